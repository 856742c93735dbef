"""CPU oracle for the Granite greedy-decode hot path.

TEST INFRASTRUCTURE ONLY.  Nothing in the product package imports this
directory; only ``tests/``, ``__graft_entry__.smoke()`` and the CPU-baseline
leg of ``bench.py`` use it, and only as the checker (or as the timed CPU
reference), never as a fallback for the CUDA path.

Parity status: pinned.  ``tests/golden/`` holds vectors produced by running the
reference decoders themselves on CPU (``tests/golden/make_golden.py``), and
``tests/test_oracle_golden.py`` checks this restatement against them
bit-for-bit.
"""
