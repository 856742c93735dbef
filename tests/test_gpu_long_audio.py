"""The long-audio chunk feeder on the GPU: chunks of different prompt lengths
decoded in lock-step mini-batches (the last one padded with a copy of its
first chunk) must give every chunk the greedy ids of its own B=1 decode by
the oracle (the reference's batched path equals its B=1 path up to
near-ties, tests/test_batched.py:85-134)."""

import pytest
import torch

from oracle import granite_ref as gr

pytestmark = pytest.mark.gpu

if not torch.cuda.is_available():
    pytest.skip("needs a CUDA device", allow_module_level=True)

from starling_b200.batched import BatchedLLMMega  # noqa: E402
from starling_b200.long_audio import decode_chunks  # noqa: E402

torch.set_grad_enabled(False)
NO_EOS = -1


@pytest.mark.parametrize("fmt", ["bf16", "fp8"])
def test_chunk_feeder_matches_per_chunk_b1(golden_dir, fmt):
    g = torch.load(golden_dir / "b1_greedy.pt")
    d = gr.Dims(**g["dims"])
    w = gr.make_weights(d, seed=g["seed"], std=g["std"], norm_jitter=g["norm_jitter"])
    gen = torch.Generator().manual_seed(21)
    lengths = [24, 19, 24, 21, 16]
    chunks = [torch.randn(T, d.hidden, generator=gen).to(torch.bfloat16) for T in lengths]
    n_new = 12
    dec = BatchedLLMMega(weights=w, dims=d.__dict__, weight_format=fmt, max_cache_len=96, max_batch_size=2,
                         steps_per_replay=4)
    res = decode_chunks(dec, [c.cuda() for c in chunks], max_new_tokens=n_new, eos_token_id=NO_EOS,
                        distributed=False)
    assert res.n_chunks == 5 and [c.index for c in res.chunks] == list(range(5))
    om = gr.OracleModel(d, w, fmt=fmt)
    with gr.accumulate("f64"):
        for i, c in enumerate(chunks):
            ref, logits = gr.OracleDecoder(om, 96).generate(c[None], n_new, NO_EOS, record_logits=True)
            got = res.chunks[i].ids
            assert len(got) == n_new
            tol = 1e-2 * float(logits[0].float().abs().max())
            for j in range(n_new):
                if got[j] != ref[j]:
                    t = logits[j].float().topk(2).values
                    assert float(t[0] - t[1]) <= tol, f"chunk {i} step {j}: {got[j]} vs {ref[j]}"
                    break
