"""Pin the CPU oracle to vectors produced by the reference itself.

The fixtures in ``tests/golden`` were made by ``tests/golden/make_golden.py``,
which runs the reference's ``LLMMega`` / ``FusedLLMMega`` / ``BatchedLLMMega``
/ ``SpeculativeDecoder`` on CPU.  The oracle restates the same torch ops, so on
CPU it must agree bit-for-bit (ids and logits).
"""

import torch
import pytest

from oracle import granite_ref as gr

torch.set_grad_enabled(False)
EOS = 100257
PAD = 100256


@pytest.fixture(scope="module")
def tiny(golden_dir):
    g = torch.load(golden_dir / "b1_greedy.pt")
    d = gr.Dims(**g["dims"])
    w = gr.make_weights(d, seed=g["seed"], std=g["std"], norm_jitter=g["norm_jitter"])
    assert abs(gr.weights_checksum(w) - g["checksum"]) < 1e-6 * abs(g["checksum"]) + 1e-6
    return d, w, gr.OracleModel(d, w), g


def test_b1_greedy_ids_and_logits(tiny):
    d, w, m, g = tiny
    dec = gr.OracleDecoder(m, g["max_cache_len"])
    ids, logs = dec.generate(g["inputs_embeds"], g["max_new_tokens"], EOS, record_logits=True)
    assert ids == g["ids"].tolist()
    assert torch.equal(logs[0], g["prefill_logits"])
    assert torch.equal(torch.stack(logs[1:]), g["step_logits"])


def test_batched_padded(tiny, golden_dir):
    d, w, m, _ = tiny
    g = torch.load(golden_dir / "batched_padded.pt")
    B = g["inputs_embeds"].shape[0]
    dec = gr.OracleDecoder(m, g["max_cache_len"], B=B)
    gen = dec.generate_batched(g["inputs_embeds"], g["prompt_lengths"], g["max_new_tokens"], EOS, PAD)
    assert gen == [x.tolist() for x in g["ids"]]


def test_speculative(tiny, golden_dir):
    d, w, m, _ = tiny
    g = torch.load(golden_dir / "speculative.pt")
    dec = gr.OracleDecoder(m, g["max_cache_len"])
    ids, st = gr.speculative_generate(dec, g["inputs_embeds"], g["draft"], g["max_new_tokens"], EOS)
    assert ids == g["ids"].tolist()
    assert st["accepted"] == g["accepted"]
    assert st["verify_forwards"] == g["verify_forwards"]
    assert st["decode_steps"] == g["decode_steps"]


def test_layer_step_baseline_dims(golden_dir):
    g = torch.load(golden_dir / "layer_step.pt")
    D = gr.GRANITE_1B_DIMS
    w, kc, vc, x, past = gr.layer_step_case(D, seed=g["seed"], past=g["past"], std=g["std"])
    assert torch.equal(x, g["x"])
    L = gr.make_layer(D, w, 0)
    y = gr.layer_step(D, L, kc, vc, x, past)
    assert torch.equal(y.reshape(-1), g["y"])
    assert torch.equal(kc[0, :, past], g["k_new"])
    assert torch.equal(vc[0, :, past], g["v_new"])
