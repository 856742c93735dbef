"""sb_lm_head_argmax_static: the lm_head + argmax entry point for callers that
cannot allocate device memory (its scratch is a fixed array inside the
library).  Called through the C ABI, it must give the same logits and token
ids as sb_lm_head_argmax with a caller workspace, on two calls in a row, and
reject shapes whose scratch would not fit.

This file is named so that pytest collects it last.
"""

import ctypes as C

import pytest
import torch

pytestmark = pytest.mark.gpu

if not torch.cuda.is_available():
    pytest.skip("needs a CUDA device", allow_module_level=True)

from starling_b200 import _lib  # noqa: E402
from starling_b200.engine import GraniteDims, GraniteEngine  # noqa: E402

torch.set_grad_enabled(False)


SMALL = dict(hidden=512, n_q=4, n_kv=2, inter=1024)
# the Granite-1B decoder's lm_head dimensions (hidden 2048, 16 / 4 heads)
FULL = dict(hidden=2048, n_q=16, n_kv=4, inter=8192)


def _engine(vocab, fmt, tensor_cores=True, dims=SMALL):
    d = GraniteDims(vocab=vocab, layers=1, **dims)
    H, I, NQ, NKV = d.hidden, d.inter, d.n_q * 128, d.n_kv * 128
    g = torch.Generator(device="cuda").manual_seed(7)
    w = {}
    for name, shape in [("embed_tokens.weight", (vocab, H)), ("norm.weight", (H,)),
                        ("layers.0.input_layernorm.weight", (H,)), ("layers.0.post_attention_layernorm.weight", (H,)),
                        ("layers.0.self_attn.q_proj.weight", (NQ, H)), ("layers.0.self_attn.k_proj.weight", (NKV, H)),
                        ("layers.0.self_attn.v_proj.weight", (NKV, H)), ("layers.0.self_attn.o_proj.weight", (H, NQ)),
                        ("layers.0.mlp.gate_proj.weight", (I, H)), ("layers.0.mlp.up_proj.weight", (I, H)),
                        ("layers.0.mlp.down_proj.weight", (H, I))]:
        w[name] = (torch.randn(shape, generator=g, device="cuda") * (0.05 if len(shape) == 2 else 1.0)).to(torch.bfloat16)
    return GraniteEngine(d, w, fmt, max_cache_len=64, max_batch=16, tensor_cores=tensor_cores)


@pytest.mark.parametrize("vocab,fmt,batch,dims,null_ws", [
    (100352, "nvfp4", 1, SMALL, False), (2051, "bf16", 1, SMALL, False), (100352, "fp8", 2, SMALL, False),
    (100352, "nvfp4", 1, FULL, True), (100352, "fp8", 2, FULL, True), (100352, "fp8", 16, FULL, True),
    (100352, "bf16", 1, FULL, True)])
def test_static_scratch_matches_workspace_version(vocab, fmt, batch, dims, null_ws):
    """null_ws: the state carries no workspace at all (pointer NULL, 0 bytes),
    as a caller without a device allocator would pass it."""
    eng = _engine(vocab, fmt, dims=dims)
    lib = eng.lib
    H = eng.dims.hidden
    ref = eng.new_state(batch, 1, _lib.SB_MODE_FIRST, out_steps=1)
    new = eng.new_state(batch, 1, _lib.SB_MODE_FIRST, out_steps=1)
    if null_ws:
        new.c.workspace, new.c.workspace_bytes = None, 0
    h = torch.randn(batch, H, generator=torch.Generator(device="cuda").manual_seed(1), device="cuda").to(torch.bfloat16)
    ref.hidden.copy_(h)
    new.hidden.copy_(h)
    s = _lib.current_stream()
    _lib.check(lib.sb_lm_head_argmax(C.byref(eng.cmodel), C.byref(ref.c), 0, s), "sb_lm_head_argmax")
    for call in range(2):  # two calls in a row share (and must re-clear) the fixed scratch
        new.out_ids.zero_()
        new.logits.zero_()
        _lib.check(lib.sb_lm_head_argmax_static(C.byref(eng.cmodel), C.byref(new.c), 0, s),
                   "sb_lm_head_argmax_static")
        torch.cuda.synchronize()
        # same kernel and configuration: results are identical (the tests'
        # tolerance for a bf16 logit is one rounding step; here it is zero)
        assert torch.equal(new.logits, ref.logits), f"call {call}: logits differ"
        assert torch.equal(new.out_ids[:batch], ref.out_ids[:batch]), f"call {call}: token ids differ"
        assert torch.equal(new.out_ids[:batch], ref.logits.float().argmax(-1))


def test_static_scratch_rejects_too_many_rows():
    # the mma.sync GEMV (no tensor-core tile copy) keeps one argmax partial per
    # CTA of a large grid: 32 rows of a 100352-row lm_head exceed the array
    eng = _engine(100352, "fp8", tensor_cores=False)
    rows = 32
    assert eng.lib.sb_workspace_bytes(C.byref(eng.cmodel), rows) > 256 * 1024  # does not fit the fixed array
    st = eng.new_state(1, rows, _lib.SB_MODE_VERIFY, out_steps=1)
    rc = eng.lib.sb_lm_head_argmax_static(C.byref(eng.cmodel), C.byref(st.c), 0, _lib.current_stream())
    assert rc == 1002  # SB_ERR_CONFIG
    assert b"scratch" in eng.lib.sb_last_error()
