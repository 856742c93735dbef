"""The fused decode step (one cooperative launch per forward of <= 8 token
rows, starling_b200/csrc/step.cu) against the per-op kernels, which the
decode tests pin to the CPU oracle and the reference's golden vectors.

Tolerances: logits within rel 1e-2 of the logit range (the two paths sum in
different fp32 orders and split the attention keys differently); greedy ids
identical unless the per-op top-2 margin is within that tolerance.
"""

import ctypes as C

import pytest
import torch

pytestmark = pytest.mark.gpu

if not torch.cuda.is_available():
    pytest.skip("needs a CUDA device", allow_module_level=True)

from starling_b200 import _lib  # noqa: E402
from starling_b200 import synthetic as syn  # noqa: E402
from starling_b200._lib import StarlingError  # noqa: E402
from starling_b200.engine import GraniteDims, GraniteEngine  # noqa: E402

torch.set_grad_enabled(False)
DEV = torch.device("cuda")
SMALL = GraniteDims(hidden=512, n_q=4, n_kv=2, inter=1024, vocab=2051, layers=2)
REAL = GraniteDims(layers=2)  # Granite 1B layer shapes, vocab 100352


def _engine(d, fmt, max_len, B, seed=0):
    w = syn.make_weights(d, seed=seed, device=DEV)
    eng = GraniteEngine(d, w, fmt, max_cache_len=max_len, max_batch=B, device=DEV)
    g = torch.Generator(device="cuda").manual_seed(seed + 1)
    eng.kv.normal_(generator=g)
    return eng


def _run(eng, st, path, ids, slot, pad_len):
    eng.step_path = path
    st.ids.copy_(ids)
    st.set_slot(slot, pad_len=pad_len)
    st.ctrl[_lib.SB_CTRL_ERR] = 0
    eng.decode_step(st, 0)
    torch.cuda.synchronize()
    return (st.logits.float().clone(), st.out_ids.clone(), int(st.ctrl[_lib.SB_CTRL_ERR]),
            int(st.ctrl[_lib.SB_CTRL_SLOT]), int(st.ctrl[_lib.SB_CTRL_ACCEPT]))


CASES = [
    # (dims, fmt, batch, m, mode, max_len, slot, prompt lengths or None)
    ("real", "nvfp4", 1, 1, _lib.SB_MODE_DECODE, 640, 320, None),
    ("real", "bf16", 1, 1, _lib.SB_MODE_DECODE, 640, 300, None),
    ("real", "fp8", 1, 1, _lib.SB_MODE_DECODE, 640, 77, None),
    ("real", "int8", 1, 1, _lib.SB_MODE_DECODE, 640, 500, None),
    ("real", "nvfp4", 1, 8, _lib.SB_MODE_VERIFY, 700, 600, None),
    ("small", "fp8", 4, 1, _lib.SB_MODE_DECODE, 160, 100, None),
    ("small", "nvfp4", 3, 1, _lib.SB_MODE_DECODE, 160, 90, [40, 81, 64]),
    ("small", "bf16", 1, 4, _lib.SB_MODE_VERIFY, 160, 120, None),
    ("small", "int8", 8, 1, _lib.SB_MODE_DECODE, 96, 70, [10, 64, 33, 64, 1, 50, 64, 63]),
]


@pytest.mark.parametrize("dims,fmt,B,m,mode,max_len,slot,plen", CASES)
def test_fused_step_matches_per_op(dims, fmt, B, m, mode, max_len, slot, plen):
    d = REAL if dims == "real" else SMALL
    eng = _engine(d, fmt, max_len, B)
    kw = {}
    pad = slot
    if plen is not None:
        pad = max(plen)
        pl = torch.tensor(plen, dtype=torch.int32)
        kw = dict(prompt_len=pl, rope_off=pad - pl)
        slot = pad + (slot - pad if slot > pad else 3)
    st = eng.new_state(B, m, mode, out_steps=4, **kw)
    assert eng.fused_step_ok(st)
    g = torch.Generator(device="cuda").manual_seed(7)
    tol = None
    for step in range(3):  # teacher-forced: both paths get the same ids at the same slot
        ids = torch.randint(0, d.vocab, (B * m,), device=DEV, generator=g)
        f = _run(eng, st, "fused", ids, slot + step, pad)
        o = _run(eng, st, "ops", ids, slot + step, pad)
        assert f[2] == 0 and o[2] == 0, "a bounded wait expired"
        assert f[3] == o[3] and f[4] == o[4], "slot / accept feedback differs"
        lf, lo = f[0], o[0]
        tol = 1e-2 * float(lo.abs().max())
        err = float((lf - lo).abs().max())
        assert err <= tol, f"step {step}: logits differ by {err:.4g} > {tol:.4g}"
        rows = B * m
        gf, go = f[1][:rows].tolist(), o[1][:rows].tolist()
        for r in range(rows):
            if gf[r] != go[r]:
                top = lo[r].topk(2).values
                assert float(top[0] - top[1]) <= tol, f"step {step} row {r}: id {gf[r]} vs {go[r]}"


def test_fused_step_serves_b1_and_refuses_large_batches():
    eng = _engine(SMALL, "nvfp4", 160, 9)
    assert eng.fused_step_ok(eng.new_state(1, 1))
    assert eng.fused_step_ok(eng.new_state(1, 8, _lib.SB_MODE_VERIFY))
    st9 = eng.new_state(9, 1)
    assert not eng.fused_step_ok(st9)
    eng.step_path = "fused"
    with pytest.raises(StarlingError):
        eng.decode_step(st9, 0)
    eng.step_path = "ops"
    eng.decode_step(st9, 0)  # the per-op kernels serve it
    torch.cuda.synchronize()


def test_fused_step_wait_expiry_reports_error_and_recovers():
    """A wait that can never complete (the attention-statistics counter of
    stream 0 / KV head 0 pushed out of reach) expires after its time bound:
    the step records SB_CTRL_ERR = 4, ends, resets its counters, and the
    next forward is correct again."""
    eng = _engine(SMALL, "bf16", 160, 1)
    st = eng.new_state(1, 1)
    off = int(eng.lib.sb_decode_step_scratch_offset(C.byref(eng.cmodel), 1))
    assert off % 4 == 0 and off < st.workspace.numel()
    ids = torch.tensor([5], device=DEV)
    ref = _run(eng, st, "ops", ids, 50, 50)
    ws = st.workspace.view(torch.int32)
    stats_word = off // 4 + 64  # the first per-(stream, KV head) statistics counter
    ws[stats_word] = -1000  # count - target stays below zero: the first attention wait never completes
    torch.cuda.synchronize()
    bad = _run(eng, st, "fused", ids, 50, 50)
    assert bad[2] == 4
    assert int(ws[stats_word]) == 0, "counters not reset after the failed forward"
    good = _run(eng, st, "fused", ids, 50, 50)
    assert good[2] == 0
    assert float((good[0] - ref[0]).abs().max()) <= 1e-2 * float(ref[0].abs().max())
    assert good[1][0] == ref[1][0]


# ---- the fused step against the CPU oracle and the reference's golden run ------------
from oracle import granite_ref as gr  # noqa: E402
from starling_b200.llm_mega import LLMMega  # noqa: E402
from starling_b200.multistep import MultiStepLLMMega  # noqa: E402
from starling_b200.speculative import SpeculativeDecoder  # noqa: E402


@pytest.fixture(scope="module")
def golden(golden_dir):
    g = torch.load(golden_dir / "b1_greedy.pt")
    d = gr.Dims(**g["dims"])
    w = gr.make_weights(d, seed=g["seed"], std=g["std"], norm_jitter=g["norm_jitter"])
    return d, w, g


def _tol(ref):
    return 1e-2 * float(ref.float().abs().max())


@pytest.mark.parametrize("fmt", ["bf16", "nvfp4"])
def test_fused_step_teacher_forced_vs_oracle(golden, fmt):
    """Every fused forward from the oracle's own cache state vs the oracle's step."""
    d, w, g = golden
    emb = g["inputs_embeds"]
    eng = GraniteEngine(d, w, fmt, max_cache_len=96, max_batch=1)
    eng.step_path = "fused"
    st = eng.new_state(1, 1, _lib.SB_MODE_DECODE, out_steps=1)
    assert eng.fused_step_ok(st)
    st.hidden.copy_(eng.prefill(emb.cuda()))
    T = emb.shape[1]
    odec = gr.OracleDecoder(gr.OracleModel(d, w, fmt=fmt), 96)
    odec.prefill(emb)
    ids = g["ids"].tolist()
    for i in range(12):
        eng.load_cache_from(odec.cache.k, odec.cache.v)
        st.ids[0] = ids[i]
        st.set_slot(T + i, pad_len=T)
        eng.decode_step(st, 0)
        valid = (torch.arange(96) <= T + i).view(1, -1)
        ref = odec.step(torch.tensor([ids[i]]), torch.tensor([T + i]), valid)[0]
        err = (st.logits[0].cpu().float() - ref.float()).abs().max()
        assert err <= _tol(ref), f"{fmt} step {i}: {err:.4g}"
        assert int(st.ctrl[_lib.SB_CTRL_ERR]) == 0


def test_fused_multistep_greedy_vs_golden(golden):
    d, w, g = golden
    eng = GraniteEngine(d, w, "bf16", max_cache_len=96, max_batch=1)
    eng.step_path = "fused"
    dec = MultiStepLLMMega(engine=eng, steps_per_replay=8)
    res = dec.generate(g["inputs_embeds"].cuda(), max_new_tokens=g["max_new_tokens"])
    got, ref = res.ids[0].tolist(), g["ids"].tolist()
    margins = [float(x.float().topk(2).values.diff().abs()) for x in [g["prefill_logits"]] + list(g["step_logits"])]
    tol = _tol(g["prefill_logits"])
    for i in range(min(len(got), len(ref))):
        if got[i] != ref[i]:
            assert margins[i] <= tol, f"id mismatch at {i} with margin {margins[i]:.4g}"
            return
    assert len(got) == len(ref)


def test_fused_speculative_vs_golden(golden, golden_dir):
    d, w, _ = golden
    g = torch.load(golden_dir / "speculative.pt")
    eng = GraniteEngine(d, w, "bf16", max_cache_len=g["max_cache_len"], max_batch=1)
    eng.step_path = "prefer_fused"  # verify forwards above 8 tokens stay per-op
    sd = SpeculativeDecoder(LLMMega(engine=eng))
    res = sd.generate(g["inputs_embeds"].cuda(), g["draft"], max_new_tokens=g["max_new_tokens"])
    assert res.ids[0].tolist() == g["ids"].tolist()
    assert res.verify_forwards == g["verify_forwards"]
