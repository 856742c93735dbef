"""Kernel-level parity on the GPU, through the C ABI, against the CPU oracle.

* dequantisation: bit-exact vs oracle/quant_ref.py for every format;
* dequant-GEMV: vs ``bf16(x.float() @ W_deq.T)`` (fp32 reference), tolerance
  stated below;
* glue ops: vs the reference's torch ops (oracle/granite_ref.py);
* argmax: torch tie rule (first maximal index).
"""

import ctypes as C

import numpy as np
import pytest
import torch

from oracle import granite_ref as gr
from oracle import quant_ref as qr

pytestmark = pytest.mark.gpu

if not torch.cuda.is_available():  # collected on CPU hosts too; skip there
    pytest.skip("needs a CUDA device", allow_module_level=True)

from starling_b200 import _lib, pack  # noqa: E402
from starling_b200._lib import check, ptr  # noqa: E402
from starling_b200.rope import rope_tables  # noqa: E402

BF16 = torch.bfloat16
lib = _lib.load()
S = lambda: _lib.current_stream()  # noqa: E731


def _w(n, k, seed, std=0.02):
    g = torch.Generator().manual_seed(seed)
    return (torch.randn(n, k, generator=g) * std).to(BF16)


def _to_dev(p: pack.PackedLinear) -> pack.PackedLinear:
    p.w = p.w.cuda()
    p.scale = None if p.scale is None else p.scale.cuda()
    return p


def _oracle_dense(w, fmt):
    if fmt == "bf16":
        return w.float()
    return torch.from_numpy(qr.dequantize(fmt, qr.quantize(fmt, w.float().numpy())))


@pytest.mark.parametrize("fmt", ["fp8", "int8", "nvfp4"])
@pytest.mark.parametrize("shape,std", [((96, 512), 0.05), ((2064, 512), 0.2), ((100, 1024), 1e-3)])
def test_quantizer_on_gpu_matches_oracle(fmt, shape, std):
    """Packing runs on the GPU at load time; its arithmetic must be the oracle's
    (IEEE division, RNE conversions) bit-for-bit."""
    from starling_b200 import quant

    w = _w(*shape, seed=shape[0], std=std)
    ours = quant.quantize(fmt, w.cuda())
    ref = qr.quantize(fmt, w.float().numpy())
    a = qr.dequantize(fmt, ref)
    b = quant.dequantize(fmt, ours).cpu().numpy()
    assert np.array_equal(a.view(np.uint32), b.view(np.uint32))


@pytest.mark.parametrize("fmt", ["bf16", "fp8", "int8", "nvfp4"])
def test_dequant_bit_exact(fmt):
    w = _w(100, 320 if fmt != "nvfp4" else 384, seed=11)
    p = _to_dev(pack.pack_matrix(w, fmt))
    out = torch.empty(p.n, p.k, dtype=torch.float32, device="cuda")
    check(lib.sb_dequant_f32(C.byref(p.c_struct()), ptr(out), S()))
    got = out.cpu().numpy()
    want = _oracle_dense(w, fmt).numpy()
    assert np.array_equal(got.view(np.uint32), want.view(np.uint32))
    outb = torch.empty(p.n, p.k, dtype=BF16, device="cuda")
    check(lib.sb_dequant_bf16(C.byref(p.c_struct()), ptr(outb), S()))
    assert torch.equal(outb.cpu(), torch.from_numpy(want).to(BF16))


# GEMV tolerance: the kernel accumulates in fp32 in a different order than
# the fp32 reference, so a bf16 output may differ by one rounding step.
def _close_bf16(got, ref):
    g, r = got.float(), ref.float()
    tol = 2.0 ** -7 * r.abs() + 1e-3 * r.abs().max()  # one bf16 ulp + tiny absolute slack
    bad = (g - r).abs() > tol
    assert bad.float().mean() < 1e-4, f"{int(bad.sum())} of {bad.numel()} outside one bf16 ulp"
    assert (g - r).abs().max() <= 4 * 2.0 ** -7 * r.abs().max()


@pytest.mark.parametrize("fmt", ["bf16", "fp8", "int8", "nvfp4"])
@pytest.mark.parametrize("n,k,m", [(3072, 2048, 1), (2048, 8192, 1), (1000, 2048, 3), (512, 1024, 9),
                                   (2048, 2048, 48), (4096, 1024, 16)])
def test_linear(fmt, n, k, m):
    w = _w(n, k, seed=n + k + m)
    x = torch.randn(m, k, generator=torch.Generator().manual_seed(5)).to(BF16)
    p = _to_dev(pack.pack_matrix(w, fmt))
    y = torch.empty(m, n, dtype=BF16, device="cuda")
    xd = x.cuda()
    check(lib.sb_linear(C.byref(p.c_struct()), ptr(xd), ptr(y), m, 0, S()), "sb_linear")
    ref = (x.float() @ _oracle_dense(w, fmt).T).to(BF16)
    _close_bf16(y.cpu(), ref)


def _linear_tc(p, x, pdl=0):
    m = x.shape[0]
    c = p.c_struct()
    need = int(lib.sb_linear_workspace_bytes(C.byref(c), m))
    assert need > 0, "tensor-core path not selected"
    ws = torch.zeros(need, dtype=torch.uint8, device="cuda")  # zeroed once: it holds counters
    y = torch.empty(m, p.n, dtype=BF16, device="cuda")
    check(lib.sb_linear_ex(C.byref(c), ptr(x), ptr(y), m, ptr(ws), need, pdl, S()), "sb_linear_ex")
    return y


@pytest.mark.parametrize("fmt", ["bf16", "fp8"])
@pytest.mark.parametrize("n,k,m", [(3072, 2048, 48), (2048, 8192, 48), (16384, 2048, 48), (2051, 512, 9),
                                   (4096, 1024, 16), (1000, 2048, 33), (2048, 2048, 64), (640, 1024, 128),
                                   (384, 512, 300), (2048, 2048, 1000), (1000, 1024, 8300),
                                   (1024, 4096, 300), (512, 8192, 200)])
def test_linear_tensor_cores(fmt, n, k, m):
    """tcgen05 GEMM (9..128 rows per block, fp8 activations as two e4m3 terms)
    vs the fp32 reference over the exactly dequantised weight: same bar as the
    GEMV (one bf16 rounding step).  Above 128 rows with K = 2048 x (1, 2, 4)
    the activation operand is prepared with each row in registers (one warp
    per 2048-element section); other K use one warp per row."""
    w = _w(n, k, seed=n + k + m)
    x = torch.randn(m, k, generator=torch.Generator().manual_seed(6)).to(BF16)
    p = pack.pack_matrix(w, fmt, tc=True)
    p = _to_dev(p)
    p.w_tc = p.w_tc.cuda()
    y = _linear_tc(p, x.cuda())
    ref = (x.float() @ _oracle_dense(w, fmt).T).to(BF16)
    _close_bf16(y.cpu(), ref)


@pytest.mark.parametrize("fmt", ["int8", "nvfp4"])
@pytest.mark.parametrize("n,k,m", [(2048, 2048, 65), (3072, 2048, 300), (1000, 1024, 1000), (2051, 512, 128)])
def test_linear_tensor_cores_bf16_copy(fmt, n, k, m):
    """INT8 / NVFP4 above 64 rows (prefill): tcgen05 GEMM on the bf16 tile copy
    (codes, code x block scale), fp32 row / tensor scale in the epilogue."""
    w = _w(n, k, seed=n + k + m)
    x = torch.randn(m, k, generator=torch.Generator().manual_seed(6)).to(BF16)
    p = _to_dev(pack.pack_matrix(w, fmt, tc=True))
    p.w_tc = p.w_tc.cuda()
    y = _linear_tc(p, x.cuda())
    ref = (x.float() @ _oracle_dense(w, fmt).T).to(BF16)
    _close_bf16(y.cpu(), ref)


def _linear(p, x, pdl=0):
    m = x.shape[0]
    y = torch.empty(m, p.n, dtype=BF16, device="cuda")
    check(lib.sb_linear(C.byref(p.c_struct()), ptr(x), ptr(y), m, pdl, S()), "sb_linear")
    return y


def _bs(w):
    p = _to_dev(pack.pack_matrix(w, "nvfp4", bs=True))
    p.w_bs = p.w_bs.cuda()
    return p


@pytest.fixture
def block_scaled():
    """Every NVFP4 linear of 1..8 rows with a w_bs copy on the block-scaled
    kernel (not only the shapes the automatic choice gives it)."""
    prev = lib.sb_set_nvfp4_path(_lib.SB_NVFP4_BLOCK_SCALED)
    yield
    lib.sb_set_nvfp4_path(prev)


@pytest.mark.parametrize("n,k,m", [(3072, 2048, 1), (2048, 8192, 1), (2048, 2048, 1), (16384, 2048, 1),
                                   (20000, 256, 2), (1000, 2048, 3), (2048, 2048, 8), (2048, 8192, 8),
                                   (512, 1024, 5), (200, 256, 4)])
def test_linear_block_scaled_nvfp4(block_scaled, n, k, m):
    """NVFP4 at 1..8 token rows on the block-scaled tcgen05 kernel
    (kind::mxf4nvf4: the weight's codes and e4m3 block scales as they are, the
    activation as eight e2m1 terms) vs the fp32 reference over the exactly
    dequantised weight: same bar as the GEMV (one bf16 rounding step).  Shapes
    cover K split over clusters of 2..8 CTAs, one and several tiles per
    persistent CTA, partial tiles and N = 8..64."""
    w = _w(n, k, seed=n + k + m)
    x = torch.randn(m, k, generator=torch.Generator().manual_seed(8)).to(BF16)
    y = _linear(_bs(w), x.cuda())
    ref = (x.float() @ _oracle_dense(w, "nvfp4").T).to(BF16)
    _close_bf16(y.cpu(), ref)


def test_linear_block_scaled_wide_range_rows(block_scaled):
    """Activation terms: rows spanning many binades, an all-zero row and a row
    near 1e-20 still match the fp32 reference."""
    n, k, m = 512, 1024, 6
    w = _w(n, k, seed=5)
    g = torch.Generator().manual_seed(3)
    x = torch.randn(m, k, generator=g) * torch.exp2(torch.randint(-12, 6, (m, k), generator=g).float())
    x[3] = 0
    x[5] *= 1e-20
    x = x.to(BF16)
    y = _linear(_bs(w), x.cuda()).cpu()
    ref = (x.float() @ _oracle_dense(w, "nvfp4").T).to(BF16)
    assert torch.all(y[3] == 0)
    _close_bf16(y, ref)


def test_linear_block_scaled_runs_deterministic_and_agrees_with_gemv(block_scaled):
    """The block-scaled kernel is the one that runs (kernel names from the
    profiler), repeats bit for bit with and without programmatic dependent
    launch, and agrees with the mma.sync GEMV over the same packed weight."""
    w = _w(3072, 2048, seed=21)
    x = torch.randn(1, 2048, device="cuda").to(BF16)
    p = _bs(w)
    with torch.profiler.profile(activities=[torch.profiler.ProfilerActivity.CUDA]) as prof:
        y0 = _linear(p, x, 0)
        torch.cuda.synchronize()
    names = [e.name for e in prof.events()]
    assert any("k_bs_gemm" in s for s in names), names[:10]
    y1 = _linear(p, x, 1)
    y2 = _linear(p, x, 0)
    assert torch.equal(y0, y1) and torch.equal(y0, y2)
    yg = _linear(_to_dev(pack.pack_matrix(w, "nvfp4")), x)  # no w_bs: the mma.sync GEMV
    _close_bf16(y0.cpu(), yg.cpu())


def test_nvfp4_path_switch():
    """sb_set_nvfp4_path returns the previous mode and rejects unknown ones;
    in automatic mode a 1-row layer projection stays on the GEMV and the
    lm_head-sized matrix takes the block-scaled kernel."""
    prev = lib.sb_set_nvfp4_path(_lib.SB_NVFP4_AUTO)
    try:
        assert lib.sb_set_nvfp4_path(_lib.SB_NVFP4_AUTO) == _lib.SB_NVFP4_AUTO
        assert lib.sb_set_nvfp4_path(7) not in (0, 1, 2)
        x = torch.randn(1, 256, device="cuda").to(BF16)
        for n, want in ((2048, False), (40000, True)):
            p = _bs(_w(n, 256, seed=n))
            with torch.profiler.profile(activities=[torch.profiler.ProfilerActivity.CUDA]) as prof:
                _linear(p, x)
                torch.cuda.synchronize()
            assert any("k_bs_gemm" in e.name for e in prof.events()) == want, n
    finally:
        lib.sb_set_nvfp4_path(prev)


def test_linear_tensor_cores_many_tiles_two_ctas_per_sm():
    """A matrix of hundreds of 128-row tiles at 48 rows: the persistent plan
    with two CTAs per SM (296 CTAs, half the ring and TMEM each), fp8 and
    bf16, vs the fp32 reference."""
    for fmt in ("fp8", "bf16"):
        n, k, m = 90000, 256, 48
        w = _w(n, k, seed=17)
        x = torch.randn(m, k, generator=torch.Generator().manual_seed(9)).to(BF16)
        p = _to_dev(pack.pack_matrix(w, fmt, tc=True))
        p.w_tc = p.w_tc.cuda()
        y = _linear_tc(p, x.cuda())
        ref = (x.float() @ _oracle_dense(w, fmt).T).to(BF16)
        _close_bf16(y.cpu(), ref)


def test_linear_tensor_cores_wide_range_rows():
    """fp8 activation split: rows spanning many binades (and an all-zero row)
    still match the fp32 reference."""
    n, k, m = 512, 1024, 24
    w = _w(n, k, seed=1)
    g = torch.Generator().manual_seed(2)
    x = torch.randn(m, k, generator=g) * torch.exp2(torch.randint(-12, 6, (m, k), generator=g).float())
    x[3] = 0
    x[5] *= 1e-20
    x = x.to(BF16)
    p = _to_dev(pack.pack_matrix(w, "fp8", tc=True))
    p.w_tc = p.w_tc.cuda()
    y = _linear_tc(p, x.cuda()).cpu()
    ref = (x.float() @ _oracle_dense(w, "fp8").T).to(BF16)
    assert torch.all(y[3] == 0)
    _close_bf16(y, ref)


def test_linear_tensor_cores_deterministic_and_pdl():
    w = _w(2048, 8192, seed=4)
    p = _to_dev(pack.pack_matrix(w, "fp8", tc=True))
    p.w_tc = p.w_tc.cuda()
    x = torch.randn(48, 8192, device="cuda").to(BF16)
    y0 = _linear_tc(p, x, 0)
    y1 = _linear_tc(p, x, 1)
    y2 = _linear_tc(p, x, 0)
    assert torch.equal(y0, y1) and torch.equal(y0, y2)


def test_linear_pdl_same_as_plain():
    w = _w(2048, 2048, seed=3)
    p = _to_dev(pack.pack_matrix(w, "nvfp4"))
    x = torch.randn(1, 2048, device="cuda").to(BF16)
    y0 = torch.empty(1, 2048, dtype=BF16, device="cuda")
    y1 = torch.empty_like(y0)
    check(lib.sb_linear(C.byref(p.c_struct()), ptr(x), ptr(y0), 1, 0, S()))
    check(lib.sb_linear(C.byref(p.c_struct()), ptr(x), ptr(y1), 1, 1, S()))
    assert torch.equal(y0, y1)


def test_glue_rmsnorm_silu_residual():
    g = torch.Generator().manual_seed(9)
    x = (torch.randn(4, 2048, generator=g) * 3).to(BF16)
    w = (1 + 0.1 * torch.randn(2048, generator=g)).to(BF16)
    y = torch.empty_like(x, device="cuda")
    xd, wd = x.cuda(), w.cuda()  # keep device copies alive until the kernel has run
    check(lib.sb_rmsnorm(ptr(xd), ptr(wd), ptr(y), 4, 2048, C.c_float(1e-5), S()))
    ref = gr.rmsnorm(x, w, 1e-5)
    diff = (y.cpu().float() != ref.float())
    assert diff.float().mean() < 1e-3  # rare 1-ulp flips from the sum order of mean(x^2)
    assert torch.allclose(y.cpu().float(), ref.float(), rtol=2 ** -7, atol=0)

    gt = (torch.randn(8192, generator=g) * 4).to(BF16)
    up = torch.randn(8192, generator=g).to(BF16)
    o = torch.empty(8192, dtype=BF16, device="cuda")
    gd, ud = gt.cuda(), up.cuda()
    check(lib.sb_silu_mul(ptr(gd), ptr(ud), ptr(o), 8192, S()))
    ref = gr.silu_mul(gt, up)
    assert (o.cpu().float() != ref.float()).float().mean() < 1e-3
    assert torch.allclose(o.cpu().float(), ref.float(), rtol=2 ** -7, atol=1e-30)

    a = torch.randn(2048, generator=g).to(BF16)
    b = torch.randn(2048, generator=g).to(BF16)
    z = torch.empty(2048, dtype=BF16, device="cuda")
    ad, bd = a.cuda(), b.cuda()
    check(lib.sb_residual_scale(ptr(ad), ptr(bd), ptr(z), 2048, C.c_float(0.22), S()))
    assert torch.equal(z.cpu(), gr.residual_scale(a, b, 0.22))  # bf16 products: exact


def test_glue_rope_bit_exact():
    d = gr.GRANITE_1B_DIMS
    cs, sn = rope_tables(128, d.theta, 1024)
    pos = torch.tensor([0, 7, 300, 1023], dtype=torch.int32)
    q = (torch.randn(4, 16, 128, generator=torch.Generator().manual_seed(2)) * 20).to(BF16)
    qd = q.cuda().contiguous()
    pd, csd, snd = pos.cuda(), cs.cuda(), sn.cuda()
    check(lib.sb_rope(ptr(qd), 64, 16, ptr(pd), ptr(csd), ptr(snd), S()))
    c4, s4 = gr.rope_cos_sin(d, pos.long().view(4, 1))  # (4, 1, 128)
    ref = q * c4 + gr.rotate_half(q) * s4  # llm_mega.py:542 with per-position cos/sin
    assert torch.equal(qd.cpu(), ref)


def test_rope_table_matches_hf_formula():
    d = gr.GRANITE_1B_DIMS
    cs, sn = rope_tables(128, d.theta, 700)
    c, s = gr.rope_cos_sin(d, torch.arange(700).view(1, -1))
    assert torch.equal(cs, c[0, :, :64]) and torch.equal(sn, s[0, :, :64])
    assert torch.equal(c[0, :, :64], c[0, :, 64:])


def test_argmax_first_max():
    x = torch.zeros(3, 100353, dtype=BF16)
    x[0, 17] = 5.0
    x[0, 90000] = 5.0
    x[1, :] = -1.0
    x[2, 100352] = 1.0
    out = torch.empty(3, dtype=torch.int64, device="cuda")
    xd = x.cuda()
    check(lib.sb_argmax_bf16(ptr(xd), 3, 100353, ptr(out), S()))
    assert out.cpu().tolist() == [17, 0, 100352]
    assert out.cpu().tolist() == x.float().argmax(-1).tolist()


def _attn_engine(B, max_len, n_q=8, n_kv=4):
    from starling_b200.engine import GraniteDims, GraniteEngine

    d = GraniteDims(hidden=1024, n_q=n_q, n_kv=n_kv, inter=1024, vocab=256, layers=1)
    g = torch.Generator(device="cuda").manual_seed(1)
    shapes = {"embed_tokens.weight": (256, 1024), "norm.weight": (1024,),
              "layers.0.input_layernorm.weight": (1024,), "layers.0.post_attention_layernorm.weight": (1024,),
              "layers.0.self_attn.q_proj.weight": (n_q * 128, 1024), "layers.0.self_attn.k_proj.weight": (n_kv * 128, 1024),
              "layers.0.self_attn.v_proj.weight": (n_kv * 128, 1024), "layers.0.self_attn.o_proj.weight": (1024, n_q * 128),
              "layers.0.mlp.gate_proj.weight": (1024, 1024), "layers.0.mlp.up_proj.weight": (1024, 1024),
              "layers.0.mlp.down_proj.weight": (1024, 1024)}
    w = {k: (torch.randn(s, generator=g, device="cuda") * 0.02).to(BF16) for k, s in shapes.items()}
    return GraniteEngine(d, w, "bf16", max_cache_len=max_len, max_batch=B, tensor_cores=False)


def _attn_reference(q, kc, vc, valid, n_q, n_kv, m, mult):
    """The reference's eager attention (llm_mega.py:549-556, modeling_granite.py:89-112)
    on CPU: bf16 matmuls, additive -max mask, fp32 softmax cast to bf16."""
    B = kc.shape[0]
    qh = q.view(B, m, n_q, 128).transpose(1, 2)  # (B, n_q, m, 128)
    kr, vr = gr.repeat_kv(kc, n_q // n_kv), gr.repeat_kv(vc, n_q // n_kv)
    sc = torch.matmul(qh, kr.transpose(2, 3)) * mult
    mask = torch.zeros(valid.shape, dtype=BF16).masked_fill_(~valid, gr.NEG)  # (B, m, L)
    sc = sc + mask[:, None]
    pr = torch.nn.functional.softmax(sc, dim=-1, dtype=torch.float32).to(BF16)
    return torch.matmul(pr, vr).transpose(1, 2).reshape(B * m, n_q * 128)


@pytest.mark.parametrize("B,m,max_len,slot,holes", [(40, 1, 700, 650, True), (40, 1, 700, 650, False),
                                                     (3, 1, 700, 400, True), (1, 9, 640, 600, False),
                                                     (2, 4, 300, 120, True)])
def test_attention_vs_reference(B, m, max_len, slot, holes):
    """sb_attention (one CTA per (stream, head) when the groups fill the GPU,
    else a cluster split; multi-tile key rings; right-padding holes; verify
    rows with the causal block) vs the reference's eager attention."""
    eng = _attn_engine(B, max_len)
    d = eng.dims
    g = torch.Generator().manual_seed(B * 1000 + slot)
    pad_len = slot - 5 if holes else slot
    pl = torch.randint(pad_len // 3, pad_len + 1, (B,), generator=g) if holes else torch.full((B,), pad_len)
    pl[0] = pad_len
    st = eng.new_state(B, m, _lib.SB_MODE_DECODE, out_steps=1, prompt_len=pl, rope_off=pad_len - pl)
    kc = (torch.randn(B, d.n_kv, max_len, 128, generator=g) * 2).to(BF16)
    vc = torch.randn(B, d.n_kv, max_len, 128, generator=g).to(BF16)
    q = (torch.randn(B * m, d.n_q * 128, generator=g) * 2).to(BF16)
    eng.kv[0, 0, :B].copy_(kc)
    eng.kv[0, 1, :B].copy_(vc)
    st.q.copy_(q)
    st.set_slot(slot, pad_len=pad_len)
    check(lib.sb_attention(C.byref(eng.cmodel), C.byref(st.c), 0, S()), "sb_attention")
    kpos = torch.arange(max_len)
    # row token mi sees [0, prompt_len) and [pad_len, slot + mi]
    valid = ((kpos[None, None, :] < pl[:, None, None]) |
             ((kpos[None, None, :] >= pad_len) & (kpos[None, None, :] <= slot + torch.arange(m)[None, :, None])))
    ref = _attn_reference(q, kc, vc, valid, d.n_q, d.n_kv, m, d.attn_mult)
    _close_bf16(st.attn.cpu(), ref)
    assert int(st.ctrl[_lib.SB_CTRL_ERR]) == 0
