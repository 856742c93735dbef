"""The numpy quantiser restatement vs torch's own fp8 / fp4 conversions."""

import numpy as np
import torch

from oracle import quant_ref as q


def _randw(n, k, seed=0, std=0.02):
    g = torch.Generator().manual_seed(seed)
    return (torch.randn(n, k, generator=g) * std).to(torch.bfloat16).float().numpy()


def test_e4m3_round_matches_torch():
    g = torch.Generator().manual_seed(3)
    x = torch.cat([torch.randn(20000, generator=g) * s for s in (1e-3, 0.1, 1, 30, 300)])
    x = x.clamp(-448, 448)
    ref = x.to(torch.float8_e4m3fn)
    ours = q.e4m3_round(x.numpy())
    assert np.array_equal(ref.float().numpy(), ours)
    assert np.array_equal(ref.view(torch.uint8).numpy() & 0x7F, q.e4m3_encode(ours) & 0x7F)
    assert np.array_equal(q.e4m3_decode(q.e4m3_encode(ours)), ours)


def test_all_e4m3_codes_roundtrip():
    bits = np.array([b for b in range(256) if (b & 0x7F) != 0x7F], dtype=np.uint8)
    vals = q.e4m3_decode(bits)
    ref = torch.from_numpy(bits).view(torch.float8_e4m3fn).float().numpy()
    assert np.array_equal(vals, ref)
    nz = vals != 0
    assert np.array_equal(q.e4m3_encode(vals)[nz], bits[nz])


def test_e2m1_grid_and_ties():
    v = np.array([0.0, 0.25, 0.26, 0.75, 1.25, 1.75, 2.5, 3.5, 5.0, 5.1, 7.0, -0.75, -6.0, -0.1], np.float32)
    got = q.e2m1_decode(q.e2m1_round_codes(v))
    want = np.array([0, 0, 0.5, 1.0, 1.0, 2.0, 2.0, 4.0, 4.0, 6.0, 6.0, -1.0, -6.0, 0.0], np.float32)
    assert np.array_equal(got, want)


def test_e2m1_matches_torch_fp4_when_available():
    if not hasattr(torch, "float4_e2m1fn_x2"):
        return
    codes = np.arange(16, dtype=np.uint8)
    packed = torch.from_numpy((codes[0::2] | (codes[1::2] << 4)).astype(np.uint8))
    try:
        f = packed.view(torch.float4_e2m1fn_x2)
        # no general cast exists; decode through the documented e2m1 table
    except Exception:
        return
    assert q.e2m1_decode(codes).tolist() == [0, .5, 1, 1.5, 2, 3, 4, 6, -0.0, -.5, -1, -1.5, -2, -3, -4, -6]


def test_fp8_int8_nvfp4_roundtrip_error():
    w = _randw(64, 256)
    for fmt, tol in (("fp8", 0.07), ("int8", 0.01), ("nvfp4", 0.3)):
        parts = q.quantize(fmt, w)
        dq = q.dequantize(fmt, parts)
        rel = np.abs(dq - w).max() / np.abs(w).max()
        assert rel < tol, (fmt, rel)


def test_nvfp4_block_structure():
    w = _randw(16, 64)
    codes, sb, g = q.quant_nvfp4(w)
    assert codes.shape == (16, 64) and sb.shape == (16, 4)
    assert codes.max() < 16
    assert np.float32(g) == np.float32(np.abs(w).max() / np.float32(2688.0))
