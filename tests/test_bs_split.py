"""The activation split of the block-scaled NVFP4 kernel (gemm_bs.cu), restated
in numpy: per 16-element block one power-of-two scale 2^e >= max / 6 (the
smallest), y0 = x 2^-e, c_t = e2m1(y_t) (round to nearest, ties to even),
y_{t+1} = 4 (y_t - c_t), eight terms.  The kernel's comment claims every step
is exact, every bf16 element within 2^-9 of its block maximum is reproduced
exactly and the rest to below 2^-17 of the block maximum; this pins those
bounds on seeded bf16 data spanning many binades (CPU only)."""

import numpy as np
import torch

E2M1 = np.array([0.0, 0.5, 1.0, 1.5, 2.0, 3.0, 4.0, 6.0])


def _e2m1_rne(y):
    """Round to the e2m1 grid, ties to the even code (the hardware conversion's rule)."""
    a = np.minimum(np.abs(y), 6.0)
    lo = np.searchsorted(E2M1, a, side="right") - 1
    lo = np.clip(lo, 0, 7)
    hi = np.minimum(lo + 1, 7)
    dl, dh = a - E2M1[lo], E2M1[hi] - a
    pick_hi = (dh < dl) | ((dh == dl) & (hi % 2 == 0) & (hi != lo))
    return np.sign(y) * np.where(pick_hi, E2M1[hi], E2M1[lo])


def _split(x):
    """x: [blocks, 16] float64 (bf16 values) -> reconstruction from 8 terms."""
    bm = np.abs(x).max(axis=1, keepdims=True)
    f, ex = np.frexp(bm)
    e = np.where(f <= 0.75, ex - 3, ex - 2)
    y = x * np.exp2(-e)
    assert np.all(np.abs(y) <= 6.0)
    rec = np.zeros_like(x)
    for t in range(8):
        c = _e2m1_rne(y)
        rec += c * np.exp2(e - 2.0 * t)
        y = (y - c) * 4.0
        assert np.all(np.abs(y) <= 6.0)
    return rec, bm


def test_block_scaled_activation_terms_bounds():
    g = torch.Generator().manual_seed(0)
    x = torch.randn(4096, 16, generator=g) * torch.exp2(torch.randint(-14, 8, (4096, 16), generator=g).float())
    x = x.to(torch.bfloat16).double().numpy()
    rec, bm = _split(x)
    err = np.abs(rec - x)
    assert np.all(err <= bm * 2.0 ** -17)
    big = np.abs(x) >= bm * 2.0 ** -9
    assert np.array_equal(rec[big], x[big])
