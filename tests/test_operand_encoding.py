"""The fp8 activation operand's arithmetic, on CPU: a row block x is stored
as two e4m3 terms with a power-of-two scale 2^s (max |x| 2^s in [128, 256)),
x 2^s = t0 + t1 / 16, t0 = e4m3(x 2^s), t1 = e4m3(16 (x 2^s - t0)), both
round-to-nearest-even and saturating.  The tensor-core GEMM uses it with one
scale per row (the prepared operand) and the fp8 decode chain with one UE8M0
scale per 32 elements (operand.cuh).  The claims checked here are the ones
the kernels rely on: every bf16 value within 2^13 of the block maximum is
represented exactly, and the rest to 2^-14 absolute in the scaled units."""

import numpy as np
import pytest
import torch


def e4m3_rn(v):
    """Round float64 values to e4m3 (1 sign, 4 exponent bits with bias 7, 3
    mantissa bits, subnormals down to 2^-9, largest finite 448),
    round-to-nearest-even, saturating to +-448."""
    v = np.asarray(v, dtype=np.float64)
    a = np.abs(v)
    e = np.floor(np.log2(np.where(a > 0, a, 1.0)))
    e = np.maximum(e, -6.0)  # below 2^-6 the grid is the subnormal one, 2^-9
    step = np.exp2(e - 3.0)
    q = np.rint(a / step) * step
    q = np.minimum(q, 448.0)
    return np.sign(v) * q


def encode(x):
    """x: a block of values (float64) -> (t0, t1, s)."""
    am = float(np.max(np.abs(x)))
    e2 = np.frexp(am)[1] if am > 0 else 0
    s = 8 - int(e2)
    y = np.ldexp(x, s)
    t0 = e4m3_rn(y)
    t1 = e4m3_rn(16.0 * (y - t0))
    return t0, t1, s


def bf16_values(n, log2_range, seed):
    g = torch.Generator().manual_seed(seed)
    mag = torch.exp2(-torch.rand(n, generator=g, dtype=torch.float64) * log2_range)
    sign = torch.where(torch.rand(n, generator=g) < 0.5, -1.0, 1.0).double()
    scale = float(torch.exp2(torch.randint(-20, 21, (1,), generator=g).double()))
    return (sign * mag * scale).to(torch.bfloat16).double().numpy()


@pytest.mark.parametrize("log2_range", [4, 13, 20, 30])
@pytest.mark.parametrize("seed", range(8))
def test_two_term_block_encoding(log2_range, seed):
    x = bf16_values(32, log2_range, seed)
    t0, t1, s = encode(x)
    am_scaled = np.max(np.abs(np.ldexp(x, s)))
    assert 128.0 <= am_scaled < 256.0
    # every term is an e4m3 value, so no conversion saturated
    assert np.all(np.abs(t0) <= 448.0) and np.all(np.abs(t1) <= 448.0)
    assert np.array_equal(e4m3_rn(t0), t0) and np.array_equal(e4m3_rn(t1), t1)
    y = np.ldexp(x, s)
    back = t0 + t1 / 16.0
    err = np.abs(back - y)
    near = np.abs(x) >= np.max(np.abs(x)) * 2.0 ** -13
    assert np.all(err[near] == 0.0), "a value within 2^13 of the block maximum is not exact"
    assert np.all(err <= 2.0 ** -14), "the residual error exceeds 2^-14 in the scaled units"


def test_ue8m0_scale_code_range():
    """The block scale 2^-s is stored as the UE8M0 code 127 - s; the kernels
    clamp s to [-126, 126] so that 2^s and 2^-s are normal floats and the code
    stays in [1, 253] (255 is the NaN code)."""
    for am in [0.0, 2.0 ** -140, 1e-30, 1.0, 3.0e38]:
        e2 = np.frexp(am)[1] if am > 0 else 0
        s = min(max(8 - int(e2), -126), 126)
        code = 127 - s
        assert 1 <= code <= 253
