"""Oracle restatement (numpy, CPU) of the weight-only quantisation formats.

TEST INFRASTRUCTURE ONLY -- see ``oracle/__init__.py``.

The reference has no quantised path (README.md:87-88 records that INT8 and FP8
were tried and dropped; no code remains), so the three formats are defined
here, once, and the product quantiser (``starling_b200/quant.py``, torch) and
the CUDA dequantiser are both checked against these functions bit-for-bit.

Formats (all per ``nn.Linear`` weight ``W[N, K]``, bf16 in):

* ``fp8``  : ``q = e4m3(W / s_row)``, ``s_row = amax_row / 448`` (fp32);
             dequant ``fp32(q) * s_row``.
* ``int8`` : ``q = clamp(rint(W / s_row), -127, 127)``,
             ``s_row = amax_row / 127``; dequant ``fp32(q) * s_row``.
* ``nvfp4``: ``g = amax / (6 * 448)``; per 16-element K block
             ``s_b = e4m3(amax_b / 6 / g)``; ``code = e2m1(W / (fp32(s_b) * g))``;
             dequant ``(fp32(code) * fp32(s_b)) * g``.

Rounding is round-to-nearest-even everywhere; e2m1 and e4m3 saturate at their
largest finite magnitude (6 and 448).  A value that rounds to zero is stored as
+0 (code 0).
"""

from __future__ import annotations

import numpy as np

E4M3_MAX = 448.0
E2M1_MAX = 6.0

# e2m1 magnitudes by 3-bit code (sign in bit 3).
E2M1_VALUES = np.array([0.0, 0.5, 1.0, 1.5, 2.0, 3.0, 4.0, 6.0], dtype=np.float32)


def _f32(x) -> np.ndarray:
    return np.asarray(x, dtype=np.float32)


def e4m3_round(x: np.ndarray) -> np.ndarray:
    """Round fp32 values to the nearest e4m3fn value (RNE), saturating at 448.

    Returns the rounded values as fp32 (every e4m3 value is exact in fp32).
    e4m3fn: 1 sign, 4 exponent (bias 7), 3 mantissa bits; smallest normal
    2^-6, subnormal step 2^-9.
    """
    x = _f32(x)
    a = np.abs(x).astype(np.float64)
    out = np.zeros_like(a)
    nz = a > 0
    # exponent of the value, clamped to the normal range floor (-6) so that
    # subnormals share the 2^-9 quantum.
    e = np.floor(np.log2(np.where(nz, a, 1.0)))
    e = np.maximum(e, -6.0)
    q = np.exp2(e - 3.0)  # quantum: 3 mantissa bits
    out = np.where(nz, np.rint(a / q) * q, 0.0)  # np.rint is half-to-even
    out = np.minimum(out, E4M3_MAX)
    return (np.sign(x) * out).astype(np.float32)


def e4m3_encode(v: np.ndarray) -> np.ndarray:
    """Encode exact e4m3 values (output of :func:`e4m3_round`) to uint8 bits."""
    v = _f32(v)
    a = np.abs(v).astype(np.float64)
    sign = (np.signbit(v) & (a > 0)).astype(np.uint8) << 7
    bits = np.zeros(v.shape, dtype=np.uint8)
    nz = a > 0
    e = np.floor(np.log2(np.where(nz, a, 1.0)))
    sub = nz & (e < -6)
    norm = nz & ~sub
    # normal: exp field = e + 7, mantissa = (a / 2^e - 1) * 8
    ef = (e + 7).astype(np.int64)
    man = np.rint((a / np.exp2(e) - 1.0) * 8.0).astype(np.int64)
    bits = np.where(norm, (ef << 3) | man, bits).astype(np.int64)
    # subnormal: value = man * 2^-9
    mans = np.rint(a / 2.0**-9).astype(np.int64)
    bits = np.where(sub, mans, bits)
    return (bits.astype(np.uint8) | sign).astype(np.uint8)


def e4m3_decode(bits: np.ndarray) -> np.ndarray:
    """Decode e4m3fn bytes to fp32."""
    b = np.asarray(bits, dtype=np.uint8).astype(np.int64)
    s = np.where(b & 0x80, -1.0, 1.0)
    ef = (b >> 3) & 0xF
    m = b & 0x7
    val = np.where(ef == 0, m * 2.0**-9, (1.0 + m / 8.0) * np.exp2(ef - 7.0))
    # 0x7F / 0xFF are NaN in e4m3fn; the quantiser never produces them.
    return (s * val).astype(np.float32)


def e2m1_round_codes(v: np.ndarray) -> np.ndarray:
    """Round fp32 values to e2m1 (RNE, saturating at 6); return 4-bit codes."""
    v = _f32(v)
    a = np.abs(v)
    # Thresholds between neighbouring grid points; ties go to the even
    # mantissa (0, 1.0, 2.0, 4.0 are "even").
    idx = np.select(
        [a <= 0.25, a < 0.75, a <= 1.25, a < 1.75, a <= 2.5, a < 3.5, a <= 5.0],
        [0, 1, 2, 3, 4, 5, 6],
        default=7,
    ).astype(np.uint8)
    sign = ((v < 0) & (idx != 0)).astype(np.uint8) << 3
    return (idx | sign).astype(np.uint8)


def e2m1_decode(codes: np.ndarray) -> np.ndarray:
    c = np.asarray(codes, dtype=np.uint8)
    mag = E2M1_VALUES[c & 0x7]
    return np.where(c & 0x8, -mag, mag).astype(np.float32)


# --------------------------------------------------------------------------- #
# quantisers: canonical (unpacked) representation
# --------------------------------------------------------------------------- #
def quant_fp8(w: np.ndarray):
    """Return (q_bits uint8 [N,K], scale fp32 [N])."""
    w = _f32(w)
    amax = np.max(np.abs(w), axis=1)
    s = (amax / np.float32(E4M3_MAX)).astype(np.float32)
    s = np.where(s == 0, np.float32(1.0), s).astype(np.float32)
    v = (w / s[:, None]).astype(np.float32)
    v = np.clip(v, -E4M3_MAX, E4M3_MAX)
    return e4m3_encode(e4m3_round(v)), s


def dequant_fp8(q: np.ndarray, s: np.ndarray) -> np.ndarray:
    return (e4m3_decode(q) * _f32(s)[:, None]).astype(np.float32)


def quant_int8(w: np.ndarray):
    """Return (q int8 [N,K], scale fp32 [N])."""
    w = _f32(w)
    amax = np.max(np.abs(w), axis=1)
    s = (amax / np.float32(127.0)).astype(np.float32)
    s = np.where(s == 0, np.float32(1.0), s).astype(np.float32)
    q = np.clip(np.rint((w / s[:, None]).astype(np.float32)), -127, 127)
    return q.astype(np.int8), s


def dequant_int8(q: np.ndarray, s: np.ndarray) -> np.ndarray:
    return (q.astype(np.float32) * _f32(s)[:, None]).astype(np.float32)


def quant_nvfp4(w: np.ndarray):
    """Return (codes uint8 [N,K] (4-bit), block scales uint8 e4m3 [N,K/16], g fp32)."""
    w = _f32(w)
    n, k = w.shape
    assert k % 16 == 0
    amax = np.float32(np.max(np.abs(w)))
    g = np.float32(amax / np.float32(E2M1_MAX * E4M3_MAX))
    if g == 0:
        g = np.float32(1.0)
    wb = w.reshape(n, k // 16, 16)
    amax_b = np.max(np.abs(wb), axis=2).astype(np.float32)
    sb = e4m3_round(((amax_b / np.float32(E2M1_MAX)).astype(np.float32) / g).astype(np.float32))
    sf = (sb * g).astype(np.float32)
    safe = np.where(sf == 0, np.float32(1.0), sf).astype(np.float32)
    v = (wb / safe[:, :, None]).astype(np.float32)
    v = np.where(sf[:, :, None] == 0, np.float32(0.0), v)
    codes = e2m1_round_codes(v).reshape(n, k)
    return codes, e4m3_encode(sb), g


def dequant_nvfp4(codes: np.ndarray, sbits: np.ndarray, g) -> np.ndarray:
    n, k = codes.shape
    c = e2m1_decode(codes).reshape(n, k // 16, 16)
    sb = e4m3_decode(sbits)
    out = (c * sb[:, :, None]).astype(np.float32) * np.float32(g)
    return out.astype(np.float32).reshape(n, k)


QUANTIZERS = {"fp8": quant_fp8, "int8": quant_int8, "nvfp4": quant_nvfp4}


def quantize(fmt: str, w: np.ndarray):
    return QUANTIZERS[fmt](w)


def dequantize(fmt: str, parts) -> np.ndarray:
    if fmt == "fp8":
        return dequant_fp8(*parts)
    if fmt == "int8":
        return dequant_int8(*parts)
    if fmt == "nvfp4":
        return dequant_nvfp4(*parts)
    raise ValueError(fmt)
