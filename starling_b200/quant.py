"""Weight-only quantisers (torch; run on the GPU at load time).

Formats (per weight ``W[N, K]``; activations stay bf16):

* ``fp8``  : e4m3 with an fp32 scale per output row, ``s = amax_row / 448``;
* ``int8`` : symmetric int8, round-half-even, ``s = amax_row / 127``;
* ``nvfp4``: e2m1 codes, an e4m3 scale per 16 K-elements and an fp32
  tensor scale ``g = amax / (6 * 448)``; block scale ``e4m3(amax_b / 6 / g)``.

Dequantisation is ``fp32(q) * s`` (fp8/int8) and ``(fp32(code) * fp32(s_b)) * g``
(nvfp4).  The reference has no quantised path (its README.md:87-88 records INT8
and FP8 experiments with no code left), so these definitions are this
library's own; a value rounding to zero is stored as +0.
"""

from __future__ import annotations

import torch

E4M3_MAX = 448.0
E2M1_MAX = 6.0


def _div(a: torch.Tensor, b: float) -> torch.Tensor:
    """a / b with IEEE division on every device.  (On CUDA, torch evaluates
    ``tensor / python_scalar`` as a multiply by the rounded reciprocal, which
    is not the correctly rounded quotient; dividing by a tensor is.)"""
    return a / torch.full_like(a, b)


def _e4m3_bits(v: torch.Tensor) -> torch.Tensor:
    """fp32 (already within +-448) -> e4m3fn bits (RNE), with -0 canonicalised to +0."""
    b = v.to(torch.float8_e4m3fn).view(torch.uint8)
    return torch.where(b == 0x80, torch.zeros_like(b), b)


def e4m3_to_f32(bits: torch.Tensor) -> torch.Tensor:
    return bits.view(torch.float8_e4m3fn).to(torch.float32)


def quant_fp8(w: torch.Tensor):
    """-> (q uint8 [N,K] e4m3 bits, s fp32 [N])."""
    w = w.float()
    s = _div(w.abs().amax(dim=1), E4M3_MAX)
    s = torch.where(s == 0, torch.ones_like(s), s)
    v = (w / s[:, None]).clamp(-E4M3_MAX, E4M3_MAX)
    return _e4m3_bits(v), s


def quant_int8(w: torch.Tensor):
    """-> (q int8 [N,K], s fp32 [N])."""
    w = w.float()
    s = _div(w.abs().amax(dim=1), 127.0)
    s = torch.where(s == 0, torch.ones_like(s), s)
    q = torch.round(w / s[:, None]).clamp(-127, 127).to(torch.int8)
    return q, s


_E2M1_THRESH = (
    (0.25, False), (0.75, True), (1.25, False), (1.75, True), (2.5, False), (3.5, True), (5.0, False),
)


def e2m1_codes(v: torch.Tensor) -> torch.Tensor:
    """fp32 -> 4-bit e2m1 codes (RNE on the grid 0,.5,1,1.5,2,3,4,6; saturating)."""
    a = v.abs()
    idx = torch.zeros(v.shape, dtype=torch.uint8, device=v.device)
    for t, inclusive in _E2M1_THRESH:
        idx += (a >= t if inclusive else a > t).to(torch.uint8)
    sign = ((v < 0) & (idx != 0)).to(torch.uint8) << 3
    return idx | sign


E2M1_VALUES = torch.tensor([0.0, 0.5, 1.0, 1.5, 2.0, 3.0, 4.0, 6.0])


def e2m1_to_f32(codes: torch.Tensor) -> torch.Tensor:
    mag = E2M1_VALUES.to(codes.device)[(codes & 7).long()]
    return torch.where((codes & 8) != 0, -mag, mag)


def quant_nvfp4(w: torch.Tensor):
    """-> (codes uint8 [N,K] (4-bit values), block scales uint8 e4m3 [N,K/16], g float)."""
    w = w.float()
    n, k = w.shape
    if k % 16:
        raise ValueError("nvfp4 needs K % 16 == 0")
    g = _div(w.abs().amax().reshape(1), E2M1_MAX * E4M3_MAX)
    g = torch.where(g == 0, torch.ones_like(g), g)
    wb = w.view(n, k // 16, 16)
    amax_b = wb.abs().amax(dim=2)
    sb_bits = _e4m3_bits((_div(amax_b, E2M1_MAX) / g).clamp(max=E4M3_MAX))
    sf = e4m3_to_f32(sb_bits) * g
    safe = torch.where(sf == 0, torch.ones_like(sf), sf)
    v = wb / safe[:, :, None]
    v = torch.where(sf[:, :, None] == 0, torch.zeros_like(v), v)
    return e2m1_codes(v).view(n, k), sb_bits, float(g.item())


def quantize(fmt: str, w: torch.Tensor):
    if fmt == "fp8":
        return quant_fp8(w)
    if fmt == "int8":
        return quant_int8(w)
    if fmt == "nvfp4":
        return quant_nvfp4(w)
    raise ValueError(f"unknown weight format {fmt!r}")


def dequantize(fmt: str, parts) -> torch.Tensor:
    """Exact fp32 dequantisation (same values the CUDA dequant produces)."""
    if fmt == "fp8":
        q, s = parts
        return e4m3_to_f32(q) * s[:, None]
    if fmt == "int8":
        q, s = parts
        return q.float() * s[:, None]
    if fmt == "nvfp4":
        codes, sb, g = parts
        n, k = codes.shape
        c = e2m1_to_f32(codes).view(n, k // 16, 16)
        return ((c * e4m3_to_f32(sb)[:, :, None]) * torch.tensor(g, dtype=torch.float32, device=codes.device)).view(n, k)
    raise ValueError(fmt)
