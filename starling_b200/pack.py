"""Packing of linear layers into the tensor-core fragment layout the
dequant-GEMV streams (see include/starling_b200.h, ``SbLinear``).

Logical weight ``W[N, K]`` (row = output feature).  Rows are padded to a
multiple of 16; row tile ``t`` covers rows ``16t..16t+15``.  K is cut into
kgroups of 16 bytes per lane (64 nvfp4, 32 fp8/int8, 16 bf16 elements).  For
kgroup ``kg``, k-step ``ks`` (16 K-elements) and lane ``(g, c) = (lane//4,
lane%4)`` the lane holds the eight ``mma.m16n8k16`` A-fragment elements

    e0,e1 = (g,   2c..2c+1)   e2,e3 = (g+8, 2c..2c+1)
    e4,e5 = (g,   2c+8..2c+9) e6,e7 = (g+8, 2c+8..2c+9)

in that order (two e2m1 codes per byte, low nibble first).  nvfp4 block
scales are stored per (tile, kgroup) as 8 lanes-groups x 8 bytes
``[s(g,ks0), s(g+8,ks0), s(g,ks1), ...]``.

Fused matrices: ``qkv`` = rows ``[q | k | v]`` where inside every q and k
head the RoPE halves are interleaved (packed row ``2j`` = dim ``j``, ``2j+1`` =
dim ``j+64``) so that the GEMV epilogue holds both operands of each RoPE pair;
``gate_up`` interleaves gate row ``i`` (``2i``) and up row ``i`` (``2i+1``) for the
SwiGLU epilogue.  Quantised fused matrices are quantised as one tensor.

Tensor-core tile copy (``w_tc``): the same packed rows as raw bytes (e4m3
codes for fp8; bf16 values otherwise: the weights, the int8 codes, or the
nvfp4 code x block scale, all exact in bf16, with the row / tensor scale kept
for the epilogue), rows padded to a multiple of 128, cut into
128-row x 128-byte blocks, each block in the no-swizzle K-major canonical
layout of ``tcgen05.mma``: byte ``(row, kbyte)`` of block ``(tile, kb)`` sits at
``rg*1024 + kc*128 + r*16 + b`` with ``row = 128*tile + 8*rg + r`` and
``kbyte = 128*kb + 16*kc + b``.
"""

from __future__ import annotations

from dataclasses import dataclass
from typing import Optional

import torch

from . import quant
from ._lib import KGROUP_ELEMS, SB_FMT, SbLinear


@dataclass
class PackedLinear:
    fmt: str
    n: int
    k: int
    n_pad: int
    w: torch.Tensor  # uint8, packed fragments
    scale: Optional[torch.Tensor]  # fp32 [n_pad] (fp8/int8) or uint8 (nvfp4) or None
    global_scale: float = 1.0
    row_perm: Optional[torch.Tensor] = None  # packed row r holds logical row row_perm[r]
    w_tc: Optional[torch.Tensor] = None  # uint8 tensor-core tile copy (fp8 / bf16)
    w_bs: Optional[torch.Tensor] = None  # uint8 block-scaled tensor-core copy (nvfp4)

    def c_struct(self) -> SbLinear:
        s = SbLinear()
        s.fmt = SB_FMT[self.fmt]
        s.n, s.k, s.n_pad = self.n, self.k, self.n_pad
        s.w = self.w.data_ptr()
        s.scale = self.scale.data_ptr() if self.scale is not None else None
        s.global_scale = float(self.global_scale)
        s.w_tc = self.w_tc.data_ptr() if self.w_tc is not None else None
        s.w_bs = self.w_bs.data_ptr() if self.w_bs is not None else None
        return s

    @property
    def nbytes(self) -> int:
        return self.w.numel() * self.w.element_size() + (
            0 if self.scale is None else self.scale.numel() * self.scale.element_size()
        )


def _frag_order(q: torch.Tensor, kge: int) -> torch.Tensor:
    """[n_pad, K] elements -> [tiles, kgroups, lane(g,c), ks, e] order (flattened)."""
    n_pad, k = q.shape
    T, KG, KS = n_pad // 16, k // kge, kge // 16
    # n = t*16 + hr*8 + g ; k = kg*kge + ks*16 + hk*8 + c*2 + lo
    v = q.reshape(T, 2, 8, KG, KS, 2, 4, 2)
    # -> (T, KG, g, c, KS, hk, hr, lo): e = hk*4 + hr*2 + lo
    v = v.permute(0, 3, 2, 6, 4, 5, 1, 7)
    return v.reshape(-1)


TC_FORMATS = ("fp8", "bf16", "int8", "nvfp4")


def _bf16_rows(v: torch.Tensor) -> torch.Tensor:
    """fp32 values exactly representable in bf16 [n, k] -> bf16 bytes [n, 2k]."""
    b = v.to(torch.bfloat16)
    assert torch.equal(b.float(), v), "tile-copy values must be exact in bf16"
    return b.view(torch.int16).view(torch.uint8).reshape(v.shape[0], 2 * v.shape[1])


def tc_tiles(rows: torch.Tensor) -> torch.Tensor:
    """Row-major bytes ``[n, kbytes]`` (uint8) -> the tensor-core tile copy."""
    n, kbytes = rows.shape
    if kbytes % 128:
        raise ValueError(f"row bytes {kbytes} must be a multiple of 128")
    n_pad = (n + 127) // 128 * 128
    if n_pad != n:
        rows = torch.cat([rows, torch.zeros(n_pad - n, kbytes, dtype=torch.uint8, device=rows.device)])
    T, KB = n_pad // 128, kbytes // 128
    v = rows.reshape(T, 16, 8, KB, 8, 16)  # (tile, rg, r, kb, kc, b)
    return v.permute(0, 3, 1, 4, 2, 5).contiguous().view(-1)


def tc_untile(t: torch.Tensor, n: int, kbytes: int) -> torch.Tensor:
    """Inverse of :func:`tc_tiles` (layout check)."""
    n_pad = (n + 127) // 128 * 128
    T, KB = n_pad // 128, kbytes // 128
    v = t.view(T, KB, 16, 8, 8, 16).permute(0, 2, 4, 1, 3, 5)
    return v.reshape(n_pad, kbytes)[:n]


def bs_tiles(codes: torch.Tensor, sb: torch.Tensor) -> torch.Tensor:
    """NVFP4 codes ``[n, k]`` (4-bit values in uint8) and block scales
    ``[n, k/16]`` (e4m3 bytes) -> the block-scaled tensor-core copy
    (``SbLinear.w_bs``): per (128-row tile, 256-element K block) the codes, two
    per byte (lower K index in the low nibble), in the tile layout of
    :func:`tc_tiles`, then four 512-byte scale chunks (chunk ``j`` = K elements
    ``64j..64j+63``), byte ``(r % 32)*16 + (r // 32)*4 + i`` for tile row ``r``
    and 16-element block ``i`` of the chunk."""
    n, k = codes.shape
    if k % 256:
        raise ValueError(f"K={k} must be a multiple of 256 for the block-scaled copy")
    n_pad = (n + 127) // 128 * 128
    if n_pad != n:
        codes = torch.cat([codes, torch.zeros(n_pad - n, k, dtype=torch.uint8, device=codes.device)])
        sb = torch.cat([sb, torch.zeros(n_pad - n, k // 16, dtype=torch.uint8, device=sb.device)])
    T, KB = n_pad // 128, k // 256
    packed = (codes[:, 0::2] | (codes[:, 1::2] << 4)).contiguous()  # [n_pad, k/2]
    ct = packed.reshape(T, 16, 8, KB, 8, 16).permute(0, 3, 1, 4, 2, 5).reshape(T, KB, 16384)
    st = sb.reshape(T, 4, 32, KB, 4, 4).permute(0, 3, 4, 2, 1, 5).reshape(T, KB, 2048)
    return torch.cat([ct, st], dim=2).contiguous().view(-1)


def bs_untile(t: torch.Tensor, n: int, k: int):
    """Inverse of :func:`bs_tiles` (layout check) -> (codes [n, k], scales [n, k/16])."""
    n_pad = (n + 127) // 128 * 128
    T, KB = n_pad // 128, k // 256
    v = t.view(T, KB, 18432)
    packed = v[:, :, :16384].reshape(T, KB, 16, 8, 8, 16).permute(0, 2, 4, 1, 3, 5).reshape(n_pad, k // 2)
    codes = torch.stack([packed & 15, packed >> 4], dim=2).reshape(n_pad, k)
    sb = v[:, :, 16384:].reshape(T, KB, 4, 32, 4, 4).permute(0, 4, 3, 1, 2, 5).reshape(n_pad, k // 16)
    return codes[:n], sb[:n]


def pack_matrix(w: torch.Tensor, fmt: str, tc: bool = False, bs: bool = False) -> PackedLinear:
    """Quantise (if needed) and pack a logical weight [N, K] (bf16 or fp32).

    tc: also build the tensor-core tile copy (fp8 / bf16 only).
    bs: also build the block-scaled tensor-core copy (nvfp4, K % 256 == 0)."""
    n, k = w.shape
    kge = KGROUP_ELEMS[fmt]
    if k % 64:
        raise ValueError(f"K={k} must be a multiple of 64")
    n_pad = (n + 15) // 16 * 16
    dev = w.device
    tc = tc and fmt in TC_FORMATS
    if fmt == "bf16":
        q = w.to(torch.bfloat16).view(torch.int16)
        w_tc = tc_tiles(q.view(torch.uint8).reshape(n, 2 * k)) if tc else None
        if n_pad != n:
            q = torch.cat([q, torch.zeros(n_pad - n, k, dtype=torch.int16, device=dev)])
        packed = _frag_order(q, kge).contiguous().view(torch.uint8)
        return PackedLinear(fmt, n, k, n_pad, packed, None, w_tc=w_tc)
    parts = quant.quantize(fmt, w)
    if fmt in ("fp8", "int8"):
        q, s = parts
        if tc:  # fp8: the e4m3 bytes; int8: the integer codes as bf16 (exact)
            w_tc = tc_tiles(q.view(torch.uint8)) if fmt == "fp8" else tc_tiles(_bf16_rows(q.float()))
        else:
            w_tc = None
        q = q.view(torch.uint8)
        if n_pad != n:
            q = torch.cat([q, torch.zeros(n_pad - n, k, dtype=torch.uint8, device=dev)])
            s = torch.cat([s, torch.ones(n_pad - n, dtype=torch.float32, device=dev)])
        packed = _frag_order(q, kge).contiguous()
        return PackedLinear(fmt, n, k, n_pad, packed, s.contiguous(), w_tc=w_tc)
    codes, sb, g = parts
    w_bs = bs_tiles(codes, sb) if bs and k % 256 == 0 else None
    w_tc = None
    if tc:  # code x block scale as bf16 (<= 6 significant bits: exact); the tensor scale stays apart
        cb = quant.e2m1_to_f32(codes).view(n, k // 16, 16) * quant.e4m3_to_f32(sb)[:, :, None]
        w_tc = tc_tiles(_bf16_rows(cb.view(n, k)))
    if n_pad != n:
        codes = torch.cat([codes, torch.zeros(n_pad - n, k, dtype=torch.uint8, device=dev)])
        sb = torch.cat([sb, torch.zeros(n_pad - n, k // 16, dtype=torch.uint8, device=dev)])
    e = _frag_order(codes, kge).view(-1, 2)
    packed = (e[:, 0] | (e[:, 1] << 4)).contiguous()
    T, KG = n_pad // 16, k // 64
    sv = sb.reshape(T, 2, 8, KG, 4).permute(0, 3, 2, 4, 1).contiguous().view(-1)
    return PackedLinear(fmt, n, k, n_pad, packed, sv, g, w_tc=w_tc, w_bs=w_bs)


def rope_pair_perm(n_heads: int, head_dim: int = 128) -> torch.Tensor:
    """Packed row order for RoPE heads: within each head, (j, j+hd/2) adjacent."""
    half = head_dim // 2
    within = torch.stack([torch.arange(half), torch.arange(half) + half], dim=1).reshape(-1)
    return (torch.arange(n_heads)[:, None] * head_dim + within[None, :]).reshape(-1)


def qkv_perm(n_q: int, n_kv: int, head_dim: int = 128) -> torch.Tensor:
    qk = rope_pair_perm(n_q + n_kv, head_dim)
    v = torch.arange((n_q + n_kv) * head_dim, (n_q + 2 * n_kv) * head_dim)
    return torch.cat([qk, v])


def gate_up_perm(inter: int) -> torch.Tensor:
    return torch.stack([torch.arange(inter), torch.arange(inter) + inter], dim=1).reshape(-1)


def pack_qkv(wq, wk, wv, n_q, n_kv, fmt, head_dim=128, tc: bool = False, bs: bool = False) -> PackedLinear:
    perm = qkv_perm(n_q, n_kv, head_dim).to(wq.device)
    w = torch.cat([wq, wk, wv], dim=0)[perm]
    p = pack_matrix(w, fmt, tc=tc, bs=bs)
    p.row_perm = perm
    return p


def pack_gate_up(wg, wu, fmt, tc: bool = False, bs: bool = False) -> PackedLinear:
    perm = gate_up_perm(wg.shape[0]).to(wg.device)
    w = torch.cat([wg, wu], dim=0)[perm]
    p = pack_matrix(w, fmt, tc=tc, bs=bs)
    p.row_perm = perm
    return p


def unpack_reference(p: PackedLinear) -> torch.Tensor:
    """Inverse of the packing for bf16 (pure layout check, CPU or GPU)."""
    assert p.fmt == "bf16"
    T, KG, KS = p.n_pad // 16, p.k // 16, 1
    v = p.w.view(torch.int16).reshape(T, KG, 8, 4, KS, 2, 2, 2)
    v = v.permute(0, 6, 2, 1, 4, 5, 3, 7).reshape(p.n_pad, p.k)
    return v[: p.n].view(torch.bfloat16)
