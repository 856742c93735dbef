"""CPU checks of the product quantiser and the packed fragment layout.

* the torch quantiser (starling_b200/quant.py) must equal the numpy oracle
  (oracle/quant_ref.py) bit-for-bit;
* decoding the packed bytes with an independent Python reader must give back
  exactly the quantiser's codes / the oracle's dequantised weights.
"""

import numpy as np
import pytest
import torch

from oracle import quant_ref as qr
from starling_b200 import pack, quant


def _w(n, k, seed=0, std=0.02):
    g = torch.Generator().manual_seed(seed)
    w = torch.randn(n, k, generator=g) * std
    w[1] = 0.0  # an all-zero row
    w[2, :5] = torch.tensor([3.0, -2.5, 1e-8, -1e-9, 0.0]) * std
    return w.to(torch.bfloat16)


@pytest.mark.parametrize("fmt", ["fp8", "int8", "nvfp4"])
@pytest.mark.parametrize("shape", [(48, 128), (33, 256), (16, 64)])
def test_torch_quant_matches_oracle(fmt, shape):
    w = _w(*shape, seed=shape[0])
    ours = quant.quantize(fmt, w)
    ref = qr.quantize(fmt, w.float().numpy())
    if fmt == "nvfp4":
        assert np.array_equal(ours[0].numpy(), ref[0])
        assert np.array_equal(ours[1].numpy(), ref[1])
        assert np.float32(ours[2]) == np.float32(ref[2])
    else:
        q = ours[0].numpy()
        assert np.array_equal(q.view(np.uint8), ref[0].view(np.uint8))
        assert np.array_equal(ours[1].numpy(), ref[1])
    dq = quant.dequantize(fmt, ours).numpy()
    assert np.array_equal(dq.view(np.uint32), qr.dequantize(fmt, ref).view(np.uint32))


# ---- independent reader of the packed layout (mirror of the CUDA indexing) ----
def read_packed(p: pack.PackedLinear) -> np.ndarray:
    """Return the logical [n, k] fp32 weights encoded in a PackedLinear."""
    kge = {"bf16": 16, "fp8": 32, "int8": 32, "nvfp4": 64}[p.fmt]
    ks_n = kge // 16
    T, KG = p.n_pad // 16, p.k // kge
    raw = p.w.numpy().reshape(T, KG, 32, 16)
    out = np.zeros((p.n_pad, p.k), np.float32)
    rofs = lambda g: [g, g, g + 8, g + 8, g, g, g + 8, g + 8]
    kofs = lambda c: [2 * c, 2 * c + 1, 2 * c, 2 * c + 1, 2 * c + 8, 2 * c + 9, 2 * c + 8, 2 * c + 9]
    if p.fmt == "nvfp4":
        sc = p.scale.numpy().reshape(T, KG, 8, 8)
    for t in range(T):
        for kg in range(KG):
            for lane in range(32):
                g, c = lane // 4, lane % 4
                b = raw[t, kg, lane]
                for ks in range(ks_n):
                    for e in range(8):
                        row = t * 16 + rofs(g)[e]
                        k = kg * kge + ks * 16 + kofs(c)[e]
                        if p.fmt == "bf16":
                            u = int(b[2 * (ks * 8 + e)]) | (int(b[2 * (ks * 8 + e) + 1]) << 8)
                            v = np.array([u << 16], np.uint32).view(np.float32)[0]
                        elif p.fmt in ("fp8", "int8"):
                            byte = b[ks * 8 + e]
                            v = qr.e4m3_decode(np.array([byte]))[0] if p.fmt == "fp8" else np.float32(np.int8(byte))
                            v = np.float32(v) * p.scale.numpy()[row]
                        else:
                            byte = b[ks * 4 + e // 2]
                            code = (byte >> 4) if e % 2 else (byte & 0xF)
                            hr = rofs(g)[e] >= 8
                            s = qr.e4m3_decode(np.array([sc[t, kg, g, ks * 2 + int(hr)]]))[0]
                            v = np.float32(np.float32(qr.e2m1_decode(np.array([code]))[0] * s) * np.float32(p.global_scale))
                        out[row, k] = v
    return out[: p.n]


@pytest.mark.parametrize("fmt", ["bf16", "fp8", "int8", "nvfp4"])
def test_packed_layout_roundtrip(fmt):
    w = _w(20, 128, seed=7)  # n not a multiple of 16 -> padded tile
    p = pack.pack_matrix(w, fmt)
    assert p.n_pad == 32
    got = read_packed(p)
    if fmt == "bf16":
        want = w.float().numpy()
    else:
        want = qr.dequantize(fmt, qr.quantize(fmt, w.float().numpy()))
    assert np.array_equal(got.view(np.uint32), want.view(np.uint32))


def test_bf16_unpack_reference():
    w = _w(40, 192, seed=3)
    p = pack.pack_matrix(w, "bf16")
    assert torch.equal(pack.unpack_reference(p), w)


def test_row_permutations():
    perm = pack.qkv_perm(2, 1, 128)
    assert perm.numel() == 4 * 128
    assert perm[:4].tolist() == [0, 64, 1, 65]
    assert perm[128:130].tolist() == [128, 192]
    assert perm[3 * 128:3 * 128 + 2].tolist() == [384, 385]  # v rows unpermuted
    assert sorted(perm.tolist()) == list(range(512))
    gu = pack.gate_up_perm(4)
    assert gu.tolist() == [0, 4, 1, 5, 2, 6, 3, 7]


def _bf16_bytes(v: np.ndarray) -> torch.Tensor:
    t = torch.from_numpy(np.ascontiguousarray(v, dtype=np.float32)).to(torch.bfloat16)
    assert torch.equal(t.float(), torch.from_numpy(np.ascontiguousarray(v, dtype=np.float32)))
    return t.view(torch.int16).view(torch.uint8).reshape(v.shape[0], 2 * v.shape[1])


@pytest.mark.parametrize("fmt", ["bf16", "fp8", "int8", "nvfp4"])
def test_tensor_core_tile_layout(fmt):
    """w_tc: byte (row, kbyte) of block (tile, kb) at rg*1024 + kc*128 + r*16 + b
    (the no-swizzle K-major canonical layout of tcgen05.mma), padded rows zero,
    holding the oracle's quantised rows: e4m3 bytes for fp8; bf16 values for
    the others (the weights, the int8 codes, the nvfp4 code x block scale)."""
    n, k = 200, 256
    w = _w(n, k, seed=9)
    p = pack.pack_matrix(w, fmt, tc=True)
    assert p.w_tc is not None
    if fmt == "bf16":
        rows = w.view(torch.int16).view(torch.uint8).reshape(n, 2 * k)
    elif fmt == "fp8":
        q, _ = qr.quantize("fp8", w.float().numpy())
        rows = torch.from_numpy(q.view(np.uint8).copy()).reshape(n, k)
    elif fmt == "int8":
        q, _ = qr.quantize("int8", w.float().numpy())
        rows = _bf16_bytes(q.astype(np.float32))
    else:
        codes, sb, _ = qr.quantize("nvfp4", w.float().numpy())
        cb = qr.e2m1_decode(codes).reshape(n, k // 16, 16) * qr.e4m3_decode(sb)[:, :, None]
        rows = _bf16_bytes(cb.reshape(n, k))
    kbytes = rows.shape[1]
    t = p.w_tc
    assert t.numel() == 256 * kbytes  # 200 rows -> 2 tiles of 128
    KB = kbytes // 128
    g = torch.Generator().manual_seed(0)
    for _ in range(500):
        row = int(torch.randint(0, 256, (1,), generator=g))
        kb_ = int(torch.randint(0, kbytes, (1,), generator=g))
        tile, rr = divmod(row, 128)
        rg, r = divmod(rr, 8)
        kb, kk = divmod(kb_, 128)
        kc, b = divmod(kk, 16)
        off = (tile * KB + kb) * 16384 + rg * 1024 + kc * 128 + r * 16 + b
        want = int(rows[row, kb_]) if row < n else 0
        assert int(t[off]) == want
    assert torch.equal(pack.tc_untile(t, n, kbytes), rows)


def test_block_scaled_copy_layout():
    """w_bs (nvfp4): per (tile, 256-element K block) 16384 bytes of codes, two
    per byte (lower K index in the low nibble) at rg*1024 + kc*128 + r*16 + b,
    then four 512-byte scale chunks, byte (r % 32)*16 + (r // 32)*4 + i for
    chunk j (K elements 64j..64j+63) and 16-element block i; padded rows zero;
    codes and scales are the oracle's quantisation."""
    n, k = 200, 512
    w = _w(n, k, seed=13)
    p = pack.pack_matrix(w, "nvfp4", bs=True)
    assert p.w_bs is not None and p.w_bs.numel() == 2 * (k // 256) * 18432
    codes, sb, _ = qr.quantize("nvfp4", w.float().numpy())
    codes = torch.from_numpy(np.asarray(codes, dtype=np.uint8).reshape(n, k))
    sb = torch.from_numpy(np.asarray(sb, dtype=np.uint8).reshape(n, k // 16))
    t = p.w_bs
    KB = k // 256
    g = torch.Generator().manual_seed(1)
    for _ in range(500):
        row = int(torch.randint(0, 256, (1,), generator=g))
        e = int(torch.randint(0, k, (1,), generator=g))
        tile, rr = divmod(row, 128)
        rg, r = divmod(rr, 8)
        kb, ke = divmod(e, 256)
        kc, b = divmod(ke // 2, 16)
        blk = (tile * KB + kb) * 18432
        byte = int(t[blk + rg * 1024 + kc * 128 + r * 16 + b])
        want = int(codes[row, e]) if row < n else 0
        assert (byte >> (4 * (e & 1))) & 15 == want
        j, i = divmod((ke % 256) // 16, 4)
        s = int(t[blk + 16384 + j * 512 + (rr % 32) * 16 + (rr // 32) * 4 + i])
        assert s == (int(sb[row, kb * 16 + j * 4 + i]) if row < n else 0)
    c2, s2 = pack.bs_untile(t, n, k)
    assert torch.equal(c2, codes) and torch.equal(s2, sb)
    assert pack.pack_matrix(w[:, :448], "nvfp4", bs=True).w_bs is None  # K % 256 != 0: no copy
