"""The C ABI without a GPU: the library loads, exports every function that
include/starling_b200.h declares, and the ctypes structs match the C layout
(checked by compiling a small C program against the header)."""

import ctypes as C
import re
import subprocess
import tempfile
from pathlib import Path

import pytest

from starling_b200 import _lib
from starling_b200.flags import OptFlags, flags, get_default_flags

REPO = Path(__file__).resolve().parent.parent
HEADER = REPO / "include" / "starling_b200.h"


def declared_functions():
    text = HEADER.read_text()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"\b(sb_[a-z0-9_]+)\s*\(", text)))


@pytest.fixture(scope="module")
def lib():
    if not _lib.LIB_PATH.exists():
        from starling_b200 import build

        build.build()
    return _lib.load()


def test_exports_every_declared_symbol(lib):
    names = declared_functions()
    assert len(names) >= 14
    for n in names:
        assert hasattr(lib, n), f"{n} declared in the header but not exported"
    assert set(names) == set(_lib.EXPORTS)


def test_host_only_calls(lib):
    assert lib.sb_version() == 1
    assert isinstance(lib.sb_last_error(), bytes)
    assert lib.sb_workspace_bytes(None, 1) == 0


def test_struct_layout_matches_header(tmp_path):
    src = tmp_path / "layout.c"
    src.write_text(
        '#include <stdio.h>\n#include <stddef.h>\n#include "starling_b200.h"\n'
        "#define P(T, f) printf(#T \".\" #f \" %zu\\n\", offsetof(T, f));\n"
        "int main(void){\n"
        'printf("SbLinear %zu\\nSbLayer %zu\\nSbModel %zu\\nSbState %zu\\nSbSpecLoop %zu\\n", sizeof(SbLinear),'
        " sizeof(SbLayer), sizeof(SbModel), sizeof(SbState), sizeof(SbSpecLoop));\n"
        "P(SbLinear, w) P(SbLinear, global_scale) P(SbLinear, w_tc) P(SbLinear, w_bs) P(SbLayer, qkv) P(SbLayer, k_cache) P(SbModel, eps)"
        " P(SbModel, embed) P(SbModel, lm_head) P(SbModel, layers) P(SbState, eos_id) P(SbState, ids)"
        " P(SbState, workspace_bytes) P(SbSpecLoop, max_chunk) P(SbSpecLoop, eos_id) P(SbSpecLoop, spec)"
        " P(SbSpecLoop, draft)\nreturn 0;}\n"
    )
    exe = tmp_path / "layout"
    subprocess.run(["gcc", "-I", str(REPO / "include"), str(src), "-o", str(exe)], check=True)
    out = dict(line.split() for line in subprocess.run([str(exe)], capture_output=True, text=True).stdout.splitlines())
    assert int(out["SbLinear"]) == C.sizeof(_lib.SbLinear)
    assert int(out["SbLayer"]) == C.sizeof(_lib.SbLayer)
    assert int(out["SbModel"]) == C.sizeof(_lib.SbModel)
    assert int(out["SbState"]) == C.sizeof(_lib.SbState)
    assert int(out["SbSpecLoop"]) == C.sizeof(_lib.SbSpecLoop)
    for key, val in out.items():
        if "." in key:
            t, f = key.split(".")
            assert int(val) == getattr(_lib, t).__dict__[f].offset, key


def test_missing_library_fails_loudly(monkeypatch, tmp_path):
    monkeypatch.setattr(_lib, "LIB_PATH", tmp_path / "nope.so")
    monkeypatch.setattr(_lib, "_lib", None)
    with pytest.raises(_lib.StarlingError):
        _lib.load()


def test_flags():
    assert get_default_flags().multistep_graph
    with pytest.raises(ValueError):
        OptFlags(batched_encoder=True)
    with pytest.raises(ValueError):
        OptFlags(weight_format="fp16")
    with flags(weight_format="nvfp4") as f:
        assert f.weight_format == "nvfp4" and get_default_flags().weight_format == "nvfp4"
    assert get_default_flags().weight_format == "bf16"


def _fake_model(fmt, gate_up_n=None, hidden=2048, inter=8192, n_q=16, n_kv=4, layers=2):
    """An SbModel of the Granite-1B decoder's dimensions whose device pointers
    are placeholders: only host-side planning (sb_workspace_bytes) may see it."""
    fake = 0x10000

    def lin(n, k):
        return _lib.SbLinear(fmt=_lib.SB_FMT[fmt], n=n, k=k, n_pad=(n + 127) // 128 * 128, w=fake, scale=fake,
                             global_scale=1.0, w_tc=fake, w_bs=None)

    arr = (_lib.SbLayer * layers)()
    for i in range(layers):
        arr[i].in_norm = arr[i].post_norm = arr[i].k_cache = arr[i].v_cache = fake
        arr[i].qkv = lin((n_q + 2 * n_kv) * 128, hidden)
        arr[i].o = lin(hidden, n_q * 128)
        arr[i].gate_up = lin(gate_up_n or 2 * inter, hidden)
        arr[i].down = lin(hidden, inter)
    md = _lib.SbModel(hidden=hidden, n_q=n_q, n_kv=n_kv, head_dim=128, inter=inter, vocab=100352, n_layers=layers,
                      max_len=1040, max_batch=64, rope_max_pos=4096, eps=1e-5, attn_mult=1.0, emb_mult=12.0,
                      res_mult=0.22, logits_mult=0.125, embed=fake, final_norm=fake, rope_cos=fake, rope_sin=fake,
                      lm_head=lin(100352, hidden), layers=arr)
    return md, arr


@pytest.mark.parametrize("fmt,T", [("fp8", 8), ("fp8", 9), ("fp8", 12), ("fp8", 48), ("fp8", 64), ("fp8", 65),
                                   ("bf16", 48)])
def test_decode_chain_workspace(lib, fmt, T):
    """The workspace of an fp8 model at 9..64 token rows holds the decode
    chain's buffers -- the hidden-wide and inter-wide block-scaled operands
    (per 128-element K block: 2 x pad8(T) rows of 128 e4m3 bytes + 512 bytes
    of scales) and the [64][hidden / 32] sums of squares -- and no other
    case does.  The comparison model differs only in a gate/up row count
    that breaks gate/up = 2 x inter, which the chain requires."""
    def bs_bytes(k):
        return (k // 128) * (2 * ((T + 7) // 8 * 8) * 128 + 512)

    def up(x):
        return (x + 255) // 256 * 256

    md, keep = _fake_model(fmt)
    md2, keep2 = _fake_model(fmt, gate_up_n=2 * 8192 + 128)
    diff = lib.sb_workspace_bytes(C.byref(md), T) - lib.sb_workspace_bytes(C.byref(md2), T)
    if fmt == "fp8" and 9 <= T <= 64:
        chain = up(bs_bytes(2048)) + up(bs_bytes(8192)) + 2048 // 32 * 64 * 4
        assert 0 <= diff - chain < 256  # plus the region's 256-byte alignment
    else:
        assert diff == 0
