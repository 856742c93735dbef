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
