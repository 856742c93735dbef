"""ctypes binding of libstarling_b200.so (include/starling_b200.h).

The product path has no fallback: if the library is missing or a call fails,
this module raises.  Structures mirror the C structs field for field.
"""

from __future__ import annotations

import ctypes as C
import os
from pathlib import Path

_PKG = Path(__file__).resolve().parent
LIB_PATH = Path(os.environ.get("STARLING_B200_LIB", _PKG / "libstarling_b200.so"))

SB_FMT = {"bf16": 0, "fp8": 1, "int8": 2, "nvfp4": 3}
KGROUP_ELEMS = {"bf16": 16, "fp8": 32, "int8": 32, "nvfp4": 64}

SB_CTRL_SLOT, SB_CTRL_PADLEN, SB_CTRL_ACCEPT, SB_CTRL_ERR, SB_CTRL_WORDS = 0, 1, 2, 3, 8
SB_MODE_DECODE, SB_MODE_VERIFY, SB_MODE_FIRST = 0, 1, 2
SB_OP_QKV, SB_OP_ATTN, SB_OP_O, SB_OP_GATE_UP, SB_OP_DOWN, SB_OP_LM_HEAD = range(6)
SB_STEP_PER_OP, SB_STEP_FUSED = 1, 2
SB_NVFP4_AUTO, SB_NVFP4_BLOCK_SCALED, SB_NVFP4_MMA_SYNC = 0, 1, 2
(SB_SPEC_N_EMIT, SB_SPEC_CACHE_POS, SB_SPEC_DRAFT_POS, SB_SPEC_CHUNK, SB_SPEC_STUCK, SB_SPEC_ACCEPTED,
 SB_SPEC_VERIFIES, SB_SPEC_STOPPED, SB_SPEC_ROUNDS, SB_SPEC_K, SB_SPEC_ERR, SB_SPEC_N_DRAFT, SB_SPEC_MAX_NEW,
 SB_SPEC_PROMPT, SB_SPEC_MAX_ROUNDS) = range(15)
SB_SPEC_WORDS = 16

vp = C.c_void_p


class SbLinear(C.Structure):
    _fields_ = [
        ("fmt", C.c_int32), ("n", C.c_int32), ("k", C.c_int32), ("n_pad", C.c_int32),
        ("w", vp), ("scale", vp), ("global_scale", C.c_float), ("_pad", C.c_int32),
        ("w_tc", vp), ("w_bs", vp),
    ]


class SbLayer(C.Structure):
    _fields_ = [
        ("in_norm", vp), ("post_norm", vp),
        ("qkv", SbLinear), ("o", SbLinear), ("gate_up", SbLinear), ("down", SbLinear),
        ("k_cache", vp), ("v_cache", vp),
    ]


class SbModel(C.Structure):
    _fields_ = [
        ("hidden", C.c_int32), ("n_q", C.c_int32), ("n_kv", C.c_int32), ("head_dim", C.c_int32),
        ("inter", C.c_int32), ("vocab", C.c_int32), ("n_layers", C.c_int32), ("max_len", C.c_int32),
        ("max_batch", C.c_int32), ("rope_max_pos", C.c_int32),
        ("eps", C.c_float), ("attn_mult", C.c_float), ("emb_mult", C.c_float), ("res_mult", C.c_float),
        ("logits_mult", C.c_float),
        ("embed", vp), ("final_norm", vp), ("rope_cos", vp), ("rope_sin", vp),
        ("lm_head", SbLinear), ("layers", C.POINTER(SbLayer)),
    ]


class SbState(C.Structure):
    _fields_ = [
        ("batch", C.c_int32), ("m", C.c_int32), ("mode", C.c_int32), ("use_pdl", C.c_int32),
        ("eos_id", C.c_int64), ("pad_id", C.c_int64),
        ("ids", vp), ("ctrl", vp), ("prompt_len", vp), ("rope_off", vp), ("finished", vp),
        ("out_ids", vp), ("hidden", vp), ("q", vp), ("attn", vp), ("act", vp), ("xnorm", vp), ("logits", vp),
        ("workspace", vp), ("workspace_bytes", C.c_size_t),
    ]


class SbSpecLoop(C.Structure):
    _fields_ = [
        ("verify", C.POINTER(SbState)), ("max_chunk", C.c_int32), ("draft_capacity", C.c_int32),
        ("emit_capacity", C.c_int32), ("_pad", C.c_int32), ("eos_id", C.c_int64),
        ("spec", vp), ("emitted", vp), ("draft", vp),
    ]


EXPORTS = [
    "sb_last_error", "sb_version", "sb_workspace_bytes", "sb_decode_step", "sb_lm_head_argmax",
    "sb_linear", "sb_dequant_f32", "sb_dequant_bf16", "sb_rmsnorm", "sb_silu_mul",
    "sb_residual_scale", "sb_rope", "sb_argmax_bf16", "sb_attention", "sb_decode_op",
    "sb_lm_head_argmax_static", "sb_linear_ex", "sb_linear_workspace_bytes", "sb_launch_count",
    "sb_prefill", "sb_prefill_workspace_bytes", "sb_prefill_block_rows", "sb_decode_step_ex",
    "sb_decode_step_fused_ok", "sb_decode_step_scratch_offset", "sb_set_nvfp4_path",
    "sb_spec_loop_create", "sb_spec_loop_launch", "sb_spec_loop_destroy",
]


class StarlingError(RuntimeError):
    pass


_lib = None


def load() -> C.CDLL:
    """Load the library once.  Raises if it is absent: there is no CPU path."""
    global _lib
    if _lib is not None:
        return _lib
    if not LIB_PATH.exists():
        raise StarlingError(
            f"{LIB_PATH} not found: build it with `python -m starling_b200.build` "
            "(the decode path has no fallback implementation)"
        )
    lib = C.CDLL(str(LIB_PATH))
    lib.sb_last_error.restype = C.c_char_p
    lib.sb_launch_count.restype = C.c_uint64
    lib.sb_set_nvfp4_path.restype = C.c_int32
    lib.sb_set_nvfp4_path.argtypes = [C.c_int32]
    lib.sb_prefill_workspace_bytes.restype = C.c_size_t
    lib.sb_prefill_workspace_bytes.argtypes = [C.POINTER(SbModel), C.c_int32, C.c_int32]
    lib.sb_prefill_block_rows.restype = C.c_int32
    lib.sb_prefill_block_rows.argtypes = [C.POINTER(SbModel), C.c_int32, C.c_int32]
    lib.sb_prefill.argtypes = [C.POINTER(SbModel), vp, C.c_int32, C.c_int32, vp, vp, vp, vp, vp, C.c_size_t, vp]
    lib.sb_workspace_bytes.restype = C.c_size_t
    lib.sb_workspace_bytes.argtypes = [C.POINTER(SbModel), C.c_int32]
    lib.sb_decode_step.argtypes = [C.POINTER(SbModel), C.POINTER(SbState), C.c_int32, vp]
    lib.sb_decode_step_ex.argtypes = [C.POINTER(SbModel), C.POINTER(SbState), C.c_int32, C.c_int32, vp]
    lib.sb_decode_step_fused_ok.argtypes = [C.POINTER(SbModel), C.POINTER(SbState)]
    lib.sb_decode_step_fused_ok.restype = C.c_int32
    lib.sb_decode_step_scratch_offset.argtypes = [C.POINTER(SbModel), C.c_int32]
    lib.sb_decode_step_scratch_offset.restype = C.c_size_t
    lib.sb_lm_head_argmax.argtypes = [C.POINTER(SbModel), C.POINTER(SbState), C.c_int32, vp]
    lib.sb_lm_head_argmax_static.argtypes = [C.POINTER(SbModel), C.POINTER(SbState), C.c_int32, vp]
    lib.sb_attention.argtypes = [C.POINTER(SbModel), C.POINTER(SbState), C.c_int32, vp]
    lib.sb_decode_op.argtypes = [C.POINTER(SbModel), C.POINTER(SbState), C.c_int32, C.c_int32, C.c_int32, vp]
    lib.sb_linear.argtypes = [C.POINTER(SbLinear), vp, vp, C.c_int32, C.c_int32, vp]
    lib.sb_linear_ex.argtypes = [C.POINTER(SbLinear), vp, vp, C.c_int32, vp, C.c_size_t, C.c_int32, vp]
    lib.sb_linear_workspace_bytes.restype = C.c_size_t
    lib.sb_linear_workspace_bytes.argtypes = [C.POINTER(SbLinear), C.c_int32]
    lib.sb_dequant_f32.argtypes = [C.POINTER(SbLinear), vp, vp]
    lib.sb_dequant_bf16.argtypes = [C.POINTER(SbLinear), vp, vp]
    lib.sb_rmsnorm.argtypes = [vp, vp, vp, C.c_int32, C.c_int32, C.c_float, vp]
    lib.sb_silu_mul.argtypes = [vp, vp, vp, C.c_int64, vp]
    lib.sb_residual_scale.argtypes = [vp, vp, vp, C.c_int64, C.c_float, vp]
    lib.sb_rope.argtypes = [vp, C.c_int32, C.c_int32, vp, vp, vp, vp]
    lib.sb_argmax_bf16.argtypes = [vp, C.c_int32, C.c_int32, vp, vp]
    lib.sb_spec_loop_create.argtypes = [C.POINTER(SbModel), C.POINTER(SbSpecLoop), C.POINTER(vp)]
    lib.sb_spec_loop_launch.argtypes = [vp, vp]
    lib.sb_spec_loop_destroy.argtypes = [vp]
    lib.sb_spec_loop_destroy.restype = None
    _lib = lib
    return lib


def check(rc: int, what: str = "") -> None:
    if rc != 0:
        msg = load().sb_last_error().decode(errors="replace")
        raise StarlingError(f"{what or 'starling_b200'} failed (code {rc}): {msg}")


def ptr(t) -> int:
    """Device (or host) address of a torch tensor, or 0 for None."""
    return 0 if t is None else int(t.data_ptr())


def current_stream() -> int:
    import torch

    return int(torch.cuda.current_stream().cuda_stream)
