"""GraniteEngine: packed weights, static KV cache and device state for the
native decode path, plus the prefill that fills the cache (``sb_prefill``).

The decode / verify forward itself is one C-ABI call per step
(``sb_decode_step``) issuing the fused sm_100a kernels; everything it reads
(token ids, cache slot, finished flags) lives in device tensors owned here, so
a CUDA graph captured once is replayed for every chunk.
"""

from __future__ import annotations

import ctypes as C
from dataclasses import dataclass, fields
from typing import Optional

import torch

from . import _lib
from ._lib import SB_CTRL_PADLEN, SB_CTRL_SLOT, SB_CTRL_WORDS, SbLayer, SbModel, SbState, check, ptr
from .config import LLM_EOS_TOKEN_ID, LLM_PAD_TOKEN_ID
from .pack import PackedLinear, pack_gate_up, pack_matrix, pack_qkv
from .rope import rope_tables

BF16 = torch.bfloat16


@dataclass(frozen=True)
class GraniteDims:
    hidden: int = 2048
    n_q: int = 16
    n_kv: int = 4
    head_dim: int = 128
    inter: int = 8192
    vocab: int = 100352
    layers: int = 40
    eps: float = 1e-5
    theta: float = 10000.0
    attn_mult: float = 0.0078125
    emb_mult: float = 12.0
    res_mult: float = 0.22
    logits_scaling: float = 8.0

    @classmethod
    def from_hf_config(cls, cfg) -> "GraniteDims":
        rp = getattr(cfg, "rope_parameters", None) or {}
        theta = rp.get("rope_theta", getattr(cfg, "rope_theta", 10000.0))
        return cls(
            hidden=cfg.hidden_size, n_q=cfg.num_attention_heads, n_kv=cfg.num_key_value_heads,
            head_dim=getattr(cfg, "head_dim", None) or cfg.hidden_size // cfg.num_attention_heads,
            inter=cfg.intermediate_size, vocab=cfg.vocab_size, layers=cfg.num_hidden_layers,
            eps=cfg.rms_norm_eps, theta=float(theta), attn_mult=cfg.attention_multiplier,
            emb_mult=cfg.embedding_multiplier, res_mult=cfg.residual_multiplier,
            logits_scaling=cfg.logits_scaling,
        )

    @classmethod
    def coerce(cls, d) -> "GraniteDims":
        if isinstance(d, cls):
            return d
        names = {f.name for f in fields(cls)}
        src = d if isinstance(d, dict) else d.__dict__
        return cls(**{k: v for k, v in src.items() if k in names})


def weights_from_hf(language_model, lm_head=None) -> dict:
    """HF GraniteModel (+ lm_head) -> {HF parameter name: tensor}."""
    w = {k: v for k, v in language_model.state_dict().items() if "rotary" not in k}
    if lm_head is not None and lm_head.weight.data_ptr() != w["embed_tokens.weight"].data_ptr():
        w["lm_head.weight"] = lm_head.weight
    return w


class EngineState:
    """Device buffers and the C ``SbState`` for one forward shape (batch, m)."""

    def __init__(self, eng: "GraniteEngine", batch: int, m: int, mode: int, out_steps: int = 1,
                 finished: bool = False, prompt_len: Optional[torch.Tensor] = None,
                 rope_off: Optional[torch.Tensor] = None, keep_logits: bool = True,
                 use_pdl: bool = True, share: Optional["EngineState"] = None):
        """share: use that state's ids, ctrl and out_ids buffers (at least as
        large as this state's) instead of new ones."""
        d, dev = eng.dims, eng.device
        T = batch * m
        self.batch, self.m = batch, m
        if share is not None and (share.ids.numel() < T or share.out_ids.numel() < max(out_steps, 1) * max(batch, m)):
            raise ValueError("the shared state's buffers are smaller than this state's")
        self.ids = share.ids if share is not None else torch.zeros(T, dtype=torch.int64, device=dev)
        self.ctrl = share.ctrl if share is not None else torch.zeros(SB_CTRL_WORDS, dtype=torch.int32, device=dev)
        self.prompt_len = None if prompt_len is None else prompt_len.to(dev, torch.int32).contiguous()
        self.rope_off = None if rope_off is None else rope_off.to(dev, torch.int32).contiguous()
        self.finished = torch.zeros(batch, dtype=torch.int32, device=dev) if finished else None
        self.out_ids = (share.out_ids if share is not None else
                        torch.zeros(max(out_steps, 1) * max(batch, m), dtype=torch.int64, device=dev))
        self.hidden = torch.zeros(T, d.hidden, dtype=BF16, device=dev)
        self.q = torch.zeros(T, d.n_q * d.head_dim, dtype=BF16, device=dev)
        self.attn = torch.zeros(T, d.n_q * d.head_dim, dtype=BF16, device=dev)
        self.act = torch.zeros(T, d.inter, dtype=BF16, device=dev)
        self.xnorm = torch.zeros(T, d.hidden, dtype=BF16, device=dev)
        self.logits = torch.zeros(T, d.vocab, dtype=BF16, device=dev) if keep_logits else None
        nbytes = eng.lib.sb_workspace_bytes(C.byref(eng.cmodel), T)
        self.workspace = torch.zeros(max(nbytes, 256), dtype=torch.uint8, device=dev)
        s = SbState()
        s.batch, s.m, s.mode, s.use_pdl = batch, m, mode, int(use_pdl)
        s.eos_id, s.pad_id = LLM_EOS_TOKEN_ID, LLM_PAD_TOKEN_ID
        s.ids, s.ctrl = ptr(self.ids), ptr(self.ctrl)
        s.prompt_len, s.rope_off, s.finished = ptr(self.prompt_len), ptr(self.rope_off), ptr(self.finished)
        s.out_ids, s.hidden, s.q, s.attn, s.act = (ptr(self.out_ids), ptr(self.hidden), ptr(self.q),
                                                   ptr(self.attn), ptr(self.act))
        s.logits = ptr(self.logits)
        s.xnorm = ptr(self.xnorm)
        s.workspace, s.workspace_bytes = ptr(self.workspace), self.workspace.numel()
        self.c = s

    def set_mode(self, mode: int) -> None:
        self.c.mode = mode

    def set_slot(self, slot: int, pad_len: Optional[int] = None) -> None:
        self.ctrl[SB_CTRL_SLOT] = int(slot)
        if pad_len is not None:
            self.ctrl[SB_CTRL_PADLEN] = int(pad_len)


class GraniteEngine:
    def __init__(self, dims, weights: dict, fmt: str = "bf16", max_cache_len: int = 640,
                 max_batch: int = 1, device="cuda", rope_max_pos: Optional[int] = None,
                 tensor_cores: bool = True, block_scaled: bool = True):
        """tensor_cores: also keep the tcgen05 tile copy of every fp8 / bf16
        weight, which serves 9..128 token rows (batched decode, verify,
        prefill); it doubles the weight memory of those formats.
        block_scaled: also keep the block-scaled tcgen05 copy of every NVFP4
        weight (same bytes as the packed weight), which the library uses for
        1..8 token rows where it is faster (sb_set_nvfp4_path)."""
        self.lib = _lib.load()
        self.dims = d = GraniteDims.coerce(dims)
        if d.head_dim != 128:
            raise ValueError("the native kernels use head_dim 128")
        self.fmt = fmt
        self.device = torch.device(device)
        self.max_cache_len = int(max_cache_len)
        self.max_batch = int(max_batch)
        dev = self.device

        def W(name):
            return weights[name].detach().to(dev, BF16)

        self.embed = W("embed_tokens.weight").contiguous()
        self.final_norm = W("norm.weight").contiguous()
        head_w = weights.get("lm_head.weight", None)
        tc = bool(tensor_cores)
        bs = bool(block_scaled)
        self.lm_head = pack_matrix(self.embed if head_w is None else W("lm_head.weight"), fmt, tc=tc, bs=bs)
        self.layers = []
        for i in range(d.layers):
            p = f"layers.{i}."
            L = dict(
                in_norm=W(p + "input_layernorm.weight").contiguous(),
                post_norm=W(p + "post_attention_layernorm.weight").contiguous(),
                qkv=pack_qkv(W(p + "self_attn.q_proj.weight"), W(p + "self_attn.k_proj.weight"),
                             W(p + "self_attn.v_proj.weight"), d.n_q, d.n_kv, fmt, tc=tc, bs=bs),
                o=pack_matrix(W(p + "self_attn.o_proj.weight"), fmt, tc=tc, bs=bs),
                gate_up=pack_gate_up(W(p + "mlp.gate_proj.weight"), W(p + "mlp.up_proj.weight"), fmt, tc=tc, bs=bs),
                down=pack_matrix(W(p + "mlp.down_proj.weight"), fmt, tc=tc, bs=bs),
            )
            self.layers.append(L)
        # static KV cache: [layer][k|v][batch][n_kv][max_len][128] (StaticLayer layout per layer)
        self.kv = torch.zeros(d.layers, 2, max_batch, d.n_kv, self.max_cache_len, d.head_dim, dtype=BF16, device=dev)
        self.rope_max_pos = int(rope_max_pos or max(4096, self.max_cache_len))
        cs, sn = rope_tables(d.head_dim, d.theta, self.rope_max_pos)
        self.rope_cos, self.rope_sin = cs.to(dev), sn.to(dev)
        self._build_c()

    # ------------------------------------------------------------------ #
    def _build_c(self) -> None:
        d = self.dims
        arr = (SbLayer * d.layers)()
        for i, L in enumerate(self.layers):
            arr[i].in_norm = ptr(L["in_norm"])
            arr[i].post_norm = ptr(L["post_norm"])
            arr[i].qkv = L["qkv"].c_struct()
            arr[i].o = L["o"].c_struct()
            arr[i].gate_up = L["gate_up"].c_struct()
            arr[i].down = L["down"].c_struct()
            arr[i].k_cache = ptr(self.kv[i, 0])
            arr[i].v_cache = ptr(self.kv[i, 1])
        m = SbModel()
        m.hidden, m.n_q, m.n_kv, m.head_dim = d.hidden, d.n_q, d.n_kv, d.head_dim
        m.inter, m.vocab, m.n_layers = d.inter, d.vocab, d.layers
        m.max_len, m.max_batch, m.rope_max_pos = self.max_cache_len, self.max_batch, self.rope_max_pos
        m.eps, m.attn_mult, m.emb_mult, m.res_mult = d.eps, d.attn_mult, d.emb_mult, d.res_mult
        m.logits_mult = 1.0 / d.logits_scaling
        m.embed, m.final_norm = ptr(self.embed), ptr(self.final_norm)
        m.rope_cos, m.rope_sin = ptr(self.rope_cos), ptr(self.rope_sin)
        m.lm_head = self.lm_head.c_struct()
        m.layers = C.cast(arr, C.POINTER(SbLayer))
        self._layer_arr = arr
        self.cmodel = m

    @property
    def weight_bytes(self) -> int:
        n = self.lm_head.nbytes
        for L in self.layers:
            n += sum(L[k].nbytes for k in ("qkv", "o", "gate_up", "down"))
        return n

    def new_state(self, batch: int = 1, m: int = 1, mode: int = _lib.SB_MODE_DECODE, **kw) -> EngineState:
        if batch > self.max_batch:
            raise ValueError(f"batch {batch} > engine max_batch {self.max_batch}")
        return EngineState(self, batch, m, mode, **kw)

    # ---- native calls ----------------------------------------------------- #
    # decode-step kernel path: "auto" (the library's default: the fused step for
    # forwards of one stream where it serves them, else the per-op kernels),
    # "fused" (required), "prefer_fused" (fused wherever it serves the
    # forward) or "ops" (per-op kernels only)
    step_path = "auto"

    def decode_step(self, st: EngineState, step: int = 0) -> None:
        if not 0 <= step < st.out_ids.numel() // max(st.batch, st.m):
            raise ValueError(f"step {step} outside the state's output ring")
        path = self.step_path
        if path == "prefer_fused":
            path = "fused" if self.fused_step_ok(st) else "ops"
        flags = {"auto": 0, "ops": _lib.SB_STEP_PER_OP, "fused": _lib.SB_STEP_FUSED}[path]
        check(self.lib.sb_decode_step_ex(C.byref(self.cmodel), C.byref(st.c), int(step), flags,
                                         _lib.current_stream()), "sb_decode_step")

    def fused_step_ok(self, st: EngineState) -> bool:
        """Whether the one-launch fused step serves forwards of this state."""
        return bool(self.lib.sb_decode_step_fused_ok(C.byref(self.cmodel), C.byref(st.c)))

    def lm_head_argmax(self, st: EngineState, step: int = 0) -> None:
        check(self.lib.sb_lm_head_argmax(C.byref(self.cmodel), C.byref(st.c), int(step), _lib.current_stream()),
              "sb_lm_head_argmax")

    def dequant(self, p: PackedLinear, f32: bool = True) -> torch.Tensor:
        """Packed -> dense weight in LOGICAL row order (fp32 exact, or bf16)."""
        out = torch.empty(p.n, p.k, dtype=torch.float32 if f32 else BF16, device=self.device)
        fn = self.lib.sb_dequant_f32 if f32 else self.lib.sb_dequant_bf16
        c = p.c_struct()
        check(fn(C.byref(c), ptr(out), _lib.current_stream()), "sb_dequant")
        if p.row_perm is not None:
            out = out[self._inverse_perm(p)]
        return out

    # ---- single linears and prefill --------------------------------------- #
    def linear(self, x: torch.Tensor, p: PackedLinear) -> torch.Tensor:
        """y = x W^T through the native dequant-GEMV (any number of rows; fp32
        accumulation over the exactly dequantised weight).  Output columns in
        LOGICAL row order."""
        shp = x.shape
        x2 = x.reshape(-1, shp[-1]).to(BF16).contiguous()
        y = torch.empty(x2.shape[0], p.n, dtype=BF16, device=self.device)
        c = p.c_struct()
        need = int(self.lib.sb_linear_workspace_bytes(C.byref(c), x2.shape[0]))
        ws = getattr(self, "_lin_ws", None)
        if need and (ws is None or ws.numel() < need):
            self._lin_ws = ws = torch.zeros(need, dtype=torch.uint8, device=self.device)
        check(self.lib.sb_linear_ex(C.byref(c), ptr(x2), ptr(y), x2.shape[0], ptr(ws) if need else None,
                                    ws.numel() if need else 0, 0, _lib.current_stream()), "sb_linear_ex")
        if p.row_perm is not None:
            y = y[:, self._inverse_perm(p)]
        return y.view(*shp[:-1], p.n)

    def _inverse_perm(self, p: PackedLinear) -> torch.Tensor:
        inv = getattr(p, "_inv", None)
        if inv is None:
            inv = torch.empty_like(p.row_perm)
            inv[p.row_perm] = torch.arange(p.row_perm.numel(), device=p.row_perm.device)
            p._inv = inv = inv.to(self.device)
        return inv

    @torch.inference_mode()
    def prefill(self, inputs_embeds: torch.Tensor, prompt_lengths: Optional[torch.Tensor] = None) -> torch.Tensor:
        """Prefill over ``inputs_embeds`` (B, T, H) (before the x12 embedding
        multiplier), writing cache slots [0, T) of streams 0..B-1: the
        ``GraniteModel.forward`` with a causal (+ right-padding) mask of
        llm_mega.py:176-202 / batched.py:222-276, run by the library's
        ``sb_prefill``.  Returns the last real position's hidden row per
        stream, before the final norm: (B, H).  Raises ``StarlingError`` where
        the library does not serve the shape (there is no other path)."""
        d = self.dims
        B, T, _ = inputs_embeds.shape
        if T >= self.max_cache_len:
            raise ValueError(f"prompt {T} >= max_cache_len {self.max_cache_len}")
        Tp = (T + 7) // 8 * 8  # sb_prefill takes whole query blocks of 8 positions
        if Tp > self.max_cache_len or B > self.max_batch:
            raise ValueError(f"prefill needs T rounded up to 8 ({Tp}) <= max_cache_len {self.max_cache_len} "
                             f"and B ({B}) <= max_batch {self.max_batch}")
        dev = self.device
        hidden = torch.zeros(B, Tp, d.hidden, dtype=BF16, device=dev)
        hidden[:, :T] = inputs_embeds.to(dev, BF16) * d.emb_mult
        pl = None
        if prompt_lengths is not None:
            pl = prompt_lengths.to(dev, torch.int32).contiguous()
        elif Tp != T:
            pl = torch.full((B,), T, dtype=torch.int32, device=dev)
        m = C.byref(self.cmodel)
        ws_bytes = int(self.lib.sb_prefill_workspace_bytes(m, B, Tp))
        rows = int(self.lib.sb_prefill_block_rows(m, B, Tp))
        q = torch.empty(B * Tp, d.n_q * d.head_dim, dtype=BF16, device=dev)
        attn = torch.empty_like(q)
        act = torch.empty(rows, d.inter, dtype=BF16, device=dev)
        ws = torch.zeros(ws_bytes, dtype=torch.uint8, device=dev)
        check(self.lib.sb_prefill(m, ptr(hidden), B, Tp, ptr(pl), ptr(q), ptr(attn), ptr(act), ptr(ws), ws_bytes,
                                  _lib.current_stream()), "sb_prefill")
        last = (pl.long() - 1) if pl is not None else torch.full((B,), T - 1, device=dev)
        return hidden[torch.arange(B, device=dev), last, :].contiguous()

    def load_cache_from(self, k_list, v_list, batch_index: int = 0) -> None:
        """Copy externally computed K/V (per layer (n_kv, S, 128) or (B, n_kv, S, 128)) into slots [0, S)."""
        for li, (k, v) in enumerate(zip(k_list, v_list)):
            if k.dim() == 3:
                k, v = k[None], v[None]
            S = k.shape[2]
            b1 = batch_index + k.shape[0]
            self.kv[li, 0, batch_index:b1, :, :S] = k.to(self.device, BF16)
            self.kv[li, 1, batch_index:b1, :, :S] = v.to(self.device, BF16)
