"""Single-step graphed greedy decoder on the native B200 path.

Drop-in for the reference's ``LLMMega`` / ``FusedLLMMega``
(src/starling/granite/llm_mega.py:85-589): same constructor arguments, the
same ``prefill`` / ``capture`` / ``generate`` / ``bench`` methods and result
types, and the attributes ``SpeculativeDecoder`` reaches for
(``static_input_ids``, ``static_logits``, ``_graph``, ``_captured``,
``_reset_cache_pos``, ``_set_mask``, ``max_cache_len``, ``vocab_size`` ...).

What differs underneath: one decode step is ``sb_decode_step`` (about five
fused sm_100a kernels per layer plus the lm_head/argmax kernel) instead of
~240 torch/cuBLAS/Triton launches, the argmax and token feedback happen on
the device, and the cache slot / valid length is a device counter instead of
a host-built mask.
"""

from __future__ import annotations

import statistics
import time
from dataclasses import dataclass
from typing import Any, Optional

import torch

from . import _lib
from .config import LLM_EOS_TOKEN_ID
from .engine import GraniteDims, GraniteEngine, weights_from_hf
from .flags import get_default_flags


@dataclass
class GenerateResult:
    """Output of :meth:`LLMMega.generate` (llm_mega.py:59-67)."""

    ids: torch.Tensor  # (1, n_new) int64 on CPU
    text: str
    n_tokens: int
    total_ms: float
    tok_per_s: float


@dataclass
class BenchReport:
    """Benchmark numbers (llm_mega.py:70-79)."""

    prefill_ms: float = 0.0
    decode_ms_per_token: float = 0.0
    decode_tok_per_s: float = 0.0
    total_ms: float = 0.0
    total_tok_per_s: float = 0.0
    notes: str = ""


def _engine_args(language_model, lm_head, weights, dims):
    if weights is None:
        if language_model is None:
            raise ValueError("pass language_model (HF GraniteModel) or weights=")
        weights = weights_from_hf(language_model, lm_head)
        dims = GraniteDims.from_hf_config(language_model.config)
    if dims is None:
        raise ValueError("dims= is required with weights=")
    return weights, GraniteDims.coerce(dims)


class LLMMega:
    """CUDA-graph-captured greedy decoder (B=1) on the native kernels.

    Args mirror the reference (llm_mega.py:102-110); extra keyword-only
    arguments: ``weight_format`` (bf16 | fp8 | int8 | nvfp4, default from
    :func:`starling_b200.flags.get_default_flags`), ``weights``/``dims`` to
    build from a plain ``{hf_param_name: tensor}`` dict instead of HF modules,
    ``engine`` to share an already packed :class:`GraniteEngine`.
    """

    out_steps = 1

    def __init__(self, language_model: Any = None, lm_head: Any = None, max_cache_len: int = 640,
                 warmup_iters: int = 3, device: str = "cuda", dtype: torch.dtype = torch.bfloat16, *,
                 weight_format: Optional[str] = None, weights: Optional[dict] = None, dims=None,
                 engine: Optional[GraniteEngine] = None, use_pdl: Optional[bool] = None) -> None:
        fl = get_default_flags()
        if dtype != torch.bfloat16:
            raise ValueError("activations are bf16 (the reference's dtype)")
        if engine is None:
            weights, dims = _engine_args(language_model, lm_head, weights, dims)
            engine = GraniteEngine(dims, weights, weight_format or fl.weight_format, max_cache_len, 1, device)
        self.engine = engine
        self.lm = language_model
        self.lm_head = lm_head
        self.config = getattr(language_model, "config", None)
        self.max_cache_len = engine.max_cache_len
        self.warmup_iters = int(warmup_iters)
        self.device = device
        self.dtype = dtype
        self.vocab_size = engine.dims.vocab
        self.num_layers = engine.dims.layers
        self.use_pdl = fl.use_pdl if use_pdl is None else use_pdl
        self.state = engine.new_state(1, 1, _lib.SB_MODE_DECODE, out_steps=self.out_steps, use_pdl=self.use_pdl)
        self.static_input_ids = self.state.ids.view(1, 1)
        self.static_logits = self.state.logits.view(1, 1, self.vocab_size)
        self._neg_val = torch.finfo(dtype).min
        self._graph: Optional[torch.cuda.CUDAGraph] = None
        self._captured = False

    # ------------------------------------------------------------------ #
    @property
    def static_position_ids(self) -> torch.Tensor:
        """Cache slot / RoPE position of the next decode step (device, int32)."""
        return self.state.ctrl[_lib.SB_CTRL_SLOT:_lib.SB_CTRL_SLOT + 1].view(1, 1)

    def _reset_cache_pos(self, n: int) -> None:
        """Set the write slot of the next forward to ``n`` (llm_mega.py:147-150)."""
        self.state.set_slot(n)

    def _set_mask(self, valid_len: int) -> None:
        """Attend to keys [0, valid_len): the next token sits at slot valid_len-1."""
        self.state.set_slot(valid_len - 1)

    def _decode_step_eager(self) -> None:
        self.engine.decode_step(self.state, 0)

    # ------------------------------------------------------------------ #
    @torch.inference_mode()
    def prefill(self, inputs_embeds: torch.Tensor) -> torch.Tensor:
        """Fill the cache with the prompt and return the first token, (1, 1) int64."""
        T = inputs_embeds.shape[1]
        assert T < self.max_cache_len, f"prompt {T} >= max_cache_len {self.max_cache_len}"
        last = self.engine.prefill(inputs_embeds)
        st = self.state
        st.hidden[:1].copy_(last)
        st.set_mode(_lib.SB_MODE_FIRST)
        self.engine.lm_head_argmax(st, 0)
        st.set_mode(_lib.SB_MODE_DECODE)
        st.set_slot(T, pad_len=T)
        return st.ids[:1].view(1, 1).clone()

    def _prime(self, first_token: torch.Tensor, pos: int) -> None:
        self.state.ids[:1].copy_(first_token.reshape(-1)[:1])
        self.state.set_slot(pos, pad_len=pos)

    @torch.inference_mode()
    def capture(self, first_token: torch.Tensor, prefill_len: int) -> None:
        """Capture one decode step into a CUDA graph (llm_mega.py:207-244)."""
        self._prime(first_token, prefill_len)
        for _ in range(self.warmup_iters):
            self._decode_step_eager()
        torch.cuda.synchronize()
        self._prime(first_token, prefill_len)
        self._graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(self._graph):
            self._decode_step_eager()
        self._prime(first_token, prefill_len)
        self._captured = True

    # ------------------------------------------------------------------ #
    def _check_budget(self, T: int, max_new_tokens: int, batch: int) -> None:
        max_safe = self.max_cache_len - T + 1
        if max_new_tokens > max_safe:
            raise ValueError(
                f"max_new_tokens={max_new_tokens} would overflow the static KV cache "
                f"(prompt T={T}, max_cache_len={self.max_cache_len}; at most "
                f"{max_safe} new tokens fit). Increase max_cache_len or reduce max_new_tokens."
            )
        if batch != 1:
            raise ValueError(f"{type(self).__name__} only supports batch=1, got batch={batch}.")

    @torch.inference_mode()
    def generate(self, inputs_embeds: torch.Tensor, max_new_tokens: int = 100,
                 eos_token_id: int = LLM_EOS_TOKEN_ID, tokenizer: Any = None,
                 capture: bool = True) -> GenerateResult:
        """Greedy decode, one graph replay + one host sync per token (llm_mega.py:250-324)."""
        T = inputs_embeds.shape[1]
        self._check_budget(T, max_new_tokens, inputs_embeds.shape[0])
        if max_new_tokens <= 0:
            return self._finalize([], 0.0, tokenizer)
        tok = self.prefill(inputs_embeds)
        gen = [int(tok.item())]
        if max_new_tokens <= 1:
            return self._finalize(gen, 0.0, tokenizer)
        if capture and not self._captured:
            self.capture(tok, T)
        self._prime(tok, T)
        t0 = time.perf_counter()
        for _ in range(max_new_tokens - 1):
            if self._captured:
                self._graph.replay()
            else:
                self._decode_step_eager()
            nxt = int(self.state.out_ids[0].item())
            gen.append(nxt)
            if nxt == eos_token_id:
                break
        torch.cuda.synchronize()
        return self._finalize(gen, (time.perf_counter() - t0) * 1000.0, tokenizer)

    def _finalize(self, gen_ids: list, decode_wall_ms: float, tokenizer: Any) -> GenerateResult:
        ids = torch.tensor(gen_ids, dtype=torch.int64).unsqueeze(0)
        n = len(gen_ids)
        text = tokenizer.decode(ids[0], skip_special_tokens=True) if tokenizer is not None else ""
        return GenerateResult(ids=ids, text=text, n_tokens=n, total_ms=decode_wall_ms,
                              tok_per_s=n / max(decode_wall_ms / 1000.0, 1e-9))

    # ------------------------------------------------------------------ #
    @staticmethod
    def _cuda_timer(fn, warmup: int = 3, iters: int = 20) -> float:
        """Median GPU time (ms) of ``fn`` with CUDA events (llm_mega.py:415-433)."""
        torch.cuda.synchronize()
        for _ in range(warmup):
            fn()
        torch.cuda.synchronize()
        times = []
        for _ in range(iters):
            s = torch.cuda.Event(enable_timing=True)
            e = torch.cuda.Event(enable_timing=True)
            s.record()
            fn()
            e.record()
            torch.cuda.synchronize()
            times.append(s.elapsed_time(e))
        return statistics.median(times)

    @torch.inference_mode()
    def bench(self, inputs_embeds: torch.Tensor, max_new_tokens: int = 100,
              eos_token_id: int = LLM_EOS_TOKEN_ID, decode_iters: int = 20) -> BenchReport:
        """Prefill time, per-token replay time at a fixed position, and a full
        generate (llm_mega.py:347-413)."""
        T = inputs_embeds.shape[1]
        prefill_ms = self._cuda_timer(lambda: self.engine.prefill(inputs_embeds), warmup=1, iters=3)
        first = self.prefill(inputs_embeds)
        self.capture(first, T)

        def one():
            self._graph.replay()
            self._prime(first, T)

        decode_ms = self._cuda_timer(one, warmup=3, iters=decode_iters)
        self._captured = False
        res = self.generate(inputs_embeds, max_new_tokens=max_new_tokens, eos_token_id=eos_token_id)
        return BenchReport(prefill_ms=prefill_ms, decode_ms_per_token=decode_ms,
                           decode_tok_per_s=1000.0 / decode_ms if decode_ms > 0 else 0.0,
                           total_ms=res.total_ms, total_tok_per_s=res.tok_per_s,
                           notes=f"decoded {res.n_tokens} tokens; cache_len={self.max_cache_len}; fmt={self.engine.fmt}")


# The reference's fused variant differs only in its glue kernels; the native
# step is fused already.
FusedLLMMega = LLMMega
