"""Batched (B streams, lock-step) graphed greedy decoder.

Drop-in for the reference's ``BatchedLLMMega`` / ``BatchedFusedLLMMega``
(src/starling/granite/batched.py:101-588): same constructor and
``generate(inputs_embeds, prompt_lengths, max_new_tokens, eos_token_id)``
returning :class:`BatchedGenerateResult`, same right-padding semantics (each
stream decodes at the shared cache slot with RoPE position
``slot - (T - T_b)`` and never attends to its padding hole
``[T_b, T)``, batched.py:180-200,373-380), same EOS rule (a finished stream
feeds the pad token and its outputs are dropped, batched.py:425-434).

Unlike the reference, which syncs with the host after every step
(batched.py:425-426), the per-stream EOS / pad feedback runs on the device
inside a K-step graph, so the host syncs once per K steps.
"""

from __future__ import annotations

import time
from dataclasses import dataclass
from typing import Any, Optional

import torch

from . import _lib
from .config import LLM_EOS_TOKEN_ID, LLM_PAD_TOKEN_ID
from .engine import GraniteEngine
from .flags import get_default_flags
from .llm_mega import _engine_args


@dataclass
class BatchedGenerateResult:
    """Output of :meth:`BatchedLLMMega.generate` (batched.py:66-95)."""

    ids_list: list
    n_tokens_per_stream: list
    total_tokens: int
    n_streams: int
    prefill_ms: float = 0.0
    decode_ms: float = 0.0
    total_ms: float = 0.0
    max_new_tokens: int = 0

    @property
    def decode_tok_per_s(self) -> float:
        return self.total_tokens / max(self.decode_ms / 1000.0, 1e-9)

    def to_dict(self) -> dict:
        return {
            "n_streams": self.n_streams,
            "total_tokens": self.total_tokens,
            "prefill_ms": round(self.prefill_ms, 3),
            "decode_ms": round(self.decode_ms, 3),
            "total_ms": round(self.total_ms, 3),
            "decode_tok_per_s": round(self.decode_tok_per_s, 1),
            "max_new_tokens": self.max_new_tokens,
        }


class BatchedLLMMega:
    def __init__(self, language_model: Any = None, lm_head: Any = None, max_cache_len: int = 640,
                 max_batch_size: int = 8, warmup_iters: int = 3, device: str = "cuda",
                 dtype: torch.dtype = torch.bfloat16, *, steps_per_replay: int = 8,
                 weight_format: Optional[str] = None, weights: Optional[dict] = None, dims=None,
                 engine: Optional[GraniteEngine] = None, use_pdl: Optional[bool] = None) -> None:
        fl = get_default_flags()
        B = int(max_batch_size)
        if engine is None:
            weights, dims = _engine_args(language_model, lm_head, weights, dims)
            engine = GraniteEngine(dims, weights, weight_format or fl.weight_format, max_cache_len, B, device)
        self.engine = engine
        self.lm, self.lm_head = language_model, lm_head
        self.config = getattr(language_model, "config", None)
        self.max_cache_len = engine.max_cache_len
        self.max_batch_size = B
        self.warmup_iters = int(warmup_iters)
        self.device, self.dtype = device, dtype
        self.vocab_size = engine.dims.vocab
        self.K = max(1, int(steps_per_replay))
        self.use_pdl = fl.use_pdl if use_pdl is None else use_pdl
        self.state = engine.new_state(
            B, 1, _lib.SB_MODE_DECODE, out_steps=self.K, finished=True,
            prompt_len=torch.zeros(B, dtype=torch.int32), rope_off=torch.zeros(B, dtype=torch.int32),
            use_pdl=self.use_pdl,
        )
        self.static_input_ids = self.state.ids.view(B, 1)
        self.static_logits = self.state.logits.view(B, 1, self.vocab_size)
        self._neg_val = torch.finfo(dtype).min
        self._graph: Optional[torch.cuda.CUDAGraph] = None
        self._captured = False

    # ------------------------------------------------------------------ #
    def _reset_cache_pos(self, n: int) -> None:
        self.state.set_slot(n)

    def _set_streams(self, T: int, prompt_lengths: Optional[torch.Tensor]) -> None:
        st = self.state
        pl = torch.full((self.max_batch_size,), T, dtype=torch.int32) if prompt_lengths is None \
            else prompt_lengths.to(torch.int32).cpu()
        st.prompt_len.copy_(pl.to(st.prompt_len.device))
        st.rope_off.copy_((T - pl).to(st.rope_off.device))
        st.set_slot(T, pad_len=T)

    @torch.inference_mode()
    def prefill(self, inputs_embeds: torch.Tensor, prompt_lengths: Optional[torch.Tensor] = None) -> torch.Tensor:
        """Batched prefill + first token per stream, (B, 1) int64 (batched.py:222-276)."""
        B, T = inputs_embeds.shape[:2]
        assert T < self.max_cache_len, f"prompt {T} >= max_cache_len {self.max_cache_len}"
        last = self.engine.prefill(inputs_embeds, prompt_lengths)
        st = self.state
        st.finished.zero_()
        self._set_streams(T, prompt_lengths)
        st.hidden.copy_(last)
        st.set_mode(_lib.SB_MODE_FIRST)
        self.engine.lm_head_argmax(st, 0)
        st.set_mode(_lib.SB_MODE_DECODE)
        return st.out_ids[:B].view(B, 1).clone()

    def _run_k_steps(self) -> None:
        for j in range(self.K):
            self.engine.decode_step(self.state, j)

    def _snapshot(self):
        st = self.state
        return st.ids.clone(), st.finished.clone(), st.ctrl.clone()

    def _restore(self, snap) -> None:
        st = self.state
        st.ids.copy_(snap[0])
        st.finished.copy_(snap[1])
        st.ctrl.copy_(snap[2])

    @torch.inference_mode()
    def capture(self, first_tokens: torch.Tensor = None, prefill_len: int = None,
                prompt_lengths: Optional[torch.Tensor] = None) -> None:
        """Capture K lock-step decode steps into one CUDA graph (batched.py:281-325)."""
        snap = self._snapshot()
        for _ in range(self.warmup_iters):
            self._run_k_steps()
        torch.cuda.synchronize()
        self._restore(snap)
        self._graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(self._graph):
            self._run_k_steps()
        self._restore(snap)
        self._captured = True

    @torch.inference_mode()
    def generate(self, inputs_embeds: torch.Tensor, prompt_lengths: Optional[torch.Tensor] = None,
                 max_new_tokens: int = 200, eos_token_id: int = LLM_EOS_TOKEN_ID) -> BatchedGenerateResult:
        B, T = inputs_embeds.shape[:2]
        if B != self.max_batch_size:
            raise ValueError(
                f"inputs_embeds batch {B} != max_batch_size {self.max_batch_size}; "
                f"construct BatchedLLMMega(max_batch_size={B}) for this batch."
            )
        max_safe = self.max_cache_len - T + 1
        if max_new_tokens > max_safe:
            raise ValueError(
                f"max_new_tokens={max_new_tokens} would overflow the static KV cache "
                f"(prompt T={T}, max_cache_len={self.max_cache_len}; at most {max_safe} new tokens fit)."
            )
        if eos_token_id != self.state.c.eos_id:
            self.state.c.eos_id = int(eos_token_id)
            self._captured = False
        t0 = time.perf_counter()
        first = self.prefill(inputs_embeds, prompt_lengths)
        first_list = first.view(-1).tolist()
        prefill_ms = (time.perf_counter() - t0) * 1000.0
        gen = [[t] for t in first_list]
        finished = [t == eos_token_id for t in first_list]
        if max_new_tokens <= 1 or all(finished):
            return self._finalize(gen, prefill_ms, 0.0, max_new_tokens)
        n_steps = max_new_tokens - 1
        n_chunks = (n_steps + self.K - 1) // self.K
        if T - 1 + n_chunks * self.K >= self.max_cache_len:
            raise ValueError(
                f"K-step rounded-up decode ({n_chunks * self.K} steps, K={self.K}) would overflow the "
                f"static KV cache (prompt T={T}, max_cache_len={self.max_cache_len})."
            )
        if not self._captured:
            self.capture()
        t1 = time.perf_counter()
        steps = 0
        for _ in range(n_chunks):
            self._graph.replay()
            out = self.state.out_ids[: self.K * B].view(self.K, B).tolist()  # one sync per K steps
            for row in out:
                if steps >= n_steps:
                    break
                steps += 1
                for b in range(B):
                    if not finished[b]:
                        gen[b].append(row[b])
                        if row[b] == eos_token_id:
                            finished[b] = True
            if all(finished) or steps >= n_steps:
                break
        torch.cuda.synchronize()
        return self._finalize(gen, prefill_ms, (time.perf_counter() - t1) * 1000.0, max_new_tokens)

    def _finalize(self, gen, prefill_ms, decode_ms, max_new_tokens) -> BatchedGenerateResult:
        ids_list = [torch.tensor(g, dtype=torch.int64) for g in gen]
        n_per = [len(g) for g in gen]
        return BatchedGenerateResult(ids_list=ids_list, n_tokens_per_stream=n_per, total_tokens=sum(n_per),
                                     n_streams=len(gen), prefill_ms=prefill_ms, decode_ms=decode_ms,
                                     total_ms=prefill_ms + decode_ms, max_new_tokens=max_new_tokens)

    def reset(self) -> None:
        """Drop the captured graph and clear the cache (batched.py:459-465)."""
        self._graph = None
        self._captured = False
        self.engine.kv.zero_()


BatchedFusedLLMMega = BatchedLLMMega
