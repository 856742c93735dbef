"""K-step graphed greedy decoder (drop-in for the reference's
``MultiStepLLMMega``, src/starling/granite/multistep.py:69-401).

One CUDA graph holds K consecutive ``sb_decode_step`` calls.  Each step's
lm_head kernel computes the argmax on the device, writes it to
``output_ids[j]``, feeds it back as the next step's input id and advances the
cache slot (multistep.py:157-188), so one replay emits K tokens and the host
syncs once per replay.  Tokens after an EOS inside a chunk are trimmed on the
host (multistep.py:31-41).
"""

from __future__ import annotations

import time
from typing import Any, Optional

import torch

from .config import LLM_EOS_TOKEN_ID
from .llm_mega import BenchReport, GenerateResult, LLMMega


class MultiStepLLMMega(LLMMega):
    def __init__(self, language_model: Any = None, lm_head: Any = None, max_cache_len: int = 640,
                 steps_per_replay: int = 16, warmup_iters: int = 3, device: str = "cuda",
                 dtype: torch.dtype = torch.bfloat16, **kw) -> None:
        self.steps_per_replay = max(1, int(steps_per_replay))
        self.K = self.steps_per_replay
        self.out_steps = self.K
        super().__init__(language_model, lm_head, max_cache_len=max_cache_len, warmup_iters=warmup_iters,
                         device=device, dtype=dtype, **kw)
        self.output_ids = self.state.out_ids[: self.K]
        self._ms_graph: Optional[torch.cuda.CUDAGraph] = None
        self._ms_captured = False

    def _reset_to_chunk_start(self, base: int, first_token: torch.Tensor) -> None:
        """Slot -> base, input id -> first_token (multistep.py:128-152)."""
        self._prime(first_token, base)

    def _run_k_steps(self) -> None:
        for j in range(self.K):
            self.engine.decode_step(self.state, j)

    @torch.inference_mode()
    def capture(self, first_token: torch.Tensor, prefill_len: int) -> None:
        T = int(prefill_len)
        if T + self.K > self.max_cache_len:
            raise ValueError(
                f"K={self.K} captured steps would overflow the static KV cache "
                f"(prompt T={T}, max_cache_len={self.max_cache_len}; need "
                f"T + K <= max_cache_len). Reduce K or max_cache_len."
            )
        super().capture(first_token, T)  # single-step graph, for SpeculativeDecoder
        self._reset_to_chunk_start(T, first_token)
        for _ in range(self.warmup_iters):
            self._run_k_steps()
        torch.cuda.synchronize()
        self._reset_to_chunk_start(T, first_token)
        self._ms_graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(self._ms_graph):
            self._run_k_steps()
        self._reset_to_chunk_start(T, first_token)
        self._ms_captured = True

    @torch.inference_mode()
    def generate(self, inputs_embeds: torch.Tensor, max_new_tokens: int = 100,
                 eos_token_id: int = LLM_EOS_TOKEN_ID, tokenizer: Any = None,
                 capture: bool = True) -> GenerateResult:
        T = inputs_embeds.shape[1]
        max_safe = self.max_cache_len - T + 1
        if max_new_tokens > max_safe:
            raise ValueError(
                f"max_new_tokens={max_new_tokens} would overflow the static KV "
                f"cache (prompt T={T}, max_cache_len={self.max_cache_len}; at "
                f"most {max_safe} new tokens fit)."
            )
        if inputs_embeds.shape[0] != 1:
            raise ValueError(f"MultiStepLLMMega only supports batch=1, got batch={inputs_embeds.shape[0]}.")
        if max_new_tokens <= 0:
            return self._finalize([], 0.0, tokenizer)
        K = self.K
        n_decode = max_new_tokens - 1
        tok = self.prefill(inputs_embeds)
        gen = [int(tok.item())]
        if max_new_tokens <= 1 or n_decode <= 0:
            return self._finalize(gen, 0.0, tokenizer)
        n_chunks = (n_decode + K - 1) // K
        total_steps = n_chunks * K
        if T - 1 + total_steps >= self.max_cache_len:
            raise ValueError(
                f"multi-step rounded-up decode ({total_steps} steps across "
                f"{n_chunks} chunks of K={K}) would overflow the static KV cache "
                f"(prompt T={T}, max_cache_len={self.max_cache_len}). Reduce K "
                f"or max_new_tokens."
            )
        if capture and not self._ms_captured:
            self.capture(tok, T)
        self._reset_to_chunk_start(T, tok)
        t0 = time.perf_counter()
        done = False
        for _ in range(n_chunks):
            if self._ms_captured:
                self._ms_graph.replay()
            else:
                self._run_k_steps()
            for t in self.output_ids.tolist():  # one device->host sync per K tokens
                if len(gen) >= max_new_tokens:
                    done = True
                    break
                gen.append(t)
                if t == eos_token_id:
                    done = True
                    break
            if done:
                break
        torch.cuda.synchronize()
        return self._finalize(gen, (time.perf_counter() - t0) * 1000.0, tokenizer)

    @torch.inference_mode()
    def bench(self, inputs_embeds: torch.Tensor, max_new_tokens: int = 100,
              eos_token_id: int = LLM_EOS_TOKEN_ID, decode_iters: int = 10) -> BenchReport:
        """Per-token time = K-step replay / K (multistep.py:338-401)."""
        T = inputs_embeds.shape[1]
        prefill_ms = self._cuda_timer(lambda: self.engine.prefill(inputs_embeds), warmup=1, iters=3)
        first = self.prefill(inputs_embeds)
        self.capture(first, T)

        def k_replay():
            self._ms_graph.replay()
            self._reset_to_chunk_start(T, first)

        replay_ms = self._cuda_timer(k_replay, warmup=3, iters=decode_iters)
        decode_ms = replay_ms / self.K
        self._ms_captured = False
        res = self.generate(inputs_embeds, max_new_tokens=max_new_tokens, eos_token_id=eos_token_id)
        return BenchReport(prefill_ms=prefill_ms, decode_ms_per_token=decode_ms,
                           decode_tok_per_s=1000.0 / decode_ms if decode_ms > 0 else 0.0,
                           total_ms=res.total_ms, total_tok_per_s=res.tok_per_s,
                           notes=f"decoded {res.n_tokens} tokens; K={self.K}; cache_len={self.max_cache_len}; "
                                 f"fmt={self.engine.fmt}")
