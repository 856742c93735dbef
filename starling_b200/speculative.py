"""Self-speculative greedy decoding on the native verify forward.

Drop-in for the reference's ``SpeculativeDecoder``
(src/starling/granite/speculative.py:242-852), keeping its loop exactly:
verify ``[last_token, draft_chunk]`` (L = k+1 tokens) in one forward, accept
the longest prefix whose greedy argmax equals the draft, emit the greedy
correction (or the free bonus token on full acceptance), rewind the cache to
the last emitted token, re-align the draft pointer, adapt the chunk size
8 -> 12 -> 16 (2 inside formatting boundaries), and fall back to single-step
decode once the draft is exhausted (speculative.py:400-567).

The verify forward is ``sb_decode_step`` with m = L: every projection is a
skinny GEMM over the L rows, attention applies the causal verify mask
(query i sees keys [0, start+i], speculative.py:755-765) on the device, and
the lm_head kernel returns the L argmaxes plus the accepted-prefix length.
One CUDA graph per L is captured up front (speculative.py:685-781).

By default (``device_loop=True``) the whole verify / accept loop runs on the
device as one CUDA graph (``sb_spec_loop_*``): a WHILE node over rounds whose
body switches to the captured verify forward of the round's chunk length,
followed by a control kernel that applies the rules above and plans the next
round, so the host reads the emitted ids once, after the loop, instead of
after every verify.  ``device_loop=False`` runs the same loop on the host, one
graph replay and one device->host read per round, as the reference does.
The CTC draft extraction (speculative.py:93-236) belongs to the encoder side
and is not part of this package: callers pass the draft ids.
"""

from __future__ import annotations

import ctypes as C
import time
from dataclasses import dataclass
from typing import Any, Optional

import torch

from . import _lib
from ._lib import check, ptr
from .config import LLM_EOS_TOKEN_ID


@dataclass
class SpecResult:
    """Output of :meth:`SpeculativeDecoder.generate` (speculative.py:60-87)."""

    ids: torch.Tensor
    text: str
    n_tokens: int
    total_ms: float
    tok_per_s: float
    draft_count: int
    accepted: int
    verify_forwards: int
    acceptance_rate: float
    decode_steps: int = 0
    decode_probes: int = 0


class SpeculativeDecoder:
    MIN_CHUNK: int = 8
    BOUNDARY_CHUNK: int = 2
    MAX_CHUNK: int = 16

    def __init__(self, llm: Any, embed_tokens: Any = None, device_loop: bool = True) -> None:
        self.llm = llm
        self.engine = llm.engine
        self.embed_tokens = embed_tokens
        self.device_loop = bool(device_loop)
        self._verify_graphs: dict = {}
        self._pinned = torch.zeros(self.MAX_CHUNK + 1, dtype=torch.int64).pin_memory()
        self._loop = None  # the device loop's graph and buffers, built on first use

    # ------------------------------------------------------------------ #
    def _capture_verify_graph(self, L: int) -> None:
        llm = self.llm
        st = self.engine.new_state(1, L, _lib.SB_MODE_VERIFY, out_steps=1, use_pdl=llm.use_pdl)
        capture_pos = llm.max_cache_len - L - 2
        st.ids.fill_(1)
        for _ in range(3):
            st.set_slot(capture_pos)
            self.engine.decode_step(st, 0)
        torch.cuda.synchronize()
        st.set_slot(capture_pos)
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g):
            self.engine.decode_step(st, 0)
        self._verify_graphs[L] = (st, g)

    def warmup_graphs(self, chunk_sizes: Optional[tuple] = None) -> None:
        if chunk_sizes is None:
            chunk_sizes = tuple(range(1, self.MAX_CHUNK + 1))
        for cs in chunk_sizes:
            if cs + 1 not in self._verify_graphs:
                self._capture_verify_graph(cs + 1)

    def verify(self, ids: list, start_pos: int):
        """One verify forward of ``ids`` (L tokens) at cache slots
        [start_pos, start_pos+L).  Returns (argmax per position, accepted
        prefix length vs ids[1:]) with one device->host sync."""
        L = len(ids)
        if L not in self._verify_graphs:
            self._capture_verify_graph(L)
        st, g = self._verify_graphs[L]
        self._pinned[:L] = torch.tensor(ids, dtype=torch.int64)
        st.ids.copy_(self._pinned[:L], non_blocking=True)
        st.set_slot(start_pos)
        g.replay()
        res = torch.cat([st.out_ids[:L], st.ctrl[_lib.SB_CTRL_ACCEPT:_lib.SB_CTRL_ACCEPT + 1].long()]).tolist()
        return res[:L], res[L]

    # ------------------------------------------------------------------ #
    def _device_loop(self, eos: int, n_draft: int) -> dict:
        """The loop graph (sb_spec_loop_create) and its buffers: built once,
        rebuilt only for a new EOS id or a longer draft."""
        lp = self._loop
        if lp is not None and lp["eos"] == eos and lp["draft"].numel() >= n_draft:
            return lp
        if lp is not None:
            self.engine.lib.sb_spec_loop_destroy(lp["handle"])
            self._loop = None
        eng, llm = self.engine, self.llm
        dev = eng.device
        big = eng.new_state(1, self.MAX_CHUNK + 1, _lib.SB_MODE_VERIFY, out_steps=1, use_pdl=False)
        states = [eng.new_state(1, k + 1, _lib.SB_MODE_VERIFY, out_steps=1, use_pdl=False, share=big)
                  for k in range(1, self.MAX_CHUNK)] + [big]
        for st in states:  # every kernel configuration runs once before it is captured
            st.ids.fill_(1)
            st.set_slot(llm.max_cache_len - st.m - 2)
            eng.decode_step(st, 0)
        torch.cuda.synchronize()
        cap = max(4096, n_draft)
        buf = dict(spec=torch.zeros(_lib.SB_SPEC_WORDS, dtype=torch.int32, device=dev),
                   emitted=torch.zeros(llm.max_cache_len + 2, dtype=torch.int64, device=dev),
                   draft=torch.zeros(cap, dtype=torch.int64, device=dev))
        arr = (_lib.SbState * self.MAX_CHUNK)(*[st.c for st in states])
        spec = _lib.SbSpecLoop()
        spec.verify = C.cast(arr, C.POINTER(_lib.SbState))
        spec.max_chunk = self.MAX_CHUNK
        spec.draft_capacity = cap
        spec.emit_capacity = buf["emitted"].numel()
        spec.eos_id = int(eos)
        spec.spec, spec.emitted, spec.draft = ptr(buf["spec"]), ptr(buf["emitted"]), ptr(buf["draft"])
        handle = C.c_void_p()
        check(eng.lib.sb_spec_loop_create(C.byref(eng.cmodel), C.byref(spec), C.byref(handle)), "sb_spec_loop_create")
        self._loop = dict(handle=handle, states=states, eos=eos, **buf)
        return self._loop

    def __del__(self):
        lp = getattr(self, "_loop", None)
        if lp is not None:
            try:
                self.engine.lib.sb_spec_loop_destroy(lp["handle"])
            except Exception:
                pass

    @torch.inference_mode()
    def generate(self, inputs_embeds: torch.Tensor, draft: list, max_new_tokens: int = 200,
                 eos_token_id: int = LLM_EOS_TOKEN_ID) -> SpecResult:
        if not self.device_loop:
            return self._generate_host(inputs_embeds, draft, max_new_tokens, eos_token_id)
        llm = self.llm
        P = inputs_embeds.shape[1]
        draft = [int(t) for t in draft]
        draft_count = len(draft)
        max_safe = llm.max_cache_len - P + 1
        if max_new_tokens > max_safe:
            raise ValueError(
                f"max_new_tokens={max_new_tokens} would overflow the static KV "
                f"cache (prompt T={P}, max_cache_len={llm.max_cache_len})."
            )
        if inputs_embeds.shape[0] != 1:
            raise ValueError("SpeculativeDecoder only supports batch=1.")
        if max_new_tokens <= 0:
            return self._finalize([], 0.0, draft_count, 0, 0, 0, 0)
        first = llm.prefill(inputs_embeds)
        emitted = [int(first.item())]
        if emitted[-1] == eos_token_id or len(emitted) >= max_new_tokens:
            return self._finalize(emitted, 0.0, draft_count, 0, 0, 0, 0)
        if not llm._captured:
            llm.capture(first, P)
        lp = self._device_loop(int(eos_token_id), draft_count)
        t0 = time.perf_counter()
        inputs = torch.zeros(_lib.SB_SPEC_WORDS, dtype=torch.int32)
        inputs[_lib.SB_SPEC_N_DRAFT] = draft_count
        inputs[_lib.SB_SPEC_MAX_NEW] = max_new_tokens
        inputs[_lib.SB_SPEC_PROMPT] = P
        # each round advances the draft or emits a token, except up to 8 stuck rounds in a row
        inputs[_lib.SB_SPEC_MAX_ROUNDS] = 8 * (draft_count + max_new_tokens) + 16
        lp["spec"].copy_(inputs)
        lp["emitted"][:1].copy_(first.reshape(-1)[:1])
        if draft_count:
            lp["draft"][:draft_count].copy_(torch.tensor(draft, dtype=torch.int64))
        check(self.engine.lib.sb_spec_loop_launch(lp["handle"], _lib.current_stream()), "sb_spec_loop_launch")
        out = torch.cat([lp["spec"].long(), lp["emitted"]]).tolist()  # the one device->host read
        spec, ids = out[:_lib.SB_SPEC_WORDS], out[_lib.SB_SPEC_WORDS:]
        if spec[_lib.SB_SPEC_ERR]:
            raise _lib.StarlingError(f"speculative loop stopped at its round limit or capacity (state {spec})")
        emitted = ids[:spec[_lib.SB_SPEC_N_EMIT]]
        accepted, verify_forwards = spec[_lib.SB_SPEC_ACCEPTED], spec[_lib.SB_SPEC_VERIFIES]
        cache_pos = spec[_lib.SB_SPEC_CACHE_POS]
        decode_steps = 0
        if not spec[_lib.SB_SPEC_STOPPED]:
            # single-step fallback once the draft is exhausted (speculative.py:541-560)
            while len(emitted) < max_new_tokens:
                llm._prime(torch.tensor([emitted[-1]], device=llm.state.ids.device), cache_pos)
                if llm._captured:
                    llm._graph.replay()
                else:
                    llm._decode_step_eager()
                decode_steps += 1
                tid = int(llm.state.out_ids[0].item())
                emitted.append(tid)
                cache_pos += 1
                if tid == eos_token_id:
                    break
        torch.cuda.synchronize()
        return self._finalize(emitted, (time.perf_counter() - t0) * 1000.0, draft_count, accepted,
                              verify_forwards, decode_steps, 0)

    @torch.inference_mode()
    def _generate_host(self, inputs_embeds: torch.Tensor, draft: list, max_new_tokens: int = 200,
                       eos_token_id: int = LLM_EOS_TOKEN_ID) -> SpecResult:
        llm = self.llm
        P = inputs_embeds.shape[1]
        draft = [int(t) for t in draft]
        draft_count = len(draft)
        max_safe = llm.max_cache_len - P + 1
        if max_new_tokens > max_safe:
            raise ValueError(
                f"max_new_tokens={max_new_tokens} would overflow the static KV "
                f"cache (prompt T={P}, max_cache_len={llm.max_cache_len})."
            )
        if inputs_embeds.shape[0] != 1:
            raise ValueError("SpeculativeDecoder only supports batch=1.")
        if max_new_tokens <= 0:
            return self._finalize([], 0.0, draft_count, 0, 0, 0, 0)

        first = llm.prefill(inputs_embeds)
        emitted = [int(first.item())]
        if emitted[-1] == eos_token_id or len(emitted) >= max_new_tokens:
            return self._finalize(emitted, 0.0, draft_count, 0, 0, 0, 0)
        if not llm._captured:
            llm.capture(first, P)
        self.warmup_graphs()
        t0 = time.perf_counter()
        cache_pos = P
        accepted = verify_forwards = decode_steps = 0
        draft_pos = 0
        chunk_size = self.MIN_CHUNK
        SEARCH_WIN, STUCK_LIMIT = 40, 8
        stuck = 0
        while draft_pos < draft_count and len(emitted) < max_new_tokens:
            before = draft_pos
            k = min(chunk_size, draft_count - draft_pos, max_new_tokens - len(emitted),
                    llm.max_cache_len - cache_pos - 1)
            if k <= 0:
                break
            chunk = draft[draft_pos:draft_pos + k]
            preds_all, _ = self.verify([emitted[-1]] + chunk, cache_pos)
            verify_forwards += 1
            preds, bonus = preds_all[:k], preds_all[k]
            j = 0
            mismatch = full = stopped = False
            while j < k and preds[j] == chunk[j]:
                emitted.append(chunk[j])
                accepted += 1
                if chunk[j] == eos_token_id:
                    j += 1
                    stopped = True
                    break
                j += 1
            if not stopped:
                if j < k:
                    emitted.append(preds[j])
                    mismatch = True
                    stopped = preds[j] == eos_token_id
                else:
                    full = True
                    emitted.append(bonus)
                    stopped = bonus == eos_token_id
            if full:
                cache_pos += k + 1
                draft_pos += k
            elif mismatch:
                cache_pos += j + 1
                draft_pos += j
            else:
                cache_pos += j
                draft_pos += j
            last_val = emitted[-1]
            realigned = False
            if not stopped and draft_pos < draft_count:
                for dd in range(draft_pos, min(draft_pos + SEARCH_WIN, draft_count)):
                    if draft[dd] == last_val:
                        draft_pos = dd + 1
                        accepted += 1
                        realigned = True
                        break
            stuck = 0 if draft_pos > before else stuck + 1
            if stuck >= STUCK_LIMIT and not stopped and draft_pos < draft_count:
                draft_pos = before + 1
                stuck = 0
            if not stopped:
                if full:
                    chunk_size = min(chunk_size + 4, self.MAX_CHUNK)
                elif mismatch and j == 0 and not realigned:
                    chunk_size = self.BOUNDARY_CHUNK
                else:
                    chunk_size = self.MIN_CHUNK
            if stopped or len(emitted) >= max_new_tokens:
                torch.cuda.synchronize()
                return self._finalize(emitted, (time.perf_counter() - t0) * 1000.0, draft_count, accepted,
                                      verify_forwards, decode_steps, 0)
        # single-step fallback once the draft is exhausted (speculative.py:541-560)
        while len(emitted) < max_new_tokens:
            llm._prime(torch.tensor([emitted[-1]], device=llm.state.ids.device), cache_pos)
            if llm._captured:
                llm._graph.replay()
            else:
                llm._decode_step_eager()
            decode_steps += 1
            tid = int(llm.state.out_ids[0].item())
            emitted.append(tid)
            cache_pos += 1
            if tid == eos_token_id:
                break
        torch.cuda.synchronize()
        return self._finalize(emitted, (time.perf_counter() - t0) * 1000.0, draft_count, accepted,
                              verify_forwards, decode_steps, 0)

    def _finalize(self, emitted, wall_ms, draft_count, accepted, verify_forwards, decode_steps=0, decode_probes=0):
        ids = torch.tensor(emitted, dtype=torch.int64).unsqueeze(0)
        n = len(emitted)
        return SpecResult(ids=ids, text="", n_tokens=n, total_ms=wall_ms, tok_per_s=n / max(wall_ms / 1000.0, 1e-9),
                          draft_count=draft_count, accepted=accepted, verify_forwards=verify_forwards,
                          acceptance_rate=accepted / draft_count if draft_count > 0 else 0.0,
                          decode_steps=decode_steps, decode_probes=decode_probes)
