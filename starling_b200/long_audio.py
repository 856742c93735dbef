"""Batched long-audio decode feeder, on one GPU or across the GPUs of a box.

The LLM half of the reference's ``transcribe_long_batched``
(src/starling/granite/long_audio.py:310-397) and of
``BatchedPipeline.run_batch`` (src/starling/granite/batched.py:780-858): the
chunks of a long recording, each already turned into its prompt embeddings
(audio projector output + prompt tokens, before the x12 multiplier), are
decoded ``B = decoder.max_batch_size`` at a time in lock-step.  As in the
reference, a short last mini-batch is filled up to B with copies of its
first chunk (the decoder's buffers, cache and graph are sized for B) whose
outputs are dropped; prompts of different lengths are right-padded with
zeros and masked through ``prompt_lengths``; each mini-batch's token budget
is ``max(1, min(max_new_tokens, max_cache_len - T_max - 1))``.

Across GPUs (one process per GPU, a ``torch.distributed`` process group for
the host-side gather only) the chunks are dealt round-robin to the ranks;
every rank decodes its own chunks with its own decoder and no collective on
the data path, and the token ids come back to one rank in chunk order at the
end (``shard.gather_ids``).  The audio chunking, the encoder and the text
joining belong to the encoder side and are not part of this package.
"""

from __future__ import annotations

import time
from dataclasses import dataclass, field
from typing import Any, Optional, Sequence

import torch

from .config import LLM_EOS_TOKEN_ID


@dataclass
class ChunkDecode:
    """One chunk's greedy output (the id half of the reference's ChunkResult,
    long_audio.py:61-69)."""

    index: int
    ids: list
    n_tokens: int
    ms: float  # the chunk's share of its mini-batch's wall time, as the reference reports it


@dataclass
class LongDecodeResult:
    """All chunks in chunk order (long_audio.py:72-85, without the text)."""

    chunks: list = field(default_factory=list)
    total_ms: float = 0.0
    n_chunks: int = 0
    total_tokens: int = 0
    n_ranks: int = 1


def _as_rows(e: torch.Tensor) -> torch.Tensor:
    if e.dim() == 3:
        if e.shape[0] != 1:
            raise ValueError(f"a chunk's embeddings must be (T, H) or (1, T, H), got {tuple(e.shape)}")
        e = e[0]
    if e.dim() != 2:
        raise ValueError(f"a chunk's embeddings must be (T, H) or (1, T, H), got {tuple(e.shape)}")
    return e


def run_batch(decoder: Any, chunk_embeds: Sequence[torch.Tensor], max_new_tokens: int = 200,
              eos_token_id: int = LLM_EOS_TOKEN_ID):
    """Decode up to ``decoder.max_batch_size`` chunks in lock-step
    (batched.py:780-858 after the encoder): fill the batch to B with copies of
    the first chunk, right-pad to the longest prompt, generate, and return
    the results of the real chunks only (``BatchedGenerateResult``)."""
    n = len(chunk_embeds)
    B = int(decoder.max_batch_size)
    if n < 1 or n > B:
        raise ValueError(f"got {n} streams but the decoder is sized for max_batch_size={B}")
    rows = [_as_rows(e) for e in chunk_embeds]
    rows += [rows[0]] * (B - n)
    Ts = [int(r.shape[0]) for r in rows]
    T_max = max(Ts)
    H = int(rows[0].shape[1])
    emb = torch.zeros(B, T_max, H, dtype=rows[0].dtype, device=rows[0].device)
    for b, r in enumerate(rows):
        emb[b, : Ts[b]] = r
    prompt_lengths = None if all(T == T_max for T in Ts) else torch.tensor(Ts, dtype=torch.long)
    budget = max(1, min(int(max_new_tokens), int(decoder.max_cache_len) - T_max - 1))
    res = decoder.generate(emb, prompt_lengths=prompt_lengths, max_new_tokens=budget, eos_token_id=eos_token_id)
    if n < B:
        res.ids_list = res.ids_list[:n]
        res.n_tokens_per_stream = res.n_tokens_per_stream[:n]
        res.total_tokens = sum(res.n_tokens_per_stream)
        res.n_streams = n
    return res


def deal_chunks(n_chunks: int, world: int) -> list:
    """Chunk indices of each rank: round-robin, so every rank's mini-batches
    are consecutive stretches of the recording and the ranks' loads differ
    by at most one chunk."""
    if world < 1:
        raise ValueError("world must be >= 1")
    return [list(range(r, n_chunks, world)) for r in range(world)]


def decode_chunks(decoder: Any, chunk_embeds: Sequence[torch.Tensor], max_new_tokens: int = 200,
                  eos_token_id: int = LLM_EOS_TOKEN_ID, group=None, dst: Optional[int] = 0,
                  distributed: Optional[bool] = None) -> Optional[LongDecodeResult]:
    """Decode every chunk: ``decoder`` is this process's batched decoder
    (``BatchedLLMMega`` or anything with its ``max_batch_size``,
    ``max_cache_len`` and ``generate``).  With a process group (``group``,
    or the default one when ``torch.distributed`` is initialised and
    ``distributed`` is not False) every rank passes the SAME chunk list and
    decodes its share; rank ``dst`` receives the merged result (``dst=None``:
    every rank), the other ranks get None."""
    import torch.distributed as dist

    use_pg = (dist.is_available() and dist.is_initialized()) if distributed is None else bool(distributed)
    world = dist.get_world_size(group) if use_pg else 1
    rank = dist.get_rank(group) if use_pg else 0
    n = len(chunk_embeds)
    mine = deal_chunks(n, world)[rank]
    B = int(decoder.max_batch_size)
    t0 = time.perf_counter()
    local = {}
    for s in range(0, len(mine), B):
        idx = mine[s: s + B]
        c0 = time.perf_counter()
        res = run_batch(decoder, [chunk_embeds[i] for i in idx], max_new_tokens, eos_token_id)
        if torch.cuda.is_available():
            torch.cuda.synchronize()
        per_ms = (time.perf_counter() - c0) * 1000.0 / len(idx)
        for j, i in enumerate(idx):
            ids = res.ids_list[j]
            ids = ids.tolist() if hasattr(ids, "tolist") else list(ids)
            local[i] = (ids, per_ms)
    my_ms = (time.perf_counter() - t0) * 1000.0
    if use_pg:
        from .shard import gather_ids

        merged = gather_ids(local, n, group=group, dst=dst)
        t = torch.tensor([my_ms], dtype=torch.float64)
        if dist.get_backend(group) == "nccl":
            t = t.cuda()
        dist.all_reduce(t, op=dist.ReduceOp.MAX, group=group)
        total_ms = float(t.item())
        if merged is None:
            return None
    else:
        merged = [local[i] for i in range(n)]
        total_ms = my_ms
    chunks = [ChunkDecode(i, ids, len(ids), ms) for i, (ids, ms) in enumerate(merged)]
    return LongDecodeResult(chunks=chunks, total_ms=total_ms, n_chunks=n,
                            total_tokens=sum(c.n_tokens for c in chunks), n_ranks=world)
