"""Stream sharding across the GPUs of one box (batched long-audio decode).

The reference decodes on one GPU (batched.py:20-33) and has no distributed
code.  Here independent streams are dealt to ranks (one process per GPU):
every rank holds a full weight replica, its own KV cache and graph, and
decodes its own streams with no collective on the data path; the token ids
are gathered on the host at the end.

* :func:`shard_streams` sorts streams by prompt length and deals them
  round-robin, so each rank's longest prompt (its padded prefill length and
  cache footprint) is as balanced as possible.
* :func:`gather_ids` brings every rank's per-stream id lists back to rank 0
  (or all ranks) in the original stream order.
* :class:`ShardedBatchedDecoder` wraps :class:`BatchedLLMMega` with both.
"""

from __future__ import annotations

from typing import Optional, Sequence

import torch


def shard_streams(prompt_lengths: Sequence[int], world: int) -> list:
    """Return ``world`` lists of stream indices.  Streams are sorted by prompt
    length (longest first, stable) and dealt round-robin."""
    if world < 1:
        raise ValueError("world must be >= 1")
    order = sorted(range(len(prompt_lengths)), key=lambda i: (-int(prompt_lengths[i]), i))
    shards = [[] for _ in range(world)]
    for j, i in enumerate(order):
        shards[j % world].append(i)
    return [sorted(s) for s in shards]


def gather_ids(local: dict, n_streams: int, group=None, dst: Optional[int] = 0) -> Optional[list]:
    """Gather ``{stream index: list of ids}`` from every rank.

    With ``dst`` an int only that rank receives the merged list (others get
    None); with ``dst=None`` every rank does.  Host objects only: works on
    gloo (CPU) and nccl process groups alike.
    """
    import torch.distributed as dist

    world = dist.get_world_size(group)
    rank = dist.get_rank(group)
    if dst is None:
        parts = [None] * world
        dist.all_gather_object(parts, local, group=group)
    else:
        parts = [None] * world if rank == dst else None
        dist.gather_object(local, parts, dst=dst, group=group)
        if rank != dst:
            return None
    out = [None] * n_streams
    for p in parts:
        for i, ids in p.items():
            if out[i] is not None:
                raise RuntimeError(f"stream {i} decoded by two ranks")
            out[i] = ids
    missing = [i for i, v in enumerate(out) if v is None]
    if missing:
        raise RuntimeError(f"streams {missing[:8]} were decoded by no rank")
    return out


class ShardedBatchedDecoder:
    """Decode a batch of streams split across the ranks of a process group.

    Every rank passes the SAME full batch; rank r decodes
    ``shard_streams(...)[r]`` with its local :class:`BatchedLLMMega`
    (constructed with ``max_batch_size`` = its shard size) and the ids are
    gathered to ``dst``.
    """

    def __init__(self, make_decoder, group=None):
        self.make_decoder = make_decoder  # callable(batch_size) -> BatchedLLMMega-like
        self.group = group
        self._decoders = {}

    def generate(self, inputs_embeds: torch.Tensor, prompt_lengths: torch.Tensor, max_new_tokens: int,
                 eos_token_id: int, dst: Optional[int] = 0):
        import torch.distributed as dist

        world = dist.get_world_size(self.group)
        rank = dist.get_rank(self.group)
        B = inputs_embeds.shape[0]
        mine = shard_streams(prompt_lengths.tolist(), world)[rank]
        local = {}
        if mine:
            pl = prompt_lengths[mine]
            T = int(pl.max())
            emb = inputs_embeds[mine, :T]
            dec = self._decoders.get(len(mine))
            if dec is None:
                dec = self._decoders[len(mine)] = self.make_decoder(len(mine))
            res = dec.generate(emb, prompt_lengths=pl, max_new_tokens=max_new_tokens, eos_token_id=eos_token_id)
            local = {i: res.ids_list[j].tolist() for j, i in enumerate(mine)}
        return gather_ids(local, B, group=self.group, dst=dst)
