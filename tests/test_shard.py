"""Multi-rank host logic on CPU with gloo (world_size 2): stream sharding,
the host gather of ids, a sharded decode with a fake decoder, and a rank that
fails before the gather (the other rank must get an error, not hang)."""

import datetime
import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from starling_b200.shard import ShardedBatchedDecoder, gather_ids, shard_streams


def test_shard_streams_balanced_and_complete():
    pl = [300, 900, 450, 880, 310, 700, 650, 420]
    shards = shard_streams(pl, 2)
    assert sorted(sum(shards, [])) == list(range(8))
    assert max(pl[i] for i in shards[0]) == 900 and max(pl[i] for i in shards[1]) == 880
    assert abs(len(shards[0]) - len(shards[1])) <= 1
    assert shard_streams([5, 5, 5], 4)[3] == []
    with pytest.raises(ValueError):
        shard_streams(pl, 0)


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


class _FakeResult:
    def __init__(self, ids_list):
        self.ids_list = ids_list


class _FakeDecoder:
    """Stands in for BatchedLLMMega on CPU: stream ids = [T_b, T_b + 1, ...]."""

    def __init__(self, b):
        self.b = b

    def generate(self, emb, prompt_lengths, max_new_tokens, eos_token_id):
        assert emb.shape[0] == self.b
        return _FakeResult([torch.arange(int(t), int(t) + max_new_tokens) for t in prompt_lengths])


def _worker(rank, world, port, mode, q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    try:
        dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=5))
        if mode == "gather":
            local = {i: [i, rank] for i in range(rank, 6, world)}
            out = gather_ids(local, 6, dst=None)
            q.put((rank, out))
        elif mode == "sharded":
            pl = torch.tensor([300, 900, 450, 880, 310])
            emb = torch.zeros(5, 900, 4)
            dec = ShardedBatchedDecoder(lambda b: _FakeDecoder(b))
            out = dec.generate(emb, pl, 3, -1, dst=0)
            q.put((rank, out))
        elif mode == "fail":
            if rank == 1:
                raise RuntimeError("rank 1: decoder failed")
            try:
                gather_ids({0: [1]}, 2, dst=0)
                q.put((rank, "no error"))
            except Exception as e:  # the gather must end with an error, not hang
                q.put((rank, f"error: {type(e).__name__}"))
    except RuntimeError as e:
        q.put((rank, f"raised: {e}"))
    finally:
        if dist.is_initialized():
            try:
                dist.destroy_process_group()
            except Exception:
                pass


def _run(mode, world=2):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    ps = [ctx.Process(target=_worker, args=(r, world, port, mode, q)) for r in range(world)]
    for p in ps:
        p.start()
    res = dict(q.get(timeout=120) for _ in range(world))
    for p in ps:
        p.join(timeout=60)
        if p.is_alive():
            p.kill()
    return res


def test_gather_ids_all_ranks():
    res = _run("gather")
    want = [[i, i % 2] for i in range(6)]
    assert res[0] == want and res[1] == want


def test_sharded_decode_gathers_in_stream_order():
    res = _run("sharded")
    assert res[1] is None
    assert res[0] == [[300, 301, 302], [900, 901, 902], [450, 451, 452], [880, 881, 882], [310, 311, 312]]


def test_failed_rank_does_not_hang_the_others():
    res = _run("fail")
    assert res[1].startswith("raised: rank 1")
    assert res[0].startswith("error")
