"""The long-audio chunk feeder's host logic on CPU: mini-batching with the
reference's padding rule and token budget (long_audio.py:310-397,
batched.py:780-858), the round-robin dealing of chunks to ranks, and the
same chunks decoded on two gloo ranks giving the single-process result."""

import datetime
import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from starling_b200.long_audio import deal_chunks, decode_chunks, run_batch


class _Res:
    def __init__(self, ids_list):
        self.ids_list = ids_list
        self.n_tokens_per_stream = [len(x) for x in ids_list]
        self.total_tokens = sum(self.n_tokens_per_stream)
        self.n_streams = len(ids_list)


class _FakeDecoder:
    """BatchedLLMMega's interface on CPU.  A stream's ids (``budget`` of
    them, budget >= 3) encode what the decoder saw: [sum of its real prompt
    rows' first feature (rounded), prompt length, budget, 7, ...] -- so the
    tests can check padding, lengths and the budget."""

    def __init__(self, B, max_cache_len=64):
        self.max_batch_size = B
        self.max_cache_len = max_cache_len
        self.calls = []

    def generate(self, emb, prompt_lengths=None, max_new_tokens=200, eos_token_id=0):
        B, T, _ = emb.shape
        assert B == self.max_batch_size
        pl = [T] * B if prompt_lengths is None else [int(x) for x in prompt_lengths]
        self.calls.append((T, pl, max_new_tokens))
        out = []
        for b in range(B):
            assert torch.all(emb[b, pl[b]:] == 0), "right padding must be zeros"
            tag = int(round(float(emb[b, : pl[b], 0].sum())))
            out.append(torch.tensor([tag, pl[b], max_new_tokens] + [7] * (max_new_tokens - 3)))
        return _Res(out)


def _chunks(n, H=4, T0=10):
    g = torch.Generator().manual_seed(0)
    out = []
    for i in range(n):
        T = T0 + (i % 3)  # prompts of different lengths
        e = torch.zeros(T, H)
        e[:, 0] = float(i + 1) / T  # sums to i + 1
        e[:, 1:] = torch.randn(T, H - 1, generator=g)
        out.append(e)
    return out


def test_run_batch_pads_with_first_chunk_and_drops_it():
    dec = _FakeDecoder(4, max_cache_len=64)
    ch = _chunks(3)
    res = run_batch(dec, ch, max_new_tokens=100, eos_token_id=0)
    T, pl, budget = dec.calls[0]
    assert T == 12 and pl == [10, 11, 12, 10]  # the fourth stream is a copy of the first
    assert budget == 64 - 12 - 1  # max(1, min(max_new_tokens, max_cache_len - T_max - 1))
    assert len(res.ids_list) == 3 and res.n_streams == 3
    assert [int(x[0]) for x in res.ids_list] == [1, 2, 3]
    assert res.total_tokens == 3 * budget
    with pytest.raises(ValueError):
        run_batch(dec, _chunks(5))


def test_run_batch_equal_lengths_pass_no_prompt_lengths():
    dec = _FakeDecoder(2)
    run_batch(dec, [torch.ones(8, 4), torch.ones(1, 8, 4)], max_new_tokens=5)
    assert dec.calls[0] == (8, [8, 8], 5)


def test_deal_chunks_round_robin():
    assert deal_chunks(7, 3) == [[0, 3, 6], [1, 4], [2, 5]]
    assert sorted(sum(deal_chunks(11, 4), [])) == list(range(11))
    assert deal_chunks(2, 4)[3] == []
    with pytest.raises(ValueError):
        deal_chunks(3, 0)


def test_decode_chunks_single_process_order():
    dec = _FakeDecoder(2)
    res = decode_chunks(dec, _chunks(5), max_new_tokens=4, distributed=False)
    assert res.n_chunks == 5 and res.n_ranks == 1
    assert [c.ids[0] for c in res.chunks] == [1, 2, 3, 4, 5]
    assert [c.index for c in res.chunks] == list(range(5))
    assert res.total_tokens == 5 * 4
    assert len(dec.calls) == 3  # mini-batches of 2, 2 and 1 (padded to 2)


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _worker(rank, world, port, q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    try:
        dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=10))
        dec = _FakeDecoder(2)
        res = decode_chunks(dec, _chunks(7), max_new_tokens=4, dst=0)
        q.put((rank, None if res is None else [c.ids for c in res.chunks], len(dec.calls)))
        dist.destroy_process_group()
    except Exception as e:  # reported to the parent
        q.put((rank, repr(e), -1))


def test_decode_chunks_two_ranks_matches_one():
    ref = decode_chunks(_FakeDecoder(2), _chunks(7), max_new_tokens=4, distributed=False)
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    out = {}
    for _ in range(2):
        r, ids, calls = q.get(timeout=120)
        out[r] = (ids, calls)
    for p in procs:
        p.join(timeout=60)
    assert out[1][0] is None  # only dst gets the merged result
    assert out[0][0] == [c.ids for c in ref.chunks]
    assert out[0][1] == 2 and out[1][1] == 2  # 4 and 3 chunks, in mini-batches of 2
