"""Decode throughput benchmark for the native B200 Granite decode path.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--workload b48|b1] [--fmt F]
    python bench.py --impl reference ...          # the reference's eager CPU path

One timed "step" is one greedy decode step of every stream (B tokens per
GPU).  Workloads (synthetic, seeded; see starling_b200/synthetic.py):

* ``b48`` (default, the headline): 48 streams per GPU (weak scaling), FP8
  e4m3 per-channel weights, prompt lengths U[300, 900], 128 greedy steps,
  40-layer decoder;
* ``b1``: one stream, NVFP4 weights, 300 audio embeddings + 20 prompt ids,
  128 greedy steps as K=8-step graph replays;
* ``verify``: one stream, NVFP4 weights, verify forwards of 8 tokens over a
  600-position cache, 64 rounds, the cache rewound to 600 after each.

On one GPU the headline line also carries a ``b1`` and a ``verify`` object
(each with its own value, roofline, e2e and CPU baseline).  Under torchrun
each rank decodes its own 48 streams with no collective on the data path
(streams are independent); only the timing barrier and the max-over-ranks
reduction use the process group.  With N > 1 the line adds
``strong_scaling``: a fixed batch of 48 streams dealt over the N ranks
(``shard.shard_streams``), 48 x K tokens over the max-over-ranks time.
"""

from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import threading
import time
from pathlib import Path

import torch

REPO = Path(__file__).resolve().parent
sys.path.insert(0, str(REPO))

GEN_STEPS = 128  # greedy steps of one workload instance (e2e: prefill + these)
WORKLOADS = {
    "b48": dict(batch=48, fmt="fp8", max_len=1040, k_replay=8, desc="batched long-audio decode, B=48/GPU, FP8 e4m3 per-channel, prompts U[300,900], 128 greedy steps"),
    "b1": dict(batch=1, fmt="nvfp4", max_len=640, k_replay=8, desc="B=1 greedy decode, NVFP4, 300 audio embeds + 20 prompt ids, 128 steps as K=8 graph replays"),
}
VERIFY = dict(fmt="nvfp4", max_len=640, ctx=600, m=8, rounds=64,
              desc="self-speculative verify, B=1, NVFP4, 8 tokens per verify over a 600-position cache, 64 rounds "
                   "with the cache rewound after each")


def _env_int(name, default):
    try:
        return int(os.environ.get(name, default))
    except ValueError:
        return default


def _peaks():
    p = REPO / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        return float(d["hbm_gbs"]), "measured"
    return 6650.0, "fallback"


# --------------------------------------------------------------------------- #
class ClockSampler:
    """SM clocks and clock-event reasons sampled during the timed region.

    NVML is queried (read-only) every 5 ms from a thread, so that a timed
    region of tens of milliseconds still holds samples; without NVML,
    nvidia-smi's 200 ms loop.  Only samples taken between mark_start() and
    mark_end() are summarised."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")
    NAMES = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
    # NVML clock-event reason bits of the names above, and of the power brake
    BITS = {"sw_power_cap": 0x4, "hw_slowdown": 0x8, "sw_thermal_slowdown": 0x20, "hw_thermal_slowdown": 0x40,
            "hw_power_brake_slowdown": 0x80}

    def __init__(self, device_index: int):
        try:  # address the GPU by UUID: robust to CUDA_VISIBLE_DEVICES remapping
            self.idx = "GPU-" + str(torch.cuda.get_device_properties(device_index).uuid)
        except Exception:
            self.idx = str(device_index)
        self.proc = None
        self.stop = None
        self.samples = []  # (time, sm MHz, max sm MHz, set of active reasons)
        self.t0 = self.t1 = None

    def mark_start(self):
        self.t0 = time.perf_counter()

    def mark_end(self):
        self.t1 = time.perf_counter()

    def __enter__(self):
        if self._start_nvml():
            return self
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits", "-lms", "200",
                 "-i", self.idx], stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self._t = threading.Thread(target=self._read, daemon=True)
            self._t.start()
        except (FileNotFoundError, OSError):
            self.proc = None
        return self

    def _start_nvml(self) -> bool:
        try:
            import pynvml

            pynvml.nvmlInit()
            h = pynvml.nvmlDeviceGetHandleByUUID(self.idx) if self.idx.startswith("GPU-") else \
                pynvml.nvmlDeviceGetHandleByIndex(int(self.idx))
            mx = float(pynvml.nvmlDeviceGetMaxClockInfo(h, pynvml.NVML_CLOCK_SM))
        except Exception:
            return False
        self.stop = threading.Event()

        def loop():
            while not self.stop.is_set():
                try:
                    t = time.perf_counter()
                    sm = float(pynvml.nvmlDeviceGetClockInfo(h, pynvml.NVML_CLOCK_SM))
                    r = int(pynvml.nvmlDeviceGetCurrentClocksEventReasons(h))
                    self.samples.append((t, sm, mx, {n for n, b in self.BITS.items() if r & b}))
                except Exception:
                    return
                self.stop.wait(0.005)

        self._t = threading.Thread(target=loop, daemon=True)
        self._t.start()
        return True

    def _read(self):
        for line in self.proc.stdout:
            parts = [x.strip() for x in line.strip().split(",")]
            if len(parts) < 9:
                continue
            try:
                sm, mx = float(parts[1]), float(parts[2])
            except ValueError:
                continue
            self.samples.append((time.perf_counter(), sm, mx,
                                 {n for n, v in zip(self.NAMES, parts[5:9]) if v.lower() == "active"}))

    def __exit__(self, *a):
        if self.stop is not None:
            self.stop.set()
            self._t.join(timeout=5)
        if self.proc is not None:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()

    def summary(self):
        t0 = self.t0 if self.t0 is not None else float("-inf")
        t1 = self.t1 if self.t1 is not None else float("inf")
        inside = [x for x in list(self.samples) if t0 <= x[0] <= t1]
        sm = [x[1] for x in inside]
        reasons = set().union(*[x[3] for x in inside]) if inside else set()
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": inside[-1][2] if inside else None,
                "reasons": sorted(reasons), "samples": len(sm),
                "source": "nvml" if self.stop is not None else "nvidia-smi"}


# --------------------------------------------------------------------------- #
def _barrier(world):
    if world > 1:
        import torch.distributed as dist

        dist.barrier()


def _max_over_ranks(x: float, world: int, dev) -> float:
    t = torch.tensor([x], device=dev, dtype=torch.float64)
    if world > 1:
        import torch.distributed as dist

        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def decode_timing(eng, B, emb, prompt_lengths, T, K, W, kr, world, dev, local_rank):
    """Prefill ``B`` streams, capture the K-step decode graph, run W warm-up
    steps, then time exactly K steps (barrier + synchronize on both sides,
    CUDA events on the launching stream, max over ranks).  Returns the
    timing, the launch count per step and a ``reset`` that puts the state
    back at the first decode position."""
    from starling_b200.batched import BatchedLLMMega
    from starling_b200.multistep import MultiStepLLMMega

    if B == 1:
        dec = MultiStepLLMMega(engine=eng, steps_per_replay=kr)
        first = dec.prefill(emb.to(dev))
        st = dec.state
        snap_ids = first.view(-1).clone()
        fin0 = None
    else:
        dec = BatchedLLMMega(engine=eng, max_batch_size=B, steps_per_replay=kr)
        dec.prefill(emb.to(dev), prompt_lengths)
        st = dec.state
        snap_ids = st.ids.clone()
        fin0 = st.finished.clone()
    if T + K + W > eng.max_cache_len:
        raise SystemExit(f"steps+warmup exceed the cache ({T}+{K}+{W} > {eng.max_cache_len})")

    def reset():
        st.ids.copy_(snap_ids)
        if fin0 is not None:
            st.finished.copy_(fin0)
        st.set_slot(T, pad_len=T)

    def capture(n):
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g):
            for j in range(n):
                eng.decode_step(st, j)
        return g

    reset()
    for _ in range(2):  # eager warm-up of every kernel configuration before capture
        n0 = int(eng.lib.sb_launch_count())
        eng.decode_step(st, 0)
        launches_per_step = int(eng.lib.sb_launch_count()) - n0
    torch.cuda.synchronize()
    graphs = {kr: capture(kr)}
    if K % kr or W % kr:
        graphs[1] = capture(1)
    reset()

    def run_steps(n):
        for _ in range(n // kr):
            graphs[kr].replay()
        for _ in range(n % kr):
            graphs[1].replay()

    with ClockSampler(local_rank) as clk:
        run_steps(W)  # warm-up (untimed), then back to the first decode position
        torch.cuda.synchronize()
        reset()
        stream = torch.cuda.current_stream()
        ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        _barrier(world)
        torch.cuda.synchronize()
        torch.cuda.nvtx.range_push("timed_steps")  # ncu --nvtx-include "timed_steps/" selects these launches
        clk.mark_start()
        ev0.record(stream)
        run_steps(K)
        ev1.record(stream)
        torch.cuda.nvtx.range_pop()
        torch.cuda.synchronize()
        clk.mark_end()
        _barrier(world)
    ms = _max_over_ranks(ev0.elapsed_time(ev1), world, dev)
    reset()
    graphs.clear()
    return dict(ms=ms, launches_per_step=launches_per_step, state=st, reset=reset, clocks=clk.summary())


# DRAM traffic per launch (dram__bytes_read.sum + dram__bytes_write.sum) from
# one ncu capture of the same kernel and shape (profiles/), with the
# algorithmic bytes of the captured case: the bench scales the traffic to its
# own launch by the ratio of algorithmic bytes (same kernel, same tiling).
PROFILED_TRAFFIC = {
    ("b48", "attention"): (66.056448e6 + 0.626432e6, 61.5e6, "profiles/attention_b48_decode.md"),
    ("b48", "gate_up"): (33.9008e6, 33.62e6, "profiles/tcgen05_gemm_gate_up_fp8_b48.md"),
    ("b1", "gate_up"): (18.93376e6, 18.87e6, "profiles/gemv_gate_up_nvfp4_b1.md"),
    # 4 layers + lm_head: 4 x 34.21 MB + 115.61 MB of NVFP4 weights + K/V rows
    ("b1", "step"): (255.986688e6 + 4.75648e6, 4 * 34.21e6 + 115.61e6 + 2.6e6, "profiles/fused_step_b1_nvfp4.md"),
}


def dominant_kernel(eng, st, d, B, T, fmt, reset, workload=None):
    """Time the step's largest kernel alone (same configuration), rotating over
    the 40 layers so its operands come from HBM.  Returns the roofline entry."""
    from starling_b200 import _lib
    import ctypes as C

    peak, _ = _peaks()
    lib = eng.lib
    stream = torch.cuda.current_stream()
    L = d.layers
    ctx = T  # decode position at the first timed step
    # K and V rows of the valid keys only: each stream's prompt part plus the new slot
    plens = getattr(st, "prompt_len", None)
    valid = int(plens[:B].sum().item()) + B if plens is not None else B * (ctx + 1)
    kv_bytes = 2 * d.n_kv * 128 * 2 * valid
    cands = {}
    for name, op in (("gate_up", _lib.SB_OP_GATE_UP), ("attention", _lib.SB_OP_ATTN), ("down", _lib.SB_OP_DOWN)):
        if name == "attention":
            nbytes = kv_bytes
        else:
            p = eng.layers[0][name]
            nbytes = p.nbytes + B * p.k * 2 + B * (p.n // (2 if name == "gate_up" else 1)) * 2
        reset()

        def launch_all():
            for l in range(L):
                _lib.check(lib.sb_decode_op(C.byref(eng.cmodel), C.byref(st.c), l, op, 0, _lib.current_stream()))

        launch_all()  # eager once (kernel attributes), then one graph of the 40 launches
        torch.cuda.synchronize()
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g):
            launch_all()
        for _ in range(2):
            g.replay()
        torch.cuda.synchronize()
        reps = 5
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        for _ in range(reps):
            g.replay()
        e1.record(stream)
        torch.cuda.synchronize()
        del g
        us = e0.elapsed_time(e1) * 1000.0 / (reps * L)
        cands[name] = dict(us=us, bytes=nbytes, gbs=nbytes / (us * 1e-6) / 1e9)
    reset()
    # dominant = largest total time per step
    name = max(cands, key=lambda n: cands[n]["us"])
    c = cands[name]
    traffic, tsrc = None, None
    prof = PROFILED_TRAFFIC.get((workload, name))
    if prof is not None:
        traffic = round(prof[0] * c["bytes"] / prof[1])
        tsrc = f"ncu capture in {prof[2]}, scaled by algorithmic bytes"
    return {
        "roofline": {"bound": "hbm", "achieved": round(c["gbs"], 1), "peak": peak, "unit": "GB/s",
                     "frac": round(c["gbs"] / peak, 4), "traffic": traffic, "traffic_source": tsrc, "kernel": name,
                     "algorithmic_bytes_per_launch": c["bytes"], "avg_launch_us": round(c["us"], 3)},
        "info": {k: {kk: round(vv, 3) for kk, vv in v.items()} for k, v in cands.items()},
    }


def run_e2e(eng, wl, inp, B, dev, world):
    """One workload instance through the public generate() call with inputs in
    pinned host memory: H2D of the prompt embeddings, prefill, GEN_STEPS greedy
    steps, D2H of the token ids (one read per K-step replay)."""
    from starling_b200.batched import BatchedLLMMega
    from starling_b200.multistep import MultiStepLLMMega

    emb = inp.inputs_embeds.pin_memory()
    n_new = GEN_STEPS + 1  # the prefill's first token + GEN_STEPS decode steps
    if B == 1:
        dec = MultiStepLLMMega(engine=eng, steps_per_replay=wl["k_replay"])
        call = lambda: dec.generate(emb, max_new_tokens=n_new, eos_token_id=-1)  # noqa: E731
    else:
        dec = BatchedLLMMega(engine=eng, max_batch_size=B, steps_per_replay=wl["k_replay"])
        call = lambda: dec.generate(emb, prompt_lengths=inp.prompt_lengths, max_new_tokens=n_new,  # noqa: E731
                                    eos_token_id=-1)
    call()  # warm-up: the decoder captures its K-step graph once and keeps it
    torch.cuda.synchronize()
    secs = []
    for _ in range(3):  # median of three calls: one call's host-clock time swings with host load
        t0 = time.perf_counter()
        res = call()
        ntok = res.n_tokens if B == 1 else res.total_tokens
        torch.cuda.synchronize()
        secs.append(time.perf_counter() - t0)
    sec = _max_over_ranks(sorted(secs)[1], world, dev)
    n = torch.tensor([float(ntok)], device=dev)
    if world > 1:
        import torch.distributed as dist

        dist.all_reduce(n, op=dist.ReduceOp.SUM)
    h2d = emb.numel() * emb.element_size()
    d2h = ntok * 8
    return {"value": round(float(n.item()) / sec, 2), "unit": "tok/s",
            "h2d_bytes_per_step": int(h2d // GEN_STEPS), "d2h_bytes_per_step": int(d2h // GEN_STEPS),
            "note": f"one workload instance per GPU through the public generate(): prefill + {GEN_STEPS} greedy "
                    f"steps ({B * n_new} tokens per GPU), median of 3 calls after one warm-up call, host clock, "
                    f"max over ranks; the prefill is inside the timed region, so e2e grows with the step count"}

# --------------------------------------------------------------------------- #
_ORACLE = {}


def _oracle_model():
    """The reference's eager decode path restated on the CPU (bf16 weights:
    the reference has no quantised path), built once per process."""
    from oracle import granite_ref as gr

    if "m" not in _ORACLE:
        torch.set_grad_enabled(False)
        d = gr.GRANITE_1B_DIMS
        _ORACLE["m"] = gr.OracleModel(d, gr.make_weights(d, seed=0, std=0.02))
    return _ORACLE["m"]


def _timed_loop(fn, seconds: float, max_iters: int = 64):
    times = []
    t_end = time.perf_counter() + seconds
    while True:
        t0 = time.perf_counter()
        fn()
        times.append(time.perf_counter() - t0)
        if time.perf_counter() > t_end or len(times) >= max_iters:
            return times


def cpu_baseline(B: int, seconds: float, prompt_lengths=None, T: int = None, max_len: int = None):
    """The reference's eager decode step (oracle restatement of
    FusedLLMMega._decode_step_eager, bf16, torch CPU) on a bounded sample: as
    many full 40-layer decode steps of the GPU arm's B streams as fit in
    ``seconds``.  Each stream has the GPU arm's prompt length (random cache
    contents in its prompt slots, right-padded to T) and attends, as the
    reference does, over the whole static cache through its mask."""
    from oracle import granite_ref as gr

    m = _oracle_model()
    d = m.d
    pl = torch.full((B,), T) if prompt_lengths is None else prompt_lengths.long()
    T = int(pl.max()) if T is None else T
    dec = gr.OracleDecoder(m, max_len, B=B)
    g = torch.Generator().manual_seed(0)
    for li in range(d.layers):
        for c in (dec.cache.k[li], dec.cache.v[li]):
            c[:, :, :T] = torch.randn(B, d.n_kv, T, d.head_dim, generator=g).to(torch.bfloat16)
    dec.pos = T
    kpos = torch.arange(max_len)
    state = {"toks": torch.randint(0, d.vocab, (B,), generator=g)}

    def step():
        valid = (kpos[None, :] < pl[:, None]) | ((kpos >= T) & (kpos <= dec.pos))[None, :]
        lg = dec.step(state["toks"], dec.pos - (T - pl), valid)
        state["toks"] = lg.argmax(-1)

    times = _timed_loop(step, seconds)
    per_step = statistics.median(times)
    return {"value": round(B / per_step, 3), "unit": "tok/s", "cores": torch.get_num_threads(),
            "kind": "port", "sample": f"{len(times)} full decode steps of {B} stream(s), 40 layers, bf16, the GPU "
            f"arm's prompt lengths (mean {float(pl.float().mean()):.0f}, padded to {T}), static cache {max_len}, "
            f"median step {per_step * 1000:.1f} ms; decode only (no prefill)",
            "affinity_cpus": len(os.sched_getaffinity(0))}


def cpu_verify(seconds: float):
    """The reference's verify forward (oracle restatement of
    SpeculativeDecoder._verify_step_fused, bf16, CPU): 8 tokens at cache slot
    600 over a random 600-position cache, repeated (each call rewinds)."""
    from oracle import granite_ref as gr

    m = _oracle_model()
    d = m.d
    dec = gr.OracleDecoder(m, VERIFY["max_len"])
    g = torch.Generator().manual_seed(0)
    for li in range(d.layers):
        for c in (dec.cache.k[li], dec.cache.v[li]):
            c[:, :, :VERIFY["ctx"]] = torch.randn(1, d.n_kv, VERIFY["ctx"], d.head_dim, generator=g).to(torch.bfloat16)
    ids = torch.randint(0, d.vocab, (VERIFY["m"],), generator=g)
    times = _timed_loop(lambda: dec.verify(ids, VERIFY["ctx"]).argmax(-1), seconds)
    per = statistics.median(times)
    return {"value": round(1.0 / per, 3), "unit": "verify/s", "cores": torch.get_num_threads(), "kind": "port",
            "sample": f"{len(times)} verify forwards of {VERIFY['m']} tokens at cache 600, 40 layers, bf16, median "
                      f"{per * 1000:.1f} ms", "affinity_cpus": len(os.sched_getaffinity(0))}

# --------------------------------------------------------------------------- #
def _engine(name, fmt, dev):
    from starling_b200 import synthetic as syn
    from starling_b200.engine import GraniteDims, GraniteEngine

    wl = WORKLOADS[name]
    d = GraniteDims()
    weights = syn.make_weights(d, seed=0, device=dev)
    eng = GraniteEngine(d, weights, fmt, max_cache_len=wl["max_len"], max_batch=wl["batch"], device=dev)
    embed = weights["embed_tokens.weight"]
    del weights
    torch.cuda.empty_cache()
    return eng, embed


def bench_workload(name, args, rank, world, local_rank, dev, with_cpu):
    """Device-timed decode tok/s of one workload (all ranks), its dominant
    kernel's roofline, e2e through generate(), and the CPU baseline."""
    from starling_b200 import synthetic as syn

    wl = WORKLOADS[name]
    fmt = (args.fmt if name == args.workload else None) or wl["fmt"]
    B, K, W, kr = wl["batch"], args.steps, args.warmup, wl["k_replay"]
    eng, embed = _engine(name, fmt, dev)
    d = eng.dims
    inp = syn.b1_inputs(embed, seed=0) if B == 1 else syn.batched_inputs(d.hidden, batch=B, seed=rank)
    del embed
    t = decode_timing(eng, B, inp.inputs_embeds, None if B == 1 else inp.prompt_lengths, inp.T, K, W, kr, world,
                      dev, local_rank)
    value = B * K * world / (t["ms"] / 1000.0)
    peak, peak_kind = _peaks()
    dom = dominant_kernel(eng, t["state"], d, B, inp.T, fmt, t["reset"], name)
    if eng.fused_step_ok(t["state"]) and B == 1:
        # the step is ONE launch of the fused kernel: its roofline is the
        # step's algorithmic bytes (every weight once + the valid K/V rows)
        # over the device time of a step
        wbytes = eng.lm_head.nbytes + sum(L[k].nbytes for L in eng.layers for k in ("qkv", "o", "gate_up", "down"))
        kvb = (inp.T + 1 + K // 2) * d.layers * 2 * d.n_kv * d.head_dim * 2  # mean context over the timed steps
        step_s = t["ms"] / K / 1e3
        gbs = (wbytes + kvb) / step_s / 1e9
        prof = PROFILED_TRAFFIC[("b1", "step")]
        dom["roofline"] = {"bound": "hbm", "achieved": round(gbs, 1), "peak": peak, "unit": "GB/s",
                           "frac": round(gbs / peak, 4), "traffic": round(prof[0] * (wbytes + kvb) / prof[1]),
                           "traffic_source": f"ncu capture in {prof[2]}, scaled by algorithmic bytes",
                           "kernel": "k_step (the whole decode step, one cooperative launch)",
                           "algorithmic_bytes_per_launch": wbytes + kvb, "avg_launch_us": round(step_s * 1e6, 3)}
    dom["roofline"]["peak_kind"] = peak_kind
    e2e = run_e2e(eng, wl, inp, B, dev, world)
    out = {
        "value": round(value, 2), "unit": "tok/s", "ms_per_step": round(t["ms"] / K, 5),
        "dtype": f"bf16 activations, {fmt} weights",
        "config": {
            "workload": wl["desc"], "model": "Granite-style 40-layer decoder (hidden 2048, 16/4 heads, inter 8192, "
            "vocab 100352)", "streams_per_gpu": B, "global_batch": B * world, "prompt_len_padded": inp.T,
            "weight_format": fmt, "graph_steps_per_replay": kr, "max_cache_len": eng.max_cache_len,
            "l2": f"inputs larger than L2 (weights {eng.weight_bytes / 1e9:.2f} GB/step)",
        },
        "gpu_launches": K * t["launches_per_step"],
        "clocks": t["clocks"],
        "roofline": dom["roofline"],
        "dominant_kernel": dom["info"],
        "e2e": e2e,
    }
    if with_cpu and rank == 0 and world == 1 and not args.no_cpu:
        pl = None if B == 1 else inp.prompt_lengths
        out["cpu_baseline"] = cpu_baseline(B, args.cpu_seconds if B > 1 else args.cpu_seconds / 2, pl, inp.T,
                                           wl["max_len"])
    return out, eng


def bench_strong(eng, args, rank, world, local_rank, dev):
    """Strong scaling: one fixed batch of 48 streams (prompts U[300,900],
    seed 0) dealt over the ranks by prompt length; each rank decodes its share
    with no collective; value = 48 x K tokens over the max-over-ranks time."""
    from starling_b200 import synthetic as syn
    from starling_b200.shard import shard_streams

    wl = WORKLOADS["b48"]
    inp = syn.batched_inputs(eng.dims.hidden, batch=48, seed=0)
    mine = shard_streams(inp.prompt_lengths.tolist(), world)[rank]
    pl = inp.prompt_lengths[mine]
    T = int(pl.max())
    emb = inp.inputs_embeds[mine, :T].contiguous()
    t = decode_timing(eng, len(mine), emb, pl, T, args.steps, args.warmup, wl["k_replay"], world, dev, local_rank)
    return {"value": round(48 * args.steps / (t["ms"] / 1000.0), 2), "unit": "tok/s",
            "ms_per_step": round(t["ms"] / args.steps, 5), "global_batch": 48, "streams_per_gpu": len(mine),
            "scaling": "strong",
            "note": "every GPU still streams all weights each step, so a fixed 48-stream batch scales far below N x"}


def bench_verify(eng, args, dev, with_cpu):
    """Verify forwards of 8 tokens at cache slot 600 (NVFP4, B=1): graph
    replays back to back, each rewinding to slot 600 (a verify forward leaves
    the slot where it was), timed with CUDA events; e2e through
    SpeculativeDecoder.verify with the ids in host memory."""
    from starling_b200 import _lib
    from starling_b200.multistep import MultiStepLLMMega
    from starling_b200.speculative import SpeculativeDecoder

    v = VERIFY
    d = eng.dims
    g = torch.Generator().manual_seed(3)
    eng.prefill(torch.randn(1, v["ctx"], d.hidden, generator=g).to(torch.bfloat16).to(dev))
    ids = torch.randint(0, d.vocab, (v["m"],), generator=g)
    st = eng.new_state(1, v["m"], _lib.SB_MODE_VERIFY, out_steps=1)
    st.ids.copy_(ids.to(dev))
    st.set_slot(v["ctx"], pad_len=v["ctx"])
    for _ in range(2):
        n0 = int(eng.lib.sb_launch_count())
        eng.decode_step(st, 0)
        launches = int(eng.lib.sb_launch_count()) - n0
    torch.cuda.synchronize()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        eng.decode_step(st, 0)
    for _ in range(args.warmup):
        graph.replay()
    stream = torch.cuda.current_stream()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    torch.cuda.synchronize()
    e0.record(stream)
    for _ in range(v["rounds"]):
        graph.replay()
    e1.record(stream)
    torch.cuda.synchronize()
    ms = e0.elapsed_time(e1) / v["rounds"]
    del graph
    peak, peak_kind = _peaks()
    wbytes = eng.lm_head.nbytes + sum(L[k].nbytes for L in eng.layers for k in ("qkv", "o", "gate_up", "down"))
    kvb = (v["ctx"] + v["m"]) * d.layers * 2 * d.n_kv * d.head_dim * 2
    gbs = (wbytes + kvb) / (ms * 1e-3) / 1e9
    # e2e: the public verify call, ids from pinned host memory, argmaxes + accept length read back
    spec = SpeculativeDecoder(MultiStepLLMMega(engine=eng, steps_per_replay=8))
    id_list = ids.tolist()
    spec.verify(id_list, v["ctx"])
    torch.cuda.synchronize()
    t0 = time.perf_counter()
    for _ in range(v["rounds"]):
        spec.verify(id_list, v["ctx"])
    e2e_s = (time.perf_counter() - t0) / v["rounds"]
    out = {
        "metric": "verify forwards/s", "value": round(1000.0 / ms, 2), "unit": "verify/s", "ms_per_verify": round(ms, 5),
        "tokens_per_verify": v["m"], "rounds": v["rounds"], "dtype": "bf16 activations, nvfp4 weights",
        "config": {"workload": v["desc"], "cache_positions": v["ctx"], "weight_format": "nvfp4"},
        "gpu_launches": v["rounds"] * launches,
        "roofline": {"bound": "hbm", "achieved": round(gbs, 1), "peak": peak, "unit": "GB/s",
                     "frac": round(gbs / peak, 4), "traffic": None, "kernel": "whole verify forward",
                     "algorithmic_bytes_per_launch": wbytes + kvb, "peak_kind": peak_kind},
        "e2e": {"value": round(1.0 / e2e_s, 2), "unit": "verify/s", "h2d_bytes_per_step": 8 * v["m"],
                "d2h_bytes_per_step": 8 * (v["m"] + 1),
                "note": "SpeculativeDecoder.verify: pinned H2D of the ids, graph replay, one D2H of argmaxes + "
                        "accept length per round; host clock"},
    }
    if with_cpu and not args.no_cpu:
        out["cpu_baseline"] = cpu_verify(args.cpu_seconds / 2)
    return out

# --------------------------------------------------------------------------- #
def run_native(args, rank, world, local_rank):
    torch.cuda.set_device(local_rank)
    dev = torch.device("cuda", local_rank)
    name = args.workload
    head, eng = bench_workload(name, args, rank, world, local_rank, dev, with_cpu=True)
    out = {
        "metric": "decode tok/s", "value": head["value"], "unit": "tok/s", "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": head["ms_per_step"], "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": head["dtype"],
        "data": "synthetic (seeded random-init weights N(0,0.02), N(0,1) embeddings)",
        "config": {**head["config"], "parallelism": f"stream sharding x{world}, no collective"},
    }
    for k in ("gpu_launches", "clocks", "roofline", "dominant_kernel", "e2e", "cpu_baseline"):
        if k in head:
            out[k] = head[k]
    if world > 1 and name == "b48":
        out["strong_scaling"] = bench_strong(eng, args, rank, world, local_rank, dev)
    if world == 1 and not args.headline_only:
        if name == "b48":
            del eng
            torch.cuda.empty_cache()
            out["b1"], eng = bench_workload("b1", args, rank, world, local_rank, dev, with_cpu=True)
        out["verify"] = bench_verify(eng, args, dev, with_cpu=True)
    return out


def run_reference(args, rank, world):
    """Reference arm: the reference's eager CPU decode path (oracle
    restatement of FusedLLMMega._decode_step_eager, bf16) on the host cores,
    on the GPU arm's workloads (same prompt lengths); rank 0 only."""
    if rank != 0:
        return None
    from starling_b200 import synthetic as syn

    torch.set_num_threads(len(os.sched_getaffinity(0)))
    wl = WORKLOADS[args.workload]
    B = wl["batch"]
    if B == 1:
        cpu = cpu_baseline(1, args.cpu_seconds, None, 320, wl["max_len"])
    else:
        inp = syn.batched_inputs(2048, batch=B, seed=0)
        cpu = cpu_baseline(B, args.cpu_seconds, inp.prompt_lengths, inp.T, wl["max_len"])
    v = cpu["value"]
    out = {
        "impl": "reference", "metric": "decode tok/s", "value": v, "unit": "tok/s", "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(1000.0 * B / v, 3),
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "bf16",
        "data": "synthetic", "config": {"workload": wl["desc"] + " (CPU eager reference path; bf16 weights)",
                                        "streams": B},
        "cpu_baseline": cpu,
        "e2e": {"value": v, "unit": "tok/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    if args.workload == "b48" and not args.headline_only:
        b1 = cpu_baseline(1, args.cpu_seconds / 2, None, 320, WORKLOADS["b1"]["max_len"])
        out["b1"] = {"value": b1["value"], "unit": "tok/s", "cpu_baseline": b1}
        vf = cpu_verify(args.cpu_seconds / 2)
        out["verify"] = {"value": vf["value"], "unit": "verify/s", "cpu_baseline": vf}
    return out


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=128)
    ap.add_argument("--warmup", type=int, default=8)
    ap.add_argument("--impl", default="native", choices=["native", "reference"])
    ap.add_argument("--workload", default="b48", choices=sorted(WORKLOADS))
    ap.add_argument("--fmt", default=None)
    ap.add_argument("--cpu-seconds", type=float, default=16.0)
    ap.add_argument("--no-cpu", action="store_true")
    ap.add_argument("--headline-only", action="store_true", help="skip the b1 / verify objects")
    args = ap.parse_args()
    if args.warmup < 3:
        raise SystemExit("--warmup must be >= 3")
    # stdout carries exactly one JSON line: anything libraries print (NCCL's
    # banner, warnings) goes to stderr instead
    json_out = os.fdopen(os.dup(1), "w")
    os.dup2(2, 1)
    rank, world, local_rank = _env_int("RANK", 0), _env_int("WORLD_SIZE", 1), _env_int("LOCAL_RANK", 0)
    if args.impl == "reference":
        out = run_reference(args, rank, world)
        if out is not None:
            print(json.dumps(out), file=json_out, flush=True)
        return
    if world > 1:
        import datetime

        import torch.distributed as dist

        torch.cuda.set_device(local_rank)
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300),
                                device_id=torch.device("cuda", local_rank))
    try:
        out = run_native(args, rank, world, local_rank)
        if rank == 0:
            print(json.dumps(out), file=json_out, flush=True)
    finally:
        if world > 1:
            import torch.distributed as dist

            dist.destroy_process_group()


if __name__ == "__main__":
    main()
