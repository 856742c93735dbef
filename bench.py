"""Decode throughput benchmark for the native B200 Granite decode path.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--workload b48|b1] [--fmt F]
    python bench.py --impl reference ...          # the reference's eager CPU path

One timed "step" is one greedy decode step of every stream (B tokens per
GPU).  Workloads (synthetic, seeded; see starling_b200/synthetic.py):

* ``b48`` (default): 48 streams per GPU (weak scaling), FP8 e4m3 per-channel
  weights, prompt lengths U[300, 900], 128 greedy steps, 40-layer decoder;
* ``b1``: one stream, NVFP4 weights, 300 audio embeddings + 20 prompt ids,
  128 greedy steps as K=8-step graph replays.

Under torchrun each rank decodes its own 48 streams with no collective on the
data path (streams are independent); only the timing barrier and the
max-over-ranks reduction use the process group.
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

WORKLOADS = {
    "b48": dict(batch=48, fmt="fp8", max_len=1040, k_replay=8, desc="batched long-audio decode, B=48/GPU, FP8 e4m3 per-channel, prompts U[300,900], 128 greedy steps"),
    "b1": dict(batch=1, fmt="nvfp4", max_len=640, k_replay=8, desc="B=1 greedy decode, NVFP4, 300 audio embeds + 20 prompt ids, 128 steps as K=8 graph replays"),
}


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
    """nvidia-smi clocks / throttle reasons sampled during the timed region."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, device_index: int):
        try:  # address the GPU by UUID: robust to CUDA_VISIBLE_DEVICES remapping
            self.idx = "GPU-" + str(torch.cuda.get_device_properties(device_index).uuid)
        except Exception:
            self.idx = str(device_index)
        self.proc = None
        self.lines = []

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits", "-lms", "200",
                 "-i", self.idx], stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self._t = threading.Thread(target=self._read, daemon=True)
            self._t.start()
        except (FileNotFoundError, OSError):
            self.proc = None
        return self

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def __exit__(self, *a):
        if self.proc is not None:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()

    def summary(self):
        sm, mx, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for ln in self.lines:
            parts = [x.strip() for x in ln.split(",")]
            if len(parts) < 9:
                continue
            try:
                sm.append(float(parts[1]))
                mx = float(parts[2])
            except ValueError:
                continue
            for n, v in zip(names, parts[5:9]):
                if v.lower() == "active":
                    reasons.add(n)
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": mx, "reasons": sorted(reasons),
                "samples": len(sm)}


# --------------------------------------------------------------------------- #
def run_native(args, rank, world, local_rank):
    import torch.distributed as dist

    from starling_b200 import _lib
    from starling_b200.batched import BatchedLLMMega
    from starling_b200.engine import GraniteDims, GraniteEngine
    from starling_b200.multistep import MultiStepLLMMega
    from starling_b200 import synthetic as syn

    torch.cuda.set_device(local_rank)
    dev = torch.device("cuda", local_rank)
    wl = dict(WORKLOADS[args.workload])
    fmt = args.fmt or wl["fmt"]
    d = GraniteDims()
    B = wl["batch"]
    K = args.steps
    weights = syn.make_weights(d, seed=0, device=dev)
    eng = GraniteEngine(d, weights, fmt, max_cache_len=wl["max_len"], max_batch=B, device=dev)
    embed_cpu = weights["embed_tokens.weight"]
    del weights
    torch.cuda.empty_cache()

    # ---- inputs (this rank's streams) and prefill ------------------------------
    if B == 1:
        inp = syn.b1_inputs(embed_cpu, seed=0)
        dec = MultiStepLLMMega(engine=eng, steps_per_replay=wl["k_replay"])
        first = dec.prefill(inp.inputs_embeds.to(dev))
        st = dec.state
        T = inp.T
        snap_ids = first.view(-1).clone()
        fin0 = None
    else:
        inp = syn.batched_inputs(d.hidden, batch=B, seed=rank)
        dec = BatchedLLMMega(engine=eng, max_batch_size=B, steps_per_replay=wl["k_replay"])
        dec.prefill(inp.inputs_embeds.to(dev), inp.prompt_lengths)
        st = dec.state
        T = inp.T
        snap_ids = st.ids.clone()
        fin0 = st.finished.clone()
    if T + K + args.warmup > eng.max_cache_len:
        raise SystemExit(f"steps+warmup exceed the cache ({T}+{K}+{args.warmup} > {eng.max_cache_len})")

    kr = wl["k_replay"]
    graphs = {}

    def capture(n):
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g):
            for j in range(n):
                eng.decode_step(st, j)
        return g

    def reset():
        st.ids.copy_(snap_ids)
        if fin0 is not None:
            st.finished.copy_(fin0)
        st.set_slot(T, pad_len=T)

    reset()
    for _ in range(2):  # eager warm-up of every kernel configuration before capture
        n0 = int(eng.lib.sb_launch_count())
        eng.decode_step(st, 0)
        launches_per_step = int(eng.lib.sb_launch_count()) - n0
    torch.cuda.synchronize()
    graphs[kr] = capture(kr)
    if K % kr:
        graphs[1] = capture(1)
    reset()

    def run_steps(n):
        for _ in range(n // kr):
            graphs[kr].replay()
        for _ in range(n % kr):
            graphs[1].replay() if 1 in graphs else eng.decode_step(st, 0)

    # warm-up (untimed), then reset to the first decode position
    if args.warmup % kr and 1 not in graphs:
        graphs[1] = capture(1)
        reset()
    run_steps(args.warmup)
    torch.cuda.synchronize()
    reset()
    torch.cuda.synchronize()

    def barrier():
        if world > 1:
            dist.barrier()

    stream = torch.cuda.current_stream()
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    barrier()
    torch.cuda.synchronize()
    with ClockSampler(local_rank) as clk:
        torch.cuda.nvtx.range_push("timed_steps")  # ncu --nvtx-include "timed_steps/" selects these launches
        ev0.record(stream)
        run_steps(K)
        ev1.record(stream)
        torch.cuda.nvtx.range_pop()
        torch.cuda.synchronize()
    barrier()
    ms = ev0.elapsed_time(ev1)
    t = torch.tensor([ms], device=dev)
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    ms_max = float(t.item())
    tokens = B * K * world
    value = tokens / (ms_max / 1000.0)

    # ---- dominant kernel, timed live on the launching stream ----------------------
    peak, peak_kind = _peaks()
    dom = dominant_kernel(eng, st, d, B, T, fmt, reset, args.workload)

    # ---- e2e through the public API with host (pinned) buffers --------------------
    e2e = run_e2e(eng, wl, inp, B, K, dev, world)

    # ---- CPU baseline (rank 0, N=1 only) -------------------------------------------
    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu:
        cpu = cpu_baseline(B, args.cpu_seconds)

    reset()
    for g in graphs.values():
        del g
    out = {
        "metric": "decode tok/s",
        "value": round(value, 2),
        "unit": "tok/s",
        "n_gpus": world,
        "steps": K,
        "warmup": args.warmup,
        "ms_per_step": round(ms_max / K, 5),
        "higher_is_better": True,
        "scaling": "weak",
        "vs_baseline": None,
        "dtype": f"bf16 activations, {fmt} weights",
        "data": "synthetic (seeded random-init weights N(0,0.02), N(0,1) embeddings)",
        "config": {
            "workload": wl["desc"], "model": "Granite-style 40-layer decoder (hidden 2048, 16/4 heads, inter 8192, vocab 100352)",
            "streams_per_gpu": B, "global_batch": B * world, "prompt_len_padded": T,
            "weight_format": fmt, "graph_steps_per_replay": kr, "max_cache_len": eng.max_cache_len,
            "parallelism": f"stream sharding x{world}, no collective", "l2": "inputs larger than L2 (weights "
            f"{eng.weight_bytes / 1e9:.2f} GB/step)",
        },
        "gpu_launches": K * launches_per_step,
        "clocks": clk.summary(),
        "roofline": dom["roofline"],
        "dominant_kernel": dom["info"],
        "e2e": e2e,
    }
    out["roofline"]["peak_kind"] = peak_kind
    if cpu is not None:
        out["cpu_baseline"] = cpu
    return out


# DRAM traffic per launch (dram__bytes_read.sum + dram__bytes_write.sum) from
# one ncu capture of the same kernel and shape (profiles/), with the
# algorithmic bytes of the captured case: the bench scales the traffic to its
# own launch by the ratio of algorithmic bytes (same kernel, same tiling).
PROFILED_TRAFFIC = {
    ("b48", "attention"): (80.179456e6 + 2.41664e6, 61.5e6, "profiles/attention_b48_decode.md"),
    ("b48", "gate_up"): (33.9008e6, 33.62e6, "profiles/tcgen05_gemm_gate_up_fp8_b48.md"),
    ("b1", "gate_up"): (18.93376e6, 18.87e6, "profiles/gemv_gate_up_nvfp4_b1.md"),
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


def run_e2e(eng, wl, inp, B, K, dev, world):
    """The public generate() call with inputs in pinned host memory: H2D of the
    prompt embeddings, prefill, K decode steps, D2H of the token ids."""
    import torch.distributed as dist
    from starling_b200.batched import BatchedLLMMega
    from starling_b200.multistep import MultiStepLLMMega

    emb = inp.inputs_embeds.pin_memory()
    if B == 1:
        dec = MultiStepLLMMega(engine=eng, steps_per_replay=wl["k_replay"])
        call = lambda: dec.generate(emb, max_new_tokens=K + 1, eos_token_id=-1)  # noqa: E731
    else:
        dec = BatchedLLMMega(engine=eng, max_batch_size=B, steps_per_replay=wl["k_replay"])
        call = lambda: dec.generate(emb, prompt_lengths=inp.prompt_lengths, max_new_tokens=K + 1,  # noqa: E731
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
    sec = sorted(secs)[1]
    t = torch.tensor([sec], device=dev)
    n = torch.tensor([float(ntok)], device=dev)
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        dist.all_reduce(n, op=dist.ReduceOp.SUM)
    h2d = emb.numel() * emb.element_size()
    d2h = ntok * 8
    return {"value": round(float(n.item()) / float(t.item()), 2), "unit": "tok/s",
            "h2d_bytes_per_step": int(h2d // K), "d2h_bytes_per_step": int(d2h // K),
            "note": "public generate() calls per GPU (after one warm-up call), median of 3, each incl. prefill "
                    "of the prompts (timed on the host clock)"}


# --------------------------------------------------------------------------- #
def cpu_baseline(B: int, seconds: float):
    """The reference's eager decode step (oracle restatement, bf16, torch CPU)
    on a bounded sample: as many full 40-layer decode steps of B streams as fit
    in ``seconds`` (at least one), at context ~T with random cache contents."""
    from oracle import granite_ref as gr

    torch.set_grad_enabled(False)
    d = gr.BASELINE_DIMS
    w = gr.make_weights(d, seed=0, std=0.02)
    m = gr.OracleModel(d, w)
    max_len = 640 if B == 1 else 1040
    T = 320 if B == 1 else 900
    dec = gr.OracleDecoder(m, max_len, B=B)
    g = torch.Generator().manual_seed(0)
    for li in range(d.layers):
        dec.cache.k[li][:, :, :T] = torch.randn(B, d.n_kv, T, 128, generator=g).to(torch.bfloat16)
        dec.cache.v[li][:, :, :T] = torch.randn(B, d.n_kv, T, 128, generator=g).to(torch.bfloat16)
    dec.pos = T
    toks = torch.randint(0, d.vocab, (B,), generator=g)
    kpos = torch.arange(max_len)
    times = []
    t_end = time.perf_counter() + seconds
    while True:
        valid = (kpos <= dec.pos).view(1, -1).expand(B, -1)
        t0 = time.perf_counter()
        lg = dec.step(toks, torch.full((B,), dec.pos), valid)
        times.append(time.perf_counter() - t0)
        toks = lg.argmax(-1)
        if time.perf_counter() > t_end or len(times) >= 64:
            break
    per_step = statistics.median(times)
    return {"value": round(B / per_step, 3), "unit": "tok/s", "cores": torch.get_num_threads(),
            "kind": "port", "sample": f"{len(times)} full decode steps of {B} stream(s), 40 layers, bf16, "
            f"context {T}, median step {per_step * 1000:.1f} ms",
            "affinity_cpus": len(os.sched_getaffinity(0))}


def run_reference(args, rank, world):
    """Reference arm: the reference's eager CPU decode path (oracle
    restatement of FusedLLMMega._decode_step_eager) on the host cores."""
    if rank != 0:
        return None
    wl = WORKLOADS[args.workload]
    B = wl["batch"]
    torch.set_num_threads(len(os.sched_getaffinity(0)))
    cpu = cpu_baseline(B, args.cpu_seconds)
    v = cpu["value"]
    return {
        "impl": "reference", "metric": "decode tok/s", "value": v, "unit": "tok/s", "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(1000.0 * B / v, 3),
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "bf16",
        "data": "synthetic", "config": {"workload": wl["desc"] + " (CPU eager reference path; bf16 weights)",
                                        "streams": B},
        "cpu_baseline": cpu,
        "e2e": {"value": v, "unit": "tok/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=128)
    ap.add_argument("--warmup", type=int, default=8)
    ap.add_argument("--impl", default="native", choices=["native", "reference"])
    ap.add_argument("--workload", default="b48", choices=sorted(WORKLOADS))
    ap.add_argument("--fmt", default=None)
    ap.add_argument("--cpu-seconds", type=float, default=20.0)
    ap.add_argument("--no-cpu", action="store_true")
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
