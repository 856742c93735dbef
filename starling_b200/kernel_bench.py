"""Per-kernel timings of the decode path on one GPU (also the small cases the
ncu summaries under profiles/ are captured on).

    python -m starling_b200.kernel_bench ops --workload b48        # every op of a step, graphs of 40 launches;
                                                                   # the whole step per-op and fused (one launch)
    python -m starling_b200.kernel_bench attention --batch 48      # sb_attention alone
    python -m starling_b200.kernel_bench linear --fmt fp8 --n 16384 --k 2048 --m 48
    python -m starling_b200.kernel_bench step --workload b48 --layers 4   # one eager step in NVTX range "step"
    python -m starling_b200.kernel_bench step --workload b1 --path fused  # the one-launch fused step
    python -m starling_b200.kernel_bench prefill --layers 40       # one native prefill of the b48 prompts
    python -m starling_b200.kernel_bench verify --layers 40        # one 8-token verify forward, B=1, NVFP4
    python -m starling_b200.kernel_bench gemv-table                # dequant-GEMV microbench, B=1, 3 formats

Workloads (same as bench.py): b48 = 48 streams, FP8 weights, prompts
U[300,900]; b1 = one stream, NVFP4 weights, 320 prompt positions.  Weights are
seeded random-init N(0,0.02); every time is taken with CUDA events on the
launching stream after warm-up, device time per launch.
"""

from __future__ import annotations

import argparse
import ctypes as C
import sys

import torch

from . import _lib, pack
from . import synthetic as syn
from ._lib import check, ptr
from .batched import BatchedLLMMega
from .engine import GraniteDims, GraniteEngine
from .multistep import MultiStepLLMMega

WORKLOADS = {"b48": (48, "fp8", 1040), "b1": (1, "nvfp4", 640)}
OPS = ["qkv", "attention", "o", "gate_up", "down"]


def _graph_time(fn, reps: int = 5) -> float:
    """Device microseconds of one call of fn (captured once into a graph)."""
    fn()
    torch.cuda.synchronize()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        fn()
    g.replay()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(reps):
        g.replay()
    e1.record()
    torch.cuda.synchronize()
    return e0.elapsed_time(e1) * 1000.0 / reps


def _decoder(workload: str, layers: int):
    B, fmt, max_len = WORKLOADS[workload]
    dev = torch.device("cuda")
    d = GraniteDims(layers=layers)
    w = syn.make_weights(d, seed=0, device=dev)
    eng = GraniteEngine(d, w, fmt, max_cache_len=max_len, max_batch=B, device=dev)
    emb = w["embed_tokens.weight"]
    del w
    torch.cuda.empty_cache()
    if B == 1:
        inp = syn.b1_inputs(emb, seed=0)
        dec = MultiStepLLMMega(engine=eng, steps_per_replay=8)
        dec.prefill(inp.inputs_embeds.to(dev))
    else:
        inp = syn.batched_inputs(d.hidden, batch=B, seed=0)
        dec = BatchedLLMMega(engine=eng, max_batch_size=B, steps_per_replay=8)
        dec.prefill(inp.inputs_embeds.to(dev), inp.prompt_lengths)
    return eng, dec.state, inp.T, d


def cmd_ops(a) -> None:
    eng, st, T, d = _decoder(a.workload, a.layers)
    lib = eng.lib
    total = 0.0
    for op, name in enumerate(OPS):
        def run(op=op):
            for layer in range(d.layers):
                check(lib.sb_decode_op(C.byref(eng.cmodel), C.byref(st.c), layer, op, 0, _lib.current_stream()))
        st.set_slot(T, pad_len=T)
        us = _graph_time(run) / d.layers
        total += us * d.layers
        print(f"{a.workload} {name:9s} {us:9.2f} us per launch (mean over {d.layers} layers)")
    st.set_slot(T, pad_len=T)
    lm = _graph_time(lambda: check(lib.sb_decode_op(C.byref(eng.cmodel), C.byref(st.c), 0, _lib.SB_OP_LM_HEAD, 0,
                                                    _lib.current_stream())))
    print(f"{a.workload} lm_head   {lm:9.2f} us")
    times = {}
    for path in ("ops", "fused"):
        eng.step_path = path
        if path == "fused" and not eng.fused_step_ok(st):
            continue
        st.set_slot(T, pad_len=T)
        times[path] = _graph_time(lambda: eng.decode_step(st, 0))
    eng.step_path = "auto"
    print(f"{a.workload} sum of ops {total + lm:9.1f} us; one graphed step: " +
          ", ".join(f"{k} {v:.1f} us" for k, v in times.items()))


def cmd_step(a) -> None:
    eng, st, T, d = _decoder(a.workload, a.layers)
    eng.step_path = a.path
    for _ in range(2):
        eng.decode_step(st, 0)
    torch.cuda.synchronize()
    n0 = int(eng.lib.sb_launch_count())
    torch.cuda.nvtx.range_push("step")
    eng.decode_step(st, 0)
    torch.cuda.nvtx.range_pop()
    torch.cuda.synchronize()
    print(f"{a.workload}: one step, {d.layers} layers, {int(eng.lib.sb_launch_count()) - n0} launches")


def cmd_attention(a) -> None:
    B = a.batch
    layers = 4  # rotate over 4 layers' caches (> L2 at B=48)
    max_len = 1040 if B > 1 else 640
    d = GraniteDims(layers=layers, inter=256, vocab=256)
    g = torch.Generator(device="cuda").manual_seed(1)
    w = {"embed_tokens.weight": (256, 2048), "norm.weight": (2048,)}
    for i in range(layers):
        p = f"layers.{i}."
        w.update({p + "input_layernorm.weight": (2048,), p + "post_attention_layernorm.weight": (2048,),
                  p + "self_attn.q_proj.weight": (2048, 2048), p + "self_attn.k_proj.weight": (512, 2048),
                  p + "self_attn.v_proj.weight": (512, 2048), p + "self_attn.o_proj.weight": (2048, 2048),
                  p + "mlp.gate_proj.weight": (256, 2048), p + "mlp.up_proj.weight": (256, 2048),
                  p + "mlp.down_proj.weight": (2048, 256)})
    w = {k: (torch.randn(s, generator=g, device="cuda") * 0.02).to(torch.bfloat16) for k, s in w.items()}
    eng = GraniteEngine(d, w, "bf16", max_cache_len=max_len, max_batch=B, tensor_cores=False)
    gen = torch.Generator().manual_seed(0)
    if B > 1:
        pl = torch.randint(300, 901, (B,), generator=gen)
        T = int(pl.max())
    else:
        pl, T = torch.tensor([320]), 320
    st = eng.new_state(B, 1, _lib.SB_MODE_DECODE, out_steps=1, prompt_len=pl, rope_off=T - pl)
    eng.kv.normal_()
    st.q.normal_()
    st.set_slot(T, pad_len=T)

    def run():
        for layer in range(a.reps):
            check(eng.lib.sb_attention(C.byref(eng.cmodel), C.byref(st.c), layer % layers, _lib.current_stream()))

    us = _graph_time(run) / a.reps
    nbytes = (int(pl.sum()) + B) * d.n_kv * 2 * 256
    print(f"attention B={B} ctx<= {T}: {us:.2f} us per launch; valid K/V bytes {nbytes / 1e6:.1f} MB "
          f"-> {nbytes / us / 1e3:.0f} GB/s; err={int(st.ctrl[_lib.SB_CTRL_ERR])}")


def cmd_prefill(a) -> None:
    """One native prefill of the b48 workload (48 prompts U[300,900], FP8), the
    timed call inside NVTX range "prefill"."""
    B, fmt, max_len = WORKLOADS["b48"]
    dev = torch.device("cuda")
    d = GraniteDims(layers=a.layers)
    w = syn.make_weights(d, seed=0, device=dev)
    eng = GraniteEngine(d, w, fmt, max_cache_len=max_len, max_batch=B, device=dev)
    del w
    torch.cuda.empty_cache()
    inp = syn.batched_inputs(d.hidden, batch=B, seed=0)
    emb = inp.inputs_embeds.to(dev)
    eng.prefill(emb, inp.prompt_lengths)
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    torch.cuda.nvtx.range_push("prefill")
    e0.record()
    eng.prefill(emb, inp.prompt_lengths)
    e1.record()
    torch.cuda.nvtx.range_pop()
    torch.cuda.synchronize()
    print(f"prefill b48 ({B} prompts, padded to {inp.T}, {int(inp.prompt_lengths.sum())} positions), "
          f"{a.layers} layers: {e0.elapsed_time(e1):.1f} ms")


def cmd_verify(a) -> None:
    """One graphed verify forward of 8 draft tokens at B = 1 (NVFP4, cache of
    600 positions: the speculative-verify workload) on each NVFP4 kernel
    choice, and its per-op times."""
    dev = torch.device("cuda")
    d = GraniteDims(layers=a.layers)
    w = syn.make_weights(d, seed=0, device=dev)
    eng = GraniteEngine(d, w, "nvfp4", max_cache_len=640, max_batch=1, device=dev)
    del w
    torch.cuda.empty_cache()
    eng.kv.normal_(generator=torch.Generator(device="cuda").manual_seed(1))
    st = eng.new_state(1, 8, _lib.SB_MODE_VERIFY, out_steps=1)
    st.ids.copy_(torch.randint(0, d.vocab, (8,), generator=torch.Generator().manual_seed(2)).to(dev))
    lib = eng.lib
    prev = lib.sb_set_nvfp4_path(_lib.SB_NVFP4_AUTO)
    try:
        for name, path in (("auto", _lib.SB_NVFP4_AUTO), ("mma_sync", _lib.SB_NVFP4_MMA_SYNC)):
            lib.sb_set_nvfp4_path(path)
            ops = []
            for op, opname in enumerate(OPS):
                def run(op=op):
                    for layer in range(d.layers):
                        check(lib.sb_decode_op(C.byref(eng.cmodel), C.byref(st.c), layer, op, 0,
                                               _lib.current_stream()))
                st.set_slot(600, pad_len=600)
                ops.append(f"{opname} {_graph_time(run) / d.layers:.2f}")
            st.set_slot(600, pad_len=600)
            lm = _graph_time(lambda: check(lib.sb_decode_op(C.byref(eng.cmodel), C.byref(st.c), 0,
                                                            _lib.SB_OP_LM_HEAD, 0, _lib.current_stream())))
            eng.step_path = "ops"
            st.set_slot(600, pad_len=600)
            full = _graph_time(lambda: eng.decode_step(st, 0))
            eng.step_path = "auto"
            print(f"verify 8 tokens, cache 600, {d.layers} layers, NVFP4 {name}: forward {full:.1f} us "
                  f"(per launch: {', '.join(ops)}, lm_head {lm:.2f} us)")
        lib.sb_set_nvfp4_path(_lib.SB_NVFP4_AUTO)
        if eng.fused_step_ok(st):
            eng.step_path = "fused"
            st.set_slot(600, pad_len=600)
            fused = _graph_time(lambda: eng.decode_step(st, 0))
            eng.step_path = "auto"
            print(f"verify 8 tokens, cache 600, {d.layers} layers, NVFP4 fused step: forward {fused:.1f} us")
    finally:
        lib.sb_set_nvfp4_path(prev)


def cmd_linear(a) -> None:
    lib = _lib.load()
    lib.sb_set_nvfp4_path({"auto": _lib.SB_NVFP4_AUTO, "block_scaled": _lib.SB_NVFP4_BLOCK_SCALED,
                           "mma_sync": _lib.SB_NVFP4_MMA_SYNC}[a.nvfp4_path])
    w = (torch.randn(a.n, a.k, device="cuda") * 0.02).to(torch.bfloat16)
    # rotate: 4 copies > L2 at large n
    copies = [pack.pack_matrix(w, a.fmt, tc=True, bs=a.fmt == "nvfp4") for _ in range(4)]
    cs = [p.c_struct() for p in copies]
    x = torch.randn(a.m, a.k, device="cuda").to(torch.bfloat16)
    y = torch.empty(a.m, a.n, dtype=torch.bfloat16, device="cuda")
    need = int(lib.sb_linear_workspace_bytes(C.byref(cs[0]), a.m))
    ws = torch.zeros(max(need, 16), dtype=torch.uint8, device="cuda")

    def run():
        for i in range(a.reps):
            check(lib.sb_linear_ex(C.byref(cs[i % 4]), ptr(x), ptr(y), a.m, ptr(ws), need, 1, _lib.current_stream()))

    us = _graph_time(run) / a.reps
    nbytes = copies[0].nbytes
    path = "tcgen05" if need else ("nvfp4 " + a.nvfp4_path if a.fmt == "nvfp4" else "gemv")
    print(f"linear {a.fmt} n={a.n} k={a.k} m={a.m} ({path}): {us:.2f} us per launch; weight bytes "
          f"{nbytes / 1e6:.2f} MB -> {nbytes / us / 1e3:.0f} GB/s")


def cmd_gemv_table(a) -> None:
    """The dequant-GEMV microbench at B = 1: NVFP4 / FP8 / INT8 weights of
    [8192 x 2048], [2048 x 8192] and the [100352 x 2048] lm_head, N(0, 0.02)
    weights, an N(0, 1) bf16 activation row, bf16 out.  Launches rotate over
    enough weight copies that they span >= 8x the 126 MB L2 (at least 16), so
    every launch streams its weight from HBM.  Algorithmic bytes = packed
    weight + scales + x + y; fraction of the measured copy peak."""
    import json
    from pathlib import Path

    lib = _lib.load()
    lib.sb_set_nvfp4_path(_lib.SB_NVFP4_AUTO)
    peak_file = Path(__file__).resolve().parent.parent / "MEASURED_PEAKS.json"
    peak = json.loads(peak_file.read_text())["hbm_gbs"] if peak_file.exists() else 6650.0
    g = torch.Generator(device="cuda").manual_seed(0)
    rows = []
    for n, k in ((8192, 2048), (2048, 8192), (100352, 2048)):
        w = (torch.randn(n, k, device="cuda", generator=g) * 0.02).to(torch.bfloat16)
        x = torch.randn(1, k, device="cuda", generator=g).to(torch.bfloat16)
        y = torch.empty(1, n, dtype=torch.bfloat16, device="cuda")
        for fmt in ("nvfp4", "fp8", "int8"):
            first = pack.pack_matrix(w, fmt, tc=False, bs=fmt == "nvfp4")
            ncopy = max(16, -(-8 * 126_000_000 // first.nbytes))
            copies = [first] + [pack.pack_matrix(w, fmt, tc=False, bs=fmt == "nvfp4") for _ in range(ncopy - 1)]
            cs = [c.c_struct() for c in copies]
            reps = ncopy

            def run():
                for i in range(reps):
                    check(lib.sb_linear(C.byref(cs[i]), ptr(x), ptr(y), 1, 1, _lib.current_stream()))

            us = _graph_time(run, reps=3) / reps
            nbytes = first.nbytes + 2 * k + 2 * n
            gbs = nbytes / us / 1e3
            rows.append(dict(fmt=fmt, n=n, k=k, us=round(us, 3), bytes=nbytes, gbs=round(gbs, 1),
                             frac=round(gbs / peak, 4), copies=ncopy))
            del copies, cs, first
            torch.cuda.empty_cache()
    print(f"| format | W [n x k] | us / launch | algorithmic bytes | GB/s | of measured {peak:.0f} GB/s |")
    print("|---|---|---|---|---|---|")
    for r in rows:
        print(f"| {r['fmt']} | {r['n']} x {r['k']} | {r['us']:.2f} | {r['bytes'] / 1e6:.2f} MB | {r['gbs']:.0f} | "
              f"{r['frac']:.3f} |")
    print(json.dumps({"gemv_b1": rows, "peak_gbs": peak}))


def main(argv=None) -> None:
    ap = argparse.ArgumentParser(description=__doc__.split("\n\n")[0])
    sub = ap.add_subparsers(dest="cmd", required=True)
    p = sub.add_parser("ops")
    p.add_argument("--workload", choices=list(WORKLOADS), default="b48")
    p.add_argument("--layers", type=int, default=40)
    p = sub.add_parser("step")
    p.add_argument("--workload", choices=list(WORKLOADS), default="b48")
    p.add_argument("--layers", type=int, default=4)
    p.add_argument("--path", choices=["auto", "ops", "fused"], default="auto")
    p = sub.add_parser("attention")
    p.add_argument("--batch", type=int, default=48)
    p.add_argument("--reps", type=int, default=20)
    p = sub.add_parser("verify")
    p.add_argument("--layers", type=int, default=40)
    p = sub.add_parser("prefill")
    p.add_argument("--layers", type=int, default=40)
    p = sub.add_parser("linear")
    p.add_argument("--fmt", default="fp8")
    p.add_argument("--n", type=int, default=16384)
    p.add_argument("--k", type=int, default=2048)
    p.add_argument("--m", type=int, default=48)
    p.add_argument("--reps", type=int, default=20)
    p.add_argument("--nvfp4-path", choices=["auto", "block_scaled", "mma_sync"], default="auto",
                   help="kernel for 1..8-row NVFP4 launches (sb_set_nvfp4_path)")
    sub.add_parser("gemv-table")
    a = ap.parse_args(argv)
    torch.set_grad_enabled(False)
    {"ops": cmd_ops, "step": cmd_step, "attention": cmd_attention, "linear": cmd_linear, "prefill": cmd_prefill,
     "verify": cmd_verify, "gemv-table": cmd_gemv_table}[a.cmd](a)


if __name__ == "__main__":
    sys.exit(main())
