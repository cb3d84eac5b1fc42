"""Benchmark of the int4 quantized-matmul hot path on B200 (prints ONE JSON line on rank 0).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

Headline workload ("1024-tok prefill"): one step is the
layers-outer prefill projection stack of a Gemma-4-E2B-shaped int4 model --
35 layers x {q, k, v, o, gate, up, down} fused dequant+tcgen05 GEMMs at
M = 1024 tokens (group-32 f16 scales, f16 activations, f32 accumulate), all
captured in one CUDA graph.  value = 1024 tokens / step time (whole job:
N replicas x 1024 / max-over-ranks time, weak scaling; there is no collective
on this path).  The 620 MB of packed weights exceed the 126 MB L2, so no flush
is needed between steps.  Attention, norms and RoPE are not part of this
workload (they are not in config 2).

Also reported (sub-objects): the decode GEMV stack (35 layers x 7 GEMVs at
M=1 plus the fused 262144-row lm_head+argmax, one CUDA graph per token) as
decode-GEMV tok/s and achieved HBM GB/s, and the lm_head alone (config 3).

--impl reference times the reference's algorithm on the host cores: the numpy
oracle (a restatement of the reference's numpy code; the reference itself is
Python and cannot travel to the GPU box) on a bounded sample of the same
workload, scaled to the same unit.
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

M_TOK = 1024
N_LAYERS = 35
SHAPES = {"q": (2048, 1536), "k": (256, 1536), "v": (256, 1536), "o": (1536, 2048),
          "gate": (6144, 1536), "up": (6144, 1536), "down": (1536, 6144)}
VOCAB, HID = 262144, 1536


def parse():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--kernel", default="", choices=["", "gemm_q4", "gemm_f16", "gemv", "lmhead"],
                    help="run one kernel --iters times on a single shape and exit (for ncu captures)")
    ap.add_argument("--shape", default="6144,1536", help="N,K of the weight for --kernel")
    ap.add_argument("--m", type=int, default=1024, help="rows of the activation for --kernel")
    ap.add_argument("--iters", type=int, default=3)
    return ap.parse_args()


def run_kernel_case(args):
    """One kernel on one shape, --iters launches after one warm-up (ncu target)."""
    import torch

    from slang_b200 import kernels as kern
    dev = torch.device("cuda", 0)
    n, k = (int(v) for v in args.shape.split(","))
    m = args.m
    g = torch.Generator(device=dev)
    g.manual_seed(0)
    w = torch.randint(0, 256, (n, k // 2), dtype=torch.uint8, device=dev, generator=g)
    s = (torch.randn((n, k // 32), device=dev, generator=g) * 0.02).abs().half()
    if args.kernel in ("gemm_q4", "gemm_f16"):
        a = torch.randn((m, k), device=dev, generator=g).half()
        c = torch.empty((m, n), dtype=torch.float16, device=dev)
        wf = kern.dequant_f16(w, s, k, n) if args.kernel == "gemm_f16" else None

        def op():
            if wf is None:
                kern.gemm_q4(a, w, s, C=c)
            else:
                kern.gemm(a, wf, c, m, n, k)
    else:
        x = torch.randn((m, k), device=dev, generator=g)
        y = torch.empty((m, n), device=dev)

        def op():
            if args.kernel == "gemv":
                kern.gemv_q4(w, s, x, y=y)
            else:
                kern.lmhead_argmax(w, s, x)
    op()
    torch.cuda.synchronize()
    # replay a CUDA graph of --iters launches so host overhead is not timed
    stream = torch.cuda.Stream()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph, stream=stream):
        for _ in range(args.iters):
            op()
    graph.replay()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    graph.replay()
    e1.record()
    e1.synchronize()
    us = e0.elapsed_time(e1) * 1e3 / args.iters
    kern.device_status()
    if args.kernel in ("gemm_q4", "gemm_f16"):
        rate = f"{2 * m * n * k / us / 1e6:.1f} TFLOP/s"
    else:
        rate = f"{(n * k // 2 + n * (k // 32) * 2 + m * k * 4 + m * n * 4) / us / 1e3:.1f} GB/s"
    print(f"ran {args.kernel} m={m} n={n} k={k} x{args.iters + 1}: {us:.2f} us/launch, {rate} "
          f"(graph of back-to-back launches; operands L2-warm when they fit in L2)")


# ------------------------------------------------------------------ helpers
class Clocks:
    """Sample SM clocks and throttle reasons with nvidia-smi during the timed region."""

    FIELDS = ["clocks.sm", "clocks.max.sm", "power.draw", "clocks_event_reasons.hw_slowdown",
              "clocks_event_reasons.hw_thermal_slowdown", "clocks_event_reasons.sw_thermal_slowdown",
              "clocks_event_reasons.sw_power_cap"]

    def __init__(self, gpu_id: str):
        self.proc = None
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", "-i", gpu_id, "--query-gpu=" + ",".join(self.FIELDS),
                 "--format=csv,noheader,nounits", "-lms", "200"],
                stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except OSError:
            self.proc = None

    def stop(self) -> dict:
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        self.proc.terminate()
        out, _ = self.proc.communicate(timeout=10)
        sm, smax, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for line in out.strip().splitlines():
            parts = [p.strip() for p in line.split(",")]
            if len(parts) < 7:
                continue
            try:
                sm.append(float(parts[0]))
                smax = float(parts[1])
            except ValueError:
                continue
            for nm, val in zip(names, parts[3:7]):
                if val.lower().startswith("active"):
                    reasons.add(nm)
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": smax,
                "reasons": sorted(reasons), "samples": len(sm)}


def gpu_id_for(torch, dev) -> str:
    try:
        return "GPU-" + str(torch.cuda.get_device_properties(dev).uuid)
    except Exception:
        vis = os.environ.get("CUDA_VISIBLE_DEVICES", "")
        return vis.split(",")[dev.index] if vis else str(dev.index)


def timed_graph(torch, graph, steps, warmup, stream):
    for _ in range(warmup):
        graph.replay()
    torch.cuda.synchronize()
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    start.record(stream)
    for _ in range(steps):
        graph.replay()
    end.record(stream)
    end.synchronize()
    return start.elapsed_time(end) / steps  # ms per step


def load_peaks():
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            p = json.load(f)
        return p["hbm_gbs"], p["bf16_tflops"], "measured"
    except Exception:
        return 6650.0, 1590.0, "fallback"


# ------------------------------------------------------------------ CPU baseline (oracle)
def cpu_sample_prefill(seconds_budget: float = 20.0) -> dict:
    """Time the numpy oracle on a bounded sample: the layer-0 gate projection at M=1024
    (dequant to f16 then f32 GEMM, the reference's _dq + _gemm math); scaled to the
    35-layer stack by parameter count (both dequant and matmul scale with it)."""
    import numpy as np

    from oracle import q4
    from slang_b200 import synth
    rng = np.random.default_rng(1)
    n, k = SHAPES["gate"]
    packed, scales = synth.q4_weight(rng, n, k)
    a = synth.activations(rng, M_TOK, k)
    times = []
    t_start = time.perf_counter()
    q4.gemm_q4(a, packed, scales)  # warm-up
    while len(times) < 5 and time.perf_counter() - t_start < seconds_budget:
        t0 = time.perf_counter()
        q4.gemm_q4(a, packed, scales)
        times.append(time.perf_counter() - t0)
    t = min(times)
    stack_params = N_LAYERS * sum(nn * kk for nn, kk in SHAPES.values())
    scale = stack_params / (n * k)
    return {"value": M_TOK / (t * scale), "unit": "tok/s", "cores": os.cpu_count(), "kind": "port",
            "sample": f"oracle q4.gemm_q4 (dq_f16 + fp32 numpy GEMM) of one gate projection "
                      f"[{n}x{k}] at M={M_TOK}, min of {len(times)} runs = {t*1e3:.1f} ms, "
                      f"scaled x{scale:.1f} by parameter count to the 35-layer stack"}


def run_reference(args):
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    vals = []
    for _ in range(args.warmup):
        cpu_sample_prefill(5.0)
    t0 = time.perf_counter()
    for _ in range(max(1, args.steps // 10)):
        vals.append(cpu_sample_prefill(5.0))
    wall = time.perf_counter() - t0
    v = statistics.median([x["value"] for x in vals])
    cb = dict(vals[0])
    cb["value"] = v
    line = {"metric": "1024-tok prefill tok/s (35-layer int4 projection GEMMs)", "value": v, "unit": "tok/s",
            "impl": "reference", "n_gpus": args.gpus, "steps": len(vals), "warmup": args.warmup,
            "ms_per_step": 1e3 * M_TOK / v, "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "f16", "data": "synthetic",
            "config": {"workload": "cfg2_prefill_proj_stack", "tokens": M_TOK, "layers": N_LAYERS,
                       "matrices": list(SHAPES), "parallelism": "cpu"},
            "cpu_baseline": cb,
            "e2e": {"value": v, "unit": "tok/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
            "wall_s": wall}
    print(json.dumps(line), flush=True)


# ------------------------------------------------------------------ GPU arm
def main():
    args = parse()
    if args.kernel:
        return run_kernel_case(args)
    if args.impl == "reference":
        return run_reference(args)

    import torch
    import torch.distributed as dist

    from slang_b200 import kernels as kern

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    dev = torch.device("cuda", local)
    torch.cuda.set_device(dev)
    if world > 1:
        from datetime import timedelta
        dist.init_process_group("nccl", timeout=timedelta(seconds=120), device_id=dev)
    stream = torch.cuda.Stream(device=dev)
    gen = torch.Generator(device=dev)
    gen.manual_seed(1234 + rank)

    def q4w(n, k):
        w = torch.randint(0, 256, (n, k // 2), dtype=torch.uint8, device=dev, generator=gen)
        s = (torch.randn((n, k // 32), device=dev, generator=gen) * 0.02).abs().half()
        return w, s

    with torch.cuda.stream(stream):
        layers = [{nm: q4w(*shp) for nm, shp in SHAPES.items()} for _ in range(N_LAYERS)]
        emb = q4w(VOCAB, HID)
        X = torch.randn((M_TOK, HID), device=dev, generator=gen).half()
        QO = torch.empty((M_TOK, 2048), dtype=torch.float16, device=dev)
        KO = torch.empty((M_TOK, 256), dtype=torch.float16, device=dev)
        VO = torch.empty((M_TOK, 256), dtype=torch.float16, device=dev)
        OO = torch.empty((M_TOK, HID), dtype=torch.float16, device=dev)
        GO = torch.empty((M_TOK, 6144), dtype=torch.float16, device=dev)
        UO = torch.empty((M_TOK, 6144), dtype=torch.float16, device=dev)
        DO = torch.empty((M_TOK, HID), dtype=torch.float16, device=dev)
        ws_bytes = max(kern.gemm_q4_workspace_size(M_TOK, n, k) for n, k in SHAPES.values())
        ws = torch.empty(max(1, ws_bytes // 4), dtype=torch.float32, device=dev)

    launches = {"n": 0}

    def gemm(A, name, L, out, alpha=1.0):
        w, s = L[name]
        kern.gemm_q4(A, w, s, C=out, alpha=alpha, workspace=ws)
        n, k = SHAPES[name]
        launches["n"] += 1 + (1 if kern.gemm_q4_workspace_size(M_TOK, n, k) else 0)

    flops_step = 2 * M_TOK * N_LAYERS * sum(n * k for n, k in SHAPES.values())

    def prefill_step(rec=None):
        # layers outer, tokens inner (gemma4_150/prefill_gpu.py:316-395 GEMM sequence)
        for L in layers:
            for name, A, out in (("q", X, QO), ("k", X, KO), ("v", X, VO), ("o", QO, OO),
                                 ("gate", X, GO), ("up", X, UO), ("down", GO, DO)):
                if rec is not None:
                    e0 = torch.cuda.Event(enable_timing=True)
                    e0.record(stream)
                gemm(A, name, L, out)
                if rec is not None:
                    e1 = torch.cuda.Event(enable_timing=True)
                    e1.record(stream)
                    rec.append((name, e0, e1))

    # warm-up outside capture (first calls set kernel attributes, resolve symbols)
    with torch.cuda.stream(stream):
        prefill_step()
    torch.cuda.synchronize()
    launches["n"] = 0
    g_prefill = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g_prefill, stream=stream):
        prefill_step()
    launches_prefill = launches["n"]

    # decode GEMV stack: 35 x 7 GEMVs at M=1 (f32 activations) + fused lm_head argmax
    with torch.cuda.stream(stream):
        xin = {k: torch.randn((1, k), device=dev, generator=gen) for k in (1536, 2048, 6144)}
        yout = {nm: torch.empty((1, n), device=dev) for nm, (n, k) in SHAPES.items()}
        keys = torch.empty(1, dtype=torch.int64, device=dev)
        tok = torch.empty(1, dtype=torch.int32, device=dev)
    gemv_bytes = sum(n * k // 2 + n * (k // 32) * 2 + k * 4 + n * 4 for n, k in SHAPES.values()) * N_LAYERS
    lm_bytes = VOCAB * HID // 2 + VOCAB * (HID // 32) * 2 + HID * 4

    def decode_step():
        for L in layers:
            for nm, (n, k) in SHAPES.items():
                kern.gemv_q4(L[nm][0], L[nm][1], xin[k], y=yout[nm])
        kern.lmhead_argmax(emb[0], emb[1], xin[1536], keys=keys, tokens=tok)

    with torch.cuda.stream(stream):
        decode_step()
    torch.cuda.synchronize()
    g_decode = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g_decode, stream=stream):
        decode_step()
    g_lm = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g_lm, stream=stream):
        kern.lmhead_argmax(emb[0], emb[1], xin[1536], keys=keys, tokens=tok)

    # ---------------- timed region: the headline (prefill stack)
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    clk = Clocks(gpu_id_for(torch, dev))
    with torch.cuda.stream(stream):
        ms = timed_graph(torch, g_prefill, args.steps, args.warmup, stream)
    clocks = clk.stop()
    torch.cuda.synchronize()
    if world > 1:
        t = torch.tensor([ms], device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms = float(t.item())
        dist.barrier()
    value = world * M_TOK / (ms / 1e3)

    # ---------------- end to end through the public API with host buffers
    xh = torch.empty((M_TOK, HID), dtype=torch.float16, pin_memory=True)
    xh.copy_(X.cpu())
    outh = torch.empty((M_TOK, HID), dtype=torch.float16, pin_memory=True)
    with torch.cuda.stream(stream):
        for i in range(args.warmup + args.steps):
            if i == args.warmup:
                torch.cuda.synchronize()
                e0 = torch.cuda.Event(enable_timing=True)
                e0.record(stream)
            X.copy_(xh, non_blocking=True)
            g_prefill.replay()
            outh.copy_(DO, non_blocking=True)
        e1 = torch.cuda.Event(enable_timing=True)
        e1.record(stream)
    e1.synchronize()
    e2e_ms = e0.elapsed_time(e1) / args.steps
    if world > 1:
        t = torch.tensor([e2e_ms], device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        e2e_ms = float(t.item())

    # ---------------- roofline: per-launch durations of the fused GEMM kernel
    rec = []
    with torch.cuda.stream(stream):
        prefill_step(rec)
    torch.cuda.synchronize()
    per = {}
    for name, e0_, e1_ in rec:
        per.setdefault(name, []).append(e0_.elapsed_time(e1_))
    gemm_ms = sum(sum(v) for v in per.values())
    hbm_peak, tc_peak, peak_kind = load_peaks()
    achieved_tflops = flops_step / (gemm_ms / 1e3) / 1e12
    by_shape = {nm: {"avg_us": 1e3 * statistics.mean(v),
                     "tflops": 2 * M_TOK * SHAPES[nm][0] * SHAPES[nm][1] / (statistics.mean(v) / 1e3) / 1e12}
                for nm, v in per.items()}

    # ---------------- decode GEMV stack + lm_head (sub-measurements)
    with torch.cuda.stream(stream):
        dms = timed_graph(torch, g_decode, max(5, args.steps), args.warmup, stream)
        lms = timed_graph(torch, g_lm, max(20, args.steps), args.warmup, stream)
    dec_gbs = (gemv_bytes + lm_bytes) / (dms / 1e3) / 1e9
    lm_gbs = lm_bytes / (lms / 1e3) / 1e9

    if rank == 0:
        cpu = None
        if not args.no_cpu_baseline and world == 1:
            cpu = cpu_sample_prefill()
        line = {
            "metric": "1024-tok prefill tok/s (35-layer int4 projection GEMMs)",
            "value": value, "unit": "tok/s", "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": ms, "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
            "dtype": "f16", "data": "synthetic",
            "config": {"workload": "cfg2_prefill_proj_stack", "tokens": M_TOK, "layers": N_LAYERS,
                       "matrices": {k: list(v) for k, v in SHAPES.items()}, "group": 32,
                       "parallelism": f"replicas x{world}", "l2": "weights 620 MB > 126 MB L2, no flush",
                       "graph": "one CUDA graph per step"},
            "roofline": {"bound": "tensor", "achieved": achieved_tflops, "peak": tc_peak, "unit": "TFLOP/s",
                         "frac": achieved_tflops / tc_peak, "traffic": None, "peak_kind": peak_kind,
                         "kernel": "gemm_tc_kernel<MODE_Q4> (+ split-K finalize)", "by_matrix": by_shape},
            "cpu_baseline": cpu,
            "e2e": {"value": world * M_TOK / (e2e_ms / 1e3), "unit": "tok/s",
                    "h2d_bytes_per_step": M_TOK * HID * 2, "d2h_bytes_per_step": M_TOK * HID * 2},
            "gpu_launches": launches_prefill,
            "clocks": clocks,
            "decode_gemv": {"metric": "decode GEMV-stack tok/s (35x7 GEMVs + lm_head argmax, M=1)",
                            "value": 1e3 / dms, "unit": "tok/s", "ms_per_token": dms,
                            "hbm_gbs": dec_gbs, "frac_of_hbm": dec_gbs / hbm_peak,
                            "bytes_per_token": gemv_bytes + lm_bytes},
            "lmhead": {"metric": "q4 GEMV HBM GB/s (lm_head 262144x1536 + argmax)", "value": lm_gbs,
                       "unit": "GB/s", "us": lms * 1e3, "frac_of_hbm": lm_gbs / hbm_peak, "peak": hbm_peak},
        }
        print(json.dumps(line), flush=True)
    del g_prefill, g_decode, g_lm
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
