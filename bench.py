"""Benchmark of the B200 int4 quantized-matmul path (prints ONE JSON line on rank 0).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

Headline: "1024-tok prefill tok/s" of the random-init Gemma-4-E2B-shaped int4
decoder (BASELINE config 4 architecture: 35 layers, hidden 1536, FFN 6144,
8q/1kv heads at head_dim 256, vocab 262144, group-32 f16 scales).  One step is
the full layers-outer prefill of a 1024-token prompt -- embed, per layer the
fused int4 tcgen05 projection GEMMs (q|k|v, o, gate|up with GEGLU in its
epilogue, down), q/k norm + RoPE + KV-cache store, the fused causal tcgen05
attention and its split merge, the residual norms -- ending in the final norm
and the lm_head argmax of the first generated token; it is captured as one
CUDA graph.  value = N x 1024 tokens /
max-over-ranks step time (replicas, weak scaling: there is no collective on
this path).  The ~1 GB of weights exceeds the 126 MB L2, so no flush is needed.

Sub-objects: decode tok/s (graph-captured greedy decode step at context
~1024, batch 1) with its bytes/token and HBM GB/s, the lm_head GEMV + argmax
alone (config 3, HBM GB/s), the projection GEMMs inside the prefill (config 2
shapes at M=1024, per matrix TFLOP/s), config 5 (batched decode by batch size
on the GEMV and tcgen05 GEMM paths, and the gate|up crossover), the
per-layer-embedding work of the real checkpoint per decode token and per
prompt ("ple"), and at N>1 the vocabulary-sharded lm_head with its exchange
in peer memory and its NCCL key all-reduce.

--impl reference times the reference's algorithm on the host cores through the
numpy oracle (the reference itself is Python and does not travel to the GPU
box) on a bounded sample, scaled to the same unit.
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
    ap.add_argument("--steps", type=int, default=60)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--kernel", default="",
                    choices=["", "gemm_q4", "gemm_q4_geglu", "gemm_f16", "gemv", "lmhead", "attn", "attn_decode", "gemv_q8",
                             "gemv_bf16", "ple_block", "prefill",
                             "decode", "decode_fused", "decode_batch"],
                    help="run one kernel --iters times on a single shape and exit (for ncu captures)")
    ap.add_argument("--shape", default="6144,1536", help="N,K of the weight for --kernel")
    ap.add_argument("--m", type=int, default=1024, help="rows of the activation for --kernel")
    ap.add_argument("--iters", type=int, default=3)
    ap.add_argument("--batch", type=int, default=256, help="sequences for --kernel decode_batch")
    ap.add_argument("--bits", type=int, default=4, choices=[2, 4],
                    help="code width of the weight for --kernel gemv / lmhead / gemm_q4 / gemm_q4_geglu")
    return ap.parse_args()


def run_model_case(args):
    """Full-model prefill (--m tokens) or decode step, run eagerly (no graph) so a
    profiler sees each launch: one warm-up pass, then --iters profiled passes."""
    import torch

    from slang_b200 import runner, synth
    dev = torch.device("cuda", 0)
    cfg = synth.e2b_config()
    model = synth.random_model(cfg, seed=1234)
    dm = runner.DeviceModel(model, dev, args.m + 8 + 4 * args.iters)
    r = runner.Runner(dm, 1, fused=args.kernel == "decode_fused")
    prompt = synth.prompt_tokens(args.m, cfg["vocab"], seed=99)
    r.prefill(prompt, graph=False)
    torch.cuda.synchronize()
    if args.kernel == "decode_batch":
        # --batch sequences on the tcgen05 GEMM path, each at sequence 0's context (--m tokens)
        rb = runner.Runner(dm, args.batch, proj="gemm")
        for li in range(len(dm.layers)):
            rb.kc[li].copy_(r.kc[li][0:1].expand(args.batch, -1, -1))
            rb.vc[li].copy_(r.vc[li][0:1].expand(args.batch, -1, -1))
        rb.pos.fill_(int(r.pos[0].item()))
        rb.cur.copy_(r.cur[0:1].expand(args.batch))
        torch.cuda.synchronize()
        for _ in range(1 + args.iters):
            with torch.cuda.stream(rb.stream):
                rb._decode_ops()
        torch.cuda.synchronize()
        print(f"ran decode_batch x{1 + args.iters} (batch {args.batch}, context {args.m}) eagerly")
        return
    for _ in range(args.iters):
        if args.kernel == "prefill":
            r.prefill(prompt, graph=False)
        else:
            with torch.cuda.stream(r.stream):
                (r._fused_ops if r.fused else r._decode_ops)()
    torch.cuda.synchronize()
    print(f"ran {args.kernel} x{args.iters} (prompt {args.m}) eagerly")


def run_kernel_case(args):
    """One kernel on one shape, --iters launches after one warm-up (ncu target)."""
    import torch

    if args.kernel in ("prefill", "decode", "decode_fused", "decode_batch"):
        return run_model_case(args)
    from slang_b200 import kernels as kern
    dev = torch.device("cuda", 0)
    n, k = (int(v) for v in args.shape.split(","))
    m = args.m
    g = torch.Generator(device=dev)
    g.manual_seed(0)
    bits = args.bits
    w = torch.randint(0, 256, (n, k * bits // 8), dtype=torch.uint8, device=dev, generator=g)
    s = (torch.randn((n, k // 32), device=dev, generator=g) * 0.02).abs().half()
    if args.kernel == "attn_decode":
        # batched decode attention: --batch sequences at context --m, 8 query heads, head_dim from --shape's K
        hd, B, ctx = k, args.batch, args.m
        max_seq = ctx + 61
        q = torch.randn((B, 8, hd), device=dev, generator=g) * 0.2
        kc = torch.randn((B, max_seq, hd), device=dev, generator=g)
        vc = torch.randn((B, max_seq, hd), device=dev, generator=g)
        pos = torch.full((B,), ctx - 1, dtype=torch.int32, device=dev)
        out16 = torch.empty((B, 8, hd), dtype=torch.float16, device=dev)

        def op():
            kern.attn_decode(q, kc, vc, pos, out=out16, f16=True)
    elif args.kernel == "attn":
        # fused causal prefill attention: --m tokens, 8 query heads, head_dim from --shape's K
        hd = k
        q = torch.randn((m, 8, hd), device=dev, generator=g).half()
        kk = torch.randn((m, hd), device=dev, generator=g).half()
        vv = torch.randn((m, hd), device=dev, generator=g).half()
        out = torch.empty_like(q)

        def op():
            kern.attn_prefill(q, kk, vv, out)
    elif args.kernel in ("gemv_q8", "gemv_bf16", "ple_block"):
        # PLE kernels: weights rotated over copies totalling > 256 MB so every launch reads HBM
        esz = 2 if args.kernel == "gemv_bf16" else 1
        per = (2 * 256 * 1536 if args.kernel == "ple_block" else n * k * esz)
        copies = max(2, -(-(256 << 20) // per))
        x = torch.randn((m, 1536 if args.kernel == "ple_block" else k), device=dev, generator=g)
        if args.kernel == "ple_block":
            ple_in = torch.randn((m, 256), device=dev, generator=g)
            layers = [{"gate": (torch.randint(0, 256, (256, 1536), dtype=torch.uint8, device=dev, generator=g),
                                torch.full((256,), 1e-4, device=dev)),
                       "proj": (torch.randint(0, 256, (1536, 256), dtype=torch.uint8, device=dev, generator=g),
                                torch.full((1536,), 1e-3, device=dev)),
                       "post_norm": torch.ones(1536, device=dev), "scalar": 1.0} for _ in range(copies)]
            if m > kern.PLE_GEMV_ROWS:  # the GEMM route's f16 weights are made once per layer, not timed
                for layer in layers:
                    kern.ple_block(x.clone(), ple_in, layer, 1e-6)
        else:
            ws = [torch.randint(0, 256, (n, k * esz), dtype=torch.uint8, device=dev, generator=g)
                  for _ in range(copies)]
            if esz == 2:
                ws = [t.view(torch.int16) for t in ws]
            scale = torch.full((n,), 1e-3, device=dev)
            y = torch.empty((m, n), device=dev)
        turn = [0]

        def op():
            i = turn[0] % copies
            turn[0] += 1
            if args.kernel == "ple_block":
                kern.ple_block(x, ple_in, layers[i], 1e-6)
            elif esz == 2:
                kern.gemv_bf16(ws[i], x, alpha=0.03, out=y)
            else:
                kern.gemv_q8(ws[i], scale, x, out=y)
    elif args.kernel in ("gemm_q4", "gemm_q4_geglu", "gemm_f16"):
        a = torch.randn((m, k), device=dev, generator=g).half()
        geglu = args.kernel == "gemm_q4_geglu"
        c = torch.empty((m, n // 2 if geglu else n), dtype=torch.float16, device=dev)
        wf = kern.dequant_f16(w, s, k, n) if args.kernel == "gemm_f16" else None

        def op():
            if wf is None:
                kern.gemm_q4(a, w, s, C=c, geglu=geglu, bits=bits)
            else:
                kern.gemm(a, wf, c, m, n, k)
    else:
        x = torch.randn((m, k), device=dev, generator=g)
        y = torch.empty((m, n), device=dev)

        def op():
            if args.kernel == "gemv":
                kern.gemv_q4(w, s, x, y=y, bits=bits)
            else:
                kern.lmhead_argmax(w, s, x, bits=bits)
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
    if args.kernel == "attn_decode":
        rate = f"{2 * args.batch * m * k * 4 / us / 1e3:.1f} GB/s of K/V"
    elif args.kernel == "attn":
        rate = f"{2 * 2 * 8 * m * m / 2 * k / us / 1e6:.1f} TFLOP/s (causal: half of S x S)"
    elif args.kernel in ("gemv_q8", "gemv_bf16"):
        rate = f"{(n * k * esz + n * 4 * (esz == 1) + m * k * 4 + m * n * 4) / us / 1e3:.1f} GB/s (weights rotated over copies > L2)"
    elif args.kernel == "ple_block":
        rate = f"{(2 * 256 * 1536 + 1792 * 4 + m * 1536 * 16) / us / 1e3:.1f} GB/s over gate + proj + tail (3 launches)"
    elif args.kernel in ("gemm_q4", "gemm_q4_geglu", "gemm_f16"):
        rate = f"{2 * m * n * k / us / 1e6:.1f} TFLOP/s"
    else:
        rate = f"{(n * k * bits // 8 + n * (k // 32) * 2 + m * k * 4 + m * n * 4) / us / 1e3:.1f} GB/s"
    print(f"ran {args.kernel} ({bits}-bit) m={m} n={n} k={k} x{args.iters + 1}: {us:.2f} us/launch, {rate} "
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


def ple_measure(torch, kern, dev, stream, warmup, hbm_peak, prompt):
    """The per-layer-embedding (PLE) work of the Gemma-4-E2B checkpoint (not in
    the benchmark model): per decode token the bf16 model projection
    [8960 x 1536] + table gather + combine, then 35 blocks of two 8-bit GEMVs
    and the norm-add tail; per prompt the same as GEMMs.  Random E2B-shaped
    weights (table cut to 4096 rows), three copies rotated so a token reads HBM."""
    H, nL, d, V = 1536, 35, 256, 4096
    g = torch.Generator(device=dev)
    g.manual_seed(7)
    u8 = lambda *s: torch.randint(0, 256, s, dtype=torch.uint8, device=dev, generator=g)  # noqa: E731

    def weights():
        proj = (torch.randn(nL * d, H, device=dev, generator=g) * 0.02).to(torch.bfloat16)
        return {"table": u8(V, nL * d // 2), "table_scale": torch.rand(V, nL, device=dev, generator=g) * 0.01,
                "proj": proj, "proj16": proj.to(torch.float16),
                "norm": torch.ones(d, device=dev),
                "layers": [{"gate": (u8(d, H), torch.full((d,), 2e-4, device=dev)),
                            "proj": (u8(H, d), torch.full((H,), 1e-3, device=dev)),
                            "post_norm": torch.ones(H, device=dev), "scalar": 1.0} for _ in range(nL)]}

    sets = [weights() for _ in range(3)]
    out = {}
    for m in (1, prompt):
        x = torch.randn(m, H, device=dev, generator=g)
        ids = torch.randint(0, V, (m,), dtype=torch.int32, device=dev, generator=g)
        ple_in = torch.empty(m, nL, d, device=dev)

        def token(P):
            kern.ple_input(x, ids, P["table"], P["table_scale"], P["proj"], P["norm"], nL, d, 1e-6, 16.0,
                           out=ple_in, w_proj16=P["proj16"])
            for li, L in enumerate(P["layers"]):
                kern.ple_block(x, ple_in[:, li], L, 1e-6)

        with torch.cuda.stream(stream):
            for P in sets:  # outside capture: kernel attributes, f16 weight copies of the GEMM route
                token(P)
            torch.cuda.synchronize()
            graph = torch.cuda.CUDAGraph()
            with torch.cuda.graph(graph, stream=stream):
                for P in sets:
                    token(P)
            us = timed_graph(torch, graph, 5, warmup, stream) / len(sets) * 1e3
        del graph
        w_bytes = nL * d * H * 2 + nL * 2 * d * H + nL * (d + H) * 4 + m * (nL * d // 2 + nL * 4)
        if m == 1:
            out["decode"] = {"us_per_token": us, "weight_bytes_per_token": w_bytes,
                             "hbm_gbs": w_bytes / us / 1e3, "frac_of_hbm": w_bytes / us / 1e3 / hbm_peak,
                             "gpu_launches_per_token": 2 + (2 if kern.PLE_FUSED_TAIL_ROWS >= 1 else 3) * nL}
        else:
            out["prefill"] = {"tokens": m, "us_per_prompt": us, "gpu_launches_per_prompt": 3 + 5 * nL,
                              "tflops": (2 * m * H * nL * d + nL * 4 * m * H * d) / us / 1e6}
    return {"metric": "PLE work per decode token / per prompt (35 layers, d 256; not in the benchmark model)", **out}


def config5_sweep(torch, kern, runner, dm, r0, warmup, steps, max_over_ranks, world):
    """Config 5 on one replica: decode tok/s at batch B, every sequence at the
    context of r0's sequence 0 (copied into all B), on the GEMV path (B <= 8)
    and on the tcgen05 GEMM path; and per-call times of the gate|up projection
    [12288 x 1536] both ways, rotating over the 35 layers' weights (371 MB,
    past L2) as a decode step does, to locate the GEMV -> GEMM crossover."""
    out = {"decode": [], "gateup": []}
    S0 = int(r0.pos[0].item())
    for B, proj in ((1, "gemv"), (1, "gemm"), (2, "gemv"), (2, "gemm"), (4, "gemv"), (4, "gemm"), (8, "gemv"),
                    (8, "gemm"), (32, "gemm"), (128, "gemm"), (256, "gemm")):
        rb = runner.Runner(dm, B, proj=proj)
        with torch.cuda.stream(rb.stream):
            for li in range(len(dm.layers)):
                rb.kc[li].copy_(r0.kc[li][0:1].expand(B, -1, -1))
                rb.vc[li].copy_(r0.vc[li][0:1].expand(B, -1, -1))
            rb.pos.fill_(S0)
            rb.cur.copy_(r0.cur[0:1].expand(B))
        torch.cuda.synchronize()
        rb.capture()
        with torch.cuda.stream(rb.stream):
            ms = timed_graph(torch, rb.graph, steps, warmup, rb.stream)
        ms = max_over_ranks(ms)
        out["decode"].append({"batch": B, "proj": proj, "ms_per_step": ms, "tok_s": world * B * 1e3 / ms,
                              "context": S0, "gpu_launches_per_step": rb.kernel_launches_per_step()})
        del rb
        torch.cuda.empty_cache()
    # gate|up projection alone: GEMV (f32 x, M <= 8) and GEMM (f16 A) per call
    dev = dm.device
    nL = len(dm.layers)
    N, K = dm.layers[0]["gu"][0].shape[0], dm.layers[0]["gu"][0].shape[1] * 2
    stream = torch.cuda.Stream(device=dev)
    gemv_us = {}
    for M in (1, 2, 4, 8, 16, 32, 64, 128, 256):
        row = {"M": M}
        for path in ("gemv", "gemm"):
            if path == "gemv" and M > 8:
                continue
            x = torch.randn((M, K), device=dev, dtype=torch.float32 if path == "gemv" else torch.float16)
            y = torch.empty((M, N), device=dev, dtype=torch.float32 if path == "gemv" else torch.float16)
            ws = kern._workspace(dev, kern.gemm_q4_workspace_size(M, N, K)) if path == "gemm" else None

            def call(li):
                w, sc = dm.layers[li]["gu"]
                if path == "gemv":
                    kern.gemv_q4(w, sc, x, y=y)
                else:
                    kern.gemm_q4(x, w, sc, C=y, workspace=ws)
            with torch.cuda.stream(stream):
                for li in range(nL):
                    call(li)
                torch.cuda.synchronize()
                g = torch.cuda.CUDAGraph()
                with torch.cuda.graph(g, stream=stream):
                    for li in range(nL):
                        call(li)
                us = timed_graph(torch, g, 3, 1, stream) * 1e3 / nL
            row[path + "_us"] = us
            row[path + "_weight_gbs"] = (N * K // 2 + N * (K // 32) * 2) / (us * 1e3)
        if M <= 8:
            gemv_us[M] = row["gemv_us"]
        else:
            row["gemv_equivalent_us"] = (M + 7) // 8 * gemv_us[8]  # M/8 launches of the 8-row GEMV
        out["gateup"].append(row)
    cross = [r["M"] for r in out["gateup"] if r["gemm_us"] < r.get("gemv_us", r.get("gemv_equivalent_us", 1e30))]
    out["gateup_crossover_M"] = min(cross) if cross else None
    best = {}
    for d in out["decode"]:
        if d["batch"] not in best or d["tok_s"] > best[d["batch"]]["tok_s"]:
            best[d["batch"]] = d
    both = sorted(b for b in best if {x["proj"] for x in out["decode"] if x["batch"] == b} == {"gemv", "gemm"})
    gemm_wins = [b for b in both if best[b]["proj"] == "gemm"]
    out["decode_crossover_batch"] = min(gemm_wins) if gemm_wins else None
    return out


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
    line = {"metric": "1024-tok prefill tok/s", "value": v, "unit": "tok/s",
            "impl": "reference", "n_gpus": args.gpus, "steps": len(vals), "warmup": args.warmup,
            "ms_per_step": 1e3 * M_TOK / v, "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "f16", "data": "synthetic",
            "config": {"workload": "cfg4_full_model_prefill_1024", "prompt_tokens": M_TOK,
                       "parallelism": "cpu", "sample": "see cpu_baseline.sample"},
            "cpu_baseline": cb,
            "e2e": {"value": v, "unit": "tok/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
            "wall_s": wall}
    print(json.dumps(line), flush=True)


# ------------------------------------------------------------------ GPU arm
PROMPT = 1024
DECODE_STEPS = 64
# DRAM bytes (dram__bytes_read.sum + dram__bytes_write.sum) of one launch of the
# fused int4 GEMM at M = 1024, keyed by the weight's (N, K), from one ncu capture
# per shape: `ncu --metrics gpu__time_duration.sum,dram__bytes_read.sum,
# dram__bytes_write.sum --clock-control none -k regex:gemm_q4 -s 1 -c 2 python
# bench.py --kernel gemm_q4 --shape N,K --m 1024 --iters 3` (gemm_q4_geglu for
# the gate|up weight).  Each equals the operands read once (A, packed W,
# scales); C stays in L2 within the launch.
GEMM_DRAM_BYTES = {(2560, 1536): 5_419_264, (1536, 2048): 6_022_144, (12288, 1536): 13_820_928,
                   (1536, 6144): 17_949_696}


def main():
    args = parse()
    if args.kernel:
        return run_kernel_case(args)
    if args.impl == "reference":
        return run_reference(args)

    import torch
    import torch.distributed as dist

    from slang_b200 import kernels as kern
    from slang_b200 import lmhead, runner, synth

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    dev = torch.device("cuda", local)
    torch.cuda.set_device(dev)
    if world > 1:
        from datetime import timedelta
        dist.init_process_group("nccl", timeout=timedelta(seconds=120), device_id=dev)

    def max_over_ranks(x):
        if world == 1:
            return x
        t = torch.tensor([x], device=dev, dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    cfg = synth.e2b_config()
    model = synth.random_model(cfg, seed=1234 + rank)
    dm = runner.DeviceModel(model, dev, PROMPT + args.warmup + args.steps + DECODE_STEPS + 8)
    del model
    r = runner.Runner(dm, 1)
    prompt = synth.prompt_tokens(PROMPT, cfg["vocab"], seed=99 + rank)
    r.prefill(prompt)                  # eager run + capture
    g_prefill = r.prefill_graph(PROMPT)
    stream = r.stream

    # ---------------- timed region: the headline (prefill graph replays)
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    clk = Clocks(gpu_id_for(torch, dev))
    with torch.cuda.stream(stream):
        ms = timed_graph(torch, g_prefill, args.steps, args.warmup, stream)
    clocks = clk.stop()
    ms = max_over_ranks(ms)
    value = world * PROMPT / (ms / 1e3)

    # ---------------- end to end through the public API (pinned H2D prompt, D2H first token)
    for _ in range(args.warmup):
        r.prefill(prompt)
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for _ in range(args.steps):
        r.prefill(prompt)
    e1.record(stream)
    e1.synchronize()
    e2e_ms = max_over_ranks(e0.elapsed_time(e1) / args.steps)

    # ---------------- roofline of the dominant kernel (fused int4 GEMM) inside the prefill
    rec = r.prefill_timed_gemms(prompt)
    hbm_peak, tc_peak, peak_kind = load_peaks()
    gemm_ms = sum(x[4] for x in rec)
    gemm_flops = sum(2 * m * n * k for _, m, n, k, _ in rec)
    achieved = gemm_flops / (gemm_ms / 1e3) / 1e12
    by = {}
    for name, m, n, k, t in rec:
        b = by.setdefault(name, {"shape": [m, n, k], "ms": 0.0, "count": 0})
        b["ms"] += t
        b["count"] += 1
    for b in by.values():
        m, n, k = b["shape"]
        b["avg_us"] = 1e3 * b["ms"] / b["count"]
        b["tflops"] = 2 * m * n * k / (b["avg_us"] / 1e6) / 1e12
        b["algorithmic_read_bytes"] = m * k * 2 + n * k // 2 + n * (k // 32) * 2
        b["dram_bytes_per_launch"] = GEMM_DRAM_BYTES.get((n, k)) if m == PROMPT else None
        del b["ms"]
    traffic = (sum(b["dram_bytes_per_launch"] * b["count"] for b in by.values())
               if all(b["dram_bytes_per_launch"] for b in by.values()) else None)

    # ---------------- decode (graph-captured step, batch 1, context from PROMPT)
    # the persistent one-kernel step (the product path) and the per-op graph
    rf = runner.Runner(dm, 1, fused=True)
    rf.prefill(prompt)
    rf.capture()
    with torch.cuda.stream(rf.stream):
        dms = timed_graph(torch, rf.graph, DECODE_STEPS, args.warmup, rf.stream)
    dms = max_over_ranks(dms)
    r.capture()
    with torch.cuda.stream(stream):
        dms_ops = timed_graph(torch, r.graph, DECODE_STEPS, args.warmup, stream)
    dms_ops = max_over_ranks(dms_ops)
    ctx = PROMPT + args.warmup + DECODE_STEPS // 2
    w_bytes = sum(t.numel() * t.element_size() for L in dm.layers for key in ("qkv", "o", "gu", "down") for t in L[key])
    lm_bytes = dm.embed_q.numel() + dm.embed_s.numel() * 2
    kv_bytes = len(dm.layers) * 2 * ctx * r.hd * 4
    dec_bytes = w_bytes + lm_bytes + kv_bytes

    # ---------------- lm_head GEMV + argmax alone (config 3)
    g_lm = torch.cuda.CUDAGraph()
    with torch.cuda.stream(stream):
        kern.lmhead_argmax(dm.embed_q, dm.embed_s, r.h, keys=r.keys, tokens=r.tok)
        torch.cuda.synchronize()
        with torch.cuda.graph(g_lm, stream=stream):
            for _ in range(10):
                kern.lmhead_argmax(dm.embed_q, dm.embed_s, r.h, keys=r.keys, tokens=r.tok)
        lms = timed_graph(torch, g_lm, 5, 2, stream) / 10
    lm_alg = VOCAB * HID // 2 + VOCAB * (HID // 32) * 2 + HID * 4

    # ---------------- per-layer embeddings of the real checkpoint (kernels of csrc/ple.cu)
    ple = ple_measure(torch, kern, dev, stream, args.warmup, hbm_peak, PROMPT)

    # ---------------- config 5: batched decode sweep and the GEMV -> tcgen05 GEMM crossover
    c5 = config5_sweep(torch, kern, runner, dm, r, args.warmup, 10, max_over_ranks, world)

    # ---------------- vocabulary-sharded lm_head over NCCL (N > 1)
    sharded = None
    if world > 1:
        sh = lmhead.ShardedLMHead(dm.embed_q, dm.embed_s, rank, world)
        keys = torch.zeros(1, dtype=torch.int64, device=dev)
        toks = torch.zeros(1, dtype=torch.int32, device=dev)
        with torch.cuda.stream(stream):
            for _ in range(args.warmup):
                sh(r.h, keys, toks)
            torch.cuda.synchronize()
            s0, s1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            s0.record(stream)
            for _ in range(args.steps):
                sh(r.h, keys, toks)
            s1.record(stream)
        s1.synchronize()
        sms_ = max_over_ranks(s0.elapsed_time(s1) / args.steps)
        sharded = {"metric": "vocab-sharded lm_head + argmax (NCCL MAX of keys), tok/s", "value": 1e3 / sms_,
                   "unit": "tok/s", "us": sms_ * 1e3, "shards": world,
                   "hbm_gbs_aggregate": lm_alg / (sms_ / 1e3) / 1e9, "scaling": "strong"}
        # the same shards with the exchange in peer memory (atomic MAX over NVLink in the GEMV, one
        # counting kernel per rank), captured as a graph of 10 steps
        try:
            ph = lmhead.PeerLMHead(dm.embed_q, dm.embed_s, rank, world)
        except Exception as exc:  # noqa: BLE001 - CUDA IPC unavailable: report, keep the NCCL numbers
            sharded["peer"] = {"unavailable": str(exc)[:200]}
            ph = None
        if ph is not None:
            with torch.cuda.stream(stream):
                for _ in range(args.warmup):
                    ph(r.h, keys, toks)
                torch.cuda.synchronize()
                gp = torch.cuda.CUDAGraph()
                with torch.cuda.graph(gp, stream=stream):
                    for _ in range(10):
                        ph(r.h, keys, toks)
                dist.barrier()
                pms = timed_graph(torch, gp, max(1, args.steps // 10), 1, stream) / 10
            pms = max_over_ranks(pms)
            # (each rank holds its own random model here; the sharded tokens are checked in the tests)
            sharded["peer"] = {"metric": "vocab-sharded lm_head + argmax, exchange in peer memory over NVLink, tok/s",
                               "value": 1e3 / pms, "us": pms * 1e3, "hbm_gbs_aggregate": lm_alg / (pms / 1e3) / 1e9,
                               "gpu_launches_per_token": 2}
            del gp
            ph.close()

    if rank == 0:
        cpu = cpu_sample_prefill() if (not args.no_cpu_baseline and world == 1) else None
        line = {
            "metric": "1024-tok prefill tok/s", "value": value, "unit": "tok/s", "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms, "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": "f16", "data": "synthetic",
            "config": {"workload": "cfg4_full_model_prefill_1024", "prompt_tokens": PROMPT,
                       "model": "random-init Gemma-4-E2B-shaped int4 decoder (35L, H1536, F6144, 8q/1kv hd256, "
                                "V262144, group-32 f16 scales)",
                       "parallelism": f"replicas x{world}", "l2": "weights ~1 GB > 126 MB L2, no flush",
                       "graph": "one CUDA graph per prefill"},
            "roofline": {"bound": "tensor", "achieved": achieved, "peak": tc_peak, "unit": "TFLOP/s",
                         "frac": achieved / tc_peak, "traffic": traffic, "peak_kind": peak_kind,
                         "traffic_unit": "DRAM bytes per prefill step over all GEMM launches (ncu, per shape)",
                         "kernel": "gemm_q4_pair_kernel (fused int4 dequant + tcgen05 CTA pair; split-K "
                                   "reduced in-cluster)",
                         "flops_per_step": gemm_flops, "gemm_ms_per_step": gemm_ms,
                         "gemm_share_of_step": gemm_ms / ms, "by_matrix": by},
            "cpu_baseline": cpu,
            "e2e": {"value": world * PROMPT / (e2e_ms / 1e3), "unit": "tok/s",
                    "h2d_bytes_per_step": PROMPT * 4, "d2h_bytes_per_step": 4},
            "gpu_launches": r.prefill_launches(PROMPT),
            "clocks": clocks,
            "decode": {"metric": "decode tok/s (batch 1, greedy, context ~%d)" % ctx, "value": world * 1e3 / dms,
                       "unit": "tok/s", "ms_per_token": dms, "bytes_per_token": dec_bytes,
                       "hbm_gbs": dec_bytes / (dms / 1e3) / 1e9, "frac_of_hbm": dec_bytes / (dms / 1e3) / 1e9 / hbm_peak,
                       "kernel": "decode_step_kernel (persistent, one cooperative launch per token)",
                       "gpu_launches_per_token": rf.kernel_launches_per_step(),
                       "per_op_graph": {"value": world * 1e3 / dms_ops, "ms_per_token": dms_ops,
                                        "gpu_launches_per_token": r.kernel_launches_per_step()}},
            "config5": {"metric": "batched decode tok/s (all replicas) by batch and projection path; gate|up "
                                  "per-call time GEMV vs tcgen05 GEMM", "scaling": "weak (replicas)", **c5},
            "lmhead": {"metric": "q4 GEMV HBM GB/s (lm_head 262144x1536 + argmax)", "value": lm_alg / (lms / 1e3) / 1e9,
                       "unit": "GB/s", "us": lms * 1e3, "frac_of_hbm": lm_alg / (lms / 1e3) / 1e9 / hbm_peak,
                       "peak": hbm_peak},
            "lmhead_sharded": sharded,
            "ple": ple,
        }
        print(json.dumps(line), flush=True)
    del g_prefill, g_lm
    r.graph = None
    rf.graph = None
    r._pgraphs.clear()
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
