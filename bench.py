"""Benchmark of the Newton-Schulz / Muon hot path on B200.

    python bench.py [--gpus N] [--steps K] [--warmup W]
                    [--workload muon8b|muon1b|ns|sweep] [--impl ours|reference]

Workloads:
  muon8b  configs[4], the default at every N: FusedMuon.step() over the 224
          matrices of the 8B-class Llama shape set, grads N(0, 1e-3), lr 0.02,
          momentum 0.95, nesterov, matrices sharded across the N ranks
          (FLOP-balanced) with an NCCL all-gather.  The same workload at
          N = 1, 2, 4, 8 makes one strong-scaling curve.  At N = 1 the line
          also carries, under "ns_4096", the configs[1] headline below.
  muon1b  configs[3]: the same over the 112 matrices of the 1B-class set.
  ns      configs[1] headline: 5-step Newton-Schulz on one (4096, 4096) bf16
          N(0,1) matrix (seed 0); --shape picks another (m, n).  One step =
          one fused_newton_schulz call.  L2 (126 MB) is flushed with a 256 MB
          write before every timed step (outside the step's events).
  sweep   configs[0..2]: every NS shape of the config-1 case and the square
          and wide sweeps, timed with the reference's own protocol
          (benchmarks/bench_ns_step.py:41-81: 200 warm-ups, 50 timed calls,
          median), beside the reference's PyTorch NS on the same GPU, eager
          and under torch.compile.  One JSON line per shape.
  prep    the normalisation / transpose kernels alone, HBM GB/s per shape.
  gemm_compare  each NS GEMM alone against cuBLAS (torch.mm) doing the same
          product, per shape (default (4096,4096), (4096,14336), (2048,8192));
          --sweep-shapes picks others.  One JSON line per shape.

The metric is dense-equivalent Newton-Schulz TFLOP/s (the reference's count,
5·(4m²n + 2m³) per matrix; docs/optimization_report.md:24-29), whole job, max
over ranks; µs per NS / ms per step are reported beside it.

--impl reference times the reference's own algorithm on the host CPU cores
(the oracle's op-for-op restatement of muon_fused/ns_step.py:25-55, since the
reference's path is pure PyTorch and is not installed on the GPU box), on a
bounded sample of the same workload.
"""

from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import time

import torch

ROOT = os.path.dirname(os.path.abspath(__file__))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)

PEAKS_FALLBACK = {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0}
NS_STEPS = 5
SHAPE_NS = (4096, 4096)


def ns_flops(m: int, n: int, steps: int = NS_STEPS) -> float:
    m, n = min(m, n), max(m, n)
    return steps * (4.0 * m * m * n + 2.0 * m ** 3)


def llama_shapes(kind: str):
    """Per-layer Muon matrices of the 1B / 8B Llama-style sets."""
    if kind == "muon1b":
        h, kv, ffn, layers = 2048, 512, 8192, 16
    else:
        h, kv, ffn, layers = 4096, 1024, 14336, 32
    per_layer = [(h, h), (kv, h), (kv, h), (h, h), (ffn, h), (ffn, h), (h, ffn)]  # q k v o gate up down
    return [s for _ in range(layers) for s in per_layer]


def load_peaks():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        with open(p) as f:
            d = json.load(f)
        return d, "measured"
    return PEAKS_FALLBACK, "fallback"


class ClockSampler:
    """nvidia-smi clocks / throttle reasons sampled every 200 ms."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, index: int):
        self.index = index
        self.proc = None

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", "-i", str(self.index), f"--query-gpu={self.FIELDS}",
                 "--format=csv,noheader,nounits", "-lms", "200"],
                stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except OSError:
            self.proc = None
        return self

    def __exit__(self, *exc):
        self.lines = []
        if self.proc is not None:
            self.proc.terminate()
            try:
                out, _ = self.proc.communicate(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()
                out, _ = self.proc.communicate()
            self.lines = [l for l in out.splitlines() if l.strip()]

    def summary(self):
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        sm, smax, reasons = [], 0.0, set()
        for l in getattr(self, "lines", []):
            f = [x.strip() for x in l.split(",")]
            if len(f) < 9:
                continue
            try:
                sm.append(float(f[1]))
                smax = max(smax, float(f[2]))
            except ValueError:
                continue
            for nm, v in zip(names, f[5:9]):
                if v.lower() == "active":
                    reasons.add(nm)
        if not sm:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unsampled"]}
        return {"sm_mhz": statistics.median(sm), "sm_max_mhz": smax, "reasons": sorted(reasons),
                "samples": len(sm)}


# --------------------------------------------------------------------------- helpers
def dist_env():
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    return world, rank, local


def barrier_max(x: float, world: int) -> float:
    if world == 1:
        return x
    import torch.distributed as dist

    t = torch.tensor([x], dtype=torch.float64, device="cuda")
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def flush_l2(buf: torch.Tensor) -> None:
    buf.fill_(1)


def pipelined_ns_e2e(G_host, G_dev, out_host, ws, flush, steps, ns) -> float:
    """ms per step of `steps` NS calls whose inputs come from pinned host memory
    and whose results go back to it, with copies overlapping the computation
    (two device input buffers, two host result buffers, one copy stream per
    direction).  One CUDA-event pair on the compute stream brackets the whole
    run; every copy is ordered inside it."""
    stream = torch.cuda.current_stream()
    up, down = torch.cuda.Stream(), torch.cuda.Stream()
    uploaded = [torch.cuda.Event() for _ in range(2)]
    computed = [torch.cuda.Event() for _ in range(2)]
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    torch.cuda.synchronize()
    start.record(stream)
    up.wait_stream(stream)
    down.wait_stream(stream)
    with torch.cuda.stream(up):
        G_dev[0].copy_(G_host, non_blocking=True)
        uploaded[0].record(up)
    for i in range(steps):
        b = i & 1
        stream.wait_event(uploaded[b])
        flush_l2(flush)
        out = ns(G_dev[b], NS_STEPS, ws)
        computed[b].record(stream)
        if i + 1 < steps:
            with torch.cuda.stream(up):
                if i >= 1:
                    up.wait_event(computed[b ^ 1])  # step i-1 has read that buffer
                G_dev[b ^ 1].copy_(G_host, non_blocking=True)
                uploaded[b ^ 1].record(up)
        down.wait_event(computed[b])
        with torch.cuda.stream(down):
            out_host[b].copy_(out, non_blocking=True)
        out.record_stream(down)
    stream.wait_stream(down)
    end.record(stream)
    torch.cuda.synchronize()
    return start.elapsed_time(end) / steps


def torch_eager_ns(G: torch.Tensor, steps: int) -> torch.Tensor:
    """The reference's pure-PyTorch NS (muon_fused/ns_step.py:25-55) on the GPU:
    the path a reference user gets on B200, where its sm_80 extension is not
    built.  Reported beside our number, not used as an oracle."""
    a, b, c = 3.4445, -4.7750, 2.0315
    X = G.bfloat16()
    if G.size(0) > G.size(1):
        X = X.T
    X = X / (X.norm() + 1e-7)
    for _ in range(steps):
        A = X @ X.T
        B = b * A + c * A @ A
        X = a * X + B @ X
    if G.size(0) > G.size(1):
        X = X.T
    return X


# --------------------------------------------------------------------------- CPU arms
def cpu_ns_sample(budget_s: float, shapes):
    """Time the reference's algorithm (oracle restatement) on the host cores
    over ``shapes`` (one seeded bf16 matrix each, one pass = every matrix
    once); returns (TFLOP/s, seconds per pass, passes, threads)."""
    from oracle import ns_oracle as O

    threads = os.cpu_count() or 1
    torch.set_num_threads(threads)
    gs = [torch.randn(*s, generator=torch.Generator().manual_seed(i)).bfloat16()
          for i, s in enumerate(shapes)]
    O.ns_reference_bf16(gs[0][:512, :512], NS_STEPS)  # warm the BLAS
    times = []
    t_end = time.perf_counter() + budget_s
    while True:
        t0 = time.perf_counter()
        for g in gs:
            O.ns_reference_bf16(g, NS_STEPS)
        times.append(time.perf_counter() - t0)
        if time.perf_counter() > t_end or len(times) >= 5:
            break
    med = statistics.median(times)
    return sum(ns_flops(*sh) for sh in shapes) / med / 1e12, med, len(times), threads


def run_reference_arm(args, world, rank):
    if rank != 0:
        return
    from oracle import ns_oracle as O

    threads = os.cpu_count() or 1
    torch.set_num_threads(threads)
    wl = args.workload
    if wl == "ns":
        m, n = args.shape
        G = torch.randn(m, n, generator=torch.Generator().manual_seed(0)).bfloat16()
        unit_flops, sample = ns_flops(m, n), f"one 5-step NS on ({m},{n}) per step"
        fn = lambda: O.ns_reference_bf16(G, NS_STEPS)
    else:
        # one layer of the set (7 matrices) per step; the metric is a rate, so
        # the per-layer rate stands for the whole step
        shapes = llama_shapes(wl)[:7]
        gs = [torch.randn(s, generator=torch.Generator().manual_seed(1000 + i)) * 1e-3
              for i, s in enumerate(shapes)]
        unit_flops = sum(ns_flops(*s) for s in shapes)
        sample = f"one layer ({len(shapes)} matrices) of the {wl} set per step, NS only"
        fn = lambda: [O.ns_reference_bf16(g, NS_STEPS) for g in gs]
    # warm-up: W passes, but at most ~20 s of CPU work (at least one pass)
    t_w = time.perf_counter()
    for _ in range(args.warmup):
        fn()
        if time.perf_counter() - t_w > 20.0:
            break
    # bounded sample: stop timing after ~60 s of CPU work (at least one step)
    times = []
    t_start = time.perf_counter()
    for _ in range(args.steps):
        t0 = time.perf_counter()
        fn()
        times.append(time.perf_counter() - t0)
        if time.perf_counter() - t_start > 60.0:
            break
    t = statistics.mean(times)
    value = unit_flops / t / 1e12
    line = {
        "impl": "reference", "metric": metric_name(wl, tuple(args.shape)), "value": round(value, 4),
        "unit": "TFLOP/s", "n_gpus": world, "steps": len(times), "warmup": args.warmup,
        "steps_requested": args.steps,
        "ms_per_step": round(t * 1e3, 3), "higher_is_better": True,
        "scaling": "weak" if wl == "ns" else "strong", "vs_baseline": None, "dtype": "bf16",
        "data": "synthetic",
        "config": config_for(wl, world, tuple(args.shape)),
        "cpu_baseline": {"value": round(value, 4), "unit": "TFLOP/s", "cores": threads,
                         "kind": "port", "sample": sample},
        "e2e": {"value": round(value, 4), "unit": "TFLOP/s", "h2d_bytes_per_step": 0,
                "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


def metric_name(wl: str, shape=SHAPE_NS) -> str:
    if wl == "ns":
        return f"5-step Newton-Schulz dense-equivalent TFLOP/s, ({shape[0]},{shape[1]}) bf16"
    return f"FusedMuon.step Newton-Schulz dense-equivalent TFLOP/s, {wl} shape set"


def config_for(wl: str, world: int, shape=SHAPE_NS):
    if wl == "ns":
        return {"workload": f"ns_5step_{shape[0]}x{shape[1]}", "shape": list(shape),
                "ns_steps": NS_STEPS,
                "seed": 0, "l2": "flushed (256 MB write) before every timed step",
                "parallelism": "replicas" if world > 1 else "single"}
    shapes = llama_shapes(wl)
    return {"workload": f"fusedmuon_step_{wl}", "matrices": len(shapes), "ns_steps": NS_STEPS,
            "lr": 0.02, "momentum": 0.95, "nesterov": True,
            "l2": "working set (params+grads+momentum) far above L2",
            "parallelism": f"matrix-sharded dp{world}" if world > 1 else "single",
            "exchange": "n/a"}


# --------------------------------------------------------------------------- our arm
def bench_ns(args, peaks, peak_src):
    from muon_fused import _lib, fused_newton_schulz, workspace_size

    dev = torch.device("cuda")
    m, n = args.shape
    G = torch.randn(m, n, generator=torch.Generator(device=dev).manual_seed(0), device=dev,
                    dtype=torch.bfloat16)
    ws = torch.empty(workspace_size(m, n), dtype=torch.uint8, device=dev)
    flush = torch.empty(256 << 20, dtype=torch.uint8, device=dev)
    stream = torch.cuda.current_stream()
    for _ in range(args.warmup):
        fused_newton_schulz(G, NS_STEPS, ws)
    torch.cuda.synchronize()

    evs = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
           for _ in range(args.steps)]
    n_launch0 = _lib.launch_count()
    with ClockSampler(torch.cuda.current_device()) as clk:
        for s, e in evs:
            flush_l2(flush)
            s.record(stream)
            fused_newton_schulz(G, NS_STEPS, ws)
            e.record(stream)
        torch.cuda.synchronize()
    launches = _lib.launch_count() - n_launch0
    t_ms = [s.elapsed_time(e) for s, e in evs]
    ms = statistics.mean(t_ms)
    flops = ns_flops(m, n)

    # per-kernel timing pass (events around every launch, same stream)
    _lib.stage_timing(True)
    for _ in range(args.steps):
        flush_l2(flush)
        fused_newton_schulz(G, NS_STEPS, ws)
    st = _lib.stage_times()
    _lib.stage_timing(False)
    mo, no = min(m, n), max(m, n)  # the kernels work on the wide orientation
    stage_flops = {"gemm1_syrk": 2.0 * mo * mo * no, "gemm2_poly": 2.0 * mo ** 3,
                   "gemm3_bx": 2.0 * mo * mo * no}
    stages = {}
    for k, (tot, cnt) in st.items():
        if cnt:
            avg = tot / cnt
            d = {"launches": cnt, "avg_us": round(avg * 1e3, 2),
                 "share": round(tot / sum(v[0] for v in st.values()), 4)}
            if k in stage_flops:
                d["dense_eq_tflops"] = round(stage_flops[k] / (avg * 1e-3) / 1e12, 1)
            stages[k] = d
    if st["gemm3_bx"][1]:
        dom = "gemm3_bx"
        kname = "ns_gemm_pair_kernel<kBX> (X' = d*X + Boff*X)"
    else:
        # single matrices up to m = 4096 run all iterations in one persistent
        # kernel: it is the dominant (only) tensor kernel, credited with the
        # MMA work it does (the SYRKs' lower triangles: "useful" FLOPs)
        dom = "fused_ns"
        stage_flops[dom] = NS_STEPS * (mo * (mo + 1) * no + mo * mo * (mo + 1) + 2.0 * mo * mo * no)
        mt = (mo + 127) // 128
        kname = ("ns_fused_kernel<128> (all 5 iterations, 128x128 tiles)" if mt * (mt + 1) // 2 <= 148
                 else "ns_fused_pair_kernel (all 5 iterations, CTA-pair 256x256 tiles)")
    avg_dom = st[dom][0] / st[dom][1]
    achieved = stage_flops[dom] / (avg_dom * 1e-3) / 1e12
    peak = float(peaks["bf16_tflops"])
    roofline = {"bound": "tensor", "kernel": kname,
                "achieved": round(achieved, 1), "peak": peak, "unit": "TFLOP/s",
                "frac": round(achieved / peak, 4), "peak_source": f"{peak_src} bf16_tflops (burst)",
                "traffic": None, "stages": stages}

    extra = {"us_per_ns": round(ms * 1e3, 1),
             "useful_tflops": round(NS_STEPS * (mo * (mo + 1) * no + mo * mo * (mo + 1)
                                                + 2.0 * mo * mo * no) / (ms * 1e-3) / 1e12, 1)}
    if args.quick:
        return {"ms": ms, "flops": flops, "t_ms": t_ms, "roofline": roofline,
                "clocks": clk.summary(), "e2e": None, "launches": launches,
                "extra": extra}

    # end to end: pinned host G -> device -> NS -> pinned host result.
    # Serial: each step's copies and NS back to back on one stream.
    G_host = G.cpu().pin_memory()
    out_host = [torch.empty((m, n), dtype=torch.bfloat16).pin_memory() for _ in range(2)]
    G_dev = [torch.empty_like(G) for _ in range(2)]
    for _ in range(2):
        G_dev[0].copy_(G_host, non_blocking=True)
        out_host[0].copy_(fused_newton_schulz(G_dev[0], NS_STEPS, ws), non_blocking=True)
    torch.cuda.synchronize()
    evs2 = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
            for _ in range(args.steps)]
    for s, e in evs2:
        flush_l2(flush)
        s.record(stream)
        G_dev[0].copy_(G_host, non_blocking=True)
        out_host[0].copy_(fused_newton_schulz(G_dev[0], NS_STEPS, ws), non_blocking=True)
        e.record(stream)
    torch.cuda.synchronize()
    serial_ms = statistics.mean(s.elapsed_time(e) for s, e in evs2)
    # Pipelined (the headline e2e): step i+1's input upload and step i-1's
    # result download run on two copy streams while step i computes;
    # double-buffered device inputs, every byte still crosses the link in the
    # timed region.
    e2e_ms = pipelined_ns_e2e(G_host, G_dev, out_host, ws, flush, args.steps, fused_newton_schulz)

    # the reference's PyTorch path on this GPU (what a reference user runs on B200)
    for _ in range(3):
        torch_eager_ns(G, NS_STEPS)
    torch.cuda.synchronize()
    evs3 = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
            for _ in range(args.steps)]
    for s, e in evs3:
        flush_l2(flush)
        s.record(stream)
        torch_eager_ns(G, NS_STEPS)
        e.record(stream)
    torch.cuda.synchronize()
    eager_ms = statistics.mean(s.elapsed_time(e) for s, e in evs3)

    return {
        "ms": ms, "flops": flops, "t_ms": t_ms, "roofline": roofline, "clocks": clk.summary(),
        "e2e": {"value": round(flops / (e2e_ms * 1e-3) / 1e12, 2), "unit": "TFLOP/s",
                "ms_per_step": round(e2e_ms, 4), "h2d_bytes_per_step": G_host.nbytes,
                "d2h_bytes_per_step": out_host[0].nbytes,
                "mode": "pipelined: uploads/downloads on copy streams overlap the next/previous "
                        "step's NS",
                "serial_ms_per_step": round(serial_ms, 4),
                "serial_value": round(flops / (serial_ms * 1e-3) / 1e12, 2)},
        "launches": launches,
        "extra": dict(extra, torch_eager_gpu_ms=round(eager_ms, 4),
                      speedup_vs_torch_eager_gpu=round(eager_ms / ms, 3)),
    }


def bench_muon(args, world, rank, peaks, peak_src):
    from muon_fused import FusedMuon, _lib
    from muon_fused.sharding import ShardPlan

    dev = torch.device("cuda")
    shapes = llama_shapes(args.workload)
    params = []
    for i, s in enumerate(shapes):
        g = torch.Generator(device=dev).manual_seed(i)
        p = torch.nn.Parameter(torch.randn(s, generator=g, device=dev, dtype=torch.bfloat16) * 0.02)
        p.grad = torch.randn(s, generator=torch.Generator(device=dev).manual_seed(1000 + i),
                             device=dev, dtype=torch.bfloat16) * 1e-3
        params.append(p)
    opt = FusedMuon([{"params": params, "use_muon": True}], lr=0.02, momentum=0.95, nesterov=True,
                    ns_steps=NS_STEPS, collective=args.collective,
                    bucket_bytes=args.bucket_mib << 20)
    for _ in range(args.warmup):
        opt.step()
    torch.cuda.synchronize()
    stream = torch.cuda.current_stream()

    def barrier():
        if world > 1:
            import torch.distributed as dist

            dist.barrier()
        torch.cuda.synchronize()

    barrier()
    s_ev, e_ev = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    n_launch0 = _lib.launch_count()
    with ClockSampler(torch.cuda.current_device()) as clk:
        s_ev.record(stream)
        for _ in range(args.steps):
            opt.step()
        e_ev.record(stream)
        torch.cuda.synchronize()
    launches = _lib.launch_count() - n_launch0
    barrier()
    ms = barrier_max(s_ev.elapsed_time(e_ev) / args.steps, world)
    flops = sum(ns_flops(*s) for s in shapes)

    # GEMM3 roofline: per-launch events over a few steps; FLOPs of the
    # matrices this rank owns (all of them at N = 1).
    owner = ShardPlan.assign([tuple(s) for s in shapes], world) if world > 1 else [0] * len(shapes)
    mine = [s for s, o in zip(shapes, owner) if o == rank]
    prof_steps = 3
    _lib.stage_timing(True)
    for _ in range(prof_steps):
        opt.step()
    st = _lib.stage_times()
    _lib.stage_timing(False)
    barrier()
    g3_flops = prof_steps * NS_STEPS * sum(2.0 * min(s) ** 2 * max(s) for s in mine)
    g3_ms = st["gemm3_bx"][0]
    achieved = g3_flops / (g3_ms * 1e-3) / 1e12 if g3_ms > 0 else 0.0
    peak = float(peaks.get("bf16_tflops_sustained", peaks["bf16_tflops"]))
    total = sum(v[0] for v in st.values())
    roofline = {"bound": "tensor", "kernel": "ns_gemm_pair_kernel<kBX> (X' = d*X + Boff*X), batched",
                "achieved": round(achieved, 1), "peak": peak, "unit": "TFLOP/s",
                "frac": round(achieved / peak, 4),
                "peak_source": f"{peak_src} bf16_tflops_sustained (kernel timed inside a long step)",
                "traffic": None, "rank": rank,
                "stages": {k: {"launches": c, "ms_per_step": round(t / prof_steps, 3),
                               "share_of_ns_time": round(t / total, 4) if total else 0.0}
                           for k, (t, c) in st.items() if c}}

    # End to end: every step uploads the gradients of the matrices this rank
    # owns (the only ones its step reads) from pinned host memory and reads
    # two bytes of the updated parameters back; uploads for step i+1 run on a
    # copy stream, into the second of two device gradient sets, during step i.
    own = [p for p, o in zip(params, owner) if o == rank]
    host = [p.grad.detach().cpu().pin_memory() for p in own]
    sets = [[p.grad for p in own], [torch.empty_like(p.grad) for p in own]]
    probe = torch.empty(1, dtype=torch.bfloat16).pin_memory()
    up = torch.cuda.Stream()
    uploaded = [torch.cuda.Event() for _ in range(2)]
    stepped = [torch.cuda.Event() for _ in range(2)]
    e2e_steps = max(3, min(args.steps, 20))
    barrier()
    s2, e2 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    s2.record(stream)
    up.wait_stream(stream)
    with torch.cuda.stream(up):
        for d, h in zip(sets[0], host):
            d.copy_(h, non_blocking=True)
        uploaded[0].record(up)
    for i in range(e2e_steps):
        b = i & 1
        stream.wait_event(uploaded[b])
        for p, d in zip(own, sets[b]):
            p.grad = d
        opt.step()
        stepped[b].record(stream)
        probe.copy_(params[-1].detach().view(-1)[:1], non_blocking=True)
        if i + 1 < e2e_steps:
            with torch.cuda.stream(up):
                if i >= 1:
                    up.wait_event(stepped[b ^ 1])  # step i-1 has read that set
                for d, h in zip(sets[b ^ 1], host):
                    d.copy_(h, non_blocking=True)
                uploaded[b ^ 1].record(up)
    e2.record(stream)
    torch.cuda.synchronize()
    barrier()
    e2e_ms = barrier_max(s2.elapsed_time(e2) / e2e_steps, world)
    h2d = sum(h.nbytes for h in host)
    e2e = {"value": round(flops / (e2e_ms * 1e-3) / 1e12, 2), "unit": "TFLOP/s",
           "ms_per_step": round(e2e_ms, 4), "h2d_bytes_per_step": h2d,
           "d2h_bytes_per_step": probe.nbytes, "steps": e2e_steps,
           "mode": "pipelined: owned gradients uploaded from pinned host memory on a copy "
                   "stream during the previous step; rank 0's bytes"}
    extra = {"matrices": len(shapes)}
    if world > 1:
        extra["bucket_mib"] = args.bucket_mib
        extra["ranks_agree"], extra["owner_check"] = verify_sharded(opt, params, shapes, owner,
                                                                    world, rank)
    return {"ms": ms, "flops": flops, "roofline": roofline, "clocks": clk.summary(), "e2e": e2e,
            "launches": launches, "extra": extra}


def verify_sharded(opt, params, shapes, owner, world, rank):
    """Correctness of the sharded step, after the timed loops (outside them).

    1. Every rank holds bit-identical parameters: a float64 sum per matrix,
       all-reduced with MAX and MIN, must agree exactly.
    2. One more sharded step is replayed on rank 0 for three large matrices
       owned by different ranks: their owners broadcast the momentum buffer,
       rank 0 recomputes momentum (the reference's torch ops), a single-matrix
       fused_newton_schulz and the update, and compares with the parameters
       the sharded step produced (bit-identical expected: at these sizes the
       batched and single calls run the same unsplit tiles; the line reports
       the relative Frobenius difference of the deltas too)."""
    import torch.distributed as dist

    from muon_fused import fused_newton_schulz

    sums = torch.stack([p.detach().double().sum() for p in params])
    hi, lo = sums.clone(), sums.clone()
    dist.all_reduce(hi, op=dist.ReduceOp.MAX)
    dist.all_reduce(lo, op=dist.ReduceOp.MIN)
    same = bool(torch.equal(hi, lo))

    picked, ranks_seen = [], set()
    for i, s in enumerate(shapes):
        if min(s) >= 3072 and owner[i] not in ranks_seen:
            picked.append(i)
            ranks_seen.add(owner[i])
        if len(picked) == 3:
            break
    before, bufs = {}, {}
    for i in picked:
        p = params[i]
        buf = opt.state[p]["momentum_buffer"] if owner[i] == rank else torch.empty_like(p.grad)
        dist.broadcast(buf, src=owner[i])
        bufs[i] = buf.clone()
        before[i] = p.detach().clone()
    opt.step()
    torch.cuda.synchronize()
    group = opt.param_groups[0]
    lr, wd, mu = group["lr"], group["wd"], group["momentum"]
    worst, exact = 0.0, True
    if rank == 0:
        for i in picked:
            g = params[i].grad
            buf = bufs[i].mul_(mu).add_(g)
            d = g.add(buf, alpha=mu)
            u = fused_newton_schulz(d, NS_STEPS)
            want = before[i].clone()
            want.mul_(1 - lr * wd).add_(u, alpha=-opt.adjust_lr_for_muon(lr, want.shape))
            got = params[i].detach()
            exact = exact and bool(torch.equal(got, want))
            dg = got.double() - before[i].double()
            dw = want.double() - before[i].double()
            worst = max(worst, float((dg - dw).norm() / dw.norm()))
    flag = torch.tensor([1.0 if (same and worst <= 5e-3) else 0.0], device="cuda")
    dist.broadcast(flag, src=0)
    check = {"matrices": [list(shapes[i]) for i in picked], "owners": [owner[i] for i in picked],
             "bit_identical": exact, "max_rel_fro_delta": worst, "checksums_equal": same}
    return bool(flag.item() == 1.0), check


SWEEP_SHAPES = [(896, 1152),  # configs[0]
                (2048, 2048), (3584, 3584), (4096, 4096), (8192, 8192),  # configs[1]
                (2048, 2560), (2560, 6144), (2560, 9728), (3584, 4608), (4096, 14336),
                (4096, 28672)]  # configs[2]


def bench_sweep(args, peaks, peak_src):
    """Every NS shape of configs[0..2] with the reference's protocol
    (benchmarks/bench_ns_step.py:62-81: warm-ups, then CUDA-event-timed calls,
    median): ours, the reference's PyTorch NS eager, and the same under
    torch.compile (the reference's published comparison compiles
    zeropower_via_newtonschulz5, benchmarks/reference_muon.py:13-37).
    Inputs are seeded N(0,1) bf16 resident on the GPU; no L2 flush (the
    reference's harness has none)."""
    from muon_fused import fused_newton_schulz, workspace_size

    dev = torch.device("cuda")
    compiled = torch.compile(torch_eager_ns)
    peak = float(peaks["bf16_tflops"])
    warm, timed = args.sweep_warmup, args.sweep_timed

    def median_ms(fn, G, n_warm):
        for _ in range(n_warm):
            fn(G)
        torch.cuda.synchronize()
        evs = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
               for _ in range(timed)]
        for s_, e_ in evs:
            s_.record()
            fn(G)
            e_.record()
        torch.cuda.synchronize()
        return statistics.median(s_.elapsed_time(e_) for s_, e_ in evs)

    lines = []
    for m, n in (args.sweep_shapes or SWEEP_SHAPES):
        G = torch.randn(m, n, generator=torch.Generator(device=dev).manual_seed(0), device=dev,
                        dtype=torch.bfloat16)
        ws = torch.empty(workspace_size(m, n), dtype=torch.uint8, device=dev)
        with ClockSampler(torch.cuda.current_device()) as clk:
            ours = median_ms(lambda x: fused_newton_schulz(x, NS_STEPS, ws), G, warm)
        eager = median_ms(lambda x: torch_eager_ns(x, NS_STEPS), G, 10)
        try:
            comp = median_ms(lambda x: compiled(x, NS_STEPS), G, 10)
        except Exception as e:  # noqa: BLE001 - reported, not fatal
            comp = None
            comp_err = repr(e)[:200]
        mo, no = min(m, n), max(m, n)
        dense = ns_flops(m, n)
        useful = NS_STEPS * (mo * (mo + 1) * no + mo * mo * (mo + 1) + 2.0 * mo * mo * no)
        line = {"workload": "ns_sweep", "shape": [m, n], "us_per_ns": round(ours * 1e3, 1),
                "dense_eq_tflops": round(dense / (ours * 1e-3) / 1e12, 1),
                "useful_tflops": round(useful / (ours * 1e-3) / 1e12, 1),
                "frac_of_measured_peak": round(dense / (ours * 1e-3) / 1e12 / peak, 4),
                "peak": f"{peak} TFLOP/s ({peak_src} bf16_tflops, burst)",
                "torch_eager_us": round(eager * 1e3, 1),
                "torch_compile_us": None if comp is None else round(comp * 1e3, 1),
                "speedup_vs_eager": round(eager / ours, 3),
                "speedup_vs_compile": None if comp is None else round(comp / ours, 3),
                "protocol": f"{warm} warm-ups, median of {timed} CUDA-event-timed calls",
                "clocks": clk.summary()}
        if comp is None:
            line["torch_compile_error"] = comp_err
        print(json.dumps(line), flush=True)
        lines.append(line)
        del G, ws
        torch.cuda.empty_cache()
    return lines


GEMM_COMPARE_SHAPES = [(4096, 4096), (4096, 14336), (2048, 8192)]


def bench_gemm_compare(args, peaks, peak_src):
    """Each Newton-Schulz GEMM alone against cuBLAS (torch.mm, bf16) doing the
    same product on the same B200, per (m, n): GEMM1 A = X·Xᵀ (m x m, K = n),
    GEMM2 A·A (m x m, K = m), GEMM3 B·X (m x n, K = m).  Ours: one
    newton_schulz_step per call with per-launch CUDA events around each GEMM
    (fm_stage_timing); cuBLAS: CUDA events around torch.mm.  Ours computes only
    the lower triangle of the two SYRKs and fuses its epilogues; the TFLOP/s
    columns use the dense product's 2·M·N·K for both, so they compare times at
    equal work.  Medians over 30 calls after 20 warm-ups, clocks sampled."""
    from muon_fused import _fused_muon_C as _C
    from muon_fused import _lib

    dev = torch.device("cuda")
    peak = float(peaks["bf16_tflops"])
    for m, n in (args.sweep_shapes or GEMM_COMPARE_SHAPES):
        gen = torch.Generator(device=dev).manual_seed(0)
        X = torch.randn(m, n, generator=gen, device=dev, dtype=torch.bfloat16)
        X = (X.float() / X.float().norm()).bfloat16()
        ws = torch.empty(_C.workspace_size(m, max(m, n)), dtype=torch.uint8, device=dev)
        A = X @ X.T
        B = torch.randn(m, m, generator=gen, device=dev, dtype=torch.bfloat16)
        with ClockSampler(torch.cuda.current_device()) as clk:
            for _ in range(20):
                _C.newton_schulz_step(X, ws)
            torch.cuda.synchronize()
            per = {k: [] for k in ("gemm1_syrk", "gemm2_poly", "gemm3_bx")}
            for _ in range(30):
                _lib.stage_timing(True)
                _C.newton_schulz_step(X, ws)
                st = _lib.stage_times()
                for k in per:
                    per[k].append(st[k][0] / max(st[k][1], 1))
            _lib.stage_timing(False)
            ours = {k: statistics.median(v) for k, v in per.items()}

            def mm_ms(a, b):
                for _ in range(20):
                    torch.mm(a, b)
                torch.cuda.synchronize()
                evs = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
                       for _ in range(30)]
                for s_, e_ in evs:
                    s_.record()
                    torch.mm(a, b)
                    e_.record()
                torch.cuda.synchronize()
                return statistics.median(s_.elapsed_time(e_) for s_, e_ in evs)

            cub = {"gemm1_syrk": mm_ms(X, X.T), "gemm2_poly": mm_ms(A, A),
                   "gemm3_bx": mm_ms(B, X)}
        flops = {"gemm1_syrk": 2.0 * m * m * n, "gemm2_poly": 2.0 * m ** 3,
                 "gemm3_bx": 2.0 * m * m * n}
        line = {"workload": "gemm_compare", "shape": [m, n], "clocks": clk.summary(),
                "peak": f"{peak} TFLOP/s ({peak_src} bf16_tflops, burst)"}
        for k in flops:
            line[k] = {"ours_us": round(ours[k] * 1e3, 2), "cublas_us": round(cub[k] * 1e3, 2),
                       "ours_dense_eq_tflops": round(flops[k] / (ours[k] * 1e-3) / 1e12, 1),
                       "cublas_tflops": round(flops[k] / (cub[k] * 1e-3) / 1e12, 1),
                       "ratio_cublas_over_ours": round(cub[k] / ours[k], 3)}
        print(json.dumps(line), flush=True)


PREP_SHAPES = [(1, 4096, 4096), (1, 4096, 14336), (1, 14336, 4096), (8, 14336, 4096),
               (64, 1024, 4096), (1, 896, 1152)]


def bench_prep(args, peaks, peak_src):
    """The normalisation kernels alone (HBM-bound): sum of squares of bf16(G)
    and the scaled copy X0 = bf16(bf16(G) / (||G||_F + 1e-7)), transposed for
    tall inputs.  Algorithmic bytes per matrix: 2mn read for the norm, 2mn
    read + 2mn write for the copy (bf16 input).  Per shape (batch, rows,
    cols): the prep kernels' summed CUDA-event time per call (fm_stage_timing
    stage "prep"), averaged over 20 calls of a 1-step Newton-Schulz after 5
    warm-ups, L2 flushed (256 MB write) before each call."""
    from muon_fused import _fused_muon_C as _C
    from muon_fused import _lib

    dev = torch.device("cuda")
    peak = float(peaks["hbm_gbs"])
    flush = torch.empty(256 << 20, dtype=torch.uint8, device=dev)
    for b, r, c in PREP_SHAPES:
        G = torch.randn(b, r, c, generator=torch.Generator(device=dev).manual_seed(0),
                        device=dev, dtype=torch.bfloat16)
        ws = torch.empty(_C.workspace_size_batched(b, r, c), dtype=torch.uint8, device=dev)
        out = torch.empty_like(G)
        for _ in range(5):
            _C.fused_newton_schulz_batched(G, 1, ws, out=out)
        torch.cuda.synchronize()
        tot = 0.0
        for _ in range(20):
            flush_l2(flush)
            _lib.stage_timing(True)
            _C.fused_newton_schulz_batched(G, 1, ws, out=out)
            tot += _lib.stage_times()["prep"][0]
        _lib.stage_timing(False)
        ms = tot / 20
        nbytes = 6.0 * b * r * c
        gbs = nbytes / (ms * 1e-3) / 1e9
        print(json.dumps({"workload": "prep", "batch": b, "shape": [r, c],
                          "kernels": "sumsq + " + ("scale_transpose" if r > c else "scale"),
                          "us": round(ms * 1e3, 2), "algorithmic_bytes": int(nbytes),
                          "gbs": round(gbs, 1), "frac_of_hbm": round(gbs / peak, 4),
                          "peak": f"{peak} GB/s ({peak_src} hbm_gbs)"}), flush=True)
        del G, ws, out


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=None,
                    help="timed steps (default: 400 for ns, 40 for the optimizer-step workloads, "
                         "so the timed work stays within about a minute)")
    ap.add_argument("--warmup", type=int, default=20)
    ap.add_argument("--workload",
                    choices=["ns", "muon1b", "muon8b", "sweep", "gemm_compare", "prep"],
                    default="muon8b")
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--collective", choices=["nccl", "param_gather"], default="param_gather",
                    help="sharded-step exchange: all-gather of the updates + apply on every "
                         "rank, or owner apply + in-place all-gather of the parameters")
    ap.add_argument("--bucket-mib", type=int, default=256,
                    help="sharded step: per-rank all-gather bucket size in MiB (FusedMuon's "
                         "bucket_bytes)")
    ap.add_argument("--shape", type=int, nargs=2, default=list(SHAPE_NS),
                    help="ns workload matrix shape (default: the headline 4096 4096)")
    ap.add_argument("--quick", action="store_true",
                    help="ns workload: timed loop and per-kernel pass only (for ncu launch lists)")
    ap.add_argument("--no-ns-headline", action="store_true",
                    help="optimizer-step workloads at N = 1: skip the ns_4096 sub-object")
    ap.add_argument("--cpu-budget", type=float, default=12.0,
                    help="seconds of host-CPU baseline sampling per baseline (rank 0, N=1)")
    ap.add_argument("--sweep-warmup", type=int, default=200)
    ap.add_argument("--sweep-timed", type=int, default=50)
    ap.add_argument("--sweep-shapes", type=int, nargs="+", default=None,
                    help="sweep: flat list of m n pairs (default: all BASELINE shapes)")
    args = ap.parse_args()
    if args.sweep_shapes:
        v = args.sweep_shapes
        args.sweep_shapes = [(v[i], v[i + 1]) for i in range(0, len(v) - 1, 2)]
    world, rank, local = dist_env()
    if args.steps is None:
        args.steps = 400 if args.workload == "ns" else 40
    args.warmup = max(args.warmup, 3)
    args.shape = tuple(args.shape)

    if args.impl == "reference":
        run_reference_arm(args, world, rank)
        return

    torch.cuda.set_device(local)
    if world > 1:
        import torch.distributed as dist

        dist.init_process_group("nccl", device_id=torch.device("cuda", local))
    peaks, peak_src = load_peaks()
    if args.workload in ("sweep", "gemm_compare", "prep"):
        if rank == 0:
            {"sweep": bench_sweep, "gemm_compare": bench_gemm_compare,
             "prep": bench_prep}[args.workload](args, peaks, peak_src)
        if world > 1:
            import torch.distributed as dist

            dist.barrier()
            dist.destroy_process_group()
        return
    ns_sub = None
    if args.workload == "ns":
        r = bench_ns(args, peaks, peak_src)
        r["ms"] = barrier_max(r["ms"], world)
        value = world * r["flops"] / (r["ms"] * 1e-3) / 1e12
    else:
        # the (4096, 4096) sub-measurement first, on a fresh process state
        # (its pipelined end-to-end copies are sensitive to what ran before)
        if world == 1 and not args.no_ns_headline:
            ns_sub = ns_headline(args, peaks, peak_src)
            torch.cuda.empty_cache()
        r = bench_muon(args, world, rank, peaks, peak_src)
        value = r["flops"] / (r["ms"] * 1e-3) / 1e12

    if rank == 0:
        line = {
            "metric": metric_name(args.workload, args.shape), "value": round(value, 2),
            "unit": "TFLOP/s",
            "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": round(r["ms"], 4), "higher_is_better": True,
            "scaling": "weak" if args.workload == "ns" else "strong",
            "vs_baseline": None, "dtype": "bf16", "data": "synthetic",
            "config": dict(config_for(args.workload, world, args.shape),
                           **({"exchange": args.collective}
                              if world > 1 and args.workload != "ns" else {})),
            "clocks": r["clocks"], "gpu_launches": r["launches"],
        }
        if r["e2e"] is not None:
            line["e2e"] = r["e2e"]
        if r["roofline"] is not None:
            line["roofline"] = r["roofline"]
        line.update(r["extra"])
        if world == 1 and not args.quick:
            if args.workload == "ns":
                shapes, what = [args.shape], f"5-step NS on ({args.shape[0]},{args.shape[1]})"
            else:
                shapes = llama_shapes(args.workload)[:7]
                what = f"5-step NS of one layer (7 matrices) of the {args.workload} set"
            v, sec, calls, threads = cpu_ns_sample(args.cpu_budget, shapes)
            line["cpu_baseline"] = {"value": round(v, 4), "unit": "TFLOP/s", "cores": threads,
                                    "kind": "port",
                                    "sample": f"{calls} x {what}, median {sec:.2f} s"}
        if ns_sub is not None:
            line["ns_4096"] = ns_sub
        print(json.dumps(line), flush=True)
    if world > 1:
        import torch.distributed as dist

        dist.barrier()
        dist.destroy_process_group()


def ns_headline(args, peaks, peak_src):
    """configs[1] headline inside the N = 1 line: the (4096, 4096) 5-step NS
    with its own device-timed rate, GEMM3 roofline, end-to-end rate from
    pinned host memory, the reference's PyTorch path on this GPU and the host
    CPU baseline of the same matrix."""
    import argparse as _ap

    a = _ap.Namespace(**vars(args))
    a.shape, a.steps, a.warmup, a.quick = SHAPE_NS, 100, 20, False
    r = bench_ns(a, peaks, peak_src)
    v, sec, calls, threads = cpu_ns_sample(args.cpu_budget, [SHAPE_NS])
    out = {"metric": metric_name("ns", SHAPE_NS), "unit": "TFLOP/s",
           "value": round(r["flops"] / (r["ms"] * 1e-3) / 1e12, 2),
           "ms_per_step": round(r["ms"], 4), "steps": a.steps, "warmup": a.warmup,
           "config": config_for("ns", 1, SHAPE_NS), "clocks": r["clocks"], "e2e": r["e2e"],
           "roofline": r["roofline"],
           "cpu_baseline": {"value": round(v, 4), "unit": "TFLOP/s", "cores": threads,
                            "kind": "port",
                            "sample": f"{calls} x 5-step NS on (4096,4096), median {sec:.2f} s"}}
    out.update(r["extra"])
    return out


if __name__ == "__main__":
    main()
