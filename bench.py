#!/usr/bin/env python
"""Benchmark of the entropy-gated mixed-precision step on B200.

Workload ("gated_step_llama3_8b", BASELINE configs 1-3 at Llama-3-8B shapes): per GPU
M = 4096 token rows.  One step =
  1. fused softmax + entropy + dual-threshold route + bucket compaction over the gating
     logits [M, 4096] fp16 (tau = 0.41 / 1.68),
  2. for each Llama-3-8B projection -- attention (K=4096, N=4096), MLP up/gate
     (K=4096, N=14336), MLP down (K=14336, N=4096) -- per-row quantisation of that
     projection's activations [M, K] into the INT8 / FP8 / FP16 buckets and one
     persistent tcgen05 GEMM over all three buckets, scattered back in row order.
Inputs are seeded synthetic data: logits rows ~ N(0, s^2) with s log-uniform in
[7, 9.5] (routes about 20 / 60 / 20 % of the rows to INT8 / FP8 / FP16, the config-3
mix), activations ~ N(0, 1) with 1 % of the entries x20, weights ~ N(0, 0.02) quantised
per output channel.  The metric is TFLOPS of the whole step (sum of 2*M*N*K over the
three projections divided by the step's device time).

  python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

N > 1 is launched by torchrun (one process per GPU, NCCL); rows partition across GPUs
(every rank runs its own M rows, weak scaling) and no collective runs inside a step.
``--impl reference`` times the reference's path restated with its own PyTorch ops on
the host CPU (oracle/ee_cpu_reference.py) on a bounded sample of rows.
"""
from __future__ import annotations

import argparse
import json
import math
import os
import statistics
import subprocess
import sys
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)

METRIC = "gated GEMM TFLOPS & softmax+entropy GB/s (Llama-3-8B shapes), tokens/s 1–8 B200"
UNIT = "TFLOPS"
TAU = (0.41, 1.68)
N_LOGIT = 4096
PROJECTIONS = [("attn_proj", 4096, 4096), ("mlp_up_gate", 4096, 14336), ("mlp_down", 14336, 4096)]  # (name, K, N)
SCALE_RANGE = (7.0, 9.5)
FLUSH_BYTES = 256 << 20  # > 126 MB L2


class L2Flush:
    """Between timed steps: write a buffer larger than L2, then read a second one, so
    the lines left behind are clean and no write-back of the flush lands in the next
    step's timed region."""

    def __init__(self, torch, dev):
        self.w = torch.empty(FLUSH_BYTES, dtype=torch.uint8, device=dev)
        self.r = torch.ones(FLUSH_BYTES // 4, dtype=torch.float32, device=dev)

    def __call__(self):
        self.w.zero_()
        self.r.sum()


DTYPE = "s8/e4m3/f16 operands, s32/f32 accumulate"


def parse_args(argv=None):
    ap = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=400)
    ap.add_argument("--warmup", type=int, default=10)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--rows", type=int, default=4096, help="token rows per GPU")
    ap.add_argument("--e2e-steps", type=int, default=20)
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--cpu-seconds", type=float, default=12.0, help="CPU-baseline sample budget")
    return ap.parse_args(argv)


def step_flops(M: int) -> float:
    return float(sum(2 * M * K * N for _, K, N in PROJECTIONS))


def config_dict(M: int, world: int, mix=None) -> dict:
    cfg = {
        "workload": "gated_step_llama3_8b",
        "rows_per_gpu": M,
        "global_rows": M * world,
        "logits": [M, N_LOGIT],
        "projections": {name: {"K": K, "N": N} for name, K, N in PROJECTIONS},
        "tau": list(TAU),
        "logit_scale_loguniform": list(SCALE_RANGE),
        "activations": "N(0,1), 1% x20 outliers",
        "weights": "N(0,0.02), INT8 per-channel",
        "parallelism": f"rows{world}",
        "l2": "flushed between timed steps (256 MiB write then 256 MiB read, outside the step's events)",
    }
    if mix is not None:
        cfg["route_mix"] = mix
    return cfg


# ----------------------------------------------------------------------------- clocks
class ClockSampler:
    """nvidia-smi sampling during the timed region (start before, stop after)."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_indices):
        self.gpus = {str(i) for i in gpu_indices}
        self.proc = None
        self.path = os.path.join(ROOT, "gpurun_out", f"clocks_{os.getpid()}.csv")

    def start(self):
        try:
            os.makedirs(os.path.dirname(self.path), exist_ok=True)
            self.fh = open(self.path, "w")
            self.proc = subprocess.Popen(["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                                          "-lms", "100"], stdout=self.fh, stderr=subprocess.DEVNULL)
        except OSError:
            self.proc = None

    def stop(self) -> dict:
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        time.sleep(0.15)
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
        self.fh.close()
        sm, smax, reasons = [], [], set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        with open(self.path) as f:
            for line in f:
                parts = [p.strip() for p in line.split(",")]
                if len(parts) < 9 or parts[0] not in self.gpus:
                    continue
                try:
                    sm.append(float(parts[1]))
                    smax.append(float(parts[2]))
                except ValueError:
                    continue
                for name, val in zip(names, parts[5:9]):
                    if val.lower() == "active":
                        reasons.add(name)
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": max(smax) if smax else None,
                "reasons": sorted(reasons), "samples": len(sm)}


# ----------------------------------------------------------------------------- peaks
def measured_peaks(torch, dev) -> dict:
    """bf16 / HBM from the driver-written MEASURED_PEAKS.json; dense fp8 and int8
    library peaks (cuBLAS via torch._scaled_mm / torch._int_mm at 8192^3) measured here."""
    peaks = {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "source": "fallback"}
    path = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(path):
        with open(path) as f:
            mp = json.load(f)
        peaks = {"hbm_gbs": float(mp["hbm_gbs"]), "bf16_tflops": float(mp["bf16_tflops"]),
                 "bf16_tflops_sustained": float(mp.get("bf16_tflops_sustained", 0.0)),
                 "source": "MEASURED_PEAKS.json"}
    n = 8192
    flops = 2.0 * n ** 3

    def best(fn, reps=10):
        for _ in range(3):
            fn()
        s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        t = []
        for _ in range(reps):
            s.record()
            fn()
            e.record()
            e.synchronize()
            t.append(s.elapsed_time(e) / 1e3)
        return flops / min(t) / 1e12

    try:
        a = torch.randn(n, n, device=dev).to(torch.float8_e4m3fn)
        b = torch.randn(n, n, device=dev).to(torch.float8_e4m3fn).t()
        one = torch.ones((), device=dev)
        peaks["fp8_tflops"] = best(lambda: torch._scaled_mm(a, b, scale_a=one, scale_b=one, out_dtype=torch.bfloat16))
        del a, b
    except Exception as exc:  # library without an fp8 GEMM: keep the nominal 2x of bf16
        peaks["fp8_tflops"] = 2.0 * peaks["bf16_tflops"]
        peaks["fp8_note"] = f"2x bf16 (torch._scaled_mm failed: {type(exc).__name__})"
    try:
        a = torch.randint(-127, 127, (n, n), device=dev, dtype=torch.int8)
        b = torch.randint(-127, 127, (n, n), device=dev, dtype=torch.int8)
        peaks["int8_tops"] = best(lambda: torch._int_mm(a, b))
        del a, b
    except Exception as exc:
        peaks["int8_tops"] = 2.0 * peaks["bf16_tflops"]
        peaks["int8_note"] = f"2x bf16 (torch._int_mm failed: {type(exc).__name__})"
    torch.cuda.empty_cache()
    return peaks


# ----------------------------------------------------------------------------- inputs
def make_inputs(torch, pkg, dev, M: int, seed: int):
    g = torch.Generator(device=dev).manual_seed(seed)
    lo, hi = math.log(SCALE_RANGE[0]), math.log(SCALE_RANGE[1])
    s = torch.exp(torch.rand(M, 1, generator=g, device=dev) * (hi - lo) + lo)
    logits = (torch.randn(M, N_LOGIT, generator=g, device=dev) * s).to(torch.float16)
    acts, packs, w_host = [], [], []
    for p, (_, K, N) in enumerate(PROJECTIONS):
        a = torch.randn(M, K, generator=g, device=dev)
        a = torch.where(torch.rand(M, K, generator=g, device=dev) < 0.01, a * 20.0, a)
        acts.append(a.to(torch.float16))
        del a
        gw = torch.Generator(device=dev).manual_seed(1000 + p)  # same weights on every rank
        w = (torch.randn(N, K, generator=gw, device=dev) * 0.02).to(torch.float16)
        w_kn, w_s = pkg.quantize_weights_int8(w)
        packs.append(pkg.WeightPack(w_kn, w_s))
        w_host.append((w_kn, w_s))
        del w
    torch.cuda.empty_cache()
    return logits, acts, packs, w_host


# ----------------------------------------------------------------------------- CPU
def cpu_baseline(torch, logits, acts, w_host, budget_s: float) -> dict:
    """The reference's PyTorch path on the host CPU over a bounded sample of rows."""
    from oracle import ee_cpu_reference as ref

    torch.set_num_threads(os.cpu_count() or 1)
    R = 128
    lg = logits[:R].cpu()
    a_cpu = [a[:R].cpu() for a in acts]
    weights = [ref.CpuWeights(w_kn.cpu(), w_s.cpu()) for w_kn, w_s in w_host]
    ref.gated_step(lg, a_cpu, weights, *TAU)  # warm-up
    times = []
    t_end = time.perf_counter() + budget_s
    while len(times) < 3 or time.perf_counter() < t_end:
        t0 = time.perf_counter()
        ref.gated_step(lg, a_cpu, weights, *TAU)
        times.append(time.perf_counter() - t0)
        if len(times) >= 200:
            break
    t = statistics.median(times)
    return {"value": step_flops(R) / t / 1e12, "unit": UNIT, "cores": torch.get_num_threads(), "kind": "port",
            "sample": f"{R} of the {logits.shape[0]} rows per step, all three projections, median of {len(times)} "
                      f"steps (oracle/ee_cpu_reference.py: the reference's torch ops on the CPU)",
            "ms_per_sample_step": t * 1e3}


def run_reference(args) -> int:
    """--impl reference: the reference's path restated with its own torch ops on the CPU."""
    import torch
    from oracle import ee_cpu_reference as ref

    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", str(args.gpus)))
    if rank != 0:
        return 0
    torch.set_num_threads(os.cpu_count() or 1)
    g = torch.Generator().manual_seed(1234)
    pool = 256
    lo, hi = math.log(SCALE_RANGE[0]), math.log(SCALE_RANGE[1])
    s = torch.exp(torch.rand(pool, 1, generator=g) * (hi - lo) + lo)
    logits = (torch.randn(pool, N_LOGIT, generator=g) * s).to(torch.float16)
    acts, weights = [], []
    for p, (_, K, N) in enumerate(PROJECTIONS):
        a = torch.randn(pool, K, generator=g)
        a = torch.where(torch.rand(pool, K, generator=g) < 0.01, a * 20.0, a)
        acts.append(a.to(torch.float16))
        w = (torch.randn(N, K, generator=torch.Generator().manual_seed(1000 + p)) * 0.02).to(torch.float16)
        weights.append(ref.CpuWeights(*ref.quantize_weights_int8(w)))
        del w
    # size the per-step sample so the whole run stays within about two minutes
    t0 = time.perf_counter()
    ref.gated_step(logits[:16], [a[:16] for a in acts], weights, *TAU)
    per_row = (time.perf_counter() - t0) / 16
    R = int(max(1, min(pool, 120.0 / max(args.steps + args.warmup, 1) / max(per_row, 1e-9))))
    for _ in range(args.warmup):
        ref.gated_step(logits[:R], [a[:R] for a in acts], weights, *TAU)
    times = []
    for k in range(args.steps):
        r0 = (k * R) % max(pool - R + 1, 1)
        t0 = time.perf_counter()
        ref.gated_step(logits[r0:r0 + R], [a[r0:r0 + R] for a in acts], weights, *TAU)
        times.append(time.perf_counter() - t0)
    t = sum(times) / len(times)
    value = step_flops(R) / t / 1e12
    line = {
        "impl": "reference", "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": t * 1e3, "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": DTYPE, "data": "synthetic",
        "config": config_dict(args.rows, world),
        "cpu_baseline": {"value": value, "unit": UNIT, "cores": torch.get_num_threads(), "kind": "port",
                         "sample": f"{R} rows per step (of {args.rows} per GPU), all three projections; "
                                   "the reference's torch ops on the CPU (oracle/ee_cpu_reference.py)"},
        "e2e": {"value": value, "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)
    return 0


# ----------------------------------------------------------------------------- GPU
def main(argv=None) -> int:
    args = parse_args(argv)
    if args.impl == "reference":
        return run_reference(args)
    import torch
    import torch.distributed as dist
    from datetime import timedelta

    import __graft_entry__ as ge

    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    dev = torch.device("cuda", local)
    torch.cuda.set_device(dev)
    if world > 1:
        dist.init_process_group("nccl", timeout=timedelta(seconds=300), device_id=dev)

    def barrier():
        if world > 1:
            dist.barrier(device_ids=[local])

    pkg = ge.load_package()
    M = args.rows
    peaks = measured_peaks(torch, dev) if rank == 0 else None
    logits, acts, packs, w_host = make_inputs(torch, pkg, dev, M, seed=4242 + rank)
    ys = [torch.empty(M, N, dtype=torch.float16, device=dev) for _, _, N in PROJECTIONS]
    router = pkg.EntropyRouter(*TAU)
    router.reserve(M, max(K for _, K, _ in PROJECTIONS), dev)
    flush = L2Flush(torch, dev)
    n_proj = len(PROJECTIONS)

    def step(ev=None):
        if ev is not None:
            ev[0].record()
        router.route(logits)
        if ev is not None:
            ev[1].record()
        for p in range(n_proj):
            router.pack_rows(acts[p])
            if ev is not None:
                ev[2 + 2 * p].record()
            router.gemm_packed(packs[p], out=ys[p])
            if ev is not None:
                ev[3 + 2 * p].record()

    launches_per_step = 1 + 2 * n_proj  # softmax/route/compaction + (pack + GEMM) per projection
    for _ in range(max(args.warmup, 3)):
        flush()
        step()
    torch.cuda.synchronize()
    pkg._lib.device_check()
    counts = router.counts.cpu().tolist()
    mix = {"INT8": counts[0], "FP8": counts[1], "FP16": counts[2]}

    # the timed step is the C++ engine's CUDA graph of the same launches (one host call)
    engine = pkg.GatedLayerEngine([(logits, [(acts[p], packs[p], ys[p]) for p in range(n_proj)])], *TAU)
    engine.capture()
    for _ in range(max(args.warmup, 3)):
        flush()
        engine.launch()
    torch.cuda.synchronize()

    E = lambda: torch.cuda.Event(enable_timing=True)  # noqa: E731
    step_evs = [(E(), E()) for _ in range(args.steps)]
    sampler = ClockSampler(range(world)) if rank == 0 else None
    barrier()
    torch.cuda.synchronize()
    if sampler:
        sampler.start()
        time.sleep(0.3)
    for k in range(args.steps):
        flush()  # between steps, outside the step's events
        step_evs[k][0].record()
        engine.launch()
        step_evs[k][1].record()
    torch.cuda.synchronize()
    barrier()
    clocks = sampler.stop() if sampler else None
    pkg._lib.device_check()
    total_ms = sum(a.elapsed_time(b) for a, b in step_evs)
    if world > 1:
        t = torch.tensor([total_ms], dtype=torch.float64, device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        total_ms = float(t.item())

    # per-kernel breakdown: eager launches bracketed by events; a GPU-side sleep before
    # each step lets the host enqueue the whole step first, so no launch latency leaks in
    n_instr = min(args.steps, 50)
    evs = [[E() for _ in range(2 + 2 * n_proj)] for _ in range(n_instr)]
    for k in range(n_instr):
        flush()
        torch.cuda._sleep(4_000_000)
        step(evs[k])
    torch.cuda.synchronize()
    gate_ms = [ev[0].elapsed_time(ev[1]) for ev in evs]
    pack_ms = [[ev[1 + 2 * p if p == 0 else 3 + 2 * (p - 1)].elapsed_time(ev[2 + 2 * p]) for p in range(n_proj)]
               for ev in evs]
    gemm_ms = [[ev[2 + 2 * p].elapsed_time(ev[3 + 2 * p]) for p in range(n_proj)] for ev in evs]

    # ------------------------------------------------------------------ e2e (public API, host buffers)
    e2e = None
    if not args.no_e2e:
        h_logits = logits.cpu().pin_memory()
        h_acts = [a.cpu().pin_memory() for a in acts]
        h_ys = [torch.empty(y.shape, dtype=y.dtype, pin_memory=True) for y in ys]
        h2d = h_logits.numel() * 2 + sum(a.numel() * 2 for a in h_acts)
        d2h = sum(y.numel() * 2 for y in ys)
        K2 = max(1, args.e2e_steps)
        evs2 = [(E(), E()) for _ in range(K2)]

        def e2e_step(ev):
            ev[0].record()
            logits.copy_(h_logits, non_blocking=True)
            for a, ha in zip(acts, h_acts):
                a.copy_(ha, non_blocking=True)
            router.route(logits)
            for p in range(n_proj):
                router.gated_linear(acts[p], packs[p], out=ys[p])
            for y, hy in zip(ys, h_ys):
                hy.copy_(y, non_blocking=True)
            ev[1].record()

        for _ in range(2):
            e2e_step((E(), E()))
        torch.cuda.synchronize()
        barrier()
        for ev in evs2:
            flush()
            e2e_step(ev)
        torch.cuda.synchronize()
        barrier()
        e2e_total = sum(a.elapsed_time(b) for a, b in evs2)
        if world > 1:
            t = torch.tensor([e2e_total], dtype=torch.float64, device=dev)
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
            e2e_total = float(t.item())
        e2e = {"value": world * step_flops(M) * K2 / (e2e_total / 1e3) / 1e12, "unit": UNIT,
               "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h, "ms_per_step": e2e_total / K2,
               "path": "EntropyRouter.route + EntropyRouter.gated_linear per projection, pinned host in/out"}

    if rank == 0:
        cpu = None
        if world == 1 and not args.no_cpu_baseline:
            cpu = cpu_baseline(torch, logits, acts, w_host, args.cpu_seconds)
        # roofline of the dominant kernel (the bucketed GEMM): effective mixed peak
        c = counts
        f_b = [sum(2.0 * c[b] * K * N for _, K, N in PROJECTIONS) for b in range(3)]
        p_b = [peaks["int8_tops"], peaks["fp8_tflops"], peaks["bf16_tflops"]]
        f_tot = sum(f_b)
        peak_eff = f_tot / sum(f / p for f, p in zip(f_b, p_b))
        gemm_total_ms = sum(sum(x) for x in gemm_ms)
        achieved = f_tot * n_instr / (gemm_total_ms / 1e3) / 1e12
        traffic = None
        tpath = os.path.join(ROOT, "profiles", "gemm_traffic.json")
        if os.path.exists(tpath):
            with open(tpath) as f:
                traffic = json.load(f).get("dram_bytes_per_launch")
        gate_bytes = 2.0 * M * N_LOGIT + 4 * M + M
        gate_gbs = gate_bytes * n_instr / (sum(gate_ms) / 1e3) / 1e9
        value = world * step_flops(M) * args.steps / (total_ms / 1e3) / 1e12
        line = {
            "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": total_ms / args.steps, "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": DTYPE, "data": "synthetic",
            "config": config_dict(M, world, mix),
            "tokens_per_s": world * M * args.steps / (total_ms / 1e3),
            "softmax_entropy": {"gbs": gate_gbs, "frac": gate_gbs / peaks["hbm_gbs"],
                                "us_per_launch": 1e3 * sum(gate_ms) / len(gate_ms),
                                "bytes_per_launch": gate_bytes,
                                "note": "route kernel incl. compaction; algorithmic bytes 2Mn + 4M + M"},
            "per_projection_tflops": {
                name: 2.0 * M * K * N * n_instr / (sum(g[p] for g in gemm_ms) / 1e3) / 1e12
                for p, (name, K, N) in enumerate(PROJECTIONS)},
            "per_kernel_us": {
                "softmax_entropy_route": 1e3 * sum(gate_ms) / n_instr,
                **{f"pack_{name}": 1e3 * sum(x[p] for x in pack_ms) / n_instr for p, (name, _, _) in enumerate(PROJECTIONS)},
                **{f"gemm_{name}": 1e3 * sum(x[p] for x in gemm_ms) / n_instr for p, (name, _, _) in enumerate(PROJECTIONS)},
                "note": f"eager launches, {n_instr} steps, events around each kernel"},
            "timing": "value / ms_per_step: CUDA-graph replays of the step (GatedLayerEngine), events around each replay",
            "roofline": {"bound": "tensor", "achieved": achieved, "peak": peak_eff, "unit": "TFLOP/s",
                         "frac": achieved / peak_eff, "traffic": traffic,
                         "kernel": "gated_gemm_kernel (3 launches per step, one per projection)",
                         "peak_basis": "effective peak of the bucket mix: fp16 bucket at measured bf16 burst "
                                       "(MEASURED_PEAKS.json), FP8 / INT8 buckets at cuBLAS fp8 / int8 8192^3 "
                                       "measured in this run"},
            "peaks": peaks,
            "cpu_baseline": cpu,
            "e2e": e2e,
            "gpu_launches": launches_per_step * args.steps,
            "clocks": clocks,
        }
        print(json.dumps(line), flush=True)
    if world > 1:
        barrier()
        dist.destroy_process_group()
    return 0


if __name__ == "__main__":
    sys.exit(main())
