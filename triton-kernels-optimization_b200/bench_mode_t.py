"""Mode T against mode R for the gated SwiGLU MLP on the GPUs of one node (config 5's
MLP: d = 4096, I = 14336, 16384 token rows split evenly across the ranks).  Run under
torchrun, one process per GPU:

    python -m torch.distributed.run --nnodes=1 --nproc-per-node 2 --master-addr 127.0.0.1 \\
        --master-port 29534 triton-kernels-optimization_b200/bench_mode_t.py

Mode T: ``ColumnParallelGatedMLP`` (gate / up split by column, rows all-gathered and
exchanged).  Mode R: the same class at world size 1 on each rank's own rows with the
full weights (no collective).  Times are CUDA events over 10 calls, max over ranks.
"""
from __future__ import annotations

import json
import os
import sys
from datetime import timedelta

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)


def main() -> int:
    import torch
    import torch.distributed as dist

    import __graft_entry__ as ge

    rank, world = int(os.environ.get("RANK", "0")), int(os.environ.get("WORLD_SIZE", "1"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    dev = torch.device("cuda", local)
    torch.cuda.set_device(dev)
    dist.init_process_group("nccl", timeout=timedelta(seconds=120), device_id=dev)
    pkg = ge.load_package()
    from importlib import import_module

    sh = import_module(pkg.__name__ + ".sharding")
    M_total, d, inter = 16384, 4096, 14336
    m = M_total // world
    g = torch.Generator(device=dev).manual_seed(7)
    wg = (torch.randn(inter, d, generator=g, device=dev) * 0.02).half()
    wu = (torch.randn(inter, d, generator=g, device=dev) * 0.02).half()
    wd = (torch.randn(d, inter, generator=g, device=dev) * 0.02).half()
    x = torch.randn(m, d, generator=g, device=dev).half()
    H = torch.rand(m, generator=g, device=dev) * 2.5
    mode_t = sh.ColumnParallelGatedMLP(wg, wu, wd, world, rank)
    mode_r = sh.ColumnParallelGatedMLP(wg, wu, wd, 1, 0)

    def timed(fn, n=10):
        for _ in range(3):
            fn()
        torch.cuda.synchronize()
        dist.barrier(device_ids=[local])
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record()
        for _ in range(n):
            fn()
        b.record()
        b.synchronize()
        t = torch.tensor([a.elapsed_time(b) / n], device=dev, dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    t_t = timed(lambda: mode_t.forward(x, H))
    t_r = timed(lambda: mode_r.forward(x, H))
    flops = 2.0 * M_total * 3 * d * inter
    if rank == 0:
        print(json.dumps({"world": world, "rows_total": M_total, "d": d, "inter": inter,
                          "mode_t_ms": round(t_t, 3), "mode_t_tflops_total": round(flops / t_t / 1e9, 1),
                          "mode_r_ms": round(t_r, 3), "mode_r_tflops_total": round(flops / t_r / 1e9, 1)}))
    dist.barrier(device_ids=[local])
    dist.destroy_process_group()
    return 0


if __name__ == "__main__":
    sys.exit(main())
