"""Runs one small case of the gated path a few times, for kernel captures with ncu.

Each repetition launches, in order: the router (softmax + entropy + route +
compaction) over logits [rows, 4096], the row packing of A [rows, K] and the gated
GEMM against a [N, K] weight.  Inputs follow bench.py's laws (route mix about
24 / 55 / 21 %); device footprint is about 4*N*K + 5*rows*K + 2*rows*N bytes.

    python triton-kernels-optimization_b200/profile_case.py --rows 2048 --K 4096 --N 14336 --reps 4
    ncu --set full --clock-control none -k regex:gated_gemm -s 3 -c 1 -o prof <same command>
"""
from __future__ import annotations

import argparse
import math
import os
import sys

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)


def main(argv=None) -> int:
    ap = argparse.ArgumentParser()
    ap.add_argument("--rows", type=int, default=2048)
    ap.add_argument("--K", type=int, default=4096)
    ap.add_argument("--N", type=int, default=14336)
    ap.add_argument("--n-logits", type=int, default=4096)
    ap.add_argument("--reps", type=int, default=4)
    args = ap.parse_args(argv)

    import torch

    import __graft_entry__ as ge

    pkg = ge.load_package()
    dev = torch.device("cuda:0")
    g = torch.Generator(device=dev).manual_seed(7)
    M, K, N = args.rows, args.K, args.N
    s = torch.exp(torch.rand(M, 1, generator=g, device=dev) * (math.log(9.5) - math.log(7.0)) + math.log(7.0))
    logits = (torch.randn(M, args.n_logits, generator=g, device=dev) * s).half()
    a = torch.randn(M, K, generator=g, device=dev)
    a = torch.where(torch.rand(M, K, generator=g, device=dev) < 0.01, a * 20.0, a).half()
    w = (torch.randn(N, K, generator=g, device=dev) * 0.02).half()
    pack = pkg.WeightPack(*pkg.quantize_weights_int8(w))
    del w
    y = torch.empty(M, N, dtype=torch.float16, device=dev)
    router = pkg.EntropyRouter(0.41, 1.68)
    router.reserve(M, K, dev)
    for _ in range(args.reps):
        router.route(logits)
        router.pack_rows(a)
        router.gemm_packed(pack, out=y)
    torch.cuda.synchronize()
    pkg._lib.device_check()
    print("buckets", router.counts.cpu().tolist(), "rows", M, "K", K, "N", N)
    return 0


if __name__ == "__main__":
    sys.exit(main())
