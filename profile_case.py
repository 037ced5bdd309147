"""Runs one small case of the gated path a few times, for kernel captures with ncu.

--case gated (default): each repetition launches, in order, the router (softmax +
entropy + route + bucket scan) over logits [rows, 4096], the row packing of A [rows, K]
and the gated GEMM against a [N, K] weight (the router's workspace has room for K-split
partials, as EntropyRouter sizes it by default).  Inputs follow bench.py's laws (route
mix about 24 / 55 / 21 %); device footprint is about 4*N*K + 5*rows*K + 2*rows*N bytes
(+ 77 MB of split room above 64 rows).

--case attention: each repetition runs flash_attention_entropy (causal, output and
per-row entropy) on q [B, Hq, S, D], k / v [B, Hkv, S, D]; with --exact the exact-entropy
mode instead (flash_attention_rope_entropy with cos = 1, sin = 0 on [B, S, H * D] rows:
the flash pass, then the second pass that rounds each probability to fp16).

--case kv: an entropy-tied KV cache of --B sequences x --S tokens (8 KV heads of 128, tokens
stored at about 24 / 55 / 21 % INT8 / FP8 / FP16, the bench's seeds), then per repetition
one decode step's attention of 32 query heads against it (+ its own new K / V).

--case forward: each repetition runs one eager forward of the decoder-stack engine over
--layers Llama-3-8B-shaped layers (hidden 4096, 32 / 8 heads of 128, intermediate 14336;
random-init weights) for --B sequences of --S tokens, per-token routing at (0.41, 1.68).

    python profile_case.py --rows 2048 --K 4096 --N 14336 --reps 4
    ncu --set full --clock-control none -k regex:gated_gemm -s 3 -c 1 -o prof <same command>
    python profile_case.py --case attention --B 1 --Hq 32 --Hkv 4 --S 2048 --D 64
    python profile_case.py --case attention --exact --B 2 --Hq 32 --Hkv 8 --S 2048 --D 128
    python profile_case.py --case forward --layers 1 --B 8 --S 2048 --reps 2
    python profile_case.py --case kv --B 8 --S 8192 --reps 3
"""
from __future__ import annotations

import argparse
import math
import os
import sys

ROOT = os.path.dirname(os.path.abspath(__file__))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)


def main(argv=None) -> int:
    ap = argparse.ArgumentParser()
    ap.add_argument("--rows", type=int, default=2048)
    ap.add_argument("--K", type=int, default=4096)
    ap.add_argument("--N", type=int, default=14336)
    ap.add_argument("--n-logits", type=int, default=4096)
    ap.add_argument("--reps", type=int, default=4)
    ap.add_argument("--case", choices=("gated", "attention", "forward", "kv"), default="gated")
    ap.add_argument("--layers", type=int, default=1)
    ap.add_argument("--B", type=int, default=1)
    ap.add_argument("--Hq", type=int, default=32)
    ap.add_argument("--Hkv", type=int, default=4)
    ap.add_argument("--S", type=int, default=2048)
    ap.add_argument("--D", type=int, default=64)
    ap.add_argument("--exact", action="store_true", help="attention: the exact-entropy mode")
    args = ap.parse_args(argv)

    import torch

    import __graft_entry__ as ge

    pkg = ge.load_package()
    dev = torch.device("cuda:0")
    g = torch.Generator(device=dev).manual_seed(7)
    if args.case == "forward":
        from transformers import LlamaConfig
        from transformers.models.llama.modeling_llama import LlamaModel

        torch.manual_seed(4242)
        cfg = LlamaConfig(hidden_size=4096, num_hidden_layers=args.layers, num_attention_heads=32,
                          num_key_value_heads=8, intermediate_size=14336, vocab_size=1024, rms_norm_eps=1e-5,
                          rope_theta=5e5, max_position_embeddings=8192, attn_implementation="eager",
                          initializer_range=0.02)
        with torch.device(dev):
            model = LlamaModel(cfg)
        model = model.half().eval().requires_grad_(False)
        eng = pkg.DecoderEngine.from_model(model, args.B, args.S, 0.41, 1.68, routing="token")
        x = torch.randn(args.B * args.S, 4096, generator=g, device=dev).half() * 0.02
        for _ in range(args.reps):
            eng.run(x)
        torch.cuda.synchronize()
        pkg._lib.device_check()
        print("forward", args.layers, "layers", args.B, "x", args.S, "mix", eng.layer_counts.sum(dim=0).tolist())
        return 0
    if args.case == "kv":
        kv, d, hq = 8, 128, 32
        gk = torch.Generator(device=dev).manual_seed(21)
        cache = pkg.EntropyKVCache(args.B, kv, d, args.S + 64, device=dev)
        k = torch.randn(args.B * args.S, kv * d, generator=gk, device=dev).half()
        v = torch.randn(args.B * args.S, kv * d, generator=gk, device=dev).half()
        u = torch.rand(args.B * args.S, generator=gk, device=dev)
        tier = torch.where(u < 0.24, 0, torch.where(u < 0.79, 1, 2)).to(torch.int8)
        cache.append(k, v, tier)
        del k, v
        q = torch.randn(args.B, hq * d, generator=gk, device=dev).half()
        kn = torch.randn(args.B, kv * d, generator=gk, device=dev).half()
        vn = torch.randn(args.B, kv * d, generator=gk, device=dev).half()
        out = torch.empty_like(q)
        for _ in range(args.reps):
            cache.decode_attention(q, kn, vn, d ** -0.5, out=out)
        torch.cuda.synchronize()
        pkg._lib.device_check()
        print("kv decode", args.B, "x", args.S, "tiers", [int((tier == t).sum()) for t in range(3)])
        return 0
    if args.case == "attention" and args.exact:
        B, S, D = args.B, args.S, args.D
        q = torch.randn(B, S, args.Hq * D, generator=g, device=dev).half()
        k = torch.randn(B, S, args.Hkv * D, generator=g, device=dev).half()
        v = torch.randn(B, S, args.Hkv * D, generator=g, device=dev).half()
        cos = torch.ones(B, S, D, device=dev, dtype=torch.float16)
        sin = torch.zeros_like(cos)
        for _ in range(args.reps):
            out, hb = pkg.flash_attention_rope_entropy(q, k, v, cos, sin, args.Hq, args.Hkv, exact_entropy=True)
        torch.cuda.synchronize()
        pkg._lib.device_check()
        print("exact-entropy attention", tuple(q.shape), "kv", tuple(k.shape), "batch entropy", hb.cpu().tolist())
        return 0
    if args.case == "attention":
        q = torch.randn(args.B, args.Hq, args.S, args.D, generator=g, device=dev).half()
        k = torch.randn(args.B, args.Hkv, args.S, args.D, generator=g, device=dev).half()
        v = torch.randn(args.B, args.Hkv, args.S, args.D, generator=g, device=dev).half()
        for _ in range(args.reps):
            out, hb = pkg.flash_attention_entropy(q, k, v, causal=True)
        torch.cuda.synchronize()
        pkg._lib.device_check()
        print("attention", tuple(q.shape), "kv", tuple(k.shape), "batch entropy", hb.cpu().tolist())
        return 0
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
