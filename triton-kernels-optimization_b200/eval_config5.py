"""Config 5 of the path's scope: 4 Llama-3-8B-shaped layers (hidden 4096, 32 query / 8 KV
heads of 128, intermediate 14336; random-init weights, the same seed on every rank) over
16384 tokens = 8 sequences of 2048, split by sequence across the GPUs of one node (mode R:
no collective inside the forward).  Reports the forward's tokens/s over all ranks (time =
max over ranks, CUDA events) and TFLOPS from the config's FLOPs per token
(2 x 872.4 M parameters + 4 x layers x hidden x (S + 1) / 2 for causal attention).  The
embedding (vocabulary 128256) is looked up, there is no lm_head.

    python -m torch.distributed.run --nnodes=1 --nproc-per-node 2 --master-addr 127.0.0.1 \\
        --master-port 29535 triton-kernels-optimization_b200/eval_config5.py
"""
from __future__ import annotations

import argparse
import json
import os
import sys
from datetime import timedelta

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)


def main(argv=None) -> int:
    ap = argparse.ArgumentParser()
    ap.add_argument("--layers", type=int, default=4)
    ap.add_argument("--seqs", type=int, default=8)
    ap.add_argument("--seq", type=int, default=2048)
    ap.add_argument("--reps", type=int, default=3)
    args = ap.parse_args(argv)

    import torch
    import torch.distributed as dist
    from transformers import LlamaConfig
    from transformers.models.llama.modeling_llama import LlamaModel

    import __graft_entry__ as ge

    rank, world = int(os.environ.get("RANK", "0")), int(os.environ.get("WORLD_SIZE", "1"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    dev = torch.device("cuda", local)
    torch.cuda.set_device(dev)
    if world > 1:
        dist.init_process_group("nccl", timeout=timedelta(seconds=300), device_id=dev)
    pkg = ge.load_package()
    from importlib import import_module

    sh = import_module(pkg.__name__ + ".sharding")
    hidden, heads, kv, inter, vocab = 4096, 32, 8, 14336, 128256
    torch.manual_seed(4242)
    cfg = LlamaConfig(hidden_size=hidden, num_hidden_layers=args.layers, num_attention_heads=heads,
                      num_key_value_heads=kv, intermediate_size=inter, vocab_size=vocab, rms_norm_eps=1e-5,
                      rope_theta=5e5, max_position_embeddings=max(8192, args.seq), attn_implementation="eager",
                      initializer_range=0.02)
    model = LlamaModel(cfg).to(dev).half().eval()
    s0, s1 = sh.row_shard(args.seqs, world, rank)
    g = torch.Generator().manual_seed(7)
    ids_all = torch.randint(0, vocab, (args.seqs, args.seq), generator=g)
    ids = ids_all[s0:s1].to(dev)
    B = ids.shape[0]
    tokens_total = args.seqs * args.seq

    wrap = torch.nn.Module()  # build_dispatched_llama reads model.model.layers
    wrap.model = model
    params = sum(p.numel() for n, p in model.named_parameters() if "embed_tokens" not in n)
    flops_tok = 2.0 * params + 4.0 * args.layers * hidden * (args.seq + 1) / 2
    results = {}
    for name, routing, attention in (("token_flash", "token", "flash"), ("batch_flash", "batch", "flash")):
        blocks, disp = pkg.build_dispatched_llama(wrap, 0.41, 1.68, routing=routing, attention=attention)

        @torch.no_grad()
        def forward():
            h = model.embed_tokens(ids).half()
            pos = torch.arange(args.seq, device=dev).unsqueeze(0).expand(B, args.seq)
            pe = model.rotary_emb(h, pos)
            for blk in blocks:
                h = blk(h, dispatcher=disp, position_ids=pos, position_embeddings=pe)[0]
            return model.norm(h)

        forward()
        torch.cuda.synchronize()
        best = None
        for _ in range(args.reps):
            if world > 1:
                dist.barrier(device_ids=[local])
            a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            a.record()
            forward()
            b.record()
            b.synchronize()
            t = torch.tensor([a.elapsed_time(b)], device=dev, dtype=torch.float64)
            if world > 1:
                dist.all_reduce(t, op=dist.ReduceOp.MAX)
            ms = float(t.item())
            best = ms if best is None else min(best, ms)
        results[name] = {"ms": round(best, 2), "tokens_per_s": round(tokens_total / best * 1e3),
                         "tflops_total": round(flops_tok * tokens_total / best / 1e9, 1)}
        del blocks
        torch.cuda.empty_cache()
    if rank == 0:
        print(json.dumps({"gpus": world, "layers": args.layers, "tokens": tokens_total, "seq": args.seq,
                          "params_per_forward": params, "flops_per_token": flops_tok, "mode": "R (sequences per GPU)",
                          "runs": results}))
    if world > 1:
        dist.barrier(device_ids=[local])
        dist.destroy_process_group()
    return 0


if __name__ == "__main__":
    sys.exit(main())
