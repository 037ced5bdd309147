"""Config 4 of the path's scope: a TinyLlama-shaped model (random-init weights, seeded)
run through the entropy-dispatched blocks -- forward tokens/s and the per-token KL
divergence of the gated model's next-token distribution from the all-FP16-tier one.

TinyLlama's weights and WikiText-2 are not on this machine, so the reference's
perplexity evaluation (EE/python/quality_eval.py) is replaced by this seeded stand-in:
ids uniform in [0, vocab), KL(softmax(fp32 logits_gated) || softmax(fp32 logits_fp16))
averaged over tokens; "every linear routed" (q / k / v / o dispatched too, ``route_all``)
against the reference's MLP-only mode.  Attention is the model's own transformers module in eager mode,
as in the reference (it must return the probabilities the router reads), or this
library's flash attention with online entropy (``attention="flash"``).

    python triton-kernels-optimization_b200/eval_llama.py --batch 8 --seq 2048
"""
from __future__ import annotations

import argparse
import json
import os
import sys

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)


def main(argv=None) -> int:
    ap = argparse.ArgumentParser()
    ap.add_argument("--layers", type=int, default=22)
    ap.add_argument("--hidden", type=int, default=2048)
    ap.add_argument("--heads", type=int, default=32)
    ap.add_argument("--kv-heads", type=int, default=4)
    ap.add_argument("--inter", type=int, default=5632)
    ap.add_argument("--vocab", type=int, default=32000)
    ap.add_argument("--batch", type=int, default=8)
    ap.add_argument("--seq", type=int, default=2048)
    ap.add_argument("--reps", type=int, default=2)
    args = ap.parse_args(argv)

    import torch
    from transformers import LlamaConfig, LlamaForCausalLM

    import __graft_entry__ as ge

    pkg = ge.load_package()
    dev = torch.device("cuda:0")
    torch.manual_seed(1234)
    cfg = LlamaConfig(hidden_size=args.hidden, num_hidden_layers=args.layers, num_attention_heads=args.heads,
                      num_key_value_heads=args.kv_heads, intermediate_size=args.inter, vocab_size=args.vocab,
                      rms_norm_eps=1e-5, rope_theta=1e4, max_position_embeddings=max(2048, args.seq),
                      attn_implementation="eager", initializer_range=0.02)
    model = LlamaForCausalLM(cfg).to(dev).half().eval()
    g = torch.Generator(device=dev).manual_seed(99)
    ids = torch.randint(0, args.vocab, (args.batch, args.seq), generator=g, device=dev)
    tokens = args.batch * args.seq
    E = lambda: torch.cuda.Event(enable_timing=True)  # noqa: E731

    def timed(fn):
        fn()
        torch.cuda.synchronize()
        best = None
        for _ in range(args.reps):
            a, b = E(), E()
            a.record()
            out = fn()
            b.record()
            b.synchronize()
            ms = a.elapsed_time(b)
            best = ms if best is None else min(best, ms)
        return out, best

    result = {"config": {"layers": args.layers, "hidden": args.hidden, "heads": args.heads, "kv_heads": args.kv_heads,
                         "inter": args.inter, "vocab": args.vocab, "batch": args.batch, "seq": args.seq,
                         "weights": "random init N(0, 0.02), seed 1234", "ids": "uniform [0, vocab), seed 99"}}
    with torch.no_grad():
        _, ms_hf = timed(lambda: model(ids).logits)
    result["hf_fp16_forward"] = {"ms": round(ms_hf, 2), "tokens_per_s": round(tokens / ms_hf * 1e3)}

    def logprobs(logits):
        return torch.log_softmax(logits.float(), dim=-1)

    runs = {}
    base_lp = None
    for name, (tl, th), routing, attention in [("all_fp16_tier", (-1.0, -1.0), "batch", "eager"),
                                               ("batch_0.41_1.68", (0.41, 1.68), "batch", "eager"),
                                               ("token_0.41_1.68", (0.41, 1.68), "token", "eager"),
                                               ("batch_2.34_6.03", (2.34, 6.03), "batch", "eager"),
                                               ("token_2.34_6.03", (2.34, 6.03), "token", "eager"),
                                               ("flash_all_fp16_tier", (-1.0, -1.0), "batch", "flash"),
                                               ("flash_token_2.34_6.03", (2.34, 6.03), "token", "flash"),
                                               ("flash_batch_2.34_6.03", (2.34, 6.03), "batch", "flash"),
                                               ("flash_token_all_2.34_6.03", (2.34, 6.03), "token", "flash+all"),
                                               ("flash_token_all_0.41_1.68", (0.41, 1.68), "token", "flash+all")]:
        route_all = attention.endswith("+all")
        blocks, disp = pkg.build_dispatched_llama(model, tl, th, routing=routing, attention=attention.split("+")[0],
                                                  route_all=route_all)
        disp.reset_stats()
        logits, ms = timed(lambda: pkg.dispatched_forward(model, blocks, disp, ids))
        lp = logprobs(logits)
        entry = {"ms": round(ms, 2), "tokens_per_s": round(tokens / ms * 1e3),
                 "tiers": {k: v["count"] for k, v in disp.get_stats().items()}}
        if routing == "token":
            mix = [0, 0, 0]
            for blk in blocks:
                r = pkg.EntropyRouter(tl, th)
                r.reserve(tokens, 16, dev)
                r.route_entropy(blk.token_entropy.reshape(-1))
                c = r.counts.cpu().tolist()
                mix = [m + x for m, x in zip(mix, c)]
            entry["token_mix_INT8_FP8_FP16"] = mix
        if base_lp is None:
            base_lp = lp
        else:
            kl = (lp.exp() * (lp - base_lp)).sum(-1).mean()
            entry["kl_vs_all_fp16_tier"] = float(kl)  # against the eager all-FP16-tier run
        runs[name] = entry
        del blocks, logits, lp
        torch.cuda.empty_cache()
    result["dispatched"] = runs
    print(json.dumps(result))
    return 0


if __name__ == "__main__":
    sys.exit(main())
