"""Generates the golden vectors in tests/golden/ by running the reference's own code.

The reference (IqtedarU/triton-kernels-optimization, ``entropy-engine/python``) is
imported read-only from its checkout and executed on the CPU:
  * its Triton kernels run under the Triton 3.6 interpreter (TRITON_INTERPRET=1);
  * its GEMM launchers run unchanged; only the autotuner is pinned to the AOT
    configuration the reference ships (BLOCK 64 x 128 x 64, EE/python/compile_kernels.py:27-31),
    because autotuning needs a GPU;
  * the interpreter's fp16 -> fp8e4nv cast rounds half-up without carry or
    saturation, unlike the GPU's cvt.rn.satfinite; that one cast is replaced by
    torch's round-to-nearest-even e4m3 conversion after saturation to +-448, which is
    what the reference computes on hardware;
  * the dispatcher is constructed with pin_memory dropped (no CUDA here).
Inputs are seeded numpy draws (the reference's own tests use CUDA RNG, which a CPU
cannot reproduce).  Nothing here is needed at test time: the .npz / .json files it
writes are the fixtures.

    python tests/golden/make_golden.py --reference /path/to/reference/checkout
"""
from __future__ import annotations

import argparse
import json
import math
import os
import sys

os.environ.setdefault("TRITON_INTERPRET", "1")

import numpy as np  # noqa: E402
import torch  # noqa: E402

HERE = os.path.dirname(os.path.abspath(__file__))
PINNED = {"BLOCK_M": 64, "BLOCK_N": 128, "BLOCK_K": 64}


def _patch_fp8_cast():
    import triton.language as tl
    import triton.runtime.interpreter as interp

    original = interp._convert_float

    def convert(input, input_dtype, output_dtype, rounding_mode):
        if output_dtype == tl.float8e4nv and input_dtype in (tl.float16, tl.float32):
            x = torch.from_numpy(np.ascontiguousarray(input).astype(np.float32))
            return x.clamp(-448.0, 448.0).to(torch.float8_e4m3fn).view(torch.uint8).numpy().reshape(np.shape(input))
        if input_dtype == tl.float8e4nv and output_dtype == tl.float16:
            x = torch.from_numpy(np.ascontiguousarray(input).astype(np.uint8)).view(torch.float8_e4m3fn)
            return x.to(torch.float16).view(torch.int16).numpy().view(np.uint16).reshape(np.shape(input))
        return original(input, input_dtype, output_dtype, rounding_mode)

    interp._convert_float = convert


class _PinnedKernel:
    """Stands in for an @triton.autotune kernel: launches its JIT function with the
    reference's AOT tile config and records the arguments it was given."""

    def __init__(self, autotuned):
        self.fn = autotuned.fn
        self.calls = []

    def __getitem__(self, grid):
        def launch(*args, **kwargs):
            self.calls.append([a.clone() if isinstance(a, torch.Tensor) else a for a in args])
            return self.fn[grid](*args, **kwargs, **PINNED)
        return launch


def _config1_logits(rng, rows, n):
    s = np.exp(rng.uniform(math.log(0.05), math.log(20.0), size=rows))
    return (rng.standard_normal((rows, n)) * s[:, None]).astype(np.float16)


def main(argv=None):
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", required=True, help="reference checkout root")
    ap.add_argument("--only", choices=["attention"], default=None,
                    help="write only this fixture (the others are left as they are)")
    args = ap.parse_args(argv)
    pydir = os.path.join(args.reference, "entropy-engine (1)", "entropy-engine", "python")
    sys.path.insert(0, pydir)
    if args.only == "attention":
        import dispatch as D  # the reference's dispatch.py

        _attention_goldens(D)
        return
    _patch_fp8_cast()
    import triton
    import kernels as K  # the reference's kernels.py
    import dispatch as D  # the reference's dispatch.py

    rng = np.random.default_rng(20260101)

    # ------------------------------------------------------------ softmax + entropy
    sm = {}
    for tag, rows, n, causal in [("r64n1024", 64, 1024, False), ("r16n4096", 16, 4096, False),
                                 ("r128n64c", 128, 64, True), ("r40n48c", 40, 48, True)]:
        x = _config1_logits(rng, rows, n) if not causal else rng.standard_normal((rows, n)).astype(np.float16)
        xt = torch.from_numpy(x)
        probs = torch.empty_like(xt)
        H = torch.empty(rows, dtype=torch.float32)
        block = triton.next_power_of_2(n)
        K.fused_softmax_entropy_kernel[(rows,)](xt, probs, H, n, n, BLOCK_S=block, IS_CAUSAL=causal)
        sm[f"{tag}_x"] = x
        sm[f"{tag}_probs"] = probs.numpy()
        sm[f"{tag}_H"] = H.numpy()
    for tag, shape in [("b2h2s64", (2, 2, 64, 64)), ("b1h2s48", (1, 2, 48, 48))]:
        x = rng.standard_normal(shape).astype(np.float16)
        probs, per_batch = K.fused_softmax_entropy(torch.from_numpy(x), causal=True)
        sm[f"{tag}_x"] = x
        sm[f"{tag}_probs"] = probs.numpy()
        sm[f"{tag}_batchH"] = per_batch.numpy()
    np.savez_compressed(os.path.join(HERE, "golden_softmax.npz"), **sm)

    # ------------------------------------------------------------ GEMM launchers
    K.gemm_int8_kernel = _PinnedKernel(K.gemm_int8_kernel)
    K.gemm_fp8_kernel = _PinnedKernel(K.gemm_fp8_kernel)
    K.gemm_fp16_kernel = _PinnedKernel(K.gemm_fp16_kernel)
    gm = {}
    for tag, M, Kd, N, scale, outliers in [("m128k256n256", 128, 256, 256, 1.0, True),
                                            ("m64k512n128", 64, 512, 128, 0.1, False)]:
        a = rng.standard_normal((M, Kd)) * scale
        if outliers:
            a = np.where(rng.random((M, Kd)) < 0.01, a * 20.0, a)
        a = a.astype(np.float16)
        a[3] = 0.0  # an all-zero activation row
        W = (rng.standard_normal((N, Kd)) * 0.02).astype(np.float16)
        W[5] = 0.0  # an all-zero output channel (scale clamps to 1e-8)
        w_kn, w_s = D.quantize_weights_int8(torch.from_numpy(W))
        at = torch.from_numpy(a)
        y8 = K.triton_int8_gemm(at, w_kn, w_s)
        q_a, s_a = K.gemm_int8_kernel.calls[-1][0], K.gemm_int8_kernel.calls[-1][3]
        yf8 = K.triton_fp8_gemm(at, w_kn, w_s)
        s_a8 = K.gemm_fp8_kernel.calls[-1][3]
        y16 = K.triton_fp16_gemm(at, w_kn, w_s)
        gm.update({f"{tag}_A": a, f"{tag}_W": W, f"{tag}_wkn": w_kn.numpy(), f"{tag}_ws": w_s.numpy(),
                   f"{tag}_qa": q_a.numpy(), f"{tag}_sa": s_a.numpy(), f"{tag}_y_int8": y8.numpy(),
                   f"{tag}_sa8": s_a8.numpy(), f"{tag}_y_fp8": yf8.numpy(), f"{tag}_y_fp16": y16.numpy()})
    np.savez_compressed(os.path.join(HERE, "golden_gemm.npz"), **gm)

    # ------------------------------------------------------------ dispatcher
    real_empty = torch.empty

    def empty_unpinned(*a, **k):
        k.pop("pin_memory", None)
        return real_empty(*a, **k)

    cases = []
    for tl_, th_, seq in [(2.0, 3.5, [1.0, 2.5, 4.0]),
                          (2.0, 3.5, [2.0, 3.5, float(np.nextafter(np.float32(2.0), np.float32(0.0))), 0.0]),
                          (0.41, 1.68, [float(np.float32(0.41)), float(np.float32(1.68)), 0.4099999, 1.68, 8.3]),
                          (2.0, 3.5, [[0.5, 3.9, 1.0], [0.1, 0.2], [2.4, 2.6]])]:
        torch.empty = empty_unpinned
        try:
            d = D.PipelinedEntropyDispatcher(tau_low=tl_, tau_high=th_)
        finally:
            torch.empty = real_empty
        tiers = [int(d.get_tier())]  # before any submission
        for v in seq:
            d.submit_entropy(torch.tensor(v if isinstance(v, list) else [v], dtype=torch.float32))
            tiers.append(int(d.get_tier()))
        stats = {k: v["count"] for k, v in d.get_stats().items()}
        cases.append({"tau_low": tl_, "tau_high": th_, "submitted": seq, "tiers": tiers, "counts": stats})
    with open(os.path.join(HERE, "golden_dispatch.json"), "w") as f:
        json.dump({"cases": cases}, f, indent=1)
    _attention_goldens(D)
    print("golden vectors written to", HERE)


def _attention_goldens(D):
    """The Llama-path router input: the reference block's own
    _attention_with_fused_entropy (EE/python/dispatch.py:212-247) over a small
    transformers LlamaAttention (eager, CPU), recording the attention probabilities it
    produced and the per-batch entropy it returned."""
    from transformers import LlamaConfig
    from transformers.models.llama.modeling_llama import LlamaAttention, LlamaRotaryEmbedding

    out = {}
    for tag, (B, S, hidden, heads, kv, dtype) in {"b2s48": (2, 48, 128, 4, 2, torch.float32),
                                                   "b1s64h": (1, 64, 128, 4, 4, torch.float16),
                                                   "b3s33": (3, 33, 64, 2, 1, torch.float32)}.items():
        torch.manual_seed(1234 + S)
        cfg = LlamaConfig(hidden_size=hidden, num_attention_heads=heads, num_key_value_heads=kv,
                          intermediate_size=4 * hidden, num_hidden_layers=1, vocab_size=64,
                          attn_implementation="eager")
        attn = LlamaAttention(cfg, layer_idx=0).to(dtype).eval()
        rope = LlamaRotaryEmbedding(cfg)
        x = (torch.randn(B, S, hidden) * 2.0).to(dtype)
        pos = torch.arange(S)[None].expand(B, S)
        cos, sin = rope(x, pos)
        mask = torch.full((S, S), float("-inf")).triu(1)[None, None].to(dtype)

        class _Block:  # the attributes _attention_with_fused_entropy reads
            self_attn = attn

        captured = {}
        real = attn.forward

        def forward(*a, **k):
            res = real(*a, **k)
            captured["p"] = res[1].detach().clone()
            return res

        attn.forward = forward
        with torch.no_grad():
            _, entropy_batch, _ = D.EntropyDispatchedLlamaBlock._attention_with_fused_entropy(
                _Block(), x, attention_mask=mask, position_ids=pos, position_embeddings=(cos, sin))
        p = captured["p"]
        out[f"{tag}_p"] = p.numpy()
        out[f"{tag}_entropy"] = entropy_batch.float().numpy()
    np.savez_compressed(os.path.join(HERE, "golden_attention.npz"), **out)


if __name__ == "__main__":
    main()
