"""CPU baseline of the entropy-gated step -- TEST / BENCHMARK INFRASTRUCTURE ONLY.

The reference (IqtedarU/triton-kernels-optimization, ``entropy-engine/``; "EE/"
below) has no CPU implementation of its own: its kernels are Triton (GPU) and its
launchers are PyTorch ops.  This module restates the same path with the reference's
own PyTorch ops on the CPU, the baseline its benchmark plan names:

  * softmax + entropy        as EE/python/benchmark.py:157-160
  * dual-threshold route     as EE/python/dispatch.py:74-79 (per row)
  * INT8 launcher            EE/python/kernels.py:336-338, int32 GEMM via torch._int_mm,
                             epilogue as kernels.py:104
  * FP8 launcher             EE/python/kernels.py:361, :144-160, :176-180 with the
                             e4m3 weight operand precomputed (kernels.py:166)
  * FP16 launcher            fp32 matmul against fp16(fp16(q) * fp16(s)) (kernels.py:215-238)

Only ``bench.py`` (its cpu_baseline leg and its ``--impl reference`` arm) uses it;
the product path never does.  Weight preparation is offline and is not timed.
"""
from __future__ import annotations

import torch

INT8, FP8, FP16 = 0, 1, 2


class CpuWeights:
    """Offline CPU operand forms of one INT8-quantised weight ([K, N] + scale [N])."""

    def __init__(self, w_kn: torch.Tensor, scale: torch.Tensor):
        self.w_kn = w_kn.contiguous().cpu()
        self.scale = scale.float().contiguous().cpu()
        qh = self.w_kn.to(torch.float16)
        self.w_e4m3_f32 = qh.to(torch.float8_e4m3fn).to(torch.float32)
        self.w_f16_f32 = (qh * self.scale.to(torch.float16)[None, :]).to(torch.float32)
        self.K, self.N = self.w_kn.shape


def quantize_weights_int8(weight: torch.Tensor):
    """EE/python/dispatch.py:43-48 with torch on the CPU."""
    w = weight.detach().float().t().contiguous()
    scale = (w.abs().amax(dim=0) / 127.0).clamp(min=1e-8)
    q = (w / scale.unsqueeze(0)).round().clamp(-127, 127).to(torch.int8)
    return q.contiguous(), scale.contiguous()


def softmax_entropy_route(logits: torch.Tensor, tau_low: float, tau_high: float):
    p = torch.softmax(logits.float(), dim=-1)
    H = -(p * torch.log(p + 1e-10)).sum(dim=-1)
    route = torch.where(H < tau_low, INT8, torch.where(H < tau_high, FP8, FP16)).to(torch.int8)
    return H, route


def _int8_rows(a: torch.Tensor, w: CpuWeights) -> torch.Tensor:
    a_scale = (a.abs().amax(dim=1) / 127.0).clamp(min=1e-8).to(torch.float32)
    a_int8 = (a / a_scale[:, None]).to(torch.int8)
    if a_int8.shape[0] > 16:
        acc = torch._int_mm(a_int8, w.w_kn).to(torch.float32)
    else:  # torch._int_mm wants more than 16 rows; the exact fp64 product is the same integer
        acc = (a_int8.double() @ w.w_kn.double()).to(torch.float32)
    return (acc * a_scale[:, None] * w.scale[None, :]).to(torch.float16)


def _fp8_rows(a: torch.Tensor, w: CpuWeights) -> torch.Tensor:
    a_scale = (a.abs().amax(dim=1) / 448.0).clamp(min=1e-12).to(torch.float32)
    inv = (1.0 / a_scale).to(torch.float16)
    a8 = (a * inv[:, None]).clamp(-448, 448).to(torch.float8_e4m3fn).to(torch.float32)
    acc = a8 @ w.w_e4m3_f32
    return (acc * a_scale[:, None] * w.scale[None, :]).to(torch.float16)


def _fp16_rows(a: torch.Tensor, w: CpuWeights) -> torch.Tensor:
    return (a.float() @ w.w_f16_f32).to(torch.float16)


def gated_linear_rows(a: torch.Tensor, route: torch.Tensor, w: CpuWeights) -> torch.Tensor:
    """Y[i] = reference launcher of tier route[i] applied to row i (fp16 [M, N])."""
    y = torch.empty(a.shape[0], w.N, dtype=torch.float16)
    for b, fn in ((INT8, _int8_rows), (FP8, _fp8_rows), (FP16, _fp16_rows)):
        idx = torch.nonzero(route == b).flatten()
        if idx.numel():
            y[idx] = fn(a[idx], w)
    return y


def gated_step(logits: torch.Tensor, acts: list, weights: list, tau_low: float, tau_high: float):
    """One gated step on the CPU: route the rows once, then every projection."""
    H, route = softmax_entropy_route(logits, tau_low, tau_high)
    return H, route, [gated_linear_rows(a, route, w) for a, w in zip(acts, weights)]
