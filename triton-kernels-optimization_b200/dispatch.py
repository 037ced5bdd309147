"""The reference's dispatch surface (EE/python/dispatch.py) on the B200 engine.

* ``PrecisionTier`` / ``quantize_weights_int8`` -- same ids and weight format.
* ``PipelinedEntropyDispatcher`` -- the reference's batch-max dual-threshold rule
  (dispatch.py:55-97); the max and the tier are computed on the device and reach
  the host through pinned memory guarded by an event, not ``.item()`` on a device
  tensor.
* ``EntropyDispatchedLinear`` -- drop-in nn.Linear replacement (dispatch.py:103-143):
  ``forward(x, tier)`` runs the whole tensor in one precision as the reference does;
  ``forward_gated(x, router)`` routes every row by its own entropy on the device.
* ``EntropyRouter`` -- the on-device dispatcher: softmax + entropy + per-row route +
  stable bucket compaction in one kernel, reusable by every linear that shares the
  rows (``gated_linear``).
"""
from __future__ import annotations

import ctypes
from enum import IntEnum
from typing import Optional

import torch
import torch.nn as nn

from . import _lib
from ._lib import call
from .kernels import (
    SwiGLUPack,
    WeightPack,
    _check_act,
    _ptr,
    _require,
    _stream,
    quantize_weights_int8,
    triton_fp16_gemm,
    triton_fp8_gemm,
    triton_int8_gemm,
)

__all__ = [
    "PrecisionTier",
    "quantize_weights_int8",
    "PipelinedEntropyDispatcher",
    "EntropyDispatchedLinear",
    "EntropyRouter",
    "gated_linear",
]


class PrecisionTier(IntEnum):
    """Precision tiers ordered by compute throughput (EE/python/dispatch.py:32-36)."""
    INT8 = 0
    FP8 = 1
    FP16 = 2


def tier_of(value: float, tau_low: float, tau_high: float) -> PrecisionTier:
    """Dual-threshold rule with strict comparisons (EE/python/dispatch.py:74-79)."""
    if value < tau_low:
        return PrecisionTier.INT8
    if value < tau_high:
        return PrecisionTier.FP8
    return PrecisionTier.FP16


class PipelinedEntropyDispatcher:
    """Batch-max dual-threshold dispatcher (EE/python/dispatch.py:55-97).

    ``submit_entropy`` enqueues, on the current stream, one kernel that takes the max
    of the batch's entropies, then an asynchronous copy of that max into pinned host
    memory, and records an event.  ``get_tier`` waits for that event only (not for the
    whole device) and applies the rule on the host in double precision, exactly as the
    reference compares its Python float.  Before any submission it returns FP16.
    """

    def __init__(self, tau_low: float = 2.0, tau_high: float = 3.5):
        self.tau_low = tau_low
        self.tau_high = tau_high
        self._pinned = torch.empty(1, dtype=torch.float32, pin_memory=torch.cuda.is_available())
        self._dev: Optional[torch.Tensor] = None
        self._event: Optional[torch.cuda.Event] = None
        self._has_value = False
        self.tier_counts = {PrecisionTier.INT8: 0, PrecisionTier.FP8: 0, PrecisionTier.FP16: 0}

    def submit_entropy(self, entropy_batch: torch.Tensor) -> None:
        h = entropy_batch.detach()
        if h.dtype != torch.float32:
            h = h.float()
        h = h.contiguous().reshape(-1)
        _require(h.is_cuda and h.numel() > 0, "entropy_batch must be a non-empty CUDA tensor")
        if self._dev is None or self._dev.device != h.device:
            self._dev = torch.empty(2, dtype=torch.float32, device=h.device)
        with torch.cuda.device(h.device):
            call("ee_route_batch_max", h.data_ptr(), h.numel(), float(self.tau_low), float(self.tau_high),
                 self._dev.data_ptr(), None, _stream())
            self._pinned.copy_(self._dev[:1], non_blocking=True)
            self._event = torch.cuda.Event()
            self._event.record()
        self._has_value = True

    def get_tier(self) -> PrecisionTier:
        if not self._has_value:
            return PrecisionTier.FP16
        self._event.synchronize()
        tier = tier_of(float(self._pinned[0]), self.tau_low, self.tau_high)
        self.tier_counts[tier] += 1
        return tier

    def reset_stats(self) -> None:
        self._has_value = False
        self.tier_counts = {t: 0 for t in PrecisionTier}

    def get_stats(self) -> dict:
        total = sum(self.tier_counts.values())
        return {
            tier.name: {"count": self.tier_counts[tier], "pct": self.tier_counts[tier] / max(total, 1) * 100}
            for tier in PrecisionTier
        }


class EntropyRouter:
    """On-device per-row dispatcher.

    ``route(logits)`` launches one kernel over the fp16 logits [M, n]: per-row softmax
    entropy, dual-threshold route id, the bucket counts and the per-chunk scan that
    fixes each row's place in the stable INT8 / FP8 / FP16 order, all kept in a device
    workspace.  Every ``gated_linear(A, pack)`` that follows on the same stream reuses
    that routing for its own activations (row i of A belongs to row i of the logits).
    There is no host round trip; ``H``, ``route_ids``, ``counts`` and ``perm`` are views
    into the workspace, valid until the next ``route``.  ``H``, ``route_ids`` and
    ``counts`` are filled by ``route``; ``perm`` (position -> row) by the first
    ``pack_rows`` / ``gated_linear`` after it, which places the rows.

    ``k_split`` (default on) sizes the workspace with room for K-split partial sums
    (``ee_gated_workspace_split_bytes``: about 0.5 MiB per SM for more than 64 rows), so
    GEMMs with few tiles for the SMs split their K loops: INT8 outputs bit-identical,
    FP8 / FP16 within the last bits of the unsplit run.
    """

    def __init__(self, tau_low: float = 0.41, tau_high: float = 1.68, k_split: bool = True):
        self.tau_low = float(tau_low)
        self.tau_high = float(tau_high)
        self.k_split = bool(k_split)
        self.M = 0
        self._epoch = _lib.error_epoch
        self._ws: Optional[torch.Tensor] = None
        self._ws_k = 16
        self.H: Optional[torch.Tensor] = None
        self.route_ids: Optional[torch.Tensor] = None
        self.counts: Optional[torch.Tensor] = None
        self.perm: Optional[torch.Tensor] = None

    def reserve(self, M: int, K: int, device) -> None:
        """Size the workspace for M rows and activations up to width K."""
        self._ws_k = max(self._ws_k, int(K))
        lib = _lib.load()
        need = (lib.ee_gated_workspace_split_bytes if self.k_split else lib.ee_gated_workspace_bytes)(M, self._ws_k)
        device = torch.device(device)
        if self._ws is None or self._ws.numel() < need or self._ws.device != device:
            self._ws = torch.empty(need, dtype=torch.uint8, device=device)
            self.reset_workspace()
            self.H = None  # views of the old workspace are stale

    def reset_workspace(self) -> None:
        """Zero the workspace head (bucket and tile counters, the router's scan state).
        Done at allocation; every kernel of the path leaves the head consistent after a
        clean run, so ``route`` skips the memset.  After ``_lib.device_check`` has found
        a kernel's error word set, the next ``route`` / ``route_entropy`` of every router
        zeroes it again by itself."""
        if self._ws is not None:
            self._ws[: _lib.load().ee_gated_workspace_head_bytes()].zero_()
        self._epoch = _lib.error_epoch

    def _recover(self) -> None:
        if self._epoch != _lib.error_epoch:  # a kernel gave up since this router last routed
            self.reset_workspace()

    def _views(self, M: int) -> None:
        off = (ctypes.c_int64 * 8)()
        call("ee_gated_workspace_layout", M, 0, off)
        ws = self._ws
        self.counts = ws[off[0]:off[0] + 12].view(torch.int32)
        self.perm = ws[off[1]:off[1] + 4 * M].view(torch.int32)
        self.route_ids = ws[off[3]:off[3] + M].view(torch.int8)
        self.H = ws[off[4]:off[4] + 4 * M].view(torch.float32)

    def route(self, logits: torch.Tensor) -> torch.Tensor:
        _require(logits.is_cuda and logits.dim() == 2 and logits.dtype == torch.float16,
                 "logits must be a CUDA fp16 [M, n] tensor")
        if logits.stride(1) != 1:
            logits = logits.contiguous()
        M, n = logits.shape
        self.reserve(M, self._ws_k, logits.device)
        if M != self.M or self.H is None:
            self._views(M)
        self.M = M
        self._recover()
        with torch.cuda.device(logits.device):
            call("ee_gate_rows_keep", logits.data_ptr(), M, n, logits.stride(0), self.tau_low, self.tau_high, None,
                 None, None, self._ws.data_ptr(), self._ws.numel(), _stream())
        return self.route_ids

    def route_entropy(self, H: torch.Tensor) -> torch.Tensor:
        """Route M rows from given entropies (fp32 [M] on the device) instead of logits;
        everything after is the same as after ``route``."""
        _require(H.is_cuda and H.dim() == 1, "H must be a 1-D CUDA tensor")
        H = H.detach().to(torch.float32).contiguous()
        M = H.shape[0]
        self.reserve(M, self._ws_k, H.device)
        if M != self.M or self.H is None:
            self._views(M)
        self.M = M
        self._recover()
        with torch.cuda.device(H.device):
            call("ee_gate_entropies", H.data_ptr(), M, self.tau_low, self.tau_high, None, None, self._ws.data_ptr(),
                 self._ws.numel(), _stream())
        return self.route_ids

    def _check(self, a: torch.Tensor, pack: WeightPack):
        a = _check_act(a)
        M, K = a.shape
        _require(M == self.M, f"routed {self.M} rows but A has {M}")
        _require(K == pack.K, f"K mismatch: a is [{M},{K}], weight is [{pack.K},{pack.N}]")
        _require(self._ws is not None and self._ws.numel() >= _lib.load().ee_gated_workspace_bytes(M, K),
                 "workspace too small for this K: call reserve(M, K, device) before route()")
        return a

    def pack_rows(self, a: torch.Tensor) -> None:
        """Quantise / copy A's rows into the bucket buffers (first half of gated_linear)."""
        a = _check_act(a)
        M, K = a.shape
        _require(M == self.M, f"routed {self.M} rows but A has {M}")
        with torch.cuda.device(a.device):
            call("ee_gated_pack", a.data_ptr(), a.stride(0), M, K, self._ws.data_ptr(), self._ws.numel(), _stream())
        self._packed_k = K

    def gemm_packed(self, pack: WeightPack, out: Optional[torch.Tensor] = None) -> torch.Tensor:
        """Bucketed tcgen05 GEMM over the rows packed by ``pack_rows`` (second half)."""
        M, K = self.M, pack.K
        _require(getattr(self, "_packed_k", None) == K, "pack_rows(A) with A of width K must come first")
        y = out if out is not None else torch.empty(M, pack.N, dtype=torch.float16, device=self._ws.device)
        with torch.cuda.device(y.device):
            call("ee_gated_gemm_packed", M, K, pack.w_i8.data_ptr(), pack.w_e4m3.data_ptr(), pack.w_f16.data_ptr(),
                 pack.scale.data_ptr(), pack.N, y.data_ptr(), y.stride(0), self._ws.data_ptr(), self._ws.numel(),
                 _stream())
        return y

    def swiglu_packed(self, pack: "SwiGLUPack", out: Optional[torch.Tensor] = None) -> torch.Tensor:
        """silu(gate) * up over the rows packed by ``pack_rows``, in one bucketed GEMM with
        the SwiGLU epilogue; the same values as ``silu(gemm_packed(gate)) * gemm_packed(up)``."""
        M, K = self.M, pack.K
        _require(getattr(self, "_packed_k", None) == K, "pack_rows(A) with A of width K must come first")
        y = out if out is not None else torch.empty(M, pack.I, dtype=torch.float16, device=self._ws.device)
        with torch.cuda.device(y.device):
            call("ee_gated_swiglu_packed", M, K, pack.w_i8.data_ptr(), pack.w_e4m3.data_ptr(), pack.w_f16.data_ptr(),
                 pack.scale.data_ptr(), pack.I, y.data_ptr(), y.stride(0), self._ws.data_ptr(), self._ws.numel(),
                 _stream())
        return y

    def gated_linear(self, a: torch.Tensor, pack: WeightPack, out: Optional[torch.Tensor] = None) -> torch.Tensor:
        a = self._check(a, pack)
        self.pack_rows(a)
        return self.gemm_packed(pack, out)


def gated_linear(logits: torch.Tensor, a: torch.Tensor, pack: WeightPack, tau_low: float = 0.41,
                 tau_high: float = 1.68):
    """Entropy-gated linear in one call: returns (Y fp16 [M, N], H fp32 [M],
    route int8 [M], bucket counts int32 [3]) -- the last three are copies."""
    r = EntropyRouter(tau_low, tau_high)
    r.reserve(a.shape[0], a.shape[1], a.device)
    r.route(logits)
    y = r.gated_linear(a, pack)
    return y, r.H.clone(), r.route_ids.clone(), r.counts.clone()


class EntropyDispatchedLinear(nn.Module):
    """nn.Linear stand-in with three precision tiers (EE/python/dispatch.py:103-143).

    Holds the reference's buffers (``weight_int8`` [K, N], ``weight_scale`` [N]) plus
    the K-major operand packs the sm_100a kernels read.
    """

    def __init__(self, in_features: int, out_features: int, bias: bool = False):
        super().__init__()
        self.in_features = in_features
        self.out_features = out_features
        self.register_buffer("weight_int8", None)
        self.register_buffer("weight_scale", None)
        if bias:
            self.register_buffer("bias", None)
        else:
            self.bias = None
        self.pack: Optional[WeightPack] = None

    @classmethod
    def from_linear(cls, linear: nn.Linear) -> "EntropyDispatchedLinear":
        has_bias = linear.bias is not None
        layer = cls(linear.in_features, linear.out_features, bias=has_bias)
        w_int8, w_scale = quantize_weights_int8(linear.weight)
        layer.weight_int8 = w_int8
        layer.weight_scale = w_scale
        layer._pack()
        if has_bias:
            layer.bias = linear.bias.detach().to(torch.float16)
        return layer

    @classmethod
    def from_pack(cls, pack: WeightPack, bias: Optional[torch.Tensor] = None,
                  scale_dtype: torch.dtype = torch.float32) -> "EntropyDispatchedLinear":
        """A routed linear over a ready pack (a weight-pack file), with no quantisation at
        load: ``weight_int8`` [K, N] is a view of the pack's int8 [N, K] and ``weight_scale``
        the pack's scale (as ``scale_dtype``: fp16 for blocks that ``.half()`` converts, as
        build_dispatched_llama does, so the conversion leaves the pack in place)."""
        layer = cls(pack.K, pack.N, bias=bias is not None)
        layer.weight_int8 = pack.w_i8.t()
        layer.weight_scale = pack.scale.to(scale_dtype)
        layer.pack = pack
        w, s = layer.weight_int8, layer.weight_scale
        layer._pack_key = (w.data_ptr(), w._version, w.device, s.data_ptr(), s._version, s.dtype)
        if bias is not None:
            layer.bias = bias.detach().to(torch.float16)
        return layer

    def _pack(self) -> WeightPack:
        """The operand packs of the current buffers.  Rebuilt when a buffer moved or
        changed: ``module.half()`` (as the reference's build_dispatched_llama applies,
        EE/python/dispatch.py:254) turns ``weight_scale`` into fp16, and the reference
        kernels then read those fp16-rounded scales -- so do these packs."""
        w, s = self.weight_int8, self.weight_scale
        key = (w.data_ptr(), w._version, w.device, s.data_ptr(), s._version, s.dtype)
        if self.pack is None or getattr(self, "_pack_key", None) != key:
            self.pack = WeightPack(w, s.to(torch.float32))
            self._pack_key = key
        return self.pack

    def forward(self, x: torch.Tensor, tier: PrecisionTier = PrecisionTier.FP16) -> torch.Tensor:
        orig_shape = x.shape
        x_2d = x.reshape(-1, self.in_features).contiguous().to(torch.float16)
        p = self._pack()
        if tier == PrecisionTier.INT8:
            out = triton_int8_gemm(x_2d, p)
        elif tier == PrecisionTier.FP8:
            out = triton_fp8_gemm(x_2d, p)
        else:
            out = triton_fp16_gemm(x_2d, p)
        if self.bias is not None:
            out = out + self.bias.unsqueeze(0)
        return out.reshape(orig_shape[:-1] + (self.out_features,))

    def forward_gated(self, x: torch.Tensor, router: EntropyRouter) -> torch.Tensor:
        """Per-row routed forward: row i of x runs in the precision the router chose
        for row i (route the logits first with ``router.route``)."""
        orig_shape = x.shape
        x_2d = x.reshape(-1, self.in_features).contiguous().to(torch.float16)
        out = router.gated_linear(x_2d, self._pack())
        if self.bias is not None:
            out = out + self.bias.unsqueeze(0)
        return out.reshape(orig_shape[:-1] + (self.out_features,))

    def extra_repr(self):
        return f"in={self.in_features}, out={self.out_features}, bias={self.bias is not None}"
