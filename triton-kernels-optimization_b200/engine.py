"""Native launchers: the reference's ``CubinEngine`` contract and the CUDA-Graph layer loop.

* ``CubinEngine`` keeps the constructor, ``from_metadata`` and ``forward`` of the
  reference's pybind11 class (EE/csrc/engine.cpp:64-215).  The reference loads a Triton
  sm_89 cubin; here the sm_100a kernels are compiled into libee_b200.so, so the cubin
  path and the tile metadata are accepted for compatibility and validated, and
  ``forward`` launches the tcgen05 INT8 GEMM on the caller's stream.
* ``GatedLayerEngine`` drives the C++ engine of include/ee_b200.h: a fixed list of gated
  layers (routing logits + projections at fixed device addresses) enqueued with no
  host round trip, eagerly or as one CUDA graph recorded once and replayed.
"""
from __future__ import annotations

import ctypes
import json
import os
from typing import Optional, Sequence

import torch

from . import _lib
from ._lib import call
from .kernels import WeightPack, _require, gemm_int8_prequant


class CubinEngine:
    """Reference-compatible INT8 launcher (EE/csrc/engine.cpp:73-104, :106-166)."""

    SUPPORTED = ("gemm_int8_kernel",)

    def __init__(self, cubin_path: Optional[str] = None, func_name: str = "gemm_int8_kernel",
                 shared_mem: int = 49152, num_warps: int = 4, block_m: int = 64, block_n: int = 128):
        if func_name not in self.SUPPORTED:
            raise RuntimeError(f"cuModuleGetFunction failed for '{func_name}': this engine launches the INT8 "
                               "contract only (use triton_fp8_gemm / triton_fp16_gemm for the other tiers)")
        for name, v in (("shared_mem", shared_mem), ("num_warps", num_warps), ("block_m", block_m),
                        ("block_n", block_n)):
            if int(v) <= 0:
                raise RuntimeError(f"{name} must be positive")
        self.cubin_path = cubin_path
        self.func_name = func_name
        self.shared_mem, self.num_warps, self.block_m, self.block_n = shared_mem, num_warps, block_m, block_n
        _lib.load()

    @staticmethod
    def from_metadata(cubin_path: Optional[str], meta_json_path: str,
                      func_name: str = "gemm_int8_kernel") -> "CubinEngine":
        """EE/csrc/engine.cpp:168-199: reads shared / num_warps / BLOCK_M / BLOCK_N."""
        if not os.path.exists(meta_json_path):
            raise RuntimeError(f"Cannot open {meta_json_path}")
        with open(meta_json_path) as f:
            meta = json.load(f)
        for key in ("shared", "num_warps", "BLOCK_M", "BLOCK_N"):
            if key not in meta:
                raise RuntimeError(f"Missing key: {key}")
        return CubinEngine(cubin_path, func_name, int(meta["shared"]), int(meta["num_warps"]),
                           int(meta["BLOCK_M"]), int(meta["BLOCK_N"]))

    def forward(self, a_int8: torch.Tensor, b_int8: torch.Tensor, a_scale: torch.Tensor,
                b_scale: torch.Tensor) -> torch.Tensor:
        """int8 [M, K] (pre-quantised) x int8 [K, N] -> fp16 [M, N] with
        y = fp16((fp32(acc) * a_scale[m]) * b_scale[n])."""
        _require(b_int8.dtype == torch.int8, "b must be int8")
        _require(b_scale.dtype == torch.float32, "b_scale must be fp32")
        _require(b_int8.is_contiguous(), "b must be contiguous")
        _require(a_int8.dim() == 2 and b_int8.dim() == 2 and a_int8.shape[1] == b_int8.shape[0],
                 f"K mismatch: a is {list(a_int8.shape)}, b is {list(b_int8.shape)}")
        return gemm_int8_prequant(a_int8, b_int8, a_scale, b_scale)

    __call__ = forward


class _Projection(ctypes.Structure):
    _fields_ = [("K", ctypes.c_int64), ("N", ctypes.c_int64), ("A", ctypes.c_void_p), ("lda", ctypes.c_int64),
                ("w_i8_nk", ctypes.c_void_p), ("w_e4m3_nk", ctypes.c_void_p), ("w_f16_nk", ctypes.c_void_p),
                ("w_scale", ctypes.c_void_p), ("Y", ctypes.c_void_p), ("ldy", ctypes.c_int64)]


class _Layer(ctypes.Structure):
    _fields_ = [("logits", ctypes.c_void_p), ("n_logits", ctypes.c_int64), ("ld_logits", ctypes.c_int64),
                ("n_proj", ctypes.c_int32), ("proj", ctypes.POINTER(_Projection))]


class GatedLayerEngine:
    """The gated layer loop as one native object.

    ``layers`` is a list of ``(logits, [(A, WeightPack, Y), ...])``: per layer the fp16
    routing logits [rows, n] and its projections (fp16 A [rows, K] in, fp16 Y [rows, N]
    out).  The tensors are referenced, not copied: refill ``logits`` / ``A`` in place and
    call ``launch()`` again.  Every layer routes its own rows per row (tau_low / tau_high)
    on the device.
    """

    def __init__(self, layers: Sequence, tau_low: float = 0.41, tau_high: float = 1.68):
        _require(len(layers) > 0, "need at least one layer")
        rows = layers[0][0].shape[0]
        dev = layers[0][0].device
        self._keep = []  # keeps every tensor the engine points to alive
        self._projs = []
        c_layers = (_Layer * len(layers))()
        for li, (logits, projs) in enumerate(layers):
            _require(logits.is_cuda and logits.dtype == torch.float16 and logits.dim() == 2 and
                     logits.shape[0] == rows and logits.stride(1) == 1, "logits must be fp16 [rows, n], unit stride")
            arr = (_Projection * max(len(projs), 1))()
            for pi, (a, pack, y) in enumerate(projs):
                _require(isinstance(pack, WeightPack), "projections take a WeightPack")
                _require(a.dtype == torch.float16 and a.shape == (rows, pack.K) and a.stride(1) == 1,
                         f"A of layer {li} projection {pi} must be fp16 [{rows}, {pack.K}]")
                _require(y.dtype == torch.float16 and y.shape == (rows, pack.N) and y.stride(1) == 1,
                         f"Y of layer {li} projection {pi} must be fp16 [{rows}, {pack.N}]")
                arr[pi] = _Projection(pack.K, pack.N, a.data_ptr(), a.stride(0), pack.w_i8.data_ptr(),
                                      pack.w_e4m3.data_ptr(), pack.w_f16.data_ptr(), pack.scale.data_ptr(),
                                      y.data_ptr(), y.stride(0))
                self._keep += [a, pack, y]
            self._projs.append(arr)
            c_layers[li] = _Layer(logits.data_ptr(), logits.shape[1], logits.stride(0), len(projs),
                                  ctypes.cast(arr, ctypes.POINTER(_Projection)))
            self._keep.append(logits)
        lib = _lib.load()
        nbytes = lib.ee_engine_workspace_bytes(rows, len(layers), c_layers)
        _require(nbytes > 0, "malformed layer description")
        self.workspace = torch.empty(nbytes, dtype=torch.uint8, device=dev)
        self.rows = rows
        self.device = dev
        self.stream = torch.cuda.Stream(device=dev)  # graphs are recorded on a created stream
        self._handle = ctypes.c_void_p()
        with torch.cuda.device(dev):
            call("ee_engine_create", rows, float(tau_low), float(tau_high), len(layers), c_layers,
                 self.workspace.data_ptr(), self.workspace.numel(), ctypes.byref(self._handle))
        self._layers = c_layers

    def run(self) -> None:
        """Enqueue every layer eagerly on the current stream."""
        with torch.cuda.device(self.device):
            call("ee_engine_run", self._handle, torch.cuda.current_stream(self.device).cuda_stream)

    def capture(self) -> None:
        """Record the loop into a CUDA graph (on the engine's own stream, ordered after
        the caller's current stream)."""
        cur = torch.cuda.current_stream(self.device)
        self.stream.wait_stream(cur)
        with torch.cuda.device(self.device):
            call("ee_engine_capture", self._handle, self.stream.cuda_stream)
        cur.wait_stream(self.stream)
        self._captured = True

    def launch(self) -> None:
        """Replay the recorded graph on the current stream (records it on first use)."""
        if not getattr(self, "_captured", False):
            self.capture()
        with torch.cuda.device(self.device):
            call("ee_engine_launch", self._handle, torch.cuda.current_stream(self.device).cuda_stream)

    def close(self) -> None:
        if getattr(self, "_handle", None) and self._handle.value:
            _lib.load().ee_engine_destroy(self._handle)
            self._handle = ctypes.c_void_p()

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass
