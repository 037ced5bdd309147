"""Native launchers: the reference's ``CubinEngine`` contract and the CUDA-Graph layer loop.

* ``CubinEngine`` keeps the constructor, ``from_metadata`` and ``forward`` of the
  reference's pybind11 class (EE/csrc/engine.cpp:64-215).  The reference loads a Triton
  sm_89 cubin; here the sm_100a kernels are compiled into libee_b200.so, so the cubin
  path and the tile metadata are accepted for compatibility and validated, and
  ``forward`` launches the tcgen05 INT8 GEMM on the caller's stream.
* ``GatedLayerEngine`` drives the C++ engine of include/ee_b200.h: a fixed list of gated
  layers (routing logits + projections at fixed device addresses) enqueued with no
  host round trip, eagerly or as one CUDA graph recorded once and replayed.
* ``DecoderEngine`` drives the C++ decoder-stack engine (``ee_decoder_*``): the whole
  Llama decoder stack of ``EntropyDispatchedLlamaBlock`` layers -- norms, projections,
  rotary flash attention with row entropies, per-token or batch-max routing, fused
  SwiGLU MLP -- for one batch shape, as one CUDA graph per forward.
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


class _WeightPackC(ctypes.Structure):
    _fields_ = [("w_i8", ctypes.c_void_p), ("w_e4m3", ctypes.c_void_p), ("w_f16", ctypes.c_void_p),
                ("scale", ctypes.c_void_p)]


class _DecoderLayerC(ctypes.Structure):
    _fields_ = [("input_norm", ctypes.c_void_p), ("post_norm", ctypes.c_void_p), ("qkv_f16", ctypes.c_void_p),
                ("o_f16", ctypes.c_void_p), ("qkv", _WeightPackC), ("o", _WeightPackC), ("gate_up", _WeightPackC),
                ("down", _WeightPackC)]


class _DecoderConfigC(ctypes.Structure):
    _fields_ = [("batch", ctypes.c_int64), ("seq", ctypes.c_int64), ("hidden", ctypes.c_int64),
                ("heads", ctypes.c_int64), ("kv_heads", ctypes.c_int64), ("head_dim", ctypes.c_int64),
                ("intermediate", ctypes.c_int64), ("rms_eps", ctypes.c_float), ("attn_scale", ctypes.c_float),
                ("tau_low", ctypes.c_double), ("tau_high", ctypes.c_double), ("routing", ctypes.c_int32),
                ("route_all", ctypes.c_int32), ("exact_entropy", ctypes.c_int32)]


def _pack_c(p) -> _WeightPackC:
    return _WeightPackC(p.w_i8.data_ptr(), p.w_e4m3.data_ptr(), p.w_f16.data_ptr(), p.scale.data_ptr())


class DecoderEngine:
    """The decoder stack of a Llama-architecture model as one native object (the
    reference's per-layer Python loop, EE/python/quality_eval.py:133-141, with every step
    on the device).

    ``blocks`` are ``EntropyDispatchedLlamaBlock`` layers built with ``attention="flash"``
    (their weight packs, norms, attention weights and entropy mode are used in place); ``final_norm``
    the model's last RMSNorm weight; ``position_embeddings`` the (cos, sin) tables of the
    rotary embedding for [batch, seq] positions (fp16 [batch, seq, head_dim], what
    transformers' rotary module returns).  ``routing`` / ``route_all`` as the blocks'.
    ``forward(hidden)`` copies fp16 [batch, seq, hidden] into the engine's input buffer
    and replays the recorded graph; the result (after the final norm) is ``self.output``
    and the last block's output (before it) ``self.residual``.  ``layer_counts`` [layers,
    3] holds each layer's MLP INT8 / FP8 / FP16 row counts of the latest forward.
    """

    def __init__(self, blocks: Sequence, final_norm: torch.Tensor, position_embeddings, batch: int, seq: int,
                 tau_low: float = 0.41, tau_high: float = 1.68, routing: str = "token", route_all: bool = False):
        _require(len(blocks) > 0, "need at least one block")
        _require(routing in ("token", "batch"), "routing must be 'token' or 'batch'")
        b0 = blocks[0]
        attn = b0.self_attn
        dev = final_norm.device
        hidden = b0.input_layernorm.weight.numel()
        d = attn.head_dim
        heads = b0._qkv_split[0] // d
        kv = b0._qkv_split[1] // d
        inter = b0.down_proj.in_features
        eps = float(b0.input_layernorm.variance_epsilon)
        self.batch, self.seq, self.hidden = int(batch), int(seq), int(hidden)
        M = self.batch * self.seq
        cfg = _DecoderConfigC(self.batch, self.seq, hidden, heads, kv, d, inter, eps, float(attn.scaling),
                              float(tau_low), float(tau_high), 0 if routing == "token" else 1, int(bool(route_all)),
                              int(bool(b0.exact_entropy)))
        self._keep = []
        layers = (_DecoderLayerC * len(blocks))()
        for i, blk in enumerate(blocks):
            _require(blk.attention == "flash", "DecoderEngine needs blocks built with attention='flash'")
            _require(blk.exact_entropy == b0.exact_entropy, "every block must use the same entropy mode")
            _require(float(blk.input_layernorm.variance_epsilon) == eps and
                     float(blk.post_attention_layernorm.variance_epsilon) == eps, "every RMSNorm must share eps")
            gu = blk.swiglu_pack()
            _require(gu is not None, "the intermediate size must be a multiple of 128")
            w_in = blk.input_layernorm.weight.detach().to(torch.float16).contiguous()
            w_post = blk.post_attention_layernorm.weight.detach().to(torch.float16).contiguous()
            down = blk.down_proj._pack()
            L = _DecoderLayerC()
            L.input_norm, L.post_norm = w_in.data_ptr(), w_post.data_ptr()
            L.gate_up, L.down = _pack_c(gu), _pack_c(down)
            keep = [w_in, w_post, gu, down]
            if route_all:
                qp, op = blk.qkv_proj._pack(), blk.o_proj._pack()
                L.qkv, L.o = _pack_c(qp), _pack_c(op)
                keep += [qp, op]
            else:
                wq = blk.qkv_weight()
                wo = blk.self_attn.o_proj.weight.detach().to(torch.float16).contiguous()
                L.qkv_f16, L.o_f16 = wq.data_ptr(), wo.data_ptr()
                keep += [wq, wo]
            layers[i] = L
            self._keep += keep
        cos, sin = position_embeddings
        self.cos = cos.to(torch.float16).reshape(M, d).contiguous()
        self.sin = sin.to(torch.float16).reshape(M, d).contiguous()
        self.final_norm = final_norm.detach().to(torch.float16).contiguous()
        self.layer_counts = torch.zeros(len(blocks), 3, dtype=torch.int32, device=dev)
        lib = _lib.load()
        nbytes = lib.ee_decoder_workspace_bytes(ctypes.byref(cfg))
        _require(nbytes > 0, "unsupported decoder shape")
        self.workspace = torch.empty(nbytes, dtype=torch.uint8, device=dev)
        self.input = torch.empty(M, hidden, dtype=torch.float16, device=dev)
        self.output = torch.empty(M, hidden, dtype=torch.float16, device=dev)
        self.residual = torch.empty(M, hidden, dtype=torch.float16, device=dev)
        self.device = dev
        self.stream = torch.cuda.Stream(device=dev)  # graphs are recorded on a created stream
        self._cfg, self._layers = cfg, layers
        self._handle = ctypes.c_void_p()
        with torch.cuda.device(dev):
            call("ee_decoder_create", ctypes.byref(cfg), len(blocks), layers, self.final_norm.data_ptr(),
                 self.cos.data_ptr(), self.sin.data_ptr(), self.layer_counts.data_ptr(), self.workspace.data_ptr(),
                 self.workspace.numel(), ctypes.byref(self._handle))
        self._captured = False

    @classmethod
    def from_model(cls, model, batch: int, seq: int, tau_low: float = 0.41, tau_high: float = 1.68,
                   routing: str = "token", route_all: bool = False, exact_entropy: bool = False) -> "DecoderEngine":
        """Engine over every decoder layer of a transformers Llama model (LlamaForCausalLM
        or LlamaModel, fp16 on the device): the layers are wrapped as the reference's
        build_dispatched_llama does (EE/python/dispatch.py:250-259), with flash attention;
        positions 0 .. seq - 1 in every sequence.  ``self.blocks`` keeps the wrapped layers."""
        from .llama import build_dispatched_llama

        base = model.model if hasattr(model, "model") else model
        wrap = model
        if not hasattr(model, "model"):
            wrap = torch.nn.Module()
            wrap.model = base
        blocks, _ = build_dispatched_llama(wrap, tau_low, tau_high, routing=routing, attention="flash",
                                           route_all=route_all, exact_entropy=exact_entropy)
        dev = base.norm.weight.device
        pos = torch.arange(seq, device=dev).unsqueeze(0).expand(batch, seq)
        probe = torch.empty(batch, seq, base.norm.weight.numel(), dtype=torch.float16, device=dev)
        with torch.no_grad():
            pe = base.rotary_emb(probe, pos)
        eng = cls(blocks, base.norm.weight, pe, batch, seq, tau_low, tau_high, routing=routing, route_all=route_all)
        eng.blocks = blocks
        return eng

    def run(self, hidden: Optional[torch.Tensor] = None) -> torch.Tensor:
        """One eager forward on the current stream (reads ``hidden`` in place when given,
        else the input buffer); returns the output buffer."""
        x = self.input if hidden is None else hidden
        _require(x.dtype == torch.float16 and x.is_contiguous() and x.numel() == self.input.numel(),
                 "hidden must be contiguous fp16 [batch, seq, hidden]")
        with torch.cuda.device(self.device):
            call("ee_decoder_run", self._handle, x.data_ptr(), self.output.data_ptr(), self.residual.data_ptr(),
                 torch.cuda.current_stream(self.device).cuda_stream)
        return self.output

    def capture(self) -> None:
        """Record one forward over the engine's buffers into a CUDA graph (on the engine's
        own stream, ordered after the caller's current stream)."""
        cur = torch.cuda.current_stream(self.device)
        self.stream.wait_stream(cur)
        with torch.cuda.device(self.device):
            call("ee_decoder_capture", self._handle, self.input.data_ptr(), self.output.data_ptr(),
                 self.residual.data_ptr(), self.stream.cuda_stream)
        cur.wait_stream(self.stream)
        self._captured = True

    def launch(self) -> None:
        """Replay the recorded forward on the current stream (records it on first use)."""
        if not self._captured:
            self.capture()
        with torch.cuda.device(self.device):
            call("ee_decoder_launch", self._handle, torch.cuda.current_stream(self.device).cuda_stream)

    def forward(self, hidden: torch.Tensor) -> torch.Tensor:
        """hidden fp16 [batch, seq, hidden] -> the final-norm output (a view of the
        engine's output buffer, valid until the next forward)."""
        self.input.view_as(hidden).copy_(hidden)
        self.launch()
        return self.output.view(hidden.shape)

    __call__ = forward

    def close(self) -> None:
        if getattr(self, "_handle", None) and self._handle.value:
            _lib.load().ee_decoder_destroy(self._handle)
            self._handle = ctypes.c_void_p()

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass
