"""Entropy-tied KV-cache compression (the reference's listed next step, README "Work In
Progress": "dynamic KV-Cache compression tied to the entropy metric"; it has no code).

Every cached token keeps its keys and values at the precision of its entropy tier --
the dual-threshold route ids of the linears (0 INT8, 1 FP8-e4m3, 2 FP16) -- in two slot
pools (8-bit codes with an fp32 scale per token and KV head, and fp16), and the decode
attention reads the mixed cache directly (include/ee_b200.h, ``ee_kv_*``).  A prompt's
tokens take the tiers their prefill attention entropies route them to; a decoded token
the tier of its own decode-step entropy (``decode_attention`` returns it).
"""
from __future__ import annotations

import ctypes
from typing import Optional

import torch

from . import _lib
from ._lib import call
from .kernels import _require, _stream


class _KvCacheC(ctypes.Structure):
    _fields_ = [("batch", ctypes.c_int64), ("kv_heads", ctypes.c_int64), ("head_dim", ctypes.c_int64),
                ("max_tokens", ctypes.c_int64), ("slots8", ctypes.c_int64), ("slots16", ctypes.c_int64),
                ("k8", ctypes.c_void_p), ("v8", ctypes.c_void_p), ("k16", ctypes.c_void_p), ("v16", ctypes.c_void_p),
                ("k_scale", ctypes.c_void_p), ("v_scale", ctypes.c_void_p), ("slot", ctypes.c_void_p),
                ("length", ctypes.c_void_p), ("pool_used", ctypes.c_void_p)]


class EntropyKVCache:
    """A KV cache for ``batch`` sequences of up to ``max_tokens`` tokens with ``kv_heads``
    heads of ``head_dim`` (64 or 128).  ``slots8`` / ``slots16``: token slots of the 8-bit
    and fp16 pools shared by all sequences (default: room for every token in either)."""

    def __init__(self, batch: int, kv_heads: int, head_dim: int, max_tokens: int, slots8: Optional[int] = None,
                 slots16: Optional[int] = None, device="cuda"):
        self.batch, self.kv_heads, self.head_dim, self.max_tokens = int(batch), int(kv_heads), int(head_dim), int(max_tokens)
        self.slots8 = int(batch * max_tokens if slots8 is None else slots8)
        self.slots16 = int(batch * max_tokens if slots16 is None else slots16)
        lib = _lib.load()
        nbytes = lib.ee_kv_cache_bytes(self.batch, self.kv_heads, self.head_dim, self.max_tokens, self.slots8,
                                       self.slots16)
        _require(nbytes > 0, "unsupported KV-cache shape (head_dim 64 or 128)")
        self.device = torch.device(device)
        self.memory = torch.empty(nbytes, dtype=torch.uint8, device=self.device)
        self.c = _KvCacheC()
        with torch.cuda.device(self.device):
            call("ee_kv_cache_init", ctypes.byref(self.c), self.memory.data_ptr(), nbytes, self.batch, self.kv_heads,
                 self.head_dim, self.max_tokens, self.slots8, self.slots16, _stream())
        self._ws: Optional[torch.Tensor] = None

    def _view(self, ptr: int, n: int, dtype) -> torch.Tensor:
        off = ptr - self.memory.data_ptr()
        size = torch.tensor([], dtype=dtype).element_size()
        return self.memory[off:off + n * size].view(dtype)

    @property
    def lengths(self) -> torch.Tensor:
        return self._view(self.c.length, self.batch, torch.int32)

    @property
    def pool_used(self) -> torch.Tensor:
        return self._view(self.c.pool_used, 2, torch.int32)

    def raw(self) -> dict:
        """The cache's arrays as tensors (views): k8 / v8 [slots8, kv_heads, d] uint8,
        k16 / v16 [slots16, kv_heads, d] fp16, k_scale / v_scale [slots8, kv_heads],
        slot [batch, max_tokens] int32 ((tier << 28) | index)."""
        h, d = self.kv_heads, self.head_dim
        return {"k8": self._view(self.c.k8, self.slots8 * h * d, torch.uint8).view(self.slots8, h, d),
                "v8": self._view(self.c.v8, self.slots8 * h * d, torch.uint8).view(self.slots8, h, d),
                "k16": self._view(self.c.k16, self.slots16 * h * d, torch.float16).view(self.slots16, h, d),
                "v16": self._view(self.c.v16, self.slots16 * h * d, torch.float16).view(self.slots16, h, d),
                "k_scale": self._view(self.c.k_scale, self.slots8 * h, torch.float32).view(self.slots8, h),
                "v_scale": self._view(self.c.v_scale, self.slots8 * h, torch.float32).view(self.slots8, h),
                "slot": self._view(self.c.slot, self.batch * self.max_tokens, torch.int32).view(self.batch,
                                                                                               self.max_tokens)}

    def append(self, k_rows: torch.Tensor, v_rows: torch.Tensor, tier: torch.Tensor) -> None:
        """Append T tokens to every sequence: k_rows / v_rows fp16 [batch * T, kv_heads * d]
        (K after the rotary embedding), tier int8 [batch * T] (route ids)."""
        _require(k_rows.dtype == torch.float16 and v_rows.dtype == torch.float16, "K / V rows must be fp16")
        _require(k_rows.dim() == 2 and k_rows.shape == v_rows.shape and k_rows.shape[0] % self.batch == 0,
                 "K / V rows must be [batch * T, kv_heads * head_dim]")
        _require(k_rows.stride(1) == 1 and v_rows.stride(1) == 1, "K / V rows need unit column stride")
        t_new = k_rows.shape[0] // self.batch
        tier = tier.to(torch.int8).contiguous()
        _require(tier.numel() == k_rows.shape[0], "one tier per row")
        with torch.cuda.device(self.device):
            call("ee_kv_append", ctypes.byref(self.c), k_rows.data_ptr(), k_rows.stride(0), v_rows.data_ptr(),
                 v_rows.stride(0), tier.data_ptr(), t_new, _stream())

    def decode_attention(self, q: torch.Tensor, k_new: torch.Tensor, v_new: torch.Tensor, scale: float,
                         out: Optional[torch.Tensor] = None):
        """One decode step: q fp16 [batch, heads * d] against every sequence's cached
        tokens and its own k_new / v_new [batch, kv_heads * d] (not yet appended).
        Returns (out fp16 [batch, heads * d], H fp32 [batch, heads])."""
        B = self.batch
        heads = q.shape[1] // self.head_dim
        _require(q.dtype == torch.float16 and q.shape == (B, heads * self.head_dim), "q must be fp16 [batch, heads * d]")
        _require(k_new.shape == (B, self.kv_heads * self.head_dim) and v_new.shape == k_new.shape and
                 k_new.stride(0) == v_new.stride(0), "k_new / v_new must be [batch, kv_heads * d] with one row stride")
        y = out if out is not None else torch.empty_like(q)
        H = torch.empty(B, heads, dtype=torch.float32, device=q.device)
        lib = _lib.load()
        need = lib.ee_kv_decode_workspace_bytes(ctypes.byref(self.c), heads)
        if self._ws is None or self._ws.numel() < need:
            self._ws = torch.empty(need, dtype=torch.uint8, device=self.device)
        with torch.cuda.device(self.device):
            call("ee_kv_decode_attention", ctypes.byref(self.c), q.data_ptr(), q.stride(0), heads, k_new.data_ptr(),
                 v_new.data_ptr(), k_new.stride(0), float(scale), y.data_ptr(), y.stride(0), H.data_ptr(),
                 self._ws.data_ptr(), self._ws.numel(), _stream())
        return y, H

    def bytes_per_token(self, tier: int) -> int:
        """Cache bytes one token takes (keys and values of every KV head, with scales)."""
        row = self.kv_heads * self.head_dim
        return 4 * row if tier == 2 else 2 * row + 8 * self.kv_heads
