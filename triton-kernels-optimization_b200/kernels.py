"""The reference's operator surface (EE/python/kernels.py), backed by the sm_100a kernels.

Same names, argument meaning and output dtypes as the reference's launchers; every
call goes through the C ABI of libee_b200.so on torch's current CUDA stream.  The
weight argument keeps the reference's format -- int8 [K, N] plus fp32 scale [N] from
``quantize_weights_int8`` -- and is converted once into the K-major operand packs the
tensor-core kernels read (cached per weight tensor, see ``WeightPack``).
"""
from __future__ import annotations

from collections import OrderedDict

import torch

from . import _lib
from ._lib import call


def _stream() -> int:
    return torch.cuda.current_stream().cuda_stream


def _ptr(t) -> int | None:
    return None if t is None else t.data_ptr()


def _require(cond: bool, msg: str) -> None:
    if not cond:
        raise RuntimeError(msg)


def _check_cuda(t: torch.Tensor, name: str) -> None:
    _require(t.is_cuda, f"{name} must be a CUDA tensor")


class WeightPack:
    """K-major [N, K] operand packs of one INT8-quantised weight.

    Built from the reference's weight format (int8 [K, N] + fp32 scale [N],
    EE/python/dispatch.py:43-48):
      * ``w_i8``   int8  [N, K]  -- the INT8 bucket's B operand
      * ``w_e4m3`` uint8 [N, K]  -- e4m3(fp16(q)), the FP8 bucket's B operand
                                    (EE/python/kernels.py:166)
      * ``w_f16``  fp16  [N, K]  -- fp16(fp16(q) * fp16(s)), the FP16 bucket's B
                                    operand (EE/python/kernels.py:215, :233)
      * ``scale``  fp32  [N]
    """

    def __init__(self, w_int8: torch.Tensor, scale: torch.Tensor):
        _check_cuda(w_int8, "b_int8")
        _require(w_int8.dtype == torch.int8 and w_int8.dim() == 2, "b_int8 must be a 2-D int8 tensor [K, N]")
        _require(scale.dtype == torch.float32 and scale.numel() == w_int8.shape[1], "b_scale must be fp32 [N]")
        w_int8 = w_int8.contiguous()
        K, N = w_int8.shape
        dev = w_int8.device
        self.K, self.N = int(K), int(N)
        self.scale = scale.contiguous().to(dev)
        self.w_i8 = torch.empty(N, K, dtype=torch.int8, device=dev)
        self.w_e4m3 = torch.empty(N, K, dtype=torch.uint8, device=dev)
        self.w_f16 = torch.empty(N, K, dtype=torch.float16, device=dev)
        with torch.cuda.device(dev):
            call("ee_pack_weights", w_int8.data_ptr(), self.scale.data_ptr(), K, N, self.w_i8.data_ptr(),
                 self.w_e4m3.data_ptr(), self.w_f16.data_ptr(), _stream())

    @classmethod
    def from_arrays(cls, w_i8: torch.Tensor, w_e4m3: torch.Tensor, w_f16: torch.Tensor,
                    scale: torch.Tensor) -> "WeightPack":
        """A pack from its four arrays as stored (a weight-pack file): int8, e4m3 codes and
        fp16 [N, K] and the fp32 scale [N], all on one device; nothing is recomputed."""
        N, K = w_i8.shape
        _require(w_i8.dtype == torch.int8 and w_e4m3.dtype == torch.uint8 and w_f16.dtype == torch.float16 and
                 scale.dtype == torch.float32, "pack arrays must be int8 / uint8 / fp16 / fp32")
        _require(w_e4m3.shape == (N, K) and w_f16.shape == (N, K) and scale.shape == (N,), "pack array shapes")
        self = cls.__new__(cls)
        self.K, self.N = int(K), int(N)
        self.w_i8, self.w_e4m3, self.w_f16 = w_i8.contiguous(), w_e4m3.contiguous(), w_f16.contiguous()
        self.scale = scale.contiguous()
        return self

    @classmethod
    def from_weight(cls, weight: torch.Tensor) -> "WeightPack":
        """Quantise an nn.Linear weight [N, K] on the device, then pack it."""
        w_int8, scale = quantize_weights_int8(weight)
        return cls(w_int8, scale)

    def nbytes(self) -> int:
        return sum(t.numel() * t.element_size() for t in (self.w_i8, self.w_e4m3, self.w_f16, self.scale))


class SwiGLUPack:
    """Gate and up weight packs of a gated SwiGLU MLP, interleaved for the fused GEMM
    (``ee_gated_swiglu_packed``): rows 256t .. 256t+127 are gate channels 128t .., the
    next 128 rows the same up channels; ``N`` = 2I rows, ``I`` output channels."""

    def __init__(self, gate: WeightPack, up: WeightPack):
        _require(gate.K == up.K and gate.N == up.N, "gate and up must have the same shape")
        _require(gate.N % 128 == 0, f"the intermediate size ({gate.N}) must be a multiple of 128")
        self.K, self.I, self.N = gate.K, gate.N, 2 * gate.N
        groups = gate.N // 128

        def interleave(a: torch.Tensor, b: torch.Tensor) -> torch.Tensor:
            rest = tuple(a.shape[1:])
            return torch.stack([a.reshape(groups, 128, *rest), b.reshape(groups, 128, *rest)], dim=1) \
                .reshape(2 * gate.N, *rest).contiguous()

        self.w_i8 = interleave(gate.w_i8, up.w_i8)
        self.w_e4m3 = interleave(gate.w_e4m3, up.w_e4m3)
        self.w_f16 = interleave(gate.w_f16, up.w_f16)
        self.scale = interleave(gate.scale, up.scale)


_PACK_CACHE: "OrderedDict[tuple, WeightPack]" = OrderedDict()
_PACK_CACHE_SIZE = 8


def pack_for(b_int8: torch.Tensor, b_scale: torch.Tensor) -> WeightPack:
    """WeightPack of (b_int8, b_scale), cached on the tensors' storage and version."""
    key = (b_int8.data_ptr(), b_int8._version, tuple(b_int8.shape), tuple(b_int8.stride()), b_int8.device,
           b_scale.data_ptr(), b_scale._version)
    pack = _PACK_CACHE.get(key)
    if pack is None:
        pack = WeightPack(b_int8, b_scale)
        _PACK_CACHE[key] = pack
        while len(_PACK_CACHE) > _PACK_CACHE_SIZE:
            _PACK_CACHE.popitem(last=False)
    else:
        _PACK_CACHE.move_to_end(key)
    return pack


def _as_pack(b, b_scale) -> WeightPack:
    return b if isinstance(b, WeightPack) else pack_for(b, b_scale)


def _check_act(a: torch.Tensor) -> torch.Tensor:
    _check_cuda(a, "a")
    _require(a.dim() == 2, "a must be 2-D [M, K]")
    _require(a.dtype == torch.float16, "a must be fp16")
    if a.stride(1) != 1 or a.stride(0) % 8 != 0 or a.data_ptr() % 16 != 0:
        a = a.contiguous()
    return a


def _workspace(nbytes: int, device) -> torch.Tensor:
    return torch.empty(max(int(nbytes), 256), dtype=torch.uint8, device=device)


# ------------------------------------------------------------------------ weights
def quantize_weights_int8(weight: torch.Tensor, div_mode: int = 0):
    """Per-output-channel INT8 quantisation (EE/python/dispatch.py:43-48).

    weight [N, K] (any float dtype; converted to fp16 on the device) ->
    (int8 [K, N], fp32 scale [N]).  ``div_mode`` 0 reproduces torch's CUDA evaluation
    of ``amax / 127.0`` (multiplication by the fp32 reciprocal), 1 its CPU evaluation
    (IEEE division).
    """
    _check_cuda(weight, "weight")
    w = weight.detach()
    _require(w.dim() == 2, "weight must be 2-D [out, in]")
    if w.dtype != torch.float16:
        w = w.to(torch.float16)
    w = w.contiguous()
    N, K = w.shape
    w_kn = torch.empty(K, N, dtype=torch.int8, device=w.device)
    scale = torch.empty(N, dtype=torch.float32, device=w.device)
    with torch.cuda.device(w.device):
        call("ee_quantize_weights_int8", w.data_ptr(), N, K, K, w_kn.data_ptr(), None, scale.data_ptr(),
             int(div_mode), _stream())
    return w_kn, scale


# ------------------------------------------------------------------------ activations
def quant_rows_int8(a: torch.Tensor):
    """Per-row INT8 activation quantisation of the reference's INT8 launcher
    (EE/python/kernels.py:336-338): returns (int8 [M, K], fp32 scale [M])."""
    a = _check_act(a)
    M, K = a.shape
    q = torch.empty(M, K, dtype=torch.int8, device=a.device)
    s = torch.empty(M, dtype=torch.float32, device=a.device)
    with torch.cuda.device(a.device):
        call("ee_quant_rows_int8", a.data_ptr(), M, K, a.stride(0), q.data_ptr(), s.data_ptr(), _stream())
    return q, s


def quant_rows_e4m3(a: torch.Tensor):
    """Per-row e4m3 activation quantisation of the reference's FP8 kernel
    (EE/python/kernels.py:361, :144-160): returns (uint8 e4m3 bytes [M, K], fp32 scale [M])."""
    a = _check_act(a)
    M, K = a.shape
    q = torch.empty(M, K, dtype=torch.uint8, device=a.device)
    s = torch.empty(M, dtype=torch.float32, device=a.device)
    with torch.cuda.device(a.device):
        call("ee_quant_rows_e4m3", a.data_ptr(), M, K, a.stride(0), q.data_ptr(), s.data_ptr(), _stream())
    return q, s


# ------------------------------------------------------------------------ GEMMs
def triton_int8_gemm(a: torch.Tensor, b_int8, b_scale: torch.Tensor | None = None) -> torch.Tensor:
    """fp16 [M, K] x INT8 weight -> fp16 [M, N] (EE/python/kernels.py:330-351).

    Per-row activation quantisation is fused in front of a tcgen05 kind::i8 GEMM with
    an int32 accumulator; y = fp16((fp32(acc) * a_scale[m]) * b_scale[n]).
    ``b_int8`` is the reference's int8 [K, N] (with ``b_scale``) or a WeightPack.
    """
    a = _check_act(a)
    p = _as_pack(b_int8, b_scale)
    M, K = a.shape
    _require(K == p.K, f"K mismatch: a is [{M},{K}], b is [{p.K},{p.N}]")
    y = torch.empty(M, p.N, dtype=torch.float16, device=a.device)
    with torch.cuda.device(a.device):
        nbytes = _lib.load().ee_linear_workspace_bytes(M, K)
        ws = _workspace(nbytes, a.device)
        call("ee_linear_int8", a.data_ptr(), a.stride(0), p.w_i8.data_ptr(), p.scale.data_ptr(), y.data_ptr(), M,
             p.N, K, p.N, ws.data_ptr(), ws.numel(), _stream())
    return y


def triton_fp8_gemm(a: torch.Tensor, b_int8, b_scale: torch.Tensor | None = None) -> torch.Tensor:
    """fp16 [M, K] x weight in e4m3 -> fp16 [M, N] (EE/python/kernels.py:354-373).

    Per-row e4m3 quantisation of a (scale amax/448) is fused in front of a tcgen05
    kind::f8f6f4 GEMM with an fp32 accumulator; y = fp16((acc * a_scale[m]) * b_scale[n]).
    """
    a = _check_act(a)
    p = _as_pack(b_int8, b_scale)
    M, K = a.shape
    _require(K == p.K, f"K mismatch: a is [{M},{K}], b is [{p.K},{p.N}]")
    y = torch.empty(M, p.N, dtype=torch.float16, device=a.device)
    with torch.cuda.device(a.device):
        nbytes = _lib.load().ee_linear_workspace_bytes(M, K)
        ws = _workspace(nbytes, a.device)
        call("ee_linear_fp8", a.data_ptr(), a.stride(0), p.w_e4m3.data_ptr(), p.scale.data_ptr(), y.data_ptr(), M,
             p.N, K, p.N, ws.data_ptr(), ws.numel(), _stream())
    return y


def triton_fp16_gemm(a: torch.Tensor, b_int8, b_scale: torch.Tensor | None = None) -> torch.Tensor:
    """fp16 [M, K] x dequantised fp16 weight -> fp16 [M, N] (EE/python/kernels.py:380-409).

    tcgen05 kind::f16 GEMM with an fp32 accumulator over the weight dequantised as
    the reference does per tile, fp16(fp16(q) * fp16(s)).
    """
    a = _check_act(a)
    p = _as_pack(b_int8, b_scale)
    M, K = a.shape
    _require(K == p.K, f"K mismatch: a is [{M},{K}], b is [{p.K},{p.N}]")
    if a.stride(0) != K:
        a = a.contiguous()
    y = torch.empty(M, p.N, dtype=torch.float16, device=a.device)
    with torch.cuda.device(a.device):
        call("ee_gemm_fp16", a.data_ptr(), p.w_f16.data_ptr(), y.data_ptr(), M, p.N, K, p.N, _stream())
    return y


def linear_f16(x: torch.Tensor, weight: torch.Tensor, out: torch.Tensor | None = None) -> torch.Tensor:
    """fp16 x [M, K] @ weight[N, K]^T -> fp16 [M, N] (nn.Linear without bias) on the
    tcgen05 kind::f16 GEMM with an fp32 accumulator: the Llama block's unrouted
    projections (q / k / v / o of the reference's MLP-only mode)."""
    x = _check_act(x)
    if x.stride(0) != x.shape[1]:
        x = x.contiguous()
    _check_cuda(weight, "weight")
    _require(weight.dtype == torch.float16 and weight.dim() == 2 and weight.shape[1] == x.shape[1],
             "weight must be fp16 [N, K] with K = x.shape[1]")
    w = weight.contiguous()
    M, K = x.shape
    N = w.shape[0]
    y = out if out is not None else torch.empty(M, N, dtype=torch.float16, device=x.device)
    _require(y.shape == (M, N) and y.stride(1) == 1, "out must be fp16 [M, N] rows")
    with torch.cuda.device(x.device):
        call("ee_gemm_fp16", x.data_ptr(), w.data_ptr(), y.data_ptr(), M, N, K, y.stride(0), _stream())
    return y


def head_mean_entropy(rows: torch.Tensor):
    """Router inputs from the attention's row entropies [B, Hq, S] (fp32): per token the
    mean over the heads [B, S], and per batch the mean over heads and positions [B]
    (the reference's entropy_batch, EE/python/dispatch.py:244-245), in one fixed order."""
    _check_cuda(rows, "rows")
    _require(rows.dim() == 3 and rows.dtype == torch.float32, "rows must be fp32 [B, Hq, S]")
    rows = rows.contiguous()
    B, Hq, S = rows.shape
    token = torch.empty(B, S, dtype=torch.float32, device=rows.device)
    batch = torch.empty(B, dtype=torch.float32, device=rows.device)
    with torch.cuda.device(rows.device):
        call("ee_head_mean_entropy", rows.data_ptr(), B, Hq, S, token.data_ptr(), batch.data_ptr(), _stream())
    return token, batch


def gemm_int8_prequant(a_int8: torch.Tensor, b, a_scale: torch.Tensor, b_scale: torch.Tensor | None = None):
    """Pre-quantised INT8 GEMM (the CubinEngine.forward contract, EE/csrc/engine.cpp:106-166)."""
    _check_cuda(a_int8, "a")
    _require(a_int8.dtype == torch.int8, "a must be int8")
    _require(a_scale.dtype == torch.float32, "a_scale must be fp32")
    _require(a_int8.is_contiguous(), "a must be contiguous")
    p = _as_pack(b, b_scale)
    M, K = a_int8.shape
    _require(K == p.K, f"K mismatch: a is [{M},{K}], b is [{p.K},{p.N}]")
    a_scale = a_scale.contiguous()
    y = torch.empty(M, p.N, dtype=torch.float16, device=a_int8.device)
    with torch.cuda.device(a_int8.device):
        call("ee_gemm_int8", a_int8.data_ptr(), a_scale.data_ptr(), p.w_i8.data_ptr(), p.scale.data_ptr(),
             y.data_ptr(), M, p.N, K, p.N, _stream())
    return y


def gemm_accumulators(kind: str, a_q: torch.Tensor, w_nk: torch.Tensor) -> torch.Tensor:
    """Raw tcgen05 accumulators (int32 for 'int8', fp32 for 'fp8' / 'fp16') of
    a_q [M, K] . w_nk [N, K]^T, for verification."""
    M, K = a_q.shape
    N = w_nk.shape[0]
    out = torch.empty(M, N, dtype=torch.int32 if kind == "int8" else torch.float32, device=a_q.device)
    name = {"int8": "ee_gemm_int8_acc", "fp8": "ee_gemm_fp8_acc", "fp16": "ee_gemm_fp16_acc"}[kind]
    with torch.cuda.device(a_q.device):
        call(name, a_q.data_ptr(), w_nk.data_ptr(), out.data_ptr(), M, N, K, _stream())
    return out


# ------------------------------------------------------------------------ softmax + entropy
def softmax_entropy_rows(logits: torch.Tensor, causal: bool = False, S: int | None = None,
                         want_probs: bool = True, tau_low: float | None = None, tau_high: float | None = None):
    """Per-row softmax + entropy of a 2-D fp16 [rows, n] matrix (the reference kernel
    EE/python/kernels.py:264-312 without the 4-D wrapper).

    Returns (probs fp16 [rows, n] or None, entropy fp32 [rows], route int8 [rows] or
    None).  The route (dual-threshold tier per row) is produced when both thresholds
    are given.
    """
    _check_cuda(logits, "logits")
    _require(logits.dim() == 2 and logits.dtype == torch.float16, "logits must be fp16 [rows, n]")
    if logits.stride(1) != 1:
        logits = logits.contiguous()
    rows, n = logits.shape
    H = torch.empty(rows, dtype=torch.float32, device=logits.device)
    probs = torch.empty(rows, n, dtype=torch.float16, device=logits.device) if want_probs else None
    route = None
    if tau_low is not None and tau_high is not None:
        route = torch.empty(rows, dtype=torch.int8, device=logits.device)
    with torch.cuda.device(logits.device):
        call("ee_softmax_entropy", logits.data_ptr(), rows, n, logits.stride(0), int(bool(causal)),
             int(S if S is not None else n), _ptr(probs), n, H.data_ptr(), _ptr(route),
             float(tau_low or 0.0), float(tau_high or 0.0), _stream())
    return probs, H, route


def fused_softmax_entropy(logits: torch.Tensor, causal: bool = True):
    """EE/python/kernels.py:416-453: logits fp16 [B, H, S, S] ->
    (probs fp16 [B, H, S, S], per-batch mean entropy fp32 [B])."""
    _check_cuda(logits, "logits")
    B, Hh, S, S2 = logits.shape
    assert S == S2
    if not logits.is_contiguous():
        logits = logits.contiguous()
    if logits.dtype != torch.float16:
        logits = logits.to(torch.float16)
    probs = torch.empty_like(logits, dtype=torch.float16)
    row_entropies = torch.empty(B * Hh * S, dtype=torch.float32, device=logits.device)
    per_batch = torch.empty(B, dtype=torch.float32, device=logits.device)
    with torch.cuda.device(logits.device):
        call("ee_fused_softmax_entropy_4d", logits.data_ptr(), B, Hh, S, int(bool(causal)), probs.data_ptr(),
             row_entropies.data_ptr(), per_batch.data_ptr(), _stream())
    return probs, per_batch


def attention_entropy(attn_weights: torch.Tensor, return_rows: bool = False):
    """Entropy of attention probabilities as the reference's Llama block computes it
    (EE/python/dispatch.py:243-245): ``-(p * log(p + 1e-10)).sum(-1)`` in fp32, then
    the mean over heads and query positions.

    attn_weights: fp16 or fp32 [B, H, S, S_k] (any leading shape with the batch first;
    the last dim is reduced) -> per-batch mean entropy fp32 [B] (and the per-row
    entropies [B, H, S] when ``return_rows``).
    """
    _check_cuda(attn_weights, "attn_weights")
    _require(attn_weights.dim() >= 2, "attn_weights needs a batch and a key dimension")
    p = attn_weights
    if p.dtype not in (torch.float16, torch.float32):
        p = p.float()
    if p.stride(-1) != 1 or not p.is_contiguous():
        p = p.contiguous()
    B, n = p.shape[0], p.shape[-1]
    rows = p.numel() // n if n else 0
    row_h = torch.empty(p.shape[:-1], dtype=torch.float32, device=p.device)
    batch_h = torch.empty(B, dtype=torch.float32, device=p.device)
    dtype = 1 if p.dtype == torch.float32 else 0
    with torch.cuda.device(p.device):
        call("ee_attention_entropy", p.data_ptr(), dtype, rows, n, n, row_h.data_ptr(), B,
             batch_h.data_ptr() if rows else None, _stream())
    return (batch_h, row_h) if return_rows else batch_h


def flash_attention_entropy(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, causal: bool = True,
                            scale: float | None = None, return_rows: bool = False, return_token: bool = False):
    """Attention with the entropy of every query row in one pass (no [B, H, S, S]
    probabilities): q fp16 [B, Hq, S, d], k / v fp16 [B, Hkv, S, d] (grouped heads),
    d = 64 or 128.  Returns (attn_output fp16 [B, S, Hq, d] -- the layout o_proj reads --,
    per-batch mean entropy fp32 [B]) and, with ``return_rows``, the per-row entropies
    [B, Hq, S], and with ``return_token`` also the per-token mean over heads [B, S]
    (``head_mean_entropy``).  The entropy is -sum p ln p of the softmax of the reference's
    fp16 scores (EE/python/dispatch.py:243-245 computes it from the materialised
    probabilities)."""
    for t, n in ((q, "q"), (k, "k"), (v, "v")):
        _check_cuda(t, n)
        _require(t.dim() == 4 and t.dtype == torch.float16, f"{n} must be fp16 [B, H, S, d]")
    B, Hq, S, d = q.shape
    Hkv = k.shape[1]
    _require(k.shape == (B, Hkv, S, d) and v.shape == k.shape, "k and v must be [B, Hkv, S, d] like q")
    q, k, v = q.contiguous(), k.contiguous(), v.contiguous()
    scale = float(d ** -0.5 if scale is None else scale)
    out = torch.empty(B, S, Hq, d, dtype=torch.float16, device=q.device)
    rows = torch.empty(B, Hq, S, dtype=torch.float32, device=q.device)
    ws = _workspace(_lib.load().ee_attention_workspace_bytes(B, Hkv, S, d), q.device)
    with torch.cuda.device(q.device):
        call("ee_flash_attention_entropy", q.data_ptr(), k.data_ptr(), v.data_ptr(), B, Hq, Hkv, S, d,
             int(bool(causal)), scale, out.data_ptr(), rows.data_ptr(), ws.data_ptr(), ws.numel(), _stream())
    token, batch = head_mean_entropy(rows)
    if return_token:
        return out, batch, rows, token
    return (out, batch, rows) if return_rows else (out, batch)


def flash_attention_rope_entropy(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, cos: torch.Tensor,
                                 sin: torch.Tensor, num_heads: int, num_kv_heads: int, causal: bool = True,
                                 scale: float | None = None, return_rows: bool = False, return_token: bool = False,
                                 exact_entropy: bool = False):
    """flash_attention_entropy on the projections' outputs: q fp16 [B, S, Hq*d], k / v fp16
    [B, S, Hkv*d] (any row stride, unit column stride), cos / sin fp16 [B, S, d] (what
    transformers' LlamaRotaryEmbedding returns).  The rotary embedding is applied in the
    same launch chain with the roundings of transformers' apply_rotary_pos_emb on fp16
    tensors, so the result equals flash_attention_entropy(apply_rotary_pos_emb(...)) bit
    for bit.  Returns what flash_attention_entropy returns.  With ``exact_entropy`` the
    row entropies are the reference's: of the probabilities rounded to fp16 as the eager
    attention returns them (a second tensor-core pass over the keys)."""
    for t, n in ((q, "q"), (k, "k"), (v, "v"), (cos, "cos"), (sin, "sin")):
        _check_cuda(t, n)
        _require(t.dim() == 3 and t.dtype == torch.float16 and t.stride(-1) == 1, f"{n} must be fp16 [B, S, n] rows")
    B, S, _ = q.shape
    Hq, Hkv = int(num_heads), int(num_kv_heads)
    d = q.shape[2] // Hq
    _require(q.shape[2] == Hq * d and k.shape == (B, S, Hkv * d) and v.shape == k.shape, "q / k / v widths")
    _require(cos.shape == (B, S, d) and sin.shape == cos.shape, "cos / sin must be [B, S, d]")
    rows_of = lambda t: t if t.stride(0) == t.stride(1) * S else t.contiguous()  # noqa: E731
    q, k, v, cos, sin = (rows_of(t) for t in (q, k, v, cos, sin))
    scale = float(d ** -0.5 if scale is None else scale)
    out = torch.empty(B, S, Hq, d, dtype=torch.float16, device=q.device)
    rows = torch.empty(B, Hq, S, dtype=torch.float32, device=q.device)
    lib = _lib.load()
    ws_bytes = (lib.ee_attention_exact_workspace_bytes if exact_entropy else lib.ee_attention_rope_workspace_bytes)(
        B, Hq, Hkv, S, d)
    ws = _workspace(ws_bytes, q.device)
    name = "ee_flash_attention_rope_entropy_exact" if exact_entropy else "ee_flash_attention_rope_entropy"
    with torch.cuda.device(q.device):
        call(name, q.data_ptr(), q.stride(1), k.data_ptr(), k.stride(1), v.data_ptr(),
             v.stride(1), cos.data_ptr(), sin.data_ptr(), cos.stride(1), B, Hq, Hkv, S, d, int(bool(causal)), scale,
             out.data_ptr(), rows.data_ptr(), ws.data_ptr(), ws.numel(), _stream())
    token, batch = head_mean_entropy(rows)
    if return_token:
        return out, batch, rows, token
    return (out, batch, rows) if return_rows else (out, batch)


def add_rmsnorm(x: torch.Tensor, weight: torch.Tensor, eps: float, residual: torch.Tensor | None = None):
    """transformers' LlamaRMSNorm (weight, eps) of x, or of fp16(residual + x) when a
    residual is given, in one pass.  Returns y, or (y, s) with s = residual + x."""
    _check_cuda(x, "x")
    _require(x.dtype == torch.float16 and weight.dtype == torch.float16, "x and weight must be fp16")
    d = x.shape[-1]
    x2 = x.reshape(-1, d)
    if x2.stride(1) != 1:
        x2 = x2.contiguous()
    M = x2.shape[0]
    y = torch.empty(M, d, dtype=torch.float16, device=x.device)
    s = None
    r2 = None
    if residual is not None:
        _require(residual.shape == x.shape and residual.dtype == torch.float16, "residual must match x")
        r2 = residual.reshape(-1, d)
        if r2.stride(1) != 1:
            r2 = r2.contiguous()
        s = torch.empty(M, d, dtype=torch.float16, device=x.device)
    w = weight.contiguous()
    with torch.cuda.device(x.device):
        call("ee_add_rmsnorm", x2.data_ptr(), x2.stride(0), r2.data_ptr() if r2 is not None else None,
             r2.stride(0) if r2 is not None else 0, s.data_ptr() if s is not None else None, d,
             w.data_ptr(), float(eps), y.data_ptr(), d, M, d, _stream())
    y = y.reshape(x.shape)
    return y if s is None else (y, s.reshape(x.shape))

