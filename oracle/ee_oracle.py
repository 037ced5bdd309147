"""CPU oracle of the entropy-gated mixed-precision path -- TEST INFRASTRUCTURE ONLY.

A numpy restatement of the reference's algorithm (IqtedarU/triton-kernels-optimization,
``entropy-engine/``; "EE/" below), used only as the checker by tests/, by
``__graft_entry__.smoke()`` and by the CPU-baseline leg of ``bench.py``.  The product
path never imports this module.

Parity pin: tests/test_oracle_golden.py checks this module against golden vectors
produced by running the reference's own code (its Python launchers plus its Triton
kernels under the Triton 3.6 CPU interpreter) -- see tests/golden/make_golden.py.

Number formats:
  * fp16 values are numpy float16; products of two fp16 values are exact in float32,
    so numpy's float16 multiply (float32 compute, one rounding) equals an fp16 multiply.
  * e4m3 values travel as uint8 codes (OCP FP8 E4M3FN); conversion from fp16 is
    round-to-nearest-even with saturation to +-448 (the `.to(tl.float8e4nv)` cast of
    EE/python/kernels.py:160, :166 on sm_89+ hardware).
  * GEMM accumulations run in float64: exact for the INT8 path (|acc| < 2^53); for the
    fp32-accumulating FP8 / FP16 paths the difference from any fp32 order is far
    below the 1e-2 relative Frobenius tolerance the parity tests use.
"""
from __future__ import annotations

import math

import numpy as np

INT8, FP8, FP16 = 0, 1, 2  # EE/python/dispatch.py:32-36 (PrecisionTier)

# --------------------------------------------------------------------------- e4m3


def _e4m3_positive_values() -> np.ndarray:
    """Values of the finite non-negative e4m3 codes 0x00..0x7E (0x7F is NaN)."""
    codes = np.arange(0x7F, dtype=np.int64)
    e = codes >> 3
    m = codes & 7
    sub = m / 8.0 * 2.0 ** -6
    nor = (1.0 + m / 8.0) * np.power(2.0, (e - 7).astype(np.float64))
    return np.where(e == 0, sub, nor)


_E4M3_POS = _e4m3_positive_values()  # increasing, max 448


def _build_f16_to_e4m3_lut() -> np.ndarray:
    bits = np.arange(65536, dtype=np.uint32).astype(np.uint16)
    v = bits.view(np.float16).astype(np.float64)
    sign = (bits >> 15).astype(np.uint8)
    mag = np.abs(v)
    out = np.zeros(65536, dtype=np.uint8)
    nan = np.isnan(v)
    mag_c = np.where(nan, 0.0, np.minimum(mag, 448.0))  # saturate (inf included)
    hi = np.searchsorted(_E4M3_POS, mag_c, side="left")  # first value >= mag
    hi = np.minimum(hi, 0x7E)
    lo = np.maximum(hi - 1, 0)
    d_hi = _E4M3_POS[hi] - mag_c
    d_lo = mag_c - _E4M3_POS[lo]
    pick_hi = (d_hi < d_lo) | ((d_hi == d_lo) & (hi % 2 == 0))
    code = np.where(_E4M3_POS[hi] == mag_c, hi, np.where(pick_hi, hi, lo)).astype(np.uint8)
    out = code | (sign << 7)
    out[nan] = 0x7F | (sign[nan] << 7)
    return out.astype(np.uint8)


_F16_TO_E4M3 = _build_f16_to_e4m3_lut()


def f16_to_e4m3(x: np.ndarray) -> np.ndarray:
    """fp16 -> e4m3 code, RNE with saturation to +-448 (cvt.rn.satfinite semantics)."""
    x = np.asarray(x, dtype=np.float16)
    return _F16_TO_E4M3[x.view(np.uint16)]


def e4m3_to_f64(codes: np.ndarray) -> np.ndarray:
    codes = np.asarray(codes, dtype=np.uint8)
    mag = np.concatenate([_E4M3_POS, [np.nan]])[codes & 0x7F]
    return np.where(codes & 0x80, -mag, mag)


# --------------------------------------------------------------------------- softmax + entropy


def softmax_entropy(x: np.ndarray, causal: bool = False, S: int | None = None):
    """Per-row softmax and Shannon entropy (EE/python/kernels.py:264-312).

    x: fp16 [rows, n].  Causal masking hides column j of row r when j > r % S
    (kernels.py:273, :291-292).  Returns (probs fp16 [rows, n], H float64 [rows]) with
    H = log Z - sum p (x - max) (kernels.py:301-304), evaluated in float64.
    """
    x = np.asarray(x, dtype=np.float16).astype(np.float64)
    rows, n = x.shape
    if causal:
        q = np.arange(rows) % (S if S is not None else n)
        x = np.where(np.arange(n)[None, :] > q[:, None], -np.inf, x)
    m = x.max(axis=1, keepdims=True)
    sh = x - m
    e = np.exp(sh)
    Z = e.sum(axis=1, keepdims=True)
    p = e / Z
    safe = np.where(np.isneginf(sh), 0.0, sh)
    H = np.log(Z[:, 0]) - (p * safe).sum(axis=1)
    return p.astype(np.float16), H


def fused_softmax_entropy_4d(logits: np.ndarray, causal: bool = True):
    """The 4-D surface (EE/python/kernels.py:416-453): [B, H, S, S] fp16 ->
    (probs fp16 [B, H, S, S], per-batch mean entropy [B])."""
    B, Hh, S, S2 = logits.shape
    assert S == S2
    p, H = softmax_entropy(logits.reshape(-1, S), causal=causal, S=S)
    return p.reshape(logits.shape), H.reshape(B, Hh * S).mean(axis=1)


def attention_entropy(p: np.ndarray):
    """Llama-path entropy of attention probabilities (EE/python/dispatch.py:243-245):
    per row ``-sum_j p_j * ln(p_j + 1e-10)`` with p widened to fp32 and the 1e-10 added
    in fp32 (as ``attn_weights.float() + eps``), evaluated in float64; then the mean
    over every axis but the batch (the first) and the last.  Returns (per-batch [B],
    per-row [...]) as float64."""
    p32 = np.asarray(p).astype(np.float32)
    t = (p32 + np.float32(1e-10)).astype(np.float64)
    rows = -(p32.astype(np.float64) * np.log(t)).sum(axis=-1)
    return rows.reshape(rows.shape[0], -1).mean(axis=1), rows


# --------------------------------------------------------------------------- routing


def route(H: np.ndarray, tau_low: float, tau_high: float) -> np.ndarray:
    """Dual-threshold rule per value (EE/python/dispatch.py:74-79): strict `<`,
    compared in double like the reference's Python floats."""
    H = np.asarray(H, dtype=np.float64)
    return np.where(H < tau_low, INT8, np.where(H < tau_high, FP8, FP16)).astype(np.int8)


def batch_max_tier(H: np.ndarray, tau_low: float, tau_high: float) -> int:
    """The reference dispatcher's granularity: the rule on the batch max of the fp32
    entropies (EE/python/dispatch.py:63-82)."""
    val = float(np.asarray(H, dtype=np.float32).max())
    return int(route(np.array([val]), tau_low, tau_high)[0])


def compaction(route_ids: np.ndarray):
    """Stable grouping of rows by bucket: (perm [M], counts [3]); positions run over
    INT8 rows, then FP8 rows, then FP16 rows, each in increasing row order."""
    route_ids = np.asarray(route_ids)
    perm = np.concatenate([np.nonzero(route_ids == b)[0] for b in (INT8, FP8, FP16)]).astype(np.int32)
    counts = np.array([(route_ids == b).sum() for b in (INT8, FP8, FP16)], dtype=np.int32)
    return perm, counts


# --------------------------------------------------------------------------- quantisation


def quantize_weights_int8(W: np.ndarray, div_mode: str = "cuda"):
    """EE/python/dispatch.py:43-48.  W [N, K] -> (int8 [K, N], fp32 scale [N]).

    s = clamp(amax_k |W| / 127, min=1e-8) in fp32, q = clamp(round_half_even(W / s),
    -127, 127).  torch evaluates ``amax / 127.0`` on CUDA as amax * fp32(1/127)
    (``div_mode='cuda'``, the reference's deployment) and on CPU as an IEEE division
    (``div_mode='cpu'``); ``W / s`` is an IEEE division in both.
    """
    w = np.asarray(W).astype(np.float32).T  # [K, N]
    amax = np.abs(w).max(axis=0)
    if div_mode == "cuda":
        s = (amax * np.float32(np.float32(1.0) / np.float32(127.0))).astype(np.float32)
    elif div_mode == "cpu":
        s = (amax / np.float32(127.0)).astype(np.float32)
    else:
        raise ValueError(div_mode)
    s = np.maximum(s, np.float32(1e-8))
    q = np.clip(np.rint(w / s[None, :]), -127, 127).astype(np.int8)
    return np.ascontiguousarray(q), s


def _row_scale_f16(a: np.ndarray, denom: float, div_mode: str = "cuda") -> np.ndarray:
    """fp16(amax_k |a| / denom) clamped in fp16 (a no-op: the clamp bounds 1e-8 and
    1e-12 round below the smallest fp16 subnormal), widened to fp32
    (EE/python/kernels.py:336, :361).  torch evaluates the division by the Python
    scalar on CUDA as amax * fp32(1/denom) (``div_mode='cuda'``, the reference's
    deployment) and on CPU as an IEEE division (``div_mode='cpu'``); for denom 448 the
    two differ when the fp16 result is subnormal."""
    amax = np.abs(np.asarray(a, dtype=np.float16)).max(axis=1).astype(np.float32)
    if div_mode == "cuda":
        q = amax * (np.float32(1.0) / np.float32(denom))
    elif div_mode == "cpu":
        q = amax / np.float32(denom)
    else:
        raise ValueError(div_mode)
    return q.astype(np.float32).astype(np.float16).astype(np.float32)


def quant_rows_int8(a: np.ndarray, div_mode: str = "cuda"):
    """EE/python/kernels.py:336-338: s = fp32(fp16(amax/127)), q = trunc(fp32(a) / s)
    (IEEE division, conversion truncates toward zero).  Returns (int8 [M, K], s [M])."""
    s = _row_scale_f16(a, 127.0, div_mode)
    with np.errstate(divide="ignore", invalid="ignore"):
        qf = np.asarray(a, dtype=np.float16).astype(np.float32) / s[:, None]
    qf = np.where(np.isnan(qf), 0.0, qf)
    q = np.clip(np.trunc(qf), -128, 127).astype(np.int8)
    return q, s


def quant_rows_e4m3(a: np.ndarray, div_mode: str = "cuda"):
    """EE/python/kernels.py:361 (scale) and :144, :157-160 (in-kernel conversion):
    s = fp32(fp16(amax/448)), inv = fp16(1/s), a8 = e4m3(fp16(a * inv)).
    Returns (e4m3 codes [M, K], s [M])."""
    s = _row_scale_f16(a, 448.0, div_mode)
    with np.errstate(divide="ignore"):
        inv = (np.float32(1.0) / s).astype(np.float16)
    with np.errstate(invalid="ignore"):
        prod = (np.asarray(a, dtype=np.float16) * inv[:, None]).astype(np.float16)
    return f16_to_e4m3(prod), s


# --------------------------------------------------------------------------- GEMMs


def gemm_int8(q_a: np.ndarray, s_a: np.ndarray, w_kn: np.ndarray, s_w: np.ndarray, return_acc: bool = False):
    """EE/python/kernels.py:52-110: int32 acc = q_a . w_kn (exact),
    y = fp16((fp32(acc) * s_a[m]) * s_w[n]) evaluated left to right (:104)."""
    acc = np.asarray(q_a, dtype=np.float64) @ np.asarray(w_kn, dtype=np.float64)
    acc32 = acc.astype(np.float32)  # round-to-nearest, as the kernel's int32 -> fp32
    y = ((acc32 * np.asarray(s_a, np.float32)[:, None]) * np.asarray(s_w, np.float32)[None, :]).astype(np.float16)
    if return_acc:
        return y, acc.astype(np.int64)
    return y


def weight_e4m3(w_kn: np.ndarray) -> np.ndarray:
    """e4m3(fp16(q)): the FP8 kernel's B operand (EE/python/kernels.py:166)."""
    return f16_to_e4m3(np.asarray(w_kn, dtype=np.int8).astype(np.float16))


def weight_f16(w_kn: np.ndarray, s_w: np.ndarray) -> np.ndarray:
    """fp16(fp16(q) * fp16(s)): the FP16 kernel's B operand (EE/python/kernels.py:215, :233)."""
    qh = np.asarray(w_kn, dtype=np.int8).astype(np.float16)
    return (qh * np.asarray(s_w, np.float32).astype(np.float16)[None, :]).astype(np.float16)


def gemm_fp8(a: np.ndarray, w_kn: np.ndarray, s_w: np.ndarray, div_mode: str = "cuda"):
    """Full reference FP8 path (EE/python/kernels.py:354-373, :120-180):
    y = fp16((acc * s_a[m]) * s_w[n]), acc = e4m3(a) . e4m3(w)."""
    a8, s_a = quant_rows_e4m3(a, div_mode)
    acc = e4m3_to_f64(a8) @ e4m3_to_f64(weight_e4m3(w_kn))
    return ((acc.astype(np.float32) * s_a[:, None]) * np.asarray(s_w, np.float32)[None, :]).astype(np.float16)


def gemm_fp16(a: np.ndarray, w_kn: np.ndarray, s_w: np.ndarray):
    """Reference FP16 (W8A16) path (EE/python/kernels.py:380-409, :194-246)."""
    acc = np.asarray(a, dtype=np.float16).astype(np.float64) @ weight_f16(w_kn, s_w).astype(np.float64)
    return acc.astype(np.float32).astype(np.float16)


def linear_by_tier(a: np.ndarray, w_kn: np.ndarray, s_w: np.ndarray, tier: int, div_mode: str = "cuda"):
    """EntropyDispatchedLinear.forward for one tier on the whole tensor
    (EE/python/dispatch.py:126-140, bias omitted)."""
    if tier == INT8:
        q, s = quant_rows_int8(a, div_mode)
        return gemm_int8(q, s, w_kn, s_w)
    if tier == FP8:
        return gemm_fp8(a, w_kn, s_w, div_mode)
    return gemm_fp16(a, w_kn, s_w)


# --------------------------------------------------------------------------- gated linear


def gated_linear(logits: np.ndarray, A: np.ndarray, w_kn: np.ndarray, s_w: np.ndarray, tau_low: float,
                 tau_high: float, rows: np.ndarray | None = None):
    """Per-row entropy-gated linear: Y[i] = linear_by_tier(A, W, route[i])[i].

    Row independence of the per-row scales (EE/python/kernels.py:336, :361) and of the
    per-channel weight scales (EE/python/dispatch.py:45-46) makes this equal to running
    each reference launcher on the whole A and selecting the rows of its tier.
    ``rows`` restricts Y to a subset of rows (the others stay zero) so full-size
    checks stay cheap.
    """
    _, H = softmax_entropy(logits)
    r = route(H, tau_low, tau_high)
    M = A.shape[0]
    N = np.asarray(w_kn).shape[1]
    Y = np.zeros((M, N), dtype=np.float16)
    sel = np.arange(M) if rows is None else np.asarray(rows)
    for b in (INT8, FP8, FP16):
        idx = sel[r[sel] == b]
        if idx.size:
            Y[idx] = linear_by_tier(A[idx], w_kn, s_w, b)
    perm, counts = compaction(r)
    return {"H": H, "route": r, "Y": Y, "perm": perm, "counts": counts}


# --------------------------------------------------------------------------- inputs


def config1_logits(M: int, n: int, rng: np.random.Generator) -> np.ndarray:
    """Config-1 law: row i ~ N(0, s_i^2), s_i log-uniform in [0.05, 20], fp16."""
    s = np.exp(rng.uniform(math.log(0.05), math.log(20.0), size=M))
    return (rng.standard_normal((M, n)) * s[:, None]).astype(np.float16)


def activations(M: int, K: int, rng: np.random.Generator, outliers: bool = False) -> np.ndarray:
    """A ~ N(0, 1) fp16; with ``outliers`` 1% of the entries (Bernoulli) scaled x20 (config 2)."""
    a = rng.standard_normal((M, K))
    if outliers:
        a = np.where(rng.random((M, K)) < 0.01, a * 20.0, a)
    return a.astype(np.float16)


def make_gating_inputs(M: int, n: int, K: int, N: int, seed: int, outliers: bool = False) -> dict:
    """Seeded synthetic inputs of the gated step: logits [M, n] (config-1 law),
    A [M, K] ~ N(0,1), W [N, K] ~ N(0, 0.02) (nn.Linear layout), all fp16."""
    rng = np.random.default_rng(seed)
    logits = config1_logits(M, n, rng)
    A = activations(M, K, rng, outliers)
    W = (rng.standard_normal((N, K)) * 0.02).astype(np.float16)
    return {"logits": logits, "A": A, "W": W}
