"""Parity of the sm_100a path (through the C ABI) with the CPU oracle, which is pinned to
the reference's own outputs (tests/test_oracle_golden.py).

Bars: route ids, bucket compaction and int32 / INT8 outputs
bit-exact (rows within 1e-6 of a threshold excluded and counted); entropy within 1e-4
relative (plus 1e-6 nats absolute for near-zero entropies); FP8 / FP16 outputs within 1e-2
relative Frobenius error.  Full Llama-3-8B sizes are checked on sampled rows (rows are
independent) and through size-independent properties.
"""
import os

import numpy as np
import pytest
import torch

from oracle import ee_oracle as orc

pytestmark = pytest.mark.gpu

GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")
TAU = (0.41, 1.68)


def _relf(got, want):
    got = np.asarray(got, dtype=np.float64)
    want = np.asarray(want, dtype=np.float64)
    return float(np.linalg.norm(got - want) / max(np.linalg.norm(want), 1e-300))


def _far(H):
    H = np.asarray(H, dtype=np.float64)
    return (np.abs(H - TAU[0]) >= 1e-6) & (np.abs(H - TAU[1]) >= 1e-6)


def _dev(x, cuda):
    return torch.from_numpy(np.ascontiguousarray(x)).to(cuda)


# ----------------------------------------------------------------------- golden fixtures
@pytest.mark.parametrize("tag", ["m128k256n256", "m64k512n128"])
def test_gemm_launchers_against_reference_goldens(pkg, cuda, tag):
    g = np.load(os.path.join(GOLDEN, "golden_gemm.npz"))
    a = _dev(g[f"{tag}_A"], cuda)
    w_kn = _dev(g[f"{tag}_wkn"], cuda)
    w_s = _dev(g[f"{tag}_ws"], cuda)
    y8 = pkg.triton_int8_gemm(a, w_kn, w_s).cpu().numpy()
    yf8 = pkg.triton_fp8_gemm(a, w_kn, w_s).cpu().numpy()
    y16 = pkg.triton_fp16_gemm(a, w_kn, w_s).cpu().numpy()
    assert np.array_equal(y8.view(np.uint16), g[f"{tag}_y_int8"].view(np.uint16))
    ref8 = g[f"{tag}_y_fp8"]
    ok = np.isfinite(ref8).all(axis=1)  # the reference's all-zero row is NaN in FP8 ...
    assert np.isnan(yf8[~ok]).all()  # ... and here too
    assert _relf(yf8[ok], ref8[ok]) < 1e-2
    assert _relf(y16, g[f"{tag}_y_fp16"]) < 1e-2
    q, s = pkg.quant_rows_int8(a)
    assert np.array_equal(q.cpu().numpy(), g[f"{tag}_qa"])
    assert np.array_equal(s.cpu().numpy().view(np.uint32), g[f"{tag}_sa"].view(np.uint32))


def test_weight_quantisation_against_reference_goldens(pkg, cuda):
    g = np.load(os.path.join(GOLDEN, "golden_gemm.npz"))
    for tag in ("m128k256n256", "m64k512n128"):
        w_kn, w_s = pkg.quantize_weights_int8(_dev(g[f"{tag}_W"], cuda), div_mode=1)  # torch-on-CPU division
        assert np.array_equal(w_kn.cpu().numpy(), g[f"{tag}_wkn"])
        assert np.array_equal(w_s.cpu().numpy().view(np.uint32), g[f"{tag}_ws"].view(np.uint32))
        w_kn_c, w_s_c = pkg.quantize_weights_int8(_dev(g[f"{tag}_W"], cuda), div_mode=0)  # torch-on-CUDA
        q_o, s_o = orc.quantize_weights_int8(g[f"{tag}_W"], div_mode="cuda")
        assert np.array_equal(w_kn_c.cpu().numpy(), q_o)
        assert np.array_equal(w_s_c.cpu().numpy().view(np.uint32), s_o.view(np.uint32))


@pytest.mark.parametrize("tag,causal", [("r64n1024", False), ("r16n4096", False), ("r128n64c", True),
                                        ("r40n48c", True)])
def test_softmax_entropy_against_reference_goldens(pkg, cuda, tag, causal):
    g = np.load(os.path.join(GOLDEN, "golden_softmax.npz"))
    x = _dev(g[f"{tag}_x"], cuda)
    n = x.shape[1]
    probs, H, _ = pkg.softmax_entropy_rows(x, causal=causal, S=n, want_probs=True)
    np.testing.assert_allclose(H.cpu().numpy(), g[f"{tag}_H"], rtol=1e-4, atol=1e-6)
    assert np.abs(probs.cpu().numpy().astype(np.float64) - g[f"{tag}_probs"].astype(np.float64)).max() <= 1e-3


@pytest.mark.parametrize("tag", ["b2h2s64", "b1h2s48"])
def test_4d_surface_against_reference_goldens(pkg, cuda, tag):
    g = np.load(os.path.join(GOLDEN, "golden_softmax.npz"))
    probs, batch_h = pkg.fused_softmax_entropy(_dev(g[f"{tag}_x"], cuda), causal=True)
    np.testing.assert_allclose(batch_h.cpu().numpy(), g[f"{tag}_batchH"], rtol=1e-4, atol=1e-6)
    assert np.abs(probs.cpu().numpy().astype(np.float64) - g[f"{tag}_probs"].astype(np.float64)).max() <= 1e-3


@pytest.mark.parametrize("tag", ["b2s48", "b1s64h", "b3s33"])
def test_attention_entropy_against_reference_goldens(pkg, cuda, tag):
    """Probabilities produced by a transformers LlamaAttention inside the reference's
    own block code, and the entropy that code returned (fp16 and fp32; n = 33 takes
    the unvectorised path)."""
    g = np.load(os.path.join(GOLDEN, "golden_attention.npz"))
    p = g[f"{tag}_p"]
    batch, rows = pkg.attention_entropy(_dev(p, cuda), return_rows=True)
    np.testing.assert_allclose(batch.cpu().numpy(), g[f"{tag}_entropy"], rtol=1e-4, atol=1e-6)
    _, rows_ref = orc.attention_entropy(p)
    np.testing.assert_allclose(rows.cpu().numpy(), rows_ref, rtol=1e-4, atol=1e-6)


@pytest.mark.parametrize("dtype", [torch.float16, torch.float32])
def test_attention_entropy_config4_shape(pkg, cuda, dtype):
    """[B, H, S, S] causal attention probabilities at a config-4-like size."""
    B, Hh, S = 2, 8, 512
    g = torch.Generator(device=cuda).manual_seed(44)
    scores = torch.randn(B, Hh, S, S, generator=g, device=cuda) * 3.0
    scores = scores.masked_fill(torch.ones(S, S, dtype=torch.bool, device=cuda).triu(1), float("-inf"))
    p = torch.softmax(scores, dim=-1).to(dtype)
    batch, rows = pkg.attention_entropy(p, return_rows=True)
    want_b, want_r = orc.attention_entropy(p.cpu().numpy())
    np.testing.assert_allclose(batch.cpu().numpy(), want_b, rtol=1e-4)
    np.testing.assert_allclose(rows.cpu().numpy(), want_r, rtol=1e-4, atol=1e-6)
    # the reference's own torch expression on the same tensor
    ref = -(p.float() * torch.log(p.float() + 1e-10)).sum(dim=-1).mean(dim=(1, 2))
    np.testing.assert_allclose(batch.cpu().numpy(), ref.cpu().numpy(), rtol=1e-4)


# ----------------------------------------------------------------------- config 1 (gating step)
def test_config1_gated_step_against_oracle(pkg, cuda):
    inp = orc.make_gating_inputs(M=1024, n=4096, K=4096, N=4096, seed=101)
    w_kn, w_s = pkg.quantize_weights_int8(_dev(inp["W"], cuda))
    pack = pkg.WeightPack(w_kn, w_s)
    y, H, route, counts = pkg.gated_linear(_dev(inp["logits"], cuda), _dev(inp["A"], cuda), pack, *TAU)
    torch.cuda.synchronize()
    ref = orc.gated_linear(inp["logits"], inp["A"], w_kn.cpu().numpy(), w_s.cpu().numpy(), *TAU)
    H, route, y = H.cpu().numpy(), route.cpu().numpy(), y.cpu().numpy()
    np.testing.assert_allclose(H, ref["H"], rtol=1e-4, atol=1e-6)
    far = _far(ref["H"])
    assert np.array_equal(route[far], ref["route"][far]), "route ids"
    if far.all():
        assert np.array_equal(counts.cpu().numpy(), ref["counts"])
    for b in range(3):
        rows = np.nonzero(far & (ref["route"] == b))[0]
        if rows.size == 0:
            continue
        if b == orc.INT8:
            assert np.array_equal(y[rows].view(np.uint16), ref["Y"][rows].view(np.uint16)), "INT8 rows bit-exact"
        else:
            assert _relf(y[rows], ref["Y"][rows]) < 1e-2


def test_compaction_is_the_stable_bucket_order(pkg, cuda):
    inp = orc.make_gating_inputs(M=3000, n=2048, K=64, N=64, seed=5)
    r = pkg.EntropyRouter(*TAU)
    r.reserve(3000, 64, cuda)
    r.route(_dev(inp["logits"], cuda))
    r.pack_rows(_dev(inp["A"], cuda))  # places the rows: writes perm
    torch.cuda.synchronize()
    route = r.route_ids.cpu().numpy()
    perm_ref, counts_ref = orc.compaction(route)
    assert np.array_equal(r.counts.cpu().numpy(), counts_ref)
    assert np.array_equal(r.perm.cpu().numpy(), perm_ref)


# ----------------------------------------------------------------------- config 2 (standalone, outliers)
def test_config2_int8_and_fp8_against_oracle(pkg, cuda):
    rng = np.random.default_rng(202)
    a = orc.activations(1024, 4096, rng, outliers=True)
    W = (rng.standard_normal((4096, 4096)) * 0.02).astype(np.float16)
    w_kn, w_s = pkg.quantize_weights_int8(_dev(W, cuda))
    wk, ws = w_kn.cpu().numpy(), w_s.cpu().numpy()
    ad = _dev(a, cuda)
    y8 = pkg.triton_int8_gemm(ad, w_kn, w_s).cpu().numpy()
    yf8 = pkg.triton_fp8_gemm(ad, w_kn, w_s).cpu().numpy()
    y16 = pkg.triton_fp16_gemm(ad, w_kn, w_s).cpu().numpy()
    rows = np.arange(0, 1024, 7)  # sampled rows keep the float64 oracle to seconds
    assert np.array_equal(y8[rows].view(np.uint16), orc.linear_by_tier(a[rows], wk, ws, orc.INT8).view(np.uint16))
    assert _relf(yf8[rows], orc.linear_by_tier(a[rows], wk, ws, orc.FP8)) < 1e-2
    assert _relf(y16[rows], orc.linear_by_tier(a[rows], wk, ws, orc.FP16)) < 1e-2


# ----------------------------------------------------------------------- config 3 (Llama-3-8B shapes)
@pytest.mark.parametrize("M", [16, 128, 1024, 4096])
@pytest.mark.parametrize("K,N", [(4096, 4096), (4096, 14336), (14336, 4096)])
def test_config3_llama3_shapes_sampled_rows(pkg, cuda, M, K, N):
    rng = np.random.default_rng(M + K + N)
    logits = orc.config1_logits(M, 4096, rng)
    a = orc.activations(M, K, rng, outliers=True)
    g = torch.Generator(device=cuda).manual_seed(K * 31 + N)
    W = (torch.randn(N, K, generator=g, device=cuda) * 0.02).half()
    w_kn, w_s = pkg.quantize_weights_int8(W)
    pack = pkg.WeightPack(w_kn, w_s)
    y, H, route, _ = pkg.gated_linear(_dev(logits, cuda), _dev(a, cuda), pack, *TAU)
    torch.cuda.synchronize()
    assert pkg._lib.device_check() == 0
    rows = np.unique(np.linspace(0, M - 1, num=min(M, 24)).astype(int))
    ref = orc.gated_linear(logits, a, w_kn.cpu().numpy(), w_s.cpu().numpy(), *TAU, rows=rows)
    y, route = y.cpu().numpy(), route.cpu().numpy()
    far = _far(ref["H"])
    assert np.array_equal(route[far], ref["route"][far])
    for b in range(3):
        sel = rows[far[rows] & (ref["route"][rows] == b)]
        if sel.size == 0:
            continue
        if b == orc.INT8:
            assert np.array_equal(y[sel].view(np.uint16), ref["Y"][sel].view(np.uint16))
        else:
            assert _relf(y[sel], ref["Y"][sel]) < 1e-2


# ----------------------------------------------------------------------- size-independent properties
def test_rows_are_independent_of_their_batch(pkg, cuda):
    """Permuting the rows (logits and activations together) permutes the output rows
    bit for bit: routing, bucket placement and tile position never change a row."""
    M, n, K, N = 4096, 4096, 4096, 14336
    inp = orc.make_gating_inputs(M=M, n=n, K=K, N=16, seed=9)
    g = torch.Generator(device=cuda).manual_seed(99)
    W = (torch.randn(N, K, generator=g, device=cuda) * 0.02).half()
    pack = pkg.WeightPack(*pkg.quantize_weights_int8(W))
    logits, a = _dev(inp["logits"], cuda), _dev(inp["A"], cuda)
    y1, _, r1, _ = pkg.gated_linear(logits, a, pack, *TAU)
    p = torch.randperm(M, generator=torch.Generator().manual_seed(1)).to(cuda)
    y2, _, r2, _ = pkg.gated_linear(logits[p].contiguous(), a[p].contiguous(), pack, *TAU)
    torch.cuda.synchronize()
    assert torch.equal(r2, r1[p])
    assert torch.equal(y2.view(torch.int16), y1[p].view(torch.int16))


def test_step_is_deterministic(pkg, cuda):
    inp = orc.make_gating_inputs(M=2048, n=4096, K=4096, N=4096, seed=13)
    pack = pkg.WeightPack(*pkg.quantize_weights_int8(_dev(inp["W"], cuda)))
    logits, a = _dev(inp["logits"], cuda), _dev(inp["A"], cuda)
    outs = [pkg.gated_linear(logits, a, pack, *TAU)[0] for _ in range(3)]
    torch.cuda.synchronize()
    assert all(torch.equal(o.view(torch.int16), outs[0].view(torch.int16)) for o in outs[1:])


# ----------------------------------------------------------------------- edge cases
def test_single_bucket_extremes(pkg, cuda):
    """tau below every entropy: every row FP16; tau above every entropy: every row INT8."""
    inp = orc.make_gating_inputs(M=300, n=512, K=256, N=128, seed=21)
    w_kn, w_s = pkg.quantize_weights_int8(_dev(inp["W"], cuda))
    pack = pkg.WeightPack(w_kn, w_s)
    for tl, th, bucket in [(-1.0, -0.5, orc.FP16), (100.0, 200.0, orc.INT8), (-1.0, 100.0, orc.FP8)]:
        y, _, route, counts = pkg.gated_linear(_dev(inp["logits"], cuda), _dev(inp["A"], cuda), pack, tl, th)
        torch.cuda.synchronize()
        assert (route.cpu().numpy() == bucket).all()
        assert counts.cpu().tolist()[bucket] == 300
        want = orc.linear_by_tier(inp["A"], w_kn.cpu().numpy(), w_s.cpu().numpy(), bucket)
        got = y.cpu().numpy()
        if bucket == orc.INT8:
            assert np.array_equal(got.view(np.uint16), want.view(np.uint16))
        else:
            assert _relf(got, want) < 1e-2


def test_tiny_and_empty_inputs(pkg, cuda):
    inp = orc.make_gating_inputs(M=1, n=8, K=16, N=8, seed=3)
    w_kn, w_s = pkg.quantize_weights_int8(_dev(inp["W"], cuda))
    pack = pkg.WeightPack(w_kn, w_s)
    y, H, route, _ = pkg.gated_linear(_dev(inp["logits"], cuda), _dev(inp["A"], cuda), pack, *TAU)
    ref = orc.gated_linear(inp["logits"], inp["A"], w_kn.cpu().numpy(), w_s.cpu().numpy(), *TAU)
    torch.cuda.synchronize()
    np.testing.assert_allclose(H.cpu().numpy(), ref["H"], rtol=1e-4, atol=1e-6)
    if ref["route"][0] == orc.INT8:
        assert np.array_equal(y.cpu().numpy().view(np.uint16), ref["Y"].view(np.uint16))
    else:
        assert _relf(y.cpu().numpy(), ref["Y"]) < 1e-2
    empty = torch.empty(0, 16, dtype=torch.float16, device=cuda)
    assert pkg.triton_int8_gemm(empty, w_kn, w_s).shape == (0, 8)


def test_all_zero_rows_follow_the_reference(pkg, cuda):
    """An all-zero activation row has scale 0 in the reference: INT8 gives 0, FP8 NaN
    (0 * fp16(1/0)), FP16 gives 0 -- the same here."""
    a = np.zeros((4, 64), dtype=np.float16)
    a[1] = 1.0
    W = (np.random.default_rng(0).standard_normal((32, 64)) * 0.02).astype(np.float16)
    w_kn, w_s = pkg.quantize_weights_int8(_dev(W, cuda))
    ad = _dev(a, cuda)
    y8 = pkg.triton_int8_gemm(ad, w_kn, w_s).cpu().numpy()
    yf8 = pkg.triton_fp8_gemm(ad, w_kn, w_s).cpu().numpy()
    y16 = pkg.triton_fp16_gemm(ad, w_kn, w_s).cpu().numpy()
    for r in (0, 2, 3):
        assert (y8[r] == 0).all() and np.isnan(yf8[r]).all() and (y16[r] == 0).all()
    assert np.isfinite(yf8[1]).all()


@pytest.mark.parametrize("M,n", [(16, 4096), (17, 1024), (300, 64), (50000, 512), (4096, 4096)])
def test_router_bucket_scan(pkg, cuda, M, n):
    """The router fast path's bucket scan (a one-block launch chained after the router):
    one chunk, a ragged last chunk, many chunks per scan thread, and the bench's shape;
    twice in a row on the same workspace, the second without the header memset."""
    inp = orc.make_gating_inputs(M=M, n=n, K=16, N=16, seed=M + n)
    r = pkg.EntropyRouter(*TAU)
    r.reserve(M, 16, cuda)
    x = _dev(inp["logits"], cuda)
    for _ in range(2):
        r.route(x)
        r.pack_rows(_dev(inp["A"], cuda))
        torch.cuda.synchronize()
        assert pkg._lib.device_check() == 0
        route = r.route_ids.cpu().numpy()
        perm_ref, counts_ref = orc.compaction(route)
        assert np.array_equal(r.counts.cpu().numpy(), counts_ref)
        assert np.array_equal(r.perm.cpu().numpy(), perm_ref)


def test_int8_row_quantisation_exhaustive(pkg, cuda):
    """q = trunc(x / s) with the reference's IEEE division, against the oracle bit for
    bit, over every positive fp16 x up to each row's abs-max and the exact multiples
    n * s (integer quotients: the case a rounded product could miss), for abs-max values
    across the whole fp16 range (subnormal scales included)."""
    bits = np.arange(0x0001, 0x7C00, dtype=np.uint16)  # every positive finite fp16
    allv = bits.view(np.float16).astype(np.float32)
    rows = []
    for e in range(-14, 16):
        for frac in (1.0, 1.125, 1.5, 1.875, 1.99):
            amax = np.float16(2.0 ** e * frac)
            if not np.isfinite(amax) or amax == 0:
                continue
            s = np.float32(np.float16(np.float32(amax) * (np.float32(1.0) / np.float32(127.0))))
            cand = allv[allv <= np.float32(amax)]
            mult = (np.arange(1, 128, dtype=np.float32) * s).astype(np.float16).astype(np.float32)
            mult = mult[(mult <= np.float32(amax)) & (mult > 0)]
            pick = np.concatenate([mult, cand[np.linspace(0, cand.size - 1, 4096 - 1 - mult.size).astype(int)]])
            row = np.concatenate([[np.float32(amax)], pick])[:4096]
            sign = np.where(np.arange(row.size) % 3 == 1, -1.0, 1.0).astype(np.float32)
            sign[0] = 1.0
            rows.append((row * sign).astype(np.float16))
    a = np.stack(rows)
    q, s = pkg.quant_rows_int8(_dev(a, cuda))
    q_ref, s_ref = orc.quant_rows_int8(a)
    assert np.array_equal(s.cpu().numpy().view(np.uint32), s_ref.view(np.uint32))
    assert np.array_equal(q.cpu().numpy(), q_ref)
