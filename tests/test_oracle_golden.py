"""Pins the CPU oracle (oracle/ee_oracle.py) against golden vectors produced by the
reference's own code (tests/golden/make_golden.py).  CPU only."""
import json
import os

import numpy as np
import pytest

from oracle import ee_oracle as orc

GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")


@pytest.fixture(scope="module")
def sm():
    return np.load(os.path.join(GOLDEN, "golden_softmax.npz"))


@pytest.fixture(scope="module")
def gm():
    return np.load(os.path.join(GOLDEN, "golden_gemm.npz"))


GEMM_TAGS = ["m128k256n256", "m64k512n128"]


# ----------------------------------------------------------------- softmax + entropy
@pytest.mark.parametrize("tag,causal", [("r64n1024", False), ("r16n4096", False), ("r128n64c", True),
                                        ("r40n48c", True)])
def test_softmax_entropy_matches_reference_kernel(sm, tag, causal):
    x = sm[f"{tag}_x"]
    n = x.shape[1]
    probs, H = orc.softmax_entropy(x, causal=causal, S=n)
    # reference: fp32 math; the oracle: float64.  1e-4 relative, 1e-6 nats absolute
    # (the reference's fp32 log(Z) rounding when Z ~ 1).
    np.testing.assert_allclose(H, sm[f"{tag}_H"].astype(np.float64), rtol=1e-4, atol=1e-6)
    d = np.abs(probs.astype(np.float64) - sm[f"{tag}_probs"].astype(np.float64))
    ulp = np.spacing(np.abs(sm[f"{tag}_probs"]).astype(np.float16)).astype(np.float64)
    assert np.all(d <= ulp + 1e-12), d.max()


@pytest.mark.parametrize("tag", ["b2h2s64", "b1h2s48"])
def test_fused_softmax_entropy_4d(sm, tag):
    probs, batchH = orc.fused_softmax_entropy_4d(sm[f"{tag}_x"], causal=True)
    np.testing.assert_allclose(batchH, sm[f"{tag}_batchH"].astype(np.float64), rtol=1e-4, atol=1e-6)
    d = np.abs(probs.astype(np.float64) - sm[f"{tag}_probs"].astype(np.float64))
    assert d.max() <= 1e-3


# ----------------------------------------------------------------- quantisation
@pytest.mark.parametrize("tag", GEMM_TAGS)
def test_weight_quantisation_bit_exact(gm, tag):
    q, s = orc.quantize_weights_int8(gm[f"{tag}_W"], div_mode="cpu")
    assert np.array_equal(s.view(np.uint32), gm[f"{tag}_ws"].view(np.uint32))
    assert np.array_equal(q, gm[f"{tag}_wkn"])


@pytest.mark.parametrize("tag", GEMM_TAGS)
def test_weight_quantisation_cuda_semantics_within_one_ulp(gm, tag):
    # torch on CUDA multiplies by fp32(1/127); the scale may differ by one fp32 ulp
    q, s = orc.quantize_weights_int8(gm[f"{tag}_W"], div_mode="cuda")
    ref = gm[f"{tag}_ws"]
    assert np.all(np.abs(s.view(np.int32).astype(np.int64) - ref.view(np.int32).astype(np.int64)) <= 1)
    assert np.all(np.abs(q.astype(np.int32) - gm[f"{tag}_wkn"].astype(np.int32)) <= 1)


@pytest.mark.parametrize("tag", GEMM_TAGS)
def test_activation_quant_int8_bit_exact(gm, tag):
    q, s = orc.quant_rows_int8(gm[f"{tag}_A"], div_mode="cpu")
    assert np.array_equal(s.view(np.uint32), gm[f"{tag}_sa"].view(np.uint32))
    assert np.array_equal(q, gm[f"{tag}_qa"])


@pytest.mark.parametrize("tag", GEMM_TAGS)
def test_activation_scale_fp8_bit_exact(gm, tag):
    _, s = orc.quant_rows_e4m3(gm[f"{tag}_A"], div_mode="cpu")
    assert np.array_equal(s.view(np.uint32), gm[f"{tag}_sa8"].view(np.uint32))


def test_fp16_division_by_scalar_vs_reciprocal_multiply():
    # torch divides an fp16 tensor by a Python scalar on CUDA as x * fp32(1/d), on CPU
    # as x / d.  After rounding to fp16: identical for d = 127 over every finite fp16 x;
    # for d = 448 they differ only where the fp16 result is subnormal (amax < 0.0034).
    x = np.arange(0, 0x7C00, dtype=np.uint16).view(np.float16).astype(np.float32)
    for d in (127.0, 448.0):
        a = (x / np.float32(d)).astype(np.float16)
        b = (x * (np.float32(1.0) / np.float32(d))).astype(np.float16)
        diff = a.view(np.uint16) != b.view(np.uint16)
        if d == 127.0:
            assert not diff.any()
        else:
            assert np.all(np.abs(a[diff].astype(np.float32)) < np.float32(2.0 ** -14))


def test_e4m3_conversion_exhaustive():
    # every fp16 input: RNE, saturating; compared with an independent rule built from
    # the e4m3 value set (ties to the even code)
    import torch

    bits = np.arange(65536, dtype=np.uint32).astype(np.uint16)
    x = bits.view(np.float16)
    finite = np.isfinite(x)
    got = orc.f16_to_e4m3(x[finite])
    t = torch.from_numpy(x[finite].astype(np.float32)).clamp(-448, 448).to(torch.float8_e4m3fn)
    want = t.view(torch.uint8).numpy()
    assert np.array_equal(got, want)
    assert orc.f16_to_e4m3(np.array([np.inf, -np.inf], dtype=np.float16)).tolist() == [0x7E, 0xFE]


# ----------------------------------------------------------------- GEMMs
@pytest.mark.parametrize("tag", GEMM_TAGS)
def test_int8_gemm_bit_exact(gm, tag):
    y = orc.gemm_int8(gm[f"{tag}_qa"], gm[f"{tag}_sa"], gm[f"{tag}_wkn"], gm[f"{tag}_ws"])
    assert np.array_equal(y.view(np.uint16), gm[f"{tag}_y_int8"].view(np.uint16))


@pytest.mark.parametrize("tag", GEMM_TAGS)
def test_int8_launcher_end_to_end_bit_exact(gm, tag):
    y = orc.linear_by_tier(gm[f"{tag}_A"], gm[f"{tag}_wkn"], gm[f"{tag}_ws"], orc.INT8, div_mode="cpu")
    assert np.array_equal(y.view(np.uint16), gm[f"{tag}_y_int8"].view(np.uint16))


def _relf(a, b):
    a = a.astype(np.float64)
    b = b.astype(np.float64)
    ok = np.isfinite(b).all(axis=1)
    return np.linalg.norm(a[ok] - b[ok]) / np.linalg.norm(b[ok]), ok


@pytest.mark.parametrize("tag", GEMM_TAGS)
def test_fp8_gemm(gm, tag):
    y = orc.linear_by_tier(gm[f"{tag}_A"], gm[f"{tag}_wkn"], gm[f"{tag}_ws"], orc.FP8, div_mode="cpu")
    ref = gm[f"{tag}_y_fp8"]
    err, ok = _relf(y, ref)
    assert err < 1e-3, err
    # the all-zero row has scale 0 in the reference: 0 * fp16(1/0) = NaN, as here
    assert np.array_equal(np.isnan(y).all(axis=1), ~ok)


@pytest.mark.parametrize("tag", GEMM_TAGS)
def test_fp16_gemm(gm, tag):
    y = orc.linear_by_tier(gm[f"{tag}_A"], gm[f"{tag}_wkn"], gm[f"{tag}_ws"], orc.FP16)
    err, _ = _relf(y, gm[f"{tag}_y_fp16"])
    assert err < 1e-3, err


# ----------------------------------------------------------------- dispatcher
def test_dispatcher_tiers():
    with open(os.path.join(GOLDEN, "golden_dispatch.json")) as f:
        cases = json.load(f)["cases"]
    for c in cases:
        tiers = [orc.FP16]  # before any submission
        for v in c["submitted"]:
            tiers.append(orc.batch_max_tier(np.atleast_1d(np.array(v, dtype=np.float32)), c["tau_low"],
                                            c["tau_high"]))
        assert tiers == c["tiers"], (c, tiers)


@pytest.mark.parametrize("tag", ["b2s48", "b1s64h", "b3s33"])
def test_attention_entropy_matches_reference_block(tag):
    """The Llama block's router input: the oracle restatement against the entropy the
    reference's own _attention_with_fused_entropy returned on the same probabilities."""
    g = np.load(os.path.join(GOLDEN, "golden_attention.npz"))
    batch, rows = orc.attention_entropy(g[f"{tag}_p"])
    np.testing.assert_allclose(batch, g[f"{tag}_entropy"], rtol=2e-6, atol=1e-7)
    assert rows.shape == g[f"{tag}_p"].shape[:-1]

