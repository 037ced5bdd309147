"""Entropy-gated linear (route -> per-row quantisation -> bucketed tcgen05 GEMM ->
scatter) and the reference's launchers, against the reference formulas evaluated
with torch on the same device (EE/python/kernels.py:330-409)."""
import math

import pytest
import torch

pytestmark = pytest.mark.gpu


def _inputs(M, n, K, N, seed, device):
    g = torch.Generator().manual_seed(seed)
    s = torch.exp(torch.empty(M).uniform_(math.log(0.05), math.log(20.0), generator=g))
    logits = (torch.randn(M, n, generator=g) * s[:, None]).to(torch.float16)
    a = torch.randn(M, K, generator=g)
    a[torch.rand(M, K, generator=g) < 0.01] *= 20.0
    w = torch.randn(N, K, generator=g) * 0.02
    return logits.to(device), a.to(torch.float16).to(device), w.to(torch.float16).to(device)


def _ref_int8(a, p):
    s = (a.abs().amax(dim=1) / 127.0).clamp(min=1e-8).to(torch.float32)
    q = (a / s[:, None]).to(torch.int8)
    acc = (q.double() @ p.w_i8.double().T).round()
    return ((acc.float() * s[:, None]) * p.scale[None, :]).half()


def _ref_fp8(a, p):
    s = (a.abs().amax(dim=1) / 448.0).clamp(min=1e-12).to(torch.float32)
    inv = (1.0 / s).to(torch.float16)
    a8 = (a * inv[:, None]).clamp(-448, 448).to(torch.float8_e4m3fn)
    w8 = p.w_e4m3.view(torch.float8_e4m3fn)
    acc = a8.double() @ w8.double().T
    return ((acc.float() * s[:, None]) * p.scale[None, :]).half()


def _ref_fp16(a, p):
    return (a.double() @ p.w_f16.double().T).half()


def _relf(got, want):
    return ((got.double() - want.double()).norm() / want.double().norm()).item()


@pytest.mark.parametrize("M,K,N", [(256, 512, 512), (1000, 1024, 776), (1024, 4096, 4096)])
def test_reference_launchers(pkg, cuda, M, K, N):
    _, a, w = _inputs(M, 64, K, N, M + K + N, cuda)
    w_kn, ws = pkg.quantize_weights_int8(w)
    p = pkg.WeightPack(w_kn, ws)
    y8 = pkg.triton_int8_gemm(a, w_kn, ws)
    yf8 = pkg.triton_fp8_gemm(a, w_kn, ws)
    y16 = pkg.triton_fp16_gemm(a, w_kn, ws)
    torch.cuda.synchronize()
    assert torch.equal(y8.view(torch.int16), _ref_int8(a, p).view(torch.int16))
    assert _relf(yf8, _ref_fp8(a, p)) < 1e-2
    assert _relf(y16, _ref_fp16(a, p)) < 1e-2


@pytest.mark.parametrize("M,n,K,N", [(256, 1024, 512, 512), (1024, 4096, 4096, 4096), (333, 256, 1024, 264)])
def test_gated_linear(pkg, cuda, M, n, K, N):
    logits, a, w = _inputs(M, n, K, N, 3 * M + n, cuda)
    w_kn, ws = pkg.quantize_weights_int8(w)
    p = pkg.WeightPack(w_kn, ws)
    y, H, route, counts = pkg.gated_linear(logits, a, p, 0.41, 1.68)
    torch.cuda.synchronize()
    assert pkg._lib.device_check() == 0
    c = counts.cpu().tolist()
    assert c == [int((route == b).sum()) for b in range(3)]
    rows = [torch.nonzero(route == b).flatten() for b in range(3)]
    if rows[0].numel():
        want = _ref_int8(a[rows[0]], p)
        assert torch.equal(y[rows[0]].view(torch.int16), want.view(torch.int16))
    if rows[1].numel():
        assert _relf(y[rows[1]], _ref_fp8(a[rows[1]], p)) < 1e-2
    if rows[2].numel():
        assert _relf(y[rows[2]], _ref_fp16(a[rows[2]], p)) < 1e-2
