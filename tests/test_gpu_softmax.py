"""Fused softmax + entropy (+ route) on the GPU against a float64 restatement of the
reference kernel (EE/python/kernels.py:264-312) computed on the same device."""
import math

import pytest
import torch

pytestmark = pytest.mark.gpu


def _ref(x, causal=False, S=None):
    x = x.double()
    rows, n = x.shape
    if causal:
        q = torch.arange(rows, device=x.device) % S
        mask = torch.arange(n, device=x.device)[None, :] > q[:, None]
        x = x.masked_fill(mask, float("-inf"))
    p = torch.softmax(x, dim=-1)
    logp = torch.log_softmax(x, dim=-1)
    H = -(torch.where(p > 0, p * logp, torch.zeros_like(p))).sum(-1)
    return p, H


def _config1_logits(rows, n, seed, device):
    g = torch.Generator().manual_seed(seed)
    s = torch.exp(torch.empty(rows).uniform_(math.log(0.05), math.log(20.0), generator=g))
    return (torch.randn(rows, n, generator=g) * s[:, None]).to(torch.float16).to(device)


@pytest.mark.parametrize("rows,n", [(64, 256), (33, 512), (17, 1024), (9, 2048), (1024, 4096), (5, 8192),
                                    (3, 16384), (2, 20000), (7, 100)])
def test_entropy_and_probs(pkg, cuda, rows, n):
    x = _config1_logits(rows, n, rows + n, cuda)
    probs, H, _ = pkg.softmax_entropy_rows(x, want_probs=True)
    p_ref, H_ref = _ref(x)
    torch.cuda.synchronize()
    assert torch.allclose(H.double(), H_ref, rtol=1e-4, atol=1e-6), (H.double() - H_ref).abs().max()
    assert (probs.double() - p_ref).abs().max() < 1e-3


@pytest.mark.parametrize("B,Hh,S", [(2, 4, 64), (1, 3, 256), (2, 2, 100)])
def test_fused_softmax_entropy_4d_causal(pkg, cuda, B, Hh, S):
    g = torch.Generator().manual_seed(B * Hh * S)
    x = torch.randn(B, Hh, S, S, generator=g).to(torch.float16).to(cuda)
    probs, per_batch = pkg.fused_softmax_entropy(x, causal=True)
    p_ref, H_ref = _ref(x.reshape(-1, S), causal=True, S=S)
    torch.cuda.synchronize()
    assert (probs.reshape(-1, S).double() - p_ref).abs().max() < 1e-3
    want = H_ref.reshape(B, Hh * S).mean(-1)
    assert torch.allclose(per_batch.double(), want, rtol=1e-4, atol=1e-6)


def test_route_ids(pkg, cuda):
    x = _config1_logits(4096, 4096, 77, cuda)
    tl, th = 0.41, 1.68
    _, H, route = pkg.softmax_entropy_rows(x, want_probs=False, tau_low=tl, tau_high=th)
    _, H_ref = _ref(x)
    want = torch.where(H_ref < tl, 0, torch.where(H_ref < th, 1, 2)).to(torch.int8)
    far = ((H_ref - tl).abs() >= 1e-6) & ((H_ref - th).abs() >= 1e-6)
    torch.cuda.synchronize()
    assert torch.equal(route[far], want[far])


@pytest.mark.parametrize("rows,n", [(1, 8), (3, 64), (257, 1000), (20000, 1024), (9, 2048), (5000, 2048),
                                    (4096, 4096), (10000, 4096), (1, 4096)])
def test_router_rows(pkg, cuda, rows, n):
    """The router's path (entropy + route, no probabilities, no mask): one warp per row,
    rows dealt to a grid that fills the GPU once, several rows per warp at the larger
    counts; near one-hot rows (the exact pass) and rows with ties at the max included."""
    x = _config1_logits(rows, n, rows * 3 + n, cuda)
    if rows >= 3:
        x[0] = 0.0                    # uniform row: n entries at the max
        x[1, :] = -30.0
        x[1, n // 2] = 30.0           # one-hot to fp32 precision
        x[2, :] = -8.0
        x[2, : min(3, n)] = 8.0       # three-way tie at the max, tiny rest
    _, H, route = pkg.softmax_entropy_rows(x, want_probs=False, tau_low=0.41, tau_high=1.68)
    _, H_ref = _ref(x)
    torch.cuda.synchronize()
    assert torch.allclose(H.double(), H_ref, rtol=1e-4, atol=1e-6), (H.double() - H_ref).abs().max()
    want = torch.where(H_ref < 0.41, 0, torch.where(H_ref < 1.68, 1, 2)).to(torch.int8)
    far = ((H_ref - 0.41).abs() >= 1e-6) & ((H_ref - 1.68).abs() >= 1e-6)
    assert torch.equal(route[far], want[far])


def test_router_strided_rows(pkg, cuda):
    """Rows with a stride above n (a column slice of a wider matrix)."""
    x = _config1_logits(700, 3072, 9, cuda)[:, : 2048]
    _, H, _ = pkg.softmax_entropy_rows(x, want_probs=False)
    _, H_ref = _ref(x)
    torch.cuda.synchronize()
    assert torch.allclose(H.double(), H_ref, rtol=1e-4, atol=1e-6)
