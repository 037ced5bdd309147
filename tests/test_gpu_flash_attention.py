"""Flash attention with online row entropy (ee_flash_attention_entropy) against the
reference's eager attention math on the same inputs: fp16 Q K^T, times the scale, fp16,
causal mask, softmax in fp32, probabilities to fp16, P V, and the entropy
-sum p ln(p + 1e-10) of those fp16 probabilities (EE/python/dispatch.py:243-245)."""
import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu


def _eager(q, k, v, causal, scale):
    B, Hq, S, d = q.shape
    rep = Hq // k.shape[1]
    k = k.repeat_interleave(rep, dim=1)
    v = v.repeat_interleave(rep, dim=1)
    w = torch.matmul(q, k.transpose(2, 3)) * scale  # fp16, as transformers' eager attention
    if causal:
        mask = torch.full((S, S), torch.finfo(torch.float16).min, device=q.device, dtype=torch.float16).triu(1)
        w = w + mask
    p = torch.softmax(w, dim=-1, dtype=torch.float32).to(torch.float16)
    out = torch.matmul(p, v).transpose(1, 2).contiguous()  # [B, S, Hq, d]
    ent = -(p.float() * torch.log(p.float() + 1e-10)).sum(-1)  # [B, Hq, S]
    return out, ent


def _relf(a, b):
    a, b = a.double(), b.double()
    return float((a - b).norm() / b.norm())


@pytest.mark.parametrize("B,Hq,Hkv,S,d,causal", [
    (1, 2, 2, 128, 64, True), (2, 4, 2, 256, 64, True), (1, 4, 1, 384, 128, True),
    (2, 2, 2, 200, 64, True), (1, 2, 2, 256, 128, False), (1, 8, 2, 1024, 64, True)])
def test_matches_eager_attention(pkg, cuda, B, Hq, Hkv, S, d, causal):
    g = torch.Generator(device=cuda).manual_seed(B * 1000 + Hq * 100 + S + d)
    q = (torch.randn(B, Hq, S, d, generator=g, device=cuda) * 1.5).half()
    k = (torch.randn(B, Hkv, S, d, generator=g, device=cuda) * 1.5).half()
    v = torch.randn(B, Hkv, S, d, generator=g, device=cuda).half()
    out, batch, rows = pkg.flash_attention_entropy(q, k, v, causal=causal, return_rows=True)
    torch.cuda.synchronize()
    assert pkg._lib.device_check() == 0
    ref_out, ref_rows = _eager(q, k, v, causal, d ** -0.5)
    assert torch.isfinite(out.float()).all()
    assert _relf(out.float(), ref_out.float()) < 1e-2
    # the reference rounds every probability to fp16 before its entropy; this kernel
    # never materialises them, so the rows agree to that rounding
    np.testing.assert_allclose(rows.cpu().numpy(), ref_rows.cpu().numpy(), rtol=2e-3, atol=2e-3)
    np.testing.assert_allclose(batch.cpu().numpy(), ref_rows.mean(dim=(1, 2)).cpu().numpy(), rtol=1e-3)


@pytest.mark.parametrize("B,Hq,Hkv,S,d,causal,qscale", [
    (1, 2, 1, 1, 64, True, 1.5), (2, 2, 2, 7, 128, True, 1.5), (1, 4, 2, 130, 128, True, 1.5),
    (1, 2, 2, 383, 64, True, 1.5), (1, 2, 1, 300, 64, False, 1.5), (1, 2, 2, 300, 128, False, 1.5),
    (1, 2, 2, 1024, 64, True, 6.0), (1, 2, 1, 1024, 128, True, 6.0), (1, 2, 2, 640, 64, False, 6.0)])
def test_edge_sizes_and_peaked_scores(pkg, cuda, B, Hq, Hkv, S, d, causal, qscale):
    """Sequences shorter than a tile or ending mid-tile (query and key tiles partly past
    the end), non-causal calls, and peaked scores (q scaled up: the row max grows by more
    than 2^8 from one key tile to the next, so the kernel's lazy rescale of O, l and t
    runs) -- each against the eager reference math."""
    g = torch.Generator(device=cuda).manual_seed(S * 7 + d + int(qscale))
    q = (torch.randn(B, Hq, S, d, generator=g, device=cuda) * qscale).half()
    k = (torch.randn(B, Hkv, S, d, generator=g, device=cuda) * 1.5).half()
    v = torch.randn(B, Hkv, S, d, generator=g, device=cuda).half()
    out, batch, rows = pkg.flash_attention_entropy(q, k, v, causal=causal, return_rows=True)
    torch.cuda.synchronize()
    assert pkg._lib.device_check() == 0
    ref_out, ref_rows = _eager(q, k, v, causal, d ** -0.5)
    assert torch.isfinite(out.float()).all()
    assert _relf(out.float(), ref_out.float()) < 1e-2
    np.testing.assert_allclose(rows.cpu().numpy(), ref_rows.cpu().numpy(), rtol=2e-3, atol=2e-3)


def test_argument_checks(pkg, cuda):
    lib = pkg.load_library()
    p = 256
    assert lib.ee_flash_attention_entropy(p, p, p, 1, 3, 2, 128, 64, 1, 0.125, p, p, p, 1 << 20, None) == -1
    assert lib.ee_flash_attention_entropy(p, p, p, 1, 2, 2, 128, 96, 1, 0.125, p, p, p, 1 << 20, None) == -3
