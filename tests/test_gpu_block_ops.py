"""The Llama block's elementwise passes on the GPU against transformers' own modules:
the fused residual add + RMSNorm (LlamaRMSNorm, the block's `residual + x`) and the
rotary embedding folded into the flash-attention launch chain (apply_rotary_pos_emb)."""
import pytest
import torch

pytestmark = pytest.mark.gpu


def _norm(d, eps, device, seed):
    from transformers.models.llama.modeling_llama import LlamaRMSNorm

    g = torch.Generator().manual_seed(seed)
    m = LlamaRMSNorm(d, eps=eps)
    with torch.no_grad():
        m.weight.copy_(1.0 + 0.1 * torch.randn(d, generator=g))
    return m.to(device).half()


def _ulps(a, b):
    """fp16 ulp distance (same-sign finite values)."""
    ia, ib = a.view(torch.int16).to(torch.int32), b.view(torch.int16).to(torch.int32)
    return (ia - ib).abs()


@pytest.mark.parametrize("M,d", [(7, 2048), (1000, 4096), (33, 64), (5, 8192), (257, 5632), (16384, 2048)])
def test_rmsnorm_matches_transformers(pkg, cuda, M, d):
    norm = _norm(d, 1e-5, cuda, M + d)
    g = torch.Generator(device=cuda).manual_seed(M * 3 + d)
    x = (torch.randn(M, d, generator=g, device=cuda) * 3.0).half()
    y = pkg.add_rmsnorm(x, norm.weight, norm.variance_epsilon)
    with torch.no_grad():
        want = norm(x)
    torch.cuda.synchronize()
    u = _ulps(y, want)
    # the sum of squares is reduced in another order than torch's: a one-ulp change of the
    # normalised fp16 value can become two after the weight product
    assert int(u.max()) <= 2
    assert (u == 0).float().mean() > 0.99


@pytest.mark.parametrize("M,d", [(64, 2048), (3000, 4096), (5, 1024)])
def test_add_rmsnorm_matches_the_block(pkg, cuda, M, d):
    """s = residual + x (bit-exact: torch's half add) and the post-attention norm of s."""
    norm = _norm(d, 1e-6, cuda, d)
    g = torch.Generator(device=cuda).manual_seed(M + 11)
    x = torch.randn(M, d, generator=g, device=cuda).half()
    res = (torch.randn(M, d, generator=g, device=cuda) * 4.0).half()
    y, s = pkg.add_rmsnorm(x.reshape(1, M, d), norm.weight, norm.variance_epsilon, residual=res.reshape(1, M, d))
    with torch.no_grad():
        s_ref = res + x
        want = norm(s_ref)
    torch.cuda.synchronize()
    assert torch.equal(s.reshape(M, d).view(torch.int16), s_ref.view(torch.int16))
    u = _ulps(y.reshape(M, d), want)
    assert int(u.max()) <= 2
    assert (u == 0).float().mean() > 0.99


def _rotary(d, B, S, theta, device):
    from transformers import LlamaConfig
    from transformers.models.llama.modeling_llama import LlamaRotaryEmbedding

    cfg = LlamaConfig(hidden_size=d * 8, num_attention_heads=8, rope_theta=theta, max_position_embeddings=max(S, 64))
    rot = LlamaRotaryEmbedding(cfg).to(device)
    pos = torch.arange(S, device=device).unsqueeze(0).expand(B, S)
    return rot(torch.empty(1, dtype=torch.float16, device=device), pos)


@pytest.mark.parametrize("B,Hq,Hkv,S,d,fused_qkv", [(2, 8, 2, 200, 64, False), (1, 4, 4, 384, 128, False),
                                                    (2, 32, 4, 256, 64, True), (1, 8, 8, 130, 128, True)])
def test_rope_attention_equals_transformers_rotary(pkg, cuda, B, Hq, Hkv, S, d, fused_qkv):
    """The rotary embedding inside the attention's launch chain gives the same fp16 q / k
    as transformers' apply_rotary_pos_emb: output and row entropies equal bit for bit to
    flash_attention_entropy on the transformers-rotated tensors.  q / k / v either
    separate or column slices of one concatenated projection (row stride > width)."""
    from transformers.models.llama.modeling_llama import apply_rotary_pos_emb

    g = torch.Generator(device=cuda).manual_seed(B * 100 + S + d)
    if fused_qkv:
        qkv = (torch.randn(B, S, (Hq + 2 * Hkv) * d, generator=g, device=cuda) * 1.5).half()
        q, k, v = qkv.split((Hq * d, Hkv * d, Hkv * d), dim=-1)
    else:
        q = (torch.randn(B, S, Hq * d, generator=g, device=cuda) * 1.5).half()
        k = (torch.randn(B, S, Hkv * d, generator=g, device=cuda) * 1.5).half()
        v = torch.randn(B, S, Hkv * d, generator=g, device=cuda).half()
    cos, sin = _rotary(d, B, S, 1e4, cuda)
    out, batch, rows = pkg.flash_attention_rope_entropy(q, k, v, cos, sin, Hq, Hkv, causal=True, return_rows=True)
    q4 = q.reshape(B, S, Hq, d).transpose(1, 2)
    k4 = k.reshape(B, S, Hkv, d).transpose(1, 2)
    v4 = v.reshape(B, S, Hkv, d).transpose(1, 2)
    qr, kr = apply_rotary_pos_emb(q4, k4, cos, sin)
    out_ref, batch_ref, rows_ref = pkg.flash_attention_entropy(qr, kr, v4, causal=True, return_rows=True)
    torch.cuda.synchronize()
    assert pkg._lib.device_check() == 0
    assert torch.equal(out.view(torch.int16), out_ref.view(torch.int16))
    assert torch.equal(rows.view(torch.int32), rows_ref.view(torch.int32))
