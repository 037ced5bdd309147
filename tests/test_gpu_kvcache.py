"""The entropy-tied KV cache (ee_kv_*, EntropyKVCache) against torch on the same data:
the stored codes and scales of every tier bit for bit (INT8 q = rn(x / s), s = amax /
127; e4m3 of x / s, s = amax / 448; fp16 copies), the decode attention over the mixed
cache (fp32 reference of the dequantised keys and values plus the new token) within 2e-3
relative Frobenius for the output and 1e-4 relative for the row entropies, over two
decode steps in a row; a pool without room reports the error word and leaves a hole the
attention skips."""
import math

import pytest
import torch

pytestmark = pytest.mark.gpu


def _dequant(cache, b, n):
    """fp32 K, V [n, kv_heads, d] of sequence b's first n tokens, from the raw arrays."""
    r = cache.raw()
    codes = r["slot"][b, :n].to(torch.int64)
    tier, idx = codes >> 28, codes & 0x0FFFFFFF
    K = torch.empty(n, cache.kv_heads, cache.head_dim, device=codes.device)
    V = torch.empty_like(K)
    for t in (0, 1, 2):
        sel = (tier == t).nonzero().flatten()
        if sel.numel() == 0:
            continue
        i = idx[sel]
        if t == 2:
            K[sel], V[sel] = r["k16"][i].float(), r["v16"][i].float()
            continue
        if t == 0:
            kq, vq = r["k8"][i].view(torch.int8).float(), r["v8"][i].view(torch.int8).float()
        else:
            kq, vq = r["k8"][i].view(torch.float8_e4m3fn).float(), r["v8"][i].view(torch.float8_e4m3fn).float()
        K[sel] = kq * r["k_scale"][i].unsqueeze(-1)
        V[sel] = vq * r["v_scale"][i].unsqueeze(-1)
    return K, V, tier


def _codes_ref(x, t):
    """The cache's codes of rows x [n, d] (fp16) at tier t, and their scale."""
    xf = x.float()
    amax = xf.abs().amax(dim=-1, keepdim=True)
    # IEEE divisions, as the kernel's (torch turns tensor / python-scalar into a multiply)
    s = torch.where(amax > 0, torch.div(amax, torch.full_like(amax, 127.0 if t == 0 else 448.0)),
                    torch.ones_like(amax))
    y = xf * torch.div(torch.ones_like(s), s)
    if t == 0:
        return torch.clamp(torch.round(y), -127, 127).to(torch.int8).view(torch.uint8), s.squeeze(-1)
    return y.to(torch.float8_e4m3fn).view(torch.uint8), s.squeeze(-1)


@pytest.mark.parametrize("d,kv,heads", [(128, 4, 32), (64, 4, 8), (128, 8, 32), (64, 2, 2)])
@torch.no_grad()
def test_kv_cache_codes_and_decode_attention(pkg, cuda, d, kv, heads):
    B, T0, T_max = 3, 300, 512
    g = torch.Generator(device=cuda).manual_seed(d + heads)
    cache = pkg.EntropyKVCache(B, kv, d, T_max, device=cuda)
    k = (torch.randn(B * T0, kv * d, generator=g, device=cuda) * 1.5).half()
    v = torch.randn(B * T0, kv * d, generator=g, device=cuda).half()
    tier = torch.randint(0, 3, (B * T0,), generator=g, device=cuda, dtype=torch.int64).to(torch.int8)
    cache.append(k, v, tier)
    torch.cuda.synchronize()
    assert pkg._lib.device_check() == 0
    assert cache.lengths.tolist() == [T0] * B
    r = cache.raw()
    for b in range(B):
        codes = r["slot"][b, :T0].to(torch.int64)
        assert torch.equal(codes >> 28, tier.view(B, T0)[b].to(torch.int64))
        rows = slice(b * T0, (b + 1) * T0)
        kb, vb = k[rows].view(T0, kv, d), v[rows].view(T0, kv, d)
        idx = codes & 0x0FFFFFFF
        for t in (0, 1):
            sel = (codes >> 28 == t).nonzero().flatten()
            for x, name in ((kb, "k"), (vb, "v")):
                want, s = _codes_ref(x[sel], t)
                assert torch.equal(r[name + "8"][idx[sel]], want), (t, name)
                assert torch.equal(r[name + "_scale"][idx[sel]], s), (t, name)
        sel = (codes >> 28 == 2).nonzero().flatten()
        assert torch.equal(r["k16"][idx[sel]], kb[sel]) and torch.equal(r["v16"][idx[sel]], vb[sel])
    used = cache.pool_used.tolist()
    assert used == [int((tier != 2).sum()), int((tier == 2).sum())]

    scale = d ** -0.5
    G = heads // kv
    for step in range(2):
        q = torch.randn(B, heads * d, generator=g, device=cuda).half()
        k_new = torch.randn(B, kv * d, generator=g, device=cuda).half()
        v_new = torch.randn(B, kv * d, generator=g, device=cuda).half()
        out, H = cache.decode_attention(q, k_new, v_new, scale)
        torch.cuda.synchronize()
        assert pkg._lib.device_check() == 0
        n = T0 + step
        for b in range(B):
            K, V, _ = _dequant(cache, b, n)
            K = torch.cat([K, k_new[b].float().view(1, kv, d)])
            V = torch.cat([V, v_new[b].float().view(1, kv, d)])
            qb = q[b].float().view(kv, G, d)
            s = torch.einsum("hgd,thd->hgt", qb, K) * scale
            p = torch.softmax(s, dim=-1)
            o = torch.einsum("hgt,thd->hgd", p, V).reshape(heads * d)
            ent = -(p * torch.log(p.clamp_min(1e-38))).sum(-1).reshape(heads)
            rel = ((out[b].float() - o).norm() / o.norm()).item()
            assert rel < 2e-3, (step, b, rel)
            torch.testing.assert_close(H[b], ent, rtol=1e-4, atol=1e-5)
        # the new token joins the cache in the tier of its own attention entropy
        t_new = pkg.EntropyRouter(1.0, 3.0)
        t_new.reserve(B, 16, cuda)
        cache.append(k_new, v_new, t_new.route_entropy(H.mean(dim=1)).clone())
        torch.cuda.synchronize()
        assert cache.lengths.tolist() == [T0 + step + 1] * B


@torch.no_grad()
def test_kv_cache_full_pool_reports_and_is_skipped(pkg, cuda):
    B, kv, d = 1, 2, 64
    cache = pkg.EntropyKVCache(B, kv, d, 64, slots8=4, slots16=64, device=cuda)
    g = torch.Generator(device=cuda).manual_seed(9)
    k = torch.randn(8, kv * d, generator=g, device=cuda).half()
    v = torch.randn(8, kv * d, generator=g, device=cuda).half()
    cache.append(k, v, torch.zeros(8, dtype=torch.int8, device=cuda))  # 8 INT8 tokens, room for 4
    torch.cuda.synchronize()
    with pytest.raises(RuntimeError, match="EE_ERR_DEVICE"):
        pkg._lib.device_check()
    codes = cache.raw()["slot"][0, :8]
    assert int((codes >= 0).sum()) == 4 and int((codes == -1).sum()) == 4
    q = torch.randn(1, 2 * kv * d, generator=g, device=cuda).half()
    out, H = cache.decode_attention(q, k[:1], v[:1], d ** -0.5)  # the holes are skipped
    torch.cuda.synchronize()
    assert pkg._lib.device_check() == 0
    assert torch.isfinite(out.float()).all() and torch.isfinite(H).all()
