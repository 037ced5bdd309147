"""Per-token routes from the flash-attention entropies against the reference's eager
path on the same inputs.

The reference's Llama block (EE/python/dispatch.py:236-245) takes transformers' eager
attention probabilities -- fp16(Q K^T) times the scale in fp16, the causal mask,
softmax in fp32, rounded to fp16 -- and their entropy -sum p ln(p + 1e-10) in fp32; the
per-token router input is the mean of those row entropies over the heads.  Here torch
runs exactly those ops on the GPU as the reference point, and the flash kernel (which
never rounds a probability to fp16) is compared with it: the distribution of the row
entropy error, and the tokens whose route differs -- every one of them must lie within
the stated band |H_ref - tau| < 2e-3 * max(1, H_ref) of a threshold, and the test
reports how many tokens the band holds.
"""
import json
import math

import pytest
import torch

pytestmark = pytest.mark.gpu

TAUS = [(0.41, 1.68), (2.34, 6.03)]
BAND_REL = 2e-3


def _reference_rows(q, k, scale):
    """The reference's eager path with torch ops: [B, Hq, S] row entropies."""
    B, Hq, S, d = q.shape
    rep = Hq // k.shape[1]
    kr = k.repeat_interleave(rep, dim=1)
    scores = torch.matmul(q, kr.transpose(2, 3)) * scale
    mask = torch.full((S, S), torch.finfo(torch.float16).min, device=q.device, dtype=torch.float16).triu(1)
    p = torch.softmax(scores + mask, dim=-1, dtype=torch.float32).to(torch.float16)
    pf = p.float()
    return -(pf * torch.log(pf + 1e-10)).sum(dim=-1)


def _inputs(B, Hq, Hkv, S, d, device, seed):
    g = torch.Generator(device=device).manual_seed(seed)
    # per-head temperatures spread the row entropies from near 0 to about ln(S)
    temp = torch.exp(torch.linspace(math.log(0.2), math.log(8.0), Hq, device=device)).view(1, Hq, 1, 1)
    q = (torch.randn(B, Hq, S, d, generator=g, device=device) * temp).half()
    k = torch.randn(B, Hkv, S, d, generator=g, device=device).half()
    v = torch.randn(B, Hkv, S, d, generator=g, device=device).half()
    return q, k, v


@pytest.mark.parametrize("d,Hkv,S", [(64, 4, 1024), (128, 8, 1024)])
@torch.no_grad()
def test_flash_token_routes_match_eager_reference_outside_band(pkg, cuda, d, Hkv, S):
    B, Hq = 2, 32
    q, k, v = _inputs(B, Hq, Hkv, S, d, cuda, seed=11 + d)
    scale = d ** -0.5
    rows_ref = _reference_rows(q, k, scale)
    _, _, rows, token = pkg.flash_attention_entropy(q, k, v, causal=True, scale=scale, return_token=True)
    err = (rows - rows_ref).abs()
    rel = err / rows_ref.clamp_min(1e-3)
    tok_ref = rows_ref.mean(dim=1)
    stats = {"d": d, "rows": rows.numel(), "row_rel_err_max": rel.max().item(),
             "row_rel_err_p99": rel.flatten().kthvalue(int(0.99 * rel.numel())).values.item(),
             "row_rel_err_median": rel.median().item(), "row_abs_err_max": err.max().item(),
             "token_abs_err_max": (token - tok_ref).abs().max().item()}
    # the row entropies stay within the flash path's documented tolerance of the reference
    assert torch.allclose(rows, rows_ref, rtol=2e-3, atol=2e-3)
    for tl, th in TAUS:
        r_ref = pkg.EntropyRouter(tl, th)
        r_ref.reserve(B * S, 16, cuda)
        want = r_ref.route_entropy(tok_ref.reshape(-1)).clone()
        r = pkg.EntropyRouter(tl, th)
        r.reserve(B * S, 16, cuda)
        got = r.route_entropy(token.reshape(-1)).clone()
        h = tok_ref.reshape(-1)
        band = BAND_REL * h.abs().clamp_min(1.0)
        in_band = ((h - tl).abs() < band) | ((h - th).abs() < band)
        differ = got != want
        stats[f"tau_{tl}_{th}"] = {"tokens": h.numel(), "route_mismatch": int(differ.sum()),
                                   "band_tokens": int(in_band.sum()),
                                   "mismatch_outside_band": int((differ & ~in_band).sum()),
                                   "mix_ref": [int((want == t).sum()) for t in range(3)]}
        assert not (differ & ~in_band).any(), stats
    print("flash-route-parity " + json.dumps(stats))


@pytest.mark.parametrize("d,Hkv,S", [(64, 4, 1024), (128, 8, 1024)])
@torch.no_grad()
def test_exact_entropy_mode_matches_eager_reference(pkg, cuda, d, Hkv, S):
    """The exact-entropy mode (a second tensor-core pass that rounds every probability to
    fp16 as the eager attention returns it) against the same reference: row entropies
    within 1e-4 relative but for at most 1e-4 of the rows -- rows where one fp16 score of
    torch's matmul rounds the other way than the tensor core's (both sum in fp32, in
    different orders) -- and all within 1e-2; per-token routes identical outside
    |H_ref - tau| < 1e-4 * max(1, H_ref), the count of tokens in that band reported."""
    B, Hq = 2, 32
    q, k, v = _inputs(B, Hq, Hkv, S, d, cuda, seed=11 + d)
    scale = d ** -0.5
    rows_ref = _reference_rows(q, k, scale)
    # the rotary variant with cos = 1, sin = 0 is plain attention on [B, S, H * d] rows
    qb, kb, vb = (t.transpose(1, 2).reshape(B, S, -1).contiguous() for t in (q, k, v))
    cos = torch.ones(B, S, d, device=cuda, dtype=torch.float16)
    sin = torch.zeros_like(cos)
    out_on, _, rows_on, _ = pkg.flash_attention_rope_entropy(qb, kb, vb, cos, sin, Hq, Hkv, scale=scale,
                                                             return_token=True)
    out, _, rows, token = pkg.flash_attention_rope_entropy(qb, kb, vb, cos, sin, Hq, Hkv, scale=scale,
                                                           return_token=True, exact_entropy=True)
    torch.cuda.synchronize()
    assert pkg._lib.device_check() == 0
    assert torch.equal(out, out_on)  # the output is the first pass's either way
    err = (rows - rows_ref).abs()
    beyond = err > 1e-6 + 1e-4 * rows_ref.abs()
    stats = {"d": d, "rows": rows.numel(), "rows_beyond_1e-4": int(beyond.sum()),
             "rel_err_max": (err / rows_ref.clamp_min(1e-3)).max().item(),
             "online_rows_beyond_1e-4": int(((rows_on - rows_ref).abs() > 1e-6 + 1e-4 * rows_ref.abs()).sum())}
    assert int(beyond.sum()) <= max(1, rows.numel() // 10000), stats
    assert torch.allclose(rows, rows_ref, rtol=1e-2, atol=1e-4), stats
    tok_ref = rows_ref.mean(dim=1)
    for tl, th in TAUS:
        routes = []
        for h in (tok_ref, token):
            r = pkg.EntropyRouter(tl, th)
            r.reserve(B * S, 16, cuda)
            routes.append(r.route_entropy(h.reshape(-1)).clone())
        h = tok_ref.reshape(-1)
        band = 1e-4 * h.abs().clamp_min(1.0)
        in_band = ((h - tl).abs() < band) | ((h - th).abs() < band)
        differ = routes[0] != routes[1]
        stats[f"tau_{tl}_{th}"] = {"route_mismatch": int(differ.sum()), "band_tokens": int(in_band.sum()),
                                   "mismatch_outside_band": int((differ & ~in_band).sum())}
        assert not (differ & ~in_band).any(), stats
    print("exact-entropy-parity " + json.dumps(stats))
