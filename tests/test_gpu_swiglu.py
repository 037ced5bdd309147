"""The fused SwiGLU GEMM (ee_gated_swiglu_packed): gate, up, SiLU and the product in one
bucketed GEMM, against the unfused sequence on the same packed rows (two gated GEMMs,
then torch's silu and multiply on their fp16 outputs)."""
import math

import pytest
import torch

pytestmark = pytest.mark.gpu


def _case(M, K, inter, seed, dev):
    g = torch.Generator(device=dev).manual_seed(seed)
    s = torch.exp(torch.rand(M, 1, generator=g, device=dev) * (math.log(9.5) - math.log(5.0)) + math.log(5.0))
    logits = (torch.randn(M, 1024, generator=g, device=dev) * s).half()
    x = torch.randn(M, K, generator=g, device=dev)
    x = torch.where(torch.rand(M, K, generator=g, device=dev) < 0.01, x * 20.0, x).half()
    wg = (torch.randn(inter, K, generator=g, device=dev) * 0.05).half()
    wu = (torch.randn(inter, K, generator=g, device=dev) * 0.05).half()
    return logits, x, wg, wu


@pytest.fixture(params=[0, 1, 2], ids=["auto", "single_cta", "cta_pair"])
def policy(request, pkg, cuda):
    lib = pkg.load_library()
    assert lib.ee_set_gemm_policy(request.param) == 0
    yield request.param
    assert lib.ee_set_gemm_policy(0) == 0


@pytest.mark.parametrize("M,K,inter", [(1000, 512, 1024), (64, 256, 384), (4096, 2048, 2816)])
def test_fused_equals_unfused(pkg, cuda, policy, M, K, inter):
    logits, x, wg, wu = _case(M, K, inter, M + K + inter + policy, cuda)
    gate, up = pkg.WeightPack.from_weight(wg), pkg.WeightPack.from_weight(wu)
    r = pkg.EntropyRouter(0.41, 1.68)
    r.reserve(M, K, cuda)
    r.route(logits)
    r.pack_rows(x)
    want = torch.nn.functional.silu(r.gemm_packed(gate)) * r.gemm_packed(up)
    got = r.swiglu_packed(pkg.SwiGLUPack(gate, up))
    torch.cuda.synchronize()
    assert pkg._lib.device_check() == 0
    counts = r.counts.cpu().tolist()
    assert min(counts) > 0 or M < 100
    assert torch.equal(got.view(torch.int16), want.view(torch.int16))


def test_rejects_unaligned_intermediate(pkg, cuda):
    with pytest.raises(RuntimeError, match="multiple of 128"):
        g = pkg.WeightPack.from_weight(torch.randn(200, 64, device=cuda).half())
        pkg.SwiGLUPack(g, g)
    lib = pkg.load_library()
    p = 256
    assert lib.ee_gated_swiglu_packed(16, 64, p, p, p, p, 100, p, 100, p, 1 << 20, None) == -3
