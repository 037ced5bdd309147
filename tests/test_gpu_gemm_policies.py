"""Every GEMM tiling -- single-CTA 128 x 256, CTA-pair (tcgen05 cta_group::2) 256 x 256
and single-CTA 128 x 64 tiles -- forced through ee_set_gemm_policy: exact int32
accumulators, fp32 accumulators, and the gated linear per bucket against the reference
formulas."""
import pytest
import torch

pytestmark = pytest.mark.gpu

from test_gpu_gated import _inputs, _ref_fp8, _ref_fp16, _ref_int8, _relf  # noqa: E402


@pytest.fixture(params=[1, 2, 3], ids=["single_cta", "cta_pair", "single_cta_narrow"])
def policy(request, pkg, cuda):
    lib = pkg.load_library()
    assert lib.ee_set_gemm_policy(request.param) == 0
    yield request.param
    assert lib.ee_set_gemm_policy(0) == 0


@pytest.mark.parametrize("M,N,K", [(128, 256, 128), (300, 264, 1040), (1024, 4096, 4096), (257, 512, 2048)])
def test_accumulators(pkg, cuda, policy, M, N, K):
    g = torch.Generator().manual_seed(M + N + K + policy)
    a = torch.randint(-128, 128, (M, K), generator=g, dtype=torch.int32).to(torch.int8).to(cuda)
    w = torch.randint(-128, 128, (N, K), generator=g, dtype=torch.int32).to(torch.int8).to(cuda)
    acc = pkg.gemm_accumulators("int8", a, w)
    assert torch.equal(acc.to(torch.int64), (a.double() @ w.double().T).round().to(torch.int64))
    a16 = torch.randn(M, K, generator=g).half().to(cuda)
    w16 = (torch.randn(N, K, generator=g) * 0.02).half().to(cuda)
    acc = pkg.gemm_accumulators("fp16", a16, w16)
    ref = a16.double() @ w16.double().T
    assert ((acc.double() - ref).norm() / ref.norm()) < 1e-5
    a8 = a16.to(torch.float8_e4m3fn).view(torch.uint8)
    w8 = (w16 * 40).to(torch.float8_e4m3fn).view(torch.uint8)
    acc = pkg.gemm_accumulators("fp8", a8, w8)
    ref = a8.view(torch.float8_e4m3fn).double() @ w8.view(torch.float8_e4m3fn).double().T
    assert ((acc.double() - ref).norm() / ref.norm()) < 1e-5
    torch.cuda.synchronize()
    assert pkg._lib.device_check() == 0


@pytest.mark.parametrize("M,n,K,N", [(1024, 4096, 4096, 4096), (333, 256, 1024, 264), (4096, 4096, 1024, 1536)])
def test_gated_linear(pkg, cuda, policy, M, n, K, N):
    logits, a, w = _inputs(M, n, K, N, 5 * M + n + policy, cuda)
    p = pkg.WeightPack(*pkg.quantize_weights_int8(w))
    y, H, route, counts = pkg.gated_linear(logits, a, p, 0.41, 1.68)
    torch.cuda.synchronize()
    assert pkg._lib.device_check() == 0
    rows = [torch.nonzero(route == b).flatten() for b in range(3)]
    if rows[0].numel():
        assert torch.equal(y[rows[0]].view(torch.int16), _ref_int8(a[rows[0]], p).view(torch.int16))
    if rows[1].numel():
        assert _relf(y[rows[1]], _ref_fp8(a[rows[1]], p)) < 1e-2
    if rows[2].numel():
        assert _relf(y[rows[2]], _ref_fp16(a[rows[2]], p)) < 1e-2


@pytest.mark.parametrize("counts", [(100, 300, 40), (130, 257, 128), (256, 129, 1), (0, 128, 384)])
def test_bucket_edge_sizes(pkg, cuda, policy, counts):
    """Bucket sizes at the row-tile edges (a last tile of 1, 128, 129 or 256 rows: the
    CTA-pair kernel runs tiles of at most 128 rows as M = 128 pair tiles), routed from
    given entropies in a shuffled row order."""
    M, K, N = sum(counts), 512, 768
    g = torch.Generator(device=cuda).manual_seed(sum(counts) + policy)
    H = torch.cat([torch.full((c,), v, device=cuda) for c, v in zip(counts, (0.1, 1.0, 3.0))])
    H = H[torch.randperm(M, generator=g, device=cuda)]
    a = torch.randn(M, K, generator=g, device=cuda)
    a = torch.where(torch.rand(M, K, generator=g, device=cuda) < 0.01, a * 20.0, a).half()
    w = (torch.randn(N, K, generator=g, device=cuda) * 0.05).half()
    p = pkg.WeightPack(*pkg.quantize_weights_int8(w))
    r = pkg.EntropyRouter(0.41, 1.68)
    r.reserve(M, K, cuda)
    r.route_entropy(H)
    y = r.gated_linear(a, p)
    torch.cuda.synchronize()
    assert pkg._lib.device_check() == 0
    assert r.counts.cpu().tolist() == list(counts)
    route = r.route_ids
    rows = [torch.nonzero(route == b).flatten() for b in range(3)]
    if rows[0].numel():
        assert torch.equal(y[rows[0]].view(torch.int16), _ref_int8(a[rows[0]], p).view(torch.int16))
    if rows[1].numel():
        assert _relf(y[rows[1]], _ref_fp8(a[rows[1]], p)) < 1e-2
    if rows[2].numel():
        assert _relf(y[rows[2]], _ref_fp16(a[rows[2]], p)) < 1e-2

