"""The weight-streaming GEMM for calls of at most 128 rows (ee_gemm_skinny.cuh: weights as
the UMMA M operand, K split over a thread-block cluster, partials reduced through
distributed shared memory): exact int32 accumulators and INT8 outputs, FP8 / FP16 within
the reference's tolerance, for every activation-row tile size (16 / 32 / 64 / 128), forced
and automatic K splits, N and K off the tile grid, and routed buckets of every size up to
128 rows."""
import pytest
import torch

pytestmark = pytest.mark.gpu

from test_gpu_gated import _ref_fp8, _ref_fp16, _ref_int8, _relf  # noqa: E402


@pytest.fixture
def lib(pkg, cuda):
    lib = pkg.load_library()
    assert lib.ee_set_gemm_policy(4) == 0
    yield lib
    assert lib.ee_set_gemm_policy(0) == 0
    assert lib.ee_set_gemm_splits(0) == 0


@pytest.mark.parametrize("splits", [0, 1, 2, 3, 8])
@pytest.mark.parametrize("M,N,K", [(1, 128, 128), (16, 4096, 4096), (17, 264, 1040), (40, 384, 2048),
                                   (64, 136, 4096), (100, 4096, 1024), (128, 512, 14336)])
def test_accumulators(pkg, lib, cuda, splits, M, N, K):
    assert lib.ee_set_gemm_splits(splits) == 0
    g = torch.Generator().manual_seed(M * 7 + N + K + splits)
    a = torch.randint(-128, 128, (M, K), generator=g, dtype=torch.int32).to(torch.int8).to(cuda)
    w = torch.randint(-128, 128, (N, K), generator=g, dtype=torch.int32).to(torch.int8).to(cuda)
    acc = pkg.gemm_accumulators("int8", a, w)
    torch.cuda.synchronize()
    assert pkg._lib.device_check() == 0
    assert torch.equal(acc.to(torch.int64), (a.double() @ w.double().T).round().to(torch.int64))
    a16 = torch.randn(M, K, generator=g).half().to(cuda)
    w16 = (torch.randn(N, K, generator=g) * 0.02).half().to(cuda)
    # the tensor core's fp32 accumulation is not round-to-nearest at every step: measured
    # 1.7e-5 relative over K = 14336 in one pass (K split into fp32 partials lands lower)
    tol = 1e-5 if K <= 4096 else 3e-5
    acc = pkg.gemm_accumulators("fp16", a16, w16)
    ref = a16.double() @ w16.double().T
    assert ((acc.double() - ref).norm() / ref.norm()) < tol
    a8 = a16.to(torch.float8_e4m3fn).view(torch.uint8)
    w8 = (w16 * 40).to(torch.float8_e4m3fn).view(torch.uint8)
    acc = pkg.gemm_accumulators("fp8", a8, w8)
    ref = a8.view(torch.float8_e4m3fn).double() @ w8.view(torch.float8_e4m3fn).double().T
    assert ((acc.double() - ref).norm() / ref.norm()) < tol
    torch.cuda.synchronize()
    assert pkg._lib.device_check() == 0


def test_int8_equals_other_tilings(pkg, lib, cuda):
    """INT8 results do not depend on the kernel: the weight-streaming kernel with K split
    eight ways gives the 128 x 64 tiles' fp16 outputs bit for bit."""
    g = torch.Generator(device=cuda).manual_seed(3)
    M, K, N = 48, 4096, 1024
    a = torch.randn(M, K, generator=g, device=cuda).half()
    w = (torch.randn(N, K, generator=g, device=cuda) * 0.02).half()
    w_kn, ws = pkg.quantize_weights_int8(w)
    assert lib.ee_set_gemm_splits(8) == 0
    y_skinny = pkg.triton_int8_gemm(a, w_kn, ws)
    assert lib.ee_set_gemm_policy(3) == 0
    y_narrow = pkg.triton_int8_gemm(a, w_kn, ws)
    torch.cuda.synchronize()
    assert torch.equal(y_skinny.view(torch.int16), y_narrow.view(torch.int16))


@pytest.mark.parametrize("splits", [0, 1, 4])
@pytest.mark.parametrize("counts", [(5, 9, 2), (0, 16, 0), (1, 1, 1), (40, 50, 38), (128, 0, 0), (0, 0, 128),
                                    (0, 33, 31), (10, 0, 54)])
def test_routed_buckets(pkg, lib, cuda, splits, counts):
    """Routed rows in a shuffled order, bucket sizes from 0 to 128 (the tile's row count is
    chosen from the call's row capacity, so a bucket may fill it)."""
    assert lib.ee_set_gemm_splits(splits) == 0
    M, K, N = sum(counts), 2048, 640
    g = torch.Generator(device=cuda).manual_seed(sum(counts) * 3 + splits)
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


def test_auto_policy_small_calls(pkg, cuda):
    """The automatic policy takes the weight-streaming kernel at <= 128 rows: the
    reference launchers at 16 rows of a Llama-3-8B projection, INT8 bit-exact."""
    g = torch.Generator(device=cuda).manual_seed(11)
    M, K, N = 16, 4096, 14336
    a = torch.randn(M, K, generator=g, device=cuda).half()
    w = (torch.randn(N, K, generator=g, device=cuda) * 0.02).half()
    w_kn, ws = pkg.quantize_weights_int8(w)
    p = pkg.WeightPack(w_kn, ws)
    y8 = pkg.triton_int8_gemm(a, w_kn, ws)
    yf8 = pkg.triton_fp8_gemm(a, w_kn, ws)
    y16 = pkg.triton_fp16_gemm(a, w_kn, ws)
    torch.cuda.synchronize()
    assert pkg._lib.device_check() == 0
    assert torch.equal(y8.view(torch.int16), _ref_int8(a, p).view(torch.int16))
    assert _relf(yf8, _ref_fp8(a, p)) < 1e-2
    assert _relf(y16, _ref_fp16(a, p)) < 1e-2
