"""tcgen05 GEMMs through the C ABI: raw accumulators against exact float64 products
on the same device, then the dequantising epilogues against the reference formulas
(EE/python/kernels.py:104-110, :176-180, :243-246)."""
import pytest
import torch

pytestmark = pytest.mark.gpu

# (M, N, K): one tile / one K stage, several tiles, ragged M/N/K, the configs' shape
SHAPES = [(128, 256, 128), (256, 512, 512), (300, 264, 1040), (1, 8, 16), (1024, 4096, 4096)]


def _e4m3_bytes(shape, gen, device):
    # finite e4m3 codes only (0x7F / 0xFF are NaN)
    codes = torch.randint(0, 256, shape, generator=gen, dtype=torch.int32).to(torch.uint8)
    codes[(codes & 0x7F) == 0x7F] = 0x00
    return codes.to(device)


def _e4m3_to_f64(b):
    return b.view(torch.float8_e4m3fn).to(torch.float64)


@pytest.mark.parametrize("M,N,K", SHAPES)
def test_int8_accumulators_bit_exact(pkg, cuda, M, N, K):
    g = torch.Generator().manual_seed(M * 7 + N * 3 + K)
    a = torch.randint(-128, 128, (M, K), generator=g, dtype=torch.int32).to(torch.int8).to(cuda)
    w = torch.randint(-128, 128, (N, K), generator=g, dtype=torch.int32).to(torch.int8).to(cuda)
    acc = pkg.gemm_accumulators("int8", a, w)
    ref = (a.double() @ w.double().T).round().to(torch.int64)
    torch.cuda.synchronize()
    assert pkg._lib.device_check() == 0
    assert torch.equal(acc.to(torch.int64), ref)


@pytest.mark.parametrize("M,N,K", SHAPES)
def test_fp16_accumulators(pkg, cuda, M, N, K):
    g = torch.Generator().manual_seed(M + N + K)
    a = torch.randn(M, K, generator=g).to(torch.float16).to(cuda)
    w = (torch.randn(N, K, generator=g) * 0.02).to(torch.float16).to(cuda)
    acc = pkg.gemm_accumulators("fp16", a, w)
    ref = a.double() @ w.double().T
    torch.cuda.synchronize()
    err = (acc.double() - ref).norm() / ref.norm()
    assert err < 1e-5, err


@pytest.mark.parametrize("M,N,K", SHAPES)
def test_fp8_accumulators(pkg, cuda, M, N, K):
    g = torch.Generator().manual_seed(M + 2 * N + K)
    a = _e4m3_bytes((M, K), g, cuda)
    w = _e4m3_bytes((N, K), g, cuda)
    acc = pkg.gemm_accumulators("fp8", a, w)
    ref = _e4m3_to_f64(a) @ _e4m3_to_f64(w).T
    torch.cuda.synchronize()
    err = (acc.double() - ref).norm() / ref.norm()
    assert err < 1e-5, err


def test_int8_epilogue_matches_reference_formula(pkg, cuda):
    M, N, K = 256, 512, 1024
    g = torch.Generator().manual_seed(5)
    a = torch.randint(-127, 128, (M, K), generator=g, dtype=torch.int32).to(torch.int8).to(cuda)
    w_kn = torch.randint(-127, 128, (K, N), generator=g, dtype=torch.int32).to(torch.int8).to(cuda)
    sa = (torch.rand(M, generator=g) * 0.05 + 1e-3).to(cuda)
    sb = (torch.rand(N, generator=g) * 0.01 + 1e-4).to(cuda)
    y = pkg.gemm_int8_prequant(a, w_kn, sa, sb)
    acc = (a.double() @ w_kn.double()).round()
    ref = ((acc.float() * sa[:, None]) * sb[None, :]).half()
    torch.cuda.synchronize()
    assert torch.equal(y.view(torch.int16), ref.view(torch.int16))


def test_pack_weights_operands(pkg, cuda):
    K, N = 256, 384
    g = torch.Generator().manual_seed(9)
    w_kn = torch.randint(-127, 128, (K, N), generator=g, dtype=torch.int32).to(torch.int8).to(cuda)
    s = (torch.rand(N, generator=g) * 0.01 + 1e-4).to(cuda)
    p = pkg.WeightPack(w_kn, s)
    torch.cuda.synchronize()
    assert torch.equal(p.w_i8, w_kn.T.contiguous())
    want_e4m3 = w_kn.T.contiguous().to(torch.float16).to(torch.float8_e4m3fn).view(torch.uint8)
    assert torch.equal(p.w_e4m3, want_e4m3)
    want_f16 = w_kn.T.contiguous().to(torch.float16) * s.to(torch.float16)[:, None]
    assert torch.equal(p.w_f16.view(torch.int16), want_f16.view(torch.int16))
