"""The dequantising GEMM epilogues with every output layout the C ABI accepts: rows whose
stride and base allow 32-byte stores, strides that are only 16-byte multiples, a base 16
bytes past a 32-byte boundary, and a column count with a final half group (N % 16 == 8).
Every layout gives the same bits as the contiguous output, and the INT8 bucket the
reference formula fp16((acc * s_a) * s_b) (EE/python/kernels.py:104-110)."""
import pytest
import torch

pytestmark = pytest.mark.gpu


def _call(pkg, kind, a, sa, w_nk, sb, y, M, N, K, ldy):
    stream = torch.cuda.current_stream().cuda_stream
    if kind == "fp16":
        pkg._lib.call("ee_gemm_fp16", a.data_ptr(), w_nk.data_ptr(), y.data_ptr(), M, N, K, ldy, stream)
    else:
        pkg._lib.call("ee_gemm_int8" if kind == "int8" else "ee_gemm_fp8", a.data_ptr(), sa.data_ptr(),
                      w_nk.data_ptr(), sb.data_ptr(), y.data_ptr(), M, N, K, ldy, stream)


def _operands(kind, M, N, K, cuda):
    g = torch.Generator().manual_seed(M + N + K)
    if kind == "fp16":
        a = (torch.randn(M, K, generator=g) * 0.5).half().to(cuda)
        w = (torch.randn(N, K, generator=g) * 0.05).half().to(cuda)
        return a, None, w, None
    if kind == "int8":
        a = torch.randint(-127, 128, (M, K), generator=g, dtype=torch.int32).to(torch.int8).to(cuda)
        w = torch.randint(-127, 128, (N, K), generator=g, dtype=torch.int32).to(torch.int8).to(cuda)
    else:
        a = (torch.randn(M, K, generator=g) * 2).to(torch.float8_e4m3fn).to(cuda)
        w = (torch.randn(N, K, generator=g) * 2).to(torch.float8_e4m3fn).to(cuda)
    sa = (torch.rand(M, generator=g) * 0.05 + 1e-3).to(cuda)
    sb = (torch.rand(N, generator=g) * 0.01 + 1e-4).to(cuda)
    return a, sa, w, sb


@pytest.mark.parametrize("kind", ["int8", "fp8", "fp16"])
@pytest.mark.parametrize("M,N,K", [(300, 512, 512), (300, 264, 512), (1024, 4096, 1024)])
@torch.no_grad()
def test_epilogue_output_layouts(pkg, cuda, kind, M, N, K):
    a, sa, w, sb = _operands(kind, M, N, K, cuda)
    ld16 = N if N % 16 == 8 else N + 8  # a row stride of 16-byte but not 32-byte multiples
    ld32 = (N + 15) // 16 * 16  # 32-byte multiples
    layouts = {  # (row stride, base offset in elements)
        "contiguous": (N, 0),
        "stride_16B_only": (ld16, 0),
        "stride_32B": (ld32, 0),
        "stride_32B_padded": (ld32 + 16, 0),
        "base_16B_past_32B": (ld32, 8),
    }
    outs = {}
    for name, (ldy, off) in layouts.items():
        buf = torch.full((M * ldy + off + 64,), float("nan"), dtype=torch.float16, device=cuda)
        y = buf[off:off + M * ldy]
        _call(pkg, kind, a, sa, w, sb, y, M, N, K, ldy)
        torch.cuda.synchronize()
        assert pkg._lib.device_check() == 0
        view = y.view(M, ldy)
        assert torch.isnan(view[:, N:]).all(), name  # nothing written past column N
        assert torch.isnan(buf[off + M * ldy:]).all(), name  # nor past the last row
        outs[name] = view[:, :N].clone()
    base = outs["contiguous"]
    for name, o in outs.items():
        assert torch.equal(o.view(torch.int16), base.view(torch.int16)), name
    if kind == "int8":
        acc = (a.double() @ w.double().T).round()
        ref = ((acc.float() * sa[:, None]) * sb[None, :]).half()
        assert torch.equal(base.view(torch.int16), ref.view(torch.int16))
    elif kind == "fp8":
        acc = a.to(torch.float64) @ w.to(torch.float64).T
        ref = (acc * sa.double()[:, None]) * sb.double()[None, :]
        err = (base.double() - ref).norm() / ref.norm()
        assert err < 1e-3, err
    else:
        ref = a.double() @ w.double().T
        err = (base.double() - ref).norm() / ref.norm()
        assert err < 1e-3, err
