"""ee_linear_int8_noalloc: the INT8 linear for callers that cannot give the library any
device memory (a serving process whose allocator owns the whole GPU and forbids
allocation after start-up, or a plug-in whose host runtime owns the allocator).

It must produce exactly what ee_linear_int8 (caller-owned workspace) produces -- the
INT8 path is bit-exact, so that is the tolerance here -- on two calls in a row, the
second one reusing the fixed scratch the first one left behind.  The file name makes
pytest collect it last.
"""
import ctypes

import pytest
import torch

pytestmark = pytest.mark.gpu


def _inputs(M, K, N, seed, device):
    g = torch.Generator().manual_seed(seed)
    a = torch.randn(M, K, generator=g)
    a[torch.rand(M, K, generator=g) < 0.01] *= 20.0
    w = torch.randn(N, K, generator=g) * 0.02
    return a.to(torch.float16).to(device), w.to(torch.float16).to(device)


def _with_workspace(pkg, a, pack, y):
    lib = pkg.load_library()
    M, K = a.shape
    ws = torch.empty(lib.ee_linear_workspace_bytes(M, K), dtype=torch.uint8, device=a.device)
    st = lib.ee_linear_int8(a.data_ptr(), K, pack.w_i8.data_ptr(), pack.scale.data_ptr(), y.data_ptr(), M, pack.N, K,
                            pack.N, ws.data_ptr(), ws.numel(), torch.cuda.current_stream().cuda_stream)
    assert st == 0, pkg._lib.last_error()


def _no_alloc(pkg, a, pack, y):
    lib = pkg.load_library()
    M, K = a.shape
    return lib.ee_linear_int8_noalloc(a.data_ptr(), K, pack.w_i8.data_ptr(), pack.scale.data_ptr(), y.data_ptr(), M,
                                      pack.N, K, pack.N, torch.cuda.current_stream().cuda_stream)


def test_no_alloc_matches_workspace_entry_point_two_calls(pkg, cuda):
    # each call is smaller than the one before, so stale scratch rows would show up; the
    # first fills the scratch exactly (M * K = 2^24), the last takes the weight-streaming
    # kernel (at most 64 rows)
    for M, K, N, seed in [(4096, 4096, 256, 10), (1024, 4096, 4096, 11), (300, 1024, 776, 12),
                          (16, 4096, 4096, 13)]:
        a, w = _inputs(M, K, N, seed, cuda)
        w_kn, w_s = pkg.quantize_weights_int8(w)
        pack = pkg.WeightPack(w_kn, w_s)
        y_ref = torch.empty(M, N, dtype=torch.float16, device=cuda)
        y = torch.full((M, N), float("nan"), dtype=torch.float16, device=cuda)
        _with_workspace(pkg, a, pack, y_ref)
        st = _no_alloc(pkg, a, pack, y)
        assert st == 0, pkg._lib.last_error()
        torch.cuda.synchronize()
        assert pkg._lib.device_check() == 0
        assert torch.equal(y.view(torch.int16), y_ref.view(torch.int16))


def test_no_alloc_rejects_sizes_beyond_its_scratch(pkg, cuda):
    lib = pkg.load_library()
    null = ctypes.c_void_p(16)  # never dereferenced: the size check comes first
    for M, K in [(4096, 8192), (16385, 16), (1, (1 << 24) + 16), (4097, 4096)]:
        st = lib.ee_linear_int8_noalloc(null, K, null, null, null, M, 256, K, 256, None)
        assert st == -3, (M, K)  # EE_ERR_UNSUPPORTED
        assert "exceeds its fixed scratch" in pkg._lib.last_error()
