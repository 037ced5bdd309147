"""The C ABI without a GPU: the library loads, exports every entry point that
include/ee_b200.h declares, and rejects bad arguments with the documented status
codes before touching the device.  CPU only."""
import ctypes
import os
import re
import subprocess

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
HEADER = os.path.join(ROOT, "include", "ee_b200.h")

EE_ERR_INVALID, EE_ERR_MISALIGNED, EE_ERR_UNSUPPORTED = -1, -2, -3


def _declared():
    text = open(HEADER).read()
    return sorted(set(re.findall(r"EE_API\s+[\w\s\*]+?\b(ee_\w+)\s*\(", text)))


@pytest.fixture(scope="module")
def lib(pkg):
    return pkg.load_library()


def test_header_declares_entry_points():
    names = _declared()
    assert "ee_gated_linear" in names and "ee_softmax_entropy" in names
    assert len(names) >= 25


def test_library_exports_every_declared_symbol(pkg):
    out = subprocess.run(["nm", "-D", "--defined-only", pkg.LIB_PATH], capture_output=True, text=True,
                         check=True).stdout
    exported = set(re.findall(r"\bT (ee_\w+)", out))
    missing = [n for n in _declared() if n not in exported]
    assert not missing, missing
    # nothing else leaks out of the library's C interface
    assert exported == set(_declared()), sorted(exported - set(_declared()))


def test_ctypes_signatures_cover_the_header(pkg):
    from importlib import import_module

    sigs = import_module("tko_b200._lib").SIGNATURES
    assert set(sigs) == set(_declared())


def test_library_has_no_gpu_driver_dependency(pkg):
    out = subprocess.run(["ldd", pkg.LIB_PATH], capture_output=True, text=True).stdout
    assert "libcuda.so" not in out and "libcudart" not in out


def test_abi_version(lib):
    assert lib.ee_abi_version() == 1


def _msg(pkg):
    return pkg._lib.last_error()


def test_gemm_argument_checks(pkg, lib):
    p = ctypes.c_void_p(256)
    # K not a multiple of 16
    assert lib.ee_gemm_int8(p, p, p, p, p, 128, 256, 100, 256, None) == EE_ERR_UNSUPPORTED
    assert "multiple of 16" in _msg(pkg)
    # N not a multiple of 8
    assert lib.ee_gemm_fp16(p, p, p, 128, 250, 128, 250, None) == EE_ERR_UNSUPPORTED
    # ldy smaller than N
    assert lib.ee_gemm_fp8(p, p, p, p, p, 128, 256, 128, 128, None) == EE_ERR_MISALIGNED
    # negative M
    assert lib.ee_gemm_int8(p, p, p, p, p, -1, 256, 128, 256, None) == EE_ERR_INVALID
    # misaligned operand
    assert lib.ee_gemm_fp16(ctypes.c_void_p(258), p, p, 128, 256, 128, 256, None) == EE_ERR_MISALIGNED
    # M == 0 is a no-op
    assert lib.ee_gemm_int8(p, p, p, p, p, 0, 256, 128, 256, None) == 0


def test_workspace_checks(pkg, lib):
    p = ctypes.c_void_p(256)
    need = lib.ee_gated_workspace_bytes(1024, 4096)
    assert need >= 1024 * 4096 * 3
    st = lib.ee_gated_gemm(p, 4096, 1024, 4096, p, p, p, p, 4096, p, 4096, p, need - 1, None)
    assert st == EE_ERR_INVALID and "too small" in _msg(pkg)
    st = lib.ee_gated_gemm(p, 4096, 1024, 4096, p, p, p, p, 4096, p, 4096, ctypes.c_void_p(272), need, None)
    assert st == EE_ERR_MISALIGNED
    assert lib.ee_linear_workspace_bytes(-1, 5) == 0


def test_split_workspace_sizing(pkg, lib):
    """K-split room: none at <= 64 rows (the weight-streaming kernel) and above 4096 rows;
    otherwise 256 bytes of plan + four 128 KiB partial blocks per SM (148 without a GPU)."""
    for M, K in [(16, 4096), (64, 14336), (5000, 4096), (16384, 2048)]:
        assert lib.ee_gated_workspace_split_bytes(M, K) == lib.ee_gated_workspace_bytes(M, K)
    for M, K in [(65, 4096), (128, 14336), (1024, 4096), (4096, 14336)]:
        extra = lib.ee_gated_workspace_split_bytes(M, K) - lib.ee_gated_workspace_bytes(M, K)
        assert extra == 256 + 4 * 148 * 128 * 256 * 4
    assert lib.ee_gated_workspace_split_bytes(-1, 8) == 0


def test_workspace_layout_offsets(pkg, lib):
    off = (ctypes.c_int64 * 8)()
    assert lib.ee_gated_workspace_layout(1000, 512, off) == 0
    offs = list(off)
    assert offs == sorted(offs) and all(o % 256 == 0 for o in offs[1:]) and offs[0] % 16 == 0
    assert offs[7] - offs[6] >= 1000 * 512


def test_softmax_argument_checks(pkg, lib):
    p = ctypes.c_void_p(256)
    assert lib.ee_softmax_entropy(p, 4, 0, 0, 0, 1, None, 0, p, None, 0.0, 0.0, None) == EE_ERR_INVALID
    assert lib.ee_softmax_entropy(p, 4, 8, 8, 1, 0, None, 8, p, None, 0.0, 0.0, None) == EE_ERR_INVALID
    assert lib.ee_softmax_entropy(None, 4, 8, 8, 0, 1, None, 8, p, None, 0.0, 0.0, None) == EE_ERR_INVALID
    assert lib.ee_softmax_entropy(p, 0, 8, 8, 0, 1, None, 8, p, None, 0.0, 0.0, None) == 0


def test_attention_entropy_argument_checks(pkg, lib):
    p = ctypes.c_void_p(256)
    # bad dtype code
    assert lib.ee_attention_entropy(p, 7, 4, 8, 8, p, 1, p, None) == EE_ERR_INVALID
    # rows not a multiple of the batches
    assert lib.ee_attention_entropy(p, 0, 6, 8, 8, p, 4, p, None) == EE_ERR_INVALID
    # ld < n, missing row output
    assert lib.ee_attention_entropy(p, 1, 4, 8, 4, p, 1, p, None) == EE_ERR_INVALID
    assert lib.ee_attention_entropy(p, 1, 4, 8, 8, None, 1, p, None) == EE_ERR_INVALID
    # an fp32 pointer that is only 2-byte aligned
    assert lib.ee_attention_entropy(ctypes.c_void_p(258), 1, 4, 8, 8, p, 1, p, None) == EE_ERR_MISALIGNED
    # no rows: nothing to do
    assert lib.ee_attention_entropy(None, 0, 0, 8, 8, None, 0, None, None) == 0


def test_errors_raise_runtime_error_in_python(pkg):
    from importlib import import_module

    _lib = import_module("tko_b200._lib")
    with pytest.raises(RuntimeError, match="EE_ERR_UNSUPPORTED"):
        _lib.call("ee_gemm_int8", 256, 256, 256, 256, 256, 128, 256, 100, 256, None)


def test_calls_without_a_device_fail_cleanly(pkg, lib):
    import torch

    if torch.cuda.is_available():
        pytest.skip("a GPU is visible")
    # valid arguments reach the CUDA runtime, which reports the missing device
    p = ctypes.c_void_p(256)
    st = lib.ee_gemm_fp16(p, p, p, 128, 256, 128, 256, None)
    assert st == -4


def test_decoder_engine_argument_checks(pkg, lib):
    from importlib import import_module

    eng = import_module("tko_b200.engine")
    cfg = eng._DecoderConfigC(2, 256, 256, 4, 2, 64, 512, 1e-5, 0.125, 2.0, 4.0, 0, 0, 0)
    assert lib.ee_decoder_workspace_bytes(ctypes.byref(cfg)) > 0
    for field, bad in (("head_dim", 96), ("intermediate", 500), ("kv_heads", 3), ("routing", 2), ("route_all", 5),
                       ("exact_entropy", 2)):
        c = eng._DecoderConfigC.from_buffer_copy(cfg)
        setattr(c, field, bad)
        assert lib.ee_decoder_workspace_bytes(ctypes.byref(c)) == 0, field
    out = ctypes.c_void_p()
    layers = (eng._DecoderLayerC * 1)()
    p = ctypes.c_void_p(4096)
    assert lib.ee_decoder_create(ctypes.byref(cfg), 1, layers, p, p, p, None, p, 1 << 30, None) == EE_ERR_INVALID
    # a layer without its weights is rejected before anything touches the device
    st = lib.ee_decoder_create(ctypes.byref(cfg), 1, layers, p, p, p, None, p, 1 << 30, ctypes.byref(out))
    assert st == EE_ERR_INVALID and "missing a weight" in _msg(pkg) and not out.value
    assert lib.ee_decoder_run(None, p, p, None, None) == EE_ERR_INVALID
    assert lib.ee_decoder_launch(None, None) == EE_ERR_INVALID
    assert lib.ee_decoder_destroy(None) == 0
    assert lib.ee_head_mean_entropy(None, 2, 4, 8, p, None, None) == EE_ERR_INVALID
    assert lib.ee_head_mean_entropy(ctypes.c_void_p(4098), 2, 4, 8, p, None, None) == EE_ERR_MISALIGNED


def test_kv_cache_argument_checks(pkg, lib):
    from importlib import import_module

    kvc = import_module("tko_b200.kvcache")
    assert lib.ee_kv_cache_bytes(2, 8, 128, 4096, 1000, 1000) > 0
    assert lib.ee_kv_cache_bytes(2, 8, 96, 4096, 1000, 1000) == 0  # head_dim 64 or 128
    assert lib.ee_kv_cache_bytes(2, 8, 128, 4096, 1 << 28, 1) == 0  # slot index above 28 bits
    c = kvc._KvCacheC()
    p = ctypes.c_void_p(4096)
    assert lib.ee_kv_cache_init(None, p, 1 << 30, 2, 8, 128, 64, 8, 8, None) == EE_ERR_INVALID
    assert lib.ee_kv_cache_init(ctypes.byref(c), p, 16, 2, 8, 128, 64, 8, 8, None) == EE_ERR_INVALID  # too small
    assert lib.ee_kv_append(ctypes.byref(c), p, 1024, p, 1024, p, 1, None) == EE_ERR_INVALID  # not initialised
    assert lib.ee_kv_decode_workspace_bytes(None, 32) == 0
    c2 = kvc._KvCacheC(2, 8, 128, 4096, 8, 8)
    assert lib.ee_kv_decode_workspace_bytes(ctypes.byref(c2), 32) > 0
    assert lib.ee_kv_decode_attention(ctypes.byref(c), p, 4096, 32, p, p, 1024, 0.1, p, 4096, None, p, 1 << 20,
                                      None) == EE_ERR_INVALID
