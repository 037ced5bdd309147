"""ctypes binding of libee_b200.so (include/ee_b200.h).

Every wrapper raises RuntimeError carrying ee_last_error() when a call returns a
non-zero status, which is how the reference's TORCH_CHECK / CUDA_DRIVER_CHECK
failures surface in Python (EE/csrc/engine.cpp:13-21, :112-124).  There is no
fallback: when the library is missing the import fails loudly.
"""
from __future__ import annotations

import ctypes
import os
from ctypes import POINTER, c_char_p, c_double, c_float, c_int, c_int8, c_int32, c_int64, c_size_t, c_uint8, c_void_p

PKG_DIR = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(PKG_DIR, "libee_b200.so")

EE_OK = 0
STATUS_NAMES = {
    -1: "EE_ERR_INVALID",
    -2: "EE_ERR_MISALIGNED",
    -3: "EE_ERR_UNSUPPORTED",
    -4: "EE_ERR_CUDA",
    -5: "EE_ERR_DEVICE",
}

_P = c_void_p  # every device pointer crosses as an untyped address
# name -> (restype, argtypes): the exact declarations of include/ee_b200.h
SIGNATURES = {
    "ee_abi_version": (c_int, []),
    "ee_last_error": (c_char_p, []),
    "ee_set_gemm_policy": (c_int, [c_int]),
    "ee_set_gemm_splits": (c_int, [c_int]),
    "ee_device_check": (c_int, [POINTER(c_int)]),
    "ee_debug_drop_next_gemm_load": (c_int, [c_int]),
    "ee_softmax_entropy": (c_int, [_P, c_int64, c_int64, c_int64, c_int, c_int64, _P, c_int64, _P, _P, c_double,
                                   c_double, _P]),
    "ee_fused_softmax_entropy_4d": (c_int, [_P, c_int64, c_int64, c_int64, c_int, _P, _P, _P, _P]),
    "ee_attention_entropy": (c_int, [_P, c_int, c_int64, c_int64, c_int64, _P, c_int64, _P, _P]),
    "ee_attention_workspace_bytes": (c_size_t, [c_int64, c_int64, c_int64, c_int64]),
    "ee_flash_attention_entropy": (c_int, [_P, _P, _P, c_int64, c_int64, c_int64, c_int64, c_int64, c_int, c_float, _P,
                                           _P, _P, c_size_t, _P]),
    "ee_attention_rope_workspace_bytes": (c_size_t, [c_int64, c_int64, c_int64, c_int64, c_int64]),
    "ee_flash_attention_rope_entropy": (c_int, [_P, c_int64, _P, c_int64, _P, c_int64, _P, _P, c_int64, c_int64,
                                                c_int64, c_int64, c_int64, c_int64, c_int, c_float, _P, _P, _P,
                                                c_size_t, _P]),
    "ee_head_mean_entropy": (c_int, [_P, c_int64, c_int64, c_int64, _P, _P, _P]),
    "ee_attention_exact_workspace_bytes": (c_size_t, [c_int64, c_int64, c_int64, c_int64, c_int64]),
    "ee_flash_attention_rope_entropy_exact": (c_int, [_P, c_int64, _P, c_int64, _P, c_int64, _P, _P, c_int64,
                                                      c_int64, c_int64, c_int64, c_int64, c_int64, c_int, c_float,
                                                      _P, _P, _P, c_size_t, _P]),
    "ee_kv_cache_bytes": (c_size_t, [c_int64, c_int64, c_int64, c_int64, c_int64, c_int64]),
    "ee_kv_cache_init": (c_int, [_P, _P, c_size_t, c_int64, c_int64, c_int64, c_int64, c_int64, c_int64, _P]),
    "ee_kv_append": (c_int, [_P, _P, c_int64, _P, c_int64, _P, c_int64, _P]),
    "ee_kv_decode_workspace_bytes": (c_size_t, [_P, c_int64]),
    "ee_kv_decode_attention": (c_int, [_P, _P, c_int64, c_int64, _P, _P, c_int64, c_float, _P, c_int64, _P, _P,
                                       c_size_t, _P]),
    "ee_add_rmsnorm": (c_int, [_P, c_int64, _P, c_int64, _P, c_int64, _P, c_float, _P, c_int64, c_int64, c_int64,
                               _P]),
    "ee_route": (c_int, [_P, c_int64, c_double, c_double, _P, _P]),
    "ee_route_batch_max": (c_int, [_P, c_int64, c_double, c_double, _P, _P, _P]),
    "ee_quantize_weights_int8": (c_int, [_P, c_int64, c_int64, c_int64, _P, _P, _P, c_int, _P]),
    "ee_pack_weights": (c_int, [_P, _P, c_int64, c_int64, _P, _P, _P, _P]),
    "ee_quant_rows_int8": (c_int, [_P, c_int64, c_int64, c_int64, _P, _P, _P]),
    "ee_quant_rows_e4m3": (c_int, [_P, c_int64, c_int64, c_int64, _P, _P, _P]),
    "ee_gemm_int8": (c_int, [_P, _P, _P, _P, _P, c_int64, c_int64, c_int64, c_int64, _P]),
    "ee_gemm_fp8": (c_int, [_P, _P, _P, _P, _P, c_int64, c_int64, c_int64, c_int64, _P]),
    "ee_gemm_fp16": (c_int, [_P, _P, _P, c_int64, c_int64, c_int64, c_int64, _P]),
    "ee_gemm_int8_acc": (c_int, [_P, _P, _P, c_int64, c_int64, c_int64, _P]),
    "ee_gemm_fp8_acc": (c_int, [_P, _P, _P, c_int64, c_int64, c_int64, _P]),
    "ee_gemm_fp16_acc": (c_int, [_P, _P, _P, c_int64, c_int64, c_int64, _P]),
    "ee_linear_workspace_bytes": (c_size_t, [c_int64, c_int64]),
    "ee_linear_int8": (c_int, [_P, c_int64, _P, _P, _P, c_int64, c_int64, c_int64, c_int64, _P, c_size_t, _P]),
    "ee_linear_fp8": (c_int, [_P, c_int64, _P, _P, _P, c_int64, c_int64, c_int64, c_int64, _P, c_size_t, _P]),
    "ee_linear_int8_noalloc": (c_int, [_P, c_int64, _P, _P, _P, c_int64, c_int64, c_int64, c_int64, _P]),
    "ee_gated_workspace_bytes": (c_size_t, [c_int64, c_int64]),
    "ee_gated_workspace_split_bytes": (c_size_t, [c_int64, c_int64]),
    "ee_gate_rows": (c_int, [_P, c_int64, c_int64, c_int64, c_double, c_double, _P, _P, _P, _P, c_size_t, _P]),
    "ee_gate_rows_keep": (c_int, [_P, c_int64, c_int64, c_int64, c_double, c_double, _P, _P, _P, _P, c_size_t, _P]),
    "ee_gated_workspace_head_bytes": (c_size_t, []),
    "ee_gate_entropies": (c_int, [_P, c_int64, c_double, c_double, _P, _P, _P, c_size_t, _P]),
    "ee_gated_gemm": (c_int, [_P, c_int64, c_int64, c_int64, _P, _P, _P, _P, c_int64, _P, c_int64, _P, c_size_t,
                              _P]),
    "ee_gated_pack": (c_int, [_P, c_int64, c_int64, c_int64, _P, c_size_t, _P]),
    "ee_gated_gemm_packed": (c_int, [c_int64, c_int64, _P, _P, _P, _P, c_int64, _P, c_int64, _P, c_size_t, _P]),
    "ee_gated_swiglu_packed": (c_int, [c_int64, c_int64, _P, _P, _P, _P, c_int64, _P, c_int64, _P, c_size_t, _P]),
    "ee_gated_workspace_layout": (c_int, [c_int64, c_int64, POINTER(c_int64)]),
    "ee_engine_workspace_bytes": (c_size_t, [c_int64, c_int32, _P]),
    "ee_engine_create": (c_int, [c_int64, c_double, c_double, c_int32, _P, _P, c_size_t, _P]),
    "ee_engine_run": (c_int, [_P, _P]),
    "ee_engine_capture": (c_int, [_P, _P]),
    "ee_engine_launch": (c_int, [_P, _P]),
    "ee_engine_destroy": (c_int, [_P]),
    "ee_decoder_workspace_bytes": (c_size_t, [_P]),
    "ee_decoder_create": (c_int, [_P, c_int32, _P, _P, _P, _P, _P, _P, c_size_t, _P]),
    "ee_decoder_run": (c_int, [_P, _P, _P, _P, _P]),
    "ee_decoder_capture": (c_int, [_P, _P, _P, _P, _P]),
    "ee_decoder_launch": (c_int, [_P, _P]),
    "ee_decoder_destroy": (c_int, [_P]),
    "ee_gated_linear": (c_int, [_P, c_int64, c_int64, _P, c_int64, c_int64, c_int64, _P, _P, _P, _P, c_int64,
                                c_double, c_double, _P, _P, _P, _P, c_int64, _P, c_size_t, _P]),
}

_lib = None


def load(path: str = LIB_PATH) -> ctypes.CDLL:
    """Load the library once and attach the declared signatures."""
    global _lib
    if _lib is not None:
        return _lib
    if not os.path.exists(path):
        raise ImportError(
            f"{path} is missing: build it with `python triton-kernels-optimization_b200/build.py` "
            "(there is no CPU fallback)")
    lib = ctypes.CDLL(path)
    for name, (res, args) in SIGNATURES.items():
        fn = getattr(lib, name)
        fn.restype = res
        fn.argtypes = args
    _lib = lib
    return lib


def last_error() -> str:
    msg = load().ee_last_error()
    return msg.decode() if msg else ""


def check(status: int, what: str) -> None:
    if status != EE_OK:
        raise RuntimeError(f"{what}: {STATUS_NAMES.get(status, status)}: {last_error()}")


def call(name: str, *args) -> None:
    """Invoke an int-returning entry point and raise on a non-zero status."""
    check(getattr(load(), name)(*args), name)


# Bumped whenever device_check finds the error word set: a kernel that gave up may have
# left a gated workspace's header (bucket counters, tile scheduler words) dirty, so every
# EntropyRouter re-zeroes its header on its next route when the count has moved.
error_epoch = 0


def device_check() -> int:
    """Read and clear the current device's error word; raise if it was set (after
    marking every router's workspace header for re-zeroing)."""
    global error_epoch
    v = c_int(0)
    st = load().ee_device_check(ctypes.byref(v))
    if v.value != 0:
        error_epoch += 1
    check(st, "ee_device_check")
    return v.value
