"""Entropy-gated mixed-precision engine for B200 (sm_100a).

Drop-in for the hot path of IqtedarU/triton-kernels-optimization (entropy-engine):
the reference's operator names (``triton_int8_gemm``, ``triton_fp8_gemm``,
``triton_fp16_gemm``, ``fused_softmax_entropy``, ``quantize_weights_int8``,
``PrecisionTier``, ``PipelinedEntropyDispatcher``, ``EntropyDispatchedLinear``,
``EntropyDispatchedLlamaBlock``, ``build_dispatched_llama``, ``CubinEngine``) backed by
hand-written tcgen05 / TMA kernels behind the C ABI of
``libee_b200.so`` (include/ee_b200.h).  The package directory name contains dashes,
so it is imported through ``__graft_entry__.load_package()`` (module name
``tko_b200``).
"""
from . import _lib, kvcache, packfile, sharding
from .kvcache import EntropyKVCache
from .dispatch import (
    EntropyDispatchedLinear,
    EntropyRouter,
    PipelinedEntropyDispatcher,
    PrecisionTier,
    gated_linear,
    tier_of,
)
from .engine import CubinEngine, DecoderEngine, GatedLayerEngine
from .llama import EntropyDispatchedLlamaBlock, build_dispatched_llama, dispatched_forward, eval_dispatched
from .kernels import (
    SwiGLUPack,
    WeightPack,
    add_rmsnorm,
    attention_entropy,
    flash_attention_entropy,
    flash_attention_rope_entropy,
    fused_softmax_entropy,
    gemm_accumulators,
    gemm_int8_prequant,
    head_mean_entropy,
    linear_f16,
    pack_for,
    quant_rows_e4m3,
    quant_rows_int8,
    quantize_weights_int8,
    softmax_entropy_rows,
    triton_fp8_gemm,
    triton_fp16_gemm,
    triton_int8_gemm,
)

LIB_PATH = _lib.LIB_PATH


def load_library():
    """Load libee_b200.so (raises ImportError when it has not been built)."""
    return _lib.load()
