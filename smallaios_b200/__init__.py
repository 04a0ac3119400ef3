"""smallaios_b200 -- B200-native (sm_100a) LLM decode hot path of SmallAIOS onnx-rt.

GroupQueryAttention over a PolarQuant-compressed KV cache (quantize-on-append
with fused RoPE, attention that dequantizes inside the kernel) and the int4
MatMulNBits GEMV/GEMM, behind the C ABI in include/sa_b200.h
(libsa_b200.so).  This package is the host-side mirror of the reference's
operator interface; all compute runs in the CUDA library.
"""
from .kv_cache import DEFAULT_SEED, GpuKvCache, LayerView, qjl_correction
from .ops import (CapacityError, InternalError, InvalidAttribute, KvCacheDispatchCtx, OpError, PackedNBitsWeight,
                  ShapeMismatch, UnsupportedOp, dispatch_gpu_node, finalize_kv_cache, gqa_attend,
                  group_query_attention, matmul_nbits, matmul_nbits_packed, qkv_project_append, rms_norm,
                  rotary_device_status, rotary_embedding, silu_mul, supports_op)
from .layer import LayerWeights, decoder_layer_step, prefill_layer_step

__all__ = [
    "DEFAULT_SEED", "GpuKvCache", "LayerView", "CapacityError", "InternalError", "InvalidAttribute",
    "KvCacheDispatchCtx", "OpError", "ShapeMismatch", "UnsupportedOp", "dispatch_gpu_node", "finalize_kv_cache",
    "gqa_attend", "group_query_attention", "matmul_nbits", "matmul_nbits_packed", "PackedNBitsWeight",
    "qkv_project_append", "rms_norm", "silu_mul", "supports_op", "LayerWeights", "decoder_layer_step", "prefill_layer_step",
    "qjl_correction", "rotary_embedding", "rotary_device_status",
]
