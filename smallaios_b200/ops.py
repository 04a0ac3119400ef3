"""Operator-level API: the onnx-rt operators of the decode hot path on B200.

Mirrors the reference's operator interface for this path:
  * ``group_query_attention`` -- com.microsoft.GroupQueryAttention as the GPU
    executor dispatches it with a KV cache (dispatch_gqa / gqa_with_cache,
    onnx-rt/src/cuda/gpu_executor.rs:917-968; attribute parsing and
    validation as op_group_query_attention, ops/microsoft.rs:1082-1196 and
    the CPU arm executor.rs:2341-2362).
  * ``matmul_nbits`` -- com.microsoft.MatMulNBits (ORT contract; the reference
    has no such op and would register it next to MatMul in
    dispatch_gpu_node, gpu_executor.rs:490-514).
  * ``dispatch_gpu_node`` / ``KvCacheDispatchCtx`` / ``finalize_kv_cache`` --
    the executor-side glue (gpu_executor.rs:277-280, 422, 490-514).

Errors map the library's status codes onto the reference's OpError variants.
"""
from __future__ import annotations

from dataclasses import dataclass, field

import torch

from . import _lib
from ._lib import lib
from .kv_cache import GpuKvCache


# ---- OpError mirror (onnx-rt/src/operators.rs) ------------------------------
class OpError(RuntimeError):
    pass


class InvalidAttribute(OpError):
    pass


class ShapeMismatch(OpError):
    pass


class UnsupportedOp(OpError):
    pass


class InternalError(OpError):
    """CUDA failures, as the GPU executor wraps CudaError (gpu_executor.rs:963)."""


class CapacityError(InternalError):
    """kv_cache_append:position_overflow (kv_cache.rs:246-251)."""


_STATUS_TO_ERROR = {
    _lib.SA_ERR_INVALID_ATTRIBUTE: InvalidAttribute,
    _lib.SA_ERR_SHAPE_MISMATCH: ShapeMismatch,
    _lib.SA_ERR_UNSUPPORTED: UnsupportedOp,
    _lib.SA_ERR_CAPACITY: CapacityError,
    _lib.SA_ERR_INVALID_ARGUMENT: InvalidAttribute,
}


def _raise_op(status: int, op: str) -> None:
    if status == _lib.SA_OK:
        return
    msg = lib.sa_last_error_string().decode(errors="replace")
    cls = _STATUS_TO_ERROR.get(status, InternalError)
    raise cls(f"{op}: {msg} [{lib.sa_status_string(status).decode()}]")


_DTYPES = {torch.float32: _lib.SA_DTYPE_FLOAT, torch.float16: _lib.SA_DTYPE_FLOAT16,
           torch.bfloat16: _lib.SA_DTYPE_BFLOAT16}


def _dtype_code(t: torch.Tensor) -> int:
    try:
        return _DTYPES[t.dtype]
    except KeyError:
        raise UnsupportedOp(f"dtype {t.dtype} not supported") from None


def _stream_handle(stream, device) -> int:
    if stream is None:
        stream = torch.cuda.current_stream(device)
    return stream.cuda_stream if hasattr(stream, "cuda_stream") else int(stream)


def _cuda(t, what):
    if t is None:
        return None
    if not isinstance(t, torch.Tensor) or not t.is_cuda:
        raise TypeError(f"{what} must be a CUDA tensor")
    if not t.is_contiguous():
        raise ValueError(f"{what} must be contiguous")
    return t


def _rope_tables(cos_cache, sin_cache):
    for name, t in (("cos_cache", cos_cache), ("sin_cache", sin_cache)):
        if t is not None:
            _cuda(t, name)
            if t.dtype != torch.float32:
                raise UnsupportedOp(f"{name} must be float32")
            if t.dim() != 2:
                raise ShapeMismatch("apply_rope_in_place: cos/sin caches must be rank-2")
    if cos_cache is not None and sin_cache is not None and cos_cache.shape[1] != sin_cache.shape[1]:
        raise ShapeMismatch("apply_rope_in_place: cos and sin caches must share the inner dim")
    return (0 if cos_cache is None else cos_cache.shape[0])


def group_query_attention(query: torch.Tensor, key: torch.Tensor, value: torch.Tensor, cache: GpuKvCache,
                          layer: int, *, num_heads: int, kv_num_heads: int, scale: float | None = None,
                          local_window_size: int = -1, do_rotary: bool = True, rotary_interleaved: bool = False,
                          cos_cache: torch.Tensor | None = None, sin_cache: torch.Tensor | None = None,
                          out: torch.Tensor | None = None, stream=None) -> torch.Tensor:
    """GroupQueryAttention with ``cache`` as past K/V; returns attn_out (B, S, Hq_local*D).

    ``key``/``value`` (B, S, Hkv_local*D) are quantized into the cache at the
    current position (RoPE'd when ``do_rotary``); the query attends causally to
    every cached token up to its own position.  The position is not advanced
    (call ``finalize_kv_cache`` / ``cache.advance_position`` once per forward
    pass, as the reference executor does).
    """
    if query is None:
        raise ShapeMismatch("GroupQueryAttention: missing query")
    if key is None:
        raise ShapeMismatch("GroupQueryAttention: missing key")
    if value is None:
        raise ShapeMismatch("GroupQueryAttention: missing value")
    for name, t in (("query", query), ("key", key), ("value", value)):
        _cuda(t, name)
        if t.dim() != 3:
            raise ShapeMismatch("GroupQueryAttention: Q/K/V must be rank-3")
    if key.shape != value.shape:
        raise ShapeMismatch("GroupQueryAttention: key and value must have the same shape")
    if not (query.dtype == key.dtype == value.dtype):
        raise UnsupportedOp("GroupQueryAttention: Q/K/V dtypes differ")
    cfg = cache.config
    if num_heads > 0 and kv_num_heads > 0 and num_heads % kv_num_heads == 0:
        d = cfg.head_dim
        g = num_heads // kv_num_heads
        if query.shape[2] != g * cfg.kv_head_count * d or key.shape[2] != cfg.kv_head_count * d:
            raise ShapeMismatch("GroupQueryAttention: hidden sizes do not match the cache's heads/head_dim")
        if query.shape[:2] != key.shape[:2]:
            raise ShapeMismatch("GroupQueryAttention: Q and K batch/sequence differ")
    rows = _rope_tables(cos_cache, sin_cache)
    if out is None:
        out = torch.empty_like(query)
    rc = lib.sa_group_query_attention(
        cache.handle, layer, query.data_ptr(), key.data_ptr(), value.data_ptr(), out.data_ptr(),
        _dtype_code(query), query.shape[0], query.shape[1], int(num_heads), int(kv_num_heads),
        int(scale is not None), float(scale or 0.0), int(local_window_size), int(bool(do_rotary)),
        int(bool(rotary_interleaved)), None if cos_cache is None else cos_cache.data_ptr(),
        None if sin_cache is None else sin_cache.data_ptr(), rows, _stream_handle(stream, query.device))
    _raise_op(rc, "GroupQueryAttention")
    return out


def gqa_attend(query: torch.Tensor, cache: GpuKvCache, layer: int, *, num_heads: int, scale: float | None = None,
               do_rotary: bool = True, rotary_interleaved: bool = False, cos_cache=None, sin_cache=None,
               out=None, stream=None) -> torch.Tensor:
    """Attention only (no append): queries at positions [p, p+S) over cache tokens [0, p+S)."""
    _cuda(query, "query")
    rows = _rope_tables(cos_cache, sin_cache)
    if out is None:
        out = torch.empty_like(query)
    rc = lib.sa_gqa_attend(cache.handle, layer, query.data_ptr(), out.data_ptr(), _dtype_code(query),
                           query.shape[0], query.shape[1], int(num_heads), int(scale is not None),
                           float(scale or 0.0), None if cos_cache is None else cos_cache.data_ptr(),
                           None if sin_cache is None else sin_cache.data_ptr(), rows, int(bool(do_rotary)),
                           int(bool(rotary_interleaved)), _stream_handle(stream, query.device))
    _raise_op(rc, "gqa_attend")
    return out


def matmul_nbits(a: torch.Tensor, b: torch.Tensor, scales: torch.Tensor, zero_points: torch.Tensor | None = None,
                 bias: torch.Tensor | None = None, *, K: int, N: int, bits: int = 4, block_size: int = 32,
                 out: torch.Tensor | None = None, stream=None) -> torch.Tensor:
    """com.microsoft.MatMulNBits: Y[..., N] = A[..., K] . dequant(B)^T (+ bias)."""
    _cuda(a, "A")
    _cuda(b, "B")
    _cuda(scales, "scales")
    _cuda(zero_points, "zero_points")
    _cuda(bias, "bias")
    if bits != 4:
        raise UnsupportedOp(f"MatMulNBits: bits={bits} not supported (4 only)")
    if a.shape[-1] != K:
        raise ShapeMismatch(f"MatMulNBits: A inner dim {a.shape[-1]} != K={K}")
    if b.dtype != torch.uint8:
        raise UnsupportedOp("MatMulNBits: B must be uint8")
    if scales.dtype != a.dtype:
        raise UnsupportedOp("MatMulNBits: scales must have A's dtype")
    if zero_points is not None and zero_points.dtype != torch.uint8:
        raise UnsupportedOp("MatMulNBits: only packed uint8 zero_points are supported")
    nblk = (K + block_size - 1) // block_size
    if b.numel() != N * nblk * (block_size * bits // 8):
        raise ShapeMismatch("MatMulNBits: B size does not match (N, k_blocks, blob_size)")
    if scales.numel() != N * nblk:
        raise ShapeMismatch("MatMulNBits: scales size does not match N * k_blocks")
    m = a.numel() // K
    if out is None:
        out = torch.empty(*a.shape[:-1], N, dtype=a.dtype, device=a.device)
    rc = lib.sa_matmul_nbits(a.data_ptr(), b.data_ptr(), scales.data_ptr(),
                             None if zero_points is None else zero_points.data_ptr(),
                             None if bias is None else bias.data_ptr(), out.data_ptr(), _dtype_code(a), m, N, K,
                             bits, block_size, _stream_handle(stream, a.device))
    _raise_op(rc, "MatMulNBits")
    return out


def qkv_project_append(x: torch.Tensor, w_codes: torch.Tensor, w_scales: torch.Tensor, cache: GpuKvCache,
                       layer: int, *, do_rotary: bool = True, rotary_interleaved: bool = False, cos_cache=None,
                       sin_cache=None, q_out=None, k_out=None, v_out=None, stream=None):
    """Fused QKV projection of a decode step (sa_qkv_project_append).

    ``x`` (B, hidden) fp16/bf16; ``w_codes`` uint8 (n, hidden/32, 16) and
    ``w_scales`` (n, hidden/32) in x's dtype are the packed Wq/Wk/Wv
    MatMulNBits weights of this cache's heads (n = (Hq + 2*Hkv)*D, block 32,
    zero point 8).  Returns ``(q, k, v)``: q (B, Hq*D) with RoPE applied at the
    cache position, k and v (B, Hkv*D) as projected.  RoPE(k) and v are
    appended to ``layer`` at the cache position (not advanced).  The attention
    then runs with ``gqa_attend(q, ..., do_rotary=False)``.
    """
    for name, t in (("x", x), ("w_codes", w_codes), ("w_scales", w_scales)):
        _cuda(t, name)
    if x.dim() != 2:
        raise ShapeMismatch("qkv_project_append: x must be (batch, hidden)")
    if w_codes.dtype != torch.uint8:
        raise UnsupportedOp("qkv_project_append: w_codes must be uint8")
    if w_scales.dtype != x.dtype:
        raise UnsupportedOp("qkv_project_append: w_scales must have x's dtype")
    cfg = cache.config
    b, hidden = x.shape
    d = cfg.head_dim
    hkv = cfg.kv_head_count
    hq = hkv * (cfg.num_heads // cfg.num_kv_heads)
    n = (hq + 2 * hkv) * d
    if w_codes.numel() != n * hidden // 2 or w_scales.numel() != n * (hidden // 32):
        raise ShapeMismatch("qkv_project_append: weights do not match ((Hq + 2*Hkv)*D, hidden)")
    rows = _rope_tables(cos_cache, sin_cache)
    if q_out is None:
        q_out = torch.empty(b, hq * d, dtype=x.dtype, device=x.device)
    if k_out is None:
        k_out = torch.empty(b, hkv * d, dtype=x.dtype, device=x.device)
    if v_out is None:
        v_out = torch.empty(b, hkv * d, dtype=x.dtype, device=x.device)
    rc = lib.sa_qkv_project_append(cache.handle, layer, x.data_ptr(), w_codes.data_ptr(), w_scales.data_ptr(),
                                   _dtype_code(x), b, hidden, None if cos_cache is None else cos_cache.data_ptr(),
                                   None if sin_cache is None else sin_cache.data_ptr(), rows, int(bool(do_rotary)),
                                   int(bool(rotary_interleaved)), q_out.data_ptr(), k_out.data_ptr(),
                                   v_out.data_ptr(), _stream_handle(stream, x.device))
    _raise_op(rc, "qkv_project_append")
    return q_out, k_out, v_out


def rms_norm(x: torch.Tensor, weight: torch.Tensor, *, skip: torch.Tensor | None = None,
             bias: torch.Tensor | None = None, epsilon: float = 1e-5, out: torch.Tensor | None = None,
             pre_out: torch.Tensor | None = None, stream=None):
    """SkipSimplifiedLayerNormalization / SimplifiedLayerNormalization over the last axis.

    Returns ``(y, pre)``: ``pre = x + skip (+ bias)`` (``x`` itself when there
    is no skip or bias), ``y = pre / sqrt(mean(pre^2) + epsilon) * weight``.
    """
    for name, t in (("x", x), ("weight", weight), ("skip", skip), ("bias", bias)):
        _cuda(t, name)
    cols = x.shape[-1]
    if weight.numel() != cols or (bias is not None and bias.numel() != cols):
        raise ShapeMismatch("RMSNormalization: scale must match normalized region")
    if skip is not None and skip.shape != x.shape:
        raise ShapeMismatch("SkipSimplifiedLayerNormalization: x and skip must have matching shapes")
    for name, t in (("weight", weight), ("skip", skip), ("bias", bias)):
        if t is not None and t.dtype != x.dtype:
            raise UnsupportedOp(f"rms_norm: {name} must have x's dtype")
    if out is None:
        out = torch.empty_like(x)
    need_pre = skip is not None or bias is not None
    if need_pre and pre_out is None:
        pre_out = torch.empty_like(x)
    rc = lib.sa_rms_norm(x.data_ptr(), None if skip is None else skip.data_ptr(),
                         None if bias is None else bias.data_ptr(), weight.data_ptr(), out.data_ptr(),
                         pre_out.data_ptr() if need_pre else None, _dtype_code(x), x.numel() // cols, cols,
                         float(epsilon), _stream_handle(stream, x.device))
    _raise_op(rc, "RMSNormalization")
    return out, (pre_out if need_pre else x)


def silu_mul(gate: torch.Tensor, up: torch.Tensor | None = None, *, out: torch.Tensor | None = None, stream=None):
    """SwiGLU: Silu(gate) * up.  With ``up`` None, ``gate`` is one packed (rows, 2F)
    gate|up projection (gate in the first F columns)."""
    _cuda(gate, "gate")
    if up is None:
        rows, two_f = gate.shape[0], gate.shape[-1]
        if two_f % 2:
            raise ShapeMismatch("silu_mul: a packed gate|up projection has an even width")
        f, ld = two_f // 2, two_f
        g_ptr, u_ptr = gate.data_ptr(), gate.data_ptr() + f * gate.element_size()
    else:
        _cuda(up, "up")
        if up.shape != gate.shape or up.dtype != gate.dtype:
            raise ShapeMismatch("silu_mul: gate and up must have the same shape and dtype")
        rows, f = gate.shape[0], gate.shape[-1]
        ld, g_ptr, u_ptr = f, gate.data_ptr(), up.data_ptr()
    if out is None:
        out = torch.empty(rows, f, dtype=gate.dtype, device=gate.device)
    rc = lib.sa_silu_mul(g_ptr, u_ptr, ld, out.data_ptr(), _dtype_code(gate), rows, f,
                         _stream_handle(stream, gate.device))
    _raise_op(rc, "silu_mul")
    return out


_POS_DTYPES = {torch.int64: 7, torch.int32: 6}
_ROTARY_STATUS: dict = {}  # device index -> int32 device word that rotary_embedding calls flag


def rotary_device_status(device=None, clear: bool = True) -> int:
    """Bit 0 set when a ``rotary_embedding`` call on ``device`` met a position id outside its
    cos/sin table (that row was passed through unrotated).  Synchronises with the device."""
    dev = torch.device(device if device is not None else "cuda")
    idx = dev.index if dev.index is not None else torch.cuda.current_device()
    word = _ROTARY_STATUS.get(idx)
    if word is None:
        return 0
    v = int(word.item())
    if clear:
        word.zero_()
    return v


def _rotary_status_word(device) -> torch.Tensor:
    idx = device.index if device.index is not None else torch.cuda.current_device()
    word = _ROTARY_STATUS.get(idx)
    if word is None:
        word = _ROTARY_STATUS[idx] = torch.zeros(1, dtype=torch.int32, device=torch.device("cuda", idx))
    return word


def rotary_embedding(x: torch.Tensor, cos_cache: torch.Tensor, sin_cache: torch.Tensor, *,
                     position_ids: torch.Tensor | None = None, position: int = 0, interleaved: bool = False,
                     num_heads: int | None = None, rotary_embedding_dim: int = 0, out: torch.Tensor | None = None,
                     stream=None) -> torch.Tensor:
    """com.microsoft.RotaryEmbedding on the GPU (rotary_gpu, onnx-rt/src/cuda/kernels/rotary.rs:274-346;
    arithmetic and partial rotation as op_rotary_embedding / apply_rope_in_place,
    ops/microsoft.rs:137-231, 556-650).

    ``x``: rank-4 ``(B, H, S, D)`` or rank-3 ``(B, S, H*D)`` (then ``num_heads`` is needed).
    Without ``position_ids`` token s uses table row ``position + s`` (the executor passes the
    cache's current position); with ``position_ids`` (``S`` or ``B*S`` int32/int64 entries, read on
    the device) token (b, s) uses its own id.  Returns a new tensor unless ``out`` is given
    (``out`` may be ``x``).
    """
    _cuda(x, "X")
    for name, t in (("cos_cache", cos_cache), ("sin_cache", sin_cache)):
        _cuda(t, name)
        if t.dtype not in (torch.float32, torch.bfloat16):
            raise UnsupportedOp("rotary_gpu: cos/sin tables must be Float or BFloat16")
        if t.dim() != 2:
            raise ShapeMismatch("apply_rope_in_place: cos/sin caches must be rank-2")
    if cos_cache.shape != sin_cache.shape or cos_cache.dtype != sin_cache.dtype:
        raise ShapeMismatch("rotary_gpu: cos/sin tables must share max_seq_len and inner dim")
    if x.dim() == 4:
        layout, (b, h, s, d) = 0, x.shape
    elif x.dim() == 3:
        if num_heads is None or num_heads <= 0:
            raise InvalidAttribute("RotaryEmbedding: num_heads must be > 0 for rank-3 input")
        b, s, hidden = x.shape
        if hidden % num_heads:
            raise ShapeMismatch("RotaryEmbedding: hidden not divisible by num_heads")
        layout, h, d = 1, num_heads, hidden // num_heads
    else:
        raise ShapeMismatch("RotaryEmbedding: input must be rank-3 or rank-4")
    pos_ptr, pos_dtype, pos_count = None, 0, 0
    if position_ids is not None:
        if position_ids.dtype not in _POS_DTYPES:
            raise ShapeMismatch("RotaryEmbedding: position_ids must be int32 or int64")
        if not position_ids.is_cuda:
            position_ids = position_ids.to(x.device, non_blocking=True)
        position_ids = position_ids.contiguous()
        pos_ptr, pos_dtype, pos_count = position_ids.data_ptr(), _POS_DTYPES[position_ids.dtype], position_ids.numel()
    if out is None:
        out = torch.empty_like(x)
    elif out.shape != x.shape or out.dtype != x.dtype or not out.is_contiguous():
        raise ShapeMismatch("RotaryEmbedding: out must be a contiguous tensor of x's shape and dtype")
    status = _rotary_status_word(x.device) if position_ids is not None else None
    rc = lib.sa_rotary_embedding(x.data_ptr(), out.data_ptr(), _dtype_code(x), layout, b, h, s, d,
                                 cos_cache.data_ptr(), sin_cache.data_ptr(), _dtype_code(cos_cache),
                                 cos_cache.shape[0], cos_cache.shape[1], pos_ptr, pos_dtype, pos_count, int(position),
                                 int(bool(interleaved)), int(rotary_embedding_dim),
                                 None if status is None else status.data_ptr(), _stream_handle(stream, x.device))
    _raise_op(rc, "RotaryEmbedding")
    return out


class PackedNBitsWeight:
    """A MatMulNBits weight repacked once for the decode GEMV (``sa_matmul_nbits_prepack``).

    Holds the packed device buffer; ``matmul_nbits_packed`` consumes it.  The
    packed path needs fp16/bf16 scales, block 32, the default zero point, N a
    multiple of 32 and K a multiple of 1024.
    """

    def __init__(self, b: torch.Tensor, scales: torch.Tensor, *, K: int, N: int, bits: int = 4,
                 block_size: int = 32, stream=None):
        _cuda(b, "B")
        _cuda(scales, "scales")
        nbytes = lib.sa_matmul_nbits_packed_bytes(N, K, bits, block_size, _dtype_code(scales))
        if nbytes <= 0:
            raise UnsupportedOp("MatMulNBits prepack: no packed path for this dtype/shape/block size")
        self.K, self.N, self.bits, self.block_size, self.dtype = K, N, bits, block_size, scales.dtype
        self.packed = torch.empty(nbytes, dtype=torch.uint8, device=b.device)
        rc = lib.sa_matmul_nbits_prepack(b.data_ptr(), scales.data_ptr(), self.packed.data_ptr(),
                                         _dtype_code(scales), N, K, bits, block_size,
                                         _stream_handle(stream, b.device))
        _raise_op(rc, "MatMulNBits prepack")


def matmul_nbits_packed(a: torch.Tensor, w: PackedNBitsWeight, bias: torch.Tensor | None = None, *,
                        out: torch.Tensor | None = None, stream=None) -> torch.Tensor:
    """MatMulNBits (m <= 8 rows) against a ``PackedNBitsWeight``: same result as ``matmul_nbits``."""
    _cuda(a, "A")
    _cuda(bias, "bias")
    if a.shape[-1] != w.K:
        raise ShapeMismatch(f"MatMulNBits: A inner dim {a.shape[-1]} != K={w.K}")
    if a.dtype != w.dtype:
        raise UnsupportedOp("MatMulNBits: A must have the packed scales' dtype")
    m = a.numel() // w.K
    if out is None:
        out = torch.empty(*a.shape[:-1], w.N, dtype=a.dtype, device=a.device)
    rc = lib.sa_matmul_nbits_packed(a.data_ptr(), w.packed.data_ptr(), None if bias is None else bias.data_ptr(),
                                    out.data_ptr(), _dtype_code(a), m, w.N, w.K, w.bits, w.block_size,
                                    _stream_handle(stream, a.device))
    _raise_op(rc, "MatMulNBits")
    return out


# ---- executor glue ------------------------------------------------------------
SUPPORTED_OPS = ("GroupQueryAttention", "MatMulNBits", "RMSNormalization", "RotaryEmbedding",
                 "SimplifiedLayerNormalization", "SkipSimplifiedLayerNormalization")


def supports_op(op_type: str) -> bool:
    """CudaRuntime::supports_op (onnx-rt/src/cuda/mod.rs:874-889) for this path."""
    return op_type in SUPPORTED_OPS


@dataclass
class KvCacheDispatchCtx:
    """KvCacheDispatchCtx (gpu_executor.rs:277-280)."""

    cache: GpuKvCache
    next_layer_idx: int = 0
    rope: dict = field(default_factory=dict)  # optional cos_cache / sin_cache tensors


def dispatch_gpu_node(op_type: str, inputs: list, attrs: dict, kv_cache_ctx: KvCacheDispatchCtx | None = None):
    """dispatch_gpu_node (gpu_executor.rs:490-514) for the ops of this path.

    GroupQueryAttention inputs follow the ORT order (query, key, value,
    past_key, past_value, seqlens_k, total_sequence_length, cos_cache,
    sin_cache); past K/V come from the cache, so inputs 3-6 are ignored as in
    the reference GPU executor.  Returns the list of outputs ([attn_out]).
    """
    if op_type == "GroupQueryAttention":
        if kv_cache_ctx is None:
            raise InternalError("GroupQueryAttention on this path needs a KV cache context")
        inp = list(inputs) + [None] * (9 - len(inputs))
        layer = kv_cache_ctx.next_layer_idx
        kv_cache_ctx.next_layer_idx += 1
        scale = attrs.get("scale")
        out = group_query_attention(
            inp[0], inp[1], inp[2], kv_cache_ctx.cache, layer,
            num_heads=int(attrs.get("num_heads", 0)), kv_num_heads=int(attrs.get("kv_num_heads", 0)),
            scale=None if scale is None else float(scale),
            local_window_size=int(attrs.get("local_window_size", -1)),
            do_rotary=bool(int(attrs.get("do_rotary", 1))),
            rotary_interleaved=bool(int(attrs.get("rotary_interleaved", 0))),
            cos_cache=inp[7] if inp[7] is not None else kv_cache_ctx.rope.get("cos_cache"),
            sin_cache=inp[8] if inp[8] is not None else kv_cache_ctx.rope.get("sin_cache"))
        return [out]
    if op_type == "RotaryEmbedding":
        # inputs [X, position_ids, cos_cache, sin_cache] (com.microsoft) or [X, cos_cache, sin_cache]
        # (the gemma builder); resolve_rotary_inputs, gpu_executor.rs:719-759
        x = inputs[0]
        if len(inputs) >= 4:
            pos_ids, cos, sin = inputs[1], inputs[2], inputs[3]
        else:
            pos_ids, cos, sin = None, inputs[1], inputs[2]
        if x is None or cos is None or sin is None:
            raise ShapeMismatch("RotaryEmbedding: missing input")
        # no explicit ids: the cache's current position (pick_rotary_position, :761-773), read on the host
        position = kv_cache_ctx.cache.current_position() if (pos_ids is None and kv_cache_ctx is not None) else 0
        num_heads = attrs.get("num_heads")
        if x.dim() == 3 and num_heads is None:  # rotary_num_heads_for_rank3, :794-811
            hd = cos.shape[-1] * 2
            num_heads = x.shape[2] // hd if hd > 0 and x.shape[2] % hd == 0 else None
        return [rotary_embedding(x, cos, sin, position_ids=pos_ids, position=position,
                                 interleaved=bool(int(attrs.get("interleaved", 0))),
                                 num_heads=None if num_heads is None else int(num_heads),
                                 rotary_embedding_dim=int(attrs.get("rotary_embedding_dim", 0)))]
    if op_type in ("RMSNormalization", "SimplifiedLayerNormalization"):
        # inputs (X, scale[, bias]); attributes epsilon (1e-5), axis (-1: the last axis only)
        if int(attrs.get("axis", -1)) not in (-1, inputs[0].dim() - 1):
            raise InvalidAttribute(f"{op_type}: only the last axis is normalized on this path")
        inp = list(inputs) + [None] * (3 - len(inputs))
        y, _ = rms_norm(inp[0], inp[1], bias=inp[2], epsilon=float(attrs.get("epsilon", 1e-5)))
        return [y]
    if op_type == "SkipSimplifiedLayerNormalization":
        # inputs (input, skip, gamma[, bias]) -> [output, input_skip_bias_sum]
        inp = list(inputs) + [None] * (4 - len(inputs))
        y, pre = rms_norm(inp[0], inp[2], skip=inp[1], bias=inp[3], epsilon=float(attrs.get("epsilon", 1e-5)))
        return [y, pre]
    if op_type == "MatMulNBits":
        inp = list(inputs) + [None] * (6 - len(inputs))
        return [matmul_nbits(inp[0], inp[1], inp[2], inp[3], inp[5], K=int(attrs["K"]), N=int(attrs["N"]),
                             bits=int(attrs.get("bits", 4)), block_size=int(attrs.get("block_size", 32)))]
    raise InternalError(f"GPU executor: no GPU implementation for {op_type}")


def finalize_kv_cache(ctx: KvCacheDispatchCtx | None, tokens: int = 1) -> None:
    """finalize_kv_cache (gpu_executor.rs:422): one advance per forward pass."""
    if ctx is not None and ctx.next_layer_idx > 0:
        ctx.cache.advance_position(tokens)
