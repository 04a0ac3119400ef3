"""One decoder layer of a Llama-style model on this library's kernels (decode step).

The layer the reference's model loader wires (onnx-rt/src/model_loader/gemma.rs:13-36,
Llama without Gemma's embedding scale), one token per sequence:

    pre1 = x + resid                    h1 = RMSNorm(pre1) * input_norm     (SkipSimplifiedLayerNormalization)
    q, k, v = h1 . Wqkv^T, RoPE(q), RoPE(k) and v appended to the cache   (sa_qkv_project_append)
    a = GroupQueryAttention over the cache                               (sa_gqa_attend, rotary done)
    o = a . Wo^T                                                         (MatMulNBits)
    pre2 = o + pre1                     h2 = RMSNorm(pre2) * post_norm      (SkipSimplifiedLayerNormalization)
    g|u = h2 . Wgu^T                                                     (MatMulNBits, packed gate|up rows)
    m = Silu(g) * u                                                      (SwiGLU)
    d = m . Wdown^T                                                      (MatMulNBits)

and returns (d, pre2): the next layer adds them in its own first norm
(x = d, resid = pre2), so every residual add is fused into a norm.  All weights
are int4 MatMulNBits (block 32, zero point 8) with scales of the activation type.
The cache position is not advanced (once per forward pass, after the last layer).
"""
from __future__ import annotations

from dataclasses import dataclass

import torch

from .ops import gqa_attend, matmul_nbits, qkv_project_append, rms_norm, silu_mul


@dataclass
class LayerWeights:
    """Int4 MatMulNBits weights ([N][K/32][16] codes, [N][K/32] scales) of one layer."""

    wqkv_codes: torch.Tensor   # (Hq + 2*Hkv)*D rows: Wq, then Wk, then Wv
    wqkv_scales: torch.Tensor
    wo_codes: torch.Tensor     # hidden rows, K = Hq*D
    wo_scales: torch.Tensor
    wgu_codes: torch.Tensor    # 2*F rows: gate rows, then up rows, K = hidden
    wgu_scales: torch.Tensor
    wdown_codes: torch.Tensor  # hidden rows, K = F
    wdown_scales: torch.Tensor
    input_norm: torch.Tensor   # (hidden,)
    post_norm: torch.Tensor    # (hidden,)
    epsilon: float = 1e-5


def decoder_layer_step(x: torch.Tensor, resid: torch.Tensor | None, w: LayerWeights, cache, layer: int, *,
                       cos_cache=None, sin_cache=None, do_rotary: bool = True, rotary_interleaved: bool = False):
    """One decode step of one layer: ``x`` (B, hidden) plus residual ``resid`` (None for
    the first layer) -> ``(d, pre2)``, the input and residual of the next layer."""
    b, hidden = x.shape
    cfg = cache.config
    hq = cfg.kv_head_count * (cfg.num_heads // cfg.num_kv_heads)
    d_head = cfg.head_dim
    h1, pre1 = rms_norm(x, w.input_norm, skip=resid, epsilon=w.epsilon)
    q, _, _ = qkv_project_append(h1, w.wqkv_codes, w.wqkv_scales, cache, layer, do_rotary=do_rotary,
                                 rotary_interleaved=rotary_interleaved, cos_cache=cos_cache, sin_cache=sin_cache)
    a = gqa_attend(q.view(b, 1, hq * d_head), cache, layer, num_heads=hq, do_rotary=False)
    o = matmul_nbits(a.view(b, hq * d_head), w.wo_codes, w.wo_scales, K=hq * d_head, N=hidden)
    h2, pre2 = rms_norm(o, w.post_norm, skip=pre1, epsilon=w.epsilon)
    f2 = w.wgu_scales.shape[0]
    gu = matmul_nbits(h2, w.wgu_codes, w.wgu_scales, K=hidden, N=f2)
    m = silu_mul(gu)
    dn = matmul_nbits(m, w.wdown_codes, w.wdown_scales, K=f2 // 2, N=hidden)
    return dn, pre2


def prefill_layer_step(x: torch.Tensor, resid: torch.Tensor | None, w: LayerWeights, cache, layer: int, *,
                       batch: int, seq_len: int, cos_cache=None, sin_cache=None, do_rotary: bool = True,
                       rotary_interleaved: bool = False):
    """One layer over whole prompts: ``x`` (batch*seq_len, hidden) plus ``resid`` -> ``(d, pre2)``.

    The same layer as decoder_layer_step with every projection a tcgen05 MatMulNBits of
    batch*seq_len rows.  Q, K and V are three MatMulNBits calls on the row blocks of the packed
    Wqkv (GroupQueryAttention takes separate contiguous Q/K/V), and GroupQueryAttention appends
    the prompts' K/V at the cache position (RoPE, quantize-on-append) and runs the causal
    prefill attention of every query over them.  The position is not advanced.
    """
    m, hidden = x.shape
    if m != batch * seq_len:
        raise ValueError("prefill_layer_step: x must have batch * seq_len rows")
    from .ops import group_query_attention

    cfg = cache.config
    hkv = cfg.kv_head_count
    hq = hkv * (cfg.num_heads // cfg.num_kv_heads)
    d_head = cfg.head_dim
    qd, kd = hq * d_head, hkv * d_head
    h1, pre1 = rms_norm(x, w.input_norm, skip=resid, epsilon=w.epsilon)
    proj = []
    for r0, n in ((0, qd), (qd, kd), (qd + kd, kd)):
        proj.append(matmul_nbits(h1, w.wqkv_codes[r0:r0 + n], w.wqkv_scales[r0:r0 + n], K=hidden, N=n))
    q, k, v = (t.view(batch, seq_len, -1) for t in proj)
    a = group_query_attention(q, k, v, cache, layer, num_heads=cfg.num_heads, kv_num_heads=cfg.num_kv_heads,
                              do_rotary=do_rotary,
                              rotary_interleaved=rotary_interleaved, cos_cache=cos_cache, sin_cache=sin_cache)
    o = matmul_nbits(a.view(m, qd), w.wo_codes, w.wo_scales, K=qd, N=hidden)
    h2, pre2 = rms_norm(o, w.post_norm, skip=pre1, epsilon=w.epsilon)
    f2 = w.wgu_scales.shape[0]
    gu = matmul_nbits(h2, w.wgu_codes, w.wgu_scales, K=hidden, N=f2)
    mm = silu_mul(gu)
    dn = matmul_nbits(mm, w.wdown_codes, w.wdown_scales, K=f2 // 2, N=hidden)
    return dn, pre2
