"""GroupQueryAttention over the compressed cache vs the composite CPU oracle.

The reference never wires kv_compression.rs into GroupQueryAttention; the
oracle composition is ours: PolarQuantizer::encode of every token (RoPE on K
at its position), CompressedKVCache::read_k/read_v of the whole range, then
scaled_dot_product_attention with the causal mask and past_sk = T - S
(ops/microsoft.rs:380-438), reshaped to (B, S, Hq*D).  Bar: max-abs error
<= 1e-3 with f32 activations (fp32 accumulate).  bf16 activations add the
bf16 rounding of the output (half an ulp, 2^-9 relative).
"""
import numpy as np
import pytest
import torch

import oracle
from tests.helpers import interleave_v, oracle_append, oracle_attend, rng, rope_tables

pytestmark = pytest.mark.gpu

TOL = 1e-3


def _to(x, dtype, dev):
    return torch.from_numpy(np.ascontiguousarray(x)).to(dtype).to(dev)


def _decode_case(dev, *, b, hq, hkv, d, bits, t, s=1, dtype=torch.float32, theta=10000.0, seed=0,
                 interleaved=False, chunks=(64,), std=1.28, use_op=True, scale=None):
    """Fill t - s tokens through the library's own append, then run GQA on s new tokens."""
    import smallaios_b200 as sa

    r = rng(seed)
    past = t - s
    k = (r.standard_normal((b, t, hkv, d)) * std).astype(np.float32)
    v = (r.standard_normal((b, t, hkv, d)) * std).astype(np.float32)
    q = (r.standard_normal((b, s, hq, d)) * std).astype(np.float32)
    # the oracle sees the dtype-rounded values
    k = torch.from_numpy(k).to(dtype).float().numpy()
    v = torch.from_numpy(v).to(dtype).float().numpy()
    q = torch.from_numpy(q).to(dtype).float().numpy()
    cos, sin = rope_tables(t + 8, d, theta)
    cos_t, sin_t = torch.from_numpy(cos).to(dev), torch.from_numpy(sin).to(dev)
    cache = sa.GpuKvCache(1, hkv, d, t + 8, batch=b, num_heads=hq, bits=bits, device=dev)
    pos, ci = 0, 0
    while pos < past:
        n = min(chunks[ci % len(chunks)], past - pos)
        ci += 1
        cache.append(0, _to(k[:, pos:pos + n].reshape(b, n, hkv * d), dtype, dev),
                     _to(v[:, pos:pos + n].reshape(b, n, hkv * d), dtype, dev),
                     cos_cache=cos_t, sin_cache=sin_t, do_rotary=True, rotary_interleaved=interleaved)
        cache.advance_position(n)
        pos += n
    qt = _to(q.reshape(b, s, hq * d), dtype, dev)
    kt = _to(k[:, past:].reshape(b, s, hkv * d), dtype, dev)
    vt = _to(v[:, past:].reshape(b, s, hkv * d), dtype, dev)
    if use_op:
        out = sa.group_query_attention(qt, kt, vt, cache, 0, num_heads=hq, kv_num_heads=hkv, scale=scale,
                                       do_rotary=True, rotary_interleaved=interleaved, cos_cache=cos_t,
                                       sin_cache=sin_t)
    else:
        cache.append(0, kt, vt, cos_cache=cos_t, sin_cache=sin_t, do_rotary=True, rotary_interleaved=interleaved)
        out = sa.gqa_attend(qt, cache, 0, num_heads=hq, scale=scale, cos_cache=cos_t, sin_cache=sin_t,
                            do_rotary=True, rotary_interleaved=interleaved)
    torch.cuda.synchronize()
    got = out.float().cpu().numpy()
    view = cache.view(0)
    signs = view.signs.cpu().numpy().astype(np.int8)
    kc, km, vc, vm = oracle_append(k, v, signs, bits, 0, cos, sin, True, interleaved)
    # the library's cache must hold exactly the oracle's codes
    assert np.array_equal(view.k_codes[:, :, :t].cpu().numpy(), kc)
    assert np.array_equal(view.v_codes_tokens()[:, :, :t].cpu().numpy(), vc)
    assert np.array_equal(view.k_meta[:, :, :t].cpu().numpy().view(np.uint32), km.view(np.uint32))
    want = oracle_attend(q, kc, km, vc, vm, signs, bits, past, scale=scale, cos=cos, sin=sin, do_rotary=True,
                         interleaved=interleaved)
    cache.close()
    return got, want


def _check(got, want, dtype):
    err = np.abs(got - want)
    if dtype == torch.float32:
        bound = TOL
    elif dtype == torch.bfloat16:
        bound = TOL + np.abs(want) * 2.0 ** -8
    else:
        bound = TOL + np.abs(want) * 2.0 ** -11
    worst = np.unravel_index(np.argmax(err - bound), err.shape)
    assert np.all(err <= bound), f"max err {err.max():.3e} at {worst}: got {got[worst]} want {want[worst]}"


def test_c1_shape_int8(cuda_device):
    """B=1, 8 q heads / 2 KV heads, D=64, context 512, int8 KV."""
    got, want = _decode_case(cuda_device, b=1, hq=8, hkv=2, d=64, bits=8, t=512, theta=10000.0, seed=1,
                             std=0.45)
    _check(got, want, torch.float32)


def test_c3_shape_int4_small_batch(cuda_device):
    """Llama-3-8B layer shape (32/8 heads, D=128, int4, theta 5e5) at B=2, T=1500."""
    got, want = _decode_case(cuda_device, b=2, hq=32, hkv=8, d=128, bits=4, t=1500, theta=500000.0, seed=2,
                             chunks=(256, 100, 7))
    _check(got, want, torch.float32)


@pytest.mark.parametrize("bits", [3, 4, 8])
def test_bits(cuda_device, bits):
    got, want = _decode_case(cuda_device, b=2, hq=8, hkv=2, d=128, bits=bits, t=333, seed=10 + bits)
    _check(got, want, torch.float32)


@pytest.mark.parametrize("d,hq,hkv", [(16, 4, 2), (32, 6, 3), (64, 8, 8), (256, 8, 1)])
def test_head_dims_and_groups(cuda_device, d, hq, hkv):
    got, want = _decode_case(cuda_device, b=1, hq=hq, hkv=hkv, d=d, bits=4, t=200, seed=d + hq)
    _check(got, want, torch.float32)


def test_c5_shape_group8_int4(cuda_device):
    """Llama-3-70B layer shape (64/8 heads: 8 query heads per KV head, D=128, int4, theta 5e5) at B=2."""
    got, want = _decode_case(cuda_device, b=2, hq=64, hkv=8, d=128, bits=4, t=1500, theta=500000.0, seed=21,
                             chunks=(256, 100, 7))
    _check(got, want, torch.float32)


@pytest.mark.parametrize("d,hq,hkv,bits", [(128, 16, 2, 8), (64, 10, 2, 4), (64, 14, 2, 8), (128, 12, 2, 4),
                                           (64, 8, 1, 4)])
def test_groups_five_to_eight(cuda_device, d, hq, hkv, bits):
    """5..8 query heads per KV head (the eight-head decode kernel, unused heads zero)."""
    got, want = _decode_case(cuda_device, b=3, hq=hq, hkv=hkv, d=d, bits=bits, t=421, seed=d + hq + bits)
    _check(got, want, torch.float32)


def test_group8_first_tokens_and_long_context(cuda_device):
    """Group 8: contexts of 1-3 and 65 tokens, then one row of 6000 tokens cut into many warp ranges."""
    for t in (1, 2, 3, 65):
        got, want = _decode_case(cuda_device, b=1, hq=8, hkv=1, d=128, bits=4, t=t, seed=40 + t)
        _check(got, want, torch.float32)
    got, want = _decode_case(cuda_device, b=1, hq=16, hkv=2, d=128, bits=4, t=6000, seed=47, chunks=(1000,),
                             theta=500000.0)
    _check(got, want, torch.float32)


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
def test_group8_half_dtypes(cuda_device, dtype):
    got, want = _decode_case(cuda_device, b=3, hq=64, hkv=8, d=128, bits=4, t=300, dtype=dtype, seed=48,
                             theta=500000.0)
    _check(got, want, dtype)


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
def test_half_dtypes(cuda_device, dtype):
    got, want = _decode_case(cuda_device, b=3, hq=32, hkv=8, d=128, bits=4, t=700, dtype=dtype, seed=4,
                             theta=500000.0)
    _check(got, want, dtype)


def test_prefill_chunk_causal(cuda_device):
    """S=5 new tokens at once: each attends causally to [0, past + s]."""
    got, want = _decode_case(cuda_device, b=2, hq=8, hkv=2, d=64, bits=4, t=90, s=5, seed=6)
    _check(got, want, torch.float32)


@pytest.mark.parametrize("d,hq,hkv,bits", [(128, 32, 8, 4), (128, 16, 2, 8), (64, 8, 8, 4), (64, 8, 4, 8),
                                           (128, 8, 1, 4)])
def test_prefill_tensor_core(cuda_device, d, hq, hkv, bits):
    """Prefill chunks of 16+ query tokens run on the tensor-core kernel (groups 1, 2, 4, 8):
    a 200-token chunk after 60 cached tokens (past > 0, rows across CTAs, a ragged last tile)."""
    got, want = _decode_case(cuda_device, b=2, hq=hq, hkv=hkv, d=d, bits=bits, t=260, s=200, seed=d + hq + bits,
                             chunks=(60,), theta=500000.0)
    _check(got, want, torch.float32)


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
def test_prefill_whole_prompt_half(cuda_device, dtype):
    """A whole 300-token prompt in one call (empty cache), fp16/bf16 activations."""
    got, want = _decode_case(cuda_device, b=2, hq=32, hkv=8, d=128, bits=8, t=300, s=300, dtype=dtype, seed=31)
    _check(got, want, dtype)


@pytest.mark.parametrize("d,hq,hkv,bits", [(64, 6, 2, 4), (128, 10, 2, 8), (64, 12, 2, 8), (128, 14, 2, 4)])
def test_prefill_groups_not_dividing_the_row_block(cuda_device, d, hq, hkv, bits):
    """Groups 3, 5, 6 and 7: a 128-row block ends inside a position, so one position's heads are
    split between two CTAs; a 150-token chunk after 40 cached tokens."""
    got, want = _decode_case(cuda_device, b=2, hq=hq, hkv=hkv, d=d, bits=bits, t=190, s=150, seed=d + hq,
                             chunks=(40,))
    _check(got, want, torch.float32)


def test_prefill_long_sharp_softmax(cuda_device):
    """A 1100-token prompt (18 KV tiles, the running max and V reference moving across tiles)
    with wide activations (std 3), so the softmax is peaked and scores span a large range."""
    got, want = _decode_case(cuda_device, b=1, hq=8, hkv=2, d=128, bits=4, t=1100, s=1100, seed=41, std=3.0)
    _check(got, want, torch.float32)


def test_prefill_int8_tiny_values(cuda_device):
    """8-bit codes on small activations (std 0.05: V scales near 4e-4), where the products
    p * scale sit far below fp16's normal range unless they are normalised."""
    got, want = _decode_case(cuda_device, b=2, hq=8, hkv=4, d=64, bits=8, t=333, s=300, seed=42, std=0.05)
    _check(got, want, torch.float32)


def test_prefill_interleaved_rope_scale_16_tokens(cuda_device):
    got, want = _decode_case(cuda_device, b=3, hq=8, hkv=2, d=64, bits=4, t=40, s=16, seed=32, interleaved=True,
                             scale=0.2)
    _check(got, want, torch.float32)


def test_first_token_and_tiny_context(cuda_device):
    for t in (1, 2, 3, 5):
        got, want = _decode_case(cuda_device, b=1, hq=4, hkv=2, d=64, bits=4, t=t, seed=t)
        _check(got, want, torch.float32)


def test_interleaved_rope_and_scale_attr(cuda_device):
    got, want = _decode_case(cuda_device, b=2, hq=8, hkv=2, d=64, bits=4, t=130, seed=8, interleaved=True,
                             scale=0.3)
    _check(got, want, torch.float32)


def test_attend_only_entry(cuda_device):
    got, want = _decode_case(cuda_device, b=2, hq=16, hkv=4, d=128, bits=4, t=257, seed=9, use_op=False)
    _check(got, want, torch.float32)


def test_long_context_split_k(cuda_device):
    """T=6000 forces many split-K partitions and the cross-split merge."""
    got, want = _decode_case(cuda_device, b=1, hq=32, hkv=8, d=128, bits=4, t=6000, seed=12,
                             chunks=(1000,), theta=500000.0)
    _check(got, want, torch.float32)


def test_compressed_close_to_uncompressed_reference_op(cuda_device):
    """Sanity: 8-bit compressed attention stays near op_group_query_attention on raw K/V."""
    import smallaios_b200 as sa

    b, hq, hkv, d, t = 1, 8, 2, 64, 64
    r = rng(3)
    q = r.standard_normal((b, 1, hq * d)).astype(np.float32) * 0.45
    k = r.standard_normal((b, t, hkv * d)).astype(np.float32) * 0.45
    v = r.standard_normal((b, t, hkv * d)).astype(np.float32) * 0.45
    cos, sin = rope_tables(t + 1, d)
    # reference op on uncompressed tensors: prefill t-1 tokens, then one decode step
    _, pk, pv = oracle.group_query_attention(np.zeros((b, t - 1, hq * d), np.float32), k[:, :t - 1], v[:, :t - 1],
                                             cos_cache=cos, sin_cache=sin, num_heads=hq, kv_num_heads=hkv)
    want, _, _ = oracle.group_query_attention(q, k[:, t - 1:], v[:, t - 1:], pk, pv, cos, sin, num_heads=hq,
                                              kv_num_heads=hkv)
    dev = cuda_device
    cache = sa.GpuKvCache(1, hkv, d, t + 1, batch=b, num_heads=hq, bits=8, device=dev)
    cos_t, sin_t = torch.from_numpy(cos).to(dev), torch.from_numpy(sin).to(dev)
    cache.append(0, torch.from_numpy(k[:, :t - 1]).to(dev).contiguous(),
                 torch.from_numpy(v[:, :t - 1]).to(dev).contiguous(), cos_cache=cos_t, sin_cache=sin_t,
                 do_rotary=True)
    cache.advance_position(t - 1)
    out = sa.group_query_attention(torch.from_numpy(q).to(dev), torch.from_numpy(k[:, t - 1:]).to(dev).contiguous(),
                                   torch.from_numpy(v[:, t - 1:]).to(dev).contiguous(), cache, 0, num_heads=hq,
                                   kv_num_heads=hkv, cos_cache=cos_t, sin_cache=sin_t)
    got = out.cpu().numpy()
    assert np.max(np.abs(got - want)) < 0.05
    cache.close()


def test_operator_validation_errors(cuda_device):
    import smallaios_b200 as sa

    dev = cuda_device
    cache = sa.GpuKvCache(1, 2, 64, 16, batch=1, num_heads=8, bits=4, device=dev)
    q = torch.zeros(1, 1, 512, device=dev)
    kv = torch.zeros(1, 1, 128, device=dev)
    with pytest.raises(sa.InvalidAttribute):
        sa.group_query_attention(q, kv, kv, cache, 0, num_heads=8, kv_num_heads=2, local_window_size=512,
                                 do_rotary=False)
    with pytest.raises(sa.InvalidAttribute):
        sa.group_query_attention(q, kv, kv, cache, 0, num_heads=6, kv_num_heads=4, do_rotary=False)
    with pytest.raises(sa.ShapeMismatch):  # do_rotary defaults to 1 and needs caches
        sa.group_query_attention(q, kv, kv, cache, 0, num_heads=8, kv_num_heads=2)
    with pytest.raises(sa.ShapeMismatch):
        sa.group_query_attention(q, kv[:, :, :64].contiguous(), kv[:, :, :64].contiguous(), cache, 0, num_heads=8,
                                 kv_num_heads=2, do_rotary=False)
    cache.close()


def test_dispatch_gpu_node_two_layers(cuda_device):
    """Executor glue: layer counter per GQA node, one advance per forward pass."""
    import smallaios_b200 as sa

    dev = cuda_device
    b, hq, hkv, d = 1, 4, 2, 64
    cache = sa.GpuKvCache(2, hkv, d, 16, batch=b, num_heads=hq, bits=4, device=dev)
    ctx = sa.KvCacheDispatchCtx(cache)
    attrs = {"num_heads": hq, "kv_num_heads": hkv, "do_rotary": 0}
    for step in range(3):
        ctx.next_layer_idx = 0
        for _layer in range(2):
            x = torch.randn(b, 1, hq * d, device=dev)
            kv = torch.randn(b, 1, hkv * d, device=dev)
            (out,) = sa.dispatch_gpu_node("GroupQueryAttention", [x, kv, kv], attrs, ctx)
            assert out.shape == x.shape and torch.isfinite(out).all()
        sa.finalize_kv_cache(ctx)
        assert cache.current_position() == step + 1
    cache.close()
