"""Low-rank K (KVCacheConfig::kv_lowrank_k) on the GPU.

- The state (U*S per row, the rank-1 V^T row) is bit-exact with the C
  restatement of LowRankKeyDecomposer replayed as write_kv drives it
  (kv_compression.rs:842-853): the decomposition of row 0, the projections,
  and the re-decomposition at every 512th update, on every append path.
- Attention over such a cache reads keys as read_k's reconstruction
  (:870-882) and matches the composite oracle (reconstructed K, decoded V,
  causal SDPA) within 1e-3 on decode steps and prefill chunks.
"""
import numpy as np
import pytest
import torch

from tests.helpers import oracle_append, oracle_lowrank_attend, oracle_lowrank_state, rng, rope_tables

pytestmark = pytest.mark.gpu


def _bits_equal(name, got, want):
    g, w = np.ascontiguousarray(got).view(np.uint32), np.ascontiguousarray(want).view(np.uint32)
    bad = np.argwhere(g != w)
    assert bad.size == 0, f"{name}: {len(bad)} mismatches, first at {bad[:3].tolist()} " \
                          f"(got {got[tuple(bad[0])]}, want {want[tuple(bad[0])]})"


def _state(cache, t):
    view = cache.view(0)
    return view.lr_us[:, :, :t].cpu().numpy(), view.lr_vt.cpu().numpy()


@pytest.mark.parametrize("d,chunks", [(64, (600, 450, 1, 1, 1)), (128, (1, 511, 1, 513)), (16, (8,))])
def test_bulk_appends_state_bit_exact(cuda_device, d, chunks):
    """Appends in chunks across the re-decompositions at rows 512 and 1024 (and the reference's
    cache_with_lowrank shape: D = 16, 8 rows, rank 4)."""
    import smallaios_b200 as sa

    b, h, t = 2, 2, sum(chunks)
    r = rng(d + t)
    k = (r.standard_normal((b, t, h, d)) * 1.3).astype(np.float32)
    v = (r.standard_normal((b, t, h, d)) * 1.3).astype(np.float32)
    cos, sin = rope_tables(t + 1, d)
    tcos, tsin = torch.from_numpy(cos).to(cuda_device), torch.from_numpy(sin).to(cuda_device)
    cache = sa.GpuKvCache(1, h, d, t + 1, batch=b, bits=4, lowrank_k=4, device=cuda_device)
    p = 0
    for n in chunks:
        cache.append(0, torch.from_numpy(k[:, p:p + n]).reshape(b, n, h * d).to(cuda_device),
                     torch.from_numpy(v[:, p:p + n]).reshape(b, n, h * d).to(cuda_device), cos_cache=tcos,
                     sin_cache=tsin, do_rotary=True)
        cache.advance_position(n)
        p += n
    torch.cuda.synchronize()
    us, vt = _state(cache, t)
    cache.close()
    want_us, want_vt = oracle_lowrank_state(k, 4, cos, sin, True)
    _bits_equal("lr_us", us, want_us)
    _bits_equal("lr_vt", vt, want_vt)


@pytest.mark.parametrize("hq,hkv,bits", [(8, 2, 4), (16, 2, 8)])
def test_decode_steps_across_redecomposition(cuda_device, hq, hkv, bits):
    """A 508-token prompt, then decode steps through row 512: each step appends through the operator,
    and the attention reads the reconstructed keys."""
    import smallaios_b200 as sa

    b, d, past, steps = 2, 64, 508, 6
    t = past + steps
    r = rng(hq * bits)
    k = (r.standard_normal((b, t, hkv, d)) * 1.28).astype(np.float32)
    v = (r.standard_normal((b, t, hkv, d)) * 1.28).astype(np.float32)
    q = (r.standard_normal((b, t, hq, d)) * 1.28).astype(np.float32)
    cos, sin = rope_tables(t + 1, d, 500000.0)
    tcos, tsin = torch.from_numpy(cos).to(cuda_device), torch.from_numpy(sin).to(cuda_device)
    cache = sa.GpuKvCache(1, hkv, d, t + 1, batch=b, num_heads=hq, bits=bits, lowrank_k=2, device=cuda_device)
    cache.append(0, torch.from_numpy(k[:, :past]).reshape(b, past, hkv * d).to(cuda_device),
                 torch.from_numpy(v[:, :past]).reshape(b, past, hkv * d).to(cuda_device), cos_cache=tcos,
                 sin_cache=tsin, do_rotary=True)
    cache.advance_position(past)
    outs = []
    for i in range(past, t):
        out = sa.group_query_attention(torch.from_numpy(q[:, i:i + 1]).reshape(b, 1, hq * d).to(cuda_device),
                                       torch.from_numpy(k[:, i:i + 1]).reshape(b, 1, hkv * d).to(cuda_device),
                                       torch.from_numpy(v[:, i:i + 1]).reshape(b, 1, hkv * d).to(cuda_device),
                                       cache, 0, num_heads=hq, kv_num_heads=hkv, cos_cache=tcos, sin_cache=tsin)
        cache.advance_position(1)
        outs.append(out.float().cpu().numpy())
    torch.cuda.synchronize()
    us, vt = _state(cache, t)
    signs = cache.view(0).signs.cpu().numpy().astype(np.int8)
    cache.close()
    want_us, want_vt = oracle_lowrank_state(k, 2, cos, sin, True)
    _bits_equal("lr_us", us, want_us)
    _bits_equal("lr_vt", vt, want_vt)
    # attention of the last step against the composite oracle over the final state (the state of
    # rows <= 512 changes at row 512, so earlier steps are checked through their own prefixes below)
    kc, km, vc, vm = oracle_append(k, v, signs, bits, 0, cos, sin, True)
    for i, out in zip(range(past, t), outs):
        if i < 512:
            pus, pvt = oracle_lowrank_state(k[:, :i + 1], 2, cos, sin, True)
        else:
            pus, pvt = want_us[:, :, :i + 1], want_vt
        want = oracle_lowrank_attend(q[:, i:i + 1], pus, pvt, vc[:, :, :i + 1], vm[:, :, :i + 1], signs, bits, i,
                                     cos=cos, sin=sin, do_rotary=True)
        err = np.abs(out - want)
        assert err.max() <= 1e-3, f"step {i}: max err {err.max():.3e}"


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
def test_prefill_chunk_attention(cuda_device, dtype):
    """A 300-token prompt in one call, then a 40-token chunk: causal attention over reconstructed keys."""
    import smallaios_b200 as sa

    b, hq, hkv, d, bits = 2, 8, 4, 128, 4
    t = 340
    r = rng(11)
    k = torch.from_numpy((r.standard_normal((b, t, hkv, d)) * 1.28).astype(np.float32)).to(dtype)
    v = torch.from_numpy((r.standard_normal((b, t, hkv, d)) * 1.28).astype(np.float32)).to(dtype)
    q = torch.from_numpy((r.standard_normal((b, t, hq, d)) * 1.28).astype(np.float32)).to(dtype)
    cos, sin = rope_tables(t + 1, d)
    tcos, tsin = torch.from_numpy(cos).to(cuda_device), torch.from_numpy(sin).to(cuda_device)
    cache = sa.GpuKvCache(1, hkv, d, t + 1, batch=b, num_heads=hq, bits=bits, lowrank_k=1, device=cuda_device)
    outs = []
    for p0, n in ((0, 300), (300, 40)):
        outs.append(sa.group_query_attention(q[:, p0:p0 + n].reshape(b, n, hq * d).to(cuda_device),
                                             k[:, p0:p0 + n].reshape(b, n, hkv * d).to(cuda_device),
                                             v[:, p0:p0 + n].reshape(b, n, hkv * d).to(cuda_device), cache, 0,
                                             num_heads=hq, kv_num_heads=hkv, cos_cache=tcos, sin_cache=tsin))
        cache.advance_position(n)
    torch.cuda.synchronize()
    us, vt = _state(cache, t)
    signs = cache.view(0).signs.cpu().numpy().astype(np.int8)
    cache.close()
    kn, vn, qn = k.float().numpy(), v.float().numpy(), q.float().numpy()
    want_us, want_vt = oracle_lowrank_state(kn, 1, cos, sin, True)
    _bits_equal("lr_us", us, want_us)
    _bits_equal("lr_vt", vt, want_vt)
    kc, km, vc, vm = oracle_append(kn, vn, signs, bits, 0, cos, sin, True)
    ulp = 2.0 ** -8 if dtype == torch.bfloat16 else 0.0
    for (p0, n), out in zip(((0, 300), (300, 40)), outs):
        want = oracle_lowrank_attend(qn[:, p0:p0 + n], want_us[:, :, :p0 + n], want_vt, vc[:, :, :p0 + n],
                                     vm[:, :, :p0 + n], signs, bits, p0, cos=cos, sin=sin, do_rotary=True)
        got = out.float().cpu().numpy()
        err = np.abs(got - want)
        assert np.all(err <= 1e-3 + np.abs(want) * ulp), f"chunk at {p0}: max err {err.max():.3e}"


def test_fused_qkv_projection_and_qjl_together(cuda_device):
    """sa_qkv_project_append (tcgen05 epilogue, batch 20) on a cache with low-rank K and QJL residuals."""
    import smallaios_b200 as sa

    hq, hkv, d, hidden, bits, past, b = 8, 2, 128, 512, 4, 9, 20
    r = rng(70)
    n = (hq + 2 * hkv) * d
    codes = torch.from_numpy(r.integers(0, 256, size=(n, hidden // 32, 16), dtype=np.uint8))
    scales = torch.from_numpy(r.uniform(0.005, 0.02, size=(n, hidden // 32)).astype(np.float32)).to(torch.bfloat16)
    x = torch.from_numpy(r.standard_normal((b, hidden)).astype(np.float32)).to(torch.bfloat16)
    kp = torch.from_numpy((r.standard_normal((b, past, hkv, d)) * 1.28).astype(np.float32)).to(torch.bfloat16)
    vp = torch.from_numpy((r.standard_normal((b, past, hkv, d)) * 1.28).astype(np.float32)).to(torch.bfloat16)
    cos, sin = rope_tables(past + 8, d)
    tcos, tsin = torch.from_numpy(cos).to(cuda_device), torch.from_numpy(sin).to(cuda_device)
    cache = sa.GpuKvCache(1, hkv, d, past + 8, batch=b, num_heads=hq, bits=bits, qjl_residual=True, lowrank_k=8,
                          device=cuda_device)
    cache.append(0, kp.reshape(b, past, hkv * d).to(cuda_device), vp.reshape(b, past, hkv * d).to(cuda_device),
                 cos_cache=tcos, sin_cache=tsin, do_rotary=True)
    cache.advance_position(past)
    _, kn, _ = sa.qkv_project_append(x.to(cuda_device), codes.to(cuda_device), scales.to(cuda_device), cache, 0,
                                     cos_cache=tcos, sin_cache=tsin, do_rotary=True)
    torch.cuda.synchronize()
    us, vt = _state(cache, past + 1)
    kall = np.concatenate([kp.float().numpy(), kn.float().cpu().numpy().reshape(b, 1, hkv, d)], axis=1)
    cache.close()
    want_us, want_vt = oracle_lowrank_state(kall, 8, cos, sin, True)
    _bits_equal("lr_us", us, want_us)
    _bits_equal("lr_vt", vt, want_vt)


def test_general_kernel_three_bits_short_chunk(cuda_device):
    """3-bit codes and a 5-token chunk take the general split-K kernel through the operator; its
    scores read the low-rank metadata and q'.R(V^T) like the other kernels."""
    import smallaios_b200 as sa

    b, hq, hkv, d, bits, past, s = 2, 8, 2, 64, 3, 70, 5
    t = past + s
    r = rng(13)
    k = (r.standard_normal((b, t, hkv, d)) * 1.28).astype(np.float32)
    v = (r.standard_normal((b, t, hkv, d)) * 1.28).astype(np.float32)
    q = (r.standard_normal((b, s, hq, d)) * 1.28).astype(np.float32)
    cos, sin = rope_tables(t + 1, d)
    tcos, tsin = torch.from_numpy(cos).to(cuda_device), torch.from_numpy(sin).to(cuda_device)
    cache = sa.GpuKvCache(1, hkv, d, t + 1, batch=b, num_heads=hq, bits=bits, lowrank_k=2, device=cuda_device)
    cache.append(0, torch.from_numpy(k[:, :past]).reshape(b, past, hkv * d).to(cuda_device),
                 torch.from_numpy(v[:, :past]).reshape(b, past, hkv * d).to(cuda_device), cos_cache=tcos,
                 sin_cache=tsin, do_rotary=True)
    cache.advance_position(past)
    out = sa.group_query_attention(torch.from_numpy(q).reshape(b, s, hq * d).to(cuda_device),
                                   torch.from_numpy(k[:, past:]).reshape(b, s, hkv * d).to(cuda_device),
                                   torch.from_numpy(v[:, past:]).reshape(b, s, hkv * d).to(cuda_device), cache, 0,
                                   num_heads=hq, kv_num_heads=hkv, cos_cache=tcos, sin_cache=tsin)
    torch.cuda.synchronize()
    got = out.float().cpu().numpy()
    signs = cache.view(0).signs.cpu().numpy().astype(np.int8)
    cache.close()
    us, vt = oracle_lowrank_state(k, 2, cos, sin, True)
    kc, km, vc, vm = oracle_append(k, v, signs, bits, 0, cos, sin, True)
    want = oracle_lowrank_attend(q, us, vt, vc, vm, signs, bits, past, cos=cos, sin=sin, do_rotary=True)
    err = np.abs(got - want)
    assert err.max() <= 1e-3, f"max err {err.max():.3e}"


def test_no_alloc_entry_reads_low_rank_view(cuda_device):
    import ctypes

    import smallaios_b200 as sa
    from smallaios_b200 import _lib
    from smallaios_b200._lib import lib

    b, hq, hkv, d, t = 1, 4, 2, 64, 40
    r = rng(12)
    k = torch.from_numpy((r.standard_normal((b, t, hkv * d)) * 1.28).astype(np.float32))
    v = torch.from_numpy((r.standard_normal((b, t, hkv * d)) * 1.28).astype(np.float32))
    q = torch.from_numpy((r.standard_normal((b, 1, hq * d)) * 1.28).astype(np.float32)).to(cuda_device)
    cache = sa.GpuKvCache(1, hkv, d, t + 1, batch=b, num_heads=hq, bits=4, lowrank_k=2, device=cuda_device)
    cache.append(0, k.to(cuda_device), v.to(cuda_device), do_rotary=False)
    cache.advance_position(t - 1)  # the query sits at the last appended position
    want = sa.gqa_attend(q, cache, 0, num_heads=hq, do_rotary=False)
    view = _lib.KvLayerView()
    _lib.check(lib.sa_kv_cache_layer_view(cache.handle, 0, ctypes.byref(view)))
    assert view.lr_us and view.lr_vt
    got = torch.empty_like(want)
    _lib.check(lib.sa_gqa_attend_no_alloc(ctypes.byref(view), t - 1, q.data_ptr(), got.data_ptr(),
                                          _lib.SA_DTYPE_FLOAT, b, 1, hq // hkv, 0, 0.0, None, None, 0, 0, 0,
                                          torch.cuda.current_stream(cuda_device).cuda_stream))
    torch.cuda.synchronize()
    cache.close()
    # the no-alloc entry runs the general split-K kernel, the attend-only entry the decode kernel
    assert (got - want).abs().max().item() <= 1e-3
