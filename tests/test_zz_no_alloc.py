"""The allocation-free attention entry point (sa_gqa_attend_no_alloc).

It is for callers that may not allocate device memory while they run. Examples
are a real-time partition that reserves all its memory at start-up, or a host
whose device memory belongs to its own pool. The call reads the caller's cache
buffers and keeps its split-K partials in a static array the library reserves
once per GPU.

The test fills a cache through the normal API and calls both entry points
through the C ABI. The new one must match sa_gqa_attend within the attention
tolerance of the other GPU tests (1e-3), on two calls in a row, because the
second call sees the first call's leftovers in the shared array. It also checks
that a problem too large for the static array is rejected with SA_ERR_CAPACITY.

This file sorts last, so a run that stops at its first failure has already run
every other test. It also passes when run alone in a fresh process.
"""
import ctypes

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu

TOL = 1e-3


def _filled_cache(dev, b, hq, hkv, d, t, bits=4, seed=0):
    import smallaios_b200 as sa

    g = torch.Generator(device=dev)
    g.manual_seed(seed)
    cache = sa.GpuKvCache(1, hkv, d, t, batch=b, num_heads=hq, bits=bits, device=dev)
    half = d // 2
    inv = 1.0 / (500000.0 ** (np.arange(half) * 2.0 / d))
    ang = np.arange(t)[:, None] * inv[None, :]
    cos = torch.from_numpy(np.cos(ang).astype(np.float32)).to(dev)
    sin = torch.from_numpy(np.sin(ang).astype(np.float32)).to(dev)
    pos = 0
    while pos < t - 1:
        n = min(512, t - 1 - pos)
        k = torch.randn(b, n, hkv * d, device=dev, generator=g) * 1.28
        v = torch.randn(b, n, hkv * d, device=dev, generator=g) * 1.28
        cache.append(0, k, v, cos_cache=cos, sin_cache=sin, do_rotary=True)
        cache.advance_position(n)
        pos += n
    k = torch.randn(b, 1, hkv * d, device=dev, generator=g) * 1.28
    cache.append(0, k, k.clone(), cos_cache=cos, sin_cache=sin, do_rotary=True)
    return cache, cos, sin, g


def _view(cache):
    from smallaios_b200 import _lib

    v = _lib.KvLayerView()
    _lib.check(_lib.lib.sa_kv_cache_layer_view(cache.handle, 0, ctypes.byref(v)))
    return v


def test_no_alloc_matches_cached_entry_point_twice(cuda_device):
    from smallaios_b200 import _lib

    dev = cuda_device
    b, hq, hkv, d, t = 4, 32, 8, 128, 2000
    cache, cos, sin, g = _filled_cache(dev, b, hq, hkv, d, t)
    view = _view(cache)
    stream = torch.cuda.current_stream(dev).cuda_stream
    for call in range(2):  # two calls in a row share the static array
        q = torch.randn(b, 1, hq * d, device=dev, generator=g) * 1.28
        want = torch.empty_like(q)
        got = torch.full_like(q, float("nan"))
        rc = _lib.lib.sa_gqa_attend(cache.handle, 0, q.data_ptr(), want.data_ptr(), _lib.SA_DTYPE_FLOAT, b, 1, hq,
                                    0, 0.0, cos.data_ptr(), sin.data_ptr(), t, 1, 0, stream)
        _lib.check(rc)
        rc = _lib.lib.sa_gqa_attend_no_alloc(ctypes.byref(view), t - 1, q.data_ptr(), got.data_ptr(),
                                             _lib.SA_DTYPE_FLOAT, b, 1, hq // hkv, 0, 0.0, cos.data_ptr(),
                                             sin.data_ptr(), t, 1, 0, stream)
        _lib.check(rc)
        torch.cuda.synchronize(dev)
        err = (got - want).abs().max().item()
        assert err <= TOL, f"call {call}: max-abs difference {err:.3e}"
    cache.close()


def test_no_alloc_rejects_problems_beyond_the_static_maximum(cuda_device):
    from smallaios_b200 import _lib

    dev = cuda_device
    # 64 rows x 8 kv heads x group 8 x (256 + 4) floats = 4.3 MB per split: two splits exceed 8 MiB.
    b, hkv, hq, d, t = 64, 8, 64, 256, 1024
    cache, cos, sin, _ = _filled_cache(dev, b, hq, hkv, d, t)
    view = _view(cache)
    q = torch.zeros(b, 1, hq * d, device=dev)
    out = torch.zeros_like(q)
    rc = _lib.lib.sa_gqa_attend_no_alloc(ctypes.byref(view), t - 1, q.data_ptr(), out.data_ptr(),
                                         _lib.SA_DTYPE_FLOAT, b, 1, hq // hkv, 0, 0.0, cos.data_ptr(),
                                         sin.data_ptr(), t, 1, 0, torch.cuda.current_stream(dev).cuda_stream)
    assert rc == _lib.SA_ERR_CAPACITY
    assert b"static scratch maximum" in _lib.lib.sa_last_error_string()
    cache.close()
