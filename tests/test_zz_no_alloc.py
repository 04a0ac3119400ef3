"""The allocation-free attention entry point (sa_gqa_attend_no_alloc).

It is for callers that may not allocate device memory while they run. Examples
are a real-time partition that reserves all its memory at start-up, or a host
whose device memory belongs to its own pool. The call reads the caller's cache
buffers and keeps its split-K partials in a static array the library reserves
once per GPU.

The tests fill a cache through the normal API and call both entry points
through the C ABI. The new one must match sa_gqa_attend within the attention
tolerance of the other GPU tests (1e-3), on calls in a row, because each call
sees the previous call's leftovers in the shared array: the same shape twice,
then a shorter context with a different split count after a longer one. It
is also checked against the CPU oracle directly, in bf16, with 3-bit codes and
on a low-rank K view. A problem too large for the static array is rejected with
SA_ERR_CAPACITY, and one with more query rows than a launch takes with
SA_ERR_UNSUPPORTED.

This file sorts last, so a run that stops at its first failure has already run
every other test. It also passes when run alone in a fresh process.
"""
import ctypes

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu

TOL = 1e-3


def _filled_cache(dev, b, hq, hkv, d, t, bits=4, seed=0, lowrank=None):
    import smallaios_b200 as sa

    g = torch.Generator(device=dev)
    g.manual_seed(seed)
    cache = sa.GpuKvCache(1, hkv, d, t, batch=b, num_heads=hq, bits=bits, lowrank_k=lowrank, device=dev)
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


def _both(cache, view, q, dtype_code, past, cos, sin, t, dev, hq, hkv):
    """sa_gqa_attend (cache position = past) and the no-alloc entry on the same query."""
    from smallaios_b200 import _lib

    b = q.shape[0]
    stream = torch.cuda.current_stream(dev).cuda_stream
    want = torch.empty_like(q)
    got = torch.full_like(q, float("nan"))
    cache.set_position(past)
    _lib.check(_lib.lib.sa_gqa_attend(cache.handle, 0, q.data_ptr(), want.data_ptr(), dtype_code, b, 1, hq, 0, 0.0,
                                      cos.data_ptr(), sin.data_ptr(), t, 1, 0, stream))
    _lib.check(_lib.lib.sa_gqa_attend_no_alloc(ctypes.byref(view), past, q.data_ptr(), got.data_ptr(), dtype_code, b,
                                               1, hq // hkv, 0, 0.0, cos.data_ptr(), sin.data_ptr(), t, 1, 0,
                                               stream))
    torch.cuda.synchronize(dev)
    return got, want


def test_no_alloc_shorter_context_after_longer_one(cuda_device):
    """A long context (many splits) then a short one (fewer splits, other partial slots): the
    second call must not pick up the first call's partials."""
    from smallaios_b200 import _lib

    dev = cuda_device
    b, hq, hkv, d, t = 4, 32, 8, 128, 3000
    cache, cos, sin, g = _filled_cache(dev, b, hq, hkv, d, t)
    view = _view(cache)
    for past in (t - 1, 300, 2999, 17):
        q = torch.randn(b, 1, hq * d, device=dev, generator=g) * 1.28
        got, want = _both(cache, view, q, _lib.SA_DTYPE_FLOAT, past, cos, sin, t, dev, hq, hkv)
        err = (got - want).abs().max().item()
        assert err <= TOL, f"past {past}: max-abs difference {err:.3e}"
    cache.close()


def test_no_alloc_against_the_oracle(cuda_device):
    """One no-alloc call against the composite CPU oracle on the cache's own codes."""
    import oracle
    from smallaios_b200 import _lib

    dev = cuda_device
    b, hq, hkv, d, t = 2, 8, 2, 64, 700
    cache, cos, sin, g = _filled_cache(dev, b, hq, hkv, d, t)
    view = _view(cache)
    q = torch.randn(b, 1, hq * d, device=dev, generator=g) * 1.28
    got, _ = _both(cache, view, q, _lib.SA_DTYPE_FLOAT, t - 1, cos, sin, t, dev, hq, hkv)
    lv = cache.view(0)
    kc = lv.k_codes[:, :, :t].cpu().numpy()
    km = lv.k_meta[:, :, :t].cpu().numpy()
    vc = lv.v_codes_tokens()[:, :, :t].cpu().numpy()
    vm = lv.v_meta[:, :, :t].cpu().numpy()
    signs = lv.signs.cpu().numpy().astype(np.int8)
    qn = q.cpu().numpy().reshape(b, 1, hq, d).transpose(0, 2, 1, 3)
    qr = oracle.apply_rope(np.ascontiguousarray(qn), cos.cpu().numpy(), sin.cpu().numpy(), [t - 1])
    scale = np.float32(1.0) / np.float32(oracle.sqrt_f32(float(d)))
    want = oracle.compressed_gqa(qr, kc, km, vc, vm, signs, 4, scale)
    err = np.abs(got.cpu().numpy() - want).max()
    assert err <= TOL, f"max-abs error vs the oracle {err:.3e}"
    cache.close()


@pytest.mark.parametrize("case", ["bf16", "bits3", "lowrank"])
def test_no_alloc_dtypes_bits_and_lowrank_view(cuda_device, case):
    from smallaios_b200 import _lib

    dev = cuda_device
    b, hq, hkv, d, t = 3, 16, 4, 64, 900
    cache, cos, sin, g = _filled_cache(dev, b, hq, hkv, d, t, bits=3 if case == "bits3" else 4,
                                       lowrank=1 if case == "lowrank" else None)
    view = _view(cache)
    if case == "lowrank":
        assert view.lr_kmeta and view.lr_vtr
    q = torch.randn(b, 1, hq * d, device=dev, generator=g) * 1.28
    code = _lib.SA_DTYPE_FLOAT
    if case == "bf16":
        q, code = q.to(torch.bfloat16), _lib.SA_DTYPE_BFLOAT16
    for past in (t - 1, 250):
        got, want = _both(cache, view, q, code, past, cos, sin, t, dev, hq, hkv)
        bound = TOL + (want.float().abs() * 2.0 ** -8 if case == "bf16" else 0.0)
        assert torch.all((got.float() - want.float()).abs() <= bound), f"{case} past {past}"
    cache.close()


def test_query_rows_beyond_one_launch_are_rejected(cuda_device):
    """batch*seq_len above 65535 query rows: a clear SA_ERR_UNSUPPORTED from both entry points
    of the general kernel, not a failed launch."""
    import smallaios_b200 as sa
    from smallaios_b200 import _lib

    dev = cuda_device
    s = 65536
    cache = sa.GpuKvCache(1, 1, 16, s + 16, batch=1, num_heads=1, bits=4, device=dev)
    view = _view(cache)
    q = torch.zeros(1, s, 16, device=dev)
    out = torch.zeros_like(q)
    stream = torch.cuda.current_stream(dev).cuda_stream
    rc = _lib.lib.sa_gqa_attend_no_alloc(ctypes.byref(view), 0, q.data_ptr(), out.data_ptr(), _lib.SA_DTYPE_FLOAT,
                                         1, s, 1, 0, 0.0, None, None, 0, 0, 0, stream)
    assert rc == _lib.SA_ERR_UNSUPPORTED
    assert b"65535" in _lib.lib.sa_last_error_string()
    rc = _lib.lib.sa_gqa_attend(cache.handle, 0, q.data_ptr(), out.data_ptr(), _lib.SA_DTYPE_FLOAT, 1, s, 1, 0, 0.0,
                                None, None, 0, 0, 0, stream)
    assert rc == _lib.SA_ERR_UNSUPPORTED
    torch.cuda.synchronize(dev)
    cache.close()
