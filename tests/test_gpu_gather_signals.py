"""The on-device completion of the head-sharded gather, on one GPU.

With signal arrays, the kernel that writes the gathered output (the decode
merge, or the scatter after the generic attention) publishes a per-step epoch
to every rank's signal array and waits, bounded, for every rank's epoch in its
own.  On one GPU:

* a one-rank gather completes by itself and its buffer equals attn_out;
* a two-rank gather whose second "rank" never runs is a flag that nothing sets:
  the wait runs out after its short limit, the cache's device status reports
  it (bit 0, the SA_ERR_TIMEOUT condition), the context stays usable, and the
  next call is clean.
"""
import ctypes

import numpy as np
import pytest
import torch

from tests.helpers import rng, rope_tables

pytestmark = pytest.mark.gpu


def _case(dev, b=4, hq=32, hkv=8, d=128, t=300, s=1, dtype=torch.bfloat16):
    import smallaios_b200 as sa

    r = rng(90)
    cos, sin = rope_tables(t + 8, d, 500000.0)
    cos_t, sin_t = torch.from_numpy(cos).to(dev), torch.from_numpy(sin).to(dev)
    cache = sa.GpuKvCache(1, hkv, d, t + 8, batch=b, num_heads=hq, bits=4, device=dev)
    k = torch.from_numpy((r.standard_normal((b, t - s, hkv * d)) * 1.28).astype(np.float32)).to(dtype).to(dev)
    v = torch.from_numpy((r.standard_normal((b, t - s, hkv * d)) * 1.28).astype(np.float32)).to(dtype).to(dev)
    cache.append(0, k, v, cos_cache=cos_t, sin_cache=sin_t, do_rotary=True)
    cache.advance_position(t - s)
    q = torch.from_numpy((r.standard_normal((b, s, hq * d)) * 1.28).astype(np.float32)).to(dtype).to(dev)
    kn = torch.from_numpy((r.standard_normal((b, s, hkv * d)) * 1.28).astype(np.float32)).to(dtype).to(dev)
    vn = torch.from_numpy((r.standard_normal((b, s, hkv * d)) * 1.28).astype(np.float32)).to(dtype).to(dev)
    return cache, cos_t, sin_t, q, kn, vn


def _set_gather(cache, bufs, sigs, rank, timeout_us):
    from smallaios_b200._lib import check, lib

    bp = (ctypes.c_void_p * len(bufs))(*[x.data_ptr() for x in bufs])
    sp = (ctypes.c_void_p * len(sigs))(*[x.data_ptr() for x in sigs]) if sigs else None
    check(lib.sa_kv_cache_set_gather(cache.handle, bp, sp, len(bufs), rank, 0, cache.config.num_heads, timeout_us))


def _clear_gather(cache):
    from smallaios_b200._lib import check, lib

    check(lib.sa_kv_cache_set_gather(cache.handle, None, None, 0, 0, 0, 0, 0))


@pytest.mark.parametrize("s", [1, 5])  # the decode merge (1 token) and the generic path's scatter (5 tokens)
def test_one_rank_gather_completes_on_device(cuda_device, s):
    import smallaios_b200 as sa

    cache, cos, sin, q, k, v = _case(cuda_device, s=s)
    want = sa.group_query_attention(q, k, v, cache, 0, num_heads=32, kv_num_heads=8, cos_cache=cos, sin_cache=sin)
    buf = torch.full_like(want, float("nan"))
    sig = torch.zeros(16, dtype=torch.int32, device=cuda_device)
    _set_gather(cache, [buf], [sig], 0, 1_000_000)
    for step in range(3):  # the epoch advances on the device every call
        buf.fill_(float("nan"))
        sa.group_query_attention(q, k, v, cache, 0, num_heads=32, kv_num_heads=8, cos_cache=cos, sin_cache=sin)
        torch.cuda.synchronize()
        assert torch.equal(buf, want)
        assert int(sig[0]) == step + 1  # this rank's epoch, published to itself
        assert int(sig[8]) == 0 and int(sig[9]) == step + 1  # CTA counter reset, epoch
    _clear_gather(cache)
    assert cache.device_status() == 0
    cache.close()


def test_gather_wait_for_a_missing_rank_runs_out(cuda_device):
    """Buffer and signals of a second rank that never runs: nothing publishes its epoch, so the
    merge kernel's bounded wait (20 ms here) gives up and reports it; the context stays usable."""
    import smallaios_b200 as sa

    cache, cos, sin, q, k, v = _case(cuda_device)
    want = sa.group_query_attention(q, k, v, cache, 0, num_heads=32, kv_num_heads=8, cos_cache=cos, sin_cache=sin)
    bufs = [torch.zeros_like(want), torch.zeros_like(want)]
    sigs = [torch.zeros(16, dtype=torch.int32, device=cuda_device) for _ in range(2)]
    _set_gather(cache, bufs, sigs, 0, 20_000)
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    ev0.record()
    sa.group_query_attention(q, k, v, cache, 0, num_heads=32, kv_num_heads=8, cos_cache=cos, sin_cache=sin)
    ev1.record()
    torch.cuda.synchronize()
    assert ev0.elapsed_time(ev1) >= 15.0  # it waited about the limit, then returned
    assert cache.device_status(clear=True) == 1
    assert int(sigs[1][0]) == 1  # it did publish its own epoch to the other rank
    assert torch.equal(bufs[0], want) and torch.equal(bufs[1], want)  # the stores themselves completed
    _clear_gather(cache)
    out = sa.group_query_attention(q, k, v, cache, 0, num_heads=32, kv_num_heads=8, cos_cache=cos, sin_cache=sin)
    torch.cuda.synchronize()
    assert cache.device_status() == 0
    assert torch.equal(out, want)
    cache.close()


def test_set_gather_validation(cuda_device):
    from smallaios_b200._lib import SA_ERR_INVALID_ARGUMENT, lib

    cache, *_ = _case(cuda_device, t=40)
    buf = torch.zeros(4, 1, 32 * 128, dtype=torch.bfloat16, device=cuda_device)
    sig = torch.zeros(16, dtype=torch.int32, device=cuda_device)
    bp = (ctypes.c_void_p * 1)(buf.data_ptr())
    sp = (ctypes.c_void_p * 1)(sig.data_ptr())
    assert lib.sa_kv_cache_set_gather(cache.handle, bp, sp, 1, 1, 0, 32, 1000) == SA_ERR_INVALID_ARGUMENT
    assert lib.sa_kv_cache_set_gather(cache.handle, bp, sp, 1, 0, 0, 32, 0) == SA_ERR_INVALID_ARGUMENT
    assert lib.sa_kv_cache_set_gather(cache.handle, bp, sp, 1, 0, 0, 32, 1000) == 0
    assert lib.sa_kv_cache_set_gather(cache.handle, None, None, 0, 0, 0, 0, 0) == 0
    cache.close()
