"""Parity of the stream-K decode path at the sizes the benchmark runs.

The decode kernels cut every (batch row, KV head) unit's context into chunks
and give warp w of a persistent grid the flat chunk range
[w*F/W, (w+1)*F/W).  When F (all chunks) is well above W (all warps), a warp
walks several two-chunk sub-segments through its two shared-memory slots,
reuses slots and mbarrier phases across chunks, folds its integer sums across
sub-segments under a moving reference, and its range starts and ends inside
units, so several warps' records merge into one output.  The cases here make
F several times W and compare with the composite CPU oracle (PolarQuantizer::
encode of every token, read_k/read_v, causal SDPA: kv_compression.rs:814-899,
ops/microsoft.rs:380-438).  Bar: max-abs 1e-3 with f32 activations, plus half
an output ulp for bf16.

The last two cases are the benchmark's own configurations (BASELINE configs 3
and 5 at full batch and context), checked on a sample of batch rows.
"""
import numpy as np
import pytest
import torch

from tests.helpers import oracle_append, oracle_attend, rope_tables
from tests.test_gpu_gqa import _check, _decode_case

pytestmark = pytest.mark.gpu

# Warps of the persistent decode grid per SM: two CTAs of 8 warps (group <= 4),
# one CTA of 12 warps (group 5..8).
_WARPS_PER_SM = {4: 16, 8: 12}


def _chunks_per_warp(b, hq, hkv, d, bits, t):
    """(F, W) of the decode kernel for this shape on this device."""
    sms = torch.cuda.get_device_properties(0).multi_processor_count
    group = hq // hkv
    ct = 32 if d * bits // 8 > 64 else 64
    f = b * hkv * ((t + ct - 1) // ct)
    w = min(sms * _WARPS_PER_SM[4 if group <= 4 else 8], f)
    return f, w


@pytest.mark.parametrize("b,hq,hkv,d,bits,t,dtype", [
    (16, 32, 8, 128, 4, 2048 + 37, torch.float32),   # G=4, ~1.8 chunks per warp
    (16, 32, 8, 128, 4, 2048 + 37, torch.bfloat16),
    (8, 32, 8, 128, 4, 8192 + 37, torch.float32),    # ~3.5 chunks per warp
    (8, 32, 8, 128, 8, 4096 + 11, torch.float32),    # 8-bit D=128: 32-token chunks
    (8, 32, 8, 128, 8, 4096 + 11, torch.bfloat16),
    (16, 16, 8, 128, 4, 4096 + 1, torch.float32),    # G=2
    (6, 24, 8, 64, 4, 8192 + 63, torch.float16),     # D=64, G=3, a chunk of 63 tokens at the end
])
def test_many_chunks_per_warp_group4(cuda_device, b, hq, hkv, d, bits, t, dtype):
    f, w = _chunks_per_warp(b, hq, hkv, d, bits, t)
    assert f > 1.5 * w, (f, w)
    got, want = _decode_case(cuda_device, b=b, hq=hq, hkv=hkv, d=d, bits=bits, t=t, dtype=dtype, seed=100 + t + b,
                             chunks=(1000, 517), theta=500000.0)
    _check(got, want, dtype)


@pytest.mark.parametrize("b,hq,hkv,d,bits,t,dtype", [
    (8, 64, 8, 128, 4, 4096 + 5, torch.float32),     # G=8, ~2.3 chunks per warp
    (8, 64, 8, 128, 4, 4096 + 5, torch.bfloat16),
    (4, 64, 8, 128, 4, 16384 + 3, torch.float32),    # ~4.6 chunks per warp
    (12, 48, 8, 128, 8, 2048 + 29, torch.float32),   # G=6, 8-bit
])
def test_many_chunks_per_warp_group8(cuda_device, b, hq, hkv, d, bits, t, dtype):
    f, w = _chunks_per_warp(b, hq, hkv, d, bits, t)
    assert f > 1.5 * w, (f, w)
    got, want = _decode_case(cuda_device, b=b, hq=hq, hkv=hkv, d=d, bits=bits, t=t, dtype=dtype, seed=200 + t + b,
                             chunks=(1000, 517), theta=500000.0)
    _check(got, want, dtype)


def _bench_config_case(dev, *, b, hq, hkv, d, t, rows, seed, std=1.28, theta=500000.0, bits=4):
    """The benchmark's workload: the cache filled by bulk appends of device-generated bf16 K/V
    (t - 1 tokens), then one GroupQueryAttention step (append of the newest token + attention).
    The K/V of the sampled ``rows`` are kept on the host for the oracle."""
    import smallaios_b200 as sa

    g = torch.Generator(device=dev)
    g.manual_seed(seed)
    cos, sin = rope_tables(t + 8, d, theta)
    cos_t, sin_t = torch.from_numpy(cos).to(dev), torch.from_numpy(sin).to(dev)
    cache = sa.GpuKvCache(1, hkv, d, t, batch=b, num_heads=hq, bits=bits, device=dev)
    ks, vs = [], []
    pos, chunk = 0, 512
    while pos < t:
        n = min(chunk, t - 1 - pos) if pos < t - 1 else 1
        k = (torch.randn(b, n, hkv * d, device=dev, generator=g) * std).to(torch.bfloat16)
        v = (torch.randn(b, n, hkv * d, device=dev, generator=g) * std).to(torch.bfloat16)
        ks.append(k[rows].float().cpu().numpy())
        vs.append(v[rows].float().cpu().numpy())
        if pos < t - 1:
            cache.append(0, k, v, cos_cache=cos_t, sin_cache=sin_t, do_rotary=True)
            cache.advance_position(n)
        else:
            q = (torch.randn(b, 1, hq * d, device=dev, generator=g) * std).to(torch.bfloat16)
            out = sa.group_query_attention(q, k, v, cache, 0, num_heads=hq, kv_num_heads=hkv, cos_cache=cos_t,
                                           sin_cache=sin_t, do_rotary=True)
        pos += n
    torch.cuda.synchronize(dev)
    got = out[rows].float().cpu().numpy()
    qn = q[rows].float().cpu().numpy().reshape(len(rows), 1, hq, d)
    view = cache.view(0)
    kc_dev = view.k_codes[rows, :, :t].cpu().numpy()
    vc_dev = view.v_codes_tokens()[rows][:, :, :t].cpu().numpy()
    km_dev = view.k_meta[rows, :, :t].cpu().numpy()
    vm_dev = view.v_meta[rows, :, :t].cpu().numpy()
    signs = view.signs.cpu().numpy().astype(np.int8)
    cache.close()
    k_all = np.concatenate(ks, axis=1).reshape(len(rows), t, hkv, d)
    v_all = np.concatenate(vs, axis=1).reshape(len(rows), t, hkv, d)
    kc, km, vc, vm = oracle_append(k_all, v_all, signs, bits, 0, cos, sin, True, False)
    assert np.array_equal(kc_dev, kc)
    assert np.array_equal(vc_dev, vc)
    assert np.array_equal(km_dev.view(np.uint32), km.view(np.uint32))
    assert np.array_equal(vm_dev.view(np.uint32), vm.view(np.uint32))
    want = oracle_attend(qn, kc, km, vc, vm, signs, bits, t - 1, cos=cos, sin=sin, do_rotary=True)
    return got, want


def test_bench_config3_sampled_rows(cuda_device):
    """BASELINE config 3 exactly as bench.py runs it (B=64, 32/8 heads, D=128, T=8192, int4, bf16):
    about 28 chunks per warp; 6 of the 64 rows (48 of 512 units) against the oracle."""
    f, w = _chunks_per_warp(64, 32, 8, 128, 4, 8192)
    assert f > 20 * w
    rows = [0, 1, 17, 31, 46, 63]
    got, want = _bench_config_case(cuda_device, b=64, hq=32, hkv=8, d=128, t=8192, rows=rows, seed=1000)
    _check(got, want, torch.bfloat16)


def test_bench_config5_sampled_rows(cuda_device):
    """BASELINE config 5 (B=128, 64/8 heads, D=128, T=32768, int4, bf16): about 295 chunks per
    warp of the eight-head kernel; 2 of the 128 rows (16 units) against the oracle."""
    f, w = _chunks_per_warp(128, 64, 8, 128, 4, 32768)
    assert f > 200 * w
    rows = [5, 126]
    got, want = _bench_config_case(cuda_device, b=128, hq=64, hkv=8, d=128, t=32768, rows=rows, seed=1005)
    _check(got, want, torch.bfloat16)
