"""Cache persistence (state_dict / from_state_dict) and the memory footprint
(CompressedKVCache::memory_bytes, kv_compression.rs:928-957)."""
import numpy as np
import pytest
import torch

from tests.helpers import rng, rope_tables

pytestmark = pytest.mark.gpu


def _reference_memory_bytes(rows, layers, heads, batch, d, bits, qjl, lowrank):
    """The reference's accounting restated: QuantizedBlock (:166-168), QJLResidual (:352-354),
    LowRankK (:442-444) of rank 1 (the cache decomposes its first row alone)."""
    block = d * bits // 8 + 4 * 4 + 8 + 1
    per_row = 2 * block + (2 * (8 * ((d + 63) // 64) + 4 + 8) if qjl else 0)
    per_head = rows * per_row + ((rows + d) * 4 + 8 * 4 if lowrank and rows else 0)
    return layers * heads * batch * per_head


@pytest.mark.parametrize("qjl,lowrank", [(True, None), (False, None), (True, 32), (False, 4)])
def test_memory_bytes_follows_the_reference_accounting(cuda_device, qjl, lowrank):
    import smallaios_b200 as sa

    layers, heads, d, bits, rows, b = 2, 2, 64, 4, 128, 1
    cache = sa.GpuKvCache(layers, heads, d, 256, batch=b, bits=bits, qjl_residual=qjl, lowrank_k=lowrank,
                          device=cuda_device)
    assert cache.memory_bytes()[0] == 0
    r = rng(5)
    for layer in range(layers):
        k = torch.from_numpy((r.uniform(-1, 1, (b, rows, heads * d))).astype(np.float32)).to(cuda_device)
        v = torch.from_numpy((r.uniform(-1, 1, (b, rows, heads * d))).astype(np.float32)).to(cuda_device)
        cache.append(layer, k, v)
    cache.advance_position(rows)
    ref, dev = cache.memory_bytes()
    cache.close()
    assert ref == _reference_memory_bytes(rows, layers, heads, b, d, bits, qjl, lowrank)
    # integration_memory_footprint_ratio / cache_memory_footprint: compressed < f32
    assert ref < rows * layers * heads * d * 4 * 2
    assert dev >= ref


def test_state_round_trip_then_decode(cuda_device):
    """Save a cache (QJL and low-rank K on, past the re-decomposition at row 512), restore it into a
    fresh cache, then run the same decode steps on both: outputs and states stay identical."""
    import smallaios_b200 as sa

    b, hq, hkv, d, bits, past, steps = 2, 8, 2, 64, 4, 520, 3
    t = past + steps
    r = rng(21)
    k = torch.from_numpy((r.standard_normal((b, t, hkv * d)) * 1.28).astype(np.float32)).to(torch.bfloat16)
    v = torch.from_numpy((r.standard_normal((b, t, hkv * d)) * 1.28).astype(np.float32)).to(torch.bfloat16)
    q = torch.from_numpy((r.standard_normal((b, t, hq * d)) * 1.28).astype(np.float32)).to(torch.bfloat16)
    cos, sin = rope_tables(t + 4, d)
    tcos, tsin = torch.from_numpy(cos).to(cuda_device), torch.from_numpy(sin).to(cuda_device)
    kw = dict(batch=b, num_heads=hq, bits=bits, qjl_residual=True, lowrank_k=3, device=cuda_device)
    a = sa.GpuKvCache(1, hkv, d, t + 4, **kw)
    a.append(0, k[:, :past].to(cuda_device), v[:, :past].to(cuda_device), cos_cache=tcos, sin_cache=tsin,
             do_rotary=True)
    a.advance_position(past)
    state = a.state_dict()
    c = sa.GpuKvCache.from_state_dict(state, device=cuda_device)
    assert c.current_position() == past and c.memory_bytes() == a.memory_bytes()
    for i in range(past, t):
        outs = []
        for cache in (a, c):
            outs.append(sa.group_query_attention(q[:, i:i + 1].to(cuda_device), k[:, i:i + 1].to(cuda_device),
                                                 v[:, i:i + 1].to(cuda_device), cache, 0, num_heads=hq,
                                                 kv_num_heads=hkv, cos_cache=tcos, sin_cache=tsin))
            cache.advance_position(1)
        torch.cuda.synchronize()
        assert torch.equal(outs[0], outs[1]), f"step {i}"
    sa_, sc = a.state_dict(), c.state_dict()
    for name, ta in sa_["layers"][0].items():
        assert torch.equal(ta, sc["layers"][0][name]), name
    a.close()
    c.close()


def test_state_rejects_mismatched_options(cuda_device):
    import smallaios_b200 as sa

    a = sa.GpuKvCache(1, 2, 64, 32, qjl_residual=True, device=cuda_device)
    a.append(0, torch.zeros(1, 4, 128, device=cuda_device), torch.ones(1, 4, 128, device=cuda_device))
    a.advance_position(4)
    st = a.state_dict()
    a.close()
    st["config"]["qjl_residual"] = 0
    with pytest.raises(ValueError):
        sa.GpuKvCache.from_state_dict(st, device=cuda_device)
    with pytest.raises(ValueError):
        sa.GpuKvCache.from_state_dict({"format": "other"}, device=cuda_device)


def test_state_with_position_beyond_capacity_frees_the_new_cache(cuda_device):
    """A saved position past max_seq_len raises, and the cache built for it is released."""
    import smallaios_b200 as sa
    from smallaios_b200._lib import SaError

    a = sa.GpuKvCache(1, 2, 64, 32, device=cuda_device)
    a.append(0, torch.zeros(1, 4, 128, device=cuda_device), torch.ones(1, 4, 128, device=cuda_device))
    a.advance_position(4)
    st = a.state_dict()
    a.close()
    st["position"] = 33
    torch.cuda.synchronize()
    free0 = torch.cuda.mem_get_info(cuda_device)[0]
    with pytest.raises(SaError, match="position"):
        sa.GpuKvCache.from_state_dict(st, device=cuda_device)
    torch.cuda.synchronize()
    assert torch.cuda.mem_get_info(cuda_device)[0] >= free0
