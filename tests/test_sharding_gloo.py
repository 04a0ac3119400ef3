"""Multi-process host logic of the sharded modes, on CPU with ``gloo`` ranks.

World size 2.  Each rank computes its shard of heads with the CPU oracle
(signs seeded by the *global* KV-head index, as the sharded GpuKvCache does),
all-gathers through ``smallaios_b200.sharding.gather_head_shards`` and
compares with the unsharded oracle bit for bit: the per-head arithmetic is the
same, so any difference is a shard, seed or gather-layout error.
"""
import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

import oracle
from smallaios_b200 import sharding
from smallaios_b200.ops import ShapeMismatch
from tests.helpers import oracle_append, oracle_attend, rng, rope_tables

B, HQ, HKV, D, T, BITS, LAYERS, LAYER = 2, 8, 4, 32, 24, 4, 2, 1


def _inputs():
    r = rng(123)
    k = (r.standard_normal((B, T, HKV, D)) * 1.3).astype(np.float32)
    v = (r.standard_normal((B, T, HKV, D)) * 1.3).astype(np.float32)
    q = (r.standard_normal((B, 1, HQ, D)) * 1.3).astype(np.float32)
    return q, k, v


def _attend(q, k, v, signs, cos, sin):
    kc, km, vc, vm = oracle_append(k, v, signs, BITS, 0, cos, sin, True, False)
    return oracle_attend(q, kc, km, vc, vm, signs, BITS, T - 1, cos=cos, sin=sin, do_rotary=True)


def _full_reference():
    q, k, v = _inputs()
    cos, sin = rope_tables(T, D, 10000.0)
    signs = oracle.cache_signs(oracle.DEFAULT_SEED, LAYERS, HKV, D)[LAYER]
    return _attend(q, k, v, signs, cos, sin)  # (B, 1, HQ*D)


def _worker(rank, world, port, result_path):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        shard = sharding.head_shard(HQ, HKV, world, rank)
        q, k, v = _inputs()
        cos, sin = rope_tables(T, D, 10000.0)
        signs = oracle.cache_signs(oracle.DEFAULT_SEED, LAYERS, HKV, D)[LAYER]
        ks = slice(shard.kv_begin, shard.kv_begin + shard.kv_count)
        qs = slice(shard.q_begin, shard.q_begin + shard.q_count)
        local = _attend(q[:, :, qs], k[:, :, ks], v[:, :, ks], signs[ks], cos, sin)  # (B, 1, q_count*D)
        full = sharding.gather_head_shards(torch.from_numpy(np.ascontiguousarray(local)), shard)
        # batch sharding: rows partition the batch with no overlap
        rows = [sharding.batch_shard(5, world, r) for r in range(world)]
        if rank == 0:
            np.save(result_path, full.numpy())
            np.save(result_path + ".rows.npy", np.array(rows))
        dist.barrier()
    finally:
        dist.destroy_process_group()


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def test_head_sharded_gather_matches_unsharded(tmp_path):
    path = str(tmp_path / "gathered.npy")
    mp.spawn(_worker, args=(2, _free_port(), path), nprocs=2, join=True)
    got = np.load(path)
    want = _full_reference()
    assert got.shape == want.shape == (B, 1, HQ * D)
    assert np.array_equal(got.view(np.uint32), want.view(np.uint32))
    rows = np.load(path + ".rows.npy")
    assert rows.tolist() == [[0, 3], [3, 2]]


@pytest.mark.parametrize("hq,hkv,world", [(32, 8, 1), (32, 8, 2), (32, 8, 4), (32, 8, 8), (64, 8, 8), (8, 2, 2)])
def test_head_shard_covers_heads_once(hq, hkv, world):
    shards = [sharding.head_shard(hq, hkv, world, r) for r in range(world)]
    kv = [h for s in shards for h in range(s.kv_begin, s.kv_begin + s.kv_count)]
    qh = [h for s in shards for h in range(s.q_begin, s.q_begin + s.q_count)]
    assert kv == list(range(hkv)) and qh == list(range(hq))
    for s in shards:  # a rank's query heads are exactly the groups of its KV heads
        assert s.q_begin == s.kv_begin * (hq // hkv) and s.q_count == s.kv_count * (hq // hkv)


def test_head_shard_rejects_uneven_splits():
    with pytest.raises(ShapeMismatch):
        sharding.head_shard(32, 8, 3, 0)
    with pytest.raises(ShapeMismatch):
        sharding.head_shard(30, 8, 2, 0)
    with pytest.raises(ValueError):
        sharding.head_shard(32, 8, 2, 2)


def test_batch_shard_partitions_rows():
    for batch in (1, 7, 64):
        for world in (1, 2, 3, 8):
            spans = [sharding.batch_shard(batch, world, r) for r in range(world)]
            covered = [i for b0, n in spans for i in range(b0, b0 + n)]
            assert covered == list(range(batch))
