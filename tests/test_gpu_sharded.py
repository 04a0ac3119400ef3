"""KV-head-sharded GroupQueryAttention on 2 GPUs (NCCL all-gather of attn_out).

Each rank appends its KV heads' shard of a seeded prefill, then runs one
sharded decode step.  Its cache codes must equal the oracle's codes for those
global heads bit for bit, and the gathered output must match the unsharded
oracle within the operator's tolerance.  Skipped with fewer than 2 GPUs.
"""
import os
import socket
from datetime import timedelta

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

import oracle
from tests.helpers import oracle_append, oracle_attend, rng, rope_tables

pytestmark = pytest.mark.gpu

B, HQ, HKV, D, T, BITS, LAYERS, LAYER = 3, 16, 4, 128, 300, 4, 2, 1
TOL = 1e-3


def _inputs():
    r = rng(321)
    k = (r.standard_normal((B, T, HKV, D)) * 1.28).astype(np.float32)
    v = (r.standard_normal((B, T, HKV, D)) * 1.28).astype(np.float32)
    q = (r.standard_normal((B, 1, HQ, D)) * 1.28).astype(np.float32)
    return q, k, v


def _worker(rank, world, port, result_path):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dev = torch.device("cuda", rank)
    torch.cuda.set_device(dev)
    dist.init_process_group("nccl", rank=rank, world_size=world, device_id=dev, timeout=timedelta(seconds=60))
    import smallaios_b200 as sa
    from smallaios_b200 import sharding

    try:
        shard = sharding.head_shard(HQ, HKV, world, rank)
        q, k, v = _inputs()
        cos, sin = rope_tables(T, D, 10000.0)
        tcos, tsin = torch.from_numpy(cos).to(dev), torch.from_numpy(sin).to(dev)
        ks = slice(shard.kv_begin, shard.kv_begin + shard.kv_count)
        qs = slice(shard.q_begin, shard.q_begin + shard.q_count)
        cache = sa.GpuKvCache(LAYERS, HKV, D, T, batch=B, num_heads=HQ, bits=BITS, kv_head_begin=shard.kv_begin,
                              kv_head_count=shard.kv_count, device=dev)

        def local(x, sl):  # (B, S, H, D) numpy -> this rank's heads as (B, S, h*D) on the device
            x = np.ascontiguousarray(x[:, :, sl])
            return torch.from_numpy(x.reshape(x.shape[0], x.shape[1], -1)).to(dev)

        cache.append(LAYER, local(k[:, :T - 1], ks), local(v[:, :T - 1], ks), cos_cache=tcos, sin_cache=tsin,
                     do_rotary=True)
        cache.advance_position(T - 1)
        out = sharding.sharded_group_query_attention(
            local(q, qs), local(k[:, T - 1:], ks), local(v[:, T - 1:], ks), cache, LAYER, num_heads=HQ,
            kv_num_heads=HKV, shard=shard, cos_cache=tcos, sin_cache=tsin, do_rotary=True)
        torch.cuda.synchronize(dev)
        # the same step with the fused gather (decode epilogue stores into every rank's buffer)
        gather = sharding.PeerGather((B, 1, HQ * D), torch.float32, dev)
        peer_ok = True
        for _ in range(3):  # both buffers, then the first again
            cache.set_position(T - 1)
            got = sharding.sharded_group_query_attention(
                local(q, qs), local(k[:, T - 1:], ks), local(v[:, T - 1:], ks), cache, LAYER, num_heads=HQ,
                kv_num_heads=HKV, shard=shard, cos_cache=tcos, sin_cache=tsin, do_rotary=True, gather=gather)
            torch.cuda.synchronize(dev)
            peer_ok = peer_ok and torch.equal(got, out)
        # A CUDA graph of two fused steps (one per buffer), replayed with new queries each time:
        # every replay's gathered outputs must equal the NCCL gather of the same step.
        qd = local(q, qs).clone()
        kd, vd = local(k[:, T - 1:], ks).clone(), local(v[:, T - 1:], ks).clone()
        res = [torch.empty(B, 1, HQ * D, device=dev) for _ in range(2)]

        def two_steps():
            for j in range(2):
                cache.set_position(T - 1)
                g = sharding.sharded_group_query_attention(
                    qd, kd, vd, cache, LAYER, num_heads=HQ, kv_num_heads=HKV, shard=shard, cos_cache=tcos,
                    sin_cache=tsin, do_rotary=True, gather=gather)
                res[j].copy_(g)

        two_steps()
        torch.cuda.synchronize(dev)
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph):
            two_steps()
        for it in range(4):
            qn = (rng(500 + it).standard_normal((B, 1, HQ, D)) * 1.28).astype(np.float32)
            qd.copy_(local(qn, qs))
            graph.replay()
            torch.cuda.synchronize(dev)
            cache.set_position(T - 1)
            ref = sharding.sharded_group_query_attention(
                qd, kd, vd, cache, LAYER, num_heads=HQ, kv_num_heads=HKV, shard=shard, cos_cache=tcos,
                sin_cache=tsin, do_rotary=True)
            torch.cuda.synchronize(dev)
            peer_ok = peer_ok and torch.equal(res[0], ref) and torch.equal(res[1], ref)
        # The same graph replayed 16 times back to back with no host synchronisation in between (a
        # rank may run ahead of its peer by up to the gather's own wait): every step's gathered
        # output, copied out on the stream right after the step, must still equal its NCCL gather.
        qns = [local((rng(700 + it).standard_normal((B, 1, HQ, D)) * 1.28).astype(np.float32), qs)
               for it in range(16)]
        kept = []
        for qn in qns:
            qd.copy_(qn)
            graph.replay()
            kept.append((res[0].clone(), res[1].clone()))
        torch.cuda.synchronize(dev)
        for qn, (r0, r1) in zip(qns, kept):
            qd.copy_(qn)
            cache.set_position(T - 1)
            ref = sharding.sharded_group_query_attention(
                qd, kd, vd, cache, LAYER, num_heads=HQ, kv_num_heads=HKV, shard=shard, cos_cache=tcos,
                sin_cache=tsin, do_rotary=True)
            torch.cuda.synchronize(dev)
            peer_ok = peer_ok and torch.equal(r0, ref) and torch.equal(r1, ref)
        graph.reset()
        peer_ok = peer_ok and cache.device_status() == 0
        # this rank's codes against the oracle for its global heads
        signs = oracle.cache_signs(oracle.DEFAULT_SEED, LAYERS, HKV, D)[LAYER]
        kc, km, vc, vm = oracle_append(k[:, :, ks], v[:, :, ks], signs[ks], BITS, 0, cos, sin, True, False)
        view = cache.view(LAYER)
        ok = (np.array_equal(view.k_codes[:, :, :T].cpu().numpy(), kc)
              and np.array_equal(view.v_codes_tokens()[:, :, :T].cpu().numpy(), vc)
              and np.array_equal(view.k_meta[:, :, :T].cpu().numpy().view(np.uint32), km.view(np.uint32))
              and np.array_equal(view.v_meta[:, :, :T].cpu().numpy().view(np.uint32), vm.view(np.uint32)))
        flag = torch.tensor([0 if ok else 1, 0 if peer_ok else 1], device=dev)
        dist.all_reduce(flag)
        if rank == 0:
            np.save(result_path, out.float().cpu().numpy())
            np.save(result_path + ".codes.npy", flag.cpu().numpy())
        cache.close()
        dist.barrier(device_ids=[rank])
    finally:
        dist.destroy_process_group()


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs 2 GPUs")
def test_head_sharded_decode_two_gpus(tmp_path):
    path = str(tmp_path / "out.npy")
    mp.spawn(_worker, args=(2, _free_port(), path), nprocs=2, join=True)
    flags = np.load(path + ".codes.npy")
    assert flags[0] == 0, "a rank's cache codes differ from the oracle"
    assert flags[1] == 0, "the fused peer-store gather differs from the NCCL all-gather"
    got = np.load(path)
    q, k, v = _inputs()
    cos, sin = rope_tables(T, D, 10000.0)
    signs = oracle.cache_signs(oracle.DEFAULT_SEED, LAYERS, HKV, D)[LAYER]
    kc, km, vc, vm = oracle_append(k, v, signs, BITS, 0, cos, sin, True, False)
    want = oracle_attend(q, kc, km, vc, vm, signs, BITS, T - 1, cos=cos, sin=sin, do_rotary=True)
    err = np.abs(got - want).max()
    assert err <= TOL, f"max abs error {err}"
