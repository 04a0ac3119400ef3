"""Multi-GPU sharding of the decode path (one process per GPU, torch.distributed).

Every (batch row, KV head) unit of a layer is independent, so the path shards
without a collective on its data path except in the head-sharded mode:

* **KV-head sharding.** Rank r of G owns KV heads ``[r*Hkv/G, (r+1)*Hkv/G)``
  and their ``Hq/G`` query heads for every sequence.  Its cache holds only
  those heads (``GpuKvCache(kv_head_begin=..., kv_head_count=...)``); the
  PolarQuant sign seed still uses the global head index, so the shard holds
  exactly the codes the unsharded cache would.  After its local
  GroupQueryAttention the ranks all-gather ``attn_out`` over NCCL (each sends
  ``B*S*(Hq/G)*D`` activations), and the gathered ``[G][B][S][Hq/G*D]`` is
  returned in the operator's ``[B][S][Hq*D]`` head order.  With a
  ``PeerGather`` the collective disappears into the decode kernel instead: its
  merge epilogue stores every rank's copy over NVLink into symmetric-memory
  buffers (``sa_kv_cache_set_gather``) and completes the gather on the device
  with per-step epoch signals and a bounded wait.
* **Batch sharding.** Rank r owns whole sequences; no collective.

The reference runs one process on one device; its executor would call the
local operator per rank and this gather once per layer.
"""
from __future__ import annotations

import ctypes
from dataclasses import dataclass

import torch
import torch.distributed as dist

from ._lib import lib
from .ops import ShapeMismatch, _raise_op, group_query_attention


@dataclass(frozen=True)
class HeadShard:
    """The heads rank ``rank`` of ``world`` owns in the KV-head-sharded mode."""

    world: int
    rank: int
    kv_begin: int
    kv_count: int
    q_begin: int
    q_count: int


def head_shard(num_heads: int, kv_num_heads: int, world: int, rank: int) -> HeadShard:
    if world <= 0 or not 0 <= rank < world:
        raise ValueError(f"head_shard: rank {rank} outside world {world}")
    if num_heads <= 0 or kv_num_heads <= 0 or num_heads % kv_num_heads:
        raise ShapeMismatch("head_shard: num_heads must be a positive multiple of kv_num_heads")
    if kv_num_heads % world:
        raise ShapeMismatch(f"head_shard: {kv_num_heads} KV heads do not split over {world} ranks")
    kv_count = kv_num_heads // world
    group = num_heads // kv_num_heads
    return HeadShard(world, rank, rank * kv_count, kv_count, rank * kv_count * group, kv_count * group)


def batch_shard(batch: int, world: int, rank: int) -> tuple[int, int]:
    """Rows ``[begin, begin + count)`` of rank ``rank`` in the batch-sharded mode."""
    if world <= 0 or not 0 <= rank < world:
        raise ValueError(f"batch_shard: rank {rank} outside world {world}")
    base, extra = divmod(batch, world)
    begin = rank * base + min(rank, extra)
    return begin, base + (1 if rank < extra else 0)


def take_heads(x: torch.Tensor, begin: int, count: int, head_dim: int) -> torch.Tensor:
    """Columns of heads ``[begin, begin + count)`` of a ``(B, S, H*D)`` activation, contiguous."""
    return x[..., begin * head_dim:(begin + count) * head_dim].contiguous()


def gather_head_shards(local_out: torch.Tensor, shard: HeadShard, group=None,
                       out: torch.Tensor | None = None) -> torch.Tensor:
    """All-gather ``(B, S, q_count*D)`` shards into ``(B, S, Hq*D)`` in head order."""
    if local_out.dim() != 3:
        raise ShapeMismatch("gather_head_shards: attn_out must be (B, S, Hq_local*D)")
    local_out = local_out.contiguous()
    b, s, w = local_out.shape
    parts = torch.empty((shard.world, b, s, w), dtype=local_out.dtype, device=local_out.device)
    if dist.get_backend(group) == dist.Backend.NCCL:
        dist.all_gather_into_tensor(parts.view(shard.world * b, s, w), local_out, group=group)
    else:
        dist.all_gather(list(parts.unbind(0)), local_out, group=group)
    full = parts.permute(1, 2, 0, 3).reshape(b, s, shard.world * w)
    if out is not None:
        out.copy_(full)
        return out
    return full


class PeerGather:
    """Gathered-output buffers in symmetric memory for the fused head-sharded gather.

    Every rank allocates ``nbuf`` buffers of ``shape`` (``(B, S, Hq*D)``) and one
    signal array with torch's symmetric memory, so each rank's buffers and
    signals are mapped into every rank.  A step points the cache at one buffer
    set (``sa_kv_cache_set_gather``): the attention's merge kernel stores this
    rank's heads into all ranks' copies over NVLink, then its last CTA publishes
    the step's epoch to every peer and waits (bounded by ``timeout_ms``) until
    every peer has published it here.  When the operator's kernels finish, the
    gathered output is complete on this rank: no host barrier, no extra launch.
    Buffers alternate between steps, so a rank never writes a buffer a peer may
    still be reading; a CUDA graph of the loop therefore holds one step per
    buffer (the epoch itself lives on the device and advances on every replay).
    A wait that runs out sets the cache's device status (``cache.device_status()``).
    """

    SIGNAL_WORDS = 16  # one epoch per rank (up to 8), the CTA counter and the epoch, padded

    def __init__(self, shape, dtype, device, group=None, nbuf: int = 2, timeout_ms: float = 1000.0):
        from torch.distributed import _symmetric_memory as symm_mem

        if nbuf < 2:
            raise ValueError("PeerGather: at least two buffers alternate")
        group = group if group is not None else dist.group.WORLD
        self.bufs, self.handles, self.ptrs = [], [], []
        for _ in range(nbuf):
            t = symm_mem.empty(tuple(shape), dtype=dtype, device=device)
            h = symm_mem.rendezvous(t, group)
            ptrs = list(h.buffer_ptrs)
            self.bufs.append(t)
            self.handles.append(h)
            self.ptrs.append((ctypes.c_void_p * len(ptrs))(*ptrs))
        self.signals = symm_mem.empty((self.SIGNAL_WORDS,), dtype=torch.int32, device=device)
        self.signals.zero_()
        self.sig_handle = symm_mem.rendezvous(self.signals, group)
        sp = list(self.sig_handle.buffer_ptrs)
        self.sig_ptrs = (ctypes.c_void_p * len(sp))(*sp)
        self.rank = self.sig_handle.rank
        self.timeout_us = max(1, int(timeout_ms * 1000))
        # every rank's signals are zero before any rank's kernel can publish into them
        torch.cuda.synchronize(device)
        dist.barrier(group=group, device_ids=[torch.device(device).index])
        self.next = 0

    def step(self, cache, shard: HeadShard, num_heads: int, run):
        """Run ``run()`` (the local operator call) with its output gathered; returns the buffer."""
        i = self.next
        self.next = (i + 1) % len(self.bufs)
        ptrs = self.ptrs[i]
        _raise_op(lib.sa_kv_cache_set_gather(cache.handle, ptrs, self.sig_ptrs, len(ptrs), self.rank, shard.q_begin,
                                             num_heads, self.timeout_us), "kv_cache_set_gather")
        try:
            run()
        finally:
            _raise_op(lib.sa_kv_cache_set_gather(cache.handle, None, None, 0, 0, 0, 0, 0), "kv_cache_set_gather")
        return self.bufs[i]


def sharded_group_query_attention(query: torch.Tensor, key: torch.Tensor, value: torch.Tensor, cache, layer: int, *,
                                  num_heads: int, kv_num_heads: int, shard: HeadShard, group=None,
                                  local_out: torch.Tensor | None = None, out: torch.Tensor | None = None,
                                  gather: PeerGather | None = None, **kwargs) -> torch.Tensor:
    """GroupQueryAttention on this rank's heads, then the all-gather of attn_out.

    ``query``/``key``/``value`` are this rank's shards, ``(B, S, q_count*D)``
    and ``(B, S, kv_count*D)`` (the column-parallel Q/K/V projections produce
    them); ``num_heads``/``kv_num_heads`` are the model's global attributes.
    Returns ``(B, S, num_heads*D)``: NCCL all-gather of the local output, or,
    with ``gather``, the fused peer-store gather (the returned buffer belongs
    to ``gather`` and is overwritten two steps later).
    """
    cfg = cache.config
    if (cfg.kv_head_begin, cfg.kv_head_count) != (shard.kv_begin, shard.kv_count):
        raise ShapeMismatch("sharded GroupQueryAttention: the cache does not hold this rank's KV heads")
    if gather is not None:  # the decode's epilogue writes every rank's copy; no collective
        return gather.step(cache, shard, num_heads, lambda: group_query_attention(
            query, key, value, cache, layer, num_heads=num_heads, kv_num_heads=kv_num_heads, out=local_out,
            **kwargs))
    local = group_query_attention(query, key, value, cache, layer, num_heads=num_heads, kv_num_heads=kv_num_heads,
                                  out=local_out, **kwargs)
    return gather_head_shards(local, shard, group, out)
