"""Compressed, GPU-resident KV cache.

Host-side mirror of onnx-rt's ``GpuKvCache`` (onnx-rt/src/cuda/kv_cache.rs:
111-388) carrying the compression state of ``CompressedKVCache``
(onnx-rt/src/kv_compression.rs:742-925).  Storage, quantization and every
kernel live in libsa_b200.so; this class owns the handle and exposes the
layer views as torch tensors (zero-copy) for inspection.
"""
from __future__ import annotations

import ctypes
from dataclasses import dataclass

import torch

from . import _lib
from ._lib import check, lib

DEFAULT_SEED = 0xDEADBEEFCAFE1234  # KVCacheConfig::default (kv_compression.rs:724)


class _DevArray:
    """__cuda_array_interface__ wrapper so torch can view library memory."""

    def __init__(self, ptr: int, shape, typestr: str):
        self.__cuda_array_interface__ = {"shape": tuple(shape), "typestr": typestr, "data": (ptr, False),
                                         "version": 3, "strides": None}


def _view(ptr: int, shape, typestr: str, device) -> torch.Tensor:
    with torch.cuda.device(device):
        return torch.as_tensor(_DevArray(ptr, shape, typestr), device=device)


@dataclass
class LayerView:
    """GpuKvCache::view_at (kv_cache.rs:336-378), as torch tensors."""

    k_codes: torch.Tensor  # uint8 (B, H, T, CB)
    v_codes: torch.Tensor  # uint8 (B, H, T/16, CB/4, 4, 4, 4): 16-token blocks, see v_codes_tokens
    k_meta: torch.Tensor   # f32 (B, H, T, 2) {scale, zero_point}
    v_meta: torch.Tensor   # f32 (B, H, T, 2)
    signs: torch.Tensor    # f32 (H, D) +-1
    wht_scale: float
    bits: int
    code_bytes: int
    capacity: int
    # QJL residuals (KVCacheConfig::kv_qjl_residual), None unless the cache stores them
    k_qjl_bits: torch.Tensor | None = None  # uint8 (B, H, T, D/8): bit i of a vector = bit i%8 of byte i/8
    v_qjl_bits: torch.Tensor | None = None
    k_qjl_mag: torch.Tensor | None = None   # f32 (B, H, T): c_magnitude
    v_qjl_mag: torch.Tensor | None = None
    # low-rank K state (KVCacheConfig::kv_lowrank_k), None unless the cache keeps it
    lr_vt: torch.Tensor | None = None  # f32 (B, H, D): the rank-1 V^T row
    lr_us: torch.Tensor | None = None  # f32 (B, H, T): U*S, one coefficient per written row
    lr_kmeta: torch.Tensor | None = None  # f32 (B, H, T, 2): {0, U*S[t]}, the K metadata attention reads
    lr_vtr: torch.Tensor | None = None    # f32 (B, H, D): V^T rotated like the queries

    def v_codes_tokens(self) -> torch.Tensor:
        """V codes in per-token pack_bits order (B, H, T, CB).

        Library layout: per 16-token block, [chunk c][group g][byte jj][token tt]
        holds byte 4*c + jj of token 4*g + tt (16-byte chunks of the four
        4-token groups interleave, so a quarter-warp's tensor-core fragment
        loads hit 32 distinct shared-memory banks).
        """
        b, h, nblk, c4, g, jj, tt = self.v_codes.shape
        return self.v_codes.permute(0, 1, 2, 4, 6, 3, 5).reshape(b, h, nblk * g * tt, c4 * jj)


def qjl_correction(bits_a, mag_a, bits_b, mag_b, dim: int):
    """QJLResidualEncoder::correction (kv_compression.rs:401-417) of stored residual pairs, on the host.

    ``bits_*``: uint8 sign bytes (..., dim/8) as the cache stores them (LayerView.k_qjl_bits);
    ``mag_*``: their c_magnitude (...).  Returns C_a * C_b * (dim - 2 popcount(a ^ b)) / dim in
    f32, in the reference's operation order.  The reference computes the term but never applies
    it on read; this is the same helper for callers that want it.
    """
    import numpy as np

    to_np = (lambda t: t.cpu().numpy() if isinstance(t, torch.Tensor) else np.asarray(t))
    a, b = to_np(bits_a).astype(np.uint8), to_np(bits_b).astype(np.uint8)
    ma, mb = to_np(mag_a).astype(np.float32), to_np(mag_b).astype(np.float32)
    if dim == 0:
        return np.zeros(np.broadcast_shapes(ma.shape, mb.shape), np.float32)
    pop = np.unpackbits(np.bitwise_xor(a, b), axis=-1).sum(axis=-1, dtype=np.int64)
    sign_inner = np.float32(dim) - np.float32(2.0) * pop.astype(np.float32)
    return (ma * mb * sign_inner / np.float32(dim)).astype(np.float32)


class GpuKvCache:
    """Per-layer compressed K/V cache for a batch of sequences on one GPU.

    Mirrors ``GpuKvCache::allocate/append/advance_position/current_position/
    reset`` (kv_cache.rs).  ``kv_head_begin/kv_head_count`` select a shard of
    the KV heads (KV-head sharding across GPUs); the PolarQuant seed of each
    head still uses its global index, so a sharded cache holds exactly the
    codes the unsharded one would.  ``qjl_residual`` (KVCacheConfig::
    kv_qjl_residual) makes every append also store the QJL residual of each
    vector; nothing reads it back, as in the reference, so it is off by default.
    ``lowrank_k`` (KVCacheConfig::kv_lowrank_k) keeps the low-rank K state of
    LowRankKeyDecomposer; attention then reads keys as its reconstruction, as
    read_k does.
    """

    def __init__(self, num_layers: int, num_kv_heads: int, head_dim: int, max_seq_len: int, *,
                 batch: int = 1, num_heads: int | None = None, bits: int = 4, seed: int = DEFAULT_SEED,
                 kv_head_begin: int = 0, kv_head_count: int | None = None, qjl_residual: bool = False,
                 lowrank_k: int | None = None, device=None):
        self.device = torch.device(device if device is not None else "cuda", )
        if self.device.index is None:
            self.device = torch.device("cuda", torch.cuda.current_device())
        cfg = _lib.KvCacheConfig()
        cfg.num_layers = num_layers
        cfg.batch = batch
        cfg.num_heads = num_heads if num_heads is not None else num_kv_heads
        cfg.num_kv_heads = num_kv_heads
        cfg.kv_head_begin = kv_head_begin
        cfg.kv_head_count = kv_head_count if kv_head_count is not None else num_kv_heads - kv_head_begin
        cfg.head_dim = head_dim
        cfg.max_seq_len = max_seq_len
        cfg.bits = bits
        cfg.seed = seed & (2**64 - 1)
        cfg.qjl_residual = 1 if qjl_residual else 0
        # kv_lowrank_k: None = off; Some(0) means rank 1 (LowRankKeyDecomposer::new, :460-465)
        cfg.lowrank_k = 0 if lowrank_k is None else max(int(lowrank_k), 1)
        self._handle = ctypes.c_void_p()
        with torch.cuda.device(self.device):
            check(lib.sa_kv_cache_create(ctypes.byref(cfg), ctypes.byref(self._handle)))
        self.config = cfg

    # -- GpuKvCache API ------------------------------------------------------
    @classmethod
    def allocate(cls, num_layers, num_kv_heads, head_dim, max_seq_len, **kw) -> "GpuKvCache":
        return cls(num_layers, num_kv_heads, head_dim, max_seq_len, **kw)

    @property
    def handle(self) -> int:
        if not self._handle:
            raise RuntimeError("GpuKvCache used after close()")
        return self._handle.value

    def num_layers(self) -> int:
        return self.config.num_layers

    def max_seq_len(self) -> int:
        return self.config.max_seq_len

    def current_position(self) -> int:
        pos = ctypes.c_int64()
        check(lib.sa_kv_cache_position(self.handle, ctypes.byref(pos)))
        return pos.value

    def set_position(self, position: int) -> None:
        check(lib.sa_kv_cache_set_position(self.handle, position))

    def advance_position(self, n: int = 1) -> None:
        check(lib.sa_kv_cache_advance(self.handle, n))

    def reset(self) -> None:
        check(lib.sa_kv_cache_reset(self.handle))

    def append(self, layer: int, new_k: torch.Tensor, new_v: torch.Tensor, *, cos_cache=None, sin_cache=None,
               do_rotary: bool = False, rotary_interleaved: bool = False, stream=None) -> None:
        """Quantize-on-append of (B, S, H*D) K/V at the current position."""
        from .ops import _dtype_code, _stream_handle, _raise_op

        _check_tensor(new_k, self.device)
        _check_tensor(new_v, self.device)
        if new_k.shape != new_v.shape or new_k.dim() != 3:
            raise _shape("kv_cache_append: key and value must be (B, S, H*D) with equal shapes")
        rows = 0 if cos_cache is None else cos_cache.shape[0]
        rc = lib.sa_kv_append(self.handle, layer, new_k.data_ptr(), new_v.data_ptr(), _dtype_code(new_k),
                              new_k.shape[0], new_k.shape[1], _ptr_or_none(cos_cache), _ptr_or_none(sin_cache),
                              rows, int(do_rotary), int(rotary_interleaved), _stream_handle(stream, self.device))
        _raise_op(rc, "kv_cache_append")

    def view(self, layer: int) -> LayerView:
        v = _lib.KvLayerView()
        check(lib.sa_kv_cache_layer_view(self.handle, layer, ctypes.byref(v)))
        B, H, T, CB, D = v.batch, v.kv_heads, v.capacity, v.code_bytes, v.head_dim
        dev = self.device
        return LayerView(
            k_codes=_view(v.k_codes, (B, H, T, CB), "|u1", dev),
            v_codes=_view(v.v_codes, (B, H, T // 16, CB // 4, 4, 4, 4), "|u1", dev),
            k_meta=_view(v.k_meta, (B, H, T, 2), "<f4", dev),
            v_meta=_view(v.v_meta, (B, H, T, 2), "<f4", dev),
            signs=_view(v.signs, (H, D), "<f4", dev),
            wht_scale=v.wht_scale, bits=v.bits, code_bytes=CB, capacity=T,
            **({} if not v.k_qjl_bits else dict(
                k_qjl_bits=_view(v.k_qjl_bits, (B, H, T, D // 8), "|u1", dev),
                v_qjl_bits=_view(v.v_qjl_bits, (B, H, T, D // 8), "|u1", dev),
                k_qjl_mag=_view(v.k_qjl_mag, (B, H, T), "<f4", dev),
                v_qjl_mag=_view(v.v_qjl_mag, (B, H, T), "<f4", dev))),
            **({} if not v.lr_us else dict(
                lr_vt=_view(v.lr_vt, (B, H, D), "<f4", dev),
                lr_us=_view(v.lr_us, (B, H, T), "<f4", dev),
                lr_kmeta=_view(v.lr_kmeta, (B, H, T, 2), "<f4", dev),
                lr_vtr=_view(v.lr_vtr, (B, H, D), "<f4", dev))))

    def memory_bytes(self) -> tuple[int, int]:
        """(CompressedKVCache::memory_bytes of the rows written so far, summed over the batch,
        bytes held on the device) -- kv_compression.rs:928-957."""
        ref, dev = ctypes.c_uint64(), ctypes.c_uint64()
        check(lib.sa_kv_cache_memory_bytes(self.handle, ctypes.byref(ref), ctypes.byref(dev)))
        return ref.value, dev.value

    # Arrays of a layer that make up the compressed state (signs are derived from the seed).
    _STATE = ("k_codes", "v_codes", "k_meta", "v_meta", "k_qjl_bits", "v_qjl_bits", "k_qjl_mag", "v_qjl_mag",
              "lr_vt", "lr_us", "lr_kmeta", "lr_vtr")

    def state_dict(self) -> dict:
        """The compressed cache as host tensors: configuration, position and, per layer, the
        codes, metadata and optional QJL / low-rank state of the rows written so far.  The
        rotation signs are not stored; they follow from the seed (kv_compression.rs:776-779),
        so a state saved on one machine replays on another."""
        pos = self.current_position()
        torch.cuda.synchronize(self.device)
        cfg = {f: getattr(self.config, f) for f, _ in _lib.KvCacheConfig._fields_}
        layers = []
        for layer in range(self.config.num_layers):
            v = self.view(layer)
            st = {}
            for name in self._STATE:
                t = getattr(v, name)
                if t is None:
                    continue
                if name == "v_codes":  # 16-token blocks: keep whole blocks up to the position
                    t = t[:, :, :(pos + 15) // 16]
                elif name not in ("lr_vt", "lr_vtr"):
                    t = t[:, :, :pos]
                st[name] = t.cpu().clone()
            layers.append(st)
        return {"format": "smallaios_b200.kv_cache/1", "config": cfg, "position": pos, "layers": layers}

    @classmethod
    def from_state_dict(cls, state: dict, device=None) -> "GpuKvCache":
        """A cache with the saved configuration and contents, positioned where it was saved."""
        if state.get("format") != "smallaios_b200.kv_cache/1":
            raise ValueError("not a smallaios_b200 KV-cache state")
        c = state["config"]
        cache = cls(c["num_layers"], c["num_kv_heads"], c["head_dim"], c["max_seq_len"], batch=c["batch"],
                    num_heads=c["num_heads"], bits=c["bits"], seed=c["seed"], kv_head_begin=c["kv_head_begin"],
                    kv_head_count=c["kv_head_count"], qjl_residual=bool(c["qjl_residual"]),
                    lowrank_k=c["lowrank_k"] or None, device=device)
        pos = int(state["position"])
        try:
            for layer, st in enumerate(state["layers"]):
                v = cache.view(layer)
                for name, t in st.items():
                    dst = getattr(v, name)
                    if dst is None:
                        raise ValueError(f"state has {name} but the cache does not keep it")
                    if name not in ("lr_vt", "lr_vtr"):  # arrays with a token (or token-block) axis
                        dst = dst[:, :, :t.shape[2]]
                    dst.copy_(t.to(cache.device))
            torch.cuda.synchronize(cache.device)
            cache.set_position(pos)
        except Exception:
            cache.close()
            raise
        return cache

    def device_status(self, clear: bool = False) -> int:
        """Device-side status bits of the kernels that used this cache: 0, or bit 0 when a bounded
        wait inside a kernel gave up (that call's output is not valid).  Synchronises."""
        st = ctypes.c_int32()
        check(lib.sa_kv_cache_device_status(self.handle, ctypes.byref(st), int(bool(clear))))
        return st.value

    def close(self) -> None:
        if self._handle:
            with torch.cuda.device(self.device):
                lib.sa_kv_cache_destroy(self._handle.value)
            self._handle = ctypes.c_void_p()

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


def _ptr_or_none(t):
    return None if t is None else t.data_ptr()


def _shape(msg):
    from .ops import ShapeMismatch

    return ShapeMismatch(msg)


def _check_tensor(t: torch.Tensor, device) -> None:
    if not isinstance(t, torch.Tensor) or not t.is_cuda:
        raise TypeError("expected a CUDA tensor")
    if not t.is_contiguous():
        raise ValueError("expected a contiguous tensor")
