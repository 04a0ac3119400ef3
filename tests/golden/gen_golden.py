"""Write the seeded golden fixtures of the compressed decode path (tests/golden/*.npz).

The reference's tests pin no code bytes, scales or GQA outputs
(onnx-rt/src/kv_compression.rs:969-2071 check only round-trip bounds), so these
fixtures freeze today's bit-exact contract as the C restatement computes it:

* inputs: K/V for T tokens and the last token's Q, seeded normals rounded to
  bf16 (stored as their bf16 bits; the path widens them to f32);
* PolarQuantizer::encode of RoPE(K) and of V for every token (codes in
  pack_bits order, {scale, zero_point} as f32 bits), with the seeded signs of
  CompressedKVCache::new (kv_compression.rs:776-779);
* the composite GQA output of the last token: read_k/read_v of all T tokens,
  causal SDPA (ops/microsoft.rs:380-438) with RoPE on Q at position T-1.

Configs follow BASELINE: c1 (B=1, 8/2 heads, D=64, T=512, int8, theta 1e4),
c3 small (the Llama-3-8B layer's heads, D=128, int4, theta 5e5, B=1, T=40) and
c5 small (the Llama-3-70B layer's 64/8 heads, B=1, T=40).

Run from the repository root:  python tests/golden/gen_golden.py
"""
from __future__ import annotations

import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, ROOT)

import oracle  # noqa: E402

CONFIGS = {
    "c1": dict(b=1, hq=8, hkv=2, d=64, t=512, bits=8, theta=10000.0, std=0.45, seed=11),
    "c3_small": dict(b=1, hq=32, hkv=8, d=128, t=40, bits=4, theta=500000.0, std=1.28, seed=13),
    "c5_small": dict(b=1, hq=64, hkv=8, d=128, t=40, bits=4, theta=500000.0, std=1.28, seed=15),
}


def bf16_bits(x: np.ndarray) -> np.ndarray:
    """Round f32 to bf16 (nearest even) and return the 16-bit patterns."""
    u = np.ascontiguousarray(x, np.float32).view(np.uint32).astype(np.uint64)
    r = (u + 0x7FFF + ((u >> 16) & 1)) >> 16
    return r.astype(np.uint16)


def bf16_to_f32(bits: np.ndarray) -> np.ndarray:
    return (bits.astype(np.uint32) << 16).view(np.float32)


def expected(cfg: dict, k: np.ndarray, v: np.ndarray, q: np.ndarray) -> dict:
    """Codes, metadata and the last token's GQA output for inputs (B, T, H, D) / (B, 1, Hq, D)."""
    b, t, hkv, d = k.shape
    bits = cfg["bits"]
    signs = oracle.cache_signs(oracle.DEFAULT_SEED, 1, hkv, d)[0]
    cos, sin = oracle.rope_tables(t + 8, d // 2, cfg["theta"])
    kr = oracle.apply_rope(np.ascontiguousarray(k.transpose(0, 2, 1, 3)), cos, sin, np.arange(t))
    vv = np.ascontiguousarray(v.transpose(0, 2, 1, 3))
    cb = oracle.code_bytes(d, bits)
    kc = np.zeros((b, hkv, t, cb), np.uint8)
    vc = np.zeros_like(kc)
    km = np.zeros((b, hkv, t, 2), np.float32)
    vm = np.zeros_like(km)
    for h in range(hkv):
        kc[:, h], km[:, h] = oracle.polar_encode_many(kr[:, h], bits, signs[h], nthreads=1)
        vc[:, h], vm[:, h] = oracle.polar_encode_many(vv[:, h], bits, signs[h], nthreads=1)
    qr = oracle.apply_rope(np.ascontiguousarray(q.transpose(0, 2, 1, 3)), cos, sin, [t - 1])
    scale = np.float32(1.0) / np.float32(oracle.sqrt_f32(float(d)))
    out = oracle.compressed_gqa(qr, kc, km, vc, vm, signs, bits, scale, nthreads=1)
    return {"k_codes": kc, "k_meta_bits": km.view(np.uint32), "v_codes": vc, "v_meta_bits": vm.view(np.uint32),
            "signs": signs, "out": out}


def inputs(cfg: dict):
    r = np.random.default_rng(cfg["seed"])
    b, t, hq, hkv, d, std = cfg["b"], cfg["t"], cfg["hq"], cfg["hkv"], cfg["d"], cfg["std"]
    k = bf16_bits(r.standard_normal((b, t, hkv, d)) * std)
    v = bf16_bits(r.standard_normal((b, t, hkv, d)) * std)
    q = bf16_bits(r.standard_normal((b, 1, hq, d)) * std)
    return k, v, q


def main() -> None:
    oracle.build()
    for name, cfg in CONFIGS.items():
        kb, vb, qb = inputs(cfg)
        exp = expected(cfg, bf16_to_f32(kb), bf16_to_f32(vb), bf16_to_f32(qb))
        params = np.array([cfg[x] for x in ("b", "hq", "hkv", "d", "t", "bits")], np.int64)
        np.savez_compressed(os.path.join(HERE, f"{name}.npz"), params=params, theta=np.float64(cfg["theta"]),
                            k_bf16=kb, v_bf16=vb, q_bf16=qb, **exp)
        print(name, {k_: v_.shape for k_, v_ in exp.items()})


if __name__ == "__main__":
    main()
