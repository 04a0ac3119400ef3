"""Shared test helpers: seeded synthetic inputs and oracle compositions.

The oracle (oracle/) is only used here as the checker.
"""
from __future__ import annotations

import os

import numpy as np

import oracle


def rng(seed: int) -> np.random.Generator:
    return np.random.default_rng(seed)


def rope_tables(rows: int, head_dim: int, theta: float = 10000.0):
    return oracle.rope_tables(rows, head_dim // 2, theta)


def oracle_append(k_bshd: np.ndarray, v_bshd: np.ndarray, signs_hd: np.ndarray, bits: int, pos0: int,
                  cos=None, sin=None, do_rotary=False, interleaved=False):
    """Reference codes for appending K/V (B, S, H, D) at positions pos0..pos0+S-1.

    RoPE via apply_rope_in_place then PolarQuantizer::encode per vector.
    Returns k_codes, k_meta, v_codes, v_meta shaped (B, H, S, ...).
    """
    b, s, h, d = k_bshd.shape
    k = np.ascontiguousarray(np.transpose(k_bshd, (0, 2, 1, 3)), np.float32)  # (B, H, S, D)
    v = np.ascontiguousarray(np.transpose(v_bshd, (0, 2, 1, 3)), np.float32)
    if do_rotary:
        k = oracle.apply_rope(k, cos, sin, np.arange(pos0, pos0 + s), interleaved=interleaved)
    cb = oracle.code_bytes(d, bits)
    kc = np.zeros((b, h, s, cb), np.uint8)
    vc = np.zeros_like(kc)
    km = np.zeros((b, h, s, 2), np.float32)
    vm = np.zeros_like(km)
    for hi in range(h):
        c, m = oracle.polar_encode_many(k[:, hi], bits, signs_hd[hi])
        kc[:, hi], km[:, hi] = c, m
        c, m = oracle.polar_encode_many(v[:, hi], bits, signs_hd[hi])
        vc[:, hi], vm[:, hi] = c, m
    return kc, km, vc, vm


def oracle_qjl(k_bshd: np.ndarray, v_bshd: np.ndarray, signs_hd: np.ndarray, bits: int, pos0: int,
               cos=None, sin=None, do_rotary=False, interleaved=False):
    """Reference QJL residuals of an append (CompressedKVCache::write_kv, kv_compression.rs:826-840):
    QJLResidualEncoder::encode(x, PolarQuantizer::decode(encode(x))) per vector, x = RoPE(k) or v.

    Returns k_bits, k_mag, v_bits, v_mag shaped (B, H, S, D/8) and (B, H, S); the bit bytes are
    the little-endian bytes of the reference's u64 sign words.
    """
    b, s, h, d = k_bshd.shape
    kc, km, vc, vm = oracle_append(k_bshd, v_bshd, signs_hd, bits, pos0, cos, sin, do_rotary, interleaved)
    k = np.ascontiguousarray(np.transpose(k_bshd, (0, 2, 1, 3)), np.float32)
    v = np.ascontiguousarray(np.transpose(v_bshd, (0, 2, 1, 3)), np.float32)
    if do_rotary:
        k = oracle.apply_rope(k, cos, sin, np.arange(pos0, pos0 + s), interleaved=interleaved)
    out = []
    for x, codes, meta in ((k, kc, km), (v, vc, vm)):
        qbits = np.zeros((b, h, s, d // 8), np.uint8)
        qmag = np.zeros((b, h, s), np.float32)
        for bi in range(b):
            for hi in range(h):
                for si in range(s):
                    approx = oracle.polar_decode(codes[bi, hi, si], meta[bi, hi, si, 0], meta[bi, hi, si, 1], d,
                                                 bits, signs_hd[hi])
                    words, c = oracle.qjl_encode(x[bi, hi, si], approx)
                    qbits[bi, hi, si] = words.view(np.uint8)[:d // 8]
                    qmag[bi, hi, si] = c
        out += [qbits, qmag]
    return tuple(out)


def oracle_lowrank_state(k_bthd: np.ndarray, rank_cfg: int, cos=None, sin=None, do_rotary=False, interleaved=False):
    """Low-rank K state that write_kv builds over rows 0..T-1 (kv_compression.rs:842-853).

    k_bthd: (B, T, H, D) keys as appended (RoPE applied here when do_rotary).
    Returns us (B, H, T) and vt (B, H, D) -- the cache's rank is 1.
    """
    b, t, h, d = k_bthd.shape
    k = np.ascontiguousarray(np.transpose(k_bthd, (0, 2, 1, 3)), np.float32)
    if do_rotary:
        k = oracle.apply_rope(k, cos, sin, np.arange(t), interleaved=interleaved)
    us = np.zeros((b, h, t), np.float32)
    vt = np.zeros((b, h, d), np.float32)
    for bi in range(b):
        for hi in range(h):
            u_s, v_t, rank = oracle.lowrank_replay(k[bi, hi], rank_cfg)
            assert rank == 1
            us[bi, hi], vt[bi, hi] = u_s[:, 0], v_t[0]
    return us, vt


def oracle_lowrank_attend(q_bshd, us, vt, vc, vm, signs_hd, bits, pos0, scale=None, cos=None, sin=None,
                          do_rotary=False, interleaved=False):
    """Composite oracle with low-rank K: read_k returns 0 + U*S[t] * V^T (:870-882, :502-526), read_v
    decodes the codes, then causal SDPA.  q_bshd (B, S, Hq, D); us (B, H, T); vt (B, H, D); codes and
    meta (B, H, T, ...).  Returns (B, S, Hq*D)."""
    b, s, hq, d = q_bshd.shape
    h, t = us.shape[1], us.shape[2]
    q = np.ascontiguousarray(np.transpose(q_bshd, (0, 2, 1, 3)), np.float32)
    if do_rotary:
        q = oracle.apply_rope(q, cos, sin, np.arange(pos0, pos0 + s), interleaved=interleaved)
    k = (us[..., None] * vt[:, :, None, :]).astype(np.float32) + np.float32(0.0)
    v = np.zeros((b, h, t, d), np.float32)
    for bi in range(b):
        for hi in range(h):
            for ti in range(t):
                v[bi, hi, ti] = oracle.polar_decode(vc[bi, hi, ti], vm[bi, hi, ti, 0], vm[bi, hi, ti, 1], d, bits,
                                                    signs_hd[hi])
    if scale is None:
        scale = np.float32(1.0) / np.float32(oracle.sqrt_f32(float(d)))
    out = oracle.sdpa(q, k, v, past_sk=pos0, scale=scale, causal=True)  # (B, Hq, S, D)
    return np.ascontiguousarray(np.transpose(out, (0, 2, 1, 3))).reshape(b, s, hq * d)


def oracle_attend(q_bshd: np.ndarray, kc, km, vc, vm, signs_hd, bits, pos0, scale=None, cos=None, sin=None,
                  do_rotary=False, interleaved=False):
    """Composite oracle: RoPE q at positions pos0.., read_k/read_v, causal SDPA.

    q_bshd: (B, S, Hq, D); codes/meta (B, Hkv, T, ...) with T = pos0 + S.
    Returns (B, S, Hq*D).
    """
    b, s, hq, d = q_bshd.shape
    q = np.ascontiguousarray(np.transpose(q_bshd, (0, 2, 1, 3)), np.float32)
    if do_rotary:
        q = oracle.apply_rope(q, cos, sin, np.arange(pos0, pos0 + s), interleaved=interleaved)
    if scale is None:
        scale = np.float32(1.0) / np.float32(oracle.sqrt_f32(float(d)))
    return oracle.compressed_gqa(q, kc, km, vc, vm, signs_hd, bits, scale, nthreads=os.cpu_count() or 1)


def interleave_v(vc_tokens: np.ndarray) -> np.ndarray:
    """(B, H, T, CB) per-token codes -> the library's V layout, flattened per (B, H).

    16-token blocks; in a block, byte 4*c + jj of token 4*g + tt sits at
    ((c*4 + g)*4 + jj)*4 + tt (16-byte chunks of the four token groups interleave).
    """
    b, h, t, cb = vc_tokens.shape
    x = vc_tokens.reshape(b, h, t // 16, 4, 4, cb // 4, 4)  # blk, g, tt, c, jj
    return np.ascontiguousarray(x.transpose(0, 1, 2, 5, 3, 6, 4)).reshape(b, h, t * cb)
