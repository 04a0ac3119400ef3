"""Pin the CPU oracle against the reference's own known-answer tests.

Each test replays one test of the SmallAIOS onnx-rt Rust suite for this path
(inputs, seeds and thresholds as written there) against the C restatement in
oracle/.  The reference pins no code bytes, scales or GQA outputs; what it does
pin (WHT vectors, the QJL sign byte 0xD5, round-trip bounds, determinism, SDPA
and RoPE manual answers, GEMM identities, GQA shapes and errors) is here.
"""
import math

import numpy as np
import pytest

import oracle


def u64_to_f32(x: int) -> np.float32:
    return np.float32(np.uint64(x))


class Xorshift64:
    """kv_compression.rs:44-68 (used by the reference tests to make inputs)."""

    def __init__(self, seed):
        self.s = seed if seed != 0 else 0x5EEDDEADBEEFCAFE

    def next(self):
        x = self.s
        x ^= (x << 13) & (2**64 - 1)
        x ^= x >> 7
        x ^= (x << 17) & (2**64 - 1)
        self.s = x
        return x


def ref_test_vector(dim, offset):
    """kv_compression.rs:1013-1015: (i + offset) * 0.1 in f32."""
    return np.array([(np.float32(i) + np.float32(offset)) * np.float32(0.1) for i in range(dim)], np.float32)


# ---- WHT (kv_compression.rs:1021-1068) ------------------------------------
def test_wht_known_vector():
    x = oracle.wht_with_signs([1, 1, 1, 1], np.ones(4, np.int8))
    assert abs(x[0] - 2.0) < 1e-6 and np.all(np.abs(x[1:]) < 1e-6)


def test_wht_known_vector_alternating():
    x = oracle.wht_with_signs([1, -1, 1, -1], np.ones(4, np.int8))
    assert abs(x[0]) < 1e-6 and abs(x[1] - 2.0) < 1e-6 and abs(x[2]) < 1e-6 and abs(x[3]) < 1e-6


def test_wht_self_inverse_roundtrip():
    signs = np.array([1, -1, 1, 1, -1, -1, 1, -1], np.int8)
    orig = np.arange(1, 9, dtype=np.float32)
    x = oracle.inverse_wht_with_signs(oracle.wht_with_signs(orig, signs), signs)
    assert np.max(np.abs(x - orig)) < 1e-4


# ---- encode/decode round trips (kv_compression.rs:1071-1123) --------------
@pytest.mark.parametrize("dim,bits,seed,step,off,bound", [
    (64, 4, 42, 0.1, -3.0, None),
    (32, 3, 123, 0.2, -2.0, None),
    (16, 8, 999, 0.5, -4.0, 0.5),
])
def test_encode_decode_roundtrip(dim, bits, seed, step, off, bound):
    signs = oracle.polar_signs(seed, dim)
    x = np.array([np.float32(i) * np.float32(step) - np.float32(-off) for i in range(dim)], np.float32)
    codes, scale, zp, mn, mx = oracle.polar_encode(x, bits, signs)
    dec = oracle.polar_decode(codes, scale, zp, dim, bits, signs)
    err = np.max(np.abs(x - dec))
    if bound is None:
        levels = (1 << bits) - 1
        slack = 0.1 if bits == 4 else 0.2
        bound = (mx - mn) / levels + slack
    assert err < bound


@pytest.mark.parametrize("dim,bits", [(17, 4), (0, 4)])
def test_reject_non_power_of_two_dim(dim, bits):
    with pytest.raises(oracle.OracleError):
        oracle.polar_signs(42, dim)


def test_reject_invalid_bits():
    with pytest.raises(oracle.OracleError):
        oracle.polar_encode(np.zeros(16, np.float32), 5, oracle.polar_signs(42, 16))


def test_deterministic_same_seed():
    s1, s2 = oracle.polar_signs(42, 64), oracle.polar_signs(42, 64)
    assert np.array_equal(s1, s2)
    x = np.array([np.float32(i) * np.float32(0.1) for i in range(64)], np.float32)
    b1, b2 = oracle.polar_encode(x, 4, s1), oracle.polar_encode(x, 4, s2)
    assert np.array_equal(b1[0], b2[0]) and b1[1] == b2[1] and b1[2] == b2[2]


def test_different_seeds_different_signs():
    assert not np.array_equal(oracle.polar_signs(42, 64), oracle.polar_signs(99, 64))


def test_constant_input_roundtrip():
    signs = oracle.polar_signs(42, 16)
    x = np.full(16, 3.14, np.float32)
    c, s, z, _, _ = oracle.polar_encode(x, 4, signs)
    assert np.max(np.abs(x - oracle.polar_decode(c, s, z, 16, 4, signs))) < 1.5


# ---- packing (kv_compression.rs:1195-1215) ---------------------------------
@pytest.mark.parametrize("values,bits", [
    (list(range(16)), 4),
    ([0, 1, 2, 3, 4, 5, 6, 7, 0, 3, 5, 7], 3),
    (list(range(255)), 8),
])
def test_pack_unpack_roundtrip(values, bits):
    packed = oracle.pack_bits(values, bits)
    assert np.array_equal(oracle.unpack_bits(packed, len(values), bits), np.array(values, np.uint32))


def test_pack_bits_lsb_first_int4():
    # Element 2i goes to the low nibble of byte i (LSB-first bit stream).
    assert list(oracle.pack_bits([1, 2, 3, 4], 4)) == [0x21, 0x43]


# ---- QJL (kv_compression.rs:1223-1234) ------------------------------------
def test_qjl_sign_captures_correct_signs():
    words, _ = oracle.qjl_encode([1.0, -2.0, 3.0, -4.0, 0.5, -0.5, 0.0, 1.0], np.zeros(8, np.float32))
    assert int(words[0]) & 0xFF == 0xD5


# ---- CompressedKVCache (kv_compression.rs:1489-1749) ----------------------
def _cache_signs(seed, layers, heads, dim):
    return oracle.cache_signs(seed, layers, heads, dim)


def test_cache_write_read_roundtrip():
    signs = _cache_signs(42, 1, 1, 16)[0, 0]
    k, v = ref_test_vector(16, 0.0), ref_test_vector(16, 5.0)
    for x in (k, v):
        c, s, z, _, _ = oracle.polar_encode(x, 4, signs)
        assert np.max(np.abs(x - oracle.polar_decode(c, s, z, 16, 4, signs))) < 1.0


def test_cache_read_slice_8bit():
    signs = _cache_signs(42, 1, 1, 16)[0, 0]
    for pos in range(5):
        k = np.array([np.float32(i + pos * 10) * np.float32(0.1) for i in range(16)], np.float32)
        c, s, z, _, _ = oracle.polar_encode(k, 8, signs)
        assert np.max(np.abs(k - oracle.polar_decode(c, s, z, 16, 8, signs))) < 1.0


def test_cache_8bit_high_accuracy():
    signs = _cache_signs(42, 1, 1, 32)[0, 0]
    k = np.array([np.float32(i) * np.float32(0.3) - np.float32(5.0) for i in range(32)], np.float32)
    v = np.array([np.float32(i) * np.float32(0.2) + np.float32(1.0) for i in range(32)], np.float32)
    for x in (k, v):
        c, s, z, _, _ = oracle.polar_encode(x, 8, signs)
        assert np.max(np.abs(x - oracle.polar_decode(c, s, z, 32, 8, signs))) < 0.5


def test_cache_default_seed_mixing_distinct_heads():
    s = oracle.cache_signs(oracle.DEFAULT_SEED, 4, 8, 64)
    flat = {s[l, h].tobytes() for l in range(4) for h in range(8)}
    assert len(flat) == 32  # every (layer, head) gets its own quantizer


def test_integration_synthetic_gqa_compressed_vs_uncompressed():
    """kv_compression.rs:1752-1830: logits relative error < 1.0 at 4 bits."""
    dim, seq = 64, 32
    signs = _cache_signs(42, 1, 1, dim)[0, 0]
    rng = Xorshift64(12345)
    umax = u64_to_f32(2**64 - 1)

    def draw():
        return np.array([(u64_to_f32(rng.next()) / umax) * np.float32(2.0) - np.float32(1.0) for _ in range(dim)],
                        np.float32)

    ks, dec = [], []
    for _ in range(seq):
        k, _v = draw(), draw()
        ks.append(k)
        c, s, z, _, _ = oracle.polar_encode(k, 4, signs)
        dec.append(oracle.polar_decode(c, s, z, dim, 4, signs))
    q = draw()
    true = np.array([np.dot(q, k) for k in ks])
    comp = np.array([np.dot(q, k) for k in dec])
    rel = np.max(np.abs(true - comp)) / (np.mean(np.abs(true)) + 1e-6)
    assert rel < 1.0


# ---- scalar helpers ---------------------------------------------------------
def test_sqrt_approx_normalizers():
    # 1/sqrt_approx(n) is exactly 0.125 at n=64 and 0x3db504f3 at n=128.
    assert oracle.wht_normalizer(64) == np.float32(0.125)
    assert int(np.float32(oracle.wht_normalizer(128)).view(np.uint32)) == 0x3DB504F3


def test_expf_approx_close_to_exp():
    for x in [-20.0, -5.0, -1.0, -0.3, 0.0, 0.3, 1.0]:
        assert abs(oracle.expf_approx(x) - math.exp(x)) <= 5e-5 * math.exp(x) + 1e-30
    assert oracle.expf_approx(-200.0) == 0.0 or oracle.expf_approx(-200.0) < 1e-37


def test_round_f32_half_away_from_zero():
    assert oracle.round_f32(2.5) == 3.0 and oracle.round_f32(-2.5) == -3.0 and oracle.round_f32(2.49) == 2.0


# ---- RoPE (ops/microsoft.rs:1318-1400) -------------------------------------
def _taylor_cos(x):
    x = np.float32(x)
    x2 = x * x
    return np.float32(1.0) - x2 / np.float32(2.0) + x2 * x2 / np.float32(24.0) - x2 * x2 * x2 / np.float32(720.0)


def _taylor_sin(x):
    x = np.float32(x)
    x2 = x * x
    return x * (np.float32(1.0) - x2 / np.float32(6.0) + x2 * x2 / np.float32(120.0) - x2 * x2 * x2 / np.float32(5040.0))


def make_rope_caches(max_seq, half):
    cos = np.zeros((max_seq, half), np.float32)
    sin = np.zeros((max_seq, half), np.float32)
    for p in range(max_seq):
        for i in range(half):
            th = np.float32(p) * (np.float32(0.1) + np.float32(i) * np.float32(0.01))
            cos[p, i], sin[p, i] = _taylor_cos(th), _taylor_sin(th)
    return cos, sin


def test_rope_position_zero_is_identity():
    c, s = make_rope_caches(4, 2)
    x = np.array([1, 2, 3, 4], np.float32).reshape(1, 1, 1, 4)
    assert np.allclose(oracle.apply_rope(x, c, s, [0]), x, atol=1e-5)


def test_rope_interleaved_vs_noninterleaved_differ():
    c, s = make_rope_caches(4, 2)
    x = np.array([1, 2, 3, 4], np.float32).reshape(1, 1, 1, 4)
    a = oracle.apply_rope(x, c, s, [1], interleaved=False)
    b = oracle.apply_rope(x, c, s, [1], interleaved=True)
    assert np.any(np.abs(a - b) > 1e-4)


def test_rope_non_interleaved_manual_calc():
    c, s = make_rope_caches(2, 2)
    v = oracle.apply_rope(np.array([1, 2, 3, 4], np.float32).reshape(1, 1, 1, 4), c, s, [1]).ravel()
    c0, s0, c1, s1 = _taylor_cos(0.1), _taylor_sin(0.1), _taylor_cos(0.11), _taylor_sin(0.11)
    exp = [c0 * 1 - s0 * 3, c1 * 2 - s1 * 4, s0 * 1 + c0 * 3, s1 * 2 + c1 * 4]
    assert np.max(np.abs(v - np.array(exp, np.float32))) < 1e-4


# ---- SDPA (ops/microsoft.rs:1421-1530) -------------------------------------
def test_sdpa_single_head_non_causal_matches_manual():
    q = np.array([1, 0], np.float32).reshape(1, 1, 1, 2)
    k = np.array([[1, 0], [0, 1]], np.float32).reshape(1, 1, 2, 2)
    v = np.array([[1, 2], [3, 4]], np.float32).reshape(1, 1, 2, 2)
    out = oracle.sdpa(q, k, v, 0, 1.0, causal=False).ravel()
    e = np.float32(oracle.expf_approx(1.0))
    s0, s1 = e / (e + 1), 1 / (e + 1)
    assert abs(out[0] - (s0 * 1 + s1 * 3)) < 1e-4 and abs(out[1] - (s0 * 2 + s1 * 4)) < 1e-4


def test_sdpa_causal_mask_exact_zero():
    q = np.ones((1, 1, 3, 1), np.float32)
    k = np.ones((1, 1, 3, 1), np.float32)
    v = np.array([2, 4, 8], np.float32).reshape(1, 1, 3, 1)
    out = oracle.sdpa(q, k, v, 0, 1.0, causal=True).ravel()
    assert abs(out[0] - 2) < 1e-4 and abs(out[1] - 3) < 1e-4 and abs(out[2] - 14 / 3) < 1e-3


def test_sdpa_gqa_grouping():
    q = np.zeros((1, 2, 1, 2), np.float32)
    k = np.array([[1, 0], [0, 1]], np.float32).reshape(1, 1, 2, 2)
    v = np.array([[2, 3], [4, 5]], np.float32).reshape(1, 1, 2, 2)
    out = oracle.sdpa(q, k, v, 0, 1.0, causal=False).reshape(2, 2)
    assert np.allclose(out, [[3, 4], [3, 4]], atol=1e-4)


def test_sdpa_rejects_bad_grouping():
    with pytest.raises(oracle.OracleError):
        oracle.sdpa(np.zeros((1, 3, 1, 2)), np.zeros((1, 2, 1, 2)), np.zeros((1, 2, 1, 2)), 0, 1.0, False)


# ---- GroupQueryAttention (ops/microsoft.rs:1600-2180) ----------------------
def _gqa(q, k, v, pk=None, pv=None, cos=None, sin=None, nh=4, kvh=2, **kw):
    return oracle.group_query_attention(q, k, v, pk, pv, cos, sin, num_heads=nh, kv_num_heads=kvh, **kw)


def test_gqa_basic_no_rope_no_cache():
    a, pk, pv = _gqa(np.zeros((1, 1, 8)), np.array([[[1, 0, 0, 1]]]), np.array([[[1, 2, 3, 4]]]), do_rotary=False)
    assert a.shape == (1, 1, 8) and pk.shape == (1, 2, 1, 2) and pv.shape == (1, 2, 1, 2)


def test_gqa_kv_cache_mutation_across_calls():
    _, pk1, pv1 = _gqa(np.zeros((1, 2, 8)), np.ones((1, 2, 4)), np.full((1, 2, 4), 2.0), do_rotary=False)
    assert pk1.shape == (1, 2, 2, 2)
    _, pk2, _ = _gqa(np.zeros((1, 1, 8)), np.full((1, 1, 4), 3.0), np.full((1, 1, 4), 4.0), pk1, pv1,
                     do_rotary=False)
    assert pk2.shape == (1, 2, 3, 2)


def test_gqa_do_rotary_requires_caches():
    with pytest.raises(oracle.OracleError):
        _gqa(np.zeros((1, 1, 8)), np.zeros((1, 1, 4)), np.zeros((1, 1, 4)), do_rotary=True)


def test_gqa_do_rotary_default_is_on():
    # executor.rs:2349: a node without the attribute applies RoPE and needs caches.
    with pytest.raises(oracle.OracleError):
        oracle.group_query_attention(np.zeros((1, 1, 8)), np.zeros((1, 1, 4)), np.zeros((1, 1, 4)),
                                     num_heads=4, kv_num_heads=2)


def test_gqa_rejects_local_window():
    with pytest.raises(oracle.OracleError) as e:
        _gqa(np.zeros((1, 1, 8)), np.zeros((1, 1, 4)), np.zeros((1, 1, 4)), do_rotary=False, local_window_size=512)
    assert e.value.code == oracle.ORC_INVALID_ATTRIBUTE


@pytest.mark.parametrize("nh,kvh", [(3, 2), (0, 2), (4, 0)])
def test_gqa_rejects_bad_heads(nh, kvh):
    with pytest.raises(oracle.OracleError):
        _gqa(np.zeros((1, 1, 8)), np.zeros((1, 1, 4)), np.zeros((1, 1, 4)), nh=nh, kvh=kvh, do_rotary=False)


def test_integration_gqa_two_step_generation():
    o1, pk, pv = _gqa(np.full((1, 3, 8), 0.1), np.full((1, 3, 4), 0.2), np.full((1, 3, 4), 0.3), do_rotary=False)
    assert o1.shape == (1, 3, 8) and pk.shape[2] == 3
    o2, pk2, _ = _gqa(np.full((1, 1, 8), 0.4), np.full((1, 1, 4), 0.5), np.full((1, 1, 4), 0.6), pk, pv,
                      do_rotary=False)
    assert o2.shape == (1, 1, 8) and pk2.shape[2] == 4


def test_gqa_with_rope_applies_rotation():
    q = np.array([i * 0.1 + 0.05 for i in range(16)], np.float32).reshape(1, 1, 16)
    k_raw = np.array([i * 0.2 + 0.1 for i in range(8)], np.float32)
    v = np.array([i * 0.3 for i in range(8)], np.float32).reshape(1, 1, 8)
    c, s = make_rope_caches(8, 2)
    _, pk, _ = _gqa(q, k_raw.reshape(1, 1, 8), v, np.zeros((1, 2, 1, 4)), np.zeros((1, 2, 1, 4)), c, s,
                    do_rotary=True)
    assert np.any(np.abs(pk.ravel()[4:8] - k_raw[:4]) > 1e-4)


def test_gqa_present_key_has_correct_shape_with_cache():
    _, pk, pv = _gqa(np.zeros((1, 2, 8)), np.zeros((1, 2, 4)), np.zeros((1, 2, 4)),
                     np.zeros((1, 2, 3, 2)), np.zeros((1, 2, 3, 2)), do_rotary=False)
    assert pk.shape == (1, 2, 5, 2) and pv.shape == (1, 2, 5, 2)


# ---- gemm_f32 (gemm.rs tests) ------------------------------------------------
def test_gemm_identity_and_small():
    assert np.array_equal(oracle.gemm_f32(np.array([[1, 2], [3, 4]]), np.eye(2)), [[1, 2], [3, 4]])
    a = np.array([[1, 2, 3], [4, 5, 6]], np.float32)
    b = np.array([[7, 8], [9, 10], [11, 12]], np.float32)
    assert np.array_equal(oracle.gemm_f32(a, b), [[58, 64], [139, 154]])


def test_gemm_larger_than_tile_and_ones():
    assert np.allclose(oracle.gemm_f32(np.eye(16), np.eye(16)), np.eye(16), atol=1e-6)
    assert np.allclose(oracle.gemm_f32(np.ones((4, 3)), np.ones((3, 4))), 3.0, atol=1e-6)
    assert oracle.gemm_f32(np.array([[3.0]]), np.array([[5.0]]))[0, 0] == 15.0
    rng = np.random.default_rng(0)
    a, b = rng.standard_normal((70, 130)).astype(np.float32), rng.standard_normal((130, 75)).astype(np.float32)
    assert np.allclose(oracle.gemm_f32(a, b), a.astype(np.float64) @ b, atol=1e-3)


def test_matmul_nbits_matches_float_dequant():
    rng = np.random.default_rng(1)
    n, k, m = 24, 96, 3
    codes = rng.integers(0, 256, size=(n, k // 32, 16), dtype=np.uint8)
    scales = rng.uniform(0.005, 0.02, size=(n, k // 32)).astype(np.float16).astype(np.float32)
    a = rng.standard_normal((m, k)).astype(np.float32)
    y = oracle.matmul_nbits(a, codes, scales, n=n, k=k)
    lo, hi = codes & 15, codes >> 4
    q = np.stack([lo, hi], -1).reshape(n, k).astype(np.float64)
    w = (q - 8.0) * np.repeat(scales, 32, axis=1)
    assert np.allclose(y, a.astype(np.float64) @ w.T, atol=1e-4)


def test_rms_norm_known_answers():
    """generative.rs rms_norm_constant_input / rms_norm_preserves_zero_mean_direction."""
    y, _ = oracle.rms_norm(np.ones((1, 4)), np.full(4, 0.5), 1e-6)
    assert np.all(np.abs(y - 0.5) < 1e-4)
    y, _ = oracle.rms_norm(np.array([[1.0, -1.0, 1.0, -1.0]]), np.ones(4), 1e-6)
    assert np.all(np.abs(y - np.array([1.0, -1.0, 1.0, -1.0])) < 1e-3)
    # SkipSimplifiedLayerNormalization: pre = x + skip + bias is returned
    x, s, b = np.array([[1.0, 2.0]]), np.array([[3.0, -1.0]]), np.array([0.5, 0.5])
    y, pre = oracle.rms_norm(x, np.ones(2), 0.0, skip=s, bias=b)
    assert np.allclose(pre, [[4.5, 1.5]])
    assert np.allclose(y, pre / np.sqrt((pre ** 2).mean()), atol=1e-6)


def test_silu_known_answers():
    """activations.rs test_swish_at_zero / test_swish_known_values / test_swish_negative."""
    y = oracle.silu_mul(np.array([0.0, 1.0, 2.0, -1.0]), np.ones(4))
    assert abs(y[0]) < 1e-5
    assert abs(y[1] - 0.7310) < 1e-2 and abs(y[2] - 1.7616) < 1e-2 and abs(y[3] + 0.2689) < 1e-2
    assert np.allclose(oracle.silu_mul(np.array([1.0]), np.array([3.0])), 3 * 0.7310586, atol=1e-4)


# ---- LowRankKeyDecomposer (kv_compression.rs:1312-1486, 1591-1612, 1883-1953) ----

def _l2(a, b):
    return float(np.sqrt(((np.asarray(a, np.float32) - np.asarray(b, np.float32)) ** 2).sum()))


def test_lowrank_reconstruction_error_decreases_with_rank():
    m = np.array([[i + j for j in range(8)] for i in range(16)], np.float32)
    e = [_l2(m, oracle.LowRankK(m, 16, 8, r).reconstruct()) for r in (1, 2, 4)]
    assert e[1] <= e[0] + 1e-3 and e[2] <= e[1] + 1e-3


def test_lowrank_rank1_matrix():
    u = np.arange(1, 9, dtype=np.float32)
    v = np.arange(1, 5, dtype=np.float32) * 0.5
    m = np.outer(u, v).astype(np.float32)
    rec = oracle.LowRankK(m, 8, 4, 1).reconstruct()
    assert _l2(m, rec) / (np.sqrt((m ** 2).sum()) + 1e-10) < 0.6


def test_lowrank_incremental_update_and_zero_row():
    lr = oracle.LowRankK(np.arange(32, dtype=np.float32) * 0.1, 4, 8, 4)
    assert lr.rows == 4
    lr.update(np.arange(8, dtype=np.float32) * 0.5)
    assert lr.rows == 5 and lr.u_s[:5 * lr.rank].size == 5 * lr.rank
    lr = oracle.LowRankK(np.arange(16, dtype=np.float32), 2, 8, 2)
    lr.update(np.zeros(8, np.float32))
    assert lr.rows == 3


def test_lowrank_empty_full_rank_single_row():
    lr = oracle.LowRankK(np.zeros(0, np.float32), 0, 8, 4)
    assert lr.rows == 0 and lr.reconstruct().size == 0
    m = np.diag(np.arange(1, 5, dtype=np.float32))
    rec = oracle.LowRankK(m, 4, 4, 4).reconstruct()
    assert _l2(m, rec) / (np.sqrt((m ** 2).sum()) + 1e-10) < 0.01
    row = np.arange(1, 9, dtype=np.float32)
    assert _l2(row, oracle.LowRankK(row, 1, 8, 4).reconstruct()[0]) < 1.0


def test_lowrank_incremental_preserves_cols():
    lr = oracle.LowRankK(np.arange(16, dtype=np.float32), 1, 16, 4)
    for r in range(10):
        lr.update((np.arange(16) + r).astype(np.float32) * 0.1)
    assert lr.rows == 11 and lr.cols == 16


def test_lowrank_cache_replay_rank_is_one_and_bounded():
    """write_kv decomposes the first K row alone (rows = 1), so the cache's rank is
    min(rank, 1, D) = 1 from then on (:842-853, :483, :566); integration_lowrank_improves_k_accuracy."""
    dim, seq = 16, 16
    b1 = np.arange(dim, dtype=np.float32) * 0.1
    b2 = (dim - np.arange(dim)).astype(np.float32) * 0.05
    k = np.stack([np.float32(p * 0.3) * b1 + np.float32((seq - p) * 0.2) * b2 for p in range(seq)]).astype(np.float32)
    u_s, vt, rank = oracle.lowrank_replay(k, 4)
    assert rank == 1 and u_s.shape == (seq, 1) and vt.shape == (1, dim)
    rec = np.zeros((seq, dim), np.float32)
    oracle.lib().orc_lowrank_reconstruct(oracle._ptr(u_s), oracle._ptr(vt), seq, dim, 1, oracle._ptr(rec))
    assert _l2(k, rec) / (np.sqrt((k ** 2).sum()) + 1e-6) < 2.0
    # replay == decompose + update by hand, across a re-orthogonalisation (every 512 writes)
    kk = np.random.default_rng(1).standard_normal((1030, 32)).astype(np.float32)
    u_s, vt, _ = oracle.lowrank_replay(kk, 8)
    lr = oracle.LowRankK(kk[0], 1, 32, 8, capacity=1030)
    for i in range(1, 1030):
        lr.update(kk[i])
    assert np.array_equal(u_s.reshape(-1), lr.u_s[:1030]) and np.array_equal(vt.reshape(-1), lr.vt[:32])
