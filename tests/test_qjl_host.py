"""QJLResidualEncoder::correction (kv_compression.rs:401-417) on the host, against the C oracle
and the reference's own test cases (:1237-1310)."""
import numpy as np

import oracle
from tests.helpers import rng


def _bytes(words, dim):
    return np.ascontiguousarray(words, dtype=np.uint64).view(np.uint8)[:dim // 8]


def test_correction_matches_oracle_bit_for_bit():
    from smallaios_b200 import qjl_correction

    r = rng(3)
    for dim in (8, 64, 128, 256):
        for _ in range(20):
            oa, aa = r.standard_normal(dim).astype(np.float32), r.standard_normal(dim).astype(np.float32)
            ob, ab = r.standard_normal(dim).astype(np.float32), r.standard_normal(dim).astype(np.float32)
            wa, ca = oracle.qjl_encode(oa, aa)
            wb, cb = oracle.qjl_encode(ob, ab)
            want = oracle.qjl_correction(wa, ca, wb, cb, dim)
            got = qjl_correction(_bytes(wa, dim), np.float32(ca), _bytes(wb, dim), np.float32(cb), dim)
            assert np.float32(got).view(np.uint32) == want.view(np.uint32), (dim, got, want)


def test_correction_batched_shapes():
    from smallaios_b200 import qjl_correction

    r = rng(4)
    bits = r.integers(0, 256, size=(3, 5, 16), dtype=np.uint8)
    mags = r.uniform(0, 1, size=(3, 5)).astype(np.float32)
    got = qjl_correction(bits, mags, bits[:, :1], mags[:, :1], 128)
    assert got.shape == (3, 5) and got.dtype == np.float32
    # identical residuals: <sign, sign> = dim, correction = C * C (qjl_correction_nonneg_identical)
    assert np.array_equal(got[:, 0], mags[:, 0] * mags[:, 0])


def test_reference_cases():
    from smallaios_b200 import qjl_correction

    words, c = oracle.qjl_encode([1.0, 2.0, 3.0, 4.0, 5.0, 6.0, 7.0, 8.0], np.full(8, 0.5, np.float32))
    b = _bytes(words, 8)
    assert qjl_correction(b, c, b, c, 8) >= 0.0
    assert qjl_correction(b, c, ~b, c, 8) == -c * c  # every sign differs: <s, -s> = -dim
    assert qjl_correction(np.zeros(0, np.uint8), 0.0, np.zeros(0, np.uint8), 0.0, 0) == 0.0  # qjl_empty_vectors
    words, c = oracle.qjl_encode([1.0, 2.0, 3.0, 4.0], [1.0, 2.0, 3.0, 4.0])
    assert c == 0.0  # qjl_zero_residual
