"""Quantize-on-append on the GPU is bit-exact with PolarQuantizer::encode.

Codes (in pack_bits order, K and de-interleaved V), scales and zero points are
compared bit for bit against the C oracle on the same f32 inputs (inputs are
first rounded to the tested dtype so both sides see identical values).
"""
import numpy as np
import pytest
import torch

import oracle
from tests.helpers import oracle_append, rng, rope_tables

pytestmark = pytest.mark.gpu

DTYPES = {"f32": torch.float32, "bf16": torch.bfloat16, "f16": torch.float16}


def _make(shape, seed, dtype, scale=1.3):
    x = (rng(seed).standard_normal(shape) * scale).astype(np.float32)
    t = torch.from_numpy(x).to(DTYPES[dtype])
    return t, t.float().numpy()


def _run_append_case(dev, *, b, s, h, d, bits, dtype, rotary, interleaved, pos0=0, seed=0, kx=None, vx=None):
    import smallaios_b200 as sa

    max_seq = pos0 + s + 5
    cache = sa.GpuKvCache(2, h, d, max_seq, batch=b, num_heads=h * 2, bits=bits, device=dev)
    cos, sin = rope_tables(max_seq, d, 10000.0)
    if kx is None:
        kt, kn = _make((b, s, h, d), seed, dtype)
        vt, vn = _make((b, s, h, d), seed + 1, dtype)
    else:
        kt, kn = torch.from_numpy(kx), kx
        vt, vn = torch.from_numpy(vx), vx
    cache.set_position(pos0)
    layer = 1
    cache.append(layer, kt.reshape(b, s, h * d).to(dev), vt.reshape(b, s, h * d).to(dev),
                 cos_cache=torch.from_numpy(cos).to(dev), sin_cache=torch.from_numpy(sin).to(dev),
                 do_rotary=rotary, rotary_interleaved=interleaved)
    torch.cuda.synchronize()
    view = cache.view(layer)
    signs = view.signs.cpu().numpy().astype(np.int8)
    assert np.array_equal(signs, oracle.cache_signs(oracle.DEFAULT_SEED, 2, h, d)[layer])
    kc, km, vc, vm = oracle_append(kn, vn, signs, bits, pos0, cos, sin, rotary, interleaved)
    sl = slice(pos0, pos0 + s)
    g_kc = view.k_codes[:, :, sl].cpu().numpy()
    g_vc = view.v_codes_tokens()[:, :, sl].cpu().numpy()
    g_km = view.k_meta[:, :, sl].cpu().numpy()
    g_vm = view.v_meta[:, :, sl].cpu().numpy()
    # positions outside the append (the fresh cache's zeros) are left alone, in the word-interleaved
    # V layout too
    for codes in (view.k_codes.cpu().numpy(), view.v_codes_tokens().cpu().numpy()):
        assert not codes[:, :, :pos0].any() and not codes[:, :, pos0 + s:].any()
    cache.close()
    return (g_kc, g_km, g_vc, g_vm), (kc, km, vc, vm)


def _assert_bit_exact(got, want):
    names = ["k_codes", "k_meta", "v_codes", "v_meta"]
    for n, g, w in zip(names, got, want):
        if g.dtype == np.float32:
            g, w = g.view(np.uint32), w.view(np.uint32)
        mism = np.argwhere(g != w)
        assert mism.size == 0, f"{n}: {len(mism)} mismatches, first at {mism[:3].tolist()}"


@pytest.mark.parametrize("bits", [3, 4, 8])
@pytest.mark.parametrize("d", [16, 32, 64, 128])
def test_append_bit_exact_bits_dims(cuda_device, bits, d):
    if d * bits // 8 % 4:
        # a V row must pack into whole 4-byte words (D=16 at 3 bits is 6 bytes)
        import smallaios_b200 as sa
        from smallaios_b200._lib import SA_ERR_UNSUPPORTED, SaError

        with pytest.raises(SaError) as e:
            sa.GpuKvCache(1, 2, d, 8, bits=bits, device=cuda_device)
        assert e.value.status == SA_ERR_UNSUPPORTED
        return
    got, want = _run_append_case(cuda_device, b=2, s=5, h=3, d=d, bits=bits, dtype="f32", rotary=True,
                                 interleaved=False, pos0=3, seed=bits * 100 + d)
    _assert_bit_exact(got, want)


@pytest.mark.parametrize("dtype", ["bf16", "f16"])
@pytest.mark.parametrize("interleaved", [False, True])
def test_append_bit_exact_dtypes_rope(cuda_device, dtype, interleaved):
    got, want = _run_append_case(cuda_device, b=3, s=4, h=2, d=128, bits=4, dtype=dtype, rotary=True,
                                 interleaved=interleaved, pos0=17, seed=7)
    _assert_bit_exact(got, want)


def test_append_no_rotary_d256(cuda_device):
    got, want = _run_append_case(cuda_device, b=1, s=9, h=2, d=256, bits=4, dtype="f32", rotary=False,
                                 interleaved=False, pos0=0, seed=11)
    _assert_bit_exact(got, want)


def test_append_edge_vectors(cuda_device):
    """Zero, constant, signed-zero and large-magnitude vectors (first-occurrence min/max)."""
    d, h, b, s = 64, 2, 1, 8
    k = np.zeros((b, s, h, d), np.float32)
    v = np.zeros((b, s, h, d), np.float32)
    k[0, 1] = 3.14
    k[0, 2] = -0.0
    k[0, 3, :, ::2] = -0.0
    k[0, 4] = 1e30
    k[0, 5] = np.linspace(-1e-30, 1e-30, d)
    k[0, 6, 0, 0] = 1.0
    v[0, 0] = -2.5
    v[0, 7] = np.arange(d) * 1e5
    got, want = _run_append_case(cuda_device, b=b, s=s, h=h, d=d, bits=4, dtype="f32", rotary=False,
                                 interleaved=False, kx=k, vx=v)
    _assert_bit_exact(got, want)


def test_append_many_tokens_c3_shape(cuda_device):
    """Llama-3-8B KV shape (8 heads, D=128, int4) over a 1000-token prefill."""
    got, want = _run_append_case(cuda_device, b=2, s=1000, h=8, d=128, bits=4, dtype="bf16", rotary=True,
                                 interleaved=False, pos0=24, seed=5)
    _assert_bit_exact(got, want)


def test_append_capacity_and_rope_errors(cuda_device):
    import smallaios_b200 as sa

    cache = sa.GpuKvCache(1, 2, 64, 8, batch=1, num_heads=4, bits=4, device=cuda_device)
    k = torch.zeros(1, 9, 128, device=cuda_device)
    with pytest.raises(sa.CapacityError):
        cache.append(0, k, k)
    cos, sin = (torch.from_numpy(t).to(cuda_device) for t in rope_tables(4, 64))
    k4 = torch.zeros(1, 6, 128, device=cuda_device)
    with pytest.raises(sa.ShapeMismatch):  # positions 0..5 beyond 4 rope rows
        cache.append(0, k4, k4, cos_cache=cos, sin_cache=sin, do_rotary=True)
    with pytest.raises(sa.ShapeMismatch):  # do_rotary without tables
        cache.append(0, k4, k4, do_rotary=True)
    cache.close()


@pytest.mark.parametrize("bits,d", [(4, 64), (8, 256), (4, 128)])
@pytest.mark.parametrize("mag", [2.0 ** -96, 2.0 ** -88, 2.0 ** 98, 2.0 ** 102])
def test_append_scale_extremes(cuda_device, bits, d, mag):
    """Vectors whose code scale sits on either side of the range where the encoder divides by a
    reciprocal with Markstein's correction (2^-90 .. 2^100; outside it, by IEEE division): the codes
    must be the reference's either way.  Positions 2..8 give partial and full position quads."""
    r = np.random.default_rng(int(np.log2(mag)) + 200 + bits + d)
    b, s, h = 2, 7, 2
    k = (r.standard_normal((b, s, h, d)) * mag).astype(np.float32)
    v = (r.standard_normal((b, s, h, d)) * mag).astype(np.float32)
    v[0, 3] = np.float32(mag)  # a constant vector: range 0 after the first element
    got, want = _run_append_case(cuda_device, b=b, s=s, h=h, d=d, bits=bits, dtype="f32", rotary=False,
                                 interleaved=False, pos0=2, kx=k, vx=v)
    _assert_bit_exact(got, want)
