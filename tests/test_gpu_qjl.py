"""QJL residuals stored on append (KVCacheConfig::kv_qjl_residual).

With the option on, every append path -- the bulk append kernel, the
attention call's own append (decode prep kernels for groups up to 4 and for
8) and the fused QKV projection's epilogue -- also stores, per vector, the
residual sign bits and c_magnitude of QJLResidualEncoder::encode
(kv_compression.rs:365-395) against PolarQuantizer::decode of the vector's own
codes, as CompressedKVCache::write_kv does (:826-840).  Compared bit for bit
against the C oracle.  The option changes nothing else: codes and attention
outputs equal those of a cache without it, bit for bit.
"""
import numpy as np
import pytest
import torch

from tests.helpers import oracle_append, oracle_qjl, rng, rope_tables

pytestmark = pytest.mark.gpu


def _qjl_of(view, sl):
    return (view.k_qjl_bits[:, :, sl].cpu().numpy(), view.k_qjl_mag[:, :, sl].cpu().numpy(),
            view.v_qjl_bits[:, :, sl].cpu().numpy(), view.v_qjl_mag[:, :, sl].cpu().numpy())


def _assert_equal_bits(got, want, names):
    for n, g, w in zip(names, got, want):
        if g.dtype == np.float32:
            g, w = g.view(np.uint32), w.view(np.uint32)
        mism = np.argwhere(g != w)
        assert mism.size == 0, f"{n}: {len(mism)} mismatches, first at {mism[:3].tolist()}"


QJL_NAMES = ("k_qjl_bits", "k_qjl_mag", "v_qjl_bits", "v_qjl_mag")


@pytest.mark.parametrize("bits,d", [(3, 64), (3, 128), (4, 16), (4, 128), (8, 32), (8, 256)])
def test_bulk_append_stores_residuals(cuda_device, bits, d):
    import smallaios_b200 as sa

    b, s, h, pos0 = 2, 6, 3, 4
    r = rng(bits * 1000 + d)
    k = (r.standard_normal((b, s, h, d)) * 1.3).astype(np.float32)
    v = (r.standard_normal((b, s, h, d)) * 1.3).astype(np.float32)
    cos, sin = rope_tables(pos0 + s + 2, d)
    cache = sa.GpuKvCache(1, h, d, pos0 + s + 2, batch=b, bits=bits, qjl_residual=True, device=cuda_device)
    cache.set_position(pos0)
    cache.append(0, torch.from_numpy(k).reshape(b, s, h * d).to(cuda_device),
                 torch.from_numpy(v).reshape(b, s, h * d).to(cuda_device),
                 cos_cache=torch.from_numpy(cos).to(cuda_device), sin_cache=torch.from_numpy(sin).to(cuda_device),
                 do_rotary=True)
    torch.cuda.synchronize()
    view = cache.view(0)
    sl = slice(pos0, pos0 + s)
    signs = view.signs.cpu().numpy().astype(np.int8)
    got = _qjl_of(view, sl)
    codes = (view.k_codes[:, :, sl].cpu().numpy(), view.k_meta[:, :, sl].cpu().numpy(),
             view.v_codes_tokens()[:, :, sl].cpu().numpy(), view.v_meta[:, :, sl].cpu().numpy())
    cache.close()
    _assert_equal_bits(got, oracle_qjl(k, v, signs, bits, pos0, cos, sin, True), QJL_NAMES)
    _assert_equal_bits(codes, oracle_append(k, v, signs, bits, pos0, cos, sin, True),
                       ("k_codes", "k_meta", "v_codes", "v_meta"))


def test_bulk_append_bf16_interleaved(cuda_device):
    import smallaios_b200 as sa

    b, s, h, d, bits = 3, 9, 2, 128, 4
    r = rng(5)
    kt = torch.from_numpy((r.standard_normal((b, s, h, d)) * 2.0).astype(np.float32)).to(torch.bfloat16)
    vt = torch.from_numpy((r.standard_normal((b, s, h, d)) * 0.3).astype(np.float32)).to(torch.bfloat16)
    cos, sin = rope_tables(s + 1, d, 500000.0)
    cache = sa.GpuKvCache(1, h, d, s + 1, batch=b, bits=bits, qjl_residual=True, device=cuda_device)
    cache.append(0, kt.reshape(b, s, h * d).to(cuda_device), vt.reshape(b, s, h * d).to(cuda_device),
                 cos_cache=torch.from_numpy(cos).to(cuda_device), sin_cache=torch.from_numpy(sin).to(cuda_device),
                 do_rotary=True, rotary_interleaved=True)
    torch.cuda.synchronize()
    view = cache.view(0)
    got = _qjl_of(view, slice(0, s))
    signs = view.signs.cpu().numpy().astype(np.int8)
    cache.close()
    want = oracle_qjl(kt.float().numpy(), vt.float().numpy(), signs, bits, 0, cos, sin, True, True)
    _assert_equal_bits(got, want, QJL_NAMES)


@pytest.mark.parametrize("hq,hkv", [(32, 8), (16, 2)])
def test_decode_step_appends_residual(cuda_device, hq, hkv):
    """The attention call's own append of the new token (decode prep kernels, groups 4 and 8)."""
    import smallaios_b200 as sa

    b, d, bits, past = 3, 128, 4, 50
    r = rng(hq + hkv)
    k = torch.from_numpy((r.standard_normal((b, past + 1, hkv, d)) * 1.28).astype(np.float32)).to(torch.bfloat16)
    v = torch.from_numpy((r.standard_normal((b, past + 1, hkv, d)) * 1.28).astype(np.float32)).to(torch.bfloat16)
    q = torch.from_numpy((r.standard_normal((b, 1, hq * d)) * 1.28).astype(np.float32)).to(torch.bfloat16)
    cos, sin = rope_tables(past + 8, d, 500000.0)
    tcos, tsin = torch.from_numpy(cos).to(cuda_device), torch.from_numpy(sin).to(cuda_device)
    outs, got, signs = [], None, None
    for qjl in (False, True):
        cache = sa.GpuKvCache(1, hkv, d, past + 8, batch=b, num_heads=hq, bits=bits, qjl_residual=qjl,
                              device=cuda_device)
        cache.append(0, k[:, :past].reshape(b, past, hkv * d).to(cuda_device),
                     v[:, :past].reshape(b, past, hkv * d).to(cuda_device), cos_cache=tcos, sin_cache=tsin,
                     do_rotary=True)
        cache.advance_position(past)
        out = sa.group_query_attention(q.to(cuda_device), k[:, past:].reshape(b, 1, hkv * d).to(cuda_device),
                                       v[:, past:].reshape(b, 1, hkv * d).to(cuda_device), cache, 0, num_heads=hq,
                                       kv_num_heads=hkv, cos_cache=tcos, sin_cache=tsin)
        torch.cuda.synchronize()
        outs.append(out.cpu())
        if qjl:
            view = cache.view(0)
            got = _qjl_of(view, slice(0, past + 1))
            signs = view.signs.cpu().numpy().astype(np.int8)
        cache.close()
    assert torch.equal(outs[0], outs[1]), "the QJL option changed the attention output"
    want = oracle_qjl(k.float().numpy(), v.float().numpy(), signs, bits, 0, cos, sin, True)
    _assert_equal_bits(got, want, QJL_NAMES)


@pytest.mark.parametrize("b", [3, 20])
def test_fused_qkv_projection_appends_residual(cuda_device, b):
    """sa_qkv_project_append: the separate epilogue launch (batch 3) and the tcgen05 epilogue (batch 20)."""
    import smallaios_b200 as sa

    hq, hkv, d, hidden, bits, past = 8, 2, 128, 512, 4, 9
    r = rng(60 + b)
    n = (hq + 2 * hkv) * d
    codes = torch.from_numpy(r.integers(0, 256, size=(n, hidden // 32, 16), dtype=np.uint8))
    scales = torch.from_numpy(r.uniform(0.005, 0.02, size=(n, hidden // 32)).astype(np.float32)).to(torch.bfloat16)
    x = torch.from_numpy(r.standard_normal((b, hidden)).astype(np.float32)).to(torch.bfloat16)
    kp = torch.from_numpy((r.standard_normal((b, past, hkv, d)) * 1.28).astype(np.float32)).to(torch.bfloat16)
    vp = torch.from_numpy((r.standard_normal((b, past, hkv, d)) * 1.28).astype(np.float32)).to(torch.bfloat16)
    cos, sin = rope_tables(past + 8, d)
    tcos, tsin = torch.from_numpy(cos).to(cuda_device), torch.from_numpy(sin).to(cuda_device)
    cache = sa.GpuKvCache(1, hkv, d, past + 8, batch=b, num_heads=hq, bits=bits, qjl_residual=True,
                          device=cuda_device)
    cache.append(0, kp.reshape(b, past, hkv * d).to(cuda_device), vp.reshape(b, past, hkv * d).to(cuda_device),
                 cos_cache=tcos, sin_cache=tsin, do_rotary=True)
    cache.advance_position(past)
    _, kn, vn = sa.qkv_project_append(x.to(cuda_device), codes.to(cuda_device), scales.to(cuda_device), cache, 0,
                                      cos_cache=tcos, sin_cache=tsin, do_rotary=True)
    torch.cuda.synchronize()
    view = cache.view(0)
    got = _qjl_of(view, slice(0, past + 1))
    signs = view.signs.cpu().numpy().astype(np.int8)
    kall = np.concatenate([kp.float().numpy(), kn.float().cpu().numpy().reshape(b, 1, hkv, d)], axis=1)
    vall = np.concatenate([vp.float().numpy(), vn.float().cpu().numpy().reshape(b, 1, hkv, d)], axis=1)
    cache.close()
    _assert_equal_bits(got, oracle_qjl(kall, vall, signs, bits, 0, cos, sin, True), QJL_NAMES)


def test_residuals_off_by_default(cuda_device):
    import smallaios_b200 as sa

    cache = sa.GpuKvCache(1, 2, 64, 16, device=cuda_device)
    view = cache.view(0)
    assert view.k_qjl_bits is None and view.v_qjl_mag is None
    cache.close()
