"""Decoder-layer glue and one whole decoder layer (decode step) against the oracle.

- sa_rms_norm (SkipSimplifiedLayerNormalization / SimplifiedLayerNormalization)
  element for element: f32 within 1e-5 relative, fp16/bf16 within 1e-3 plus
  half an ulp of the output type; sa_silu_mul (SwiGLU) within 1e-3 (the
  oracle's Swish uses the reference's expf_approx, the kernel CUDA's expf).
- decoder_layer_step: the layer of the reference's model loader composed
  from the oracle's own ops (RMSNorm, MatMulNBits, RoPE, PolarQuant append,
  compressed attention, SwiGLU), rounding to the activation type where the
  GPU stores a tensor.  Rounding flips propagate through the chain, so the
  bar is a relative norm error of 1e-2 on the layer output and the residual.
"""
import numpy as np
import pytest
import torch

import oracle
from tests.helpers import oracle_append, oracle_attend, rng, rope_tables

pytestmark = pytest.mark.gpu

DT = {"f32": torch.float32, "f16": torch.float16, "bf16": torch.bfloat16}


def _rt(x, dtype):
    """Round an f32 array to dtype and back."""
    return torch.from_numpy(np.ascontiguousarray(x, np.float32)).to(dtype).float().numpy()


def _bound(want, dtype):
    if dtype == torch.float32:
        return 1e-5 + np.abs(want) * 1e-5
    ulp = 2.0 ** -8 if dtype == torch.bfloat16 else 2.0 ** -11
    return 1e-3 + np.abs(want) * ulp


@pytest.mark.parametrize("dt", ["f32", "f16", "bf16"])
@pytest.mark.parametrize("skip,bias", [(False, False), (True, False), (True, True)])
@pytest.mark.parametrize("cols", [4096, 8192, 1000, 4100])  # the register-held kernel; 4100: not for 16-bit
def test_rms_norm(cuda_device, dt, skip, bias, cols):
    import smallaios_b200 as sa

    dtype = DT[dt]
    r = rng(11)
    rows = 7
    x = _rt(r.standard_normal((rows, cols)) * 2.0, dtype)
    s = _rt(r.standard_normal((rows, cols)), dtype) if skip else None
    b = _rt(r.standard_normal(cols) * 0.1, dtype) if bias else None
    w = _rt(r.uniform(0.5, 1.5, cols), dtype)
    t = lambda a: None if a is None else torch.from_numpy(a).to(dtype).to(cuda_device)
    y, pre = sa.rms_norm(t(x), t(w), skip=t(s), bias=t(b), epsilon=1e-5)
    torch.cuda.synchronize()
    want, want_pre = oracle.rms_norm(x, w, 1e-5, skip=s, bias=b)
    got = y.float().cpu().numpy()
    assert np.all(np.abs(got - want) <= _bound(want, dtype)), f"max err {np.abs(got - want).max():.3e}"
    gp = pre.float().cpu().numpy()
    assert np.all(np.abs(gp - want_pre) <= _bound(want_pre, dtype))


@pytest.mark.parametrize("dt", ["f32", "bf16"])
@pytest.mark.parametrize("f", [3000, 3001])  # whole 16-byte units per row (vector kernel), or not
def test_silu_mul_packed_and_separate(cuda_device, dt, f):
    import smallaios_b200 as sa

    dtype = DT[dt]
    r = rng(12)
    rows = 5
    gu = _rt(r.standard_normal((rows, 2 * f)) * 3.0, dtype)
    t = torch.from_numpy(gu).to(dtype).to(cuda_device)
    want = oracle.silu_mul(gu[:, :f], gu[:, f:])
    for got in (sa.silu_mul(t), sa.silu_mul(t[:, :f].contiguous(), t[:, f:].contiguous())):
        torch.cuda.synchronize()
        g = got.float().cpu().numpy()
        # the oracle's Swish uses the reference's expf_approx, the kernel CUDA's expf: f32 within the 1e-3 bar
        bound = 1e-3 + np.abs(want) * 1e-5 if dtype == torch.float32 else _bound(want, dtype)
        assert np.all(np.abs(g - want) <= bound), f"max err {np.abs(g - want).max():.3e}"


def _weights(r, n, k, dtype):
    codes = r.integers(0, 256, size=(n, k // 32, 16), dtype=np.uint8)
    scales = _rt(r.uniform(0.005, 0.02, size=(n, k // 32)), dtype)
    return codes, scales


@pytest.mark.parametrize("b", [3, 24])
def test_decoder_layer_step(cuda_device, b):
    """Hidden 512, 8 query / 2 KV heads of 64, intermediate 1024, 30 cached tokens, fp16."""
    import smallaios_b200 as sa

    dev, dtype = cuda_device, torch.float16
    hidden, hq, hkv, d, f, past, bits, eps = 512, 8, 2, 64, 1024, 30, 4, 1e-5
    r = rng(100 + b)
    wqkv = _weights(r, (hq + 2 * hkv) * d, hidden, dtype)
    wo = _weights(r, hidden, hq * d, dtype)
    wgu = _weights(r, 2 * f, hidden, dtype)
    wdn = _weights(r, hidden, f, dtype)
    n_in = _rt(r.uniform(0.8, 1.2, hidden), dtype)
    n_post = _rt(r.uniform(0.8, 1.2, hidden), dtype)
    x = _rt(r.standard_normal((b, hidden)), dtype)
    resid = _rt(r.standard_normal((b, hidden)), dtype)
    kp = _rt(r.standard_normal((b, past, hkv, d)) * 1.28, dtype)
    vp = _rt(r.standard_normal((b, past, hkv, d)) * 1.28, dtype)
    cos, sin = rope_tables(past + 4, d, 10000.0)
    tcos, tsin = torch.from_numpy(cos).to(dev), torch.from_numpy(sin).to(dev)

    t = lambda a, dt=dtype: torch.from_numpy(np.ascontiguousarray(a)).to(dt).to(dev)
    w = sa.LayerWeights(t(wqkv[0], torch.uint8), t(wqkv[1]), t(wo[0], torch.uint8), t(wo[1]),
                        t(wgu[0], torch.uint8), t(wgu[1]), t(wdn[0], torch.uint8), t(wdn[1]), t(n_in), t(n_post),
                        eps)
    cache = sa.GpuKvCache(1, hkv, d, past + 4, batch=b, num_heads=hq, bits=bits, device=dev)
    cache.append(0, t(kp.reshape(b, past, -1)), t(vp.reshape(b, past, -1)), cos_cache=tcos, sin_cache=tsin,
                 do_rotary=True)
    cache.advance_position(past)
    dn, pre2 = sa.decoder_layer_step(t(x), t(resid), w, cache, 0, cos_cache=tcos, sin_cache=tsin)
    torch.cuda.synchronize()
    signs = cache.view(0).signs.cpu().numpy().astype(np.int8)
    cache.close()

    # the oracle composition, rounding where the GPU stores a tensor
    h1, pre1 = oracle.rms_norm(x, n_in, eps, skip=resid)
    h1, pre1 = _rt(h1, dtype), _rt(pre1, dtype)
    qkv = _rt(oracle.matmul_nbits(h1, wqkv[0], wqkv[1], n=(hq + 2 * hkv) * d, k=hidden), dtype)
    q, kn, vn = qkv[:, :hq * d], qkv[:, hq * d:(hq + hkv) * d], qkv[:, (hq + hkv) * d:]
    kall = np.concatenate([kp, kn.reshape(b, 1, hkv, d)], axis=1)
    vall = np.concatenate([vp, vn.reshape(b, 1, hkv, d)], axis=1)
    kc, km, vc, vm = oracle_append(kall, vall, signs, bits, 0, cos, sin, True, False)
    a = oracle_attend(q.reshape(b, 1, hq, d), kc, km, vc, vm, signs, bits, past, cos=cos, sin=sin, do_rotary=True)
    a = _rt(a.reshape(b, hq * d), dtype)
    o = _rt(oracle.matmul_nbits(a, wo[0], wo[1], n=hidden, k=hq * d), dtype)
    h2, want_pre2 = oracle.rms_norm(o, n_post, eps, skip=pre1)
    h2, want_pre2 = _rt(h2, dtype), _rt(want_pre2, dtype)
    gu = _rt(oracle.matmul_nbits(h2, wgu[0], wgu[1], n=2 * f, k=hidden), dtype)
    m = _rt(oracle.silu_mul(gu[:, :f], gu[:, f:]), dtype)
    want = oracle.matmul_nbits(m, wdn[0], wdn[1], n=hidden, k=f)

    for name, got, ref in (("down", dn.float().cpu().numpy(), want), ("residual", pre2.float().cpu().numpy(),
                                                                     want_pre2)):
        rel = np.linalg.norm(got - ref) / np.linalg.norm(ref)
        assert rel <= 1e-2, f"{name}: relative error {rel:.3e}"


def test_dispatch_norm_nodes(cuda_device):
    """dispatch_gpu_node arms for the normalization ops (ORT input orders)."""
    import smallaios_b200 as sa

    for op in ("RMSNormalization", "SimplifiedLayerNormalization", "SkipSimplifiedLayerNormalization"):
        assert sa.supports_op(op)
    r = rng(13)
    x = r.standard_normal((2, 3, 64)).astype(np.float32)
    s = r.standard_normal((2, 3, 64)).astype(np.float32)
    w = r.uniform(0.5, 1.5, 64).astype(np.float32)
    t = lambda a: torch.from_numpy(a).to(cuda_device)
    (y,) = sa.dispatch_gpu_node("SimplifiedLayerNormalization", [t(x), t(w)], {"epsilon": 1e-6})
    want, _ = oracle.rms_norm(x, w, 1e-6)
    assert np.allclose(y.cpu().numpy(), want, rtol=1e-5, atol=1e-5)
    y, pre = sa.dispatch_gpu_node("SkipSimplifiedLayerNormalization", [t(x), t(s), t(w)], {"epsilon": 1e-6})
    want, want_pre = oracle.rms_norm(x, w, 1e-6, skip=s)
    assert np.allclose(y.cpu().numpy(), want, rtol=1e-5, atol=1e-5)
    assert np.allclose(pre.cpu().numpy(), want_pre, rtol=1e-6, atol=1e-6)
    with pytest.raises(sa.InvalidAttribute):
        sa.dispatch_gpu_node("RMSNormalization", [t(x), t(w)], {"axis": 1})


@pytest.mark.parametrize("f", [8, 7])  # the vector kernel and the scalar one
def test_silu_mul_rows_beyond_one_grid_dimension(cuda_device, f):
    """More rows than a launch's grid.y takes (65535): the kernels loop over the rest."""
    import smallaios_b200 as sa

    r = rng(13)
    rows = 70001
    gu = _rt(r.standard_normal((rows, 2 * f)) * 3.0, torch.bfloat16)
    got = sa.silu_mul(torch.from_numpy(gu).to(torch.bfloat16).to(cuda_device))
    torch.cuda.synchronize()
    want = oracle.silu_mul(gu[:, :f], gu[:, f:])
    g = got.float().cpu().numpy()
    assert np.all(np.abs(g - want) <= _bound(want, torch.bfloat16)), f"max err {np.abs(g - want).max():.3e}"
