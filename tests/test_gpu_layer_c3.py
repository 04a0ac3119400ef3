"""A whole decoder layer at the Llama-3-8B decode shape, stage by stage.

B = 64 rows, hidden 4096, 32 query / 8 KV heads of 128, intermediate 14336, int4
MatMulNBits weights (block 32), an int4 PolarQuant cache of 500 tokens, bf16.
Each stage of decoder_layer_step runs on the GPU and is checked against the oracle
fed with the GPU's own input to that stage, at the operator bar: max-abs 1e-3 plus
half an ulp of bf16 (the GPU rounds each stored tensor to bf16 once; q, rounded before
and after RoPE, also gets one ulp of its rotated pair's inputs):

  SkipSimplifiedLayerNormalization -> fused QKV projection (+ RoPE, + append: the codes
  bit for bit) -> GroupQueryAttention over the cache -> o_proj -> the second norm ->
  gate|up projection -> SwiGLU -> down_proj.

The composed decoder_layer_step must give exactly the staged kernels' results.
"""
import numpy as np
import pytest
import torch

import oracle
from tests.helpers import oracle_append, rng, rope_tables

pytestmark = pytest.mark.gpu

B, HIDDEN, HQ, HKV, D, F, PAST, BITS, EPS = 64, 4096, 32, 8, 128, 14336, 500, 4, 1e-5
DT = torch.bfloat16


def _rt(x):
    return torch.from_numpy(np.ascontiguousarray(x, np.float32)).to(DT).float().numpy()


def _np(t):
    return t.float().cpu().numpy()


def _check(name, got, want, ulps=0.5):
    """max-abs 1e-3 plus `ulps` bf16 ulps (2^-7 relative) of the expected value."""
    err = np.abs(got - want)
    bound = 1e-3 + np.abs(want) * ulps * 2.0 ** -7
    worst = np.unravel_index(np.argmax(err - bound), err.shape)
    assert np.all(err <= bound), f"{name}: max err {err.max():.3e} at {worst} (got {got[worst]}, want {want[worst]})"


def _weights(r, n, k):
    codes = r.integers(0, 256, size=(n, k // 32, 16), dtype=np.uint8)
    scales = _rt(r.uniform(0.005, 0.02, size=(n, k // 32)))
    return codes, scales


def test_decoder_layer_c3_stagewise(cuda_device):
    import smallaios_b200 as sa

    dev = cuda_device
    r = rng(777)
    wqkv = _weights(r, (HQ + 2 * HKV) * D, HIDDEN)
    wo = _weights(r, HIDDEN, HQ * D)
    wgu = _weights(r, 2 * F, HIDDEN)
    wdn = _weights(r, HIDDEN, F)
    n_in, n_post = _rt(r.uniform(0.8, 1.2, HIDDEN)), _rt(r.uniform(0.8, 1.2, HIDDEN))
    x, resid = _rt(r.standard_normal((B, HIDDEN))), _rt(r.standard_normal((B, HIDDEN)))
    kp = _rt(r.standard_normal((B, PAST, HKV, D)) * 1.28)
    vp = _rt(r.standard_normal((B, PAST, HKV, D)) * 1.28)
    cos, sin = rope_tables(PAST + 8, D, 500000.0)
    tcos, tsin = torch.from_numpy(cos).to(dev), torch.from_numpy(sin).to(dev)
    t = lambda a, dt=DT: torch.from_numpy(np.ascontiguousarray(a)).to(dt).to(dev)
    w = sa.LayerWeights(t(wqkv[0], torch.uint8), t(wqkv[1]), t(wo[0], torch.uint8), t(wo[1]),
                        t(wgu[0], torch.uint8), t(wgu[1]), t(wdn[0], torch.uint8), t(wdn[1]), t(n_in), t(n_post), EPS)

    def fresh_cache():
        c = sa.GpuKvCache(1, HKV, D, PAST + 8, batch=B, num_heads=HQ, bits=BITS, device=dev)
        c.append(0, t(kp.reshape(B, PAST, -1)), t(vp.reshape(B, PAST, -1)), cos_cache=tcos, sin_cache=tsin,
                 do_rotary=True)
        c.advance_position(PAST)
        return c

    # ---- the stages, one kernel call each ----
    cache = fresh_cache()
    h1, pre1 = sa.rms_norm(t(x), w.input_norm, skip=t(resid), epsilon=EPS)
    q, k, v = sa.qkv_project_append(h1, w.wqkv_codes, w.wqkv_scales, cache, 0, cos_cache=tcos, sin_cache=tsin)
    a = sa.gqa_attend(q.view(B, 1, HQ * D), cache, 0, num_heads=HQ, do_rotary=False)
    o = sa.matmul_nbits(a.view(B, HQ * D), w.wo_codes, w.wo_scales, K=HQ * D, N=HIDDEN)
    h2, pre2 = sa.rms_norm(o, w.post_norm, skip=pre1, epsilon=EPS)
    gu = sa.matmul_nbits(h2, w.wgu_codes, w.wgu_scales, K=HIDDEN, N=2 * F)
    m = sa.silu_mul(gu)
    dn = sa.matmul_nbits(m, w.wdown_codes, w.wdown_scales, K=F, N=HIDDEN)
    torch.cuda.synchronize()
    view = cache.view(0)
    signs = view.signs.cpu().numpy().astype(np.int8)
    kc_g = view.k_codes[:, :, :PAST + 1].cpu().numpy()
    vc_g = view.v_codes_tokens()[:, :, :PAST + 1].cpu().numpy()
    km_g = view.k_meta[:, :, :PAST + 1].cpu().numpy()
    vm_g = view.v_meta[:, :, :PAST + 1].cpu().numpy()
    cache.close()

    # ---- each stage against the oracle on the GPU's own input ----
    want_h1, want_pre1 = oracle.rms_norm(x, n_in, EPS, skip=resid)
    _check("input norm", _np(h1), want_h1)
    _check("input residual", _np(pre1), want_pre1)

    proj = oracle.matmul_nbits(_np(h1), wqkv[0], wqkv[1], n=(HQ + 2 * HKV) * D, k=HIDDEN)
    q_pre = _rt(proj[:, :HQ * D]).reshape(B, HQ, 1, D)
    want_q = oracle.apply_rope(q_pre, cos, sin, [PAST]).reshape(B, HQ * D)
    # q is rounded twice on the GPU (the projection's store, then RoPE in place). The first
    # rounding may fall the other way from the oracle's on either element of a rotated pair,
    # so the bar adds one bf16 ulp of both pre-RoPE elements to half an ulp of the result.
    pair_mag = (np.abs(q_pre) + np.abs(np.roll(q_pre, D // 2, axis=-1))).reshape(B, HQ * D)
    err = np.abs(_np(q) - want_q)
    assert np.all(err <= 1e-3 + pair_mag * 2.0 ** -7 + np.abs(want_q) * 2.0 ** -8), f"q: max err {err.max():.3e}"
    _check("k (projected)", _np(k), proj[:, HQ * D:(HQ + HKV) * D])
    _check("v (projected)", _np(v), proj[:, (HQ + HKV) * D:])
    # the appended token: PolarQuantizer::encode of RoPE(k) and v as the GPU stored them (bf16)
    kall = np.concatenate([kp, _np(k).reshape(B, 1, HKV, D)], axis=1)
    vall = np.concatenate([vp, _np(v).reshape(B, 1, HKV, D)], axis=1)
    kc, km, vc, vm = oracle_append(kall, vall, signs, BITS, 0, cos, sin, True, False)
    assert np.array_equal(kc_g, kc) and np.array_equal(vc_g, vc)
    assert np.array_equal(km_g.view(np.uint32), km.view(np.uint32))
    assert np.array_equal(vm_g.view(np.uint32), vm.view(np.uint32))

    qn = _np(q).reshape(B, HQ, 1, D)
    scale = np.float32(1.0) / np.float32(oracle.sqrt_f32(float(D)))
    want_a = oracle.compressed_gqa(qn, kc, km, vc, vm, signs, BITS, scale, nthreads=8)
    _check("attention", _np(a).reshape(B, HQ * D), want_a.reshape(B, HQ * D))

    _check("o_proj", _np(o), oracle.matmul_nbits(_np(a), wo[0], wo[1], n=HIDDEN, k=HQ * D))
    want_h2, want_pre2 = oracle.rms_norm(_np(o), n_post, EPS, skip=_np(pre1))
    _check("post norm", _np(h2), want_h2)
    _check("post residual", _np(pre2), want_pre2)
    _check("gate|up", _np(gu), oracle.matmul_nbits(_np(h2), wgu[0], wgu[1], n=2 * F, k=HIDDEN))
    g_np = _np(gu)
    _check("SwiGLU", _np(m), oracle.silu_mul(g_np[:, :F], g_np[:, F:]))
    _check("down_proj", _np(dn), oracle.matmul_nbits(_np(m), wdn[0], wdn[1], n=HIDDEN, k=F))

    # ---- the composed layer runs exactly these kernels ----
    cache = fresh_cache()
    dn2, pre2b = sa.decoder_layer_step(t(x), t(resid), w, cache, 0, cos_cache=tcos, sin_cache=tsin)
    torch.cuda.synchronize()
    cache.close()
    assert torch.equal(dn2, dn) and torch.equal(pre2b, pre2)
