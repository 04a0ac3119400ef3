"""A decoder layer over whole prompts (prefill_layer_step), stage by stage.

B = 2 prompts of 80 tokens (a ragged last 64-token tile), hidden 512, 8 query / 2 KV heads of
64, intermediate 1024, int4 MatMulNBits weights (block 32), an int8 PolarQuant cache, bf16.
Every projection runs on the tcgen05 MatMulNBits (160 rows). Each stage of prefill_layer_step
runs on the GPU and is checked against the oracle fed with the GPU's own input to that stage,
at the operator bar: max-abs 1e-3 plus half an ulp of bf16 (the GPU rounds each stored tensor
to bf16 once):

  SkipSimplifiedLayerNormalization -> Q, K, V projections (row blocks of the packed Wqkv) ->
  GroupQueryAttention (RoPE and quantize-on-append of the prompts, the codes bit for bit; the
  causal prefill attention) -> o_proj -> the second norm -> gate|up -> SwiGLU -> down_proj.

A second chunk of 48 tokens then continues the same prompts at position 80. The composed
prefill_layer_step must give exactly the staged kernels' results.
"""
import numpy as np
import pytest
import torch

import oracle
from tests.helpers import oracle_append, oracle_attend, rng, rope_tables

pytestmark = pytest.mark.gpu

B, HIDDEN, HQ, HKV, D, F, BITS, EPS = 2, 512, 8, 2, 64, 1024, 8, 1e-5
S1, S2 = 80, 48
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


def _stages(sa, t, w, cache, x, resid, s, pos0, tcos, tsin):
    """The layer's kernels one call at a time (the sequence prefill_layer_step runs)."""
    m = B * s
    h1, pre1 = sa.rms_norm(t(x), w.input_norm, skip=t(resid), epsilon=EPS)
    qd, kd = HQ * D, HKV * D
    q = sa.matmul_nbits(h1, w.wqkv_codes[:qd], w.wqkv_scales[:qd], K=HIDDEN, N=qd)
    k = sa.matmul_nbits(h1, w.wqkv_codes[qd:qd + kd], w.wqkv_scales[qd:qd + kd], K=HIDDEN, N=kd)
    v = sa.matmul_nbits(h1, w.wqkv_codes[qd + kd:], w.wqkv_scales[qd + kd:], K=HIDDEN, N=kd)
    cache.set_position(pos0)
    a = sa.group_query_attention(q.view(B, s, qd), k.view(B, s, kd), v.view(B, s, kd), cache, 0, num_heads=HQ,
                                 kv_num_heads=HKV, cos_cache=tcos, sin_cache=tsin)
    o = sa.matmul_nbits(a.view(m, qd), w.wo_codes, w.wo_scales, K=qd, N=HIDDEN)
    h2, pre2 = sa.rms_norm(o, w.post_norm, skip=pre1, epsilon=EPS)
    gu = sa.matmul_nbits(h2, w.wgu_codes, w.wgu_scales, K=HIDDEN, N=2 * F)
    mm = sa.silu_mul(gu)
    dn = sa.matmul_nbits(mm, w.wdown_codes, w.wdown_scales, K=F, N=HIDDEN)
    return dict(h1=h1, pre1=pre1, q=q, k=k, v=v, a=a, o=o, h2=h2, pre2=pre2, gu=gu, m=mm, dn=dn)


def test_prefill_layer_stagewise(cuda_device):
    import smallaios_b200 as sa

    dev = cuda_device
    r = rng(4242)
    wqkv = _weights(r, (HQ + 2 * HKV) * D, HIDDEN)
    wo = _weights(r, HIDDEN, HQ * D)
    wgu = _weights(r, 2 * F, HIDDEN)
    wdn = _weights(r, HIDDEN, F)
    n_in, n_post = _rt(r.uniform(0.8, 1.2, HIDDEN)), _rt(r.uniform(0.8, 1.2, HIDDEN))
    cos, sin = rope_tables(S1 + S2 + 8, D, 500000.0)
    tcos, tsin = torch.from_numpy(cos).to(dev), torch.from_numpy(sin).to(dev)
    t = lambda a, dt=DT: torch.from_numpy(np.ascontiguousarray(a)).to(dt).to(dev)
    w = sa.LayerWeights(t(wqkv[0], torch.uint8), t(wqkv[1]), t(wo[0], torch.uint8), t(wo[1]),
                        t(wgu[0], torch.uint8), t(wgu[1]), t(wdn[0], torch.uint8), t(wdn[1]), t(n_in), t(n_post), EPS)
    cache = sa.GpuKvCache(1, HKV, D, S1 + S2 + 16, batch=B, num_heads=HQ, bits=BITS, device=dev)
    signs = cache.view(0).signs.cpu().numpy().astype(np.int8)
    k_all, v_all = [], []
    staged = []
    for s, pos0 in ((S1, 0), (S2, S1)):
        x, resid = _rt(r.standard_normal((B * s, HIDDEN))), _rt(r.standard_normal((B * s, HIDDEN)))
        g = _stages(sa, t, w, cache, x, resid, s, pos0, tcos, tsin)
        torch.cuda.synchronize()
        staged.append((x, resid, s, pos0, g))

        want_h1, want_pre1 = oracle.rms_norm(x, n_in, EPS, skip=resid)
        _check("input norm", _np(g["h1"]), want_h1)
        _check("input residual", _np(g["pre1"]), want_pre1)
        proj = oracle.matmul_nbits(_np(g["h1"]), wqkv[0], wqkv[1], n=(HQ + 2 * HKV) * D, k=HIDDEN)
        _check("q", _np(g["q"]), proj[:, :HQ * D])
        _check("k", _np(g["k"]), proj[:, HQ * D:(HQ + HKV) * D])
        _check("v", _np(g["v"]), proj[:, (HQ + HKV) * D:])

        # the prompts' K/V as the GPU stored them (bf16), appended after the earlier chunk
        k_all.append(_np(g["k"]).reshape(B, s, HKV, D))
        v_all.append(_np(g["v"]).reshape(B, s, HKV, D))
        kc, km, vc, vm = oracle_append(np.concatenate(k_all, 1), np.concatenate(v_all, 1), signs, BITS, 0, cos, sin,
                                       True, False)
        view = cache.view(0)
        tt = pos0 + s
        assert np.array_equal(view.k_codes[:, :, :tt].cpu().numpy(), kc)
        assert np.array_equal(view.v_codes_tokens()[:, :, :tt].cpu().numpy(), vc)
        assert np.array_equal(view.k_meta[:, :, :tt].cpu().numpy().view(np.uint32), km.view(np.uint32))
        assert np.array_equal(view.v_meta[:, :, :tt].cpu().numpy().view(np.uint32), vm.view(np.uint32))
        want_a = oracle_attend(_np(g["q"]).reshape(B, s, HQ, D), kc, km, vc, vm, signs, BITS, pos0, cos=cos, sin=sin,
                               do_rotary=True)
        _check("attention", _np(g["a"]).reshape(B * s, HQ * D), want_a.reshape(B * s, HQ * D))

        _check("o_proj", _np(g["o"]), oracle.matmul_nbits(_np(g["a"]).reshape(B * s, HQ * D), wo[0], wo[1],
                                                           n=HIDDEN, k=HQ * D))
        want_h2, want_pre2 = oracle.rms_norm(_np(g["o"]), n_post, EPS, skip=_np(g["pre1"]))
        _check("post norm", _np(g["h2"]), want_h2)
        _check("post residual", _np(g["pre2"]), want_pre2)
        _check("gate|up", _np(g["gu"]), oracle.matmul_nbits(_np(g["h2"]), wgu[0], wgu[1], n=2 * F, k=HIDDEN))
        gnp = _np(g["gu"])
        _check("SwiGLU", _np(g["m"]), oracle.silu_mul(gnp[:, :F], gnp[:, F:]))
        _check("down_proj", _np(g["dn"]), oracle.matmul_nbits(_np(g["m"]), wdn[0], wdn[1], n=HIDDEN, k=F))
    cache.close()

    # the composed layer runs exactly these kernels, chunk after chunk
    cache = sa.GpuKvCache(1, HKV, D, S1 + S2 + 16, batch=B, num_heads=HQ, bits=BITS, device=dev)
    for x, resid, s, pos0, g in staged:
        cache.set_position(pos0)
        dn, pre2 = sa.prefill_layer_step(t(x), t(resid), w, cache, 0, batch=B, seq_len=s, cos_cache=tcos,
                                         sin_cache=tsin)
        torch.cuda.synchronize()
        assert torch.equal(dn, g["dn"]) and torch.equal(pre2, g["pre2"])
    cache.close()
