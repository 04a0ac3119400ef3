"""Fused QKV projection + RoPE + quantize-on-append (sa_qkv_project_append).

Checks, on the same seeded inputs:

- The projections against the oracle (dequantize in f32 + gemm_f32): k and v
  within max-abs 1e-3 plus half an ulp of the output type; q after the oracle
  RoPE of the rounded projection within the same bound plus one more rounding.
- The cache codes of the new token, bit for bit, against PolarQuantizer::encode
  of RoPE(k) and v, where k and v are the op's own rounded outputs.
- The attention that follows (gqa_attend on the rotated q, do_rotary off)
  against the composite oracle, within the attention tolerance.

Both paths are covered:

- batch 17..128 with 128-column-aligned head blocks runs as one tcgen05
  launch with the epilogue fused in;
- other batches run the three projections and then one epilogue launch.
"""
import numpy as np
import pytest
import torch

import oracle
from tests.helpers import oracle_append, oracle_attend, rng, rope_tables

pytestmark = pytest.mark.gpu


def _ulp(dtype):
    return 2.0 ** -8 if dtype == torch.bfloat16 else 2.0 ** -11


def _case(dev, *, b, hq, hkv, d, hidden, dtype, past, seed, interleaved=False, bits=4, theta=10000.0):
    import smallaios_b200 as sa

    r = rng(seed)
    n = (hq + 2 * hkv) * d
    codes = r.integers(0, 256, size=(n, hidden // 32, 16), dtype=np.uint8)
    scales = torch.from_numpy(r.uniform(0.005, 0.02, size=(n, hidden // 32)).astype(np.float32)).to(dtype)
    x = torch.from_numpy(r.standard_normal((b, hidden)).astype(np.float32)).to(dtype)
    kp = torch.from_numpy((r.standard_normal((b, past, hkv, d)) * 1.28).astype(np.float32)).to(dtype)
    vp = torch.from_numpy((r.standard_normal((b, past, hkv, d)) * 1.28).astype(np.float32)).to(dtype)
    cos, sin = rope_tables(past + 8, d, theta)
    tcos, tsin = torch.from_numpy(cos).to(dev), torch.from_numpy(sin).to(dev)
    cache = sa.GpuKvCache(1, hkv, d, past + 8, batch=b, num_heads=hq, bits=bits, device=dev)
    if past:
        cache.append(0, kp.reshape(b, past, hkv * d).to(dev), vp.reshape(b, past, hkv * d).to(dev), cos_cache=tcos,
                     sin_cache=tsin, do_rotary=True, rotary_interleaved=interleaved)
        cache.advance_position(past)
    q, k, v = sa.qkv_project_append(x.to(dev), torch.from_numpy(codes).to(dev), scales.to(dev), cache, 0,
                                    cos_cache=tcos, sin_cache=tsin, do_rotary=True, rotary_interleaved=interleaved)
    # the query sits at the appended token's position: attend, then advance
    out = sa.gqa_attend(q.reshape(b, 1, hq * d), cache, 0, num_heads=hq, do_rotary=False)
    cache.advance_position(1)
    torch.cuda.synchronize()
    q, k, v = (t.float().cpu().numpy() for t in (q, k, v))
    got = out.float().cpu().numpy()
    view = cache.view(0)
    signs = view.signs.cpu().numpy().astype(np.int8)
    gcodes = (view.k_codes[:, :, :past + 1].cpu().numpy(), view.k_meta[:, :, :past + 1].cpu().numpy(),
              view.v_codes_tokens()[:, :, :past + 1].cpu().numpy(), view.v_meta[:, :, :past + 1].cpu().numpy())
    cache.close()

    # projections against the oracle
    want = oracle.matmul_nbits(x.float().numpy(), codes, scales.float().numpy(), None, n=n, k=hidden)
    qc, kc = hq * d, hkv * d
    ulp = _ulp(dtype)
    for name, g, w in (("k", k, want[:, qc:qc + kc]), ("v", v, want[:, qc + kc:])):
        err = np.abs(g - w)
        assert np.all(err <= 1e-3 + np.abs(w) * ulp), f"{name}: max err {err.max():.3e}"
    q_pre = torch.from_numpy(want[:, :qc]).to(dtype).float().numpy().reshape(b, hq, 1, d)
    q_want = oracle.apply_rope(q_pre, cos, sin, np.array([past]), interleaved=interleaved).reshape(b, qc)
    # the op rounds its f32 projection to the activation type before the rotation, like the
    # oracle's q_pre; near a rounding boundary the two sums may round one ulp (2 * ulp * |x|)
    # apart, and the rotation carries that into the element AND its rotary partner
    mag = np.abs(q_pre).reshape(b, hq, d)
    if interleaved:
        partner = mag.reshape(b, hq, d // 2, 2)[..., ::-1].reshape(b, hq, d)
    else:
        partner = np.concatenate([mag[..., d // 2:], mag[..., :d // 2]], axis=-1)
    tol = 2e-3 + 2 * ulp * (mag + partner).reshape(b, qc) + np.abs(q_want) * ulp
    err = np.abs(q - q_want)
    assert np.all(err <= tol), f"q: max err {err.max():.3e}, worst excess {(err - tol).max():.3e}"

    # cache codes: bit-exact with the encoder on the op's own k / v (past tokens: the library's append)
    kall = np.concatenate([kp.float().numpy(), k.reshape(b, 1, hkv, d)], axis=1)
    vall = np.concatenate([vp.float().numpy(), v.reshape(b, 1, hkv, d)], axis=1)
    okc, okm, ovc, ovm = oracle_append(kall, vall, signs, bits, 0, cos, sin, True, interleaved)
    assert np.array_equal(gcodes[0], okc), "k codes differ"
    assert np.array_equal(gcodes[1].view(np.uint32), okm.view(np.uint32)), "k meta differ"
    assert np.array_equal(gcodes[2], ovc), "v codes differ"
    assert np.array_equal(gcodes[3].view(np.uint32), ovm.view(np.uint32)), "v meta differ"

    # the attention that follows, on the op's rotated q
    att = oracle_attend(q.reshape(b, 1, hq, d), okc, okm, ovc, ovm, signs, bits, past)
    err = np.abs(got - att)
    assert np.all(err <= 1e-3 + np.abs(att) * ulp), f"attention: max err {err.max():.3e}"


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
@pytest.mark.parametrize("b", [17, 40])
def test_fused_tcgen05_epilogue(cuda_device, dtype, b):
    """One tcgen05 launch: head_dim 128, 8 query / 2 KV heads, hidden 512."""
    _case(cuda_device, b=b, hq=8, hkv=2, d=128, hidden=512, dtype=dtype, past=37, seed=b)


def test_fused_tcgen05_head_dim_64_interleaved(cuda_device):
    """head_dim 64: each 128-column tile holds two heads; interleaved rotary."""
    _case(cuda_device, b=24, hq=8, hkv=2, d=64, hidden=768, dtype=torch.bfloat16, past=20, seed=3, interleaved=True)


def test_fused_c3_layer_shape(cuda_device):
    """Llama-3-8B layer (hidden 4096, 32 / 8 heads, D = 128) at batch 64, theta 5e5."""
    _case(cuda_device, b=64, hq=32, hkv=8, d=128, hidden=4096, dtype=torch.bfloat16, past=100, seed=8,
          theta=500000.0)


@pytest.mark.parametrize("b", [1, 3, 16])
def test_projection_then_epilogue_launch(cuda_device, b):
    """Batches below 17: the three MatMulNBits launches, then the epilogue kernel."""
    _case(cuda_device, b=b, hq=8, hkv=2, d=128, hidden=1024, dtype=torch.float16, past=11, seed=50 + b)


def test_group8_and_first_token(cuda_device):
    """Eight query heads per KV head, an empty cache (the new token is the whole context)."""
    _case(cuda_device, b=20, hq=16, hkv=2, d=128, hidden=512, dtype=torch.bfloat16, past=0, seed=77)


def test_errors(cuda_device):
    import smallaios_b200 as sa

    cache = sa.GpuKvCache(1, 2, 128, 8, batch=2, num_heads=8, bits=4, device=cuda_device)
    x = torch.zeros(2, 512, dtype=torch.float16, device=cuda_device)
    n = (8 + 4) * 128
    codes = torch.zeros(n, 16, 16, dtype=torch.uint8, device=cuda_device)
    scales = torch.zeros(n, 16, dtype=torch.float16, device=cuda_device)
    with pytest.raises(sa.ShapeMismatch):  # weights for a different head count
        sa.qkv_project_append(x, codes[:-128], scales[:-128], cache, 0, do_rotary=False)
    with pytest.raises(sa.UnsupportedOp):
        sa.qkv_project_append(x.float(), codes, scales.float(), cache, 0, do_rotary=False)
    with pytest.raises(sa.ShapeMismatch):  # rotary without tables
        sa.qkv_project_append(x, codes, scales, cache, 0, do_rotary=True)
    cache.set_position(8)
    with pytest.raises(sa.CapacityError):
        sa.qkv_project_append(x, codes, scales, cache, 0, do_rotary=False)
    cache.close()
