"""The committed golden fixtures (tests/golden/*.npz, written by gen_golden.py).

CPU: the oracle must still reproduce every code byte, scale, zero point and
the GQA output bit for bit, so a silent change of the restatement shows up
here instead of moving both sides of the GPU parity tests together.
GPU: the library's append and GroupQueryAttention on the fixture inputs must
write the fixture's codes and metadata bit for bit and attend within 1e-3.
"""
import os

import numpy as np
import pytest

from tests.golden.gen_golden import CONFIGS, bf16_to_f32, expected, inputs

HERE = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")


def _load(name):
    z = np.load(os.path.join(HERE, f"{name}.npz"))
    return {k: z[k] for k in z.files}


@pytest.mark.parametrize("name", sorted(CONFIGS))
def test_fixture_inputs_are_the_seeded_ones(name):
    g = _load(name)
    k, v, q = inputs(CONFIGS[name])
    assert np.array_equal(g["k_bf16"], k) and np.array_equal(g["v_bf16"], v) and np.array_equal(g["q_bf16"], q)


@pytest.mark.parametrize("name", sorted(CONFIGS))
def test_oracle_reproduces_fixture_bit_for_bit(name):
    g = _load(name)
    exp = expected(CONFIGS[name], bf16_to_f32(g["k_bf16"]), bf16_to_f32(g["v_bf16"]), bf16_to_f32(g["q_bf16"]))
    for key, val in exp.items():
        got = val.view(np.uint32) if val.dtype == np.float32 else val
        want = g[key].view(np.uint32) if g[key].dtype == np.float32 else g[key]
        assert np.array_equal(got, want), f"{name}: {key} differs from the committed fixture"


@pytest.mark.gpu
@pytest.mark.parametrize("name", sorted(CONFIGS))
def test_library_matches_fixture(cuda_device, name):
    import torch

    import smallaios_b200 as sa
    import oracle

    g = _load(name)
    b, hq, hkv, d, t, bits = (int(x) for x in g["params"])
    k = torch.from_numpy(bf16_to_f32(g["k_bf16"])).to(cuda_device)
    v = torch.from_numpy(bf16_to_f32(g["v_bf16"])).to(cuda_device)
    q = torch.from_numpy(bf16_to_f32(g["q_bf16"])).to(cuda_device)
    cos, sin = oracle.rope_tables(t + 8, d // 2, float(g["theta"]))
    cos_t, sin_t = torch.from_numpy(cos).to(cuda_device), torch.from_numpy(sin).to(cuda_device)
    cache = sa.GpuKvCache(1, hkv, d, t + 8, batch=b, num_heads=hq, bits=bits, device=cuda_device)
    cache.append(0, k[:, :t - 1].reshape(b, t - 1, hkv * d).contiguous(),
                 v[:, :t - 1].reshape(b, t - 1, hkv * d).contiguous(), cos_cache=cos_t, sin_cache=sin_t,
                 do_rotary=True)
    cache.advance_position(t - 1)
    out = sa.group_query_attention(q.reshape(b, 1, hq * d), k[:, t - 1:].reshape(b, 1, hkv * d).contiguous(),
                                   v[:, t - 1:].reshape(b, 1, hkv * d).contiguous(), cache, 0, num_heads=hq,
                                   kv_num_heads=hkv, cos_cache=cos_t, sin_cache=sin_t)
    torch.cuda.synchronize()
    view = cache.view(0)
    assert np.array_equal(view.signs.cpu().numpy().astype(np.int8), g["signs"])
    assert np.array_equal(view.k_codes[:, :, :t].cpu().numpy(), g["k_codes"])
    assert np.array_equal(view.v_codes_tokens()[:, :, :t].cpu().numpy(), g["v_codes"])
    assert np.array_equal(view.k_meta[:, :, :t].cpu().numpy().view(np.uint32), g["k_meta_bits"])
    assert np.array_equal(view.v_meta[:, :, :t].cpu().numpy().view(np.uint32), g["v_meta_bits"])
    err = np.abs(out.cpu().numpy() - g["out"]).max()
    assert err <= 1e-3, f"{name}: max-abs error {err:.3e}"
    cache.close()
