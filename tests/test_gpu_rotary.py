"""RotaryEmbedding as its own node vs the CPU oracle.

The oracle is apply_rope_in_place (ops/microsoft.rs:137-231), restated in
oracle.c without fused multiply-adds; the kernel rounds every product and sum
the same way, so f32 outputs must match BIT FOR BIT (the reference's own GPU
rotary test allows 1e-5, onnx-rt/tests/test_cuda.rs:2566-2700).  fp16/bf16
inputs are rotated in f32 and rounded once, so they match the oracle applied
to the widened input and rounded to the same type.

Rank-3 inputs (B, S, H*D) follow rotary_gpu's row mapping (token s of row b
at rows (b*S + s)*H + h, onnx-rt/src/cuda/kernels/rotary.rs:54-84), i.e. the
oracle applied to the (B, H, S, D) transpose.
"""
import numpy as np
import pytest
import torch

import oracle
from tests.helpers import rng, rope_tables

pytestmark = pytest.mark.gpu


def _oracle_bhsd(x_bhsd, cos, sin, positions, interleaved, rotary_dim=None):
    return oracle.apply_rope(x_bhsd, cos, sin, positions, interleaved=interleaved, rotary_dim=rotary_dim)


@pytest.mark.parametrize("interleaved", [False, True])
@pytest.mark.parametrize("rank", [3, 4])
def test_start_position_f32_bit_exact(cuda_device, interleaved, rank):
    import smallaios_b200 as sa

    b, h, s, d, start = 3, 8, 5, 128, 17
    r = rng(70 + rank + interleaved)
    x = (r.standard_normal((b, h, s, d)) * 1.28).astype(np.float32)
    cos, sin = rope_tables(64, d, 500000.0)
    cos_t, sin_t = torch.from_numpy(cos).to(cuda_device), torch.from_numpy(sin).to(cuda_device)
    want = _oracle_bhsd(x, cos, sin, np.arange(start, start + s), interleaved)
    if rank == 4:
        xt = torch.from_numpy(x).to(cuda_device)
        got = sa.rotary_embedding(xt, cos_t, sin_t, position=start, interleaved=interleaved).cpu().numpy()
    else:
        xt = torch.from_numpy(np.ascontiguousarray(x.transpose(0, 2, 1, 3)).reshape(b, s, h * d)).to(cuda_device)
        y = sa.rotary_embedding(xt, cos_t, sin_t, position=start, interleaved=interleaved, num_heads=h)
        got = y.cpu().numpy().reshape(b, s, h, d).transpose(0, 2, 1, 3)
    assert np.array_equal(got.view(np.uint32), want.view(np.uint32))


@pytest.mark.parametrize("pos_dtype", [torch.int64, torch.int32])
@pytest.mark.parametrize("per_batch", [False, True])
def test_position_ids_on_device(cuda_device, pos_dtype, per_batch):
    """position_ids of S or B*S entries (rope_position_for, ops/microsoft.rs:112-120), read on the device."""
    import smallaios_b200 as sa

    b, h, s, d = 4, 6, 3, 64
    r = rng(80)
    x = (r.standard_normal((b, h, s, d))).astype(np.float32)
    cos, sin = rope_tables(100, d)
    pos = r.integers(0, 100, size=(b * s) if per_batch else s).astype(np.int64)
    want = _oracle_bhsd(x, cos, sin, pos, False)
    ids = torch.from_numpy(pos).to(pos_dtype).to(cuda_device)
    got = sa.rotary_embedding(torch.from_numpy(x).to(cuda_device), torch.from_numpy(cos).to(cuda_device),
                              torch.from_numpy(sin).to(cuda_device), position_ids=ids).cpu().numpy()
    assert np.array_equal(got.view(np.uint32), want.view(np.uint32))
    assert sa.rotary_device_status(cuda_device) == 0


def test_partial_rotary_dim_in_place_and_out_of_place(cuda_device):
    """rotary_embedding_dim < head_dim: the first rotary_dim elements rotate, the rest pass through."""
    import smallaios_b200 as sa

    b, h, s, d, rd = 2, 4, 7, 128, 64
    r = rng(81)
    x = r.standard_normal((b, h, s, d)).astype(np.float32)
    cos, sin = rope_tables(32, rd)
    want = _oracle_bhsd(x, cos, sin, np.arange(3, 3 + s), True, rotary_dim=rd)
    cos_t, sin_t = torch.from_numpy(cos).to(cuda_device), torch.from_numpy(sin).to(cuda_device)
    xt = torch.from_numpy(x).to(cuda_device)
    got = sa.rotary_embedding(xt, cos_t, sin_t, position=3, interleaved=True, rotary_embedding_dim=rd)
    assert np.array_equal(got.cpu().numpy().view(np.uint32), want.view(np.uint32))
    sa.rotary_embedding(xt, cos_t, sin_t, position=3, interleaved=True, rotary_embedding_dim=rd, out=xt)
    assert np.array_equal(xt.cpu().numpy().view(np.uint32), want.view(np.uint32))


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
def test_half_inputs_and_bf16_tables(cuda_device, dtype):
    """fp16/bf16 activations rotate in f32 and round once; bf16 tables are widened exactly (the GPU
    executor casts bf16 tables to f32 first, gpu_executor.rs:776-792)."""
    import smallaios_b200 as sa

    b, s, h, d = 2, 4, 32, 128
    r = rng(82)
    x = torch.from_numpy((r.standard_normal((b, s, h * d)) * 1.28).astype(np.float32)).to(dtype)
    cos, sin = rope_tables(4096, d, 500000.0)
    cos_b = torch.from_numpy(cos).to(torch.bfloat16)
    sin_b = torch.from_numpy(sin).to(torch.bfloat16)
    xw = x.float().numpy().reshape(b, s, h, d).transpose(0, 2, 1, 3)
    want = _oracle_bhsd(np.ascontiguousarray(xw), cos_b.float().numpy(), sin_b.float().numpy(),
                        np.arange(4000, 4000 + s), False)
    want = torch.from_numpy(np.ascontiguousarray(want.transpose(0, 2, 1, 3)).reshape(b, s, h * d)).to(dtype)
    got = sa.rotary_embedding(x.to(cuda_device), cos_b.to(cuda_device), sin_b.to(cuda_device), position=4000,
                              num_heads=h).cpu()
    assert torch.equal(got.view(torch.int16), want.view(torch.int16))


def test_out_of_table_position_id_flags_device_status(cuda_device):
    """A position id outside the table is a device-side check failure: the row passes through
    unrotated and the status word is set (the reference returns ShapeMismatch from the CPU op)."""
    import smallaios_b200 as sa

    b, h, s, d = 1, 2, 2, 64
    x = torch.randn(b, h, s, d, device=cuda_device)
    cos, sin = rope_tables(8, d)
    ids = torch.tensor([3, 9], dtype=torch.int64, device=cuda_device)
    y = sa.rotary_embedding(x, torch.from_numpy(cos).to(cuda_device), torch.from_numpy(sin).to(cuda_device),
                            position_ids=ids)
    assert sa.rotary_device_status(cuda_device) == 1
    assert sa.rotary_device_status(cuda_device) == 0  # cleared
    assert torch.equal(y[:, :, 1], x[:, :, 1])
    want = _oracle_bhsd(x[:, :, :1].cpu().numpy(), cos, sin, [3], False)
    assert np.array_equal(y[:, :, :1].cpu().numpy(), want)


def test_host_validation_errors(cuda_device):
    import smallaios_b200 as sa

    x = torch.zeros(1, 2, 4, 64, device=cuda_device)
    cos, sin = (torch.from_numpy(t).to(cuda_device) for t in rope_tables(8, 64))
    with pytest.raises(sa.ShapeMismatch, match="exceeds cos/sin table length"):
        sa.rotary_embedding(x, cos, sin, position=5)
    with pytest.raises(sa.ShapeMismatch, match="inner dim"):
        sa.rotary_embedding(x, cos[:, :16].contiguous(), sin[:, :16].contiguous())
    with pytest.raises(sa.InvalidAttribute):
        sa.rotary_embedding(x.reshape(1, 4, 128), cos, sin)
    with pytest.raises(sa.ShapeMismatch, match="position_ids length"):
        sa.rotary_embedding(x, cos, sin, position_ids=torch.zeros(3, dtype=torch.int64, device=cuda_device))


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
def test_graph_with_separate_rotary_nodes(cuda_device, dtype):
    """A decode step the way the gemma builder wires it (gemma.rs:13-36): RotaryEmbedding nodes on
    Q and K at the cache position, then GroupQueryAttention with do_rotary = 0.  Its codes must be
    the encoder's codes of the rotated k it was given (with f32 activations: the fused path's codes,
    bit for bit) and its output within 1e-3 of the composite oracle."""
    import smallaios_b200 as sa
    from tests.helpers import oracle_append, oracle_attend

    b, hq, hkv, d, past = 2, 8, 2, 64, 40
    r = rng(83)
    t = past + 1
    k = torch.from_numpy((r.standard_normal((b, t, hkv * d)) * 1.28).astype(np.float32)).to(dtype)
    v = torch.from_numpy((r.standard_normal((b, t, hkv * d)) * 1.28).astype(np.float32)).to(dtype)
    q = torch.from_numpy((r.standard_normal((b, 1, hq * d)) * 1.28).astype(np.float32)).to(dtype)
    cos, sin = rope_tables(t + 8, d)
    cos_t, sin_t = torch.from_numpy(cos).to(cuda_device), torch.from_numpy(sin).to(cuda_device)
    outs, views = [], []
    for fused in (True, False):
        cache = sa.GpuKvCache(1, hkv, d, t + 8, batch=b, num_heads=hq, bits=4, device=cuda_device)
        ctx = sa.KvCacheDispatchCtx(cache)
        cache.append(0, k[:, :past].to(cuda_device).contiguous(), v[:, :past].to(cuda_device).contiguous(),
                     cos_cache=cos_t, sin_cache=sin_t, do_rotary=True)
        cache.advance_position(past)
        qd, kd, vd = (x.to(cuda_device).contiguous() for x in (q, k[:, past:], v[:, past:]))
        if fused:
            (out,) = sa.dispatch_gpu_node("GroupQueryAttention", [qd, kd, vd, None, None, None, None, cos_t, sin_t],
                                          {"num_heads": hq, "kv_num_heads": hkv, "do_rotary": 1}, ctx)
        else:
            (qr,) = sa.dispatch_gpu_node("RotaryEmbedding", [qd, cos_t, sin_t], {"num_heads": hq}, ctx)
            (kr,) = sa.dispatch_gpu_node("RotaryEmbedding", [kd, cos_t, sin_t], {"num_heads": hkv}, ctx)
            (out,) = sa.dispatch_gpu_node("GroupQueryAttention", [qr, kr, vd],
                                          {"num_heads": hq, "kv_num_heads": hkv, "do_rotary": 0}, ctx)
        sa.finalize_kv_cache(ctx)
        torch.cuda.synchronize()
        view = cache.view(0)
        views.append((view.k_codes[:, :, :t].cpu().numpy(), view.k_meta[:, :, :t].cpu().numpy(),
                      view.v_codes_tokens()[:, :, :t].cpu().numpy(), view.v_meta[:, :, :t].cpu().numpy(),
                      view.signs.cpu().numpy().astype(np.int8)))
        outs.append(out.float().cpu().numpy())
        cache.close()
    kc, km, vc, vm, signs = views[0]
    kf, vf = k.float().numpy().reshape(b, t, hkv, d), v.float().numpy().reshape(b, t, hkv, d)
    okc, okm, ovc, ovm = oracle_append(kf, vf, signs, 4, 0, cos, sin, True, False)
    assert np.array_equal(okc, kc) and np.array_equal(ovc, vc)
    assert np.array_equal(okm.view(np.uint32), km.view(np.uint32))
    # The separate node rounds RoPE(k) to the activation type before the append (as the
    # reference's rotary_bf16 does); the fused append quantizes the f32 rotation.  So the new
    # token's K codes are PolarQuantizer::encode of that rounded vector; everything else matches.
    k_new = oracle.apply_rope(np.ascontiguousarray(kf[:, past:].transpose(0, 2, 1, 3)), cos, sin, [past])
    k_new = torch.from_numpy(k_new).to(dtype).float().numpy()  # (B, H, 1, D)
    ukc, ukm, uvc, uvm, _ = views[1]
    for hh in range(hkv):
        c, m = oracle.polar_encode_many(k_new[:, hh, 0], 4, signs[hh])
        assert np.array_equal(ukc[:, hh, past], c) and np.array_equal(ukm[:, hh, past].view(np.uint32),
                                                                      m.view(np.uint32))
    assert np.array_equal(ukc[:, :, :past], kc[:, :, :past]) and np.array_equal(uvc, vc)
    assert np.array_equal(uvm.view(np.uint32), vm.view(np.uint32))
    qf = q.float().numpy().reshape(b, 1, hq, d)
    want_fused = oracle_attend(qf, kc, km, vc, vm, signs, 4, past, cos=cos, sin=sin, do_rotary=True)
    # the unfused graph rounds the rotated q to the activation type before the attention
    q_rot = oracle.apply_rope(np.ascontiguousarray(qf.transpose(0, 2, 1, 3)), cos, sin, [past])
    q_rot = torch.from_numpy(q_rot).to(dtype).float().numpy().transpose(0, 2, 1, 3)
    want_unfused = oracle_attend(np.ascontiguousarray(q_rot), ukc, ukm, uvc, uvm, signs, 4, past)
    half_ulp = 0.0 if dtype == torch.float32 else 2.0 ** -8
    for got, want in ((outs[0], want_fused), (outs[1], want_unfused)):
        err = np.abs(got - want)
        assert np.all(err <= 1e-3 + half_ulp * np.abs(want)), float(err.max())
