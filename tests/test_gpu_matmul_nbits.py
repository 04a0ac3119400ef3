"""MatMulNBits on the GPU vs the oracle (dequantize in f32 + gemm_f32).

Parity is unpinned (the reference has no MatMulNBits): the oracle restates the
ORT contract on the reference's own f32 GEMM.  Bar: max-abs 1e-3 with f32
activations; fp16/bf16 outputs add half an ulp of the output dtype.
"""
import numpy as np
import pytest
import torch

import oracle
from tests.helpers import rng

pytestmark = pytest.mark.gpu


def _case(m, n, k, block=32, zp=False, bias=False, seed=0, adtype=torch.float32):
    r = rng(seed)
    nblk = k // block
    codes = r.integers(0, 256, size=(n, nblk, block // 2), dtype=np.uint8)
    scales = r.uniform(0.005, 0.02, size=(n, nblk)).astype(np.float16).astype(np.float32)
    a = r.standard_normal((m, k)).astype(np.float32)
    a = torch.from_numpy(a).to(adtype).float().numpy()
    if adtype != torch.float32:
        scales = torch.from_numpy(scales).to(adtype).float().numpy()
    zps = r.integers(0, 256, size=(n, (nblk + 1) // 2), dtype=np.uint8) if zp else None
    bvec = r.standard_normal(n).astype(np.float32) if bias else None
    if bvec is not None:
        bvec = torch.from_numpy(bvec).to(adtype).float().numpy()
    want = oracle.matmul_nbits(a, codes, scales, zps, n=n, k=k, block_size=block)
    if bvec is not None:
        want = want + bvec[None, :]
    return a, codes, scales, zps, bvec, want


def _run(dev, m, n, k, adtype=torch.float32, **kw):
    import smallaios_b200 as sa

    a, codes, scales, zps, bvec, want = _case(m, n, k, adtype=adtype, **kw)
    t = lambda x, dt: None if x is None else torch.from_numpy(x).to(dt).to(dev)
    y = sa.matmul_nbits(t(a, adtype), t(codes, torch.uint8), t(scales, adtype), t(zps, torch.uint8),
                        t(bvec, adtype), K=k, N=n, block_size=kw.get("block", 32))
    torch.cuda.synchronize()
    got = y.float().cpu().numpy()
    if adtype == torch.float32:
        bound = 1e-3
    else:
        ulp = 2.0 ** -8 if adtype == torch.bfloat16 else 2.0 ** -11
        bound = 1e-3 + np.abs(want) * ulp
    err = np.abs(got - want)
    assert np.all(err <= bound), f"max err {err.max():.3e}"


@pytest.mark.parametrize("m", [1, 3, 8, 13])
def test_gemv_f32(cuda_device, m):
    _run(cuda_device, m, 384, 1024, seed=m)


def test_c2_shape_m1_fp16(cuda_device):
    """BASELINE config 2 decode shape: K=4096, N=14336, block 32, zp 8, fp16."""
    _run(cuda_device, 1, 14336, 4096, adtype=torch.float16, seed=21)


def test_c2_shape_m64_fp16(cuda_device):
    _run(cuda_device, 64, 14336, 4096, adtype=torch.float16, seed=22)


@pytest.mark.parametrize("block", [16, 32, 64, 128])
def test_block_sizes_zero_points_bias(cuda_device, block):
    _run(cuda_device, 2, 200, 512, block=block, zp=True, bias=True, seed=block)


@pytest.mark.parametrize("m", [1, 2, 3, 4, 5, 8, 9, 16, 23, 33, 64])
@pytest.mark.parametrize("adtype", [torch.float16, torch.bfloat16])
def test_tensor_core_path(cuda_device, m, adtype):
    """The mma.sync paths (fp16/bf16, block 32, default zero point, K % 1024 == 0, m <= 64: the decode GEMV for
    m = 1, the K-split kernel above it; N = 448 is not a multiple of 128, so the tcgen05 path does not take it)."""
    _run(cuda_device, m, 448, 2048, adtype=adtype, bias=True, seed=100 + m)


@pytest.mark.parametrize("m", [24, 64])
def test_tensor_core_path_narrow_n(cuda_device, m):
    """N a multiple of 16 but not of 64: the per-warp kernel instead of the CTA-shared one."""
    _run(cuda_device, m, 272, 1024, adtype=torch.float16, bias=True, seed=200 + m)


@pytest.mark.parametrize("m", [1, 3, 8])
@pytest.mark.parametrize("adtype", [torch.float16, torch.bfloat16])
def test_packed_weights(cuda_device, m, adtype):
    """Prepacked weights (decode GEMV path): same results as the oracle."""
    import smallaios_b200 as sa

    n, k = 1024, 2048
    a, codes, scales, zps, bvec, want = _case(m, n, k, adtype=adtype, bias=True, seed=300 + m)
    t = lambda x, dt: torch.from_numpy(x).to(dt).to(cuda_device)
    w = sa.PackedNBitsWeight(t(codes, torch.uint8), t(scales, adtype), K=k, N=n)
    y = sa.matmul_nbits_packed(t(a, adtype), w, t(bvec, adtype))
    torch.cuda.synchronize()
    got = y.float().cpu().numpy()
    ulp = 2.0 ** -8 if adtype == torch.bfloat16 else 2.0 ** -11
    err = np.abs(got - want)
    assert np.all(err <= 1e-3 + np.abs(want) * ulp), f"max err {err.max():.3e}"


def test_packed_weights_rejects_unsupported(cuda_device):
    import smallaios_b200 as sa

    b = torch.zeros(48, 1024 // 2, dtype=torch.uint8, device=cuda_device)  # N = 48: not a multiple of 32
    s = torch.zeros(48, 32, dtype=torch.float16, device=cuda_device)
    with pytest.raises(sa.UnsupportedOp):
        sa.PackedNBitsWeight(b, s, K=1024, N=48)


def test_bf16(cuda_device):
    _run(cuda_device, 4, 256, 2048, adtype=torch.bfloat16, seed=5)


def test_errors(cuda_device):
    import smallaios_b200 as sa

    dev = cuda_device
    a = torch.zeros(1, 64, device=dev)
    b = torch.zeros(8, 2, 16, dtype=torch.uint8, device=dev)
    s = torch.zeros(8, 2, device=dev)
    with pytest.raises(sa.UnsupportedOp):
        sa.matmul_nbits(a, b, s, K=64, N=8, bits=3)
    with pytest.raises(sa.ShapeMismatch):
        sa.matmul_nbits(a, b, s, K=32, N=8)


@pytest.mark.parametrize("m", [17, 31, 32, 40, 64, 100, 128])
@pytest.mark.parametrize("adtype", [torch.float16, torch.bfloat16])
def test_tcgen05_path(cuda_device, m, adtype):
    """The tcgen05 path (N % 128 == 0, K % 256 == 0, 17 <= m <= 128): split-scale exact weights, f32 accumulation.
    K = 1280 is 5 stages of 256 and 20 TMEM buffer uses: both rings wrap."""
    _run(cuda_device, m, 384, 1280, adtype=adtype, bias=(m % 2 == 1), seed=300 + m)


def test_tcgen05_path_c2_shape_bf16(cuda_device):
    """BASELINE config 2 width (N=14336, K=4096) with bf16 activations and scales at m = 64."""
    _run(cuda_device, 64, 14336, 4096, adtype=torch.bfloat16, seed=42)


def test_c2_shape_m128_fp16(cuda_device):
    """128 activation rows (a prefill chunk) on the tcgen05 path."""
    _run(cuda_device, 128, 14336, 4096, adtype=torch.float16, seed=43)


@pytest.mark.parametrize("m", [129, 200, 520])
def test_tcgen05_row_blocks(cuda_device, m):
    """More than 128 rows (prefill): blocks of 128 activation rows, the last one ragged."""
    _run(cuda_device, m, 1024, 2048, adtype=torch.bfloat16, bias=True, seed=500 + m)


@pytest.mark.parametrize("m", [1, 4])
@pytest.mark.parametrize("adtype", [torch.float16, torch.bfloat16])
def test_decode_gemv_c2_shape(cuda_device, m, adtype):
    """m = 1 (the decode GEMV kernel) and m = 4 (the K-split kernel) at config 2's K=4096, N=14336, and at
    K=14336 (a down projection)."""
    _run(cuda_device, m, 14336, 4096, adtype=adtype, bias=True, seed=300 + m)
    _run(cuda_device, m, 4096, 14336, adtype=adtype, seed=310 + m)


@pytest.mark.parametrize("n,k", [(2400, 768), (7104, 256), (47360, 512), (16, 256), (28672, 4096)])
def test_m1_shapes(cuda_device, n, k):
    """m = 1 at widths and depths the decode GEMV does not take (K not a multiple of 1024, N not a
    multiple of 32: the K-split kernel) and at the fused gate|up width (28672 x 4096, the GEMV)."""
    _run(cuda_device, 1, n, k, adtype=torch.float16, bias=True, seed=n + k)
    _run(cuda_device, 1, n, k, adtype=torch.bfloat16, seed=n + k + 1)
