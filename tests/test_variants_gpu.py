"""Tile-kernel variants on the GPU, against the fp64 CPU oracle: f16 and e5m2 inputs, fp8 inputs
with an fp32 C, 64- and 32-byte operand swizzle (multi-box TMA tiles), and reducing stores
(C += A . B^T, split-K over K slices, batched, and on the skinny kernel).

Tolerances as in test_gemm_gpu.py: 1e-2 for 16-bit inputs, 5e-2 for fp8 inputs, normwise and
element-wise with a floor of 1e-2 * rms of the reference.
"""

import numpy as np
import pytest
import torch

import maia_b200 as kl

from gpu_util import FP8_MAX, TORCH_TYPES, check, random_inputs, run_kl, to_device

pytestmark = pytest.mark.gpu

TOL16 = 1e-2
FP8_TOL = 5e-2
ALGOS = pytest.mark.parametrize("algo", [kl.ALGO_1CTA, kl.ALGO_2CTA], ids=["1cta", "2cta"])
SHAPES = [(128, 256, 64), (130, 264, 200), (257, 520, 136), (512, 768, 1024)]


@ALGOS
@pytest.mark.parametrize("out", ["f16", "f32"])
@pytest.mark.parametrize("shape", SHAPES)
def test_f16_inputs(cuda, algo, out, shape):
    m, n, k = shape
    a, b, _, _ = random_inputs(m, n, k, "f16", seed=3 * m + n + k)
    c = run_kl(a, b, "f16", out, cuda, algo)
    check(c, a, b, 1.0, TOL16, kind="f16")


def test_f16_auto_small_m_uses_a_tile_kernel(cuda):
    """No skinny kernel for f16: KL_ALGO_AUTO routes 16 rows to the tile kernel."""
    a, b, _, _ = random_inputs(16, 1024, 512, "f16", seed=5)
    check(run_kl(a, b, "f16", "f16", cuda, kl.ALGO_AUTO), a, b, 1.0, TOL16, kind="f16")


@ALGOS
@pytest.mark.parametrize("dtype,out", [("e5m2", "bf16"), ("e5m2", "f32"), ("e4m3", "f32")])
@pytest.mark.parametrize("shape", [(256, 256, 256), (300, 200, 160), (512, 768, 1024)])
def test_fp8_types(cuda, algo, dtype, out, shape):
    m, n, k = shape
    a, b, sa, sb = random_inputs(m, n, k, dtype, seed=17 + m + k)
    c = run_kl(a, b, dtype, out, cuda, algo, scale_a=sa, scale_b=sb)
    check(c, a, b, sa * sb, FP8_TOL, kind=dtype)


@ALGOS
@pytest.mark.parametrize("swizzle", [64, 32])
@pytest.mark.parametrize("out", ["bf16", "f32"])
@pytest.mark.parametrize("shape", [(128, 256, 64), (130, 264, 200), (257, 520, 72), (512, 512, 1024)])
def test_operand_swizzle(cuda, algo, swizzle, out, shape):
    """Stages of 128 B of K split into 64-B or 32-B swizzle atoms: 2 or 4 TMA boxes per operand
    tile, with the MMA K-slices crossing atom columns. K values that are not multiples of 64
    leave the last boxes partly (or wholly) outside the tensor."""
    m, n, k = shape
    a, b, _, _ = random_inputs(m, n, k, "bf16", seed=swizzle + m + k)
    c = run_kl(a, b, "bf16", out, cuda, algo, swizzle=swizzle)
    check(c, a, b, 1.0, TOL16)


def test_operand_swizzle_matches_default(cuda):
    """Same inputs, same tile order and K order: the 64/32-byte kernels give the 128-byte kernel's
    fp32 result bit for bit."""
    a, b, _, _ = random_inputs(384, 512, 640, "bf16", seed=9)
    ref = run_kl(a, b, "bf16", "f32", cuda, kl.ALGO_2CTA)
    for sw in (64, 32):
        assert np.array_equal(run_kl(a, b, "bf16", "f32", cuda, kl.ALGO_2CTA, swizzle=sw), ref)


def test_operand_swizzle_limits(cuda):
    a = torch.zeros(128, 64, dtype=torch.float16, device=cuda)
    c = torch.zeros(128, 128, dtype=torch.float16, device=cuda)
    with pytest.raises(kl.KlError) as e:
        kl.gemm(a, a[:128], c, algo=kl.ALGO_1CTA, swizzle=64)
    assert e.value.status == kl.KL_ERR_NOT_SUPPORTED
    a = torch.zeros(128, 64, dtype=torch.bfloat16, device=cuda)
    with pytest.raises(kl.KlError) as e:
        kl.gemm(a, a, torch.zeros(128, 128, dtype=torch.bfloat16, device=cuda), swizzle=48)
    assert e.value.status == kl.KL_ERR_INVALID_ARGUMENT


def _c0(m, n, seed):
    rng = np.random.Generator(np.random.PCG64(seed))
    return rng.standard_normal((m, n), dtype=np.float32) * np.float32(4.0)


@pytest.mark.parametrize("algo", [kl.ALGO_1CTA, kl.ALGO_2CTA, kl.ALGO_SKINNY], ids=["1cta", "2cta", "skinny"])
@pytest.mark.parametrize("shape", [(16, 1024, 512), (100, 520, 200), (256, 768, 1024)])
def test_reduce_add_into_c(cuda, algo, shape):
    """C += A . B^T: TMA reducing stores (tile kernels) or the owning thread's read-modify-write
    (skinny kernel) on an fp32 C that already holds values."""
    m, n, k = shape
    if algo == kl.ALGO_SKINNY and m > 256:
        pytest.skip("skinny kernel: at most 256 rows")
    a, b, _, _ = random_inputs(m, n, k, "bf16", seed=m + 2 * n + k)
    c0 = _c0(m, n, seed=m)
    c = torch.from_numpy(c0).to(cuda)
    kl.gemm(to_device(a, "bf16", cuda), to_device(b, "bf16", cuda), c, algo=algo, accumulate=True)
    torch.cuda.synchronize()
    assert kl.read_status() == 0
    check(c.cpu().numpy(), a, b, 1.0, TOL16, c0=c0)


@pytest.mark.parametrize("algo", [kl.ALGO_1CTA, kl.ALGO_2CTA, kl.ALGO_SKINNY], ids=["1cta", "2cta", "skinny"])
def test_split_k_by_reducing_stores(cuda, algo):
    """Four calls over K slices, each adding into one zeroed fp32 C, equal the one-call GEMM."""
    m, n, k = (64, 2048, 2048) if algo == kl.ALGO_SKINNY else (512, 1024, 2048)
    a, b, _, _ = random_inputs(m, n, k, "bf16", seed=21)
    da, db = to_device(a, "bf16", cuda), to_device(b, "bf16", cuda)
    c = torch.zeros(m, n, dtype=torch.float32, device=cuda)
    ks = k // 4
    for s in range(4):
        kl.gemm(da[:, s * ks:(s + 1) * ks], db[:, s * ks:(s + 1) * ks], c, algo=algo, accumulate=True)
    torch.cuda.synchronize()
    assert kl.read_status() == 0
    check(c.cpu().numpy(), a, b, 1.0, TOL16)


def test_reduce_add_batched(cuda):
    L, m, n, k = 3, 256, 384, 320
    rng = np.random.Generator(np.random.PCG64(4))
    a = [random_inputs(m, n, k, "bf16", seed=40 + i) for i in range(L)]
    da = torch.stack([to_device(x[0], "bf16", cuda) for x in a])
    db = torch.stack([to_device(x[1], "bf16", cuda) for x in a])
    c0 = rng.standard_normal((L, m, n), dtype=np.float32)
    c = torch.from_numpy(c0).to(cuda)
    kl.gemm(da, db, c, algo=kl.ALGO_2CTA, accumulate=True)
    torch.cuda.synchronize()
    assert kl.read_status() == 0
    out = c.cpu().numpy()
    for i in range(L):
        check(out[i], a[i][0], a[i][1], 1.0, TOL16, c0=c0[i])


def test_reduce_add_fp8_scaled(cuda):
    m, n, k = 256, 512, 512
    a, b, sa, sb = random_inputs(m, n, k, "e4m3", seed=77)
    c0 = _c0(m, n, seed=78)
    c = torch.from_numpy(c0).to(cuda)
    dsa = torch.tensor([sa], dtype=torch.float32, device=cuda)
    dsb = torch.tensor([sb], dtype=torch.float32, device=cuda)
    kl.gemm(to_device(a, "e4m3", cuda), to_device(b, "e4m3", cuda), c, scale_a=dsa, scale_b=dsb,
            algo=kl.ALGO_2CTA, accumulate=True)
    torch.cuda.synchronize()
    assert kl.read_status() == 0
    check(c.cpu().numpy(), a, b, sa * sb, FP8_TOL, c0=c0)


def test_reduce_add_k_zero_leaves_c(cuda):
    c = torch.arange(64 * 32, dtype=torch.float32, device=cuda).reshape(64, 32)
    before = c.clone()
    a = torch.zeros(64, 0, dtype=torch.bfloat16, device=cuda)
    b = torch.zeros(32, 0, dtype=torch.bfloat16, device=cuda)
    d = kl.gemm_desc(a, b, c, c_reduce=1)
    kl.check(kl.lib().kl_gemm(kl.ctypes.byref(d), kl.ctypes.c_void_p(0)))
    torch.cuda.synchronize()
    assert torch.equal(c, before)


@pytest.mark.parametrize("algo", [kl.ALGO_1CTA, kl.ALGO_2CTA, kl.ALGO_SKINNY], ids=["1cta", "2cta", "skinny"])
@pytest.mark.parametrize("out", ["bf16", "f16"])
@pytest.mark.parametrize("shape", [(16, 1024, 512), (100, 520, 200), (256, 776, 1024)])
def test_reduce_add_into_16bit_c(cuda, algo, out, shape):
    """C += A . B^T on a bf16 / f16 C (a residual add): the epilogue reads C, adds in fp32 and the
    sum is rounded once; ragged right edges (N not a multiple of 64) included."""
    m, n, k = shape
    if algo == kl.ALGO_SKINNY and out == "f16":
        pytest.skip("the skinny kernel writes bf16 or f32 C")
    dtype = "bf16" if out == "bf16" or algo == kl.ALGO_SKINNY else "f16"
    a, b, _, _ = random_inputs(m, n, k, dtype, seed=m + n + 2 * k)
    tdt = torch.bfloat16 if out == "bf16" else torch.float16
    c = (torch.randn(m, n, generator=torch.Generator().manual_seed(m)) * 4).to(tdt)
    c0 = c.float().numpy().astype(np.float64)
    c = c.to(cuda)
    kl.gemm(to_device(a, dtype, cuda), to_device(b, dtype, cuda), c, algo=algo, accumulate=True)
    torch.cuda.synchronize()
    assert kl.read_status() == 0
    check(c.float().cpu().numpy(), a, b, 1.0, TOL16, kind=dtype, c0=c0)


def test_reduce_add_needs_out(cuda):
    a = torch.zeros(256, 64, dtype=torch.bfloat16, device=cuda)
    with pytest.raises(ValueError):
        kl.gemm(a, a, accumulate=True)

