"""GEMM parity on the GPU: libkl_b200.so through its C ABI against the fp64 CPU oracle.

Tolerances, against fp64 accumulation of the same rounded inputs: 1e-2 for bf16 inputs, 5e-2 for
e4m3 inputs, applied to both the normwise max relative error max|c - r| / max|r| and the
element-wise |c - r| / max(|r|, 1e-2 * rms(r)).
"""

import numpy as np
import pytest

import maia_b200 as kl
from maia_b200 import workloads as wl

from gpu_util import check, random_inputs, run_kl

pytestmark = pytest.mark.gpu

BF16_TOL = 1e-2
FP8_TOL = 5e-2


@pytest.mark.parametrize("algo", [kl.ALGO_1CTA, kl.ALGO_2CTA], ids=["1cta", "2cta"])
def test_c1_256_bf16_f32(cuda, algo):
    a, b, _, _ = wl.make_inputs(wl.C1)
    c = run_kl(a, b, "bf16", "f32", cuda, algo)
    _, norm = check(c, a, b, 1.0, BF16_TOL)
    assert norm < 1e-5  # fp32 output: only accumulation-order differences remain


@pytest.mark.parametrize("algo", [kl.ALGO_1CTA, kl.ALGO_2CTA], ids=["1cta", "2cta"])
def test_c2_4096_bf16(cuda, algo):
    a, b, _, _ = wl.make_inputs(wl.C2)
    c = run_kl(a, b, "bf16", "bf16", cuda, algo)
    check(c, a, b, 1.0, BF16_TOL)


RAGGED = [(1, 8, 8), (8, 16, 64), (130, 264, 200), (200, 136, 72), (257, 520, 136), (384, 512, 1024), (1000, 1000, 1000)]


@pytest.mark.parametrize("algo", [kl.ALGO_1CTA, kl.ALGO_2CTA], ids=["1cta", "2cta"])
@pytest.mark.parametrize("shape", RAGGED)
def test_ragged_bf16(cuda, algo, shape):
    m, n, k = shape
    a, b, _, _ = random_inputs(m, n, k, "bf16", seed=m * 7 + n * 3 + k)
    check(run_kl(a, b, "bf16", "bf16", cuda, algo), a, b, 1.0, BF16_TOL)
    check(run_kl(a, b, "bf16", "f32", cuda, algo), a, b, 1.0, BF16_TOL)


@pytest.mark.parametrize("algo", [kl.ALGO_1CTA, kl.ALGO_2CTA], ids=["1cta", "2cta"])
@pytest.mark.parametrize("shape", [(256, 256, 256), (512, 768, 1024), (300, 200, 160)])
def test_e4m3_scaled(cuda, algo, shape):
    m, n, k = shape
    a, b, sa, sb = random_inputs(m, n, k, "e4m3", seed=11 + m)
    c = run_kl(a, b, "e4m3", "bf16", cuda, algo, scale_a=sa, scale_b=sb)
    check(c, a, b, sa * sb, FP8_TOL)


@pytest.mark.parametrize("algo", [kl.ALGO_1CTA, kl.ALGO_2CTA], ids=["1cta", "2cta"])
def test_persistent_few_ctas(cuda, algo):
    """More tiles than CTAs: every CTA loops over several tiles and both TMEM accumulators."""
    a, b, _, _ = random_inputs(1024, 2048, 512, "bf16", seed=5)
    c = run_kl(a, b, "bf16", "bf16", cuda, algo, max_ctas=6, group_m=3)
    check(c, a, b, 1.0, BF16_TOL)


@pytest.mark.parametrize("algo", [kl.ALGO_1CTA, kl.ALGO_2CTA], ids=["1cta", "2cta"])
@pytest.mark.parametrize("prefetch", [3, 16])
def test_l2_prefetch_keeps_results(cuda, algo, prefetch):
    """L2 prefetch ahead of the loads (across tile boundaries too) changes no result."""
    a, b, _, _ = random_inputs(640, 768, 1216, "bf16", seed=prefetch)
    check(run_kl(a, b, "bf16", "bf16", cuda, algo, max_ctas=10, prefetch=prefetch), a, b, 1.0, BF16_TOL)


def test_strided_operands(cuda):
    """Leading dimensions larger than the extents (padded rows) on A, B and C."""
    import torch

    m, n, k = 384, 256, 320
    a_bits, b_bits, _, _ = random_inputs(m, n, k, "bf16", seed=9)
    from gpu_util import to_device

    a_full = torch.zeros((m, k + 64), dtype=torch.bfloat16, device=cuda)
    b_full = torch.zeros((n, k + 32), dtype=torch.bfloat16, device=cuda)
    a_full[:, :k] = to_device(a_bits, "bf16", cuda)
    b_full[:, :k] = to_device(b_bits, "bf16", cuda)
    c_full = torch.full((m, n + 24), 7.0, dtype=torch.bfloat16, device=cuda)
    kl.gemm(a_full[:, :k], b_full[:, :k], c_full[:, :n], algo=kl.ALGO_1CTA)
    torch.cuda.synchronize()
    assert (c_full[:, n:] == 7.0).all(), "wrote outside C's columns"
    check(c_full[:, :n].float().cpu().numpy(), a_bits, b_bits, 1.0, BF16_TOL)


def test_k_zero_gives_zeros(cuda):
    import torch

    a = torch.zeros((64, 0), dtype=torch.bfloat16, device=cuda)
    b = torch.zeros((32, 0), dtype=torch.bfloat16, device=cuda)
    c = torch.full((64, 32), 3.0, dtype=torch.bfloat16, device=cuda)
    d = kl.GemmDesc(m=64, n=32, k=0, a=0, lda=8, b=0, ldb=8, c=c.data_ptr(), ldc=32, ab_type=kl.KL_BF16,
                    c_type=kl.KL_BF16, alpha=1.0)
    import ctypes

    kl.check(kl.lib().kl_gemm(ctypes.byref(d), None))
    torch.cuda.synchronize()
    assert (c == 0).all()


def test_bad_alignment_is_an_error(cuda):
    import torch

    a = torch.zeros((64, 72), dtype=torch.bfloat16, device=cuda)
    b = torch.zeros((64, 64), dtype=torch.bfloat16, device=cuda)
    c = torch.zeros((64, 64), dtype=torch.bfloat16, device=cuda)
    with pytest.raises(kl.KlError) as e:
        kl.gemm(a[:, 1:65], b, c)  # A starts 2 bytes past a 16-byte boundary
    assert e.value.status == kl.KL_ERR_INVALID_ARGUMENT
    assert "16-byte aligned" in e.value.message


def test_wait_timeout_reports_instead_of_hanging(cuda):
    """A wait nobody satisfies gives up after its bound and the context stays usable."""
    import torch

    kl.read_status(clear=True)
    kl.probe_wait_timeout(2_000_000)  # 2 ms
    bits = kl.read_status(clear=True)
    assert bits & 16
    a, b, _, _ = random_inputs(128, 256, 64, "bf16", seed=1)
    check(run_kl(a, b, "bf16", "bf16", cuda, kl.ALGO_1CTA), a, b, 1.0, BF16_TOL)


def _sample_indices(n, tile, rng, extra=24):
    """Rows (or columns) at every kind of boundary the kernels have, plus random ones."""
    picks = {0, 1, 31, 32, 127, 128, 255, 256, 511, 512, n // 2 - 1, n // 2, n - 257, n - 256, n - 129, n - 128,
             n - 1}
    picks.update(int(x) for x in rng.integers(0, n, extra))
    return np.array(sorted(p for p in picks if 0 <= p < n))


@pytest.mark.parametrize("name, algo", [("c3_8192_bf16", kl.ALGO_2CTA), ("c3_8192_bf16", kl.ALGO_1CTA),
                                        ("c4_16384x16384x8192_e4m3", kl.ALGO_2CTA)],
                         ids=["c3-2cta", "c3-1cta", "c4-fp8-2cta"])
def test_full_size_sampled_rows_and_columns(cuda, name, algo):
    """The benchmark-size GEMMs, checked on whole rows and whole columns of C that cross every tile,
    CTA-pair and raster-group boundary, plus random ones (the fp64 oracle on all 5e11+ entries
    would take hours on the host)."""
    w = wl.ALL[name]
    a, b, sa, sb = wl.make_inputs(w)
    c = run_kl(a, b, w.dtype, w.out, cuda, algo, scale_a=sa, scale_b=sb)
    rng = np.random.default_rng(7)
    rows = _sample_indices(w.m, 256, rng)
    cols = _sample_indices(w.n, 256, rng)
    tol = BF16_TOL if w.dtype == "bf16" else FP8_TOL
    check(c[rows, :], a[rows], b, sa * sb, tol)
    check(c[:, cols], a, b[cols], sa * sb, tol)


def test_clock_probe_reports_the_kernel_clock(cuda):
    """kl_gemm_clock_probe: every CTA stamps clock64/%globaltimer; the ratio is a plausible SM clock."""
    import torch

    a_bits, b_bits, _, _ = random_inputs(2048, 2048, 2048, "bf16", seed=2)
    from gpu_util import to_device

    a, b = to_device(a_bits, "bf16", cuda), to_device(b_bits, "bf16", cuda)
    c = torch.empty((2048, 2048), dtype=torch.bfloat16, device=cuda)
    r = kl.clock_probe(a, b, c, algo=kl.ALGO_2CTA)
    assert r["ctas"] == 2 * (r["ctas"] // 2) > 0
    assert 300 < r["sm_mhz_min"] <= r["sm_mhz_max"] < 2500
    check(c.float().cpu().numpy(), a_bits, b_bits, 1.0, BF16_TOL)
