"""kl_gemm_skinny_noalloc, the skinny GEMM for callers that may not allocate device memory: its
scratch is a fixed array inside libkl_b200.so. Called through the C ABI and compared with the
allocating entry point kl_gemm on the same inputs (bit for bit: same kernel, same reduction
order) and with the fp64 oracle (bf16 1e-2, e4m3 5e-2), two calls in a row (the second one reuses
the array exactly as the first left it). This file is collected last on purpose.

The argument checks at the top run without a GPU: they are rejected before anything touches the
device or queues work on a stream."""

import ctypes

import numpy as np
import pytest
import torch

import maia_b200 as kl

from gpu_util import random_inputs, to_device
from oracle import gemm as og

BF16_TOL = 1e-2
FP8_TOL = 5e-2


def _noalloc(a, b, c, **kw):
    d = kl.gemm_desc(a, b, c, algo=kl.ALGO_SKINNY, **kw)
    stream = torch.cuda.current_stream(a.device).cuda_stream
    return kl.lib().kl_gemm_skinny_noalloc(ctypes.byref(d), ctypes.c_void_p(stream))


def _cpu_desc(**over):
    """A descriptor with made-up (never dereferenced) pointers, for the argument checks."""
    d = kl.GemmDesc(m=16, n=256, k=256, a=0x10000, lda=256, b=0x20000, ldb=256, c=0x30000, ldc=256,
                    ab_type=kl.KL_BF16, c_type=kl.KL_BF16, alpha=1.0, algo=kl.ALGO_SKINNY)
    for k, v in over.items():
        setattr(d, k, v)
    return d


@pytest.mark.parametrize("over, code, text", [
    (dict(c=0x30001), kl.KL_ERR_INVALID_ARGUMENT, "aligned"),                      # bf16 C at an odd address
    (dict(c=0x30002, c_type=kl.KL_F32), kl.KL_ERR_INVALID_ARGUMENT, "aligned"),    # f32 C not 4-byte aligned
    (dict(variant=2), kl.KL_ERR_NOT_SUPPORTED, "variant"),
    (dict(ab_type=kl.KL_E5M2), kl.KL_ERR_NOT_SUPPORTED, "supports"),
    (dict(m=300), kl.KL_ERR_INVALID_ARGUMENT, "256 rows"),
    (dict(algo=kl.ALGO_2CTA), kl.KL_ERR_INVALID_ARGUMENT, "skinny kernel only"),
])
def test_noalloc_rejects_before_touching_the_device(over, code, text):
    d = _cpu_desc(**over)
    assert kl.lib().kl_gemm_skinny_noalloc(ctypes.byref(d), None) == code
    assert text in kl.last_error()


@pytest.mark.gpu
@pytest.mark.parametrize("m, n, k, ctas", [(16, 28672, 8192, 0), (64, 28672, 8192, 0), (40, 3000, 2048, 29),
                                           (5, 136, 200, 0)])
def test_noalloc_matches_kl_gemm_twice(cuda, m, n, k, ctas):
    kl.set_wait_timeout_ns(1_000_000_000)
    a_bits, b_bits, _, _ = random_inputs(m, n, k, "bf16", seed=m + n)
    a = to_device(a_bits, "bf16", cuda)
    b = to_device(b_bits, "bf16", cuda)
    ref = torch.empty((m, n), dtype=torch.bfloat16, device=cuda)
    kl.gemm(a, b, ref, algo=kl.ALGO_SKINNY, max_ctas=ctas)
    want = og.gemm_f64(a_bits, b_bits) if m * n * k <= 16 * 28672 * 8192 else None
    for _ in range(2):
        c = torch.full((m, n), float("nan"), dtype=torch.bfloat16, device=cuda)
        assert _noalloc(a, b, c, max_ctas=ctas) == kl.KL_OK, kl.last_error()
        torch.cuda.synchronize()
        assert kl.read_status() == 0
        got = c.float().cpu().numpy()
        assert not np.isnan(got).any()
        elem, norm = og.rel_error(got, ref.float().cpu().numpy())
        assert norm <= BF16_TOL and elem <= BF16_TOL, (elem, norm)
        # Same kernel, same reduction order: the two entry points agree bit for bit.
        assert torch.equal(c.view(torch.int16), ref.view(torch.int16))
        if want is not None:
            elem, norm = og.rel_error(got, want)
            assert norm <= BF16_TOL and elem <= BF16_TOL, ("vs fp64 oracle", elem, norm)


@pytest.mark.gpu
@pytest.mark.parametrize("ab, out, c_reduce, shape", [
    ("bf16", "f32", 0, (24, 5000, 3072)),
    ("e4m3", "bf16", 0, (16, 28672, 8192)),
    ("bf16", "bf16", 1, (48, 2000, 1536)),
    ("bf16", "f32", 1, (7, 1100, 640)),
])
def test_noalloc_types_and_accumulate_vs_oracle(cuda, ab, out, c_reduce, shape):
    """The (bf16, f32) and (e4m3, bf16) dispatch arms and C += result, each against the fp64 oracle
    and bit for bit against kl_gemm, two calls in a row."""
    m, n, k = shape
    kl.set_wait_timeout_ns(1_000_000_000)
    a_bits, b_bits, sa, sb = random_inputs(m, n, k, ab, seed=3 * m + n + c_reduce)
    a = to_device(a_bits, ab, cuda)
    b = to_device(b_bits, ab, cuda)
    odt = torch.float32 if out == "f32" else torch.bfloat16
    scales = {}
    if ab == "e4m3":
        scales = dict(scale_a=torch.tensor([sa], dtype=torch.float32, device=cuda),
                      scale_b=torch.tensor([sb], dtype=torch.float32, device=cuda))
    g = torch.Generator().manual_seed(m + n)
    c0 = (torch.randn((m, n), generator=g) if c_reduce else torch.full((m, n), float("nan"))).to(odt).to(cuda)
    ref = c0.clone()
    kl.gemm(a, b, ref, algo=kl.ALGO_SKINNY, accumulate=bool(c_reduce), **scales)
    want = og.gemm_f64(a_bits, b_bits, sa * sb)
    if c_reduce:
        want = want + c0.float().cpu().numpy().astype(np.float64)
    tol = FP8_TOL if ab == "e4m3" else BF16_TOL
    for _ in range(2):
        c = c0.clone()
        assert _noalloc(a, b, c, c_reduce=c_reduce, **scales) == kl.KL_OK, kl.last_error()
        torch.cuda.synchronize()
        assert kl.read_status() == 0
        got = c.float().cpu().numpy()
        assert not np.isnan(got).any()
        elem, norm = og.rel_error(got, want)
        assert norm <= tol and elem <= tol, (elem, norm)
        bits = torch.int32 if out == "f32" else torch.int16
        assert torch.equal(c.view(bits), ref.view(bits))


@pytest.mark.gpu
def test_noalloc_rejects_oversized(cuda):
    a = torch.zeros((128, 8192), dtype=torch.bfloat16, device=cuda)
    b = torch.zeros((28672, 8192), dtype=torch.bfloat16, device=cuda)
    c = torch.empty((128, 28672), dtype=torch.bfloat16, device=cuda)
    assert _noalloc(a, b, c) == kl.KL_ERR_INVALID_ARGUMENT
    assert "fixed scratch" in kl.last_error()
