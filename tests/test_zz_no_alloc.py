"""kl_gemm_skinny_noalloc, the skinny GEMM for callers that may not allocate device memory: its
scratch is a fixed array inside libkl_b200.so. Called through the C ABI and compared with the
allocating entry point kl_gemm on the same inputs, two calls in a row (the second one reuses the
array exactly as the first left it). This file is collected last on purpose."""

import ctypes

import numpy as np
import pytest
import torch

import maia_b200 as kl

from gpu_util import random_inputs, to_device
from oracle import gemm as og

pytestmark = pytest.mark.gpu

BF16_TOL = 1e-2


def _noalloc(a, b, c, **kw):
    d = kl.gemm_desc(a, b, c, algo=kl.ALGO_SKINNY, **kw)
    stream = torch.cuda.current_stream(a.device).cuda_stream
    return kl.lib().kl_gemm_skinny_noalloc(ctypes.byref(d), ctypes.c_void_p(stream))


@pytest.mark.parametrize("m, n, k, ctas", [(16, 28672, 8192, 0), (64, 28672, 8192, 0), (40, 3000, 2048, 29),
                                           (5, 136, 200, 0)])
def test_noalloc_matches_kl_gemm_twice(cuda, m, n, k, ctas):
    kl.set_wait_timeout_ns(1_000_000_000)
    a_bits, b_bits, _, _ = random_inputs(m, n, k, "bf16", seed=m + n)
    a = to_device(a_bits, "bf16", cuda)
    b = to_device(b_bits, "bf16", cuda)
    ref = torch.empty((m, n), dtype=torch.bfloat16, device=cuda)
    kl.gemm(a, b, ref, algo=kl.ALGO_SKINNY, max_ctas=ctas)
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


def test_noalloc_rejects_oversized(cuda):
    a = torch.zeros((128, 8192), dtype=torch.bfloat16, device=cuda)
    b = torch.zeros((28672, 8192), dtype=torch.bfloat16, device=cuda)
    c = torch.empty((128, 28672), dtype=torch.bfloat16, device=cuda)
    assert _noalloc(a, b, c) == kl.KL_ERR_INVALID_ARGUMENT
    assert "fixed scratch" in kl.last_error()
