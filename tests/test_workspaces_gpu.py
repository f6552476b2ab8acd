"""kl_release_workspaces on the GPU: the library-owned workspaces (the skinny kernel's per-device
buffer, the tile kernels' per-stream split-tail buffers) are freed, and the next calls allocate
afresh and give the same bits as before the release; kl_gemm_skinny_noalloc looks its array's
address up again after the release."""

import ctypes

import pytest
import torch

import maia_b200 as kl

from gpu_util import check, random_inputs, to_device

pytestmark = pytest.mark.gpu

TOL16 = 1e-2


def _calls(cuda):
    a1, b1, _, _ = random_inputs(48, 3000, 2048, "bf16", seed=11)   # skinny, tiles split across CTAs
    a2, b2, _, _ = random_inputs(1024, 1024, 8192, "bf16", seed=12)  # CTA pair, forced split tail
    ta1, tb1 = to_device(a1, "bf16", cuda), to_device(b1, "bf16", cuda)
    ta2, tb2 = to_device(a2, "bf16", cuda), to_device(b2, "bf16", cuda)

    def run():
        c1 = kl.gemm(ta1, tb1, algo=kl.ALGO_SKINNY, max_ctas=29)
        c2 = kl.gemm(ta2, tb2, out_dtype=torch.float32, algo=kl.ALGO_2CTA, stream_k=1, max_ctas=20)
        c3 = torch.empty((48, 3000), dtype=torch.bfloat16, device=cuda)
        d = kl.gemm_desc(ta1, tb1, c3, algo=kl.ALGO_SKINNY, max_ctas=29)
        kl.check(kl.lib().kl_gemm_skinny_noalloc(ctypes.byref(d),
                                                 ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)))
        torch.cuda.synchronize()
        assert kl.read_status() == 0
        return c1, c2, c3

    return (a1, b1, a2, b2), run


def test_release_then_reuse_gives_the_same_bits(cuda):
    (a1, b1, a2, b2), run = _calls(cuda)
    before = run()
    check(before[0].float().cpu().numpy(), a1, b1, 1.0, TOL16)
    check(before[1].cpu().numpy(), a2, b2, 1.0, TOL16)
    for _ in range(2):
        kl.release_workspaces()
        after = run()
        for x, y in zip(before, after):
            bits = torch.int32 if x.dtype == torch.float32 else torch.int16
            assert torch.equal(x.view(bits), y.view(bits))
    # A second release with the buffers just re-allocated, then one with nothing allocated.
    kl.release_workspaces()
    kl.release_workspaces()
