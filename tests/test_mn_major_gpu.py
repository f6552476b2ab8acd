"""MN-major operands: A stored [K, M] (M contiguous) and/or B stored [K, N], read through MN-major
TMA boxes and MN-major UMMA descriptors (instruction-descriptor major bits), against the fp64
oracle on the same values."""

import numpy as np
import pytest
import torch

import maia_b200 as kl

from gpu_util import check, random_inputs, to_device

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("algo", [kl.ALGO_1CTA, kl.ALGO_2CTA], ids=["1cta", "2cta"])
@pytest.mark.parametrize("majors", [(1, 0), (0, 1), (1, 1)], ids=["A_mn", "B_mn", "AB_mn"])
@pytest.mark.parametrize("m, n, k", [(256, 256, 128), (384, 512, 640), (200, 136, 72), (1024, 768, 1000)])
def test_mn_major(cuda, algo, majors, m, n, k):
    am, bm = majors
    a_bits, b_bits, _, _ = random_inputs(m, n, k, "bf16", seed=m + 2 * n + 3 * k + 5 * am + 7 * bm)
    a_store = np.ascontiguousarray(a_bits.T) if am else a_bits  # [K, M] when MN-major
    b_store = np.ascontiguousarray(b_bits.T) if bm else b_bits
    # MN-major rows need a 16-byte pitch: pad the stored matrix's rows to a multiple of 8 elements.
    def dev(x):
        rows, cols = x.shape
        pitch = (cols + 7) // 8 * 8
        buf = torch.zeros((rows, pitch), dtype=torch.bfloat16, device=cuda)
        buf[:, :cols] = to_device(x, "bf16", cuda)
        return buf[:, :cols]
    a = dev(a_store)
    b = dev(b_store)
    c = torch.full((m, n), float("nan"), dtype=torch.bfloat16, device=cuda)
    kl.gemm(a, b, c, algo=algo, a_major=am, b_major=bm)
    torch.cuda.synchronize()
    assert kl.read_status() == 0
    check(c.float().cpu().numpy(), a_bits, b_bits, 1.0, 1e-2)


def test_mn_major_batched(cuda):
    L, m, n, k = 3, 256, 384, 256
    parts = [random_inputs(m, n, k, "bf16", seed=40 + i) for i in range(L)]
    a = torch.stack([to_device(np.ascontiguousarray(p[0].T), "bf16", cuda) for p in parts])  # [L, K, M]
    b = torch.stack([to_device(p[1], "bf16", cuda) for p in parts])                         # [L, N, K]
    c = torch.full((L, m, n), float("nan"), dtype=torch.bfloat16, device=cuda)
    kl.gemm(a, b, c, a_major=1)
    torch.cuda.synchronize()
    for i, (ab, bb, _, _) in enumerate(parts):
        check(c[i].float().cpu().numpy(), ab, bb, 1.0, 1e-2)


def test_mn_major_limits(cuda):
    a = torch.zeros((64, 128), dtype=torch.float8_e4m3fn, device=cuda)
    b = torch.zeros((128, 64), dtype=torch.float8_e4m3fn, device=cuda)
    with pytest.raises(kl.KlError) as e:
        kl.gemm(a, b, a_major=1, algo=kl.ALGO_1CTA)
    assert e.value.status == kl.KL_ERR_NOT_SUPPORTED
