"""Batched GEMM (rank-3 tensor maps): L independent problems C[i] = A[i] . B[i]^T in one launch,
each checked against the fp64 oracle; strided batches (gaps between matrices) included."""

import numpy as np
import pytest
import torch

import maia_b200 as kl

from gpu_util import check, random_inputs, to_device

pytestmark = pytest.mark.gpu


def _batch_inputs(L, m, n, k, dtype, seed):
    parts = [random_inputs(m, n, k, dtype, seed=seed + i) for i in range(L)]
    return parts


@pytest.mark.parametrize("algo", [kl.ALGO_1CTA, kl.ALGO_2CTA], ids=["1cta", "2cta"])
@pytest.mark.parametrize("L, m, n, k", [(2, 256, 512, 384), (5, 300, 200, 136), (3, 1024, 768, 512)])
@pytest.mark.parametrize("out", ["bf16", "f32"])
def test_batched_bf16(cuda, algo, L, m, n, k, out):
    parts = _batch_inputs(L, m, n, k, "bf16", seed=L * 100 + m)
    a = torch.stack([to_device(p[0], "bf16", cuda) for p in parts])
    b = torch.stack([to_device(p[1], "bf16", cuda) for p in parts])
    odt = torch.bfloat16 if out == "bf16" else torch.float32
    c = torch.full((L, m, n), float("nan"), dtype=odt, device=cuda)
    kl.gemm(a, b, c, algo=algo)
    torch.cuda.synchronize()
    assert kl.read_status() == 0
    for i, (ab, bb, _, _) in enumerate(parts):
        check(c[i].float().cpu().numpy(), ab, bb, 1.0, 1e-2)


@pytest.mark.parametrize("algo", [kl.ALGO_1CTA, kl.ALGO_2CTA], ids=["1cta", "2cta"])
def test_batched_with_gaps_between_matrices(cuda, algo):
    """Batch strides larger than rows x pitch: views into bigger buffers, nothing outside C written."""
    L, m, n, k = 3, 384, 256, 320
    parts = _batch_inputs(L, m, n, k, "bf16", seed=77)
    a_big = torch.zeros((L, m + 16, k + 64), dtype=torch.bfloat16, device=cuda)
    b_big = torch.zeros((L, n + 8, k + 32), dtype=torch.bfloat16, device=cuda)
    c_big = torch.full((L, m + 8, n + 24), 5.0, dtype=torch.bfloat16, device=cuda)
    for i, (ab, bb, _, _) in enumerate(parts):
        a_big[i, :m, :k] = to_device(ab, "bf16", cuda)
        b_big[i, :n, :k] = to_device(bb, "bf16", cuda)
    kl.gemm(a_big[:, :m, :k], b_big[:, :n, :k], c_big[:, :m, :n], algo=algo)
    torch.cuda.synchronize()
    assert (c_big[:, m:, :] == 5.0).all() and (c_big[:, :, n:] == 5.0).all(), "wrote outside C"
    for i, (ab, bb, _, _) in enumerate(parts):
        check(c_big[i, :m, :n].float().cpu().numpy(), ab, bb, 1.0, 1e-2)


def test_batched_e4m3(cuda):
    L, m, n, k = 2, 512, 512, 1024
    parts = _batch_inputs(L, m, n, k, "e4m3", seed=5)
    # One scale pair for the whole batch: requantise every matrix with the first one's scales.
    sa, sb = parts[0][2], parts[0][3]
    a = torch.stack([to_device(p[0], "e4m3", cuda) for p in parts])
    b = torch.stack([to_device(p[1], "e4m3", cuda) for p in parts])
    c = torch.full((L, m, n), float("nan"), dtype=torch.bfloat16, device=cuda)
    ta = torch.tensor([sa], dtype=torch.float32, device=cuda)
    tb = torch.tensor([sb], dtype=torch.float32, device=cuda)
    kl.gemm(a, b, c, scale_a=ta, scale_b=tb)
    torch.cuda.synchronize()
    for i, (ab, bb, _, _) in enumerate(parts):
        check(c[i].float().cpu().numpy(), ab, bb, sa * sb, 5e-2)


def test_batched_rejects_skinny(cuda):
    a = torch.zeros((2, 16, 64), dtype=torch.bfloat16, device=cuda)
    b = torch.zeros((2, 128, 64), dtype=torch.bfloat16, device=cuda)
    with pytest.raises(kl.KlError) as e:
        kl.gemm(a, b, algo=kl.ALGO_SKINNY)
    assert e.value.status == kl.KL_ERR_NOT_SUPPORTED
    c = kl.gemm(a, b)  # AUTO picks a tile kernel for batches
    torch.cuda.synchronize()
    assert c.shape == (2, 16, 128) and (c == 0).all()
