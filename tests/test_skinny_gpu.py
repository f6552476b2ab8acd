"""KL_ALGO_SKINNY (memory-bound small-M GEMM, stream-K over all SMs) against the fp64 oracle.

Covers the decode configs (M = 16, 64, 128 tokens, N = 28672, K = 8192), ragged shapes, tiles
split across several CTAs (the workspace reduction), determinism, ticket re-arming across calls,
caller-provided workspaces and e4m3 inputs. Tolerances as in test_gemm_gpu.py.
"""

import numpy as np
import pytest
import torch

import maia_b200 as kl
from maia_b200 import workloads as wl

from gpu_util import check, random_inputs, run_kl, to_device

pytestmark = pytest.mark.gpu

BF16_TOL = 1e-2
FP8_TOL = 5e-2


@pytest.mark.parametrize("variant", [1, 2], ids=["w128", "w256"])
@pytest.mark.parametrize("m", [16, 64, 128])
def test_c5_decode_shapes(cuda, m, variant):
    w = wl.C5[m]
    a, b, _, _ = wl.make_inputs(w)
    c = run_kl(a, b, "bf16", "bf16", cuda, kl.ALGO_SKINNY, variant=variant)
    check(c, a, b, 1.0, BF16_TOL)


@pytest.mark.parametrize("m", [16, 64, 128])
def test_c5_decode_shapes_default_route(cuda, m):
    """The decode configs through KL_ALGO_AUTO, the route the benchmark times (the skinny kernel
    up to 64 rows, the one-CTA tile kernel over 112 weight bands at 128), every entry against
    the fp64 oracle."""
    w = wl.C5[m]
    a, b, _, _ = wl.make_inputs(w)
    check(run_kl(a, b, "bf16", "bf16", cuda, kl.ALGO_AUTO), a, b, 1.0, BF16_TOL)


@pytest.mark.parametrize("variant", [1, 2], ids=["w128", "w256"])
@pytest.mark.parametrize("shape", [(1, 8, 64), (5, 136, 200), (17, 1000, 512), (33, 640, 1096), (100, 384, 2048),
                                   (200, 256, 640), (256, 520, 320), (128, 128, 64)])
def test_ragged(cuda, shape, variant):
    m, n, k = shape
    a, b, _, _ = random_inputs(m, n, k, "bf16", seed=m + 3 * n + 7 * k)
    check(run_kl(a, b, "bf16", "bf16", cuda, kl.ALGO_SKINNY, variant=variant), a, b, 1.0, BF16_TOL)
    check(run_kl(a, b, "bf16", "f32", cuda, kl.ALGO_SKINNY, variant=variant), a, b, 1.0, BF16_TOL)


@pytest.mark.parametrize("variant", [1, 2], ids=["w128", "w256"])
@pytest.mark.parametrize("ctas", [1, 3, 7, 50])
@pytest.mark.parametrize("prefetch", [-1, 24])
def test_tiles_split_across_ctas(cuda, ctas, prefetch, variant):
    """Few CTAs over many units: tiles shared by 2+ CTAs go through the slot reduction (with and
    without L2 prefetch of the weight tiles ahead of the loads)."""
    a, b, _, _ = random_inputs(48, 5 * 128 + 40, 64 * 37, "bf16", seed=ctas)
    check(run_kl(a, b, "bf16", "bf16", cuda, kl.ALGO_SKINNY, max_ctas=ctas, prefetch=prefetch, variant=variant),
          a, b, 1.0, BF16_TOL)


def test_deterministic_and_rearmed(cuda):
    """Repeated calls give bit-identical results: the reduction order is fixed and the tickets
    are back at zero after every call."""
    a_bits, b_bits, _, _ = random_inputs(64, 3000, 4096, "bf16", seed=4)
    a = to_device(a_bits, "bf16", cuda)
    b = to_device(b_bits, "bf16", cuda)
    outs = []
    for _ in range(4):
        c = torch.empty((64, 3000), dtype=torch.bfloat16, device=cuda)
        kl.gemm(a, b, c, algo=kl.ALGO_SKINNY, max_ctas=37)
        outs.append(c)
    torch.cuda.synchronize()
    assert kl.read_status() == 0
    for o in outs[1:]:
        assert torch.equal(o.view(torch.int16), outs[0].view(torch.int16))
    check(outs[0].float().cpu().numpy(), a_bits, b_bits, 1.0, BF16_TOL)


def test_library_workspace_across_shapes(cuda):
    """Shapes with more and fewer weight tiles in turn on the library-owned workspace: a call must
    not mistake an earlier call's partial sums for its arrival counters."""
    for n in (256, 3000, 640, 5000, 128, 3000):
        a_bits, b_bits, _, _ = random_inputs(40, n, 2048, "bf16", seed=n)
        check(run_kl(a_bits, b_bits, "bf16", "bf16", cuda, kl.ALGO_SKINNY, max_ctas=29), a_bits, b_bits, 1.0,
              BF16_TOL)


def test_caller_workspace(cuda):
    a_bits, b_bits, _, _ = random_inputs(32, 1024, 1024, "bf16", seed=8)
    a = to_device(a_bits, "bf16", cuda)
    b = to_device(b_bits, "bf16", cuda)
    c = torch.empty((32, 1024), dtype=torch.bfloat16, device=cuda)
    need = kl.workspace_size(a, b, c, algo=kl.ALGO_SKINNY, max_ctas=20)
    assert need > 0
    ws = torch.zeros(need, dtype=torch.uint8, device=cuda)
    for _ in range(2):
        kl.gemm(a, b, c, algo=kl.ALGO_SKINNY, max_ctas=20, workspace=ws)
        torch.cuda.synchronize()
        check(c.float().cpu().numpy(), a_bits, b_bits, 1.0, BF16_TOL)
    with pytest.raises(kl.KlError) as e:
        kl.gemm(a, b, c, algo=kl.ALGO_SKINNY, max_ctas=20, workspace=ws[: need - 256])
    assert e.value.status == kl.KL_ERR_INVALID_ARGUMENT


@pytest.mark.parametrize("variant", [1, 2], ids=["w128", "w256"])
@pytest.mark.parametrize("shape", [(16, 1024, 2048), (100, 640, 1024)])
def test_e4m3(cuda, shape, variant):
    m, n, k = shape
    a, b, sa, sb = random_inputs(m, n, k, "e4m3", seed=k)
    c = run_kl(a, b, "e4m3", "bf16", cuda, kl.ALGO_SKINNY, scale_a=sa, scale_b=sb, variant=variant)
    check(c, a, b, sa * sb, FP8_TOL)


def test_rejects_more_than_256_rows(cuda):
    a = torch.zeros((300, 64), dtype=torch.bfloat16, device=cuda)
    b = torch.zeros((128, 64), dtype=torch.bfloat16, device=cuda)
    with pytest.raises(kl.KlError):
        kl.gemm(a, b, algo=kl.ALGO_SKINNY)
