"""torch.ops.kl.gemm / gemm_fp8 against torch's own fp32 matmul of the same rounded operands."""

import pytest
import torch

pytestmark = pytest.mark.gpu


def rel(c, ref):
    return ((c.float() - ref).abs().max() / ref.abs().max()).item()


@pytest.mark.parametrize("m, n, k", [(64, 4096, 1024), (512, 768, 640), (2048, 2048, 2048)])
def test_kl_gemm_op_matches_torch_matmul(cuda, m, n, k):
    import maia_b200.torch_ops  # noqa: F401  (registers torch.ops.kl.*)

    g = torch.Generator(device="cuda").manual_seed(m + n + k)
    a = torch.randn((m, k), device=cuda, generator=g).to(torch.bfloat16)
    b = torch.randn((n, k), device=cuda, generator=g).to(torch.bfloat16)
    ref = a.float() @ b.float().T
    assert rel(torch.ops.kl.gemm(a, b), ref) < 1e-2
    assert rel(torch.ops.kl.gemm(a, b, torch.float32), ref) < 1e-5


def test_kl_gemm_fp8_op(cuda):
    import maia_b200.torch_ops  # noqa: F401

    g = torch.Generator(device="cuda").manual_seed(3)
    xa = torch.randn((256, 1024), device=cuda, generator=g)
    xb = torch.randn((512, 1024), device=cuda, generator=g)
    sa, sb = xa.abs().max() / 448, xb.abs().max() / 448
    a = (xa / sa).to(torch.float8_e4m3fn)
    b = (xb / sb).to(torch.float8_e4m3fn)
    ref = (a.float() @ b.float().T) * sa * sb
    assert rel(torch.ops.kl.gemm_fp8(a, b, sa.reshape(1), sb.reshape(1)), ref) < 5e-2


@pytest.mark.parametrize("kind,vec", [("e4m3", 32), ("e2m1", 32), ("e2m1", 16), ("e2m3", 32)])
def test_kl_gemm_block_scaled_op(cuda, kind, vec):
    """torch.ops.kl.gemm_block_scaled against the fp64 oracle (MXFP8, MXFP4, NVFP4, MXFP6)."""
    import numpy as np

    import maia_b200 as kl
    import maia_b200.torch_ops  # noqa: F401
    from maia_b200 import workloads as wl
    from oracle import gemm as og

    from gpu_util import to_device

    rng = np.random.default_rng(vec)
    xa = rng.standard_normal((384, 512)).astype(np.float32)
    xb = rng.standard_normal((256, 512)).astype(np.float32)
    if vec == 16:
        qa, sa, ga = wl.nv_quantize(xa)
        qb, sb, gb = wl.nv_quantize(xb)
        ref = og.gemm_nv_f64(qa, qb, sa, sb, ga * gb)
        scales = dict(scale_a=torch.tensor([ga], device=cuda), scale_b=torch.tensor([gb], device=cuda))
    else:
        qa, sa = wl.mx_quantize(xa, kind)
        qb, sb = wl.mx_quantize(xb, kind)
        ref = og.gemm_mx_f64(qa, qb, sa, sb, kind)
        scales = {"fp6": kind} if kind in ("e3m2", "e2m3") else {}
    psa = kl.pack_block_scales(torch.from_numpy(sa).to(cuda), 512, vec)
    psb = kl.pack_block_scales(torch.from_numpy(sb).to(cuda), 512, vec)
    c = torch.ops.kl.gemm_block_scaled(to_device(qa, kind, cuda), to_device(qb, kind, cuda), psa, psb, vec,
                                       torch.float32, **scales)
    torch.cuda.synchronize()
    got = c.cpu().numpy()
    assert np.abs(got - ref).max() / np.abs(ref).max() < 1e-3


def test_kl_gemm_grouped_op(cuda):
    import maia_b200.torch_ops  # noqa: F401

    g = torch.Generator(device="cuda").manual_seed(5)
    a = torch.randn((512, 256), device=cuda, generator=g).to(torch.bfloat16)
    b = torch.randn((2, 384, 256), device=cuda, generator=g).to(torch.bfloat16)
    blocks = torch.tensor([0, 0, 1, 1], dtype=torch.int32, device=cuda)
    for pairs in (False, True):
        c = torch.ops.kl.gemm_grouped(a, b, blocks, torch.float32, pairs)
        ref = torch.cat([a[:256].float() @ b[0].float().T, a[256:].float() @ b[1].float().T])
        assert rel(c, ref) < 1e-5
