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
