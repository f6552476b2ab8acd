"""torch.ops.kl.* registration and shape inference (fake tensors: no GPU, no library call)."""

import torch


def test_fake_tensor_shapes():
    import maia_b200.torch_ops  # noqa: F401
    from torch._subclasses.fake_tensor import FakeTensorMode

    with FakeTensorMode():
        a = torch.empty((8, 32), dtype=torch.bfloat16)
        b = torch.empty((16, 32), dtype=torch.bfloat16)
        c = torch.ops.kl.gemm(a, b, torch.float32)
        assert c.shape == (8, 16) and c.dtype == torch.float32
        a8 = torch.empty((8, 64), dtype=torch.float8_e4m3fn)
        b8 = torch.empty((24, 64), dtype=torch.float8_e4m3fn)
        s = torch.empty((1,), dtype=torch.float32)
        c8 = torch.ops.kl.gemm_fp8(a8, b8, s, s)
        assert c8.shape == (8, 24) and c8.dtype == torch.bfloat16


def test_fake_block_scaled_shapes():
    import maia_b200.torch_ops  # noqa: F401
    from torch._subclasses.fake_tensor import FakeTensorMode

    with FakeTensorMode():
        a = torch.empty((256, 64), dtype=torch.float4_e2m1fn_x2)   # K = 128 packed
        b = torch.empty((128, 64), dtype=torch.float4_e2m1fn_x2)
        sf = torch.empty((1024,), dtype=torch.uint8)
        c = torch.ops.kl.gemm_block_scaled(a, b, sf, sf, 16, torch.float32)
        assert c.shape == (256, 128) and c.dtype == torch.float32


def test_fake_grouped_shapes():
    import maia_b200.torch_ops  # noqa: F401
    from torch._subclasses.fake_tensor import FakeTensorMode

    with FakeTensorMode():
        a = torch.empty((512, 64), dtype=torch.bfloat16)
        b = torch.empty((3, 96, 64), dtype=torch.bfloat16)
        blocks = torch.empty((4,), dtype=torch.int32)
        c = torch.ops.kl.gemm_grouped(a, b, blocks)
        assert c.shape == (512, 96) and c.dtype == torch.bfloat16
