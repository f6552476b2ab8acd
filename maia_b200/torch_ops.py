"""PyTorch operators over the C ABI: torch.ops.kl.gemm, torch.ops.kl.gemm_fp8,
torch.ops.kl.gemm_block_scaled and torch.ops.kl.gemm_grouped.

Registered with torch.library so they compose with the rest of a PyTorch program (fake tensors
for shape inference, the dispatcher, torch.compile graphs that call them as opaque ops). The work
is the library's own kernels, launched on the tensors' current CUDA stream.
"""

from __future__ import annotations

from typing import Optional

import torch

from . import ALGO_1CTA, ALGO_2CTA, ALGO_AUTO, gemm as _kl_gemm, gemm_grouped as _kl_gemm_grouped


@torch.library.custom_op("kl::gemm", mutates_args=())
def gemm(a: torch.Tensor, b: torch.Tensor, out_dtype: torch.dtype = torch.bfloat16, alpha: float = 1.0) -> torch.Tensor:
    """alpha * a @ b.T for bf16 a [M, K] and b [N, K] (K contiguous), out bf16 or fp32."""
    if a.dtype != torch.bfloat16 or b.dtype != torch.bfloat16:
        raise TypeError("kl::gemm takes bf16 operands (use kl::gemm_fp8 for e4m3)")
    out = torch.empty((a.shape[0], b.shape[0]), dtype=out_dtype, device=a.device)
    return _kl_gemm(a, b, out, alpha=alpha, algo=ALGO_AUTO)


@gemm.register_fake
def _(a, b, out_dtype=torch.bfloat16, alpha=1.0):
    return a.new_empty((a.shape[0], b.shape[0]), dtype=out_dtype)


@torch.library.custom_op("kl::gemm_fp8", mutates_args=())
def gemm_fp8(a: torch.Tensor, b: torch.Tensor, scale_a: torch.Tensor, scale_b: torch.Tensor) -> torch.Tensor:
    """(a @ b.T) * scale_a * scale_b for e4m3 a [M, K], b [N, K] and fp32 scalar scales; bf16 out."""
    if a.dtype != torch.float8_e4m3fn or b.dtype != torch.float8_e4m3fn:
        raise TypeError("kl::gemm_fp8 takes float8_e4m3fn operands")
    out = torch.empty((a.shape[0], b.shape[0]), dtype=torch.bfloat16, device=a.device)
    return _kl_gemm(a, b, out, scale_a=scale_a.float().contiguous(), scale_b=scale_b.float().contiguous(),
                    algo=ALGO_AUTO)


@gemm_fp8.register_fake
def _(a, b, scale_a, scale_b):
    return a.new_empty((a.shape[0], b.shape[0]), dtype=torch.bfloat16)


@torch.library.custom_op("kl::gemm_block_scaled", mutates_args=())
def gemm_block_scaled(a: torch.Tensor, b: torch.Tensor, sfa: torch.Tensor, sfb: torch.Tensor, scale_vec: int = 32,
                      out_dtype: torch.dtype = torch.bfloat16, scale_a: Optional[torch.Tensor] = None,
                      scale_b: Optional[torch.Tensor] = None, fp6: str = "") -> torch.Tensor:
    """Block-scaled a @ b.T: a [M, K] and b [N, K] in float8_e4m3fn / float8_e5m2 (MXFP8, scale_vec
    32) or float4_e2m1fn_x2 ([M, K/2]; MXFP4 with scale_vec 32, NVFP4 with scale_vec 16), or with
    fp6 = "e3m2" / "e2m3" uint8 packed fp6 ([M, 3K/4], MXFP6); sfa / sfb the uint8 scales in the
    blocked layout of maia_b200.pack_block_scales, optional fp32 scalar per-tensor scales; bf16 or
    fp32 out."""
    out = torch.empty((a.shape[0], b.shape[0]), dtype=out_dtype, device=a.device)
    return _kl_gemm(a, b, out, sfa=sfa, sfb=sfb, scale_vec=scale_vec,
                    scale_a=None if scale_a is None else scale_a.float().contiguous(),
                    scale_b=None if scale_b is None else scale_b.float().contiguous(), algo=ALGO_AUTO,
                    ab_type=fp6 or None)


@gemm_block_scaled.register_fake
def _(a, b, sfa, sfb, scale_vec=32, out_dtype=torch.bfloat16, scale_a=None, scale_b=None, fp6=""):
    return a.new_empty((a.shape[0], b.shape[0]), dtype=out_dtype)


@torch.library.custom_op("kl::gemm_grouped", mutates_args=())
def gemm_grouped(a: torch.Tensor, b: torch.Tensor, m_block_group: torch.Tensor,
                 out_dtype: torch.dtype = torch.bfloat16, pairs: bool = False) -> torch.Tensor:
    """m-grouped a @ b[g].T (mixture-of-experts layout): a [M, K] with the groups' rows back to back
    (each group padded to 128 rows, or 256 with pairs=True for the CTA-pair kernel), b [G, N, K],
    m_block_group int32 [ceil(M / 128)] naming each 128-row block's group (-1 = padding)."""
    out = torch.empty((a.shape[0], b.shape[1]), dtype=out_dtype, device=a.device)
    return _kl_gemm_grouped(a, b, m_block_group, out, algo=ALGO_2CTA if pairs else ALGO_1CTA)


@gemm_grouped.register_fake
def _(a, b, m_block_group, out_dtype=torch.bfloat16, pairs=False):
    return a.new_empty((a.shape[0], b.shape[1]), dtype=out_dtype)
