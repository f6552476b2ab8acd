"""m-grouped GEMM (mixture-of-experts layout) on the GPU against the fp64 oracle: A holds the
groups' rows back to back, each group padded to 128 rows; every 128-row block multiplies the B of
its group (m_block_group), -1 blocks are padding and come out 0."""

import numpy as np
import pytest
import torch

import maia_b200 as kl
from oracle import gemm as og

from gpu_util import TORCH_TYPES, random_inputs, to_device

pytestmark = pytest.mark.gpu


def grouped_inputs(sizes, n, k, dtype, seed, pad_blocks=0):
    rows = [-(-s // 128) * 128 for s in sizes]
    m = sum(rows) + 128 * pad_blocks
    rng = np.random.Generator(np.random.PCG64(seed))
    a_bits = np.zeros((m, k), dtype=np.uint16 if dtype == "bf16" else np.uint8)
    blocks, b_list, sa, sb = [], [], 1.0, 1.0
    r0 = 0
    for g, (s, rp) in enumerate(zip(sizes, rows)):
        a, b, sa_g, sb_g = random_inputs(s, n, k, dtype, seed=int(rng.integers(1 << 30)))
        a_bits[r0:r0 + s] = a
        b_list.append(b)
        blocks += [g] * (rp // 128)
        r0 += rp
    blocks += [-1] * pad_blocks
    return a_bits, np.stack(b_list), np.array(blocks, dtype=np.int32), rows


@pytest.mark.parametrize("dtype,out", [("bf16", "bf16"), ("bf16", "f32")])
@pytest.mark.parametrize("sizes,n,k", [([100, 300, 17, 256], 512, 256), ([128], 384, 640), ([5, 250, 129], 1000, 520)])
def test_grouped_gemm(cuda, dtype, out, sizes, n, k):
    a_bits, b_bits, blocks, rows = grouped_inputs(sizes, n, k, dtype, seed=sum(sizes) + n, pad_blocks=1)
    a, b = to_device(a_bits, dtype, cuda), to_device(b_bits, dtype, cuda)
    c = torch.full((a.shape[0], n), float("nan"), dtype=TORCH_TYPES[out], device=cuda)
    kl.gemm_grouped(a, b, torch.from_numpy(blocks).to(cuda), c)
    torch.cuda.synchronize()
    assert kl.read_status() == 0
    got = c.float().cpu().numpy()
    r0 = 0
    for g, (s, rp) in enumerate(zip(sizes, rows)):
        ref = og.gemm_f64(a_bits[r0:r0 + s], b_bits[g])
        elem, norm = og.rel_error(got[r0:r0 + s], ref)
        assert elem <= 1e-2 and norm <= 1e-2, f"group {g}: {elem:.3e} / {norm:.3e}"
        assert np.all(got[r0 + s:r0 + rp] == 0), "padding rows of A are zero"
        r0 += rp
    assert np.all(got[r0:] == 0), "a -1 block computes with B = 0"


def test_grouped_gemm_fp8_and_accumulate(cuda):
    sizes, n, k = [200, 64, 384], 768, 512
    a_bits, b_bits, blocks, rows = grouped_inputs(sizes, n, k, "e4m3", seed=3)
    a, b = to_device(a_bits, "e4m3", cuda), to_device(b_bits, "e4m3", cuda)
    c0 = np.random.default_rng(4).standard_normal((a.shape[0], n)).astype(np.float32)
    c = torch.from_numpy(c0).to(cuda)
    one = torch.ones(1, device=cuda)
    kl.gemm_grouped(a, b, torch.from_numpy(blocks).to(cuda), c, scale_a=one, scale_b=one, accumulate=True)
    torch.cuda.synchronize()
    assert kl.read_status() == 0
    got = c.cpu().numpy()
    r0 = 0
    for g, (s, rp) in enumerate(zip(sizes, rows)):
        ref = og.gemm_f64(a_bits[r0:r0 + s], b_bits[g]) + c0[r0:r0 + s]
        elem, norm = og.rel_error(got[r0:r0 + s], ref)
        assert elem <= 5e-2 and norm <= 5e-2, f"group {g}: {elem:.3e} / {norm:.3e}"
        r0 += rp


@pytest.mark.parametrize("sizes,n,k", [([256, 512, 200, 256], 512, 384), ([300, 100], 1000, 520)])
def test_grouped_gemm_cta_pair(cuda, sizes, n, k):
    """The CTA-pair kernel with groups padded to 256 rows (each 256-row tile within one group)."""
    rows = [-(-s // 256) * 256 for s in sizes]
    a_bits = np.zeros((sum(rows), k), dtype=np.uint16)
    b_list, blocks, r0 = [], [], 0
    for g, (s, rp) in enumerate(zip(sizes, rows)):
        a, b, _, _ = random_inputs(s, n, k, "bf16", seed=11 * g + s)
        a_bits[r0:r0 + s] = a
        b_list.append(b)
        blocks += [g] * (rp // 128)
        r0 += rp
    b_bits = np.stack(b_list)
    a, b = to_device(a_bits, "bf16", cuda), to_device(b_bits, "bf16", cuda)
    c = torch.full((a.shape[0], n), float("nan"), dtype=torch.float32, device=cuda)
    kl.gemm_grouped(a, b, torch.tensor(blocks, dtype=torch.int32, device=cuda), c, algo=kl.ALGO_2CTA)
    torch.cuda.synchronize()
    assert kl.read_status() == 0
    got = c.cpu().numpy()
    r0 = 0
    for g, (s, rp) in enumerate(zip(sizes, rows)):
        elem, norm = og.rel_error(got[r0:r0 + s], og.gemm_f64(a_bits[r0:r0 + s], b_bits[g]))
        assert elem <= 1e-2 and norm <= 1e-2, f"group {g}: {elem:.3e} / {norm:.3e}"
        r0 += rp


def test_grouped_gemm_limits(cuda):
    a = torch.zeros(256, 64, dtype=torch.bfloat16, device=cuda)
    b = torch.zeros(2, 128, 64, dtype=torch.bfloat16, device=cuda)
    blocks = torch.zeros(2, dtype=torch.int32, device=cuda)
    d = kl.gemm_desc(a, b[0], torch.zeros(256, 128, dtype=torch.bfloat16, device=cuda), algo=kl.ALGO_SKINNY)
    d.groups, d.stride_b, d.m_block_group = 2, b.stride(0), blocks.data_ptr()
    with pytest.raises(kl.KlError) as e:
        kl.check(kl.lib().kl_gemm(kl.ctypes.byref(d), kl.ctypes.c_void_p(0)))
    assert e.value.status == kl.KL_ERR_NOT_SUPPORTED
    with pytest.raises(ValueError):
        kl.gemm_grouped(a, b, torch.zeros(1, dtype=torch.int32, device=cuda))  # too few block entries


@pytest.mark.parametrize("algo", [kl.ALGO_1CTA, kl.ALGO_2CTA], ids=["1cta", "2cta"])
@pytest.mark.parametrize("kind", ["e4m3", "e2m1", "e2m3"])
def test_grouped_block_scaled(cuda, algo, kind):
    """MoE experts in MX formats: B's block scales are the groups' blocked arrays back to back
    (packed fp6 experts: a rank-3 16U6 tensor map over the stack)."""
    from maia_b200 import workloads as wl

    sizes, n, k = [256, 512, 256], 320, 512
    rng = np.random.default_rng(len(kind))
    qa_parts, sa_parts, qb, sb = [], [], [], []
    for s in sizes:
        q, sc = wl.mx_quantize(rng.standard_normal((s, k)).astype(np.float32), kind)
        qa_parts.append(q)
        sa_parts.append(sc)
    for _ in sizes:
        q, sc = wl.mx_quantize(rng.standard_normal((n, k)).astype(np.float32), kind)
        qb.append(q)
        sb.append(sc)
    qa, sa = np.concatenate(qa_parts), np.concatenate(sa_parts)
    blocks = np.repeat(np.arange(len(sizes), dtype=np.int32), [s // 128 for s in sizes])
    a, b = to_device(qa, kind, cuda), to_device(np.stack(qb), kind, cuda)
    psa = kl.pack_block_scales(torch.from_numpy(sa).to(cuda), k)
    psb = torch.cat([kl.pack_block_scales(torch.from_numpy(x).to(cuda), k) for x in sb])
    c = torch.full((qa.shape[0], n), float("nan"), dtype=torch.float32, device=cuda)
    kl.gemm_grouped(a, b, torch.from_numpy(blocks).to(cuda), c, algo=algo, sfa=psa, sfb=psb,
                    ab_type=kind if kind in kl.FP6_TYPES else None)
    torch.cuda.synchronize()
    assert kl.read_status() == 0
    got, r0 = c.cpu().numpy(), 0
    for g, s in enumerate(sizes):
        ref = og.gemm_mx_f64(qa_parts[g], qb[g], sa_parts[g], sb[g], kind)
        elem, norm = og.rel_error(got[r0:r0 + s], ref)
        assert elem <= 5e-2 and norm <= 5e-2, f"group {g}: {elem:.3e} / {norm:.3e}"
        r0 += s
