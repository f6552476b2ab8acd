"""kl_gemm_host: operands and result in host memory, copies overlapped with the GEMM in column
blocks. Checked against the fp64 oracle, and bit for bit against kl_gemm on device copies of the
same operands where the column blocks cannot change the arithmetic (tile kernels, M > 128: every
output tile is computed the same way). The skinny kernel splits K differently when N is cut into
blocks, so there only the tolerance applies."""

import numpy as np
import pytest
import torch

import maia_b200 as kl

from gpu_util import check, random_inputs, to_device

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("m, n, k, chunks, pinned", [(512, 4096, 1024, 0, True), (256, 3000, 768, 3, True),
                                                     (64, 8192, 2048, 4, False), (1000, 1000, 520, 1, True)])
def test_host_pipeline_matches_device_gemm(cuda, m, n, k, chunks, pinned):
    """The column blocks against the fp64 oracle; with whole tiles (stream_k = -1) the blocks' tiles
    are the full GEMM's tiles, so C is bit-identical to one kl_gemm on device buffers (the default
    may cut a short block's tiles into K-ranges, another summation order)."""
    a_bits, b_bits, _, _ = random_inputs(m, n, k, "bf16", seed=m + k)
    a_dev = to_device(a_bits, "bf16", cuda)
    b_dev = to_device(b_bits, "bf16", cuda)
    ref = kl.gemm(a_dev, b_dev, stream_k=-1)
    a_host = a_dev.cpu()
    b_host = b_dev.cpu()
    c_host = torch.full((m, n), float("nan"), dtype=torch.bfloat16)
    if pinned:
        a_host, b_host, c_host = a_host.pin_memory(), b_host.pin_memory(), c_host.pin_memory()
    sa = torch.empty_like(a_dev)
    sb = torch.empty_like(b_dev)
    sc = torch.empty((m, n), dtype=torch.bfloat16, device=cuda)
    for sk in (0, -1, 0, -1):
        c_host.fill_(float("nan"))
        kl.gemm_host(a_host, b_host, c_host, sa, sb, sc, chunks=chunks, stream_k=sk)
        torch.cuda.current_stream().synchronize()
        assert kl.read_status() == 0
        check(c_host.float().numpy(), a_bits, b_bits, 1.0, 1e-2)
        if m > 128 and sk == -1:
            assert torch.equal(c_host.view(torch.int16), ref.cpu().view(torch.int16))


@pytest.mark.parametrize("m, n, k, chunks", [(512, 4096, 1024, 0), (256, 3000, 640, 3), (1000, 1024, 512, 1)])
def test_host_pipeline_mxfp8(cuda, m, n, k, chunks):
    """MXFP8 through the host-buffer path: the blocked scales travel with their column blocks of B."""
    from maia_b200 import workloads as wl
    from oracle import gemm as og

    rng = np.random.default_rng(m + n)
    qa, sfa = wl.mx_quantize(rng.standard_normal((m, k)).astype(np.float32))
    qb, sfb = wl.mx_quantize(rng.standard_normal((n, k)).astype(np.float32))
    a_dev, b_dev = to_device(qa, "e4m3", cuda), to_device(qb, "e4m3", cuda)
    psa = kl.mx_pack_scales(torch.from_numpy(sfa).to(cuda), k)
    psb = kl.mx_pack_scales(torch.from_numpy(sfb).to(cuda), k)
    ref = kl.gemm(a_dev, b_dev, sfa=psa, sfb=psb, stream_k=-1)
    c_host = torch.full((m, n), float("nan"), dtype=torch.bfloat16).pin_memory()
    kl.gemm_host(a_dev.cpu().pin_memory(), b_dev.cpu().pin_memory(), c_host, torch.empty_like(a_dev),
                 torch.empty_like(b_dev), torch.empty((m, n), dtype=torch.bfloat16, device=cuda), chunks=chunks,
                 sfa=psa.cpu().pin_memory(), sfb=psb.cpu().pin_memory(), stream_k=-1)
    torch.cuda.current_stream().synchronize()
    assert kl.read_status() == 0
    got = c_host.float().numpy()
    want = og.gemm_mx_f64(qa, qb, sfa, sfb, "e4m3")
    elem, norm = og.rel_error(got, want)
    assert elem <= 5e-2 and norm <= 5e-2
    assert torch.equal(c_host.view(torch.int16), ref.cpu().view(torch.int16))


@pytest.mark.parametrize("kind", ["e3m2", "e2m3"])
def test_host_pipeline_mxfp6(cuda, kind):
    """Packed fp6 through the host-buffer path: column blocks of B start on 256-row boundaries, so
    every block's device address keeps the 32-byte alignment the fp6 tensor maps need."""
    from maia_b200 import workloads as wl
    from oracle import gemm as og

    m, n, k = 384, 3000, 640
    rng = np.random.default_rng(17)
    qa, sfa = wl.mx_quantize(rng.standard_normal((m, k)).astype(np.float32), kind)
    qb, sfb = wl.mx_quantize(rng.standard_normal((n, k)).astype(np.float32), kind)
    a_dev, b_dev = torch.from_numpy(qa).to(cuda), torch.from_numpy(qb).to(cuda)
    psa = kl.mx_pack_scales(torch.from_numpy(sfa).to(cuda), k)
    psb = kl.mx_pack_scales(torch.from_numpy(sfb).to(cuda), k)
    ref = kl.gemm(a_dev, b_dev, sfa=psa, sfb=psb, ab_type=kind, stream_k=-1)
    c_host = torch.full((m, n), float("nan"), dtype=torch.bfloat16).pin_memory()
    kl.gemm_host(a_dev.cpu().pin_memory(), b_dev.cpu().pin_memory(), c_host, torch.empty_like(a_dev),
                 torch.empty_like(b_dev), torch.empty((m, n), dtype=torch.bfloat16, device=cuda), chunks=3,
                 sfa=psa.cpu().pin_memory(), sfb=psb.cpu().pin_memory(), ab_type=kind, stream_k=-1)
    torch.cuda.current_stream().synchronize()
    assert kl.read_status() == 0
    elem, norm = og.rel_error(c_host.float().numpy(), og.gemm_mx_f64(qa, qb, sfa, sfb, kind))
    assert elem <= 5e-2 and norm <= 5e-2
    assert torch.equal(c_host.view(torch.int16), ref.cpu().view(torch.int16))
