"""Stream capture: kl_gemm launches recorded into a CUDA graph and replayed give the eagerly
launched results bit for bit (tile kernels, the skinny kernel with its library workspace and the
no-allocation entry point, a block-scaled GEMM). Every library-side allocation or attribute call
happens on a first, eager call, so replays launch kernels only."""

import numpy as np
import pytest
import torch

import maia_b200 as kl

from gpu_util import random_inputs, to_device

pytestmark = pytest.mark.gpu


def _noalloc(a, b, c):
    d = kl.gemm_desc(a, b, c)
    s = torch.cuda.current_stream().cuda_stream
    kl.check(kl.lib().kl_gemm_skinny_noalloc(kl.ctypes.byref(d), kl.ctypes.c_void_p(s)))


def test_captured_gemms_replay_bit_exact(cuda):
    a1, b1, _, _ = random_inputs(512, 768, 1024, "bf16", seed=1)
    a2, b2, _, _ = random_inputs(16, 4096, 2048, "bf16", seed=2)
    A1, B1 = to_device(a1, "bf16", cuda), to_device(b1, "bf16", cuda)
    A2, B2 = to_device(a2, "bf16", cuda), to_device(b2, "bf16", cuda)
    c_pair = torch.empty(512, 768, dtype=torch.bfloat16, device=cuda)
    c_one = torch.empty(512, 768, dtype=torch.float32, device=cuda)
    c_skinny = torch.empty(16, 4096, dtype=torch.bfloat16, device=cuda)
    c_noalloc = torch.empty(16, 4096, dtype=torch.bfloat16, device=cuda)

    def work():
        kl.gemm(A1, B1, c_pair, algo=kl.ALGO_2CTA)
        kl.gemm(A1, B1, c_one, algo=kl.ALGO_1CTA)
        kl.gemm(A2, B2, c_skinny, algo=kl.ALGO_SKINNY)
        _noalloc(A2, B2, c_noalloc)

    side = torch.cuda.Stream()
    side.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(side):
        work()                               # eager: first-call setup, reference results
        torch.cuda.synchronize()
        want = [t.clone() for t in (c_pair, c_one, c_skinny, c_noalloc)]
        graph = torch.cuda.CUDAGraph()
        for t in (c_pair, c_one, c_skinny, c_noalloc):
            t.fill_(float("nan"))
        with torch.cuda.graph(graph, stream=side):
            work()
    torch.cuda.current_stream().wait_stream(side)
    for _ in range(3):
        for t in (c_pair, c_one, c_skinny, c_noalloc):
            t.fill_(float("nan"))
        graph.replay()
        torch.cuda.synchronize()
        assert kl.read_status() == 0
        for got, ref in zip((c_pair, c_one, c_skinny, c_noalloc), want):
            assert torch.equal(got, ref)
    del graph


def test_captured_block_scaled_gemm(cuda):
    from maia_b200 import workloads as wl

    rng = np.random.default_rng(3)
    qa, sa = wl.mx_quantize(rng.standard_normal((256, 512)).astype(np.float32), "e4m3")
    qb, sb = wl.mx_quantize(rng.standard_normal((384, 512)).astype(np.float32), "e4m3")
    a, b = to_device(qa, "e4m3", cuda), to_device(qb, "e4m3", cuda)
    psa = kl.pack_block_scales(torch.from_numpy(sa).to(cuda), 512)
    psb = kl.pack_block_scales(torch.from_numpy(sb).to(cuda), 512)
    c = torch.empty(256, 384, dtype=torch.bfloat16, device=cuda)
    side = torch.cuda.Stream()
    side.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(side):
        kl.gemm(a, b, c, sfa=psa, sfb=psb)
        torch.cuda.synchronize()
        want = c.clone()
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph, stream=side):
            kl.gemm(a, b, c, sfa=psa, sfb=psb)
    torch.cuda.current_stream().wait_stream(side)
    c.fill_(float("nan"))
    graph.replay()
    torch.cuda.synchronize()
    assert torch.equal(c, want)
    del graph
