"""Programmatic dependent launch (kl_gemm_desc.launch_overlap) keeps stream order: chained GEMMs
whose buffers ping-pong, so each launch reads what the one before it wrote (read after write) and
overwrites what the one before it read (write after read). Launched back to back with the overlap
on, the chain gives the same bits as launched one step at a time with a synchronisation between
steps and as launched with the overlap off, and every step agrees with the fp64 oracle on the bf16
input it was given. Tile kernels (one CTA, CTA pair, 256 x 512 pair tiles) and the skinny kernel,
also captured in a CUDA graph.
"""

import numpy as np
import pytest
import torch

import maia_b200 as kl
from oracle import gemm as og

from gpu_util import random_inputs, to_device

pytestmark = pytest.mark.gpu

TOL16 = 1e-2
STEPS = 6
K = 1024


def _inputs(m, seed, cuda):
    x0 = to_device(random_inputs(m, 16, K, "bf16", seed=seed)[0], "bf16", cuda)
    # Square weights scaled by 1/sqrt(K), so the chain stays of order 1.
    ws = [to_device(random_inputs(K, 16, K, "bf16", seed=seed + 1 + i, scale=K ** -0.5)[0], "bf16", cuda)
          for i in range(STEPS)]
    return x0, ws


def _launchers(bufs, ws, algo, variant, overlap, stream=None):
    return [kl.gemm_launcher(bufs[i % 2], ws[i], bufs[(i + 1) % 2], algo=algo, variant=variant, overlap=overlap,
                             stream=stream) for i in range(len(ws))]


def _back_to_back(x0, ws, algo, variant, overlap):
    """x_{i+1} = x_i . w_i^T for every w_i through two buffers, all launches queued at once."""
    bufs = [x0.clone(), torch.empty_like(x0)]
    for f in _launchers(bufs, ws, algo, variant, overlap):
        f()
    torch.cuda.synchronize()
    assert kl.read_status() == 0
    return bufs[len(ws) % 2].clone()


def _step_by_step(x0, ws, algo, variant):
    bufs = [x0.clone(), torch.empty_like(x0)]
    outs = []
    for i, f in enumerate(_launchers(bufs, ws, algo, variant, -1)):
        f()
        torch.cuda.synchronize()
        outs.append(bufs[(i + 1) % 2].clone())
    assert kl.read_status() == 0
    return outs


def _bits(t):
    return t.view(torch.int16)


CASES = pytest.mark.parametrize("m,algo,variant", [(256, kl.ALGO_2CTA, 1), (512, kl.ALGO_2CTA, 4),
                                                   (128, kl.ALGO_1CTA, 0), (16, kl.ALGO_SKINNY, 0)],
                                ids=["pair", "pair_wide", "one_cta", "skinny"])


@CASES
def test_chain_keeps_stream_order(cuda, m, algo, variant):
    x0, ws = _inputs(m, 90 + m, cuda)
    steps = _step_by_step(x0, ws, algo, variant)
    on = _back_to_back(x0, ws, algo, variant, 1)
    off = _back_to_back(x0, ws, algo, variant, -1)
    assert torch.equal(_bits(on), _bits(steps[-1]))
    assert torch.equal(_bits(off), _bits(steps[-1]))
    prev = x0
    for i, out in enumerate(steps):
        xb = _bits(prev).cpu().numpy().view(np.uint16)
        wb = _bits(ws[i]).cpu().numpy().view(np.uint16)
        elem, norm = og.rel_error(out.float().cpu().numpy(), og.gemm_f64(xb, wb, 1.0))
        assert norm <= TOL16 and elem <= TOL16, f"step {i}: element-wise {elem:.3e}, normwise {norm:.3e}"
        prev = out


@pytest.mark.parametrize("m,algo,variant", [(256, kl.ALGO_2CTA, 1), (128, kl.ALGO_1CTA, 0), (16, kl.ALGO_SKINNY, 0)],
                         ids=["pair", "one_cta", "skinny"])
def test_chain_in_a_cuda_graph(cuda, m, algo, variant):
    x0, ws = _inputs(m, 70 + m, cuda)
    want = _step_by_step(x0, ws, algo, variant)[-1]
    bufs = [x0.clone(), torch.empty_like(x0)]
    s = torch.cuda.Stream()
    fns = _launchers(bufs, ws, algo, variant, 1, stream=s.cuda_stream)
    # Warm-up on the capture stream, outside the capture: these small problems split their K across
    # the CTAs through the stream's workspace, which is made on a first eager launch and never
    # inside a capture (a capture on a stream without one records whole tiles, other bits).
    for f in fns:
        f()
    torch.cuda.synchronize()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g, stream=s):
        for f in fns:
            f()
    for _ in range(2):  # replays start from x0 again
        bufs[0].copy_(x0)
        g.replay()
        torch.cuda.synchronize()
        assert kl.read_status() == 0
        assert torch.equal(_bits(bufs[STEPS % 2]), _bits(want))
