"""The tile kernels' split tail on the GPU, against the fp64 CPU oracle.

On small problems the split is forced (stream_k = 1) and max_ctas leaves few workers, so the last
wave's tiles are cut into K-ranges on several workers and summed through the fp32 slots: every element path of the epilogue
(bf16 / f32 C, fp8 scales, MX block scales with the one-accumulator epilogue, C += result,
batched and m-grouped problems, peer-less TMA stores) goes through the split-tile reduction.
Tolerances as elsewhere: 1e-2 for 16-bit inputs, 5e-2 for fp8.
"""

import numpy as np
import pytest
import torch

import maia_b200 as kl
from maia_b200 import workloads as wl
from oracle import gemm as og

from gpu_util import check, random_inputs, run_kl, to_device

pytestmark = pytest.mark.gpu

TOL16, FP8_TOL = 1e-2, 5e-2
ALGOS = pytest.mark.parametrize("algo", [kl.ALGO_1CTA, kl.ALGO_2CTA], ids=["1cta", "2cta"])


@ALGOS
@pytest.mark.parametrize("out", ["bf16", "f32"])
@pytest.mark.parametrize("shape", [(256, 512, 2048), (300, 520, 1000), (1024, 768, 4096), (128, 256, 64)])
@pytest.mark.parametrize("ctas", [6, 10, 0])
def test_forced_tail_matches_oracle(cuda, algo, out, shape, ctas):
    m, n, k = shape
    a, b, _, _ = random_inputs(m, n, k, "bf16", seed=m + n + k + ctas)
    c = run_kl(a, b, "bf16", out, cuda, algo, stream_k=1, max_ctas=ctas)
    check(c, a, b, 1.0, TOL16)


@ALGOS
def test_tail_is_deterministic_and_close_to_data_parallel(cuda, algo):
    """The same split, the same slot order: bit-identical from run to run; whole tiles sum the
    K-blocks in another association, so they agree to fp32 rounding only."""
    a, b, _, _ = random_inputs(512, 768, 3072, "bf16", seed=3)
    runs = [run_kl(a, b, "bf16", "f32", cuda, algo, stream_k=1, max_ctas=10) for _ in range(3)]
    assert all(np.array_equal(r, runs[0]) for r in runs[1:])
    dp = run_kl(a, b, "bf16", "f32", cuda, algo, stream_k=-1, max_ctas=10)
    assert np.abs(runs[0] - dp).max() <= 1e-5 * np.abs(dp).max()


@ALGOS
def test_more_workers_than_units(cuda, algo):
    """One tile of two K-blocks: at most two K-ranges, on two workers."""
    a, b, _, _ = random_inputs(128, 256, 128, "bf16", seed=4)
    check(run_kl(a, b, "bf16", "bf16", cuda, algo, stream_k=1), a, b, 1.0, TOL16)


def test_default_splits_a_short_last_wave(cuda):
    """stream_k = 0 with 10 CTA pairs and 16 tiles (80 % of two waves), K 8192: the 6 tail tiles are
    cut into 3 K-ranges (0.67 of a wave plus the partial sums, against 1). The default's bits equal
    the forced split's (the same ranges) and differ from whole tiles (another association)."""
    a, b, _, _ = random_inputs(1024, 1024, 8192, "bf16", seed=5)
    auto = run_kl(a, b, "bf16", "f32", cuda, kl.ALGO_2CTA, max_ctas=20)
    check(auto, a, b, 1.0, TOL16)
    assert np.array_equal(auto, run_kl(a, b, "bf16", "f32", cuda, kl.ALGO_2CTA, max_ctas=20, stream_k=1))
    assert not np.array_equal(auto, run_kl(a, b, "bf16", "f32", cuda, kl.ALGO_2CTA, max_ctas=20, stream_k=-1))


@ALGOS
def test_fp8_scaled(cuda, algo):
    a, b, sa, sb = random_inputs(384, 512, 2048, "e4m3", seed=6)
    c = run_kl(a, b, "e4m3", "bf16", cuda, algo, scale_a=sa, scale_b=sb, stream_k=1, max_ctas=6)
    check(c, a, b, sa * sb, FP8_TOL, kind="e4m3")


@pytest.mark.parametrize("kind,variant", [("e4m3", 0), ("e4m3", 2), ("e2m1", 0), ("e2m3", 0)])
@ALGOS
def test_block_scaled(cuda, algo, kind, variant):
    """MX block scales; variant 0 is the one-accumulator, eight-warp early-release epilogue."""
    rng = np.random.default_rng(len(kind) + variant)
    m, n, k = 384, 512, 2048
    qa, sa = wl.mx_quantize(rng.standard_normal((m, k)).astype(np.float32), kind)
    qb, sb = wl.mx_quantize(rng.standard_normal((n, k)).astype(np.float32), kind)
    psa = kl.pack_block_scales(torch.from_numpy(sa).to(cuda), k)
    psb = kl.pack_block_scales(torch.from_numpy(sb).to(cuda), k)
    c = torch.full((m, n), float("nan"), dtype=torch.float32, device=cuda)
    kl.gemm(to_device(qa, kind, cuda), to_device(qb, kind, cuda), c, sfa=psa, sfb=psb, algo=algo, variant=variant,
            stream_k=1, max_ctas=6, ab_type=kind if kind in kl.FP6_TYPES else None)
    torch.cuda.synchronize()
    assert kl.read_status() == 0
    elem, norm = og.rel_error(c.cpu().numpy(), og.gemm_mx_f64(qa, qb, sa, sb, kind))
    assert elem <= FP8_TOL and norm <= FP8_TOL


@ALGOS
@pytest.mark.parametrize("out", ["bf16", "f32"])
def test_accumulate_into_c(cuda, algo, out):
    """C += A . B^T: only the last arrival at a split tile reads and adds C."""
    m, n, k = 512, 768, 2048
    a, b, _, _ = random_inputs(m, n, k, "bf16", seed=7)
    tdt = torch.bfloat16 if out == "bf16" else torch.float32
    c = (torch.randn(m, n, generator=torch.Generator().manual_seed(8)) * 4).to(tdt)
    c0 = c.float().numpy().astype(np.float64)
    c = c.to(cuda)
    kl.gemm(to_device(a, "bf16", cuda), to_device(b, "bf16", cuda), c, algo=algo, accumulate=True, stream_k=1,
            max_ctas=10)
    torch.cuda.synchronize()
    assert kl.read_status() == 0
    check(c.float().cpu().numpy(), a, b, 1.0, TOL16, c0=c0)


@ALGOS
def test_batched(cuda, algo):
    L, m, n, k = 3, 256, 384, 1024
    parts = [random_inputs(m, n, k, "bf16", seed=20 + i) for i in range(L)]
    da = torch.stack([to_device(p[0], "bf16", cuda) for p in parts])
    db = torch.stack([to_device(p[1], "bf16", cuda) for p in parts])
    c = torch.full((L, m, n), float("nan"), dtype=torch.float32, device=cuda)
    kl.gemm(da, db, c, algo=algo, stream_k=1, max_ctas=6)
    torch.cuda.synchronize()
    assert kl.read_status() == 0
    out = c.cpu().numpy()
    for i in range(L):
        check(out[i], parts[i][0], parts[i][1], 1.0, TOL16)


def test_grouped(cuda):
    sizes, n, k = [256, 384, 128], 320, 1536
    rng = np.random.default_rng(9)
    a_parts = [random_inputs(s, n, k, "bf16", seed=30 + i)[0] for i, s in enumerate(sizes)]
    b_parts = [random_inputs(8, n, k, "bf16", seed=40 + i)[1] for i in range(len(sizes))]
    a = to_device(np.concatenate(a_parts), "bf16", cuda)
    b = torch.stack([to_device(x, "bf16", cuda) for x in b_parts])
    blocks = torch.from_numpy(np.repeat(np.arange(len(sizes), dtype=np.int32), [s // 128 for s in sizes])).to(cuda)
    c = torch.full((a.shape[0], n), float("nan"), dtype=torch.float32, device=cuda)
    kl.gemm_grouped(a, b, blocks, c, algo=kl.ALGO_1CTA, stream_k=1)
    torch.cuda.synchronize()
    assert kl.read_status() == 0
    got, r0 = c.cpu().numpy(), 0
    for g, s in enumerate(sizes):
        check(got[r0:r0 + s], a_parts[g], b_parts[g], 1.0, TOL16)
        r0 += s
    del rng


def test_captured_in_a_graph(cuda):
    """The stream's workspace exists after an eager call; a captured launch reuses it and its
    replays give the eager result bit for bit (tickets reset themselves between launches)."""
    a_bits, b_bits, _, _ = random_inputs(512, 768, 2048, "bf16", seed=10)
    a, b = to_device(a_bits, "bf16", cuda), to_device(b_bits, "bf16", cuda)
    c = torch.empty(512, 768, dtype=torch.float32, device=cuda)
    side = torch.cuda.Stream()
    side.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(side):
        kl.gemm(a, b, c, algo=kl.ALGO_2CTA, stream_k=1, max_ctas=10)
        torch.cuda.synchronize()
        want = c.clone()
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph, stream=side):
            kl.gemm(a, b, c, algo=kl.ALGO_2CTA, stream_k=1, max_ctas=10)
    torch.cuda.current_stream().wait_stream(side)
    for _ in range(3):
        c.fill_(float("nan"))
        graph.replay()
        torch.cuda.synchronize()
        assert kl.read_status() == 0
        assert torch.equal(c, want)
    del graph
    check(want.cpu().numpy(), a_bits, b_bits, 1.0, TOL16)


def test_stream_k_argument_is_checked(cuda):
    a = torch.zeros(256, 64, dtype=torch.bfloat16, device=cuda)
    with pytest.raises(kl.KlError) as e:
        kl.gemm(a, a, torch.zeros(256, 256, dtype=torch.bfloat16, device=cuda), stream_k=2)
    assert e.value.status == kl.KL_ERR_INVALID_ARGUMENT


@pytest.mark.parametrize("a_major,b_major", [(1, 0), (0, 1), (1, 1)], ids=["a_mn", "b_mn", "both_mn"])
def test_mn_major_operands(cuda, a_major, b_major):
    """The split tail on MN-major tiles (A stored [K, M], B stored [K, N]): a K-range starts mid-K."""
    m, n, k = 512, 768, 1024
    a, b, _, _ = random_inputs(m, n, k, "bf16", seed=a_major + 2 * b_major)
    da, db = to_device(a, "bf16", cuda), to_device(b, "bf16", cuda)
    if a_major:
        da = da.t().contiguous()
    if b_major:
        db = db.t().contiguous()
    c = torch.full((m, n), float("nan"), dtype=torch.bfloat16, device=cuda)
    kl.gemm(da, db, c, algo=kl.ALGO_2CTA, a_major=a_major, b_major=b_major, stream_k=1, max_ctas=6)
    torch.cuda.synchronize()
    assert kl.read_status() == 0
    check(c.float().cpu().numpy(), a, b, 1.0, TOL16)


@pytest.mark.parametrize("swizzle", [64, 32])
def test_narrow_swizzle(cuda, swizzle):
    a, b, _, _ = random_inputs(384, 520, 1000, "bf16", seed=swizzle)
    c = run_kl(a, b, "bf16", "f32", cuda, kl.ALGO_1CTA, swizzle=swizzle, stream_k=1, max_ctas=8)
    check(c, a, b, 1.0, TOL16)


def test_f16_inputs(cuda):
    a, b, _, _ = random_inputs(300, 600, 1536, "f16", seed=15)
    c = run_kl(a, b, "f16", "f16", cuda, kl.ALGO_2CTA, stream_k=1, max_ctas=10)
    check(c, a, b, 1.0, TOL16, kind="f16")
