"""The N>1 host path on CPU: two gloo ranks shard a GEMM along N, compute their column blocks
with the CPU oracle, take the max of their timings and gather the full C, which must equal the
single-process result bit for bit."""

import os
import socket

import numpy as np
import pytest

from maia_b200 import sharding


def test_shard_ranges_cover_n():
    for n in (1, 7, 8192, 28672, 16385):
        for world in (1, 2, 3, 4, 8):
            spans = [sharding.shard_range(n, world, r) for r in range(world)]
            assert spans[0][0] == 0 and spans[-1][1] == n
            assert all(a[1] == b[0] for a, b in zip(spans, spans[1:]))
            assert max(h - l for l, h in spans) - min(h - l for l, h in spans) <= 1
    with pytest.raises(ValueError):
        sharding.shard_range(10, 2, 2)
    for n, world in ((8192, 8), (1000, 2), (28672, 3), (300, 4)):
        spans = [sharding.shard_range(n, world, r, align=256) for r in range(world)]
        assert spans[0][0] == 0 and spans[-1][1] == n
        assert all(a[1] == b[0] and a[0] <= a[1] for a, b in zip(spans, spans[1:]))
        assert all(lo % 256 == 0 for lo, _ in spans)


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank_main(rank, world, port, out_dir):
    import torch
    import torch.distributed as dist

    from gpu_util import random_inputs
    from oracle import gemm as og

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        m, n, k = 24, 67, 40
        a, b, _, _ = random_inputs(m, n, k, "bf16", seed=21)
        lo, hi = sharding.shard_range(n, world, rank)
        c_shard = torch.from_numpy(og.gemm_f64(a, b[lo:hi], threads=1))
        t = sharding.max_over_ranks(0.5 + rank, dist)
        full = sharding.gather_columns(c_shard, n, dist)
        # The same into a preallocated C, twice (a loop that reuses its buffers).
        out = torch.full((m, n), float("nan"), dtype=c_shard.dtype)
        for _ in range(2):
            got = sharding.gather_columns(c_shard, n, dist, out=out)
            assert got is out and torch.equal(out, full)
        np.save(os.path.join(out_dir, f"rank{rank}.npy"), full.numpy())
        np.save(os.path.join(out_dir, f"t{rank}.npy"), np.array([t]))
    finally:
        dist.destroy_process_group()


def test_two_rank_sharded_gemm_matches_single(tmp_path):
    import torch.multiprocessing as mp

    from gpu_util import random_inputs
    from oracle import gemm as og

    world = 2
    mp.start_processes(_rank_main, args=(world, _free_port(), str(tmp_path)), nprocs=world, start_method="spawn")
    a, b, _, _ = random_inputs(24, 67, 40, "bf16", seed=21)
    ref = og.gemm_f64(a, b, threads=1)
    for r in range(world):
        np.testing.assert_array_equal(np.load(tmp_path / f"rank{r}.npy"), ref)
        assert np.load(tmp_path / f"t{r}.npy")[0] == 1.5  # max over ranks of 0.5 + rank
