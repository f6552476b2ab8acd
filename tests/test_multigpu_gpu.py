"""N-sharded GEMM on 2+ GPUs of one node (skipped with fewer): every rank computes its column
shard with kl_gemm_gather, whose epilogue also stores the tiles into the other ranks' copies of C
over NVLink; after one collective every rank holds the whole C, equal bit for bit to a single-GPU
kl_gemm of the full problem (whole tiles on both sides), and with the split tail forced on, within
the bf16 tolerance of the fp64 oracle. The same through an NVLink multicast object
(kl_gemm_gather_multicast: one multimem store per tile, the switch writing every rank's C), where
the GPUs offer one."""

import os
import socket
import subprocess
import sys
from pathlib import Path

import pytest

pytestmark = pytest.mark.gpu

ROOT = Path(__file__).resolve().parent.parent

WORKER = r'''
import os, sys, datetime
import numpy as np
import torch
import torch.distributed as dist
sys.path.insert(0, os.environ["KL_ROOT"]); sys.path.insert(0, os.path.join(os.environ["KL_ROOT"], "tests"))
import maia_b200 as kl
from maia_b200 import sharding
from gpu_util import random_inputs, to_device

rank, world = int(os.environ["RANK"]), int(os.environ["WORLD_SIZE"])
torch.cuda.set_device(rank)
dev = torch.device("cuda", rank)
dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=60), device_id=dev)
try:
    # Small N leaves some ranks an empty shard at 4-8 GPUs (256-column boundaries): they compute
    # nothing and still receive the others' tiles.
    for (m, n, k) in [(512, 1024, 768), (384, 1000, 520), (1024, 4096, 1024), (256, 2048 + 72, 640)]:
        a_bits, b_bits, _, _ = random_inputs(m, n, k, "bf16", seed=n + k)
        a, b = to_device(a_bits, "bf16", dev), to_device(b_bits, "bf16", dev)
        # Whole tiles on both sides (stream_k = -1): a shard's tiles are then the full GEMM's tiles.
        ref = kl.gemm(a, b, stream_k=-1)                      # whole problem on this GPU
        lo, hi = sharding.shard_range(n, world, rank, align=256)
        shared = sharding.SharedC(m, n, torch.bfloat16, dev, dist)
        shared.full.fill_(float("nan"))
        dist.barrier()
        kl.gemm_gather(a, b[lo:hi], shared.full[:, lo:hi], shared.peer_ptrs(lo), stream_k=-1)
        dist.barrier()                                        # every rank's kernel has finished
        torch.cuda.synchronize()
        assert kl.read_status() == 0
        assert torch.equal(shared.full.view(torch.int16), ref.view(torch.int16)), f"rank {rank} shape {(m, n, k)}"
        dist.barrier()
        shared.close()
    # The split tail forced on (stream_k = 1): the last arrival at a split tile stores it to every
    # copy of C; checked against the fp64 oracle (the split sums in another order than whole tiles).
    from oracle import gemm as og
    m, n, k = 512, 4096, 2048
    a_bits, b_bits, _, _ = random_inputs(m, n, k, "bf16", seed=77)
    a, b = to_device(a_bits, "bf16", dev), to_device(b_bits, "bf16", dev)
    lo, hi = sharding.shard_range(n, world, rank, align=256)
    shared = sharding.SharedC(m, n, torch.float32, dev, dist)
    shared.full.fill_(float("nan"))
    dist.barrier()
    kl.gemm_gather(a, b[lo:hi], shared.full[:, lo:hi], shared.peer_ptrs(lo), stream_k=1, max_ctas=16)
    dist.barrier()
    torch.cuda.synchronize()
    assert kl.read_status() == 0
    got = shared.full.cpu().numpy()
    assert not np.isnan(got).any(), f"rank {rank}: unwritten entries"
    elem, norm = og.rel_error(got, og.gemm_f64(a_bits, b_bits, 1.0))
    assert elem <= 1e-2 and norm <= 1e-2, f"rank {rank}: split tail {elem:.3e} / {norm:.3e}"
    dist.barrier()
    shared.close()
    # End to end from host memory: each rank brings only its slab of A's rows (the last one short),
    # the ranks all-gather A over NVLink, and B's shard and C's block go through kl_gemm_host_b.
    m, n, k = 1000, 2048, 1024
    a_bits, b_bits, _, _ = random_inputs(m, n, k, "bf16", seed=91)
    lo, hi = sharding.shard_range(n, world, rank, align=256)
    hs = sharding.HostShardedGemm(m, hi - lo, k, torch.bfloat16, torch.float32, dev, dist)
    r0, r1 = hs.slab_rows()
    a_host = torch.from_numpy(a_bits[r0:r1].view(np.int16)).view(torch.bfloat16).pin_memory()
    b_host = torch.from_numpy(np.ascontiguousarray(b_bits[lo:hi]).view(np.int16)).view(torch.bfloat16).pin_memory()
    c_host = torch.full((m, hi - lo), float("nan"), dtype=torch.float32).pin_memory()
    for _ in range(2):
        hs(a_host, b_host, c_host)
        torch.cuda.synchronize()
        assert kl.read_status() == 0
        got = c_host.numpy()
        elem, norm = og.rel_error(got, og.gemm_f64(a_bits, b_bits[lo:hi], 1.0))
        assert not np.isnan(got).any() and elem <= 1e-2 and norm <= 1e-2, f"rank {rank}: host path {elem:.3e}"
    dist.barrier()
finally:
    dist.destroy_process_group()
print("OK", rank)
'''


WORKER_MC = r'''
import os, sys, datetime
import numpy as np
import torch
import torch.distributed as dist
sys.path.insert(0, os.environ["KL_ROOT"]); sys.path.insert(0, os.path.join(os.environ["KL_ROOT"], "tests"))
import maia_b200 as kl
from maia_b200 import sharding
from gpu_util import random_inputs, to_device
from oracle import gemm as og

rank, world = int(os.environ["RANK"]), int(os.environ["WORLD_SIZE"])
torch.cuda.set_device(rank)
dev = torch.device("cuda", rank)
dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=60), device_id=dev)
failures = []
try:
    # Every rank takes the same steps whatever it finds; failures are collected and raised only after
    # the multicast buffer is released by all ranks (no process leaves while bound to it).
    for (m, n, k, out, sk) in [(512, 1024, 768, torch.bfloat16, -1), (384, 1024, 520, torch.float32, -1),
                               (1024, 4096, 1024, torch.bfloat16, -1), (256, 2048 + 64, 640, torch.bfloat16, -1),
                               (512, 4096, 2048, torch.float32, 1)]:
        a_bits, b_bits, _, _ = random_inputs(m, n, k, "bf16", seed=n + k + 1)
        a, b = to_device(a_bits, "bf16", dev), to_device(b_bits, "bf16", dev)
        lo, hi = sharding.shard_range(n, world, rank, align=256)
        mc = sharding.MulticastC(m, n, out, dev, dist)
        if not mc.available:
            print("UNAVAILABLE", rank, mc.reason)
            mc.close()
            break
        mc.full.fill_(float("nan"))
        torch.cuda.synchronize()
        dist.barrier()
        kl.gemm_gather_multicast(a, b[lo:hi], mc.full[:, lo:hi], mc.mc_ptr(lo), stream_k=sk,
                                 max_ctas=16 if sk == 1 else 0)
        torch.cuda.synchronize()
        dist.barrier()                                         # every rank's kernel has finished
        got = mc.full.clone()
        status = kl.read_status()
        mc.close()
        if status != 0:
            failures.append(f"rank {rank} shape {(m, n, k)}: device wait timed out")
            continue
        if sk == -1:
            ref = kl.gemm(a, b, out_dtype=out, stream_k=-1)  # whole problem on this GPU, same tiles
            bits = torch.int16 if out == torch.bfloat16 else torch.int32
            if not torch.equal(got.view(bits), ref.view(bits)):
                failures.append(f"rank {rank} shape {(m, n, k)}: differs from the one-GPU GEMM")
        else:
            c = got.float().cpu().numpy()
            elem, norm = og.rel_error(c, og.gemm_f64(a_bits, b_bits, 1.0))
            if np.isnan(c).any() or elem > 1e-2 or norm > 1e-2:
                failures.append(f"rank {rank} split tail: {elem:.3e} / {norm:.3e}")
    else:
        print("MC-OK", rank)
finally:
    dist.barrier()
    dist.destroy_process_group()
assert not failures, failures
print("OK", rank)
'''


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def test_sharded_gemm_with_fused_gather(cuda, tmp_path):
    import torch

    world = min(torch.cuda.device_count(), 8)
    if world < 2:
        pytest.skip("needs 2+ GPUs")
    script = tmp_path / "worker.py"
    script.write_text(WORKER)
    env = dict(os.environ, KL_ROOT=str(ROOT), NCCL_NVLS_ENABLE="0")
    cmd = [sys.executable, "-m", "torch.distributed.run", "--nnodes=1", f"--nproc-per-node={world}",
           "--master-addr", "127.0.0.1", "--master-port", str(_free_port()), str(script)]
    r = subprocess.run(["timeout", "-k", "30", "300", *cmd], env=env, capture_output=True, text=True)
    assert r.returncode == 0, r.stdout[-3000:] + r.stderr[-3000:]
    assert r.stdout.count("OK") == world


def test_sharded_gemm_with_multicast_gather(cuda, tmp_path):
    import torch

    world = min(torch.cuda.device_count(), 8)
    if world < 2:
        pytest.skip("needs 2+ GPUs")
    script = tmp_path / "worker_mc.py"
    script.write_text(WORKER_MC)
    env = dict(os.environ, KL_ROOT=str(ROOT))
    cmd = [sys.executable, "-m", "torch.distributed.run", "--nnodes=1", f"--nproc-per-node={world}",
           "--master-addr", "127.0.0.1", "--master-port", str(_free_port()), str(script)]
    r = subprocess.run(["timeout", "-k", "30", "300", *cmd], env=env, capture_output=True, text=True)
    assert r.returncode == 0, r.stdout[-3000:] + r.stderr[-3000:]
    assert r.stdout.count("OK") >= world
    if "UNAVAILABLE" in r.stdout:
        pytest.skip("no NVLink multicast on these GPUs: " + r.stdout.split("UNAVAILABLE", 1)[1].splitlines()[0])
    assert r.stdout.count("MC-OK") == world
