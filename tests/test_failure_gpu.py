"""Failure detection on 2 GPUs (skipped with fewer): a rank leaves between steps, with none of its
kernels or collectives in flight. The survivor (a) notices it at the next step's check-in, before
launching anything (sharding.StepGuard on the process group's store), and (b) when it launches the
step's all-gather anyway, the bounded wait of the kl_comm communicator ends it with KL_ERR_TIMEOUT
or KL_ERR_NCCL within the deadline, aborts the communicator, and the GPU stream stays usable (a GEMM
afterwards is checked against torch). NVLS is off for NCCL; nothing here uses multicast memory, and
no kernel is made to fault, trap or hang: the only wait that runs out is NCCL's, ended by its abort."""

import os
import socket
import subprocess
import sys
from pathlib import Path

import pytest

pytestmark = pytest.mark.gpu

ROOT = Path(__file__).resolve().parent.parent

WORKER = r'''
import os, sys, time, datetime
import torch
import torch.distributed as dist
sys.path.insert(0, os.environ["KL_ROOT"])
import maia_b200 as kl
from maia_b200 import sharding

rank, world = int(os.environ["RANK"]), int(os.environ["WORLD_SIZE"])
torch.cuda.set_device(rank)
dev = torch.device("cuda", rank)
dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=30), device_id=dev)
guard = sharding.StepGuard(dist, timeout_s=3.0, prefix="gpu-failure")
comm = sharding.Comm(dist, dev, timeout_ms=60000)
send = torch.full((4096,), float(rank + 1), device=dev)
recv = torch.empty((world * 4096,), device=dev)

# Step 0: all ranks present.
guard.check(0)
comm.all_gather(send, recv)
comm.wait(20000)
ok0 = all(bool((recv[r * 4096:(r + 1) * 4096] == r + 1).all()) for r in range(world))
print(f"STEP0 {rank} {ok0}", flush=True)

if rank == world - 1:
    torch.cuda.synchronize()
    guard.leave()
    print(f"LEFT {rank}", flush=True)
    os._exit(0)

# (a) The next check-in names the rank that left, before anything of step 1 is launched.
t0 = time.monotonic()
try:
    guard.check(1)
    print(f"A {rank} not-detected", flush=True)
except sharding.RankLost as e:
    print(f"A {rank} detected left={e.left} dt={time.monotonic() - t0:.2f}", flush=True)

# (b) The all-gather launched anyway: the bounded wait ends it and aborts the communicator.
t0 = time.monotonic()
status = "completed"
try:
    comm.all_gather(send, recv)
    comm.wait(3000)
except kl.KlError as e:
    status = {kl.KL_ERR_TIMEOUT: "timeout", kl.KL_ERR_NCCL: "nccl"}.get(e.status, f"status{e.status}")
dt = time.monotonic() - t0
print(f"B {rank} {status} aborted={comm.aborted} dt={dt:.2f}", flush=True)

# The stream still works after the abort.
torch.cuda.synchronize()
a = torch.randn((512, 256), device=dev).to(torch.bfloat16)
b = torch.randn((512, 256), device=dev).to(torch.bfloat16)
c = kl.gemm(a, b, out_dtype=torch.float32)
ref = a.float() @ b.float().T
err = float((c - ref).abs().max() / ref.abs().max())
print(f"C {rank} gemm_err={err:.2e} status={kl.read_status()}", flush=True)
comm.close()
os._exit(0)  # the group's other rank is gone: no collective teardown
'''


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def test_rank_leaving_between_steps_is_detected(cuda, tmp_path):
    import torch

    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    script = tmp_path / "worker.py"
    script.write_text(WORKER)
    env = dict(os.environ, KL_ROOT=str(ROOT), NCCL_NVLS_ENABLE="0")
    cmd = [sys.executable, "-m", "torch.distributed.run", "--nnodes=1", "--nproc-per-node=2",
           "--master-addr", "127.0.0.1", "--master-port", str(_free_port()), str(script)]
    r = subprocess.run(["timeout", "-k", "30", "180", *cmd], env=env, capture_output=True, text=True)
    out = r.stdout
    assert "STEP0 0 True" in out and "STEP0 1 True" in out, out[-3000:] + r.stderr[-3000:]
    assert "LEFT 1" in out, out[-3000:]
    a = [l for l in out.splitlines() if l.startswith("A 0")]
    assert a and "detected left=[1]" in a[0], out[-3000:]
    b = [l for l in out.splitlines() if l.startswith("B 0")]
    assert b and (" timeout " in b[0] or " nccl " in b[0]) and "aborted=True" in b[0], out[-3000:] + r.stderr[-3000:]
    assert float(b[0].split("dt=")[1]) < 15.0, b[0]
    c = [l for l in out.splitlines() if l.startswith("C 0")]
    assert c and float(c[0].split("gemm_err=")[1].split()[0]) < 1e-2 and c[0].endswith("status=0"), out[-3000:]
