"""Failure detection of the N-sharded path on the host, with gloo ranks on the CPU: a rank that
leaves between steps (exits, raises, or says it leaves) is noticed by the others at their next
step's check-in, within the deadline and before they launch anything (sharding.StepGuard)."""

import os
import socket
import time

import pytest

from maia_b200 import sharding


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank_main(rank, world, port, out_dir, how):
    import datetime

    import torch
    import torch.distributed as dist

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=30))
    guard = sharding.StepGuard(dist, timeout_s=2.0, prefix=f"test/{how}")
    result = "none"
    try:
        # Step 0: everyone is there; the step's work is a collective over the group.
        guard.check(0)
        t = torch.tensor([float(rank)])
        dist.all_reduce(t)
        assert t.item() == sum(range(world))
        if rank == world - 1:
            # The last rank leaves between steps, with nothing in flight.
            if how == "leave":
                guard.leave()
                result = "left"
                return
            if how == "raise":
                raise RuntimeError("planted failure on the host")
            result = "exited"
            return  # "exit": stops checking in without a word
        t0 = time.monotonic()
        try:
            guard.check(1)
            result = "not detected"
        except sharding.RankLost as e:
            dt = time.monotonic() - t0
            result = f"lost missing={e.missing} left={e.left} dt={dt:.2f}"
    except RuntimeError as e:
        result = f"raised {e}"
    finally:
        with open(os.path.join(out_dir, f"{how}{rank}.txt"), "w") as f:
            f.write(result)
        # Ranks do not tear the group down together here: the store (rank 0) outlives the others.
        if rank == 0:
            time.sleep(0.5)


@pytest.mark.parametrize("how", ["exit", "raise", "leave"])
def test_survivors_notice_a_rank_that_left(tmp_path, how):
    import torch.multiprocessing as mp

    world = 3
    ctx = mp.start_processes(_rank_main, args=(world, _free_port(), str(tmp_path), how), nprocs=world,
                             start_method="spawn", join=False)
    while not ctx.join(timeout=60):
        pass
    for r in range(world - 1):
        text = (tmp_path / f"{how}{r}.txt").read_text()
        assert text.startswith("lost"), text
        dt = float(text.split("dt=")[1])
        if how == "leave":
            assert "left=[2]" in text and dt < 1.0, text       # seen at once
        else:
            assert "missing=[2]" in text and 1.9 <= dt < 4.0, text  # seen at the 2 s deadline
    last = (tmp_path / f"{how}{world - 1}.txt").read_text()
    assert last == {"exit": "exited", "raise": "raised planted failure on the host", "leave": "left"}[how]


def test_all_present_passes_quickly(tmp_path):
    """No rank missing: the check-in of every step returns as soon as the last rank arrives."""
    import torch.multiprocessing as mp

    mp.start_processes(_steady, args=(2, _free_port(), str(tmp_path)), nprocs=2, start_method="spawn")
    for r in range(2):
        assert float((tmp_path / f"steady{r}.txt").read_text()) < 1.0


def _steady(rank, world, port, out_dir):
    import torch.distributed as dist

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    guard = sharding.StepGuard(dist, timeout_s=5.0, prefix="test/steady")
    t0 = time.monotonic()
    for step in range(20):
        guard.check(step)
    dt = time.monotonic() - t0
    with open(os.path.join(out_dir, f"steady{rank}.txt"), "w") as f:
        f.write(str(dt))
    dist.barrier()
    dist.destroy_process_group()
