"""bench.py's reference arm on the CPU: the JSON line the driver reads (the kl arm's metric, unit,
config and direction; a `cpu_baseline` describing the timed sample; an `e2e` with no copies), on
one process and as rank 1 of a torchrun job (which exits without work)."""

import json
import os
import subprocess
import sys
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parent.parent


def _run(env_extra=None):
    env = dict(os.environ, **(env_extra or {}))
    r = subprocess.run([sys.executable, str(ROOT / "bench.py"), "--impl", "reference", "--workload", "c1_256_bf16_f32",
                        "--steps", "1", "--warmup", "1"], capture_output=True, text=True, env=env, cwd=ROOT,
                       timeout=600)
    assert r.returncode == 0, r.stdout[-2000:] + r.stderr[-2000:]
    return [json.loads(line) for line in r.stdout.splitlines() if line.startswith("{")]


def test_reference_arm_line():
    import bench  # noqa: F401  (importable without a GPU)

    (line,) = _run()
    assert line["impl"] == "reference" and line["metric"] == bench.METRIC
    assert line["unit"] == "TFLOP/s" and line["higher_is_better"] is True and line["n_gpus"] == 1
    assert line["config"]["workload"] == "c1_256_bf16_f32" and line["config"]["m"] == 256
    assert line["value"] > 0 and line["ms_per_step"] > 0
    base = line["cpu_baseline"]
    assert base["kind"] == "port" and base["cores"] >= 1 and base["value"] == line["value"] and base["sample"]
    assert line["e2e"] == {"value": line["value"], "unit": "TFLOP/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}


def test_reference_arm_other_ranks_print_nothing():
    assert _run({"RANK": "1", "WORLD_SIZE": "2"}) == []
