"""The JSON contract of `bench.py --impl reference` (the CPU arm the driver
runs beside the GPU arm), checked on the CPU: one line from rank 0 with the
same metric and config as the GPU arm, a cpu_baseline object describing the
run and an e2e object with no host-device bytes; the other ranks of a
torchrun launch print nothing and exit 0."""
from __future__ import annotations

import json
import os
import subprocess
import sys
from pathlib import Path

import pytest

REPO = Path(__file__).resolve().parents[1]
sys.path.insert(0, str(REPO))

import bench  # noqa: E402


def _run(args, env_extra=None):
    env = dict(os.environ)
    env.update(env_extra or {})
    return subprocess.run([sys.executable, str(REPO / "bench.py"), *args], cwd=REPO, env=env,
                          capture_output=True, text=True, timeout=600)


def test_reference_arm_line_matches_contract():
    r = _run(["--impl", "reference", "--steps", "1", "--warmup", "3"])
    assert r.returncode == 0, r.stderr[-2000:]
    lines = [ln for ln in r.stdout.splitlines() if ln.strip()]
    line = json.loads(lines[-1])
    assert line["impl"] == "reference"
    assert line["metric"] == bench.metric_name("cfg1")
    assert line["config"] == bench.workload_config("cfg1", 1)
    assert line["unit"] == "TFLOP/s" and line["higher_is_better"] is True
    assert line["n_gpus"] == 1 and line["steps"] == 1 and line["warmup"] == 3
    assert line["value"] > 0 and line["ms_per_step"] > 0
    cpu = line["cpu_baseline"]
    assert set(cpu) >= {"value", "unit", "cores", "kind", "sample"}
    assert cpu["kind"] in ("reference", "port") and cpu["cores"] >= 1
    assert cpu["value"] == pytest.approx(line["value"])
    e2e = line["e2e"]
    assert e2e["h2d_bytes_per_step"] == 0 and e2e["d2h_bytes_per_step"] == 0
    assert e2e["value"] == pytest.approx(line["value"]) and e2e["unit"] == line["unit"]


def test_reference_arm_other_ranks_print_nothing():
    r = _run(["--impl", "reference", "--gpus", "2", "--steps", "1", "--warmup", "3"],
             {"RANK": "1", "WORLD_SIZE": "2", "LOCAL_RANK": "1"})
    assert r.returncode == 0, r.stderr[-2000:]
    assert r.stdout.strip() == ""


@pytest.mark.parametrize("world", [1, 2, 8])
def test_large_workload_configs_name_the_default_paths(world):
    """Configs 4 and 5: both arms print large_workload_config; for config 5 its
    default describes the packed column-sharded path that ColumnShardedPolar
    runs by default."""
    cfg5 = bench.large_workload_config("cfg5", world)
    assert "BASELINE config 5" in cfg5["workload"]
    if world > 1:
        assert cfg5["parallelism"].startswith(f"column-sharded x{world}: packed")
    else:
        assert cfg5["parallelism"] == "single GPU"
    cfg4 = bench.large_workload_config("cfg4", world)
    assert "BASELINE config 4" in cfg4["workload"]
    assert cfg4["parallelism"].startswith(f"batch-sharded x{world}")
