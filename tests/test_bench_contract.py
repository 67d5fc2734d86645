"""bench.py's reference arm on the host (no GPU): the JSON line the round
driver parses, and the rule that only rank 0 of a multi-rank launch runs it.
The arm times the reference's CPU path (torch.segment_reduce on CPU and the
float64 C oracle, the faster reported), so it runs here; the GPU arm is
covered by the GPU tests.
"""
from __future__ import annotations

import json
import os
from pathlib import Path
import subprocess
import sys

import pytest

REPO = Path(__file__).resolve().parents[1]


def run_bench(*args: str, env: dict | None = None) -> subprocess.CompletedProcess:
    full_env = {**os.environ, **(env or {})}
    return subprocess.run([sys.executable, str(REPO / "bench.py"), *args], cwd=REPO, env=full_env,
                          capture_output=True, text=True, timeout=300)


@pytest.fixture(scope="module")
def reference_line():
    # 200 steps bound the oracle's timing to about one second.
    result = run_bench("--impl", "reference", "--workload", "c1", "--scale", "0.01", "--steps", "200",
                       "--warmup", "3")
    assert result.returncode == 0, result.stderr[-2000:]
    lines = [line for line in result.stdout.splitlines() if line.strip()]
    assert len(lines) == 1, result.stdout
    return json.loads(lines[0])


def test_reference_line_has_every_contract_key(reference_line):
    line = reference_line
    assert line["impl"] == "reference"
    for key in ("metric", "value", "unit", "n_gpus", "steps", "warmup", "ms_per_step", "higher_is_better",
                "scaling", "vs_baseline", "dtype", "data", "config", "cpu_baseline", "e2e"):
        assert key in line, key
    assert line["value"] > 0 and line["unit"] == "GB/s" and line["higher_is_better"] is True
    assert (line["n_gpus"], line["steps"], line["warmup"]) == (1, 200, 3)
    assert line["config"]["workload"] == "c1" and line["data"] == "synthetic"
    assert set(line["cpu_baseline"]) == {"value", "unit", "cores", "kind", "sample"}
    assert line["cpu_baseline"]["value"] == line["value"] and line["cpu_baseline"]["kind"] == "port"
    assert line["cpu_baseline"]["cores"] >= 1
    assert line["e2e"] == {"value": line["value"], "unit": "GB/s", "h2d_bytes_per_step": 0,
                           "d2h_bytes_per_step": 0}
    # Both CPU implementations were timed; the line is the one a probe call
    # found faster, over exactly `steps` calls (the other over 3).
    legs = line["legs"]
    assert set(legs) == {"torch", "oracle"}
    timed = [name for name in legs if legs[name]["calls"] == line["steps"]]
    assert len(timed) == 1 and legs[timed[0]]["value"] == line["value"]


def test_reference_arm_uses_every_host_core_under_torchrun():
    """torchrun sets OMP_NUM_THREADS=1; the CPU baseline still runs on every
    core of the process's affinity, at every rank count."""
    result = run_bench("--impl", "reference", "--workload", "c1", "--scale", "0.01", "--gpus", "4", "--steps", "5",
                       "--warmup", "1", env={"RANK": "0", "WORLD_SIZE": "4", "LOCAL_RANK": "0",
                                             "OMP_NUM_THREADS": "1"})
    assert result.returncode == 0, result.stderr[-2000:]
    line = json.loads(result.stdout.strip().splitlines()[-1])
    assert line["cpu_baseline"]["cores"] == len(os.sched_getaffinity(0))
    assert line["n_gpus"] == 4 and line["steps"] == 5


def test_reference_metric_matches_the_gpu_arm(reference_line):
    sys.path.insert(0, str(REPO))
    import bench
    assert reference_line["metric"] == bench.metric_name()


def test_only_rank_zero_runs_the_reference_arm():
    result = run_bench("--impl", "reference", "--workload", "c1", "--scale", "0.01", "--gpus", "2", "--steps",
                       "200", "--warmup", "3", env={"RANK": "1", "WORLD_SIZE": "2", "LOCAL_RANK": "1"})
    assert result.returncode == 0, result.stderr[-2000:]
    assert result.stdout.strip() == ""


def test_split_refit_from_rank_times():
    """The sharded bench's split refit (world >= 4), host half: rank times
    generated with a known end weight give that weight back, and the new
    split balances rows + weight x ends; too few ranks keep the model weight."""
    sys.path.insert(0, str(REPO))
    import numpy as np
    import bench
    from ragged import workloads
    from ragged.sharding import balanced_split, shard_rows, window_ends
    w = workloads.make("c5", scale=0.001)
    offsets = w.offsets().astype(np.int64)
    world = 8
    splits = balanced_split(offsets, world, 1.0)
    rows = [shard_rows(w.n, world, r, splits)[1] - shard_rows(w.n, world, r, splits)[0] for r in range(world)]
    ends = window_ends(offsets, world, splits)
    true_weight = 6.0
    times = [1e-6 * (r + true_weight * e) for r, e in zip(rows, ends)]
    fitted, info, new_splits = bench.split_from_rank_times(w.n, offsets, world, splits, times, 1.25)
    assert abs(fitted - true_weight) < 0.05 * true_weight, info
    assert list(new_splits) == list(balanced_split(offsets, world, fitted))
    kept, info, _ = bench.split_from_rank_times(w.n, offsets, 2, None, times[:2], 1.25)
    assert kept == 1.25 and "kept" in info["fit"]
