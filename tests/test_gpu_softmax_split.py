"""Split-class softmax segments on the classified schedule's pipelined worker.

Segments of at most 64 one-stage chunks are normalised inside the worker:
the team holding a chunk publishes its statistics, waits (bounded) for the
segment's other chunks, merges them and normalises the chunk from its
shared-memory stage.  Longer segments, and any chunk whose wait gives up,
are normalised by split_normalize_kernel from the statistics the segment's
last chunk leaves.  Both routes must match the oracle, including a run in
which every wait gives up at once (RAGGED_B200_CHUNK_WAIT_POLLS=0); the
two runs may round differently (the worker scales the terms its mass pass
kept in the stage, the normalise kernel recomputes them), each within one
ulp of the rounded exact value.
"""
from __future__ import annotations

import os
from pathlib import Path
import subprocess
import sys

import numpy as np
import pytest

from helpers import check, offsets_of, prepared, run_device

pytestmark = pytest.mark.gpu

REPO = Path(__file__).resolve().parents[1]


def _item_rows(cuda, dtype, d):
    lengths = np.array([5000, 3], dtype=np.int64)
    offsets = offsets_of(lengths)
    values = prepared(np.zeros((int(offsets[-1]), d)), dtype)
    _, report = run_device(cuda, "softmax", dtype, values, offsets, select="classified")
    return int(report.thresholds[1])


def _case(item_rows, d, dtype, seed):
    """Split segments of 2..63 chunks (normalised in the worker), one of 70
    chunks (left to the normalise kernel), segments ending mid-chunk and on
    a chunk boundary, between short and empty ones."""
    rng = np.random.default_rng(seed)
    lengths = []
    for chunks in (2, 3, 7, 16, 33, 63):
        lengths += [chunks * item_rows - int(rng.integers(0, item_rows // 2)), 0, int(rng.integers(1, 40))]
    lengths += [5 * item_rows, 70 * item_rows + 11, int(rng.integers(40, item_rows)), 0]
    offsets = offsets_of(np.array(lengths, dtype=np.int64))
    values = prepared(rng.normal(scale=3.0, size=(int(offsets[-1]), d)), dtype)
    return values, offsets


@pytest.mark.parametrize("dtype,d", [("bf16", 128), ("f32", 64), ("bf16", 256)])
def test_split_softmax_in_worker_and_late(cuda, dtype, d):
    item_rows = _item_rows(cuda, dtype, d)
    values, offsets = _case(item_rows, d, dtype, seed=d)
    actual, report = run_device(cuda, "softmax", dtype, values, offsets, select="classified")
    assert report.kernel_names == ("classify", "classified_worker", "split_normalize")
    check(actual, values, offsets, "softmax", dtype)


@pytest.mark.parametrize("dtype", ["f32", "bf16"])
def test_kept_terms_keep_special_columns(cuda, dtype):
    """Columns with NaN, +inf, only -inf, and -inf next to finite values in
    run segments and split chunks: the kept-term normalisation must give the
    oracle's NaN columns and exact zeros."""
    item_rows = _item_rows(cuda, dtype, 64)
    lengths = np.array([40, 3 * item_rows + 7, 1, 17, 0], dtype=np.int64)
    offsets = offsets_of(lengths)
    rng = np.random.default_rng(71)
    values = rng.normal(scale=4.0, size=(int(offsets[-1]), 64))
    firsts = offsets[:-1][lengths > 0]
    values[firsts, 0] = np.nan       # a NaN column in every segment
    values[firsts, 1] = np.inf       # +inf: NaN column
    values[firsts, 3] = -np.inf      # -inf beside finite values: exact zeros
    values[:40, 2] = -np.inf         # the first segment's column all -inf: NaN
    values[:, 4] = -np.inf           # every segment all -inf in this column
    values = prepared(values, dtype)
    actual, _ = run_device(cuda, "softmax", dtype, values, offsets, select="classified")
    check(actual, values, offsets, "softmax", dtype)


_CHILD = r"""
import sys
import numpy as np
sys.path[:0] = [sys.argv[1], sys.argv[1] + "/ragged-mlir_b200", sys.argv[1] + "/tests"]
from helpers import run_device
import torch
data = np.load(sys.argv[2])
actual, _ = run_device(torch, "softmax", sys.argv[3], data["values"], data["offsets"], select="classified")
np.save(sys.argv[4], actual)
"""


def test_every_wait_giving_up_still_matches(cuda, tmp_path):
    """With RAGGED_B200_CHUNK_WAIT_POLLS=0 every chunk of an in-worker segment
    that is not the last to publish goes to split_normalize_kernel; both
    runs match the oracle (and so each other within two bf16 ulps)."""
    from oracle import reference_port as rp
    item_rows = _item_rows(cuda, "bf16", 128)
    values, offsets = _case(item_rows, 128, "bf16", seed=5)
    inputs = tmp_path / "inputs.npz"
    np.savez(inputs, values=values, offsets=offsets)
    outputs = {}
    for polls in ("0", None):
        env = dict(os.environ)
        env.pop("RAGGED_B200_CHUNK_WAIT_POLLS", None)
        if polls is not None:
            env["RAGGED_B200_CHUNK_WAIT_POLLS"] = polls
        target = tmp_path / f"out_{polls}.npy"
        result = subprocess.run([sys.executable, "-c", _CHILD, str(REPO), str(inputs), "bf16", str(target)],
                                env=env, capture_output=True, text=True, timeout=600)
        assert result.returncode == 0, result.stderr[-3000:]
        outputs[polls] = np.load(target)
    for output in outputs.values():
        check(output, values, offsets, "softmax", "bf16")
    late, default = outputs["0"], outputs[None]
    finite = np.isfinite(default)
    np.testing.assert_array_equal(np.isnan(late), np.isnan(default))
    assert np.all(np.abs(late[finite] - default[finite]) <= 2 * rp.bf16_ulp(default[finite]))
