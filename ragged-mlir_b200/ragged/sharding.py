"""Row-sharded calls across the GPUs of one node (one process per GPU).

The reference runs one program on one device (README.md:457-461); this
build adds a sharded form of the row-balanced sum, max and softmax for
inputs that are spread over several GPUs.  Rank r of ``world`` holds rows
``shard_rows(N, world, r)`` of the packed values and the whole offsets
array.  Every rank reduces its rows; a segment cut by a shard boundary
leaves f32 pieces in the rank's edge record; the ranks all-gather the
records (NCCL over NVLink through ``torch.distributed``: a few KB per rank,
the only collective of the path); and the rank that holds a cut segment's
end merges its pieces in rank order.  Each output row is written by exactly
one rank: ``segment_owners`` says which.  Softmax: every rank normalises
its own rows; the (reference, mass) pieces of the segments cut at its edges
are merged from all ranks' records in rank order on every rank that holds
rows of them.

``ShardedProgram`` wraps a compiled sum or max program for one rank;
``CompiledProgram.run_sharded`` is the call it makes.
"""
from __future__ import annotations

from dataclasses import dataclass
from typing import Any, Callable

import numpy as np

from .errors import ValidationError


# Cost of one segment end in rows when balancing a split: an end writes an
# output row and restarts the accumulators.  Measured on 8 B200s with c5 (bf16,
# D=256): the even row split left the rank with the most ends (1.4M) 12%
# slower than a rank inside one segment, a weight of 2.5 left the end-free
# ranks 8% slower; 1.25 sits between.
END_WEIGHT = 1.25


def end_weight_model(op: str, dtype: str, d: int) -> float:
    """Starting weight of a segment end, in rows: an end writes one output
    row and restarts the accumulators, about 128 bytes of streaming on B200
    beyond the row (an earlier hand fit for bf16 D=256 gave 1.25 rows), so
    1 + 128 / row bytes.  Refined from measured rank times by
    ``fit_end_weight``."""
    row_bytes = d * (2 if dtype == "bf16" else 4)
    return 1.0 + 128.0 / row_bytes if op != "softmax" else 128.0 / row_bytes


def window_ends(offsets: np.ndarray, world: int, splits) -> list[int]:
    """Segment ends each rank's window consumes (ends in (row0, row1], and
    on rank 0 also the ends at row 0)."""
    offsets = np.asarray(offsets, dtype=np.int64)
    n = int(offsets[-1])
    ends = offsets[1:]
    counts = []
    for rank in range(world):
        row0, row1 = shard_rows(n, world, rank, splits)
        lo = 0 if rank == 0 else int(np.searchsorted(ends, row0, side="right"))
        counts.append(int(np.searchsorted(ends, row1, side="right")) - lo)
    return counts


def fit_end_weight(rows, ends, times_ms, fallback: float) -> tuple[float, dict]:
    """End weight from measured per-rank times of the local phase: the
    least-squares fit t = a * rows + e * ends over the ranks (a, e >= 0),
    weight e / a.  No fixed term: under a split that already balances
    rows + w * ends, the ranks' rows and ends lie on a line, and a fixed
    term would make the weight unidentifiable (a rank's fixed cost, a few
    launches, is about 1 % of a c5 window's time).  Needs at least four ranks
    with different mixes of rows and ends; otherwise ``fallback`` is
    returned."""
    rows = np.asarray(rows, dtype=np.float64)
    ends = np.asarray(ends, dtype=np.float64)
    times = np.asarray(times_ms, dtype=np.float64)
    info = {"ranks": len(times)}
    if len(times) < 4 or np.ptp(ends) == 0 or np.ptp(rows) == 0:
        return fallback, {**info, "fit": "not enough distinct ranks; model weight kept"}
    from scipy.optimize import nnls
    a = np.stack([rows / 1e6, ends / 1e6], axis=1)
    coef, residual = nnls(a, times)
    if coef[0] <= 0:
        return fallback, {**info, "fit": "no per-row cost in the fit; model weight kept"}
    weight = float(np.clip(coef[1] / coef[0], 0.0, 64.0))
    return weight, {**info, "fit": "least squares over ranks", "ms_per_mrow": round(float(coef[0]), 5),
                    "ms_per_mend": round(float(coef[1]), 5), "residual_ms": round(float(residual), 5)}


def shard_rows(n: int, world: int, rank: int, splits=None) -> tuple[int, int]:
    """Rows [row0, row1) of ``rank``: from ``splits`` (world + 1 row
    boundaries, e.g. ``balanced_split``) or the even row split (the split
    libragged_b200's rg_shard_rows computes)."""
    if n < 0 or world < 1 or not 0 <= rank < world:
        raise ValidationError("need n >= 0, world >= 1 and 0 <= rank < world")
    if splits is not None:
        if len(splits) != world + 1 or splits[0] != 0 or splits[-1] != n:
            raise ValidationError("a split has world + 1 boundaries from 0 to n")
        return int(splits[rank]), int(splits[rank + 1])
    q, rem = divmod(n, world)
    row0 = q * rank + min(rank, rem)
    return row0, row0 + q + (1 if rank < rem else 0)


def balanced_split(offsets: np.ndarray, world: int, end_weight: float = END_WEIGHT) -> list[int]:
    """Row boundaries giving every rank about the same rows + end_weight x
    segment ends (NumPy restatement of rg_shard_split; host offsets)."""
    offsets = np.asarray(offsets, dtype=np.int64)
    n, b = int(offsets[-1]), offsets.size - 1
    ends = offsets[1:]
    total = n + end_weight * b
    splits = [0]
    for k in range(1, world):
        target = total * k / world
        lo, hi = splits[-1], n
        while lo < hi:
            mid = (lo + hi) // 2
            cost = mid + end_weight * int(np.searchsorted(ends, mid, side="right"))
            if cost >= target:
                hi = mid
            else:
                lo = mid + 1
        splits.append(lo)
    splits.append(n)
    return splits


def segment_owners(offsets: np.ndarray, world: int, splits=None) -> np.ndarray:
    """Rank that writes each segment's output row: the rank whose rows
    hold the segment's end (segments ending at row 0 belong to rank 0)."""
    offsets = np.asarray(offsets, dtype=np.int64)
    n = int(offsets[-1])
    ends = np.array([shard_rows(n, world, r, splits)[1] for r in range(world)], dtype=np.int64)
    return np.searchsorted(ends, offsets[1:], side="left").astype(np.int64)


def torch_exchange(group=None) -> Callable[[Any], Any]:
    """All-gather of edge records over ``group`` (torch.distributed; NCCL on
    GPUs): returns the records of ranks 0..world-1 concatenated."""
    import torch
    import torch.distributed as dist

    def exchange(edges):
        world = dist.get_world_size(group)
        gathered = torch.empty((world * edges.numel(),), dtype=edges.dtype, device=edges.device)
        dist.all_gather_into_tensor(gathered, edges, group=group)
        return gathered

    return exchange


@dataclass
class ShardedProgram:
    """A sum or max program bound to one rank of a row-sharded call."""

    program: Any
    world: int
    rank: int
    group: Any = None
    splits: Any = None

    def rows(self, n: int) -> tuple[int, int]:
        return shard_rows(n, self.world, self.rank, self.splits)

    def run(self, values, offsets, out, *, total_rows: int, stream=None, offsets_host=None):
        return self.program.run_sharded(values, offsets, out, total_rows=total_rows, world=self.world, rank=self.rank,
                                        exchange=torch_exchange(self.group), stream=stream, splits=self.splits,
                                        offsets_host=offsets_host)
