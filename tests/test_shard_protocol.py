"""The multi-GPU sharding protocol on CPU ranks (gloo, world sizes 2 and 3).

Each rank restates, in float64 NumPy, what rg_run_shard and rg_shard_combine
do on its GPU: it owns rows ``shard_rows(N, world, rank)``; it finishes the
segments whose end lies in its rows (ends in (row0, row1], or [0, row1] on
rank 0) and that started there; it publishes an edge record with the piece of
the segment open at its start (``head``) and the one open at its end
(``tail``); the records are all-gathered (gloo here, NCCL on GPUs); and the
rank that consumed a cut segment's end merges the pieces in rank order.  The
union of what the ranks write must be every segment exactly once and equal
the oracle.  The shard split must match libragged_b200's rg_shard_rows
(callable without a GPU).
"""
from __future__ import annotations

import os
import socket

import numpy as np
import pytest

from helpers import make_lengths, offsets_of

HEADER = 3  # head_seg, head_ends, tail_seg


def _reduce(op, rows):
    if rows.shape[0] == 0:
        return np.zeros(rows.shape[1]) if op == "sum" else np.full(rows.shape[1], -np.inf)
    if op == "sum":
        return rows.sum(axis=0)
    out = rows.max(axis=0)
    out[np.isnan(rows).any(axis=0)] = np.nan
    return out


def _merge(op, a, b):
    if op == "sum":
        return a + b
    out = np.maximum(a, b)
    out[np.isnan(a) | np.isnan(b)] = np.nan
    return out


def rank_part(op, values_local, offsets, row0, row1, rank):
    """(finished {segment: row}, edge record) of one rank's window."""
    b = offsets.size - 1
    ends = offsets[1:]
    lo = 0 if rank == 0 else int(np.searchsorted(ends, row0, side="right"))  # first end consumed here
    hi = int(np.searchsorted(ends, row1, side="right"))                       # ends <= row1
    finished, head_seg, head_ends, head = {}, -1, 0, None
    for s in range(lo, hi):
        start, end = int(offsets[s]), int(offsets[s + 1])
        rows = values_local[max(start, row0) - row0:end - row0]
        if start >= row0:
            finished[s] = _reduce(op, rows)
        else:  # started on an earlier rank: this rank holds its head piece
            head_seg, head_ends, head = s, 1, _reduce(op, rows)
    tail_seg, tail = -1, None
    if hi < b and row1 > row0:
        s = hi  # the segment open at row1 (its end lies beyond)
        start = int(offsets[s])
        if start < row1:
            rows = values_local[max(start, row0) - row0:row1 - row0]
            if start >= row0:
                tail_seg, tail = s, _reduce(op, rows)
            elif head_seg < 0:  # through: the segment covers the whole window
                head_seg, head_ends, head = s, 0, _reduce(op, rows)
    d = values_local.shape[1]
    ident = np.zeros(d) if op == "sum" else np.full(d, -np.inf)
    record = np.concatenate([[head_seg, head_ends, tail_seg],
                             head if head is not None else ident, tail if tail is not None else ident])
    return finished, record


def combine(op, records, rank, d):
    """The segment this rank finishes from the gathered records, or None."""
    head_seg, head_ends = int(records[rank][0]), int(records[rank][1])
    if head_seg < 0 or head_ends == 0:
        return None
    def passes(j):  # the segment runs through rank j, or rank j holds no rows (records nothing)
        through = int(records[j][0]) == head_seg and int(records[j][1]) == 0
        return through or (int(records[j][0]) < 0 and int(records[j][2]) < 0)

    k = rank - 1
    while k >= 0 and passes(k):
        k -= 1
    head = lambda j: records[j][HEADER:HEADER + d]
    tail = lambda j: records[j][HEADER + d:]
    ident = np.zeros(d) if op == "sum" else np.full(d, -np.inf)
    total = tail(k) if k >= 0 and int(records[k][2]) == head_seg else ident
    for j in range(k + 1, rank):
        if int(records[j][0]) == head_seg:
            total = _merge(op, total, head(j))
    return head_seg, _merge(op, total, head(rank))


def _worker(rank, world, port, cases, results):
    import torch
    import torch.distributed as dist
    from ragged.sharding import shard_rows
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        out = []
        for op, values, offsets, split in cases:
            n = int(offsets[-1])
            splits = _split_of(split, offsets, world)
            row0, row1 = shard_rows(n, world, rank, splits)
            finished, record = rank_part(op, values[row0:row1], offsets, row0, row1, rank)
            mine = torch.from_numpy(record)
            gathered = [torch.empty_like(mine) for _ in range(world)]
            dist.all_gather(gathered, mine)
            extra = combine(op, [g.numpy() for g in gathered], rank, values.shape[1])
            if extra is not None:
                finished[extra[0]] = extra[1]
            out.append(finished)
        results[rank] = out
    finally:
        dist.destroy_process_group()


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _cases():
    rng = np.random.default_rng(5)
    cases = []
    for op in ("sum", "max"):
        lengths = make_lengths("long_tail", 60, 5000, seed=3)
        offsets = offsets_of(lengths)
        cases.append((op, rng.normal(size=(int(offsets[-1]), 4)), offsets))
        # A segment through whole shards, ends on shard boundaries, empty segments there.
        lengths = np.array([0, 3, 997, 0, 0, 1500, 498, 2, 0], dtype=np.int64)
        offsets = offsets_of(lengths)
        values = rng.normal(size=(int(offsets[-1]), 3))
        values[10, 1] = np.nan
        cases.append((op, values, offsets))
        cases.append((op, rng.normal(size=(2, 2)), np.array([0, 0, 2, 2], dtype=np.int64)))  # more ranks than rows
    out = [(op, values, offsets, split) for op, values, offsets in cases for split in (None, "balanced")]
    # Ranks with no rows inside one segment: repeated split boundaries (given
    # explicitly, and as the balanced split of a 3-row segment makes them).
    for op in ("sum", "max"):
        values = rng.normal(size=(3, 2))
        out.append((op, values, np.array([0, 3], dtype=np.int64), "repeat"))
        out.append((op, values, np.array([0, 3], dtype=np.int64), "balanced"))
        out.append((op, rng.normal(size=(5, 2)), np.array([0, 1, 4, 4, 5], dtype=np.int64), "repeat"))
    return out


def _split_of(split, offsets, world):
    """None (even rows), "balanced" or "repeat": every rank but the last gets
    at most one row and repeated boundaries leave ranks without rows."""
    from ragged.sharding import balanced_split
    if split == "balanced":
        return balanced_split(offsets, world)
    if split == "repeat":
        n = int(offsets[-1])
        return [0] + [min(n, (k + 1) // 2) for k in range(1, world)] + [n]
    return None


@pytest.mark.parametrize("world", [2, 3])
def test_sharding_protocol_over_gloo(world):
    import torch.multiprocessing as mp
    from oracle import reference_port as rp
    from ragged.sharding import segment_owners
    cases = _cases()
    manager = mp.get_context("spawn").Manager()
    results = manager.dict()
    mp.start_processes(_worker, args=(world, _free_port(), cases, results), nprocs=world, start_method="spawn")
    for i, (op, values, offsets, split) in enumerate(cases):
        owners = segment_owners(offsets, world, _split_of(split, offsets, world))
        seen = {}
        for rank in range(world):
            for s, row in results[rank][i].items():
                assert s not in seen, f"segment {s} written twice"
                assert owners[s] == rank, f"segment {s} written by rank {rank}, owner {owners[s]}"
                seen[s] = row
        assert sorted(seen) == list(range(offsets.size - 1)), "every segment is written exactly once"
        actual = np.stack([seen[s] for s in range(offsets.size - 1)])
        with np.errstate(all="ignore"):
            expected = rp.REFERENCES[op](values, offsets)
        np.testing.assert_allclose(actual, expected, rtol=1e-12, atol=1e-12, equal_nan=True)


def test_shard_rows_matches_native_library():
    from ragged import _native
    from ragged.sharding import shard_rows
    _native.library()
    for n in (0, 1, 7, 10, 200_000_000, 2**40 + 3):
        for world in (1, 2, 3, 8):
            for rank in range(world):
                assert shard_rows(n, world, rank) == _native.shard_rows(n, world, rank)
    assert _native.shard_edge_bytes("sum", 256) % 16 == 0 and _native.shard_edge_bytes("max", 3) % 16 == 0


# ---------------------------------------------------------------- softmax
#
# Each rank keeps (reference m, mass s) statistics, s relative to m, for the
# segments finished in its rows; the segment open at its first row (HEAD, or
# THROUGH when it covers every row) and the one that starts in its rows and is
# open at its last (TAIL) go to its edge record.  After the all-gather every
# rank merges, in rank order, the pieces of ITS cut segments from all ranks'
# records (a starting rank's TAIL piece, then the pieces of the ranks the
# segment covers) and normalises its own rows.

def _stats(rows):
    d = rows.shape[1]
    if rows.shape[0] == 0:
        return np.full(d, -np.inf), np.zeros(d)
    with np.errstate(all="ignore"):
        m = rows.max(axis=0)
        m[np.isnan(rows).any(axis=0)] = np.nan
        base = np.where(m == -np.inf, 0.0, m)
        s = np.exp(rows - base).sum(axis=0)
    return m, s


def _smerge(a, b):
    (ma, sa), (mb, sb) = a, b
    with np.errstate(all="ignore"):
        m = np.fmax(ma, mb)
        m[np.isnan(ma) | np.isnan(mb)] = np.nan
        ta = np.where(ma == -np.inf, 0.0, sa * np.exp(ma - m))
        tb = np.where(mb == -np.inf, 0.0, sb * np.exp(mb - m))
    return m, ta + tb


def rank_part_softmax(values_local, offsets, row0, row1, rank):
    """(statistics of segments finished here, edge record) of one window."""
    b = offsets.size - 1
    d = values_local.shape[1]
    ends = offsets[1:]
    lo = 0 if rank == 0 else int(np.searchsorted(ends, row0, side="right"))
    hi = int(np.searchsorted(ends, row1, side="right"))
    stats, head_seg, head_ends, head = {}, -1, 0, None
    for s in range(lo, hi):
        start, end = int(offsets[s]), int(offsets[s + 1])
        piece = _stats(values_local[max(start, row0) - row0:end - row0])
        if start >= row0:
            stats[s] = piece
        else:
            head_seg, head_ends, head = s, 1, piece
    tail_seg, tail = -1, None
    if hi < b and row1 > row0 and int(offsets[hi]) < row1:
        s, start = hi, int(offsets[hi])
        piece = _stats(values_local[max(start, row0) - row0:row1 - row0])
        if start >= row0:
            tail_seg, tail = s, piece
        elif head_seg < 0:
            head_seg, head_ends, head = s, 0, piece
    ident = (np.full(d, -np.inf), np.zeros(d))
    head, tail = head or ident, tail or ident
    return stats, np.concatenate([[head_seg, head_ends, tail_seg], head[0], head[1], tail[0], tail[1]])


def finish_softmax(values_local, offsets, row0, row1, rank, stats, records):
    d = values_local.shape[1]
    own = records[rank]
    for s in (int(own[0]), int(own[2])):
        if s < 0:
            continue
        total = (np.full(d, -np.inf), np.zeros(d))
        for rec in records:
            if int(rec[2]) == s:
                total = _smerge(total, (rec[3 + 2 * d:3 + 3 * d], rec[3 + 3 * d:3 + 4 * d]))
            elif int(rec[0]) == s:
                total = _smerge(total, (rec[3:3 + d], rec[3 + d:3 + 2 * d]))
        stats[s] = total
    out = np.empty_like(values_local)
    for s in range(offsets.size - 1):
        start, end = max(int(offsets[s]), row0), min(int(offsets[s + 1]), row1)
        if start >= end:
            continue
        m, t = stats[s]
        with np.errstate(all="ignore"):
            base = np.where(m == -np.inf, 0.0, m)
            out[start - row0:end - row0] = np.exp(values_local[start - row0:end - row0] - base) / t
    return out


def _softmax_worker(rank, world, port, cases, results):
    import torch
    import torch.distributed as dist
    from ragged.sharding import shard_rows
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        out = []
        for values, offsets, split in cases:
            n = int(offsets[-1])
            splits = _split_of(split, offsets, world)
            row0, row1 = shard_rows(n, world, rank, splits)
            local = values[row0:row1]
            stats, record = rank_part_softmax(local, offsets, row0, row1, rank)
            mine = torch.from_numpy(record)
            gathered = [torch.empty_like(mine) for _ in range(world)]
            dist.all_gather(gathered, mine)
            out.append((row0, finish_softmax(local, offsets, row0, row1, rank, stats, [g.numpy() for g in gathered])))
        results[rank] = out
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world", [2, 3])
def test_sharded_softmax_protocol_over_gloo(world):
    import torch.multiprocessing as mp
    from oracle import reference_port as rp
    rng = np.random.default_rng(8)
    cases = []
    lengths = make_lengths("long_tail", 60, 5000, seed=4)
    offsets = offsets_of(lengths)
    cases.append((rng.normal(scale=3.0, size=(int(offsets[-1]), 4)), offsets))
    lengths = np.array([0, 3, 997, 0, 0, 1500, 498, 2, 0], dtype=np.int64)
    offsets = offsets_of(lengths)
    values = rng.normal(size=(int(offsets[-1]), 3))
    values[10, 1] = np.nan
    values[1200:1300, 2] = -np.inf
    cases.append((values, offsets))
    cases = [(v, o, split) for v, o in cases for split in (None, "balanced")]
    cases += [(rng.normal(size=(3, 2)), np.array([0, 3], dtype=np.int64), split) for split in ("repeat", "balanced")]
    manager = mp.get_context("spawn").Manager()
    results = manager.dict()
    mp.start_processes(_softmax_worker, args=(world, _free_port(), cases, results), nprocs=world, start_method="spawn")
    for i, (values, offsets, _) in enumerate(cases):
        parts = sorted((results[rank][i] for rank in range(world)), key=lambda part: (part[0], part[1].shape[0]))
        actual = np.concatenate([p[1] for p in parts], axis=0)
        with np.errstate(all="ignore"):
            expected = rp.segment_softmax(values, offsets)
        np.testing.assert_allclose(actual, expected, rtol=1e-12, atol=1e-15, equal_nan=True)


def test_shard_segments_cover_every_window_row():
    """rg_shard_segments (host code, no GPU): the statistics slots of a rank
    cover every segment with rows in its window, for even and balanced
    splits, with empty segments at the boundaries."""
    from ragged import _native
    from ragged.sharding import balanced_split, shard_rows
    lengths = np.array([0, 0, 5, 0, 100, 1, 0, 0, 37, 400, 0, 2, 0], dtype=np.int64)
    offsets = offsets_of(lengths)
    n, b = int(offsets[-1]), offsets.size - 1
    for world in (1, 2, 3, 5, 8):
        for splits in (None, balanced_split(offsets, world)):
            for rank in range(world):
                row0, row1 = shard_rows(n, world, rank, splits)
                seg0, seg1 = _native.shard_segments(offsets, "i64", world, rank, splits)
                assert 0 <= seg0 <= seg1 <= b
                for s in range(b):
                    if offsets[s] < row1 and offsets[s + 1] > row0:
                        assert seg0 <= s < seg1, (world, rank, s, seg0, seg1)


@pytest.mark.parametrize("splits", [[0, 540], [0, 100, 540], [0, 100, 200, 300, 540], []])
def test_native_split_arguments_must_hold_world_plus_one_boundaries(splits):
    """The C ABI reads world + 1 boundaries from a split pointer; the
    binding refuses a list of another length before calling it."""
    from ragged import ValidationError, _native
    offsets = offsets_of(np.array([40, 0, 500], dtype=np.int64))
    with pytest.raises(ValidationError, match="world \\+ 1"):
        _native.shard_segments(offsets, "i64", 3, 1, splits)
    with pytest.raises(ValidationError, match="world \\+ 1"):
        _native.shard_workspace_bytes("sum", "f32", "i64", 4, 540, 3, 3, 1, 0, splits)


def test_end_weight_fit_recovers_the_cost_of_an_end():
    """sharding.fit_end_weight: per-rank times made from a known per-row
    and per-end cost give back their ratio (a small fixed cost moves it
    little); too few ranks keep the model weight.  window_ends counts each
    end on exactly one rank."""
    from ragged.sharding import balanced_split, end_weight_model, fit_end_weight, window_ends
    rng = np.random.default_rng(12)
    rows = rng.integers(5_000_000, 30_000_000, size=8)
    ends = rng.integers(0, 2_000_000, size=8)
    times = rows * 9e-8 + ends * 2.7e-7
    weight, info = fit_end_weight(rows, ends, times, fallback=1.25)
    assert weight == pytest.approx(3.0, rel=1e-6) and info["fit"] == "least squares over ranks"
    assert fit_end_weight(rows, ends, times + 0.01, fallback=1.25)[0] == pytest.approx(3.0, rel=0.1)
    assert fit_end_weight(rows[:2], ends[:2], times[:2], fallback=1.25)[0] == 1.25
    assert end_weight_model("sum", "bf16", 256) == 1.25
    lengths = make_lengths("long_tail", 500, 100_000, seed=2)
    lengths[:40] = 0
    offsets = offsets_of(lengths)
    for world in (1, 3, 8):
        for splits in (None, balanced_split(offsets, world, 4.0)):
            assert sum(window_ends(offsets, world, splits)) == offsets.size - 1
