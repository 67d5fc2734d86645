"""Row-sharded sum / max through the C ABI, ranks emulated on one GPU.

Every rank of a ``world``-way split runs ``rg_run_shard`` on its own rows;
their edge records are gathered in rank order, then every rank runs
``rg_shard_combine``.  No kernel waits on another rank, so running the ranks
one after another on one device is the same computation as one process per
GPU with an all-gather in between.  The assembled output (each row from the
rank ``segment_owners`` names) must match the CPU oracle, and every rank
must leave the rows it does not own untouched.
"""
from __future__ import annotations

import numpy as np
import pytest

from helpers import SENTINEL, check, make_lengths, offsets_of, prepared
from oracle import reference_port as rp

pytestmark = pytest.mark.gpu


def run_world(torch, op, dtype, values, offsets, world, splits=None):
    from ragged import _native
    from ragged.sharding import segment_owners, shard_rows
    d = values.shape[1]
    n, b = int(offsets[-1]), offsets.size - 1
    index = "i32" if offsets.dtype == np.int32 else "i64"
    tdtype = torch.float32 if dtype == "f32" else torch.bfloat16
    dev_values = torch.from_numpy(np.ascontiguousarray(values, dtype=np.float32)).to("cuda").to(tdtype)
    dev_offsets = torch.from_numpy(offsets).to("cuda")
    edge_floats = _native.shard_edge_bytes(op, d) // 4
    edges = torch.empty((world, edge_floats), dtype=torch.float32, device="cuda")
    outs = []
    for rank in range(world):
        row0, row1 = shard_rows(n, world, rank, splits)
        if splits is None:
            assert (row0, row1) == _native.shard_rows(n, world, rank)
        local = dev_values[row0:row1].contiguous()
        out = torch.full((b, d), SENTINEL, dtype=tdtype, device="cuda")
        ws = _native.shard_workspace_bytes(op, dtype, index, d, n, b, world, rank, 0, splits)
        scratch = torch.empty((max(ws, 1),), dtype=torch.uint8, device="cuda")
        _native.run_shard(op, dtype, index, d, n, b, world, rank, local.data_ptr() if local.numel() else 0,
                          dev_offsets.data_ptr(), out.data_ptr(), edges[rank].data_ptr(), scratch.data_ptr(), ws, 0,
                          torch.cuda.current_stream().cuda_stream, splits)
        outs.append(out)
    gathered = edges.reshape(-1).contiguous()
    for rank in range(world):
        _native.shard_combine(op, dtype, d, world, rank, gathered.data_ptr(), outs[rank].data_ptr(), 0,
                              torch.cuda.current_stream().cuda_stream)
    torch.cuda.synchronize()
    owners = segment_owners(offsets, world, splits)
    host = [o.float().cpu().numpy().astype(np.float64) for o in outs]
    result = np.empty((b, d), dtype=np.float64)
    for rank in range(world):
        mine = owners == rank
        result[mine] = host[rank][mine]
        untouched = host[rank][~mine]
        assert np.all(untouched == SENTINEL), f"rank {rank} wrote rows it does not own"
    return result


@pytest.mark.parametrize("op", ["sum", "max"])
@pytest.mark.parametrize("dtype,d", [("f32", 128), ("bf16", 256), ("f32", 3), ("bf16", 1024)])
@pytest.mark.parametrize("world", [2, 3, 8])
def test_sharded_matches_oracle(cuda, op, dtype, d, world):
    rng = np.random.default_rng(1000 + world + d)
    lengths = make_lengths("long_tail", 400, 60_000 if d <= 256 else 12_000, seed=world)
    lengths[5] = 0
    lengths[-1] = 0
    offsets = offsets_of(lengths)
    values = prepared(rng.normal(size=(int(offsets[-1]), d)), dtype)
    if op == "max":
        values[rng.random(values.shape) < 1e-3] = np.nan
    actual = run_world(cuda, op, dtype, values, offsets, world)
    check(actual, values, offsets, op, dtype)


@pytest.mark.parametrize("op", ["sum", "max"])
def test_sharded_giant_segment_spans_ranks(cuda, op):
    """One segment through several whole shards (ranks whose rows lie
    inside it), segments ending exactly on shard boundaries, and empty
    segments at the boundaries."""
    world = 5
    n = 50_000
    ends = [shard_end for shard_end in (10_000, 20_000, 30_000, 40_000)]
    lengths = [3, ends[0] - 3, 0, 0, 7, n - ends[0] - 7 - 11, 11, 0]
    offsets = offsets_of(np.array(lengths, dtype=np.int64))
    assert offsets[-1] == n
    values = prepared(np.random.default_rng(7).normal(size=(n, 64)), "f32")
    actual = run_world(cuda, op, "f32", values, offsets, world)
    check(actual, values, offsets, op, "f32")


@pytest.mark.parametrize("world", [2, 4])
def test_sharded_no_rows(cuda, world):
    """N = 0: every segment is empty and ends at row 0; rank 0 writes them."""
    offsets = np.array([0, 0, 0], dtype=np.int64)
    values = np.zeros((0, 4), dtype=np.float32)
    for op in ("sum", "max"):
        actual = run_world(cuda, op, "f32", values, offsets, world)
        check(actual, values, offsets, op, "f32")


@pytest.mark.parametrize("world", [2, 4])
def test_sharded_more_ranks_than_rows(cuda, world):
    lengths = np.array([0, 1, 0, 2, 0], dtype=np.int64)
    offsets = offsets_of(lengths, "i32")
    values = prepared(np.arange(3 * 8, dtype=np.float32).reshape(3, 8), "f32")
    for op in ("sum", "max"):
        actual = run_world(cuda, op, "f32", values, offsets, world + 3)
        check(actual, values, offsets, op, "f32")


def test_sharded_i32_bimodal_and_determinism(cuda):
    lengths = make_lengths("bimodal", 3000, 200_000, seed=8)
    offsets = offsets_of(lengths, "i32")
    values = prepared(np.random.default_rng(9).normal(size=(int(offsets[-1]), 32)), "bf16")
    first = run_world(cuda, "sum", "bf16", values, offsets, 4)
    again = run_world(cuda, "sum", "bf16", values, offsets, 4)
    np.testing.assert_array_equal(first, again)
    check(first, values, offsets, "sum", "bf16")


@pytest.mark.parametrize("op", ["sum", "max"])
@pytest.mark.parametrize("world", [2, 5, 8])
def test_sharded_balanced_split(cuda, op, world):
    """The work-balanced split (rows + weighted segment ends), from the C
    library's rg_shard_split and its NumPy restatement alike."""
    from ragged import _native
    from ragged.sharding import balanced_split
    lengths = make_lengths("burst", 2000, 80_000, seed=world)
    lengths[:700] = 1  # many short segments at the start pull the split forward
    offsets = offsets_of(lengths)
    splits = balanced_split(offsets, world)
    assert splits == _native.shard_split(offsets, "i64", world, 1.25)
    values = prepared(np.random.default_rng(world).normal(size=(int(offsets[-1]), 64)), "bf16")
    actual = run_world(cuda, op, "bf16", values, offsets, world, splits)
    check(actual, values, offsets, op, "bf16")


# ---------------------------------------------------------------- softmax

def run_world_softmax(torch, dtype, values, offsets, world, splits=None):
    """Every rank's statistics phase, the gathered edge records, then every
    rank's finishing phase; the ranks' rows concatenated."""
    from ragged import _native
    from ragged.sharding import shard_rows
    d = values.shape[1]
    n, b = int(offsets[-1]), offsets.size - 1
    index = "i32" if offsets.dtype == np.int32 else "i64"
    tdtype = torch.float32 if dtype == "f32" else torch.bfloat16
    stream = torch.cuda.current_stream().cuda_stream
    dev_values = torch.from_numpy(np.ascontiguousarray(values, dtype=np.float32)).to("cuda").to(tdtype)
    dev_offsets = torch.from_numpy(offsets).to("cuda")
    edges = torch.empty((world, _native.shard_edge_bytes("softmax", d) // 4), dtype=torch.float32, device="cuda")
    ranks = []
    covered = np.zeros(b, dtype=bool)
    for rank in range(world):
        row0, row1 = shard_rows(n, world, rank, splits)
        seg0, seg1 = _native.shard_segments(offsets, index, world, rank, splits)
        # every segment with rows in the window has a statistics slot
        for s in range(b):
            if offsets[s] < row1 and offsets[s + 1] > row0 and offsets[s + 1] > offsets[s]:
                assert seg0 <= s < seg1, (rank, s, seg0, seg1)
                covered[s] = True
        local = dev_values[row0:row1].contiguous()
        ws = _native.shard_softmax_workspace_bytes(dtype, index, d, n, b, world, rank, (seg0, seg1), 0, splits)
        scratch = torch.empty((max(ws, 1),), dtype=torch.uint8, device="cuda")
        _native.run_shard_softmax(dtype, index, d, n, b, world, rank, (seg0, seg1),
                                  local.data_ptr() if local.numel() else 0, dev_offsets.data_ptr(),
                                  edges[rank].data_ptr(), scratch.data_ptr(), ws, 0, stream, splits)
        ranks.append((row0, row1, (seg0, seg1), local, ws, scratch))
    gathered = edges.reshape(-1).contiguous()
    guard = torch.full((n + 2, d), SENTINEL, dtype=tdtype, device="cuda")
    for rank, (row0, row1, segments, local, ws, scratch) in enumerate(ranks):
        out = guard[1 + row0:1 + row1]
        _native.shard_softmax_finish(dtype, index, d, n, b, world, rank, segments,
                                     local.data_ptr() if local.numel() else 0, dev_offsets.data_ptr(),
                                     gathered.data_ptr(), out.data_ptr() if out.numel() else 0, scratch.data_ptr(),
                                     ws, 0, stream, splits)
    torch.cuda.synchronize()
    host = guard.float().cpu().numpy().astype(np.float64)
    assert np.all(host[0] == SENTINEL) and np.all(host[-1] == SENTINEL), "write outside the rows"
    return host[1:-1]


@pytest.mark.parametrize("dtype,d", [("f32", 128), ("bf16", 256), ("f32", 3), ("bf16", 64)])
@pytest.mark.parametrize("world", [2, 3, 8])
@pytest.mark.parametrize("balanced", [False, True])
def test_sharded_softmax_matches_oracle(cuda, dtype, d, world, balanced):
    from ragged.sharding import balanced_split
    rng = np.random.default_rng(2000 + world + d)
    lengths = make_lengths("long_tail", 400, 60_000 if d <= 128 else 20_000, seed=world + 7)
    lengths[5] = 0
    lengths[-1] = 0
    offsets = offsets_of(lengths)
    values = prepared(rng.normal(scale=2.0, size=(int(offsets[-1]), d)), dtype)
    values[rng.random(values.shape) < 1e-4] = np.nan
    splits = balanced_split(offsets, world) if balanced else None
    actual = run_world_softmax(cuda, dtype, values, offsets, world, splits)
    check(actual, values, offsets, "softmax", dtype)


def test_sharded_softmax_segment_through_whole_shards(cuda):
    """One segment covers several whole shards (through windows); a late
    maximum on a middle rank rescales every other rank's piece."""
    lengths = np.array([3, 50_000, 0, 7, 1], dtype=np.int64)
    offsets = offsets_of(lengths, "i32")
    values = prepared(np.random.default_rng(91).normal(size=(int(offsets[-1]), 64)), "bf16")
    values[30_000, 7] = 25.0
    actual = run_world_softmax(cuda, "bf16", values, offsets, 8)
    check(actual, values, offsets, "softmax", "bf16")


def test_sharded_softmax_through_the_runtime(cuda):
    """CompiledProgram.run_sharded on one rank of a world of one (the
    exchange is the identity)."""
    torch = cuda
    from helpers import program
    lengths = make_lengths("bimodal", 300, 40_000, seed=92)
    offsets = offsets_of(lengths)
    values = np.random.default_rng(93).normal(size=(int(offsets[-1]), 32)).astype(np.float32)
    dv = torch.from_numpy(values).cuda()
    out = torch.empty_like(dv)
    report = program("softmax", "f32", 32, "i64").run_sharded(
        dv, torch.from_numpy(offsets).cuda(), out, total_rows=int(offsets[-1]), world=1, rank=0,
        exchange=lambda edges: edges, offsets_host=offsets)
    torch.cuda.synchronize()
    assert "rowbalanced_normalize" in report.kernel_names
    check(out.cpu().numpy().astype(np.float64), values, offsets, "softmax", "f32")


@pytest.mark.parametrize("op", ["sum", "max"])
def test_sharded_reduction_through_the_runtime(cuda, op):
    """CompiledProgram.run_sharded for sum and max (the path bench.py takes
    on several GPUs) on one rank of a world of one, with an explicit even
    split: the exchange is the identity and every output row is this
    rank's."""
    torch = cuda
    from helpers import program
    lengths = make_lengths("long_tail", 400, 60_000, seed=94)
    lengths[::13] = 0
    offsets = offsets_of(lengths)
    n = int(offsets[-1])
    values = prepared(np.random.default_rng(95).normal(size=(n, 64)), "bf16")
    dv = torch.from_numpy(values).cuda().to(torch.bfloat16)
    out = torch.full((offsets.size - 1, 64), SENTINEL, dtype=torch.bfloat16, device="cuda")
    report = program(op, "bf16", 64, "i64").run_sharded(dv, torch.from_numpy(offsets).cuda(), out, total_rows=n,
                                                         world=1, rank=0, exchange=lambda edges: edges,
                                                         splits=[0, n])
    torch.cuda.synchronize()
    assert report.kernel_names[0].startswith("rowbalanced")
    check(out.float().cpu().numpy().astype(np.float64), values, offsets, op, "bf16")


@pytest.mark.parametrize("op", ["sum", "softmax"])
@pytest.mark.parametrize("problem", ["grad", "gathered-bf16", "gathered-strided", "gathered-short"])
def test_sharded_runtime_rejects_bad_tensors(cuda, op, problem):
    """run_sharded refuses autograd inputs and an exchange result that is
    not every rank's f32 record, contiguous, before the combine launch."""
    torch = cuda
    from ragged import ValidationError
    from helpers import program
    offsets = np.array([0, 3, 9], dtype=np.int64)
    values = torch.randn((9, 8), device="cuda")
    out = torch.full((9 if op == "softmax" else 2, 8), -64.0, device="cuda")
    exchange = {
        "gathered-bf16": lambda edges: edges.to(torch.bfloat16),
        "gathered-strided": lambda edges: torch.stack([edges, edges], 1)[:, 0],
        "gathered-short": lambda edges: edges[:-1],
    }.get(problem, lambda edges: edges)
    if problem == "grad":
        values.requires_grad_()
    kwargs = {"offsets_host": offsets} if op == "softmax" else {}
    with pytest.raises(ValidationError):
        program(op, "f32", 8, "i64").run_sharded(values, torch.from_numpy(offsets).cuda(), out, total_rows=9, world=1,
                                                 rank=0, exchange=exchange, **kwargs)
    torch.cuda.synchronize()
    if problem == "grad":
        assert torch.all(out == -64).item()


@pytest.mark.parametrize("op", ["sum", "max"])
@pytest.mark.parametrize("splits", [[0, 1, 2, 2, 3, 3, 3, 3, 3], [0, 1, 1, 1, 2, 2, 3, 3, 3], "balanced"])
def test_sharded_ranks_without_rows_inside_a_segment(cuda, op, splits):
    """Repeated split boundaries leave ranks with no rows while a segment is
    open across them: their edge records hold no piece, and the rank that
    finishes the segment must still merge the starting rank's tail piece.
    The balanced split of one 3-row segment over 8 ranks makes such a split."""
    from ragged.sharding import balanced_split
    offsets = np.array([0, 3], dtype=np.int64)
    values = prepared(np.array([[1.5, -2.0, 4.0], [0.25, 8.0, -1.0], [3.0, 0.5, 2.0]]), "f32")
    if splits == "balanced":
        splits = balanced_split(offsets, 8)
        assert len(set(splits)) < len(splits), "expected repeated boundaries"
    actual = run_world(cuda, op, "f32", values, offsets, 8, list(splits))
    check(actual, values, offsets, op, "f32")


@pytest.mark.parametrize("op", ["sum", "max"])
def test_sharded_empty_ranks_inside_a_giant_segment(cuda, op):
    """A long segment with ranks of no rows between the ranks holding it, and
    short segments around it, bf16 D=256 (the c5 row shape)."""
    lengths = np.array([5, 20_000, 0, 7, 3000, 1], dtype=np.int64)
    offsets = offsets_of(lengths)
    n = int(offsets[-1])
    splits = [0, 3000, 9000, 9000, 9000, 15000, 20003, 20003, n]
    values = prepared(np.random.default_rng(44).normal(size=(n, 256)), "bf16")
    actual = run_world(cuda, op, "bf16", values, offsets, 8, splits)
    check(actual, values, offsets, op, "bf16")
