"""In-place softmax on the GPU (ProgramSpec(alias="inplace"), out IS values):
every schedule against the oracle, the reference's alias rules, and checked
mode leaving the input untouched on rejection.  Restates the reference's
test/gpu/test_correctness.py:263-270 and test/gpu/test_checked.py:144-150,
219-222 for this build's schedules.
"""
from __future__ import annotations

import functools

import numpy as np
import pytest

from helpers import _cache_dir, check, make_lengths, offsets_of, prepared

pytestmark = pytest.mark.gpu

SCHEDULES = ("naive", "classified", "rowbalanced")


@functools.lru_cache(maxsize=64)
def inplace_program(dtype, d, index="i64"):
    from ragged import ArtifactCache, Compiler, ProgramSpec
    return Compiler().compile(ProgramSpec("softmax", dtype, d, index, alias="inplace"),
                              ArtifactCache(_cache_dir(), max_specializations=4096))


def run_inplace(torch, dtype, values, offsets, select):
    tdtype = torch.float32 if dtype == "f32" else torch.bfloat16
    d = values.shape[1]
    guard = torch.full((values.shape[0] + 2, d), -64.0, device="cuda", dtype=tdtype)
    device_values = guard[1:-1]
    device_values.copy_(torch.from_numpy(np.ascontiguousarray(values, dtype=np.float32)).to(tdtype))
    device_offsets = torch.from_numpy(offsets).to("cuda")
    report = inplace_program(dtype, d, "i32" if offsets.dtype == np.int32 else "i64").run(
        device_values, device_offsets, device_values, select=select)
    torch.cuda.synchronize()
    assert torch.all(guard[0] == -64).item() and torch.all(guard[-1] == -64).item(), "write outside the rows"
    return device_values.float().cpu().numpy().astype(np.float64), report


@pytest.mark.parametrize("select", SCHEDULES)
@pytest.mark.parametrize("dtype,d", [("f32", 1), ("f32", 7), ("f32", 128), ("f32", 256), ("bf16", 8),
                                     ("bf16", 128), ("bf16", 1024)])
@pytest.mark.parametrize("distribution", ["uniform", "long_tail", "burst"])
def test_inplace_softmax_matches_the_oracle(cuda, select, dtype, d, distribution):
    lengths = make_lengths(distribution, 300, 40_000 if d <= 256 else 6_000, seed=71)
    lengths[::23] = 0
    offsets = offsets_of(lengths)
    values = prepared(np.random.default_rng(72).normal(scale=2.0, size=(int(offsets[-1]), d)), dtype)
    actual, report = run_inplace(cuda, dtype, values, offsets, select)
    assert report.selected == select
    check(actual, values, offsets, "softmax", dtype)


@pytest.mark.parametrize("select", SCHEDULES)
def test_inplace_long_segments(cuda, select):
    """Segments split across many workers: every statistics read of a
    segment precedes the first write into it."""
    lengths = np.array([3, 70_000, 0, 9000, 1], dtype=np.int64)
    offsets = offsets_of(lengths, "i32")
    values = prepared(np.random.default_rng(73).normal(size=(int(offsets[-1]), 64)), "bf16")
    values[40_000, 3] = 30.0  # a late maximum
    actual, _ = run_inplace(cuda, "bf16", values, offsets, select)
    check(actual, values, offsets, "softmax", "bf16")


def test_inplace_matches_out_of_place_bitwise(cuda):
    torch = cuda
    from helpers import program
    lengths = make_lengths("bimodal", 400, 50_000, seed=74)
    offsets = offsets_of(lengths)
    values = np.random.default_rng(75).normal(size=(int(offsets[-1]), 32)).astype(np.float32)
    for select in SCHEDULES:
        inplace, _ = run_inplace(torch, "f32", values, offsets, select)
        dv = torch.from_numpy(values).cuda()
        out = torch.empty_like(dv)
        program("softmax", "f32", 32, "i64").run(dv, torch.from_numpy(offsets).cuda(), out, select=select)
        torch.cuda.synchronize()
        np.testing.assert_array_equal(inplace, out.cpu().numpy().astype(np.float64))


def test_alias_rules(cuda):
    torch = cuda
    from helpers import program
    from ragged import ValidationError
    big = torch.zeros((11, 8), device="cuda")
    values, shifted = big[0:10], big[1:11]
    offsets = torch.tensor([0, 4, 10], device="cuda")
    prog = inplace_program("f32", 8)
    with pytest.raises(ValidationError, match="same buffer"):
        prog.run(values, offsets, torch.empty_like(values))
    with pytest.raises(ValidationError, match="aliases values"):
        prog.run(values, offsets, shifted)  # partial overlap
    with pytest.raises(ValidationError, match="aliases values"):
        program("softmax", "f32", 8, "i64").run(values, offsets, values)  # out-of-place specialisation
    empty = torch.zeros((0, 8), device="cuda")
    prog.run(empty, torch.zeros((3,), dtype=torch.int64, device="cuda"), torch.zeros((0, 8), device="cuda"))


@pytest.mark.parametrize("select", SCHEDULES)
@pytest.mark.parametrize("index", ["i32", "i64"])
def test_checked_rejection_preserves_inplace_values(cuda, select, index):
    torch = cuda
    from ragged import ArtifactCache, Compiler, ProgramSpec, ValidationError
    prog = Compiler().compile(ProgramSpec("softmax", "f32", 3, index, alias="inplace"),
                              ArtifactCache(_cache_dir(), max_specializations=4096))
    values = torch.arange(24, device="cuda", dtype=torch.float32).reshape(8, 3) / 8
    original = values.clone()
    offsets = torch.tensor([0, 4, 3, 8], device="cuda", dtype=torch.int32 if index == "i32" else torch.int64)
    with pytest.raises(ValidationError) as caught:
        prog.run(values, offsets, values, mode="checked", select=select)
    assert caught.value.errors == {"nonmonotone": 1}
    torch.cuda.synchronize()
    assert torch.equal(values, original)
    good = torch.tensor([0, 4, 8], device="cuda", dtype=offsets.dtype)
    report = prog.run(values, good, values, mode="checked", select=select)
    torch.cuda.synchronize()
    assert report.mode == "checked"
    check(values.cpu().numpy().astype(np.float64), original.cpu().numpy().astype(np.float64),
          np.array([0, 4, 8]), "softmax", "f32")
