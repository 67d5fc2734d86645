"""Checked mode on the GPU: device validation of the offsets before any main
kernel (rg_check_offsets through ``CompiledProgram.run(mode="checked")``).

Cases restate the reference's test/gpu/test_checked.py: every condition and
its earliest index against the oracle's ``offsets_status``; a rejected call
leaves the input and every output row (and the guard rows around it)
untouched; extreme i32/i64 endpoints cannot overflow a segment length; B=0
still checks its only offset; the status is reset between calls; validation
runs on the explicit stream after work queued there; a valid call returns the
same results as validated mode.  Each schedule (naive, classified,
rowbalanced) is forced in turn; the long-segment cases reach the classified
schedule's split class.
"""
from __future__ import annotations

import functools

import numpy as np
import pytest

from helpers import _cache_dir, check, prepared
from oracle import reference_port as rp

pytestmark = pytest.mark.gpu

SCHEDULES = ("naive", "classified", "rowbalanced")
D = 3


@functools.lru_cache(maxsize=256)
def checked_program(op, index, dtype="f32", min_len=None, max_len=None, claimed=False):
    from ragged import ArtifactCache, Compiler, Hints, ProgramSpec
    spec = ProgramSpec(op, dtype, D, index, hints=Hints(max_len=max_len, min_len=min_len, offsets_checked=claimed))
    return Compiler().compile(spec, ArtifactCache(_cache_dir(), max_specializations=4096))


def _tensors(torch, op, dtype, index, offsets, n, values=None):
    tdtype = torch.float32 if dtype == "f32" else torch.bfloat16
    if values is None:
        values = np.arange(n * D, dtype=np.float32).reshape(n, D) / 8
    device_values = torch.from_numpy(np.ascontiguousarray(values, dtype=np.float32)).to("cuda").to(tdtype)
    device_offsets = torch.tensor([int(x) for x in offsets], device="cuda",
                                  dtype=torch.int32 if index == "i32" else torch.int64)
    rows = n if op == "softmax" else len(offsets) - 1
    guard = torch.full((rows + 2, D), -64.0, device="cuda", dtype=tdtype)
    return device_values, device_offsets, guard


def assert_rejected(torch, op, index, offsets, n, select, *, min_len=None, max_len=None, claimed=False):
    expected = rp.offsets_status(offsets, n, min_len, max_len)
    assert expected, "a negative case needs an independent expected violation"
    program = checked_program(op, index, "f32", min_len, max_len, claimed)
    values, device_offsets, guard = _tensors(torch, op, "f32", index, offsets, n)
    original = values.clone()
    with pytest.raises(Exception) as caught:
        program.run(values, device_offsets, guard[1:-1], mode="checked", select=select)
    from ragged import ValidationError
    assert isinstance(caught.value, ValidationError), caught.value
    error = caught.value
    assert error.errors == expected
    assert (error.condition, error.index) == next(iter(expected.items()))
    for condition, at in expected.items():
        assert f"{condition} at index {at}" in str(error)
    torch.cuda.synchronize()
    assert torch.equal(values, original), "validation changed the input"
    assert torch.all(guard == -64).item(), "an output row was written before the rejection"


def run_success(torch, op, dtype, index, offsets, select, *, min_len=None, max_len=None):
    n = int(offsets[-1])
    values = prepared(np.random.default_rng(875).normal(size=(n, D)), dtype)
    program = checked_program(op, index, dtype, min_len, max_len)
    device_values, device_offsets, guard = _tensors(torch, op, dtype, index, offsets, n, values)
    report = program.run(device_values, device_offsets, guard[1:-1], mode="checked", select=select)
    torch.cuda.synchronize()
    assert report.mode == "checked"
    assert report.validation_workspace_bytes == 56
    assert report.validation_host_ms is not None and report.validation_host_ms >= 0
    assert report.kernel_names[:2] == ("offsets_init", "offsets_check")
    if len(offsets) == 1:
        assert report.kernel_names == ("offsets_init", "offsets_check") and report.classes == ()
        assert report.workspace_bytes == 56
    else:
        assert len(report.kernel_names) > 2
    assert torch.all(guard[0] == -64).item() and torch.all(guard[-1] == -64).item()
    actual = guard[1:-1].float().cpu().numpy().astype(np.float64)
    check(actual, values, np.asarray(offsets, dtype=np.int64), op, dtype)


@pytest.mark.parametrize("op", ["sum", "max", "softmax"])
@pytest.mark.parametrize("index", ["i32", "i64"])
@pytest.mark.parametrize("select", SCHEDULES)
@pytest.mark.parametrize("offsets", [[1, 4, 8], [0, 4, 7], [0, -1, 8], [0, 9, 8], [0, 4, 3, 8]],
                         ids=["first", "final", "negative", "above-n", "nonmonotone"])
def test_checked_rejects_invalid_offsets_before_output(cuda, op, index, select, offsets):
    assert_rejected(cuda, op, index, offsets, 8, select)


@pytest.mark.parametrize("op", ["sum", "max", "softmax"])
@pytest.mark.parametrize("index", ["i32", "i64"])
@pytest.mark.parametrize("select", SCHEDULES)
@pytest.mark.parametrize("claimed", [False, True])
def test_checked_validates_both_length_hints_even_if_claimed_checked(cuda, op, index, select, claimed):
    lower = 4097 if select == "classified" else 2
    offsets = [0, lower - 1, lower - 1 + 8194]
    assert rp.offsets_status(offsets, offsets[-1], lower, 8193) == {"below_min_len": 0, "above_max_len": 1}
    assert_rejected(cuda, op, index, offsets, offsets[-1], select, min_len=lower, max_len=8193, claimed=claimed)


@pytest.mark.parametrize("op", ["sum", "max", "softmax"])
@pytest.mark.parametrize("index", ["i32", "i64"])
def test_checked_reports_all_conditions_and_earliest_indices(cuda, op, index):
    offsets = [1, -2, -3, 11, 10, 0, 1, 7, 6]
    assert rp.offsets_status(offsets, 8, 4, 4) == dict(zip(rp.CHECK_CONDITIONS, [0, 8, 1, 3, 0, 5, 6]))
    assert_rejected(cuda, op, index, offsets, 8, "naive", min_len=4, max_len=4, claimed=True)


@pytest.mark.parametrize("op", ["sum", "max", "softmax"])
@pytest.mark.parametrize("index", ["i32", "i64"])
@pytest.mark.parametrize("select", SCHEDULES)
def test_checked_extreme_endpoints_do_not_overflow_segment_lengths(cuda, op, index, select):
    bits = 32 if index == "i32" else 64
    minimum, maximum = -(1 << (bits - 1)), (1 << (bits - 1)) - 1
    # MIN -> MAX must not be subtracted; only the final 0 -> 8 segment is
    # eligible for the length bounds.
    offsets = [0, minimum, maximum, 0, 8]
    assert_rejected(cuda, op, index, offsets, 8, select, min_len=4097 if select == "classified" else 0,
                    max_len=8 if select == "naive" else 8193, claimed=True)


@pytest.mark.parametrize("op", ["sum", "max", "softmax"])
@pytest.mark.parametrize("index", ["i32", "i64"])
@pytest.mark.parametrize("n,offsets", [(0, [1]), (0, [-1]), (2, [0]), (2, [2])])
def test_checked_zero_batch_still_checks_its_only_offset(cuda, op, index, n, offsets):
    assert_rejected(cuda, op, index, offsets, n, "classified")


@pytest.mark.parametrize("op", ["sum", "max", "softmax"])
@pytest.mark.parametrize("index", ["i32", "i64"])
def test_checked_atomic_min_keeps_the_earliest_error_across_blocks(cuda, op, index):
    offsets = np.arange(4098, dtype=np.int64) * 2
    n = int(offsets[-1])
    offsets[130] = offsets[129] + 1  # below the minimum at 129, above the maximum at 130
    offsets[1026] = offsets[1025] + 1
    offsets[2051] = -1
    offsets[3077] = -2
    offsets[3001] = n + 1
    assert rp.offsets_status(offsets, n, 2, 2) == {"negative": 2051, "above_n": 3001, "nonmonotone": 2050,
                                                   "below_min_len": 129, "above_max_len": 130}
    for _ in range(3):  # repeated launches: init/check order and the reset
        assert_rejected(cuda, op, index, offsets, n, "naive", min_len=2, max_len=2)


def test_checked_earliest_index_in_a_large_batch(cuda):
    """A batch larger than the check kernel's grid (grid-stride loop): the
    minimum must still be the earliest of many offending indices."""
    b = 3_000_000
    offsets = np.arange(b + 1, dtype=np.int64) * 2
    n = int(offsets[-1])
    bad = np.array([2_999_000, 1_700_001, 900_007, 2_400_000])
    offsets[bad] = n + 5
    expected = rp.offsets_status(offsets, n)
    assert expected["above_n"] == 900_007 and expected["nonmonotone"] == 900_007
    assert_rejected(cuda, "sum", "i64", offsets, n, "rowbalanced")


@pytest.mark.parametrize("op", ["sum", "max", "softmax"])
@pytest.mark.parametrize("dtype", ["f32", "bf16"])
@pytest.mark.parametrize("index", ["i32", "i64"])
@pytest.mark.parametrize("select", SCHEDULES)
def test_checked_success_matches_the_oracle(cuda, op, dtype, index, select):
    offsets = [0, 4097, 12290] if select == "classified" else [0, 0, 1, 34, 4131]
    kwargs = {"min_len": 4097, "max_len": 8193} if select == "classified" else {}
    run_success(cuda, op, dtype, index, offsets, select, **kwargs)


@pytest.mark.parametrize("op", ["sum", "max", "softmax"])
@pytest.mark.parametrize("index", ["i32", "i64"])
@pytest.mark.parametrize("offsets", [[0], [0, 0], [0, 0, 0, 0]])
def test_checked_zero_rows_and_empty_segments_are_valid(cuda, op, index, offsets):
    run_success(cuda, op, "f32", index, offsets, "classified")


@pytest.mark.parametrize("op", ["sum", "max", "softmax"])
@pytest.mark.parametrize("index", ["i32", "i64"])
def test_checked_status_is_reset_after_a_rejected_call(cuda, op, index):
    assert_rejected(cuda, op, index, [0, -1, 8], 8, "classified")
    run_success(cuda, op, "f32", index, [0, 4, 8], "classified")


@pytest.mark.parametrize("op", ["sum", "max", "softmax"])
@pytest.mark.parametrize("target_valid", [False, True])
def test_checked_validation_follows_prior_work_on_the_explicit_stream(cuda, op, target_valid):
    torch = cuda
    from ragged import ValidationError
    program = checked_program(op, "i64")
    current, consumer = torch.cuda.Stream(), torch.cuda.Stream()
    with torch.cuda.stream(current):
        values = torch.arange(24, device="cuda", dtype=torch.float32).reshape(8, 3) / 8
        offsets = torch.tensor([0, 4, 8], dtype=torch.int64, device="cuda")
        output = torch.full((8 if op == "softmax" else 2, 3), -64.0, device="cuda")
        program.run(values, offsets, output, stream=current, mode="checked")
        offsets[-1].fill_(7 if target_valid else 8)
        output.fill_(-64)
        consumer.wait_stream(current)
        with torch.cuda.stream(consumer):
            # Queued work ahead of the mutation: validation must run after it.
            lhs = torch.ones((4096, 4096), device="cuda")
            delay = torch.empty_like(lhs)
            for _ in range(16):
                torch.mm(lhs, lhs, out=delay)
            offsets[-1].fill_(8 if target_valid else 7)
        assert torch.cuda.current_stream() == current
        if target_valid:
            assert program.run(values, offsets, output, stream=consumer, mode="checked").mode == "checked"
        else:
            with pytest.raises(ValidationError) as caught:
                program.run(values, offsets, output, stream=consumer, mode="checked")
            assert caught.value.errors == {"final_mismatch": 2}
        assert torch.cuda.current_stream() == current
        consumer.synchronize()
    if target_valid:
        host = values.cpu().numpy().astype(np.float64)
        check(output.cpu().numpy().astype(np.float64), host, np.array([0, 4, 8]), op, "f32")
    else:
        assert torch.all(output == -64).item()
