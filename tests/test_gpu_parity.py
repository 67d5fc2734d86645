"""GPU parity: every schedule of libragged_b200 against the CPU oracle.

Each call goes through the public API and the C ABI (rg_run).  Results are
checked with the reference's tolerance contract and this build's strict one
(max bit-exact; f32 sum/softmax rtol 1e-5; bf16 within 1 ulp), outputs are
guarded against out-of-bounds writes.  Cases restate the reference's
test/gpu/test_correctness.py and test/gpu/test_classified.py.
"""
from __future__ import annotations

import numpy as np
import pytest

from helpers import DISTRIBUTIONS, check, make_lengths, offsets_of, prepared, run_device
from oracle import reference_port as rp

pytestmark = pytest.mark.gpu


def schedules(op):
    from ragged.compiler import IMPLEMENTED
    return IMPLEMENTED["softmax" if op == "softmax" else "reduce"]


ALL = [(op, s) for op in ("sum", "max", "softmax") for s in ("naive", "classified", "rowbalanced")
       if not (op == "softmax" and s == "rowbalanced")]


def _run_all(cuda, op, dtype, values, offsets, **kwargs):
    """Run every implemented schedule; check each; return the outputs."""
    outputs = {}
    reference = None
    with np.errstate(all="ignore"):
        reference = rp.REFERENCES[op](values, offsets)
    for schedule in schedules(op):
        actual, report = run_device(cuda, op, dtype, values, offsets, select=schedule, **kwargs)
        assert report.selected == schedule
        check(actual, values, offsets, op, dtype, reference)
        outputs[schedule] = actual
    return outputs


def test_golden_cases(cuda, golden):
    for name, case in golden.items():
        for op in ("sum", "max", "softmax"):
            for schedule in schedules(op):
                actual, _ = run_device(cuda, op, case["dtype"], case["values"], case["offsets"], select=schedule)
                expected = case[op]
                with np.errstate(all="ignore"):
                    rp.assert_matches(actual, case["values"], case["offsets"], operation=op,
                                      input_dtype=case["dtype"], reference=expected)
                    rp.check_strict(actual, case["values"], case["offsets"], operation=op,
                                    input_dtype=case["dtype"], reference=expected)


@pytest.mark.parametrize("op", ["sum", "max", "softmax"])
@pytest.mark.parametrize("dtype", ["f32", "bf16"])
@pytest.mark.parametrize("d", [1, 2, 3, 16, 100, 128, 256, 1024])
@pytest.mark.parametrize("index", ["i32", "i64"])
@pytest.mark.parametrize("distribution", DISTRIBUTIONS)
def test_matrix(cuda, op, dtype, d, index, distribution):
    total = 4096 if d <= 256 else 1024
    lengths = make_lengths(distribution, 64, total, seed=711)
    offsets = offsets_of(lengths, index)
    values = prepared(np.random.default_rng(981).normal(size=(int(offsets[-1]), d)), dtype)
    _run_all(cuda, op, dtype, values, offsets)


@pytest.mark.parametrize("op", ["sum", "max", "softmax"])
@pytest.mark.parametrize("dtype", ["f32", "bf16"])
@pytest.mark.parametrize("offsets", [[0], [0, 0, 0], [0, 0, 1, 1, 4]])
def test_empty_all_empty_and_tail_features(cuda, op, dtype, offsets):
    values = np.arange(offsets[-1] * 3, dtype=np.float32).reshape(offsets[-1], 3)
    _run_all(cuda, op, dtype, values, np.array(offsets, dtype=np.int64))


@pytest.mark.parametrize("dtype", ["f32", "bf16"])
@pytest.mark.parametrize("rows", [2, 33, 64, 5000])
def test_softmax_special_values(cuda, dtype, rows):
    # NaN; +inf with finite; all -inf; finite with -inf; one +inf with -inf only.
    values = np.full((rows, 5), -np.inf, dtype=np.float32)
    values[0] = [np.nan, np.inf, -np.inf, -np.inf, np.inf]
    values[1] = [1, 1, -np.inf, 3, -np.inf]
    _run_all(cuda, "softmax", dtype, values, np.array([0, rows], dtype=np.int64))


@pytest.mark.parametrize("op", ["sum", "max"])
@pytest.mark.parametrize("dtype", ["f32", "bf16"])
def test_reduction_nonfinite(cuda, op, dtype):
    values = np.array([[np.nan, np.inf, -np.inf, -2], [1, -np.inf, -np.inf, -4]], dtype=np.float32)
    _run_all(cuda, op, dtype, values, np.array([0, 2, 2], dtype=np.int64))


@pytest.mark.parametrize("op", ["sum", "max", "softmax"])
def test_single_very_long_segment(cuda, op):
    values = np.tile(np.array([[1, -1, 0.5]], dtype=np.float32), (131073, 1))
    outputs = _run_all(cuda, op, "f32", values, np.array([0, len(values)], dtype=np.int64))
    if op == "sum":
        for out in outputs.values():
            np.testing.assert_array_equal(out, [[131073, -131073, 65536.5]])


@pytest.mark.parametrize("d", [128, 1024])
@pytest.mark.parametrize("op", ["sum", "softmax"])
def test_long_segment_accumulation_accuracy(cuda, d, op):
    # 0.1 is not representable: an uncompensated f32 lane accumulator drifts
    # beyond the bound; the compensated one must not (reference
    # test_correctness.py:201-216).
    rows = 16384
    if op == "sum":
        values = np.full((rows, d), np.float32(0.1), dtype=np.float32)
    else:
        values = np.full((rows, d), np.float32(-np.log(10)), dtype=np.float32)
        values[0] = 0
    _run_all(cuda, op, "f32", values, np.array([0, rows], dtype=np.int64))


@pytest.mark.parametrize("dtype", ["f32", "bf16"])
@pytest.mark.parametrize("d", [128, 1024])
def test_compensated_sum_preserves_nonfinite(cuda, dtype, d):
    values = np.zeros((12, d), dtype=np.float32)
    values[0, :5] = [np.inf, -np.inf, np.inf, np.nan, 3]
    values[4, :5] = [2, 2, -np.inf, 2, np.inf]
    values[8, :5] = [3, 3, 3, 3, 2]
    _run_all(cuda, "sum", dtype, values, np.array([0, 12], dtype=np.int64))


@pytest.mark.parametrize("op", ["sum", "max", "softmax"])
@pytest.mark.parametrize("dtype", ["f32", "bf16"])
def test_metamorphic_relations(cuda, op, dtype):
    """Permutation, empty insertion, split-sum and shift invariance
    (reference test_correctness.py:233-260), per schedule."""
    values = np.random.default_rng(90).integers(-4, 5, size=(39, 7)).astype(np.float32)
    offsets = np.array([0, 3, 3, 30, 39], dtype=np.int64)
    for schedule in schedules(op):
        run = lambda v, o: run_device(cuda, op, dtype, v, np.asarray(o, dtype=np.int64), select=schedule)[0]
        original = run(values, offsets)
        pieces = [values[a:b] for a, b in zip(offsets[:-1], offsets[1:])]
        permutation = [3, 1, 0, 2]
        permuted_values = np.concatenate([pieces[i] for i in permutation])
        permuted_offsets = [0, *np.cumsum([len(pieces[i]) for i in permutation])]
        permuted = run(permuted_values, permuted_offsets)
        expected = (np.concatenate([original[offsets[i]:offsets[i + 1]] for i in permutation])
                    if op == "softmax" else original[permutation])
        inserted = run(values, [0, 0, 3, 3, 30, 39, 39])
        if schedule == "rowbalanced" and op == "softmax":
            # The row-balanced schedule cuts the merge path by position, so a
            # segment's softmax statistics round differently when it moves.
            np.testing.assert_allclose(permuted, expected, rtol=2e-6, atol=1e-30)
            np.testing.assert_allclose(inserted, original, rtol=2e-6, atol=1e-30)
        else:
            np.testing.assert_array_equal(permuted, expected)
            np.testing.assert_array_equal(inserted if op == "softmax" else inserted[1:5], original)
        if op == "softmax":
            shifted = run(values + 5, offsets)
            np.testing.assert_allclose(shifted, original, rtol=2e-5 if dtype == "f32" else 2e-2,
                                       atol=2e-6 if dtype == "f32" else 2e-3)


@pytest.mark.parametrize("op", ["sum", "max", "softmax"])
def test_threshold_boundaries(cuda, op):
    """Segment lengths at and around every class bound (reference
    test_classified.py:23): 0, 1, 31-33, 4095-4097 and a split one."""
    lengths = np.array([0, 1, 31, 32, 33, 4095, 4096, 4097, 20000, 2, 0], dtype=np.int64)
    offsets = offsets_of(lengths)
    values = np.random.default_rng(17).normal(size=(int(offsets[-1]), 64)).astype(np.float32)
    _run_all(cuda, op, "f32", values, offsets)


@pytest.mark.parametrize("op", ["sum", "max", "softmax"])
def test_unvectorized_program(cuda, op):
    lengths = make_lengths("long_tail", 40, 3000, seed=3)
    offsets = offsets_of(lengths)
    values = np.random.default_rng(4).normal(size=(int(offsets[-1]), 16)).astype(np.float32)
    actual, report = run_device(cuda, op, "f32", values, offsets, vectorize=False, select="naive")
    assert report.d_vector == 1
    check(actual, values, offsets, op, "f32")


def test_nondefault_stream(cuda):
    torch = cuda
    lengths = make_lengths("uniform", 100, 20000, seed=9)
    offsets = offsets_of(lengths)
    values = np.random.default_rng(10).normal(size=(int(offsets[-1]), 128)).astype(np.float32)
    stream = torch.cuda.Stream()
    for op in ("sum", "max", "softmax"):
        actual, _ = run_device(cuda, op, "f32", values, offsets, stream=stream)
        check(actual, values, offsets, op, "f32")


def test_misaligned_view_is_rejected(cuda):
    torch = cuda
    from helpers import program
    from ragged import ValidationError
    prog = program("sum", "f32", 128, "i64")
    base = torch.zeros((11, 128), device="cuda")
    values = base.view(-1)[1:1 + 10 * 128].view(10, 128)  # 4-byte offset
    offsets = torch.tensor([0, 10], device="cuda")
    out = torch.empty((1, 128), device="cuda")
    with pytest.raises(ValidationError, match="aligned"):
        prog.run(values, offsets, out)


def test_validation_errors(cuda):
    torch = cuda
    from helpers import program
    from ragged import RuntimeUnavailable, ValidationError
    prog = program("sum", "f32", 4, "i64")
    values = torch.zeros((5, 4), device="cuda")
    offsets = torch.tensor([0, 5], device="cuda")
    with pytest.raises(ValidationError, match="out shape"):
        prog.run(values, offsets, torch.empty((2, 4), device="cuda"))
    with pytest.raises(ValidationError, match="dtype"):
        prog.run(values, offsets.int(), torch.empty((1, 4), device="cuda"))
    with pytest.raises(RuntimeUnavailable, match="CUDA device"):
        prog.run(values.cpu(), offsets, torch.empty((1, 4), device="cuda"))
    with pytest.raises(ValidationError, match="alias"):
        prog.run(values, offsets, values[:1])
    assert prog.run(values, offsets, torch.empty((1, 4), device="cuda"), mode="checked").mode == "checked"


@pytest.mark.parametrize("op", ["sum", "max"])
@pytest.mark.parametrize("dtype,d", [("f32", 1), ("f32", 2), ("f32", 4), ("bf16", 1), ("bf16", 2), ("bf16", 4),
                                     ("bf16", 8)])
def test_narrow_rows_packed_and_unaligned(cuda, op, dtype, d):
    """Rows of 2-16 bytes: the packed kernel (16-byte aligned values) and
    the per-row kernel it falls back to for a view that is not."""
    torch = cuda
    from helpers import program
    lengths = make_lengths("bimodal", 500, 20_000, seed=23)
    lengths[3] = 0
    offsets = offsets_of(lengths, "i32")
    values = prepared(np.random.default_rng(24).normal(size=(int(offsets[-1]), d)), dtype)
    tdtype = torch.float32 if dtype == "f32" else torch.bfloat16
    prog = program(op, dtype, d, "i32")
    device_offsets = torch.from_numpy(offsets).to("cuda")
    row_bytes = d * (4 if dtype == "f32" else 2)
    for shift in (0, 1):  # shift one row: misaligns the base for the packed loads (rows under 16 bytes)
        base = torch.zeros((values.shape[0] + 1, d), dtype=tdtype, device="cuda")
        view = base[shift:shift + values.shape[0]]
        view.copy_(torch.from_numpy(values).to(tdtype))
        out = torch.empty((offsets.size - 1, d), dtype=tdtype, device="cuda")
        report = prog.run(view, device_offsets, out, select="rowbalanced")
        torch.cuda.synchronize()
        check(out.float().cpu().numpy().astype(np.float64), values, offsets, op, dtype)
        names = set(report.kernel_names)
        if shift == 0 or row_bytes == 16:
            assert "rowbalanced_packed" in names
        else:
            assert "rowbalanced" in names and "rowbalanced_packed" not in names


@pytest.mark.parametrize("op", ["sum", "max"])
@pytest.mark.parametrize("dtype,d", [("f32", 1), ("f32", 2), ("f32", 4), ("bf16", 1), ("bf16", 4), ("bf16", 8)])
@pytest.mark.parametrize("index", ["i32", "i64"])
def test_packed_segment_ends_inside_staged_runs(cuda, op, dtype, d, index):
    """The packed kernel folds a staged run of 8 packets in one pass per
    piece between segment ends (up to two ends), row by row past that:
    lengths mixing runs of empty segments, 1-3 row segments, and lengths
    on and around packet and run boundaries (2-8 rows a packet, 16-64 a
    run), with enough rows that every lane holds several runs."""
    torch = cuda
    from helpers import program
    rng = np.random.default_rng(41)
    choices = np.array([0, 0, 1, 2, 3, 4, 5, 7, 8, 9, 15, 16, 17, 31, 32, 33, 63, 64, 65, 200, 1000])
    lengths = rng.choice(choices, size=60_000)
    lengths[100:400] = 0  # a long run of empty segments
    offsets = offsets_of(lengths, index)
    values = prepared(rng.normal(size=(int(offsets[-1]), d)), dtype)
    tdtype = torch.float32 if dtype == "f32" else torch.bfloat16
    prog = program(op, dtype, d, index)
    out = torch.empty((offsets.size - 1, d), dtype=tdtype, device="cuda")
    report = prog.run(torch.from_numpy(values).to(tdtype).to("cuda"), torch.from_numpy(offsets).to("cuda"), out,
                      select="rowbalanced")
    torch.cuda.synchronize()
    assert "rowbalanced_packed" in report.kernel_names
    check(out.float().cpu().numpy().astype(np.float64), values, offsets, op, dtype)


@pytest.mark.parametrize("op", ["sum", "max", "softmax"])
@pytest.mark.parametrize("dtype,d", [("bf16", 8), ("f32", 16)])
def test_classified_many_short_segments_long_claims(cuda, op, dtype, d):
    """Enough segments per CTA that the pipelined worker's producer claims
    128 segments at a time and runs continue across its 32-segment
    sub-batches: lengths 0-3 with runs of empty segments, a few segments
    longer than a stage (they end a run) and a final partial claim."""
    from oracle import native
    rng = np.random.default_rng(52)
    count = 200_003
    lengths = rng.integers(0, 4, size=count)
    lengths[rng.integers(0, count, size=40)] = 3000  # split class: closes the open run
    lengths[1000:1400] = 0
    offsets = offsets_of(lengths, "i64")
    values = prepared(rng.normal(size=(int(offsets[-1]), d)), dtype)
    actual, report = run_device(cuda, op, dtype, values, offsets, select="classified")
    assert "classified_worker" in report.kernel_names
    reference = native.run(op, values, offsets, dtype=dtype)
    scale = native.segment_reduce(values, offsets, "abssum", dtype=dtype) if op == "sum" else None
    native.check(actual, op, dtype, offsets, reference, scale)


@pytest.mark.parametrize("op", ["sum", "max", "softmax"])
@pytest.mark.parametrize("dtype,d", [("f32", 3), ("bf16", 128), ("f32", 1024)])
def test_classified_many_split_segments(cuda, op, dtype, d):
    """Dozens of split-class segments (several chunks each, one ending on a
    chunk boundary) between warp- and CTA-class ones and empty segments:
    the split list, chunk numbering and last-chunk merge of the classified
    schedule, across column tiles for D=1024."""
    rng = np.random.default_rng(31)
    count = 24 if d <= 128 else 6
    lengths = []
    for i in range(count):
        lengths += [int(rng.integers(4097, 20000)), 0, int(rng.integers(1, 33)), int(rng.integers(33, 4097))]
    lengths[4] = 3 * 4096  # exactly three chunks
    offsets = offsets_of(np.array(lengths, dtype=np.int64))
    values = prepared(rng.normal(size=(int(offsets[-1]), d)), dtype)
    _run_all(cuda, op, dtype, values, offsets)


@pytest.mark.parametrize("op", ["sum", "max", "softmax"])
def test_classified_is_deterministic(cuda, op):
    """Work items go to CTAs through an atomic counter; the output must not
    depend on which CTA took which item."""
    lengths = make_lengths("long_tail", 3000, 400_000, seed=41)
    offsets = offsets_of(lengths)
    values = np.random.default_rng(42).normal(size=(int(offsets[-1]), 32)).astype(np.float32)
    first, report = run_device(cuda, op, "f32", values, offsets, select="classified")
    assert report.kernel_names[:2] == ("classify", "classified_worker")
    for _ in range(3):
        again, _ = run_device(cuda, op, "f32", values, offsets, select="classified")
        np.testing.assert_array_equal(again, first)
    check(first, values, offsets, op, "f32")


@pytest.mark.parametrize("op,rows", [("sum", 200_000), ("max", 200_000), ("softmax", 150_000)])
def test_classified_chunks_grow_for_giant_segments(cuda, op, rows):
    """A split segment longer than 1024 chunks of one stage gets longer
    chunks (each streamed through several shared-memory stages by one team);
    its last chunk merges at most 1024 partials."""
    lengths = np.array([5, rows, 0, 7], dtype=np.int64)
    offsets = offsets_of(lengths)
    values = prepared(np.random.default_rng(53).normal(size=(int(offsets[-1]), 256)), "bf16")
    actual, report = run_device(cuda, op, "bf16", values, offsets, select="classified")
    assert report.thresholds[0] == 32 and 32 < report.thresholds[1] <= 4096
    assert rows > 1024 * report.thresholds[1]
    check(actual, values, offsets, op, "bf16")


@pytest.mark.parametrize("lengths", [[1, 7, 33, 300, 5000], [2, 64, 2, 900, 0, 3]])
def test_f32_softmax_terms_far_below_the_maximum(cuda, lengths):
    """f32 softmax with every logit but one per column 60 to 87 below the
    column's maximum: the exponential's relative error (about |t| * 2^-23,
    from rounding t = x - m and t * log2 e once each) reaches its largest
    there, next to the 1e-5 bound; outputs near FLT_MIN test the flush
    allowance.  Every schedule must stay within both contracts."""
    rng = np.random.default_rng(6087)
    lengths = np.array(lengths, dtype=np.int64)
    offsets = offsets_of(lengths)
    n = int(offsets[-1])
    values = rng.uniform(-87.0, -60.0, size=(n, 32)).astype(np.float32) + np.float32(12.5)
    for start, length in zip(offsets[:-1], lengths):
        if length:
            top = start + rng.integers(0, length, size=32)
            values[top, np.arange(32)] = np.float32(12.5)
    _run_all(cuda, "softmax", "f32", values, offsets)
