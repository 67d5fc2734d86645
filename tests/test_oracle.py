"""The CPU oracle: pinned against the reference oracle's own outputs.

``golden.npz`` was produced by running the reference's oracle/reference.py
(tests/golden/make_golden.py).  The NumPy port and the C port must agree
with it.  The remaining tests restate the reference's oracle self-tests
(test/python/test_oracle.py) against the port.
"""
from __future__ import annotations

import ast
from pathlib import Path

import numpy as np
import pytest

from oracle import native as coracle
from oracle import reference_port as rp

OPS = ("sum", "max", "softmax")


def _same(actual, expected):
    np.testing.assert_array_equal(np.isnan(actual), np.isnan(expected))
    finite = np.isfinite(expected)
    np.testing.assert_array_equal(actual[~finite & ~np.isnan(expected)], expected[~finite & ~np.isnan(expected)])
    np.testing.assert_allclose(actual[finite], expected[finite], rtol=1e-12, atol=1e-300)


def test_port_matches_reference_golden(golden):
    for name, case in golden.items():
        for op in OPS:
            with np.errstate(all="ignore"):
                actual = rp.REFERENCES[op](case["values"], case["offsets"])
            _same(actual, case[op])


def test_c_oracle_matches_reference_golden(golden):
    for name, case in golden.items():
        for op in OPS:
            actual = coracle.run(op, case["values"], case["offsets"], dtype=case["dtype"], threads=3)
            _same(actual, case[op])


def test_golden_outputs_pass_both_contracts(golden):
    # The reference's own answers pass its tolerance check and the strict one.
    for name, case in golden.items():
        for op in OPS:
            rounded = case[op].astype(np.float32)
            if case["dtype"] == "bf16":
                rounded = rp.quantize_bf16(rounded)
            with np.errstate(all="ignore"):
                rp.assert_matches(rounded, case["values"], case["offsets"], operation=op, input_dtype=case["dtype"])
                rp.check_strict(rounded, case["values"], case["offsets"], operation=op, input_dtype=case["dtype"])


@pytest.mark.parametrize("threads", [1, 2, 7, 16])
def test_c_oracle_threads_and_giant_segment(threads):
    rng = np.random.default_rng(5)
    lengths = np.array([0, 3, 0, 50_000, 1, 0, 7, 20_000, 0], dtype=np.int64)
    offsets = np.concatenate([[0], np.cumsum(lengths)]).astype(np.int64)
    values = rng.normal(size=(int(offsets[-1]), 4)).astype(np.float32)
    for op in OPS:
        _same(coracle.run(op, values, offsets, threads=threads), rp.REFERENCES[op](values, offsets))


@pytest.mark.parametrize("index_dtype", [np.int32, np.int64])
def test_hand_calculated(index_dtype):
    values = np.array([[1, 2], [3, 4], [-2, 7]], dtype=np.float32)
    offsets = np.array([0, 2, 2, 3], dtype=index_dtype)
    np.testing.assert_array_equal(rp.segment_sum(values, offsets), [[4, 6], [0, 0], [-2, 7]])
    np.testing.assert_array_equal(rp.segment_max(values, offsets), [[3, 4], [-np.inf, -np.inf], [-2, 7]])
    low = 1 / (1 + np.exp(2))
    np.testing.assert_allclose(rp.segment_softmax(values, offsets), [[low, low], [1 - low, 1 - low], [1, 1]])


@pytest.mark.parametrize("raw,n,condition", [
    ([1, 3], 3, r"offsets\[0\]"), ([0, 3, 2, 3], 3, "nondecreasing"), ([0, 2], 3, r"offsets\[-1\]"),
    ([0, -1, 3], 3, r"\[0, N\]"), ([0, 4, 3], 3, r"\[0, N\]"), ([], 0, "length")])
@pytest.mark.parametrize("dtype", [np.int32, np.int64])
def test_invalid_offsets(raw, n, condition, dtype):
    with pytest.raises(ValueError, match=condition):
        rp.validate_offsets(np.array(raw, dtype=dtype), n)


def test_bf16_round_ties_even_and_nonfinite():
    values = np.array([1 + 2**-8, 1 + 3 * 2**-8, np.inf, -np.inf, np.nan, -0.0], dtype=np.float32)
    actual = rp.quantize_bf16(values)
    np.testing.assert_array_equal(actual[:4], [1, 1 + 2**-6, np.inf, -np.inf])
    assert np.isnan(actual[4]) and np.signbit(actual[5])
    assert np.isnan(rp.quantize_bf16(np.array([0x7F800001], dtype=np.uint32).view(np.float32))[0])


def test_tolerance_accepts_rounding_rejects_wrong_results():
    values = np.array([[1], [2]], dtype=np.float32)
    offsets = np.array([0, 2], dtype=np.int32)
    rp.assert_matches(np.array([[3.000001]]), values, offsets, operation="sum", input_dtype="f32")
    with pytest.raises(AssertionError, match="exceed tolerance"):
        rp.assert_matches(np.array([[4]]), values, offsets, operation="sum", input_dtype="f32")
    with pytest.raises(AssertionError, match="NaN"):
        rp.assert_matches(np.array([[np.nan]]), values, offsets, operation="sum", input_dtype="f32")
    with pytest.raises(AssertionError, match="shape"):
        rp.assert_matches(np.array([3]), values, offsets, operation="sum", input_dtype="f32")


def test_tolerance_cancellation_and_overflow():
    values = np.array([[1e8], [1], [-1e8]], dtype=np.float32)
    rp.assert_matches(np.array([[0]]), values, np.array([0, 3], dtype=np.int32), operation="sum", input_dtype="f32")
    big = np.array([[3e38], [3e38]], dtype=np.float32)
    offsets = np.array([0, 2], dtype=np.int32)
    rp.assert_matches(np.array([[np.inf]]), big, offsets, operation="sum", input_dtype="f32")
    with pytest.raises(AssertionError, match="positive infinity"):
        rp.assert_matches(np.array([[np.inf]]), np.ones((2, 1), dtype=np.float32), offsets, operation="sum",
                          input_dtype="f32")


@pytest.mark.parametrize("dtype", ["f32", "bf16"])
def test_softmax_all_zero_long_segment_rejected(dtype):
    values = np.zeros((1_000_000, 1), dtype=np.float32)
    with pytest.raises(AssertionError, match="sum to one"):
        rp.assert_matches(np.zeros_like(values), values, np.array([0, len(values)], dtype=np.int64),
                          operation="softmax", input_dtype=dtype)


def test_strict_check_catches_planted_mistakes():
    """Mistakes planted in the oracle's own answer on the CPU must fail."""
    rng = np.random.default_rng(3)
    values = rp.quantize_bf16(rng.normal(size=(50, 8)).astype(np.float32))
    offsets = np.array([0, 10, 10, 50], dtype=np.int64)
    good_max = rp.segment_max(values, offsets).astype(np.float32)
    rp.check_strict(good_max, values, offsets, operation="max", input_dtype="bf16")
    bad = good_max.copy()
    bad[0, 3] = np.nextafter(bad[0, 3], np.float32(np.inf))
    with pytest.raises(AssertionError, match="bit-exact"):
        rp.check_strict(bad, values, offsets, operation="max", input_dtype="bf16")
    bad = good_max.copy()
    bad[1, 0] = 0.0   # empty segment must be -inf
    with pytest.raises(AssertionError, match="infinity"):
        rp.check_strict(bad, values, offsets, operation="max", input_dtype="bf16")
    soft = rp.quantize_bf16(rp.segment_softmax(values, offsets).astype(np.float32))
    rp.check_strict(soft, values, offsets, operation="softmax", input_dtype="bf16")
    bad = soft.copy()
    bad[5, 2] = bad[5, 2] * (1 + 2**-6)   # two bf16 ulps off
    with pytest.raises(AssertionError, match="strict softmax"):
        rp.check_strict(bad, values, offsets, operation="softmax", input_dtype="bf16")
    sums = rp.segment_sum(values.astype(np.float32), offsets)
    rp.check_strict(sums.astype(np.float32), values, offsets, operation="sum", input_dtype="f32")
    bad = sums.copy()
    bad[2, 1] += 1e-3 * rp.segment_sum(np.abs(values), offsets)[2, 1]
    with pytest.raises(AssertionError, match="strict sum"):
        rp.check_strict(bad, values, offsets, operation="sum", input_dtype="f32")


def test_oracle_imports_neither_product_nor_torch():
    for source in (Path(__file__).resolve().parents[1] / "oracle").glob("*.py"):
        for node in ast.walk(ast.parse(source.read_text())):
            if isinstance(node, ast.Import):
                names = [alias.name for alias in node.names]
            elif isinstance(node, ast.ImportFrom):
                names = [node.module or ""]
            else:
                continue
            assert all(name.split(".")[0] not in {"ragged", "torch", "triton"} for name in names), source


def test_masked_logits_match_the_reference_fixtures(masked_golden):
    """The scale / mask restatement against the reference's own
    oracle/masked.py outputs (bitwise, NaN positions included)."""
    for name, case in masked_golden.items():
        logits = rp.masked_logits(case["values"], case["mask"], scale=case["scale"])
        np.testing.assert_array_equal(logits, case["logits"], err_msg=name)
        with np.errstate(all="ignore"):
            softmax = rp.segment_softmax(logits, case["offsets"])
        np.testing.assert_allclose(softmax, case["softmax"], rtol=1e-12, atol=0, equal_nan=True, err_msg=name)


def test_masked_logits_rejects_bad_contracts():
    values = np.zeros((3, 2), dtype=np.float32)
    with pytest.raises(ValueError):
        rp.masked_logits(values, np.zeros((3, 2), dtype=np.float64))
    with pytest.raises(ValueError):
        rp.masked_logits(values, np.zeros((1, 2), dtype=np.float32))
    with pytest.raises(ValueError):
        rp.masked_logits(values, None, scale=float("inf"))


def test_chunked_checker_matches_whole_oracle():
    """oracle.device_check (the large-input checker of the GPU tests and of
    bench.py's parity gate) on host tensors: chunked float64 partials of
    sum, max and sum |x| equal the whole-array oracle, also for a window of
    rows; a result one bf16 ulp beyond the bound is rejected."""
    import torch
    from helpers import fetcher
    from oracle import device_check as dc
    rng = np.random.default_rng(12)
    lengths = np.array([3, 0, 50, 7, 0, 200, 1, 0, 90, 400], dtype=np.int64)
    offsets = np.concatenate([[0], np.cumsum(lengths)]).astype(np.int64)
    values = rp.quantize_bf16(rng.normal(size=(int(offsets[-1]), 4)).astype(np.float32))
    values[60, 2] = np.nan
    host = torch.from_numpy(values).to(torch.bfloat16)
    fetch = fetcher(host)
    n = host.shape[0]
    segments = np.array([0, 1, 2, 3, 5, 6, 8, 9])
    kinds = ("sum", "max", "abssum")
    parts = dc.segment_partials(fetch, n, 4, offsets, segments, kinds=kinds, dtype="bf16", chunk_rows=64)
    for kind, got in zip(kinds, parts):
        source = np.abs(values) if kind == "abssum" else values
        with np.errstate(all="ignore"):
            want = rp.segment_reduce(source, offsets, "max" if kind == "max" else "sum")[segments]
        np.testing.assert_allclose(got, want, rtol=1e-12, equal_nan=True)
    window, = dc.segment_partials(fetcher(host[40:300]), 260, 4, offsets, segments, kinds=("sum",), dtype="bf16",
                                  row_base=40, chunk_rows=30)
    clipped = values.copy()
    clipped[:40] = 0
    clipped[300:] = 0
    np.testing.assert_allclose(window, rp.segment_sum(clipped, offsets)[segments], rtol=1e-12, equal_nan=True)
    with np.errstate(all="ignore"):
        exact = rp.quantize_bf16(rp.segment_sum(values, offsets)[segments].astype(np.float32)).astype(np.float64)
    dc.check_reduction(exact, fetch, n, offsets, segments, op="sum", dtype="bf16", chunk_rows=64)
    wrong = exact.copy()
    wrong[-1, 0] += 4 * rp.bf16_ulp(wrong[-1:, :1])[0, 0]
    with pytest.raises(AssertionError):
        dc.check_reduction(wrong, fetch, n, offsets, segments, op="sum", dtype="bf16", chunk_rows=64)
