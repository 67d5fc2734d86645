"""CPU restatement of the reference's float64 oracle -- TEST INFRASTRUCTURE ONLY.

This module is the checker for the CUDA path, never part of it: only the
tests, ``__graft_entry__.smoke()`` and ``bench.py``'s CPU-baseline leg may
import it. It restates, in NumPy float64, the semantics of the reference's
``oracle/reference.py`` (simon-jd/ragged-mlir):

* ``validate_offsets``  follows ``oracle/reference.py:17-39``
* ``quantize_bf16``     follows ``oracle/reference.py:55-67`` (RNE, NaN kept)
* ``segment_reduce``    follows ``oracle/reference.py:70-83`` (sum: +0 for an
  empty segment; max: -inf identity, NaN propagates)
* ``segment_softmax``   follows ``oracle/reference.py:94-106``
* ``assert_matches``    follows ``oracle/reference.py:109-174`` (tolerances
  ``TOLERANCES`` of ``oracle/reference.py:14``; sum scale = sum|x|)
* ``masked_logits``     follows ``oracle/masked.py:13-25`` (x * scale, then
  + mask, each rounded to f32; the softmax oracle then runs on the result)
* ``offsets_status``    restates the checked mode's device validation
  (``lib/Conversion/ToGPU.cpp:1067-1189``, contract pinned by the
  reference's ``test/gpu/test_checked.py:23-45``)

The reference loops over segments in Python; the restatement below is
vectorised (``np.add.reduceat``-style over nonempty segments, identities
written for empty ones) so that parity checks at test sizes run in seconds.
Its outputs are pinned against fixtures produced by running the reference
oracle itself (``tests/golden/make_golden.py``).

``check_strict`` adds the stricter contract of this build (max bit-exact;
f32 sum/softmax within rtol 1e-5; bf16 output within 1 bf16 ulp of the
round-to-nearest-even of the float64 answer).
"""
from __future__ import annotations

import numpy as np

TOLERANCES = {"f32": (2e-5, 2e-6), "bf16": (2e-2, 2e-3)}

# Stricter contract of this build (see module docstring).
STRICT_RTOL_F32 = 1e-5
# Results smaller than the smallest normal f32 may be flushed to zero by a
# kernel's flush-to-zero exponential; this absolute floor admits exactly that.
FLT_MIN = float(np.finfo(np.float32).tiny)


def validate_offsets(offsets: np.ndarray, n: int) -> np.ndarray:
    """Offsets contract of ``oracle/reference.py:17-39``."""
    offsets = np.asarray(offsets)
    if isinstance(n, (bool, np.bool_)) or not isinstance(n, (int, np.integer)) or n < 0:
        raise ValueError("N must be a nonnegative integer")
    if n > np.iinfo(np.int64).max:
        raise ValueError("N exceeds the i64 indexing range")
    if offsets.ndim != 1 or offsets.size == 0:
        raise ValueError("offsets must have rank 1 and length B+1 >= 1")
    if offsets.dtype not in (np.dtype("int32"), np.dtype("int64")):
        raise TypeError("offsets dtype must be i32 or i64")
    if not offsets.flags.c_contiguous:
        raise ValueError("offsets must be contiguous")
    if int(offsets[0]) != 0:
        raise ValueError("offsets[0] must equal 0")
    if np.any(offsets < 0) or np.any(offsets > n):
        raise ValueError("offsets must lie in [0, N]")
    if np.any(offsets[1:] < offsets[:-1]):
        raise ValueError("offsets must be nondecreasing")
    if int(offsets[-1]) != n:
        raise ValueError("offsets[-1] must equal N")
    return offsets


def masked_logits(values, mask=None, *, scale=1.0) -> np.ndarray:
    """The transformed input of a scale / mask call: f32(values) * f32(scale)
    (skipped for scale 1) and then + mask, each an f32 rounding, no fused
    multiply-add; IEEE rules for non-finite values (+inf + -inf = NaN)."""
    values = np.asarray(values)
    if values.ndim != 2 or values.dtype.kind != "f":
        raise ValueError("values must be a floating-point [N, D] array")
    if mask is not None:
        mask = np.asarray(mask)
        if mask.shape != values.shape or mask.dtype != np.float32:
            raise ValueError("mask must be f32 with exactly the values shape")
    if isinstance(scale, (bool, np.bool_)) or not np.isfinite(scale):
        raise ValueError("scale must be a finite f32 value")
    with np.errstate(over="ignore", invalid="ignore"):
        x = values.astype(np.float32)
        if scale != 1.0:
            x = np.multiply(x, np.float32(scale), dtype=np.float32)
        if mask is not None:
            x = np.add(x, mask, dtype=np.float32)
    return x


CHECK_CONDITIONS = ("first_nonzero", "final_mismatch", "negative", "above_n", "nonmonotone", "below_min_len",
                    "above_max_len")


def offsets_status(offsets, n: int, min_len=None, max_len=None) -> dict[str, int]:
    """Failed checked-mode conditions -> earliest offending index, in the
    condition order.  Python integers throughout, so extreme i64 endpoints
    cannot overflow; a length is formed only for a pair with both endpoints
    in [0, N] and start <= end (the bounds apply to valid segments only)."""
    offsets = [int(x) for x in offsets]
    b = len(offsets) - 1
    found: dict[str, int] = {}

    def note(condition: str, index: int) -> None:
        found.setdefault(condition, index)

    if offsets[0] != 0:
        note("first_nonzero", 0)
    if offsets[b] != n:
        note("final_mismatch", b)
    for i, o in enumerate(offsets):
        if o < 0:
            note("negative", i)
        if o > n:
            note("above_n", i)
    for i in range(b):
        start, end = offsets[i], offsets[i + 1]
        if end < start:
            note("nonmonotone", i)
        if 0 <= start <= end <= n:
            if min_len is not None and end - start < min_len:
                note("below_min_len", i)
            if max_len is not None and end - start > max_len:
                note("above_max_len", i)
    return {name: found[name] for name in CHECK_CONDITIONS if name in found}


def _inputs(values: np.ndarray, offsets: np.ndarray) -> tuple[np.ndarray, np.ndarray]:
    values = np.asarray(values)
    if values.ndim != 2:
        raise ValueError("values must have rank 2 [N, D]")
    if not 1 <= values.shape[1] <= 1024:
        raise ValueError("D must be in [1, 1024]")
    if values.dtype.kind != "f":
        raise TypeError("values must have a real floating dtype")
    if not values.flags.c_contiguous:
        raise ValueError("values must be row-major contiguous")
    return values.astype(np.float64), validate_offsets(offsets, values.shape[0])


def quantize_bf16(values: np.ndarray) -> np.ndarray:
    """f32 -> bf16 round-to-nearest-even, returned as exact f32 (NaN kept)."""
    values = np.asarray(values, dtype=np.float32)
    bits = values.view(np.uint32)
    nan = np.isnan(values)
    with np.errstate(over="ignore"):
        rounded = (bits + np.uint32(0x7FFF) + ((bits >> 16) & 1)) & np.uint32(0xFFFF0000)
    rounded = np.where(nan, np.uint32(0x7FC00000), rounded).astype(np.uint32)
    return rounded.view(np.float32)


def _nonempty(offsets: np.ndarray) -> tuple[np.ndarray, np.ndarray]:
    starts = offsets[:-1].astype(np.int64)
    lengths = offsets[1:].astype(np.int64) - starts
    keep = lengths > 0
    return np.nonzero(keep)[0], starts[keep]


def segment_reduce(values: np.ndarray, offsets: np.ndarray, kind: str) -> np.ndarray:
    """Sum (+0 for empty) or NaN-propagating max (-inf for empty), float64."""
    if kind not in ("sum", "max"):
        raise ValueError("reduction kind must be sum or max")
    values, offsets = _inputs(values, offsets)
    b, d = len(offsets) - 1, values.shape[1]
    identity = 0.0 if kind == "sum" else -np.inf
    out = np.full((b, d), identity, dtype=np.float64)
    which, starts = _nonempty(offsets)
    if which.size:
        with np.errstate(invalid="ignore", over="ignore"):
            if kind == "sum":
                out[which] = np.add.reduceat(values, starts, axis=0)
            else:
                # np.maximum propagates NaN (fmax would erase it), as np.max does
                # in the reference.
                out[which] = np.maximum.reduceat(values, starts, axis=0)
    return out


def segment_sum(values: np.ndarray, offsets: np.ndarray) -> np.ndarray:
    return segment_reduce(values, offsets, "sum")


def segment_max(values: np.ndarray, offsets: np.ndarray) -> np.ndarray:
    return segment_reduce(values, offsets, "max")


def _segment_ids(offsets: np.ndarray, n: int) -> np.ndarray:
    lengths = np.diff(offsets.astype(np.int64))
    return np.repeat(np.arange(len(lengths), dtype=np.int64), lengths)


def segment_softmax(values: np.ndarray, offsets: np.ndarray) -> np.ndarray:
    """Per-feature exp(x - max) / sum; NaN, +inf or all -inf -> NaN column."""
    values, offsets = _inputs(values, offsets)
    n = values.shape[0]
    out = np.empty_like(values)
    if n == 0:
        return out
    maxima = segment_max(values, offsets)
    ids = _segment_ids(offsets, n)
    which, starts = _nonempty(offsets)
    with np.errstate(invalid="ignore", over="ignore", divide="ignore", under="ignore"):
        weights = np.exp(values - maxima[ids])
        totals = np.zeros_like(maxima)
        totals[which] = np.add.reduceat(weights, starts, axis=0)
        out[:] = weights / totals[ids]
    return out


def _expected(reference: np.ndarray, input_dtype: str) -> np.ndarray:
    with np.errstate(over="ignore", invalid="ignore"):
        rounded = reference.astype(np.float32)
        if input_dtype == "bf16":
            rounded = quantize_bf16(rounded)
    return np.where(np.isinf(rounded), rounded.astype(np.float64), reference)


def _compare_nonfinite(actual: np.ndarray, expected: np.ndarray) -> None:
    if actual.shape != expected.shape:
        raise AssertionError(f"shape mismatch: {actual.shape} != {expected.shape}")
    if not np.array_equal(np.isnan(actual), np.isnan(expected)):
        raise AssertionError("NaN locations differ from oracle")
    if not np.array_equal(np.isposinf(actual), np.isposinf(expected)):
        raise AssertionError("positive infinity locations differ from oracle")
    if not np.array_equal(np.isneginf(actual), np.isneginf(expected)):
        raise AssertionError("negative infinity locations differ from oracle")


REFERENCES = {"sum": segment_sum, "max": segment_max, "softmax": segment_softmax}


def assert_matches(actual: np.ndarray, values: np.ndarray, offsets: np.ndarray, *,
                   operation: str, input_dtype: str,
                   reference: np.ndarray | None = None,
                   scale: np.ndarray | None = None) -> dict[str, float | int]:
    """The reference's accuracy contract (``oracle/reference.py:109-174``).

    ``reference`` may pass a precomputed float64 answer for these inputs and,
    for sums, ``scale`` the precomputed per-segment sum of |x| (then
    ``values`` is not read).
    """
    if operation not in REFERENCES:
        raise ValueError("operation must be sum, max, or softmax")
    if input_dtype not in TOLERANCES:
        raise ValueError("input_dtype must be f32 or bf16")
    if reference is None:
        reference = REFERENCES[operation](values, offsets)
    expected = _expected(reference, input_dtype)
    actual = np.asarray(actual, dtype=np.float64)
    _compare_nonfinite(actual, expected)
    if operation != "sum":
        scale = np.abs(expected)
    elif scale is None:
        scale = segment_sum(np.abs(values), offsets)
    rtol, atol = TOLERANCES[input_dtype]
    finite = np.isfinite(expected)
    error = np.abs(actual[finite] - expected[finite])
    bound = atol + rtol * scale[finite]
    failures = error > bound
    if np.any(failures):
        raise AssertionError(
            f"{operation}/{input_dtype}: {int(np.sum(failures))} finite values exceed "
            f"tolerance; max abs error={float(np.max(error)):.9g}")
    if operation == "softmax":
        if np.any(actual[finite] < 0) or np.any(actual[finite] > 1):
            raise AssertionError("finite softmax probabilities must lie in [0, 1]")
        _check_normalization(actual, expected, offsets, rtol + atol)
    return {
        "finite_values": int(np.sum(finite)),
        "nan_values": int(np.sum(np.isnan(expected))),
        "max_abs_error": float(np.max(error, initial=0)),
        "max_fraction_of_tolerance": float(np.max(error / bound, initial=0)),
    }


def _check_normalization(actual, expected, offsets, bound) -> None:
    """Every nonempty all-finite column sums to one within ``bound``."""
    offsets = np.asarray(offsets)
    which, starts = _nonempty(offsets)
    if not which.size:
        return
    finite_rows = np.isfinite(expected)
    with np.errstate(invalid="ignore"):
        totals = np.add.reduceat(np.where(finite_rows, actual, 0.0), starts, axis=0)
        all_finite = np.logical_and.reduceat(finite_rows, starts, axis=0)
    if np.any(np.abs(totals[all_finite] - 1) > bound):
        raise AssertionError("finite softmax columns must sum to one within dtype tolerance")


def bf16_ulp(x: np.ndarray) -> np.ndarray:
    """Spacing of bf16 numbers at |x| (x already a bf16 value as float64)."""
    x = np.abs(np.asarray(x, dtype=np.float64))
    with np.errstate(divide="ignore"):
        exponent = np.floor(np.log2(np.where(x > 0, x, 1.0)))
    exponent = np.maximum(exponent, -126.0)
    return np.ldexp(1.0, (exponent - 7).astype(np.int64))


def check_strict(actual: np.ndarray, values: np.ndarray, offsets: np.ndarray, *,
                 operation: str, input_dtype: str,
                 reference: np.ndarray | None = None,
                 scale: np.ndarray | None = None) -> dict[str, float]:
    """This build's stricter contract, on top of the reference's.

    * max: bit-exact values in the output dtype (the round-to-nearest-even
      of the maximum: the maximum itself unless a scale made it
      unrepresentable), signed zero excepted, same NaN / +-inf masks;
    * f32 sum:     |a - ref| <= 1e-5 * sum|x|   (cancellation-safe scale);
    * f32 softmax: |a - ref| <= 1e-5 * |ref| + FLT_MIN;
    * bf16 output: |a - RNE(ref)| <= 1 bf16 ulp of RNE(ref) (+ for sum
      2^-22 * sum|x|, the f32 accumulation allowance under cancellation;
      + FLT_MIN for flushed subnormals).
    """
    if reference is None:
        reference = REFERENCES[operation](values, offsets)
    expected = _expected(reference, input_dtype)
    actual = np.asarray(actual, dtype=np.float64)
    _compare_nonfinite(actual, expected)
    finite = np.isfinite(expected)
    if operation == "max":
        with np.errstate(over="ignore", invalid="ignore"):
            rounded = expected.astype(np.float32)
            if input_dtype == "bf16":
                rounded = quantize_bf16(rounded)
        exact = np.where(finite, actual == rounded.astype(np.float64), True)
        if not np.all(exact):
            raise AssertionError(f"max is not bit-exact at {int(np.sum(~exact))} positions")
        return {"max_abs_error": 0.0}
    if operation == "sum":
        if scale is None:
            scale = segment_sum(np.abs(values), offsets)
    else:
        scale = None
    if input_dtype == "f32":
        target = expected
        if operation == "sum":
            bound = STRICT_RTOL_F32 * scale
        else:
            bound = STRICT_RTOL_F32 * np.abs(expected) + FLT_MIN
    else:
        with np.errstate(over="ignore", invalid="ignore"):
            target = quantize_bf16(expected.astype(np.float32)).astype(np.float64)
        bound = bf16_ulp(target) + FLT_MIN
        if operation == "sum":
            bound = bound + 2.0 ** -22 * scale
    error = np.abs(actual - target)
    fails = finite & ~(error <= bound)
    if np.any(fails):
        where = np.argwhere(fails)[0]
        raise AssertionError(
            f"strict {operation}/{input_dtype}: {int(np.sum(fails))} values exceed the bound; "
            f"first at {tuple(where)}: actual={actual[tuple(where)]!r} expected={target[tuple(where)]!r}")
    err = error[finite]
    return {"max_abs_error": float(np.max(err, initial=0))}


__all__ = ["TOLERANCES", "assert_matches", "check_strict", "quantize_bf16", "segment_max",
           "segment_reduce", "segment_softmax", "segment_sum", "validate_offsets", "bf16_ulp"]
