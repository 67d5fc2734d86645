"""Generate the golden fixtures by running the REFERENCE oracle itself.

    python tests/golden/make_golden.py --reference PATH   (or RAGGED_MLIR_REFERENCE=PATH)

Imports ``oracle/reference.py`` and ``bench/distributions.py`` of the
reference checkout (simon-jd/ragged-mlir) named by --reference or the
RAGGED_MLIR_REFERENCE environment variable and writes ``golden.npz`` +
``golden.json`` next to this script.  Each case holds its inputs (values as
f32, already bf16-quantized for bf16 cases; offsets) and the reference's
float64 outputs for sum, max and softmax.  The cases restate the
known-answer tests of the reference's test/python/test_oracle.py and
test/gpu/test_correctness.py plus seeded random cases drawn with the
reference's own length generators (bench/distributions.py:15-64).
"""
from __future__ import annotations

import argparse
import os
import json
from pathlib import Path
import sys

import numpy as np

HERE = Path(__file__).resolve().parent


def cases(reference_bench):
    """(name, values f32 [N, D], offsets, dtype) tuples."""
    make_lengths = reference_bench.make_lengths
    offsets_from_lengths = reference_bench.offsets_from_lengths
    out = []
    hand = np.array([[1, 2], [3, 4], [-2, 7]], dtype=np.float32)
    for index in ("i32", "i64"):
        out.append((f"hand_{index}", hand, np.array([0, 2, 2, 3], dtype=np.int32 if index == "i32" else np.int64), "f32"))
    out.append(("nonfinite_columns", np.array([[np.nan, np.inf, -np.inf, -np.inf, 1],
                                               [1, 1, -np.inf, 3, 2]], dtype=np.float32),
                np.array([0, 2], dtype=np.int32), "f32"))
    out.append(("opposite_infinities", np.array([[np.inf], [-np.inf]], dtype=np.float32),
                np.array([0, 2], dtype=np.int32), "f32"))
    for d in (1, 3, 16):
        for offs in ([0], [0, 0], [0, 0, 0, 0]):
            out.append((f"empty_d{d}_b{len(offs) - 1}", np.empty((0, d), dtype=np.float32),
                        np.array(offs, dtype=np.int64), "f32"))
    tail = np.arange(4 * 3, dtype=np.float32).reshape(4, 3)
    for dtype in ("f32", "bf16"):
        out.append((f"tail_features_{dtype}", tail, np.array([0, 0, 1, 1, 4], dtype=np.int64), dtype))
    special = np.full((64, 5), -np.inf, dtype=np.float32)
    special[0] = [np.nan, np.inf, -np.inf, -np.inf, np.inf]
    special[1] = [1, 1, -np.inf, 3, -np.inf]
    for rows in (2, 64):
        for dtype in ("f32", "bf16"):
            out.append((f"softmax_special_r{rows}_{dtype}", special[:rows].copy(), np.array([0, rows], dtype=np.int64),
                        dtype))
    red = np.array([[np.nan, np.inf, -np.inf, -2], [1, -np.inf, -np.inf, -4]], dtype=np.float32)
    for dtype in ("f32", "bf16"):
        out.append((f"reduction_nonfinite_{dtype}", red, np.array([0, 2, 2], dtype=np.int64), dtype))
    lane = np.zeros((12, 128), dtype=np.float32)
    lane[0, :5] = [np.inf, -np.inf, np.inf, np.nan, 3]
    lane[4, :5] = [2, 2, -np.inf, 2, np.inf]
    lane[8, :5] = [3, 3, 3, 3, 2]
    out.append(("compensated_nonfinite_lanes", lane, np.array([0, 12], dtype=np.int64), "f32"))
    meta = np.random.default_rng(90).integers(-4, 5, size=(39, 7)).astype(np.float32)
    for dtype in ("f32", "bf16"):
        out.append((f"metamorphic_base_{dtype}", meta, np.array([0, 3, 3, 30, 39], dtype=np.int64), dtype))
    extremes = np.random.default_rng(8723).normal(size=(259, 3)).astype(np.float32) * 1000
    out.append(("softmax_extremes", extremes, np.array([0, 0, 1, 258, 259], dtype=np.int64), "f32"))
    # Seeded random cases with the reference's length distributions.
    for distribution in reference_bench.DISTRIBUTIONS:
        lengths = make_lengths(distribution, 48, total_elements=600, seed=711)
        for d, index in ((1, "i32"), (3, "i64"), (16, "i64")):
            offsets = offsets_from_lengths(lengths, index)
            values = np.random.default_rng(981).normal(size=(int(offsets[-1]), d)).astype(np.float32)
            for dtype in ("f32", "bf16"):
                out.append((f"random_{distribution}_d{d}_{index}_{dtype}", values, offsets, dtype))
    return out


def main() -> None:
    parser = argparse.ArgumentParser(description=__doc__)
    parser.add_argument("--reference", default=os.environ.get("RAGGED_MLIR_REFERENCE"),
                        help="path of the reference checkout (default: $RAGGED_MLIR_REFERENCE)")
    args = parser.parse_args()
    if not args.reference:
        parser.error("name the reference checkout with --reference or RAGGED_MLIR_REFERENCE")
    sys.path.insert(0, args.reference)
    from oracle import reference as ref  # the reference's own oracle
    from bench import distributions as dist  # the reference's own generators
    arrays, index = {}, []
    for name, values, offsets, dtype in cases(dist):
        values = np.ascontiguousarray(values, dtype=np.float32)
        if dtype == "bf16":
            values = ref.quantize_bf16(values)
        arrays[f"{name}__values"] = values
        arrays[f"{name}__offsets"] = offsets
        with np.errstate(all="ignore"):
            arrays[f"{name}__sum"] = ref.segment_sum(values, offsets)
            arrays[f"{name}__max"] = ref.segment_max(values, offsets)
            arrays[f"{name}__softmax"] = ref.segment_softmax(values, offsets)
        index.append({"name": name, "dtype": dtype, "n": int(values.shape[0]), "d": int(values.shape[1]),
                      "b": int(offsets.size - 1), "offsets_dtype": str(offsets.dtype)})
    np.savez_compressed(HERE / "golden.npz", **arrays)
    (HERE / "golden.json").write_text(json.dumps({"generator": "tests/golden/make_golden.py",
                                                  "reference": "simon-jd/ragged-mlir oracle/reference.py",
                                                  "cases": index}, indent=1) + "\n")
    print(f"{len(index)} cases -> {HERE / 'golden.npz'}")


if __name__ == "__main__":
    main()
