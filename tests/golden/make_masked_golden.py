"""Generate the scale / mask golden fixtures by running the REFERENCE oracle.

    python tests/golden/make_masked_golden.py --reference PATH   (or RAGGED_MLIR_REFERENCE=PATH)

Imports ``oracle/masked.py`` and ``oracle/reference.py`` of the reference
checkout (simon-jd/ragged-mlir) named by --reference or the
RAGGED_MLIR_REFERENCE environment variable and writes ``masked.npz`` + ``masked.json`` next to this
script.  Each case holds its inputs (values as f32, already bf16-quantized
for bf16 cases; the f32 mask; the scale; offsets), the reference's
transformed logits (``masked_logits``) and its float64 softmax of them.  The
cases restate the reference's test/gpu/test_mask.py value patterns:
cancellation against the values dtype, separate f32 roundings of the scale
and the mask, non-finite masks and fully masked columns, and seeded random
masks.
"""
from __future__ import annotations

import argparse
import os
import json
from pathlib import Path
import sys

import numpy as np

HERE = Path(__file__).resolve().parent


def cases():
    """(name, values f32 [N, D], mask f32 [N, D], scale, offsets, dtype)."""
    out = []
    offsets = np.array([0, 5, 5, 6, 14], dtype=np.int64)
    n = int(offsets[-1])
    rng = np.random.default_rng(951)
    for dtype in ("f32", "bf16"):
        values = rng.normal(size=(n, 7)).astype(np.float32)
        mask = rng.uniform(-3, 3, size=(n, 7)).astype(np.float32)
        out.append((f"random_{dtype}", values, mask, 0.75, offsets, dtype))
        # Cancellation: the f32 mask must not be rounded to the values dtype.
        out.append((f"cancellation_{dtype}", np.full((n, 7), 65536, dtype=np.float32),
                    np.full((n, 7), -32772, dtype=np.float32), 0.5, offsets, dtype))
    # Two roundings: x * scale rounds before the mask is added.
    values = np.full((n, 3), np.float32(1.0) + np.float32(2.0 ** -23), dtype=np.float32)
    mask = np.full((n, 3), np.float32(-1.0), dtype=np.float32)
    out.append(("separate_roundings", values, mask, 1.0 + 2.0 ** -22, offsets, "f32"))
    # Non-finite masks and fully masked columns.
    values = rng.normal(size=(n, 5)).astype(np.float32)
    mask = np.zeros((n, 5), dtype=np.float32)
    mask[:, 0] = -np.inf                # column 0 fully masked: NaN
    mask[0:5, 1] = [-np.inf, 0, -np.inf, 0, -np.inf]
    mask[5, 2] = np.inf                 # +inf logit: NaN
    mask[6:14, 3] = np.nan
    values[7, 4] = np.inf
    mask[7, 4] = -np.inf                # +inf + -inf = NaN
    for scale in (0.0, 0.5):
        out.append((f"nonfinite_scale{scale}", values, mask, scale, offsets, "f32"))
    for d, index in ((1, "i32"), (16, "i64")):
        offs = np.array([0, 0, 3, 40, 41, 100], dtype=np.int32 if index == "i32" else np.int64)
        vals = rng.normal(scale=2.0, size=(int(offs[-1]), d)).astype(np.float32)
        msk = np.where(rng.random(size=vals.shape) < 0.2, -np.inf, rng.normal(size=vals.shape)).astype(np.float32)
        for dtype in ("f32", "bf16"):
            out.append((f"sparse_mask_d{d}_{index}_{dtype}", vals, msk, -1.25, offs, dtype))
    return out


def main() -> None:
    parser = argparse.ArgumentParser(description=__doc__)
    parser.add_argument("--reference", default=os.environ.get("RAGGED_MLIR_REFERENCE"),
                        help="path of the reference checkout (default: $RAGGED_MLIR_REFERENCE)")
    args = parser.parse_args()
    if not args.reference:
        parser.error("name the reference checkout with --reference or RAGGED_MLIR_REFERENCE")
    sys.path.insert(0, args.reference)
    from oracle import masked as ref_masked  # the reference's own oracle
    from oracle import reference as ref
    arrays, index = {}, []
    for name, values, mask, scale, offsets, dtype in cases():
        values = np.ascontiguousarray(values, dtype=np.float32)
        if dtype == "bf16":
            values = ref.quantize_bf16(values)
        logits = ref_masked.masked_logits(values, mask, scale=scale)
        arrays[f"{name}__values"] = values
        arrays[f"{name}__mask"] = mask
        arrays[f"{name}__offsets"] = offsets
        arrays[f"{name}__logits"] = logits
        with np.errstate(all="ignore"):
            arrays[f"{name}__softmax"] = ref.segment_softmax(logits, offsets)
        index.append({"name": name, "dtype": dtype, "scale": float(scale), "n": int(values.shape[0]),
                      "d": int(values.shape[1]), "b": int(offsets.size - 1), "offsets_dtype": str(offsets.dtype)})
    np.savez_compressed(HERE / "masked.npz", **arrays)
    (HERE / "masked.json").write_text(json.dumps({"generator": "tests/golden/make_masked_golden.py",
                                                  "reference": "simon-jd/ragged-mlir oracle/masked.py",
                                                  "cases": index}, indent=1) + "\n")
    print(f"{len(index)} cases -> {HERE / 'masked.npz'}")


if __name__ == "__main__":
    main()
