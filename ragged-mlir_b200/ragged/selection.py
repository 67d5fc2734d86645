"""Choosing a schedule per call from cheap host statistics.

Restates the reference's cost model (python/ragged/selection.py:1-136):
the predicted complete-call time of each schedule is linear in six terms,

    t_us = c0 + c1*M + c2*S + c3*B/1000 + c4*M*log2(skew) + c5*X

with M = N*D / 2^18 elements, S = L*span/128/1000 (the rows one thread of
the block that owns the longest segment L walks, span = d_tile*d_vector),
skew = L*B/N and X = MiB of the call's working set (input rows plus output)
beyond the device's L2, queried at run time.  Coefficients are nonnegative,
fitted per operation family ("reduce" for sum/max, "softmax") and schedule
with NNLS on B200 measurements (``python -m ragged.calibrate``) and stored
in ``cost_model.json``.  The report carries these predictions.

On B200 the linear times choose the fastest schedule for about three calls
in four of the calibration suite's held-out group; a version-4 model adds a
``TreeChooser`` that makes the choice: gradient-boosted decision trees over
``choice_features`` (logarithms of N, B, row bytes, the longest segment, the
mean length, skew and bytes, plus the dtype and operation), fitted to which
schedule was fastest on the training group.  It picks a schedule within 3%
of the fastest for about nine calls in ten of the held-out group (the
figures of the shipped model are in its ``calibration`` entry).

This build has three schedules: the reference's ``classified`` and
``naive`` (block per segment) and, for sum/max, ``rowbalanced``.  Each
family has a default schedule (used when the caller gives no ``max_len``:
without length statistics the host cannot predict block per segment, whose
time depends on the longest segment); with a version-3 (linear-only) model
another schedule is chosen only when its prediction beats the default's by
the stored margin.
"""
from __future__ import annotations

from dataclasses import dataclass
from functools import cached_property
import json
import math
from pathlib import Path
from typing import Any

import numpy as np

from .errors import CacheMismatch

MODEL_PATH = Path(__file__).with_name("cost_model.json")
SCHEDULES = ("classified", "naive", "rowbalanced")
FAMILIES = ("reduce", "softmax")
TERMS = 6
DEFAULTS = {"reduce": "rowbalanced", "softmax": "classified"}


# Softmax rows narrower than this take no row-balanced schedule from the
# cost model: with one lane per row its segment walk loads one segment end
# per step, and runs of empty segments (1.7M of them in one B200
# calibration case) made it 400x slower than the classified schedule, a
# cost the linear model cannot see.  select="rowbalanced" still runs it.
NARROW_SOFTMAX_BYTES = 64


def family(op: str) -> str:
    return "softmax" if op == "softmax" else "reduce"


def features(n: int, b: int, d: int, max_len: int, span: int, element_bytes: int = 4, op: str = "sum",
             l2_mib: float = 126.0) -> tuple[float, ...]:
    """The six terms (selection.py:56-70 of the reference, version 2)."""
    elements = n * d / 2**18
    skew = max_len * b / n if n else 1.0
    rows = n * d * element_bytes / 2**20
    output_rows = n if op == "softmax" else b
    excess = max(0.0, rows + output_rows * d * element_bytes / 2**20 - l2_mib)
    return (1.0, elements, max_len * span / 128 / 1000.0, b / 1000.0,
            elements * math.log2(max(1.0, skew)), excess)


CHOICE_FEATURES = "choice-v1"


def choice_features(op: str, n: int, b: int, d: int, max_len: int, element_bytes: int) -> np.ndarray:
    """Inputs of the tree chooser (feature set ``choice-v1``)."""
    row_bytes = d * element_bytes
    mean = n / max(b, 1)
    longest = max(max_len, 1)
    return np.array([math.log2(max(n, 1)), math.log2(max(b, 1)), math.log2(row_bytes), math.log2(longest),
                     math.log2(max(mean, 1e-3)), math.log2(longest / max(mean, 1e-3)),
                     math.log2(max(n * row_bytes, 1)), float(element_bytes == 2), float(op == "max"),
                     float(op == "softmax")], dtype=np.float64)


@dataclass(frozen=True, eq=False)
class TreeChooser:
    """Boosted trees, one per schedule and boosting round, flattened into
    node arrays: node i tests feature[i] <= threshold[i] (left, else right)
    unless it is a leaf holding value[i].  A schedule's score is its
    baseline plus its trees' leaf values; the highest score among the
    available schedules is chosen."""

    classes: tuple[str, ...]
    baseline: np.ndarray
    feature: np.ndarray
    threshold: np.ndarray
    left: np.ndarray
    right: np.ndarray
    value: np.ndarray
    leaf: np.ndarray
    roots: np.ndarray
    tree_class: np.ndarray
    max_depth: int

    @classmethod
    def from_dict(cls, data: dict[str, Any]) -> "TreeChooser":
        if data.get("features") != CHOICE_FEATURES:
            raise CacheMismatch("tree chooser built for another feature set")
        classes = tuple(str(c) for c in data["classes"])
        if not classes or len(set(classes)) != len(classes) or any(c not in SCHEDULES for c in classes):
            raise CacheMismatch("tree chooser classes must be distinct schedules")
        nodes = data["nodes"]
        feature = np.asarray(nodes["feature"], dtype=np.int64)
        count = feature.size
        arrays = dict(threshold=np.asarray(nodes["threshold"], dtype=np.float64),
                      left=np.asarray(nodes["left"], dtype=np.int64), right=np.asarray(nodes["right"], dtype=np.int64),
                      value=np.asarray(nodes["value"], dtype=np.float64), leaf=np.asarray(nodes["leaf"], dtype=bool))
        roots = np.asarray(data["roots"], dtype=np.int64)
        tree_class = np.asarray(data["tree_class"], dtype=np.int64)
        baseline = np.asarray(data["baseline"], dtype=np.float64)
        width = choice_features("sum", 1, 1, 1, 1, 4).size
        inner = ~arrays["leaf"]
        if (any(a.shape != (count,) for a in arrays.values()) or roots.shape != tree_class.shape
                or baseline.shape != (len(classes),) or not roots.size
                or np.any((roots < 0) | (roots >= count)) or np.any((tree_class < 0) | (tree_class >= len(classes)))
                or np.any(inner & ((feature < 0) | (feature >= width)))
                or np.any(inner & ((arrays["left"] < 0) | (arrays["left"] >= count)))
                or np.any(inner & ((arrays["right"] < 0) | (arrays["right"] >= count)))
                or not np.all(np.isfinite(arrays["value"][arrays["leaf"]]))):
            raise CacheMismatch("malformed tree chooser")
        max_depth = int(data["max_depth"])
        if not 0 <= max_depth <= 64:
            raise CacheMismatch("tree chooser depth out of range")
        feature = np.where(inner, feature, 0)
        chooser = cls(classes, baseline, feature, arrays["threshold"], arrays["left"], arrays["right"],
                      arrays["value"], arrays["leaf"], roots, tree_class, max_depth)
        for *x, expected in data.get("checks", []):
            if chooser.classes[int(np.argmax(chooser.scores(np.asarray(x, dtype=np.float64))))] != expected:
                raise CacheMismatch("tree chooser does not reproduce its recorded choices")
        return chooser

    @cached_property
    def native_arrays(self) -> dict:
        """The node arrays in the layout rg_tree_scores reads."""
        i32 = lambda a: np.ascontiguousarray(a, dtype=np.int32)
        f64 = lambda a: np.ascontiguousarray(a, dtype=np.float64)
        return {"feature": i32(self.feature), "threshold": f64(self.threshold), "left": i32(self.left),
                "right": i32(self.right), "value": f64(self.value), "leaf": np.ascontiguousarray(self.leaf, np.uint8),
                "roots": i32(self.roots), "tree_class": i32(self.tree_class), "baseline": f64(self.baseline)}

    def fast_scores(self, x: np.ndarray) -> np.ndarray:
        """``scores`` computed by libragged_b200 (one walk per tree in C, a few
        microseconds); the NumPy walk where the library cannot be loaded
        (fitting a model on a machine without the build).  Both make the
        same comparisons in float64."""
        from . import _native
        from .errors import RuntimeUnavailable
        try:
            _native.library()
        except RuntimeUnavailable:
            return self.scores(x)
        return _native.tree_scores(self.native_arrays, x, len(self.classes), self.max_depth)

    def scores(self, x: np.ndarray) -> np.ndarray:
        node = self.roots.copy()
        for _ in range(self.max_depth + 1):
            live = ~self.leaf[node]
            if not live.any():
                break
            at = node[live]
            node[live] = np.where(x[self.feature[at]] <= self.threshold[at], self.left[at], self.right[at])
        else:
            raise CacheMismatch("tree chooser deeper than its recorded depth")
        return self.baseline + np.bincount(self.tree_class, weights=self.value[node], minlength=len(self.classes))


@dataclass(frozen=True)
class CostModel:
    coefficients: dict[str, dict[str, tuple[float, ...]]]
    margin: float
    calibration: dict[str, Any]
    l2_mib: float = 126.0
    chooser: TreeChooser | None = None

    @classmethod
    def from_dict(cls, data: dict[str, Any]) -> "CostModel":
        try:
            if data["version"] not in (3, 4):
                raise CacheMismatch("unsupported cost model version")
            chooser = TreeChooser.from_dict(data["chooser"]) if data["version"] == 4 else None
            coefficients = {
                name: {schedule: tuple(float(v) for v in values) for schedule, values in data["coefficients"][name].items()}
                for name in FAMILIES}
            margin = float(data["margin"])
            l2_mib = float(data["l2_mib"])
        except (KeyError, TypeError, ValueError, AttributeError, IndexError) as exc:
            raise CacheMismatch(f"invalid cost model: {exc}") from exc
        for name, schedules in coefficients.items():
            if DEFAULTS[name] not in schedules or any(s not in SCHEDULES for s in schedules):
                raise CacheMismatch(f"cost model family {name} must cover its default schedule")
            if any(len(values) != TERMS or any(v < 0 for v in values) for values in schedules.values()):
                raise CacheMismatch(f"cost model coefficients must be {TERMS} nonnegative terms")
        if not 0 <= margin < 1 or not l2_mib > 0:
            raise CacheMismatch("margin must lie in [0, 1) and the L2 capacity must be positive")
        return cls(coefficients, margin, dict(data.get("calibration", {})), l2_mib, chooser)

    @classmethod
    def load(cls, path: Path = MODEL_PATH) -> "CostModel":
        return cls.from_dict(json.loads(Path(path).read_text()))

    def predict(self, schedule: str, op: str, n: int, b: int, d: int, max_len: int, span: int,
                element_bytes: int = 4, l2_mib: float | None = None) -> float:
        terms = features(n, b, d, max_len, span, element_bytes, op, self.l2_mib if l2_mib is None else l2_mib)
        return sum(c * x for c, x in zip(self.coefficients[family(op)][schedule], terms))

    def choose(self, op: str, n: int, b: int, d: int, max_len: int | None, span: int, element_bytes: int = 4,
               l2_mib: float | None = None, available: tuple[str, ...] | None = None) -> tuple[str, dict[str, Any]]:
        """The schedule to run and the predictions behind it."""
        fam = family(op)
        candidates = [s for s in (available or SCHEDULES) if s in self.coefficients[fam]]
        if (self.chooser is None and fam == "softmax" and d * element_bytes < NARROW_SOFTMAX_BYTES
                and len(candidates) > 1):
            candidates = [s for s in candidates if s != "rowbalanced"] or candidates
        default = DEFAULTS[fam] if DEFAULTS[fam] in candidates else candidates[0]
        if max_len is None:
            return default, {"max_len": None, "reason": "no length statistics on the host"}
        if l2_mib is not None and not (isinstance(l2_mib, (int, float)) and l2_mib > 0):
            raise ValueError("l2_mib must be a positive capacity in MiB")
        predicted = {s: self.predict(s, op, n, b, d, max_len, span, element_bytes, l2_mib) for s in candidates}
        details = {"max_len": max_len, "l2_mib": self.l2_mib if l2_mib is None else l2_mib,
                   "predicted_us": {s: round(v, 2) for s, v in predicted.items()}}
        ranked = [s for s in candidates if self.chooser is not None and s in self.chooser.classes]
        if ranked:
            scores = self.chooser.fast_scores(choice_features(op, n, b, d, max_len, element_bytes))
            score = {s: float(scores[self.chooser.classes.index(s)]) for s in ranked}
            details["scores"] = {s: round(v, 4) for s, v in score.items()}
            return max(ranked, key=lambda s: (score[s], s == default)), details
        best = min(candidates, key=lambda s: (predicted[s], s != default))
        selected = best if predicted[best] < predicted[default] * (1 - self.margin) else default
        return selected, details


_model: CostModel | None = None


def default_model() -> CostModel:
    global _model
    if _model is None:
        _model = CostModel.load()
    return _model
