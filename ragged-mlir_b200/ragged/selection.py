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
in ``cost_model.json``.

This build has three schedules: the reference's ``classified`` and
``naive`` (block per segment) and, for sum/max, ``rowbalanced``.  Each
family has a default schedule (used when the caller gives no ``max_len``:
without length statistics the host cannot predict block per segment, whose
time depends on the longest segment); another schedule is chosen only when
its prediction beats the default's by the stored margin.
"""
from __future__ import annotations

from dataclasses import dataclass
import json
import math
from pathlib import Path
from typing import Any

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


@dataclass(frozen=True)
class CostModel:
    coefficients: dict[str, dict[str, tuple[float, ...]]]
    margin: float
    calibration: dict[str, Any]
    l2_mib: float = 126.0

    @classmethod
    def from_dict(cls, data: dict[str, Any]) -> "CostModel":
        try:
            if data["version"] != 3:
                raise CacheMismatch("unsupported cost model version")
            coefficients = {
                name: {schedule: tuple(float(v) for v in values) for schedule, values in data["coefficients"][name].items()}
                for name in FAMILIES}
            margin = float(data["margin"])
            l2_mib = float(data["l2_mib"])
        except (KeyError, TypeError, ValueError, AttributeError) as exc:
            raise CacheMismatch(f"invalid cost model: {exc}") from exc
        for name, schedules in coefficients.items():
            if DEFAULTS[name] not in schedules or any(s not in SCHEDULES for s in schedules):
                raise CacheMismatch(f"cost model family {name} must cover its default schedule")
            if any(len(values) != TERMS or any(v < 0 for v in values) for values in schedules.values()):
                raise CacheMismatch(f"cost model coefficients must be {TERMS} nonnegative terms")
        if not 0 <= margin < 1 or not l2_mib > 0:
            raise CacheMismatch("margin must lie in [0, 1) and the L2 capacity must be positive")
        return cls(coefficients, margin, dict(data.get("calibration", {})), l2_mib)

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
        if fam == "softmax" and d * element_bytes < NARROW_SOFTMAX_BYTES and len(candidates) > 1:
            candidates = [s for s in candidates if s != "rowbalanced"] or candidates
        default = DEFAULTS[fam] if DEFAULTS[fam] in candidates else candidates[0]
        if max_len is None:
            return default, {"max_len": None, "reason": "no length statistics on the host"}
        if l2_mib is not None and not (isinstance(l2_mib, (int, float)) and l2_mib > 0):
            raise ValueError("l2_mib must be a positive capacity in MiB")
        predicted = {s: self.predict(s, op, n, b, d, max_len, span, element_bytes, l2_mib) for s in candidates}
        best = min(candidates, key=lambda s: (predicted[s], s != default))
        selected = best if predicted[best] < predicted[default] * (1 - self.margin) else default
        return selected, {"max_len": max_len, "l2_mib": self.l2_mib if l2_mib is None else l2_mib,
                          "predicted_us": {s: round(v, 2) for s, v in predicted.items()}}


_model: CostModel | None = None


def default_model() -> CostModel:
    global _model
    if _model is None:
        _model = CostModel.load()
    return _model
