"""Optimization requests (the reference's python/ragged/optimizations.py:13-60).

The eight boolean controls and ``feature_tile`` are accepted and validated
exactly as in the reference so that existing ``ProgramSpec`` values keep
working.  On B200 the kernels are built in, so the controls that select
compiler passes only select among the built-in schedules:

* ``classification=False`` makes a program use block-per-segment only;
* ``vectorize=False`` makes every thread access one feature at a time
  (``RG_FLAG_NO_VECTORIZE``);
* ``pointwise_fusion=False`` makes a scale or mask always go through
  materialised f32 logits (``RG_FLAG_NO_POINTWISE_FUSION``); otherwise a
  softmax on the classified schedule applies it as it loads;
* the other flags are recorded in the report and otherwise have no effect.
"""
from __future__ import annotations

from dataclasses import asdict, dataclass

from .errors import ValidationError

BOOL_OPTIONS = ("classification", "online_fusion", "warp_mapping", "split_mapping", "shuffle", "pointwise_fusion",
                "row_pipelining", "vectorize")
VECTOR_WIDTHS = (1, 2, 4, 8)
FEATURE_TILES = (1, 2, 4, 8, 16, 32)


@dataclass(frozen=True)
class Optimizations:
    classification: bool = True
    online_fusion: bool = True
    warp_mapping: bool = True
    split_mapping: bool = True
    shuffle: bool = True
    pointwise_fusion: bool = True
    row_pipelining: bool = True
    vectorize: bool = True
    feature_tile: int | None = None

    def __post_init__(self):
        for name in BOOL_OPTIONS:
            if type(getattr(self, name)) is not bool:
                raise ValidationError(f"optimization {name} must be bool")
        if self.feature_tile is not None and (type(self.feature_tile) is not int
                                              or self.feature_tile not in FEATURE_TILES):
            raise ValidationError("feature_tile must be None or a power of two in [1,32]")

    def to_dict(self):
        return asdict(self)

    def effects(self, *, transformed: bool = False) -> dict[str, list[str]]:
        """Which requested controls change what a call runs ("applied") and
        which are accepted but change nothing on B200 ("no_effect"); every
        ExecutionReport carries this next to the request.  ``transformed``:
        the call has a scale or mask, the only case pointwise_fusion
        selects anything for."""
        applied = ["classification", "vectorize"]
        if transformed:
            applied.append("pointwise_fusion")
        ignored = [name for name in BOOL_OPTIONS if name not in applied] + ["feature_tile"]
        return {"applied": applied, "no_effect": ignored}

    def geometry(self, d: int, dtype: str = "f32") -> tuple[int, int]:
        """(d_tile, d_vector) of the B200 kernels: each thread owns d_vector
        adjacent features (the largest power of two dividing D that fits 16
        bytes, as in the reference's rule) and d_tile = min(32,
        pow2ceil(D / d_vector)) threads span one row tile."""
        element = 2 if dtype == "bf16" else 4
        vec = 1
        if self.vectorize:
            while 2 * vec * element <= 16 and d % (2 * vec) == 0:
                vec *= 2
        columns = d // vec
        tile = 1
        while tile < columns and tile < 32:
            tile *= 2
        return tile, vec
