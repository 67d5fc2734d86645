"""Immutable program specification and per-call execution evidence.

Mirrors the reference's python/ragged/model.py (ProgramSpec 129-212, Hints
114-127, ExecutionReport 256-293) with the B200 target: the only chip is
``sm_100a`` (compute capability 10.0) and its per-CTA limits.  ``mask``
and ``scale`` take the materialised input transform (rg_run_pointwise),
``alias="inplace"`` the in-place softmax flag; ``debug_visits`` is validated
as in the reference and rejected by ``Compiler.compile`` with a
``CompilationError``.
"""
from __future__ import annotations

from dataclasses import asdict, dataclass, field
import hashlib
import json
import math
from typing import Any

from .errors import ValidationError
from .optimizations import Optimizations

DIALECT_VERSION = "1"


@dataclass(frozen=True)
class ChipLimits:
    """Per-CTA limits of a target chip: opt-in shared memory bytes, 32-bit
    registers and threads (B200: 227 KiB, 64 Ki registers, 1024 threads)."""
    shared_per_cta: int
    registers_per_cta: int
    threads_per_cta: int


DEFAULT_CHIP = "sm_100a"
CHIPS = {"sm_100a": ChipLimits(232448, 65536, 1024)}


def chip_capability(chip: str) -> tuple[int, int]:
    """(major, minor) compute capability of a supported chip name."""
    if chip not in CHIPS:
        raise ValidationError("chip must be sm_100a")
    return 10, 0


def runs_on(chip: str, capability: tuple[int, int]) -> bool:
    """sm_100a code runs only on compute capability 10.0 (the 'a' suffix
    features do not carry to later chips)."""
    return tuple(capability) == chip_capability(chip)


def canonical_json(value: Any) -> str:
    return json.dumps(value, sort_keys=True, separators=(",", ":"), allow_nan=False)


def _nonnegative_int(name: str, value: int | None) -> None:
    if value is not None and (type(value) is not int or value < 0 or value > 2**63 - 1):
        raise ValidationError(f"{name} must be an integer in [0, 2^63-1]")


@dataclass(frozen=True)
class Hints:
    max_len: int | None = None
    min_len: int | None = None
    offsets_checked: bool = False

    def __post_init__(self) -> None:
        _nonnegative_int("max_len", self.max_len)
        _nonnegative_int("min_len", self.min_len)
        if type(self.offsets_checked) is not bool:
            raise ValidationError("offsets_checked must be bool")
        if self.max_len is not None and self.min_len is not None and self.min_len > self.max_len:
            raise ValidationError("min_len must not exceed max_len")


@dataclass(frozen=True)
class ProgramSpec:
    op: str
    dtype: str = "f32"
    feature_dim: int = 128
    offsets_dtype: str = "i64"
    hints: Hints = field(default_factory=Hints)
    strategy: str = "auto"
    alias: str = "none"
    chip: str = DEFAULT_CHIP
    force_fusion: bool = False
    scale: float = 1.0
    debug_visits: bool = False
    mask: bool = False
    optimizations: Optimizations = field(default_factory=Optimizations)
    smem_per_cta: int = 232448
    regs_budget: int = 65536

    def __post_init__(self) -> None:
        if self.op not in ("sum", "max", "softmax"):
            raise ValidationError("op must be sum, max or softmax")
        if self.dtype not in ("f32", "bf16"):
            raise ValidationError("dtype must be f32 or bf16; accumulation is always f32")
        if type(self.feature_dim) is not int or not 1 <= self.feature_dim <= 1024:
            raise ValidationError("feature_dim must be a static integer in [1, 1024]")
        if self.offsets_dtype not in ("i32", "i64"):
            raise ValidationError("offsets_dtype must be i32 or i64")
        if not isinstance(self.hints, Hints):
            raise ValidationError("hints must be Hints")
        if self.strategy not in ("auto", "naive"):
            raise ValidationError("strategy must be auto or naive")
        if self.alias not in ("none", "inplace"):
            raise ValidationError("alias must be none or inplace")
        if self.alias == "inplace" and self.op != "softmax":
            raise ValidationError("in-place output is only defined for softmax")
        if self.chip not in CHIPS:
            raise ValidationError("chip must be sm_100a")
        for name in ("force_fusion", "debug_visits", "mask"):
            if type(getattr(self, name)) is not bool:
                raise ValidationError(f"{name} must be bool")
        if self.mask and self.op != "softmax":
            raise ValidationError("additive mask is only defined for softmax")
        if not isinstance(self.optimizations, Optimizations):
            raise ValidationError("optimizations must be Optimizations")
        if self.debug_visits and not self.optimizations.classification:
            raise ValidationError("debug_visits requires classification")
        if self.force_fusion and not self.optimizations.online_fusion:
            raise ValidationError("force_fusion conflicts with online_fusion disabled")
        if self.force_fusion and self.op != "softmax":
            raise ValidationError("force_fusion is only defined for softmax")
        if (type(self.scale) not in (int, float) or not math.isfinite(self.scale)
                or abs(self.scale) > 3.402823466e38):
            raise ValidationError("scale must be a finite f32 value")
        for name in ("smem_per_cta", "regs_budget"):
            value = getattr(self, name)
            if type(value) is not int or not 1 <= value <= 2**63 - 1:
                raise ValidationError(f"{name} must be a positive signed i64 integer")

    @property
    def signature(self) -> str:
        return f"{self.op}:{self.dtype}:D{self.feature_dim}:{self.offsets_dtype}:{self.chip}"

    def to_dict(self) -> dict[str, Any]:
        return asdict(self)

    @classmethod
    def from_dict(cls, data: dict[str, Any]) -> "ProgramSpec":
        data = dict(data)
        data["hints"] = Hints(**data.get("hints", {}))
        data["optimizations"] = Optimizations(**data.get("optimizations", {}))
        return cls(**data)

    def canonical_source(self) -> str:
        """Stable text naming this specialization (replaces the reference's
        generated MLIR text as the input of ``ir_hash``)."""
        return canonical_json({"dialect": DIALECT_VERSION, "spec": self.to_dict()})

    @property
    def ir_hash(self) -> str:
        return hashlib.sha256(self.canonical_source().encode()).hexdigest()


@dataclass(frozen=True)
class ExecutionReport:
    classes: tuple[str, ...]
    thresholds: tuple[int, ...]
    grids: tuple[tuple[int, int, int], ...]
    workspace_bytes: int
    cache_key: str
    fallback_reason: str | None = None
    mode: str = "validated"
    kernel_names: tuple[str, ...] = ()
    host_enqueue_ms: float | None = None
    device_elapsed_ms: float | None = None
    cache_hit: bool = False
    validation_workspace_bytes: int = 0
    validation_host_ms: float | None = None
    optimizations: dict[str, Any] | None = None
    d_tile: int | None = None
    d_vector: int = 1
    pointwise_materialized: bool = False
    resources: dict[str, Any] | None = None
    streams: int = 1
    selected: str | None = None
    selection: dict[str, Any] | None = None

    def to_dict(self) -> dict[str, Any]:
        return asdict(self)

    def to_json(self) -> str:
        return json.dumps(self.to_dict(), sort_keys=True, indent=2, allow_nan=False)
