"""Seeded synthetic workloads of the five benchmark configurations.

Lengths and offsets are generated on the host with NumPy (deterministic
PCG64 streams); values are generated where they are used (host arrays for
small cases, device tensors for the large ones; see ``bench.py``).

    c1  f32 sum, D=128, B=4096, lengths iid uniform in [1, 512], i64
    c2  f32 sum and max, D=1, B=200,000 x 64 rows, i32; the max variant has
        0.01% NaN values and 1% empty segments
    c3  bf16 softmax, D=128, B=16,384, lengths round(lognormal(3, 1.5))
        clipped to [0, 262144], 5% forced to 0, values N(0, 2^2), i64
    c4  f32 max and sum, D=2, B=10^6, 90% length 4 / 10% length 2048,
        shuffled, U[-1, 1] with 1e-4 NaN and 1e-4 -inf, i32
    c5  bf16 sum, D=256, N=200M, B=4M Zipf(1.2) lengths, i64

Recorded choices where the configuration text is ambiguous:

* c2 max: 2,000 segments (1%, seeded) become empty; to keep N = 12.8M their
  rows go one each to 128,000 of the other segments (seeded), which then
  have 65 rows.
* c5: Zipf(1.2) draws clipped to [1, 50M] and rescaled proportionally to
  the remaining rows with a floor of one row and largest-remainder rounding
  (integer arithmetic, so N is exact).  Taken alone that rule caps the
  longest segment near 2k rows (the clipped draws all tie at 50M), so no
  segment would exceed N / world_size and the cross-GPU split of giant
  segments would never run.  ``c5`` therefore reserves 3 x 50M rows for
  three giant segments (the clip bound) placed at seeded positions and
  applies the rule above to the other 4M - 3 segments and 50M rows.
  ``c5_literal`` is the rule alone, for comparison.
"""
from __future__ import annotations

from dataclasses import dataclass, field

import numpy as np

CONFIGS = ("c1", "c2_sum", "c2_max", "c3", "c4_max", "c4_sum", "c5", "c5_literal")


@dataclass
class Workload:
    name: str
    op: str
    dtype: str
    d: int
    index: str
    lengths: np.ndarray
    value_seed: int
    value_kind: str            # "normal", "normal2", "uniform"
    nan_fraction: float = 0.0
    neginf_fraction: float = 0.0
    notes: dict = field(default_factory=dict)

    @property
    def n(self) -> int:
        return int(self.lengths.sum())

    @property
    def b(self) -> int:
        return int(self.lengths.size)

    def offsets(self) -> np.ndarray:
        target = np.int32 if self.index == "i32" else np.int64
        out = np.zeros(self.b + 1, dtype=np.int64)
        np.cumsum(self.lengths, out=out[1:])
        if self.index == "i32" and out[-1] > np.iinfo(np.int32).max:
            raise ValueError("N does not fit i32 offsets")
        return out.astype(target)

    @property
    def element_bytes(self) -> int:
        return 4 if self.dtype == "f32" else 2

    def algorithmic_bytes(self) -> int:
        """values read + offsets read + output written (softmax: N rows)."""
        s_off = 4 if self.index == "i32" else 8
        rows_out = self.n if self.op == "softmax" else self.b
        return (self.n * self.d * self.element_bytes + (self.b + 1) * s_off
                + rows_out * self.d * self.element_bytes)

    def host_values(self, rows: slice | None = None) -> np.ndarray:
        """f32 values (bf16-quantised for bf16 workloads) for all rows or a
        leading slice; deterministic in ``value_seed``."""
        n = self.n if rows is None else len(range(*rows.indices(self.n)))
        rng = np.random.default_rng(self.value_seed)
        if self.value_kind == "uniform":
            values = rng.uniform(-1.0, 1.0, size=(n, self.d)).astype(np.float32)
        else:
            scale = 2.0 if self.value_kind == "normal2" else 1.0
            values = (rng.standard_normal(size=(n, self.d), dtype=np.float32) * np.float32(scale))
        special = np.random.default_rng(self.value_seed + 1)
        total = values.size
        for fraction, value in ((self.nan_fraction, np.nan), (self.neginf_fraction, -np.inf)):
            if fraction:
                count = max(1, int(round(total * fraction)))
                values.reshape(-1)[special.choice(total, size=count, replace=False)] = value
        if self.dtype == "bf16":
            values = quantize_bf16(values)
        return values


def device_values(w: Workload, rows: tuple[int, int], device) -> "torch.Tensor":  # noqa: F821
    """Values of rows [lo, hi) of ``w`` generated on a CUDA device with
    torch's generator, deterministic per chunk of 2^18 rows, so every rank
    of a sharded call builds exactly its slice of one dataset (the largest
    configuration does not fit host memory).  bf16 workloads are drawn in
    bf16 directly; NaN and -inf entries are placed at seeded positions."""
    import torch
    lo, hi = rows
    tdtype = torch.float32 if w.dtype == "f32" else torch.bfloat16
    out = torch.empty((hi - lo, w.d), dtype=tdtype, device=device)
    chunk = 1 << 18  # rows per generator chunk
    for c in range(lo // chunk, (hi + chunk - 1) // chunk):
        a, b = max(lo, c * chunk), min(hi, (c + 1) * chunk)
        g = torch.Generator(device=device)
        g.manual_seed(1_000_003 * w.value_seed + c)
        block = torch.empty((chunk, w.d), dtype=tdtype, device=device)
        if w.value_kind == "uniform":
            block.uniform_(-1.0, 1.0, generator=g)
        else:
            block.normal_(0.0, 2.0 if w.value_kind == "normal2" else 1.0, generator=g)
        if w.nan_fraction or w.neginf_fraction:
            u = torch.rand(block.shape, generator=g, device=device)
            block[u < w.nan_fraction] = float("nan")
            block[(u >= w.nan_fraction) & (u < w.nan_fraction + w.neginf_fraction)] = float("-inf")
            del u
        out[a - lo:b - lo] = block[a - c * chunk:b - c * chunk]
        del block
    return out


def quantize_bf16(values: np.ndarray) -> np.ndarray:
    """f32 -> bf16 RNE (NaN kept), as exact f32 values."""
    values = np.ascontiguousarray(values, dtype=np.float32)
    bits = values.view(np.uint32)
    with np.errstate(over="ignore"):
        rounded = (bits + np.uint32(0x7FFF) + ((bits >> 16) & 1)) & np.uint32(0xFFFF0000)
    rounded = np.where(np.isnan(values), np.uint32(0x7FC00000), rounded).astype(np.uint32)
    return rounded.view(np.float32)


def _proportional(weights: np.ndarray, total: int, floor: int = 1) -> np.ndarray:
    """Integer lengths >= floor summing to ``total``, proportional to
    ``weights`` above the floor, by largest remainder."""
    b = weights.size
    spare = total - floor * b
    if spare < 0:
        raise ValueError("total rows below the per-segment floor")
    w = np.asarray(weights, dtype=np.float64)
    share = w / w.sum() * spare
    base = np.floor(share).astype(np.int64)
    remainder = spare - int(base.sum())
    if remainder:
        order = np.argsort(-(share - base), kind="stable")[:remainder]
        base[order] += 1
    return base + floor


def make(name: str, *, scale: float = 1.0) -> Workload:
    """The workload ``name``; ``scale`` < 1 shrinks B (and N with it) for
    tests, keeping the length distribution."""
    if name not in CONFIGS:
        raise ValueError(f"workload must be one of {CONFIGS}")
    rng = np.random.default_rng(0)
    if name == "c1":
        b = max(1, int(4096 * scale))
        lengths = rng.integers(1, 513, size=b).astype(np.int64)
        return Workload(name, "sum", "f32", 128, "i64", lengths, 1, "normal")
    if name in ("c2_sum", "c2_max"):
        b = max(100, int(200_000 * scale))
        lengths = np.full(b, 64, dtype=np.int64)
        if name == "c2_sum":
            return Workload(name, "sum", "f32", 1, "i32", lengths, 1, "normal")
        empty = rng.choice(b, size=b // 100, replace=False)
        lengths[empty] = 0
        others = np.setdiff1d(np.arange(b), empty)
        extra = rng.choice(others, size=64 * empty.size, replace=False)
        lengths[extra] += 1
        return Workload(name, "max", "f32", 1, "i32", lengths, 1, "normal", nan_fraction=1e-4,
                        notes={"empty_segments": int(empty.size)})
    if name == "c3":
        b = max(16, int(16_384 * scale))
        lengths = np.clip(np.rint(rng.lognormal(3.0, 1.5, size=b)), 0, 262_144).astype(np.int64)
        lengths[rng.choice(b, size=int(round(0.05 * b)), replace=False)] = 0
        return Workload(name, "softmax", "bf16", 128, "i64", lengths, 1, "normal2")
    if name in ("c4_max", "c4_sum"):
        b = max(100, int(1_000_000 * scale))
        lengths = np.where(rng.random(b) < 0.9, 4, 2048).astype(np.int64)
        rng.shuffle(lengths)
        return Workload(name, name[3:], "f32", 2, "i32", lengths, 1, "uniform", nan_fraction=1e-4,
                        neginf_fraction=1e-4)
    # c5
    b = max(8, int(4_000_000 * scale))
    n = max(8 * b, int(200_000_000 * scale))
    cap = max(2, int(50_000_000 * scale))
    draws = np.clip(rng.zipf(1.2, size=b).astype(np.float64), 1, cap)
    if name == "c5_literal":
        lengths = _proportional(draws - 1, n, floor=1)
        return Workload(name, "sum", "bf16", 256, "i64", lengths, 1, "normal",
                        notes={"lengths_rule": "clip Zipf draws to [1, cap], proportional rescale, floor 1"})
    giants = min(3, b // 2)
    positions = rng.choice(b, size=giants, replace=False)
    body = np.setdiff1d(np.arange(b), positions)
    lengths = np.zeros(b, dtype=np.int64)
    lengths[positions] = cap
    lengths[body] = _proportional(draws[body] - 1, n - giants * cap, floor=1)
    return Workload(name, "sum", "bf16", 256, "i64", lengths, 1, "normal",
                    notes={"lengths_rule": "3 giant segments of 50M rows at seeded positions; the other "
                                           "segments: Zipf(1.2) draws clipped to [1, 50M], proportional "
                                           "rescale to the remaining rows, floor 1",
                           "giant_positions": sorted(int(p) for p in positions)})
