"""Oracle checks of device results too large to copy whole -- TEST INFRASTRUCTURE ONLY.

Used by the GPU tests at the benchmark configurations' full sizes and by
``bench.py``'s parity gate (the first call of a run, before anything is
timed).  Rows are copied from the device in bounded chunks and reduced by
the C float64 oracle (``segred_oracle.c``); the float64 partial results of a
segment's chunks are merged exactly as the oracle merges its threads'
pieces, so a 50M-row segment is checked with a few GB of host memory.
The per-segment sum of |x| (the scale of the sum tolerances) comes from
the same chunks.  Rows come from a caller's ``fetch(lo, hi)`` that returns
them as a host array the oracle reads (f32, or bf16 as raw uint16 bits), so
this module needs no device library.  Nothing here is on the product path.
"""
from __future__ import annotations

import numpy as np

from . import native

CHUNK_ROWS = 1 << 22


def segment_partials(fetch, rows: int, d: int, offsets: np.ndarray, segments: np.ndarray, *, kinds,
                     dtype: str, row_base: int = 0, chunk_rows: int = CHUNK_ROWS) -> list[np.ndarray]:
    """Float64 [len(segments), D] results, one per entry of ``kinds``
    ("sum", "max", "abssum"), of the rows of each listed segment that lie in
    the caller's rows [row_base, row_base + rows) of the whole array
    (``fetch(lo, hi)`` returns local rows lo..hi, each fetched once for all
    kinds); segments must be sorted.  Consecutive segments are fetched
    together up to ``chunk_rows``."""
    offsets = np.asarray(offsets, dtype=np.int64)
    segments = np.asarray(segments, dtype=np.int64)
    lo_row, hi_row = row_base, row_base + rows
    identity = {kind: -np.inf if kind == "max" else 0.0 for kind in kinds}
    out = [np.full((segments.size, d), identity[kind], dtype=np.float64) for kind in kinds]
    starts = np.clip(offsets[segments], lo_row, hi_row)
    ends = np.clip(offsets[segments + 1], lo_row, hi_row)
    ends = np.maximum(ends, starts)
    i = 0
    while i < segments.size:
        if ends[i] - starts[i] > chunk_rows:  # a long segment: chunk by chunk
            totals = [np.full(d, identity[kind]) for kind in kinds]
            for a in range(int(starts[i]), int(ends[i]), chunk_rows):
                b = min(int(ends[i]), a + chunk_rows)
                block = fetch(a - row_base, b - row_base)
                whole = np.array([0, b - a], dtype=np.int64)
                for k, kind in enumerate(kinds):
                    piece = native.segment_reduce(block, whole, kind, dtype=dtype)[0]
                    totals[k] = native.merge(kind, totals[k], piece)
            for k in range(len(kinds)):
                out[k][i] = totals[k]
            i += 1
            continue
        j = i  # a run of segments sharing one copy (contiguous rows)
        while j + 1 < segments.size and segments[j + 1] == segments[j] + 1 and \
                ends[j + 1] - starts[i] <= chunk_rows:
            j += 1
        a, b = int(starts[i]), int(ends[j])
        block = fetch(a - row_base, b - row_base)
        # Consecutive segments: each clipped end is the next clipped start.
        local = np.concatenate([[0], ends[i:j + 1] - a]).astype(np.int64)
        for k, kind in enumerate(kinds):
            out[k][i:j + 1] = native.segment_reduce(block, local, kind, dtype=dtype)
        i = j + 1
    return out


def check_reduction(actual: np.ndarray, fetch, rows: int, offsets: np.ndarray, segments: np.ndarray, *, op: str,
                    dtype: str, chunk_rows: int = CHUNK_ROWS) -> None:
    """``actual`` (float64 [len(segments), D], the device output rows of
    ``segments``) against the oracle over all ``rows`` rows: both tolerance
    contracts."""
    kinds = (op, "abssum") if op == "sum" else (op,)
    parts = segment_partials(fetch, rows, actual.shape[1], offsets, segments, kinds=kinds, dtype=dtype,
                             chunk_rows=chunk_rows)
    reference, scale = parts[0], (parts[1] if op == "sum" else None)
    lengths = np.asarray(offsets, dtype=np.int64)[np.asarray(segments) + 1] - \
        np.asarray(offsets, dtype=np.int64)[np.asarray(segments)]
    local = np.concatenate([[0], np.cumsum(lengths)]).astype(np.int64)
    native.check(actual, op, dtype, local, reference, scale)


def check_softmax(actual: np.ndarray, rows: np.ndarray, offsets: np.ndarray, *, dtype: str) -> None:
    """A whole softmax output (float64 [N, D]) against the oracle; ``rows``
    are all the input rows as the oracle reads them."""
    reference = native.segment_softmax(rows, np.asarray(offsets), dtype=dtype)
    native.check(actual, "softmax", dtype, np.asarray(offsets, dtype=np.int64), reference)
