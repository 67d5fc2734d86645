"""ctypes binding of ``segred_oracle.c`` -- TEST INFRASTRUCTURE ONLY.

``build()`` compiles the C restatement with gcc/OpenMP into
``oracle/_build/libsegred_oracle.so`` (git-ignored; it travels to the GPU
box with the working tree).  The functions below return float64 results,
exactly like the reference oracle.
"""
from __future__ import annotations

import ctypes
import os
from pathlib import Path
import subprocess

import numpy as np

HERE = Path(__file__).resolve().parent
SOURCE = HERE / "segred_oracle.c"
LIBRARY = HERE / "_build" / "libsegred_oracle.so"

OPS = {"sum": 0, "max": 1, "softmax": 2, "abssum": 3}
DTYPES = {"f32": 0, "bf16": 1}
INDEX = {"i32": 0, "i64": 1}

_lib = None


def build(force: bool = False) -> Path:
    """Compile the oracle library if it is missing or older than its source."""
    if not force and LIBRARY.exists() and LIBRARY.stat().st_mtime >= SOURCE.stat().st_mtime:
        return LIBRARY
    LIBRARY.parent.mkdir(parents=True, exist_ok=True)
    tmp = LIBRARY.with_suffix(f".{os.getpid()}.tmp")
    subprocess.run(["gcc", "-O3", "-march=x86-64-v2", "-fopenmp", "-fPIC", "-shared", "-std=c11",
                    str(SOURCE), "-o", str(tmp), "-lm"], check=True)
    os.replace(tmp, LIBRARY)
    return LIBRARY


def _load():
    global _lib
    if _lib is None:
        build()
        lib = ctypes.CDLL(str(LIBRARY))
        i64, p, i = ctypes.c_int64, ctypes.c_void_p, ctypes.c_int
        lib.so_segment_reduce.argtypes = [i, i, i, i64, i64, i64, p, p, p, i]
        lib.so_segment_reduce.restype = i
        lib.so_segment_softmax.argtypes = [i, i, i64, i64, i64, p, p, p, i]
        lib.so_segment_softmax.restype = i
        lib.so_max_threads.restype = i
        _lib = lib
    return _lib


def max_threads() -> int:
    """Host threads this process may run on (its CPU affinity), independent
    of OMP_NUM_THREADS (which torchrun sets to 1): the count is passed to
    every call explicitly."""
    try:
        return max(1, len(os.sched_getaffinity(0)))
    except (AttributeError, OSError):
        return max(1, os.cpu_count() or 1)


def _prepare(values: np.ndarray, dtype: str, offsets: np.ndarray):
    if dtype == "bf16":
        if values.dtype == np.uint16:
            raw = np.ascontiguousarray(values)
        else:
            # f32 arrays that already hold bf16 values: keep the high halves.
            raw = np.ascontiguousarray((np.ascontiguousarray(values, dtype=np.float32)
                                        .view(np.uint32) >> 16).astype(np.uint16))
    else:
        raw = np.ascontiguousarray(values, dtype=np.float32)
    offsets = np.ascontiguousarray(offsets)
    if offsets.dtype not in (np.int32, np.int64):
        raise TypeError("offsets must be i32 or i64")
    index = "i32" if offsets.dtype == np.int32 else "i64"
    return raw, offsets, index


def segment_reduce(values: np.ndarray, offsets: np.ndarray, kind: str, *, dtype: str = "f32",
                   threads: int | None = None) -> np.ndarray:
    """Float64 [B, D] sum, max or sum of |x| (``kind`` "abssum": the scale of
    the sum tolerance); ``values`` is [N, D] f32 (or bf16 bits/values)."""
    raw, offsets, index = _prepare(values, dtype, offsets)
    n, d = raw.shape
    b = offsets.size - 1
    out = np.empty((b, d), dtype=np.float64)
    status = _load().so_segment_reduce(OPS[kind], DTYPES[dtype], INDEX[index], n, d, b,
                                       raw.ctypes.data, offsets.ctypes.data, out.ctypes.data,
                                       threads or max_threads())
    if status:
        raise RuntimeError(f"oracle segment_reduce failed ({status})")
    return out


def segment_softmax(values: np.ndarray, offsets: np.ndarray, *, dtype: str = "f32",
                    threads: int | None = None) -> np.ndarray:
    raw, offsets, index = _prepare(values, dtype, offsets)
    n, d = raw.shape
    b = offsets.size - 1
    out = np.empty((n, d), dtype=np.float64)
    status = _load().so_segment_softmax(DTYPES[dtype], INDEX[index], n, d, b, raw.ctypes.data,
                                        offsets.ctypes.data, out.ctypes.data, threads or max_threads())
    if status:
        raise RuntimeError(f"oracle segment_softmax failed ({status})")
    return out


def run(op: str, values: np.ndarray, offsets: np.ndarray, *, dtype: str = "f32",
        threads: int | None = None) -> np.ndarray:
    if op == "softmax":
        return segment_softmax(values, offsets, dtype=dtype, threads=threads)
    return segment_reduce(values, offsets, op, dtype=dtype, threads=threads)


def merge(kind: str, into: np.ndarray, piece: np.ndarray) -> np.ndarray:
    """Merge two float64 partial results of the same segments (rows of one
    segment split in two): the oracle's own cross-thread merge."""
    if kind == "max":
        return np.maximum(into, piece)  # np.maximum propagates NaN
    return into + piece


def check(actual: np.ndarray, op: str, dtype: str, offsets: np.ndarray, reference: np.ndarray,
          scale: np.ndarray | None = None) -> None:
    """Both tolerance contracts (the reference's ``assert_matches`` and
    ``check_strict``) for a result whose float64 oracle answer, and for sums
    the per-segment sum of |x|, were computed here (large inputs: no float64
    copy of the values is ever made)."""
    from . import reference_port as rp
    with np.errstate(all="ignore"):
        rp.assert_matches(actual, None, offsets, operation=op, input_dtype=dtype, reference=reference, scale=scale)
        rp.check_strict(actual, None, offsets, operation=op, input_dtype=dtype, reference=reference, scale=scale)
