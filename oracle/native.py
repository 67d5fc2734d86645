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

OPS = {"sum": 0, "max": 1, "softmax": 2}
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
    return int(_load().so_max_threads())


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
    """Float64 [B, D] sum or max; ``values`` is [N, D] f32 (or bf16 bits/values)."""
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
