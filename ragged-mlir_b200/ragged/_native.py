"""ctypes binding of libragged_b200.so (C ABI: include/ragged_b200.h).

Replaces the reference's nanobind module ``ragged._native`` (runtime/
bindings.cpp:11-36).  The library is loaded lazily on first use; if it is
missing, ``RuntimeUnavailable`` is raised -- there is no fallback path.
Status codes map onto the reference's exceptions: invalid arguments raise
``ValidationError``, a missing or unsupported device ``RuntimeUnavailable``,
and CUDA failures ``RuntimeError`` carrying the CUDA error name and text
(as runtime/Driver.cpp:85-95 did).
"""
from __future__ import annotations

import ctypes
from pathlib import Path
import threading

from .errors import RuntimeUnavailable, ValidationError

LIBRARY = Path(__file__).resolve().parent / "_lib" / "libragged_b200.so"

RG_OK, RG_ERR_INVALID_ARGUMENT, RG_ERR_UNSUPPORTED, RG_ERR_WORKSPACE, RG_ERR_CUDA, RG_ERR_DEVICE = range(6)
OPS = {"sum": 0, "max": 1, "softmax": 2}
DTYPES = {"f32": 0, "bf16": 1}
INDEX = {"i32": 0, "i64": 1}
SCHEDULES = {"classified": 0, "naive": 1, "rowbalanced": 2}
SCHEDULE_NAMES = {value: key for key, value in SCHEDULES.items()}
FLAG_NO_VECTORIZE = 1
FLAG_IN_PLACE = 2
FLAG_NO_POINTWISE_FUSION = 4
MAX_LAUNCHES = 8

# Every symbol include/ragged_b200.h declares.
EXPORTED = ("rg_version", "rg_error_string", "rg_last_error", "rg_get_device_info", "rg_workspace_bytes",
            "rg_run", "rg_kernel_name", "rg_check_offsets", "rg_pointwise_workspace_bytes", "rg_run_pointwise",
            "rg_shard_rows", "rg_shard_split", "rg_shard_edge_bytes", "rg_shard_workspace_bytes",
            "rg_shard_segments", "rg_shard_softmax_workspace_bytes", "rg_run_shard_softmax",
            "rg_shard_softmax_finish", "rg_run_shard", "rg_shard_combine", "rg_run_noalloc", "rg_tree_scores")


class Report(ctypes.Structure):
    _fields_ = [("schedule", ctypes.c_int32), ("num_launches", ctypes.c_int32),
                ("kernel_ids", ctypes.c_int32 * MAX_LAUNCHES), ("grid", (ctypes.c_int32 * 3) * MAX_LAUNCHES),
                ("block", ctypes.c_int32 * MAX_LAUNCHES), ("shared_bytes", ctypes.c_int32 * MAX_LAUNCHES),
                ("memsets", ctypes.c_int32), ("d_vector", ctypes.c_int32), ("d_tile", ctypes.c_int32),
                ("streams", ctypes.c_int32), ("workspace_bytes", ctypes.c_int64),
                ("thresholds", ctypes.c_int64 * 2), ("status_offset", ctypes.c_int64)]


class DeviceInfo(ctypes.Structure):
    _fields_ = [("device", ctypes.c_int32), ("sm_count", ctypes.c_int32), ("cc_major", ctypes.c_int32),
                ("cc_minor", ctypes.c_int32), ("l2_bytes", ctypes.c_int64),
                ("smem_per_block_optin", ctypes.c_int32), ("max_threads_per_sm", ctypes.c_int32)]


_lock = threading.Lock()
_lib = None


def library(path: Path | None = None):
    """The loaded library (raises RuntimeUnavailable when it is missing)."""
    global _lib
    with _lock:
        if _lib is not None:
            return _lib
        target = Path(path) if path is not None else LIBRARY
        if not target.exists():
            raise RuntimeUnavailable(f"native library {target} is missing; build it with "
                                     "`python ragged-mlir_b200/build.py` (no CPU fallback exists)")
        try:
            lib = ctypes.CDLL(str(target))
        except OSError as exc:
            raise RuntimeUnavailable(f"cannot load {target}: {exc}") from exc
        i32, i64, p, u32 = ctypes.c_int, ctypes.c_int64, ctypes.c_void_p, ctypes.c_uint32
        lib.rg_version.restype = ctypes.c_char_p
        lib.rg_error_string.restype = ctypes.c_char_p
        lib.rg_error_string.argtypes = [i32]
        lib.rg_last_error.restype = ctypes.c_char_p
        lib.rg_kernel_name.restype = ctypes.c_char_p
        lib.rg_kernel_name.argtypes = [i32]
        lib.rg_get_device_info.argtypes = [i32, ctypes.POINTER(DeviceInfo)]
        lib.rg_get_device_info.restype = i32
        lib.rg_workspace_bytes.argtypes = [i32, i32, i32, i64, i64, i64, i32, i64, u32, ctypes.POINTER(i64)]
        lib.rg_workspace_bytes.restype = i32
        lib.rg_run.argtypes = [i32, i32, i32, i64, i64, i64, p, p, p, p, i64, i32, i64, u32, p,
                               ctypes.POINTER(Report)]
        lib.rg_run.restype = i32
        lib.rg_check_offsets.argtypes = [i32, i64, i64, p, i64, i64, p, p, ctypes.POINTER(Report)]
        lib.rg_check_offsets.restype = i32
        lib.rg_pointwise_workspace_bytes.argtypes = [i32, i32, i32, i64, i64, i64, i32, i64, u32,
                                                     ctypes.POINTER(i64)]
        lib.rg_pointwise_workspace_bytes.restype = i32
        lib.rg_run_pointwise.argtypes = [i32, i32, i32, i64, i64, i64, p, p, p, ctypes.c_float, p, p, i64, i32, i64,
                                         u32, p, ctypes.POINTER(Report)]
        lib.rg_run_pointwise.restype = i32
        lib.rg_run_noalloc.argtypes = [i32, i32, i32, i64, i64, i64, p, p, p, u32, p]
        lib.rg_run_noalloc.restype = i32
        lib.rg_tree_scores.argtypes = [i64, p, p, p, p, p, p, i64, p, p, i32, p, i32, p, i32, p]
        lib.rg_tree_scores.restype = i32
        pi64 = ctypes.POINTER(i64)
        lib.rg_shard_rows.argtypes = [i64, i32, i32, pi64, pi64]
        lib.rg_shard_rows.restype = i32
        lib.rg_shard_edge_bytes.argtypes = [i32, i64, pi64]
        lib.rg_shard_edge_bytes.restype = i32
        lib.rg_shard_split.argtypes = [p, i32, i64, i32, ctypes.c_double, pi64]
        lib.rg_shard_split.restype = i32
        lib.rg_shard_workspace_bytes.argtypes = [i32, i32, i32, i64, i64, i64, i32, i32, pi64, u32, pi64]
        lib.rg_shard_workspace_bytes.restype = i32
        lib.rg_run_shard.argtypes = [i32, i32, i32, i64, i64, i64, i32, i32, pi64, p, p, p, p, p, i64, u32, p,
                                     ctypes.POINTER(Report)]
        lib.rg_run_shard.restype = i32
        lib.rg_shard_combine.argtypes = [i32, i32, i64, i32, i32, p, p, u32, p]
        lib.rg_shard_combine.restype = i32
        lib.rg_shard_segments.argtypes = [p, i32, i64, i32, i32, pi64, pi64, pi64]
        lib.rg_shard_segments.restype = i32
        lib.rg_shard_softmax_workspace_bytes.argtypes = [i32, i32, i64, i64, i64, i32, i32, pi64, i64, i64, u32, pi64]
        lib.rg_shard_softmax_workspace_bytes.restype = i32
        lib.rg_run_shard_softmax.argtypes = [i32, i32, i64, i64, i64, i32, i32, pi64, i64, i64, p, p, p, p, i64, u32,
                                             p, ctypes.POINTER(Report)]
        lib.rg_run_shard_softmax.restype = i32
        lib.rg_shard_softmax_finish.argtypes = [i32, i32, i64, i64, i64, i32, i32, pi64, i64, i64, p, p, p, p, p, i64,
                                                u32, p, ctypes.POINTER(Report)]
        lib.rg_shard_softmax_finish.restype = i32
        _lib = lib
        return lib


def raise_for(status: int, what: str) -> None:
    if status == RG_OK:
        return
    lib = library()
    detail = lib.rg_last_error().decode(errors="replace")
    message = f"{what}: {lib.rg_error_string(status).decode()}: {detail}"
    if status in (RG_ERR_INVALID_ARGUMENT, RG_ERR_WORKSPACE):
        raise ValidationError(message)
    if status in (RG_ERR_DEVICE, RG_ERR_UNSUPPORTED):
        raise RuntimeUnavailable(message)
    raise RuntimeError(message)


def version() -> str:
    return library().rg_version().decode()


_kernel_names: dict[int, str] = {}


def kernel_name(kernel_id: int) -> str:
    name = _kernel_names.get(kernel_id)
    if name is None:
        name = _kernel_names[kernel_id] = library().rg_kernel_name(kernel_id).decode()
    return name


_device_info: dict[int, DeviceInfo] = {}


def device_info(device: int) -> DeviceInfo:
    info = _device_info.get(device)
    if info is None:
        info = DeviceInfo()
        raise_for(library().rg_get_device_info(device, ctypes.byref(info)), "rg_get_device_info")
        _device_info[device] = info
    return info


def workspace_bytes(op: str, dtype: str, index: str, d: int, n: int, b: int, schedule: str,
                    max_len: int | None, flags: int = 0) -> int:
    out = ctypes.c_int64(0)
    raise_for(library().rg_workspace_bytes(OPS[op], DTYPES[dtype], INDEX[index], d, n, b, SCHEDULES[schedule],
                                           -1 if max_len is None else max_len, flags, ctypes.byref(out)),
              "rg_workspace_bytes")
    return int(out.value)


def run(op: str, dtype: str, index: str, d: int, n: int, b: int, values_ptr: int, offsets_ptr: int,
        out_ptr: int, workspace_ptr: int, workspace_bytes: int, schedule: str, max_len: int | None,
        flags: int, stream: int) -> Report:
    report = Report()
    status = library().rg_run(OPS[op], DTYPES[dtype], INDEX[index], d, n, b, values_ptr, offsets_ptr, out_ptr,
                              workspace_ptr or None, workspace_bytes, SCHEDULES[schedule],
                              -1 if max_len is None else max_len, flags, stream or None, ctypes.byref(report))
    raise_for(status, "rg_run")
    return report


def pointwise_workspace_bytes(op: str, dtype: str, index: str, d: int, n: int, b: int, schedule: str,
                              max_len: int | None, flags: int) -> int:
    """Scratch of a scale / mask call: the f32 logits, results and schedule."""
    out = ctypes.c_int64(0)
    raise_for(library().rg_pointwise_workspace_bytes(OPS[op], DTYPES[dtype], INDEX[index], d, n, b,
                                                     SCHEDULES[schedule], -1 if max_len is None else max_len, flags,
                                                     ctypes.byref(out)), "rg_pointwise_workspace_bytes")
    return out.value


def run_pointwise(op: str, dtype: str, index: str, d: int, n: int, b: int, values_ptr: int, offsets_ptr: int,
                  mask_ptr: int, scale: float, out_ptr: int, workspace_ptr: int, workspace_bytes: int, schedule: str,
                  max_len: int | None, flags: int, stream: int) -> Report:
    """One call with the input transform x * scale (+ mask for softmax)."""
    report = Report()
    status = library().rg_run_pointwise(OPS[op], DTYPES[dtype], INDEX[index], d, n, b, values_ptr, offsets_ptr,
                                        mask_ptr or None, float(scale), out_ptr, workspace_ptr or None,
                                        workspace_bytes, SCHEDULES[schedule], -1 if max_len is None else max_len,
                                        flags, stream or None, ctypes.byref(report))
    raise_for(status, "rg_run_pointwise")
    return report


# ------------------------------------------------------------ sharded calls

def shard_rows(n: int, world: int, rank: int) -> tuple[int, int]:
    """Rows [row0, row1) of ``rank`` in the row-balanced split of ``n`` rows."""
    row0, row1 = ctypes.c_int64(0), ctypes.c_int64(0)
    raise_for(library().rg_shard_rows(n, world, rank, ctypes.byref(row0), ctypes.byref(row1)), "rg_shard_rows")
    return int(row0.value), int(row1.value)


def shard_edge_bytes(op: str, d: int) -> int:
    out = ctypes.c_int64(0)
    raise_for(library().rg_shard_edge_bytes(OPS[op], d, ctypes.byref(out)), "rg_shard_edge_bytes")
    return int(out.value)


def _splits_arg(splits, world: int):
    """(pointer, owner) of a split's world + 1 row boundaries, or None.  The
    library reads exactly world + 1 entries, so a list of another length is
    refused here, before it could read past the array."""
    if splits is None:
        return None
    if len(splits) != world + 1:
        raise ValidationError(f"splits must hold world + 1 = {world + 1} row boundaries, not {len(splits)}")
    array = (ctypes.c_int64 * len(splits))(*[int(x) for x in splits])
    return ctypes.cast(array, ctypes.POINTER(ctypes.c_int64)), array


def shard_split(offsets_host, index: str, world: int, end_weight: float) -> list[int]:
    """Work-balanced split (world + 1 row boundaries) of host offsets."""
    import numpy as np
    offs = np.ascontiguousarray(offsets_host, dtype=np.int32 if index == "i32" else np.int64)
    out = (ctypes.c_int64 * (world + 1))()
    raise_for(library().rg_shard_split(offs.ctypes.data, INDEX[index], offs.size - 1, world, float(end_weight),
                                       ctypes.cast(out, ctypes.POINTER(ctypes.c_int64))), "rg_shard_split")
    return [int(x) for x in out]


def shard_workspace_bytes(op: str, dtype: str, index: str, d: int, n: int, b: int, world: int, rank: int,
                          flags: int = 0, splits=None) -> int:
    out = ctypes.c_int64(0)
    arg = _splits_arg(splits, world)
    raise_for(library().rg_shard_workspace_bytes(OPS[op], DTYPES[dtype], INDEX[index], d, n, b, world, rank,
                                                 arg[0] if arg else None, flags, ctypes.byref(out)),
              "rg_shard_workspace_bytes")
    return int(out.value)


def run_shard(op: str, dtype: str, index: str, d: int, n: int, b: int, world: int, rank: int, values_ptr: int,
              offsets_ptr: int, out_ptr: int, edges_ptr: int, workspace_ptr: int, workspace_bytes: int, flags: int,
              stream: int, splits=None) -> Report:
    report = Report()
    arg = _splits_arg(splits, world)
    status = library().rg_run_shard(OPS[op], DTYPES[dtype], INDEX[index], d, n, b, world, rank, arg[0] if arg else None,
                                    values_ptr or None, offsets_ptr, out_ptr, edges_ptr, workspace_ptr or None,
                                    workspace_bytes, flags, stream or None, ctypes.byref(report))
    raise_for(status, "rg_run_shard")
    return report


def shard_combine(op: str, dtype: str, d: int, world: int, rank: int, gathered_ptr: int, out_ptr: int, flags: int,
                  stream: int) -> None:
    raise_for(library().rg_shard_combine(OPS[op], DTYPES[dtype], d, world, rank, gathered_ptr, out_ptr, flags,
                                         stream or None), "rg_shard_combine")


def shard_segments(offsets_host, index: str, world: int, rank: int, splits=None) -> tuple[int, int]:
    """Segments [seg0, seg1) whose softmax statistics rank `rank` keeps."""
    import numpy as np
    offs = np.ascontiguousarray(offsets_host, dtype=np.int32 if index == "i32" else np.int64)
    seg0, seg1 = ctypes.c_int64(0), ctypes.c_int64(0)
    arg = _splits_arg(splits, world)
    raise_for(library().rg_shard_segments(offs.ctypes.data, INDEX[index], offs.size - 1, world, rank,
                                          arg[0] if arg else None, ctypes.byref(seg0), ctypes.byref(seg1)),
              "rg_shard_segments")
    return int(seg0.value), int(seg1.value)


def shard_softmax_workspace_bytes(dtype: str, index: str, d: int, n: int, b: int, world: int, rank: int,
                                  segments: tuple[int, int], flags: int = 0, splits=None) -> int:
    out = ctypes.c_int64(0)
    arg = _splits_arg(splits, world)
    raise_for(library().rg_shard_softmax_workspace_bytes(DTYPES[dtype], INDEX[index], d, n, b, world, rank,
                                                         arg[0] if arg else None, segments[0], segments[1], flags,
                                                         ctypes.byref(out)), "rg_shard_softmax_workspace_bytes")
    return int(out.value)


def run_shard_softmax(dtype: str, index: str, d: int, n: int, b: int, world: int, rank: int,
                      segments: tuple[int, int], values_ptr: int, offsets_ptr: int, edges_ptr: int, workspace_ptr: int,
                      workspace_bytes: int, flags: int, stream: int, splits=None) -> Report:
    report = Report()
    arg = _splits_arg(splits, world)
    raise_for(library().rg_run_shard_softmax(DTYPES[dtype], INDEX[index], d, n, b, world, rank,
                                             arg[0] if arg else None, segments[0], segments[1], values_ptr or None,
                                             offsets_ptr, edges_ptr, workspace_ptr or None, workspace_bytes, flags,
                                             stream or None, ctypes.byref(report)), "rg_run_shard_softmax")
    return report


def shard_softmax_finish(dtype: str, index: str, d: int, n: int, b: int, world: int, rank: int,
                         segments: tuple[int, int], values_ptr: int, offsets_ptr: int, gathered_ptr: int, out_ptr: int,
                         workspace_ptr: int, workspace_bytes: int, flags: int, stream: int, splits=None) -> Report:
    report = Report()
    arg = _splits_arg(splits, world)
    raise_for(library().rg_shard_softmax_finish(DTYPES[dtype], INDEX[index], d, n, b, world, rank,
                                                arg[0] if arg else None, segments[0], segments[1],
                                                values_ptr or None, offsets_ptr, gathered_ptr, out_ptr or None,
                                                workspace_ptr or None, workspace_bytes, flags, stream or None,
                                                ctypes.byref(report)), "rg_shard_softmax_finish")
    return report


def check_offsets(index: str, n: int, b: int, offsets_ptr: int, min_len: int | None, max_len: int | None,
                  status_ptr: int, stream: int) -> Report:
    """Launch the checked-mode offsets validation (status: 7 int64 on the device)."""
    report = Report()
    raise_for(library().rg_check_offsets(INDEX[index], n, b, offsets_ptr, -1 if min_len is None else min_len,
                                         -1 if max_len is None else max_len, status_ptr, stream or None,
                                         ctypes.byref(report)), "rg_check_offsets")
    return report


def tree_scores(arrays: dict, x, classes: int, max_depth: int):
    """Scores of the schedule chooser's trees (rg_tree_scores); ``arrays``
    holds contiguous int32 feature/left/right/roots/tree_class, float64
    threshold/value/baseline and uint8 leaf node arrays (kept alive by the
    caller; their addresses are cached in it under "_args")."""
    import numpy as np
    lib = library()
    args = arrays.get("_args")
    if args is None:
        a = arrays
        args = arrays["_args"] = (a["feature"].size, a["feature"].ctypes.data, a["threshold"].ctypes.data,
                                  a["left"].ctypes.data, a["right"].ctypes.data, a["value"].ctypes.data,
                                  a["leaf"].ctypes.data, a["roots"].size, a["roots"].ctypes.data,
                                  a["tree_class"].ctypes.data, classes, a["baseline"].ctypes.data)
    x = np.ascontiguousarray(x, dtype=np.float64)
    scores = np.empty(classes, dtype=np.float64)
    status = lib.rg_tree_scores(*args, x.size, x.ctypes.data, max_depth, scores.ctypes.data)
    raise_for(status, "rg_tree_scores")
    return scores
