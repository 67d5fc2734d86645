"""``CompiledProgram.run``: validate, choose a schedule, launch on a stream.

Mirrors the reference's python/ragged/runtime.py (CompiledProgram 218-558):
the same signature ``run(values, offsets, out, stream=None,
mode="validated", *, debug_buffers=None, mask=None, concurrent=True,
select="auto", max_len=None) -> ExecutionReport``, the same tensor checks
and error classes (runtime.py:304-365), scratch allocated from PyTorch's
caching allocator on the execution stream (runtime.py:534-545), no device
readback and no synchronisation.  Below it there is no module loading or
launch-plan machinery: one call into libragged_b200.so (``rg_run``) chooses
grids, relocates scratch and launches the sm_100a kernels on the stream.
"""
from __future__ import annotations

from contextlib import nullcontext
from dataclasses import replace
import importlib
import threading
import time
from typing import Any

from . import _native
from .cache import Artifact
from .errors import CacheMismatch, RuntimeUnavailable, ValidationError
from .model import ExecutionReport, ProgramSpec, runs_on
from .selection import default_model
from .validation import CONDITIONS, STATUS_BYTES, raise_for_status

I64_MAX = 2**63 - 1
# Segment-length class bounds of the classified schedule (warp <= 32 rows,
# CTA <= 4096 rows, longer ones split), as in the reference's Passes.cpp:17-18.
# A call reports the bounds it used: the CTA bound shrinks to 64 KiB of one
# column tile for wide rows.
THRESHOLDS = (32, 4096)

_lock = threading.RLock()
_checked_devices: set[int] = set()
_device_l2_mib: dict[int, float | None] = {}


def _torch():
    try:
        return importlib.import_module("torch")
    except ImportError as exc:
        raise RuntimeUnavailable("PyTorch is not installed; install the GPU environment to execute") from exc


def device_l2_mib(values) -> float | None:
    """L2 capacity (MiB) of the CUDA device holding ``values``, cached."""
    device = getattr(values, "device", None)
    if getattr(device, "type", None) != "cuda":
        return None
    index = device.index if device.index is not None else 0
    if index not in _device_l2_mib:
        try:
            l2 = _native.device_info(index).l2_bytes
        except Exception:  # noqa: BLE001 - no library/device: the model's own L2 is used
            l2 = 0
        _device_l2_mib[index] = l2 / 2**20 if l2 > 0 else None
    return _device_l2_mib[index]


def _overlaps(left: Any, right: Any) -> bool:
    lstart, rstart = left.data_ptr(), right.data_ptr()
    lend = lstart + left.numel() * left.element_size()
    rend = rstart + right.numel() * right.element_size()
    return lstart < rend and rstart < lend


def _check_gathered(gathered, edges, world: int, torch):
    """The all-gather result a sharded call hands to the combine kernel:
    every rank's edge record, f32, contiguous, on this rank's device."""
    if not isinstance(gathered, torch.Tensor) or gathered.device != edges.device:
        raise ValidationError("exchange must return every rank's edge record on this device")
    if gathered.dtype != torch.float32 or not gathered.is_contiguous():
        raise ValidationError("exchange must return a contiguous f32 tensor (the records as sent)")
    if gathered.numel() != world * edges.numel():
        raise ValidationError("exchange must return every rank's edge record on this device")
    return gathered


class CompiledProgram:
    def __init__(self, spec: ProgramSpec, artifact: Artifact, *, cache_hit: bool = False,
                 naive: "CompiledProgram | None" = None):
        if not isinstance(spec, ProgramSpec):
            raise ValidationError("spec must be a ProgramSpec")
        if artifact.key.ir_hash != spec.ir_hash:
            raise CacheMismatch("artifact was recorded for a different specialization")
        self.spec, self.artifact, self.cache_hit = spec, artifact, cache_hit
        self._schedules = tuple(artifact.metadata.get("schedules", ("naive",)))
        self._digest = artifact.key.digest
        self._selects = spec.strategy == "auto" and "naive" not in self._schedules
        if naive is not None and (not self._selects or naive.spec != replace(spec, strategy="naive")):
            raise CacheMismatch("a block-per-segment companion must be the naive strategy of a classifying program")
        self.naive = naive
        self._choices: dict[tuple, tuple[str, dict[str, Any]]] = {}
        self._workspace: dict[tuple, int] = {}
        tile, vec = spec.optimizations.geometry(spec.feature_dim, spec.dtype)
        self._span = tile * vec
        self._vector = vec
        self._dtypes = None  # torch dtypes, resolved on the first call
        # The report's optimisation section, fixed per program (built once).
        self._optimization_report = {"requested": spec.optimizations.to_dict(),
                                     **spec.optimizations.effects(transformed=spec.mask or float(spec.scale) != 1.0)}
        self._flags = (0 if spec.optimizations.vectorize else _native.FLAG_NO_VECTORIZE) | (
            _native.FLAG_IN_PLACE if spec.alias == "inplace" else 0)
        # Scale or mask: rg_run_pointwise (fused into the classified worker's
        # loads for staged softmax rows, else materialised; pointwise_fusion=False
        # always materialises, the reference's route).
        self._pointwise = spec.mask or float(spec.scale) != 1.0
        if self._pointwise and not spec.optimizations.pointwise_fusion:
            self._flags |= _native.FLAG_NO_POINTWISE_FUSION

    @property
    def selects(self) -> bool:
        """Whether this program chooses among schedules per call."""
        return self._selects

    @property
    def schedules(self) -> tuple[str, ...]:
        return self._schedules + (("naive",) if self.naive is not None else ())

    def choose(self, n: int, b: int, max_len: int | None, l2_mib: float | None = None) -> tuple[str, dict[str, Any]]:
        """The schedule ``run(select="auto")`` uses and why."""
        if not self._selects:
            return self._schedules[0], {}
        key = (n, b, max_len, l2_mib)
        choice = self._choices.get(key)
        if choice is None:
            if len(self._choices) >= 256:
                self._choices.clear()
            element = 2 if self.spec.dtype == "bf16" else 4
            choice = self._choices[key] = default_model().choose(
                self.spec.op, n, b, self.spec.feature_dim, max_len, self._span, element, l2_mib=l2_mib,
                available=self.schedules)
        return choice

    def close(self) -> None:
        """Nothing to unload: kernels live in the shared library."""

    def _torch_dtypes(self, torch):
        """(values dtype, offsets dtype) of this specialization, resolved once."""
        if self._dtypes is None:
            self._dtypes = ({"f32": torch.float32, "bf16": torch.bfloat16}[self.spec.dtype],
                            {"i32": torch.int32, "i64": torch.int64}[self.spec.offsets_dtype])
        return self._dtypes

    def _validate_tensors(self, values, offsets, out, torch, checked: bool = False, mask=None) -> tuple[int, int]:
        """The reference's tensor checks and messages (its runtime.py:304-365);
        each tensor's extent is read once."""
        tensor_type = torch.Tensor
        for name, tensor in (("values", values), ("offsets", offsets), ("out", out), ("mask", mask)):
            if tensor is None and name == "mask":
                continue
            if not isinstance(tensor, tensor_type):
                raise ValidationError(f"{name} must be a torch.Tensor")
            if not tensor.is_cuda:
                raise RuntimeUnavailable(f"{name} must be on a CUDA device that runs {self.spec.chip} code; "
                                         "no CPU execution fallback exists")
            if not tensor.is_contiguous():
                raise ValidationError(f"{name} must be row-major contiguous")
            if tensor.requires_grad:
                raise ValidationError("autograd is outside the supported forward-only contract")
        device = values.device
        if device != offsets.device or device != out.device:
            raise ValidationError("values, offsets and out must use the same CUDA device")
        shape = values.shape
        if values.ndim != 2 or shape[1] != self.spec.feature_dim:
            raise ValidationError("values must have shape [N, static D]")
        count = offsets.numel()
        if offsets.ndim != 1 or count < 1:
            raise ValidationError("offsets must have shape [B+1], including [0] when B=0")
        dtype, offset_dtype = self._torch_dtypes(torch)
        if values.dtype != dtype or out.dtype != dtype or offsets.dtype != offset_dtype:
            raise ValidationError("tensor dtype differs from compiled dtype/offsets specialization")
        n, b = shape[0], count - 1
        d = shape[1]
        element = values.element_size()
        vptr, optr, fptr = values.data_ptr(), out.data_ptr(), offsets.data_ptr()
        vbytes, obytes, fbytes = n * d * element, out.numel() * element, count * offsets.element_size()
        if self._vector > 1:
            need = self._vector * element
            for name, pointer, size in (("values", vptr, vbytes), ("out", optr, obytes)):
                if size and pointer % need:
                    raise ValidationError(f"{name} must be {need}-byte aligned: this specialization accesses "
                                          f"{self._vector} features at a time (compile with vectorize=False for "
                                          "unaligned views)")
        if b == 0 and n != 0 and not checked:  # checked mode reports it from the device (final_mismatch)
            raise ValidationError("B=0 requires N=0; values cannot exist without segments")
        if self.spec.offsets_dtype == "i32" and n > 2**31 - 1:
            raise ValidationError("N exceeds the i32 offsets range")
        expected = (n if self.spec.op == "softmax" else b, d)
        if tuple(out.shape) != expected:
            raise ValidationError(f"out shape must be {expected}")

        def overlap(p1, s1, p2, s2):
            return p1 < p2 + s2 and p2 < p1 + s1

        if mask is not None:  # reference runtime.py:346-356; the mask may alias values (read only)
            if mask.dtype != torch.float32 or tuple(mask.shape) != tuple(shape):
                raise ValidationError("mask must have f32 dtype and exactly values shape [N,D]; "
                                      "broadcasting is unsupported")
            if mask.device != device:
                raise ValidationError("mask must use the values CUDA device")
            mptr, mbytes = mask.data_ptr(), n * d * 4
            if mbytes and mptr % 4:
                raise ValidationError("mask must be 4-byte aligned")
            if overlap(mptr, mbytes, optr, obytes) or overlap(mptr, mbytes, fptr, fbytes):
                raise ValidationError("mask must not overlap out or offsets")
        if overlap(fptr, fbytes, vptr, vbytes) or overlap(fptr, fbytes, optr, obytes):
            raise ValidationError("offsets must not alias values or out")
        # In place (runtime.py:358-364 of the reference): out must BE values.
        exact = vptr == optr and tuple(shape) == tuple(out.shape)
        if overlap(vptr, vbytes, optr, obytes):
            if not exact or self.spec.alias != "inplace":
                raise ValidationError("out aliases values without a compiler-proven safe in-place schedule")
        elif self.spec.alias == "inplace" and not (exact and vbytes == 0):
            raise ValidationError("in-place specialization requires out and values to be the same buffer")
        return n, b

    def workspace_bytes(self, n: int, b: int, schedule: str, max_len: int | None = None) -> int:
        key = (n, b, schedule, max_len)
        nbytes = self._workspace.get(key)
        if nbytes is None:
            if len(self._workspace) >= 256:
                self._workspace.clear()
            size = _native.pointwise_workspace_bytes if self._pointwise else _native.workspace_bytes
            nbytes = self._workspace[key] = size(
                self.spec.op, self.spec.dtype, self.spec.offsets_dtype, self.spec.feature_dim, n, b, schedule, max_len,
                self._flags)
        return nbytes

    def run(self, values, offsets, out, stream=None, mode: str = "validated", *,
            debug_buffers: dict[str, Any] | None = None, mask=None, concurrent: bool = True,
            select: str = "auto", max_len: int | None = None) -> ExecutionReport:
        """Launch on ``stream`` (default: the current stream of the values'
        device).  Validated mode reads nothing back and never synchronises.
        ``select`` is "auto" (cost model; ``max_len`` is the caller's bound on
        the longest segment, a wrong value costs time, never correctness), or
        forces "classified", "naive" or "rowbalanced"."""
        if select not in ("auto", "classified", "naive", "rowbalanced"):
            raise ValidationError("select must be auto, classified, naive or rowbalanced")
        if max_len is not None and (type(max_len) is not int or max_len < 0):
            raise ValidationError("max_len must be None or a nonnegative int")
        if mode not in ("validated", "checked"):
            raise ValidationError("mode must be validated or checked")
        if (mask is not None) != self.spec.mask:
            raise ValidationError("mask presence must match the compiled specialization")
        if debug_buffers is not None:
            raise ValidationError("debug_buffers requires an empty dict and a debug_visits specialization")
        if select != "auto" and select not in self.schedules:
            raise ValidationError(f"select={select} is not a schedule of this program ({', '.join(self.schedules)})")
        torch = _torch()
        checked = mode == "checked"
        n, b = self._validate_tensors(values, offsets, out, torch, checked, mask)
        started = time.perf_counter()
        if select == "auto":
            schedule, selection = self.choose(n, b, max_len, device_l2_mib(values))
        else:
            schedule, selection = select, {"forced": True}
        if b == 0 and not checked:
            return self._report(schedule, selection, started, None, 0)
        with torch.cuda.device(values.device):
            ordinal = values.device.index
            if ordinal not in _checked_devices:
                capability = tuple(torch.cuda.get_device_capability(values.device))
                if not runs_on(self.spec.chip, capability):
                    raise RuntimeUnavailable(f"compiled target {self.spec.chip} does not run on the current device "
                                             f"(sm_{capability[0]}{capability[1]})")
                _checked_devices.add(ordinal)
            active = stream if stream is not None else torch.cuda.current_stream(values.device)
            if not isinstance(active, torch.cuda.Stream) or active.device != values.device:
                raise ValidationError("stream must be a torch.cuda.Stream on the values device")
            validation = self._check_offsets(values, offsets, n, b, active, torch) if checked else None
            if b == 0:
                return self._report(schedule, selection, started, None, 0, validation)
            nbytes = self.workspace_bytes(n, b, schedule, max_len)
            scratch, base = None, 0
            if nbytes:
                # Scratch comes from the caching allocator ON the execution
                # stream, so reuse is ordered after this call's kernels.
                with torch.cuda.stream(active) if stream is not None else nullcontext():
                    scratch = torch.empty((nbytes,), dtype=torch.uint8, device=values.device)
                base = scratch.data_ptr()
            if stream is not None:
                for tensor in (values, offsets, out) + ((mask,) if mask is not None else ()):
                    tensor.record_stream(active)
            if self._pointwise:
                report = _native.run_pointwise(
                    self.spec.op, self.spec.dtype, self.spec.offsets_dtype, self.spec.feature_dim, n, b,
                    values.data_ptr(), offsets.data_ptr(), mask.data_ptr() if mask is not None else 0,
                    float(self.spec.scale), out.data_ptr(), base, nbytes, schedule, max_len, self._flags,
                    active.cuda_stream)
            else:
                report = _native.run(self.spec.op, self.spec.dtype, self.spec.offsets_dtype, self.spec.feature_dim,
                                     n, b, values.data_ptr(), offsets.data_ptr(), out.data_ptr(), base, nbytes,
                                     schedule, max_len, self._flags, active.cuda_stream)
            if checked and scratch is not None and getattr(report, "status_offset", -1) >= 0:
                self._check_device_status(scratch, int(report.status_offset), active, torch)
        return self._report(schedule, selection, started, report, nbytes, validation)

    @staticmethod
    def _check_device_status(scratch, offset, active, torch):
        """Checked mode, after the launch: read the call's device status word
        (rg_report.status_offset into the scratch) and raise when a bounded
        wait inside a kernel gave up, since the results are then undefined.
        Validated mode never reads it (no synchronisation)."""
        with torch.cuda.stream(active):
            host = torch.empty((1,), dtype=torch.int64, device="cpu", pin_memory=True)
            host.copy_(scratch.narrow(0, offset, 8).view(torch.int64), non_blocking=True)
        active.synchronize()
        word = int(host.tolist()[0])
        if word:
            raise RuntimeError(f"a bounded wait inside the kernel gave up (device status {word}); the call's results "
                               "are undefined")

    def _check_offsets(self, values, offsets, n, b, active, torch):
        """Checked mode (reference python/ragged/runtime.py:506-533): validate
        the offsets on the device, on the execution stream, before any main
        kernel or scratch allocation; copy the 56-byte status to pinned host
        memory, wait on that stream only and raise ValidationError on failure.
        The length bounds are the spec's hints (None: unchecked)."""
        started = time.perf_counter()
        with torch.cuda.stream(active):
            status = torch.empty((len(CONDITIONS),), dtype=torch.int64, device=values.device)
            host = torch.empty((len(CONDITIONS),), dtype=torch.int64, device="cpu", pin_memory=True)
            for tensor in (values, offsets, status):
                tensor.record_stream(active)
            report = _native.check_offsets(self.spec.offsets_dtype, n, b, offsets.data_ptr(), self.spec.hints.min_len,
                                           self.spec.hints.max_len, status.data_ptr(), active.cuda_stream)
            host.copy_(status, non_blocking=True)
        active.synchronize()
        raise_for_status(host.tolist(), b=b)
        return report, (time.perf_counter() - started) * 1000

    def run_sharded(self, values, offsets, out, *, total_rows: int, world: int, rank: int, exchange,
                    stream=None, splits=None, offsets_host=None) -> ExecutionReport:
        """One rank's part of a row-sharded call (``ragged.sharding``).

        ``values`` holds this rank's rows ``sharding.shard_rows(total_rows,
        world, rank, splits)`` of a call over ``total_rows`` rows (``splits``:
        world + 1 row boundaries, e.g. ``sharding.balanced_split``; None: the
        even row split), ``offsets`` all B+1 entries.  Sum and max: ``out``
        holds all B output rows (only the rows this rank finishes are
        written: ``sharding.segment_owners``).  Softmax: ``out`` holds this
        rank's rows, and ``offsets_host`` (the offsets in host memory) gives
        the segments whose statistics the rank keeps.  ``exchange(edges)``
        must return the edge records of ranks 0..world-1 concatenated (an
        all-gather); it is the only communication.  Launches on ``stream``
        (default: current), no host synchronisation of its own."""
        if self.spec.op == "softmax":
            return self._run_sharded_softmax(values, offsets, out, total_rows, world, rank, exchange, stream, splits,
                                             offsets_host)
        if self._pointwise:
            raise RuntimeUnavailable("sharded calls take no scale (the input transform is single-GPU only)")
        torch = _torch()
        if not 0 <= rank < world:
            raise ValidationError("need 0 <= rank < world")
        from .sharding import shard_rows
        row0, row1 = shard_rows(total_rows, world, rank, splits)
        d = self.spec.feature_dim
        b = self._validate_shard_tensors(values, offsets, out, torch)
        if tuple(values.shape) != (row1 - row0, d):
            raise ValidationError(f"values must hold this rank's {row1 - row0} rows: shape ({row1 - row0}, {d})")
        if tuple(out.shape) != (b, d):
            raise ValidationError(f"out shape must be ({b}, {d})")
        started = time.perf_counter()
        with torch.cuda.device(values.device):
            active = stream if stream is not None else torch.cuda.current_stream(values.device)
            spec = self.spec
            nbytes = _native.shard_workspace_bytes(spec.op, spec.dtype, spec.offsets_dtype, d, total_rows, b, world,
                                                   rank, self._flags, splits)
            with torch.cuda.stream(active):
                scratch = torch.empty((max(nbytes, 1),), dtype=torch.uint8, device=values.device)
                edges = torch.empty((_native.shard_edge_bytes(spec.op, d) // 4,), dtype=torch.float32,
                                    device=values.device)
                report = _native.run_shard(spec.op, spec.dtype, spec.offsets_dtype, d, total_rows, b, world, rank,
                                           values.data_ptr() if values.numel() else 0, offsets.data_ptr(),
                                           out.data_ptr(), edges.data_ptr(), scratch.data_ptr(), nbytes, self._flags,
                                           active.cuda_stream, splits)
                gathered = _check_gathered(exchange(edges), edges, world, torch)
                _native.shard_combine(spec.op, spec.dtype, d, world, rank, gathered.data_ptr(), out.data_ptr(),
                                      self._flags, active.cuda_stream)
        result = self._report("rowbalanced", {"sharded": {"world": world, "rank": rank, "rows": [row0, row1]}},
                              started, report, nbytes)
        return result

    def _run_sharded_softmax(self, values, offsets, out, total_rows, world, rank, exchange, stream, splits,
                             offsets_host):
        """Softmax of a row-sharded call: statistics of the rank's window and
        its edge record, the all-gather, then the merged statistics of the
        cut segments and the window's rows normalised into ``out``."""
        if self._pointwise:
            raise RuntimeUnavailable("sharded calls take no scale or mask (the input transform is single-GPU only)")
        if offsets_host is None:
            raise ValidationError("sharded softmax needs offsets_host (the offsets in host memory)")
        torch = _torch()
        if not 0 <= rank < world:
            raise ValidationError("need 0 <= rank < world")
        from .sharding import shard_rows
        row0, row1 = shard_rows(total_rows, world, rank, splits)
        d = self.spec.feature_dim
        b = self._validate_shard_tensors(values, offsets, out, torch)
        rows = (row1 - row0, d)
        if tuple(values.shape) != rows or tuple(out.shape) != rows:
            raise ValidationError(f"values and out must hold this rank's {row1 - row0} rows: shape {rows}")
        if len(offsets_host) != b + 1:
            raise ValidationError("offsets_host must hold the same B+1 offsets")
        spec = self.spec
        segments = _native.shard_segments(offsets_host, spec.offsets_dtype, world, rank, splits)
        started = time.perf_counter()
        with torch.cuda.device(values.device):
            active = stream if stream is not None else torch.cuda.current_stream(values.device)
            nbytes = _native.shard_softmax_workspace_bytes(spec.dtype, spec.offsets_dtype, d, total_rows, b, world,
                                                           rank, segments, self._flags, splits)
            with torch.cuda.stream(active):
                scratch = torch.empty((max(nbytes, 1),), dtype=torch.uint8, device=values.device)
                edges = torch.empty((_native.shard_edge_bytes("softmax", d) // 4,), dtype=torch.float32,
                                    device=values.device)
                ptr = values.data_ptr() if values.numel() else 0
                first = _native.run_shard_softmax(spec.dtype, spec.offsets_dtype, d, total_rows, b, world, rank,
                                                  segments, ptr, offsets.data_ptr(), edges.data_ptr(),
                                                  scratch.data_ptr(), nbytes, self._flags, active.cuda_stream, splits)
                gathered = _check_gathered(exchange(edges), edges, world, torch)
                report = _native.shard_softmax_finish(spec.dtype, spec.offsets_dtype, d, total_rows, b, world, rank,
                                                      segments, ptr, offsets.data_ptr(), gathered.data_ptr(),
                                                      out.data_ptr() if out.numel() else 0, scratch.data_ptr(),
                                                      nbytes, self._flags, active.cuda_stream, splits)
        names = tuple(_native.kernel_name(first.kernel_ids[i]) for i in range(first.num_launches))
        result = self._report("rowbalanced", {"sharded": {"world": world, "rank": rank, "rows": [row0, row1],
                                                          "segments": list(segments)}}, started, report, nbytes)
        return replace(result, kernel_names=names + result.kernel_names)

    def _validate_shard_tensors(self, values, offsets, out, torch) -> int:
        """Tensor checks shared by both sharded paths (the single-GPU rules
        of ``_validate_tensors`` that do not depend on the rank's window);
        returns B.  Pointer alignment and overlap are checked by the C ABI."""
        for name, tensor in (("values", values), ("offsets", offsets), ("out", out)):
            if not isinstance(tensor, torch.Tensor) or not tensor.is_cuda:
                raise RuntimeUnavailable(f"{name} must be a CUDA tensor; no CPU execution fallback exists")
            if not tensor.is_contiguous():
                raise ValidationError(f"{name} must be row-major contiguous")
            if tensor.requires_grad:
                raise ValidationError("autograd is outside the supported forward-only contract")
        if values.device != offsets.device or values.device != out.device:
            raise ValidationError("values, offsets and out must use the same CUDA device")
        if offsets.ndim != 1 or offsets.numel() < 1:
            raise ValidationError("offsets must have shape [B+1], including [0] when B=0")
        dtype = {"f32": torch.float32, "bf16": torch.bfloat16}[self.spec.dtype]
        offset_dtype = {"i32": torch.int32, "i64": torch.int64}[self.spec.offsets_dtype]
        if values.dtype != dtype or out.dtype != dtype or offsets.dtype != offset_dtype:
            raise ValidationError("tensor dtype differs from compiled dtype/offsets specialization")
        return offsets.numel() - 1

    def _report(self, schedule, selection, started, report, nbytes, validation=None) -> ExecutionReport:
        validation, validation_ms = validation if validation is not None else (None, None)
        thresholds = THRESHOLDS if schedule == "classified" else ()
        names, grids, vec, tile, streams = (), (), 1, None, 1
        for part in (validation, report):
            if part is None:
                continue
            count = part.num_launches
            names += tuple(_native.kernel_name(part.kernel_ids[i]) for i in range(count))
            grids += tuple(tuple(int(x) for x in part.grid[i]) for i in range(count))
        if report is not None:
            vec, tile, streams = int(report.d_vector), int(report.d_tile), int(report.streams)
            if schedule == "classified" and report.thresholds[1] > 0:
                thresholds = (int(report.thresholds[0]), int(report.thresholds[1]))
        classes = ("cta",) if schedule == "naive" else (("warp", "cta", "split") if schedule == "classified"
                                                        else ("rows",))
        if report is None:
            classes = ()
        checked_bytes = STATUS_BYTES if validation is not None else 0
        return ExecutionReport(classes, thresholds, grids, nbytes + checked_bytes, self._digest, None,
                               "checked" if validation is not None else "validated", names,
                               (time.perf_counter() - started) * 1000, cache_hit=self.cache_hit,
                               validation_workspace_bytes=checked_bytes,
                               validation_host_ms=validation_ms if validation is not None else None,
                               optimizations=dict(self._optimization_report),
                               pointwise_materialized=self._pointwise and "pointwise_logits" in names,
                               d_tile=tile, d_vector=vec, streams=streams, selected=schedule, selection=selection)
