"""Benchmark: segmented reduction throughput on B200 (one JSON line).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
                    [--workload c5] [--schedule auto] [--no-e2e] [--no-configs]

A step is one pass of the hot path over one batch: one segmented reduction
of the whole workload (default ``c5``: bf16 sum, D=256, N=200M rows, B=4M
Zipf segments -- the configuration the metric is quoted on at 1/2/4/8
GPUs).  With N GPUs (torchrun, one process per GPU) the rows are split
across ranks by work (strong scaling: the total work is fixed), each rank
reduces its rows, and the partial sums of segments cut by shard boundaries
are combined over NVLink (NCCL all-gather + a deterministic combine kernel).

Before anything is timed, the first call's output is checked against the
float64 C oracle (``"parity": "ok"`` in the line; a mismatch exits
non-zero): at N=1 the leading segments, the three 50M-row segments and the
last segments; at N>1 the same segments, each rank reducing its own rows of
them in the oracle and rank 0 merging the pieces in rank order and
comparing the rows their owners wrote.

value          = algorithmic bytes of the whole job / max-over-ranks device
                 time per step (GB/s), inputs resident in HBM;
e2e            = the same metric through the public API with the inputs in
                 pinned host memory: H2D copy, the call, D2H of the result,
                 every step inside the timed region;
roofline       = the call's achieved bandwidth per GPU vs the measured copy
                 bandwidth in MEASURED_PEAKS.json;
configs        = (N=1) c1-c4 of the configuration list, each checked against
                 the oracle at full size and timed the same way;
cpu_baseline   = the reference's CPU path on the host's cores (all of its
                 CPU affinity): torch.segment_reduce (softmax: the CPU torch
                 composition) and the float64 C oracle on a bounded sample
                 of the same workload (rank 0, N=1 only); the faster is the
                 line's value.

``--impl reference`` times that CPU path (the reference's GPU path cannot
run on sm_100) and prints its line with "impl": "reference".
"""
from __future__ import annotations

import argparse
import json
import os
from pathlib import Path
import statistics
import subprocess
import sys
import time

import numpy as np

REPO = Path(__file__).resolve().parent
sys.path.insert(0, str(REPO / "ragged-mlir_b200"))

from ragged import workloads  # noqa: E402

PEAKS_FILE = REPO / "MEASURED_PEAKS.json"

# DRAM traffic (ncu dram__bytes_read.sum + dram__bytes_write.sum) over the
# algorithmic bytes of the dominant kernel, from a capture of a smaller case
# of the same workload (traffic grows in proportion to the rows): see
# profiles/rowbal_kernel_c5.md.
TRAFFIC_RATIO = {"c5": 1.003}
FALLBACK_HBM_GBS = 6650.0
SIDE_CONFIGS = ("c1", "c2_sum", "c2_max", "c3", "c4_sum", "c4_max")


def parse_args(argv=None):
    parser = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    parser.add_argument("--gpus", type=int, default=1)
    parser.add_argument("--steps", type=int, default=10)
    parser.add_argument("--warmup", type=int, default=3)
    parser.add_argument("--impl", choices=("ours", "reference"), default="ours")
    parser.add_argument("--workload", choices=workloads.CONFIGS, default="c5")
    parser.add_argument("--schedule", default="auto")
    parser.add_argument("--scale", type=float, default=1.0, help="shrink B and N (testing only)")
    parser.add_argument("--no-e2e", action="store_true")
    parser.add_argument("--no-cpu-baseline", action="store_true")
    parser.add_argument("--no-configs", action="store_true", help="skip the c1-c4 entries (N=1)")
    parser.add_argument("--no-parity", action="store_true", help="skip the oracle check of the first call")
    parser.add_argument("--split-fit", action="store_true",
                        help="refit the split's end weight from measured per-rank times before timing (N > 1)")
    parser.add_argument("--cpu-bytes", type=float, default=2e9,
                        help="algorithmic bytes of the CPU sample (one call of each CPU implementation)")
    return parser.parse_args(argv)


def peak_hbm() -> tuple[float, str]:
    try:
        data = json.loads(PEAKS_FILE.read_text())
        return float(data["hbm_gbs"]), "measured"
    except (OSError, ValueError, KeyError):
        return FALLBACK_HBM_GBS, "fallback"


def host_threads() -> int:
    """Host threads this process may use: its CPU affinity (torchrun sets
    OMP_NUM_THREADS=1, which must not shrink the CPU baseline)."""
    try:
        return max(1, len(os.sched_getaffinity(0)))
    except (AttributeError, OSError):
        return max(1, os.cpu_count() or 1)


def metric_name() -> str:
    return "effective HBM GB/s of segmented reduction (algorithmic bytes / device time per call)"


def config_dict(w, args, flush) -> dict:
    return {"workload": w.name, "op": w.op, "values_dtype": w.dtype, "accumulate": "f32", "D": w.d, "N": w.n,
            "B": w.b, "offsets": w.index, "schedule": args.schedule, "algorithmic_bytes": w.algorithmic_bytes(),
            "parallelism": f"row-sharded x{args.gpus}", "l2": flush, **({"lengths_rule": w.notes["lengths_rule"]}
                                                                      if "lengths_rule" in w.notes else {})}


# --------------------------------------------------------------- clocks ----

class ClockSampler:
    """nvidia-smi samples during the timed region."""

    QUERY = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
             "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
             "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, device: int):
        self.device = device
        self.proc = None
        self.lines = []

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(["nvidia-smi", "-i", str(self.device), f"--query-gpu={self.QUERY}",
                                          "--format=csv,noheader,nounits", "-lms", "100"],
                                         stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except OSError:
            self.proc = None
        time.sleep(0.25)
        return self

    def __exit__(self, *exc):
        self.lines = []
        if self.proc is not None:
            time.sleep(0.15)
            self.proc.terminate()
            try:
                out, _ = self.proc.communicate(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()
                out, _ = self.proc.communicate()
            self.lines = [line for line in out.splitlines() if line.strip()]

    def summary(self) -> dict:
        sm, sm_max, reasons, power = [], 0.0, set(), []
        names = ("hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap")
        for line in self.lines:
            parts = [p.strip() for p in line.split(",")]
            if len(parts) < 9:
                continue
            try:
                sm.append(float(parts[1]))
                sm_max = max(sm_max, float(parts[2]))
                power.append(float(parts[3]))
            except ValueError:
                continue
            for name, flag in zip(names, parts[5:9]):
                if flag.lower() == "active":
                    reasons.add(name)
        if not sm:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": [], "samples": 0}
        loaded = [s for s, p in zip(sm, power) if p > 250] or sm
        return {"sm_mhz": statistics.median(loaded), "sm_max_mhz": sm_max, "reasons": sorted(reasons),
                "samples": len(sm), "power_w_max": max(power) if power else None}


# ----------------------------------------------------------- CPU legs ----

def cpu_sample(w, target_bytes: float):
    """A leading, segment-aligned sample of the workload of about
    ``target_bytes`` algorithmic bytes: (bf16/f32 host tensor, offsets,
    rows), values drawn on the host by torch's generator (same
    distribution as the device data)."""
    import torch
    row_bytes = w.d * w.element_bytes * (2 if w.op == "softmax" else 1)
    target_rows = max(1, min(w.n, int(target_bytes // row_bytes)))
    offsets = w.offsets().astype(np.int64)
    last = max(1, int(np.searchsorted(offsets, target_rows, side="right")) - 1)
    if int(offsets[last]) == 0:
        last = min(w.b, 1 + int(np.argmax(offsets[1:] > 0)))
    sample_offsets = offsets[:last + 1].copy()
    rows = int(sample_offsets[-1])
    values = workloads.device_values(w, (0, rows), torch.device("cpu"))
    index = np.int32 if w.index == "i32" else np.int64
    return values, sample_offsets.astype(index), rows


def _torch_softmax(torch, values, offsets):
    """The reference's CPU torch softmax: segment max, exp, segment sum,
    divide, in f32 (bf16 promoted first and the result cast back)."""
    work = values.float()
    lengths = offsets[1:] - offsets[:-1]
    ids = torch.repeat_interleave(torch.arange(lengths.numel()), lengths)
    maxima = torch.segment_reduce(work, "max", offsets=offsets, axis=0)
    weights = torch.exp(work - maxima[ids])
    totals = torch.segment_reduce(weights, "sum", offsets=offsets, axis=0)
    return (weights / totals[ids]).to(values.dtype)


def cpu_legs(w, target_bytes: float, timed_calls: int, warmup: int, threads: int) -> dict:
    """Both CPU implementations of the path on one bounded sample: the
    reference's torch baseline (baselines/torch_reference.py:12-16 of the
    reference: bf16 promoted to f32, torch.segment_reduce, cast back;
    softmax the CPU torch composition) with torch.set_num_threads(all), and
    the float64 C oracle on the same threads.  The faster one, by its
    median over ``timed_calls`` calls after ``warmup``, is the baseline;
    the other is timed on 3 calls."""
    import torch
    from oracle import native as coracle  # the CPU baseline leg
    torch.set_num_threads(threads)
    values, offsets, rows = cpu_sample(w, target_bytes)
    b = offsets.size - 1
    s_off = 4 if offsets.dtype == np.int32 else 8
    rows_out = rows if w.op == "softmax" else b
    nbytes = rows * w.d * w.element_bytes + (b + 1) * s_off + rows_out * w.d * w.element_bytes
    toff = torch.from_numpy(offsets.astype(np.int64))
    raw = values.view(torch.int16).numpy().view(np.uint16) if w.dtype == "bf16" else values.numpy()

    def torch_call():
        if w.op == "softmax":
            return _torch_softmax(torch, values, toff)
        work = values.float() if w.dtype == "bf16" else values
        return torch.segment_reduce(work, w.op, offsets=toff, axis=0).to(values.dtype)

    def oracle_call():
        return coracle.run(w.op, raw, offsets, dtype=w.dtype, threads=threads)

    legs = {"torch": torch_call, "oracle": oracle_call}
    probe = {}
    for name, call in legs.items():
        call()  # first touch of the sample and of the thread pool
        t0 = time.perf_counter()
        call()
        probe[name] = time.perf_counter() - t0
    fast = min(probe, key=probe.get)
    results = {}
    for name, call in legs.items():
        calls = timed_calls if name == fast else 3
        for _ in range(max(0, (warmup if name == fast else 1) - 1)):
            call()
        times = []
        for _ in range(calls):
            t0 = time.perf_counter()
            call()
            times.append(time.perf_counter() - t0)
        per_call = statistics.median(times)
        results[name] = {"value": round(nbytes / per_call / 1e9, 4), "unit": "GB/s",
                         "seconds_per_call": round(per_call, 5), "calls": calls,
                         "dtype": "f32" if name == "torch" else "f64"}
    what = {"torch": "torch.segment_reduce on CPU (f32)" if w.op != "softmax" else
            "CPU torch segment max / exp / segment sum / divide (f32)",
            "oracle": "float64 C oracle (restated oracle/reference.py)"}
    sample = (f"leading {rows} rows / {b} segments of {w.name} ({nbytes / 1e9:.3f} GB algorithmic) on "
              f"{threads} host threads")
    return {"fast": fast, "legs": results, "what": what, "sample": sample, "cores": threads, "bytes": nbytes}


def cpu_baseline_entry(legs: dict) -> dict:
    fast = legs["fast"]
    return {"value": legs["legs"][fast]["value"], "unit": "GB/s", "cores": legs["cores"], "kind": "port",
            "sample": f"{legs['sample']}; {legs['what'][fast]} (faster of the two), median of "
                      f"{legs['legs'][fast]['calls']} calls"}


def reference_arm(args) -> None:
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    w = workloads.make(args.workload, scale=args.scale)
    threads = host_threads()
    legs = cpu_legs(w, args.cpu_bytes, args.steps, args.warmup, threads)
    fast = legs["legs"][legs["fast"]]
    base = cpu_baseline_entry(legs)
    line = {"impl": "reference", "metric": metric_name(), "value": fast["value"], "unit": "GB/s",
            "n_gpus": args.gpus, "steps": fast["calls"], "warmup": args.warmup,
            "ms_per_step": round(fast["seconds_per_call"] * 1000, 3), "higher_is_better": True,
            "scaling": "strong", "vs_baseline": None, "dtype": fast["dtype"], "data": "synthetic",
            "config": config_dict(w, args, "n/a (host)"),
            "cpu_baseline": base,
            "e2e": {"value": fast["value"], "unit": "GB/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
            "legs": {name: {**leg, "impl": legs["what"][name]} for name, leg in legs["legs"].items()},
            "note": "the reference's GPU path is sm_86/sm_89 MLIR cubins and cannot load on sm_100; its CPU path "
                    "is timed instead, each step one call on a bounded sample of the workload (ms_per_step is per "
                    "sample call)"}
    print(json.dumps(line), flush=True)


# ------------------------------------------------------------ timing ----

def flush_l2(buffer):
    buffer.add_(1)  # writes 2x the L2 (read + write of a buffer > L2)


def time_calls(torch, fn, steps, warmup, stream, flush=None, dist=None):
    """Per-step device time (ms) with CUDA events on ``stream``, the K steps
    bracketed by a barrier and a synchronize on both sides; with ``dist``
    the per-step times are the maximum over ranks.  Multi-rank: the ranks'
    streams are aligned by a one-element all-reduce after the barrier (a
    host barrier returns at different times on different ranks, and the
    first collective of a step would charge that skew to step 1), and the
    last warm-up step runs after it, untimed, so the idle gap of the
    barrier is not charged to step 1 either."""
    for _ in range(warmup - (1 if dist is not None and warmup > 0 else 0)):
        if flush is not None:
            flush()
        fn()
    torch.cuda.synchronize()
    align = None
    if dist is not None:
        align = torch.zeros(1, device=torch.device("cuda", torch.cuda.current_device()))
        dist.barrier()
        torch.cuda.synchronize()
        dist.all_reduce(align)
        if warmup > 0:
            if flush is not None:
                flush()
            fn()
    starts = [torch.cuda.Event(enable_timing=True) for _ in range(steps)]
    ends = [torch.cuda.Event(enable_timing=True) for _ in range(steps)]
    for i in range(steps):
        if flush is not None:
            flush()
        starts[i].record(stream)
        fn()
        ends[i].record(stream)
    torch.cuda.synchronize()
    if dist is not None:
        dist.barrier()
    times = [s.elapsed_time(e) for s, e in zip(starts, ends)]
    if dist is not None:
        device = torch.device("cuda", torch.cuda.current_device())
        mine = torch.tensor([statistics.mean(times)], dtype=torch.float64, device=device)
        every = [torch.empty_like(mine) for _ in range(dist.get_world_size())]
        dist.all_gather(every, mine)
        RANK_MS[:] = [round(float(x.item()), 4) for x in every]
        t = torch.tensor(times, dtype=torch.float64, device=device)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        times = t.cpu().tolist()
    return times


RANK_MS: list = []  # mean step time of every rank in the last multi-GPU timing


# ------------------------------------------------------------ parity ----

def fetcher(torch, tensor):
    """``fetch(lo, hi)`` for the oracle checker: rows of a device tensor as
    the host array the C oracle reads (f32, or bf16 as raw uint16 bits)."""
    def fetch(lo, hi):
        block = tensor[lo:hi]
        if block.dtype == torch.bfloat16:
            return block.view(torch.int16).cpu().numpy().view(np.uint16)
        return block.float().cpu().numpy()
    return fetch


def host_rows(torch, out, segments=None) -> np.ndarray:
    if segments is None:
        return out.float().cpu().numpy().astype(np.float64)
    index = torch.from_numpy(np.asarray(segments, dtype=np.int64)).to(out.device)
    return out.index_select(0, index).float().cpu().numpy().astype(np.float64)


def parity_segments(offsets_host: np.ndarray, lead_rows: int = 2_000_000, tail: int = 2048) -> np.ndarray:
    """Segments checked on the benchmark's first call: the leading ones up
    to ``lead_rows`` rows, every segment of at least 1M rows (the giant
    segments cut across virtual CTAs and ranks) and the last ``tail``."""
    offsets = np.asarray(offsets_host, dtype=np.int64)
    b = offsets.size - 1
    lengths = np.diff(offsets)
    lead = int(np.searchsorted(offsets, lead_rows, side="right"))
    picked = np.concatenate([np.arange(min(b, max(1, lead))), np.nonzero(lengths >= 1_000_000)[0],
                             np.arange(max(0, b - tail), b)])
    return np.unique(picked)


def parity_single(torch, w, values, out, offsets_host) -> dict:
    """The first call's output (one GPU) against the oracle."""
    from oracle import device_check as dc  # the checker
    if w.op == "softmax":
        dc.check_softmax(host_rows(torch, out), fetcher(torch, values)(0, w.n), offsets_host, dtype=w.dtype)
        return {"parity": "ok", "parity_rows": w.n}
    whole = w.n * w.d * w.element_bytes <= 4e9  # c1-c4: every segment; c5: a sample with the giants
    segments = np.arange(w.b) if whole else parity_segments(offsets_host)
    dc.check_reduction(host_rows(torch, out, segments), fetcher(torch, values), w.n, offsets_host, segments,
                       op=w.op, dtype=w.dtype)
    rows = int(np.sum(np.diff(offsets_host.astype(np.int64))[segments]))
    return {"parity": "ok", "parity_segments": int(segments.size), "parity_rows": rows}


def parity_sharded(torch, dist, w, values, out, offsets_host, row0, rank, world, owners) -> dict:
    """The first call's output over all ranks: each rank reduces its rows of
    the checked segments in the oracle; rank 0 merges the float64 pieces in
    rank order (the oracle's own merge) and compares the rows the owners
    wrote.  Every rank takes the same collectives; the outcome is shared."""
    from oracle import device_check as dc, native  # the checker
    segments = parity_segments(offsets_host)
    kinds = (w.op, "abssum") if w.op == "sum" else (w.op,)
    parts = dc.segment_partials(fetcher(torch, values), values.shape[0], w.d, offsets_host, segments, kinds=kinds,
                                dtype=w.dtype, row_base=row0)
    device = values.device
    mine = torch.from_numpy(np.stack(parts)).to(device)
    every = [torch.empty_like(mine) for _ in range(world)]
    dist.all_gather(every, mine)
    rows_mine = out.index_select(0, torch.from_numpy(segments).to(device)).float()
    rows_every = [torch.empty_like(rows_mine) for _ in range(world)]
    dist.all_gather(rows_every, rows_mine)
    failed = torch.zeros(1, dtype=torch.int32, device=device)
    message = ""
    if rank == 0:
        pieces = [e.cpu().numpy() for e in every]
        merged = pieces[0].copy()
        for piece in pieces[1:]:
            for k, kind in enumerate(kinds):
                merged[k] = native.merge(kind, merged[k], piece[k])
        owner = owners[segments]
        gathered = np.stack([r.cpu().numpy() for r in rows_every]).astype(np.float64)
        actual = gathered[owner, np.arange(segments.size)]
        lengths = np.diff(offsets_host.astype(np.int64))[segments]
        try:
            native.check(actual, w.op, w.dtype, np.concatenate([[0], np.cumsum(lengths)]), merged[0],
                         merged[1] if w.op == "sum" else None)
        except AssertionError as exc:
            failed.fill_(1)
            message = str(exc)
    dist.all_reduce(failed, op=dist.ReduceOp.MAX)
    if int(failed.item()):
        raise SystemExit(f"parity check of the first call failed: {message or 'see rank 0'}")
    rows = int(np.sum(np.diff(offsets_host.astype(np.int64))[segments]))
    return {"parity": "ok", "parity_segments": int(segments.size), "parity_rows": rows}


# ---------------------------------------------------------------- ours ----

def ours(args) -> None:
    import torch
    from ragged import ArtifactCache, Compiler, ProgramSpec
    from ragged.sharding import (balanced_split, end_weight_model, segment_owners, shard_rows, torch_exchange)

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world != args.gpus:
        raise SystemExit(f"--gpus {args.gpus} but WORLD_SIZE={world}")
    torch.cuda.set_device(local)
    device = torch.device("cuda", local)
    dist = None
    if world > 1:
        import datetime
        import torch.distributed as dist
        dist.init_process_group("nccl", device_id=device, timeout=datetime.timedelta(seconds=120))
    w = workloads.make(args.workload, scale=args.scale)
    if world > 1 and w.op == "softmax":
        raise SystemExit("the benchmark's sharded calls compute sum and max; run softmax workloads with --gpus 1")
    offsets_host = w.offsets()
    end_weight = end_weight_model(w.op, w.dtype, w.d)
    split_fit = {"fit": "model weight"}
    splits = balanced_split(offsets_host, world, end_weight) if world > 1 else None
    rows = shard_rows(w.n, world, rank, splits)
    values = workloads.device_values(w, rows, device)
    offsets = torch.from_numpy(offsets_host).to(device)
    rows_out = w.n if w.op == "softmax" else w.b
    out = torch.empty((rows_out, w.d), dtype=values.dtype, device=device)
    cache = ArtifactCache(REPO / "_build" / "bench-cache", max_specializations=64)
    program = Compiler().compile(ProgramSpec(w.op, w.dtype, w.d, w.index), cache)
    max_len = int(w.lengths.max()) if w.b else 0
    select = args.schedule
    stream = torch.cuda.current_stream(device)
    l2 = torch.cuda.get_device_properties(device).L2_cache_size
    flush_buffer, flush_note = None, "inputs larger than L2 (no flush)"
    if values.numel() * values.element_size() < 4 * l2:
        flush_buffer = torch.empty(2 * l2 // 4, dtype=torch.float32, device=device)
        flush_note = "L2 flushed between steps (2x L2 buffer rewritten)"
    flush = (lambda: flush_l2(flush_buffer)) if flush_buffer is not None else None
    report_holder = {}
    exchange = torch_exchange() if world > 1 else None
    if world > 1 and args.split_fit:
        # Refit the split from measured local phases (the shard kernel and its
        # fix-up on each rank's rows, exchange left out), then re-shard (the
        # fit needs four ranks or more; with fewer the model weight stays).
        # Off by default: calls timed one at a time after a host
        # synchronisation run well above the back-to-back step time, which
        # skews the fit.
        end_weight, split_fit, splits = refit_split(torch, dist, program, w, values, offsets, out, offsets_host,
                                                    world, rank, splits, end_weight)
        new_rows = shard_rows(w.n, world, rank, splits)
        if new_rows != rows:
            del values
            torch.cuda.empty_cache()
            rows = new_rows
            values = workloads.device_values(w, rows, device)
    owners = segment_owners(offsets_host, world, splits) if w.op != "softmax" else None

    def step():
        if world > 1:
            report_holder["r"] = program.run_sharded(values, offsets, out, total_rows=w.n, world=world, rank=rank,
                                                     exchange=exchange, splits=splits)
        else:
            report_holder["r"] = program.run(values, offsets, out, select=select, max_len=max_len)

    # Parity gate: the first call, checked before anything is timed.
    parity = {"parity": "skipped"}
    step()
    torch.cuda.synchronize()
    if not args.no_parity:
        if world > 1:
            parity = parity_sharded(torch, dist, w, values, out, offsets_host, rows[0], rank, world, owners)
        elif rank == 0:
            parity = parity_single(torch, w, values, out, offsets_host)
    if dist is not None:
        dist.barrier()
    torch.cuda.synchronize()
    with ClockSampler(local) as clocks:
        times = time_calls(torch, step, args.steps, args.warmup, stream, flush, dist)
    report = report_holder["r"]
    ms = statistics.mean(times)
    nbytes = w.algorithmic_bytes()
    value = nbytes / (ms / 1e3) / 1e9
    peak, peak_kind = peak_hbm()
    per_rank = nbytes / world
    launches = (len(report.kernel_names) + (1 if world > 1 else 0)) * args.steps
    line = {"metric": metric_name(), "value": round(value, 2), "unit": "GB/s", "n_gpus": args.gpus,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(ms, 4), "higher_is_better": True,
            "scaling": "strong", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
            "config": config_dict(w, args, flush_note), **parity, "schedule_selected": report.selected,
            "kernels": list(report.kernel_names) + (["shard_combine"] if world > 1 else []),
            "gpu_launches": launches,
            "step_times_ms": [round(t, 4) for t in times],
            "roofline": {"bound": "hbm", "achieved": round(per_rank / (ms / 1e3) / 1e9, 2), "peak": peak,
                         "unit": "GB/s", "frac": round(per_rank / (ms / 1e3) / 1e9 / peak, 4),
                         "traffic": (round(TRAFFIC_RATIO[w.name] * per_rank) if w.name in TRAFFIC_RATIO and
                                     args.scale == 1.0 else None),
                         "peak_source": f"{peak_kind} (MEASURED_PEAKS.json hbm_gbs)" if peak_kind == "measured"
                         else "fallback 6650 GB/s",
                         "kernel": "whole call per GPU (all kernels of the schedule; the slowest rank); for c5 the "
                                   "rowbal_kernel is 99.5% of its device time (ncu launch list)"},
            "clocks": clocks.summary()}
    if world > 1:
        line["sharding"] = {"rows_per_rank": [list(shard_rows(w.n, world, r, splits)) for r in range(world)],
                            "split": f"rows + {end_weight:.4g} x segment ends balanced across ranks",
                            "end_weight_fit": split_fit,
                            "rank_ms": list(RANK_MS),
                            "collective": "NCCL all-gather of edge records",
                            "edge_bytes_per_rank": _native_edge_bytes(w),
                            "phases_ms": phase_profile(torch, dist, program, w, values, offsets, out, world, rank,
                                                       splits, exchange, flush)}
    if not args.no_e2e:
        line["e2e"] = e2e_leg(torch, args, w, program, values, offsets_host, out, max_len, select, stream, dist,
                              splits, owners, rank, world, exchange)
    if world == 1 and not args.no_configs:
        del values, out, flush_buffer
        torch.cuda.empty_cache()
        line["configs"] = side_configs(torch, args, device, stream, cache, peak)
    if not args.no_cpu_baseline and rank == 0 and world == 1:
        legs = cpu_legs(w, args.cpu_bytes, 3, 1, host_threads())
        line["cpu_baseline"] = cpu_baseline_entry(legs)
        line["cpu_legs"] = {name: {**leg, "impl": legs["what"][name]} for name, leg in legs["legs"].items()}
    if rank == 0:
        print(json.dumps(line), flush=True)
    if dist is not None:
        dist.barrier()
        dist.destroy_process_group()


def phase_profile(torch, dist, program, w, values, offsets, out, world, rank, splits, exchange, flush,
                  steps: int = 5) -> dict:
    """Per-rank device time of each phase of a sharded call, after the timed
    steps (untimed for the headline): ``local`` (rg_run_shard: the window's
    kernel and fix-up), ``exchange`` (the all-gather as the rank sees it,
    waiting for the slowest rank included), ``combine`` (shard_combine), each
    the median of ``steps`` calls with events around the phases; and
    ``allgather_alone``: the same all-gather with the ranks' streams aligned
    first, so its time is the collective's own."""
    import statistics as st
    marks = {}

    def timed_exchange(edges):
        marks["a"].record()
        gathered = exchange(edges)
        marks["b"].record()
        return gathered

    local, wait, combine, alone = [], [], [], []
    align = torch.zeros(1, device=values.device)
    for _ in range(steps):
        if flush is not None:
            flush()
        dist.barrier()
        torch.cuda.synchronize()
        dist.all_reduce(align)
        marks.update({k: torch.cuda.Event(enable_timing=True) for k in ("s", "a", "b", "e")})
        marks["s"].record()
        program.run_sharded(values, offsets, out, total_rows=w.n, world=world, rank=rank, exchange=timed_exchange,
                            splits=splits)
        marks["e"].record()
        torch.cuda.synchronize()
        local.append(marks["s"].elapsed_time(marks["a"]))
        wait.append(marks["a"].elapsed_time(marks["b"]))
        combine.append(marks["b"].elapsed_time(marks["e"]))
    edges = torch.zeros(_native_edge_bytes(w) // 4, dtype=torch.float32, device=values.device)
    for _ in range(steps):
        dist.barrier()
        torch.cuda.synchronize()
        dist.all_reduce(align)
        start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        start.record()
        exchange(edges)
        end.record()
        torch.cuda.synchronize()
        alone.append(start.elapsed_time(end))
    mine = torch.tensor([st.median(x) for x in (local, wait, combine, alone)], dtype=torch.float64,
                        device=values.device)
    every = [torch.empty_like(mine) for _ in range(world)]
    dist.all_gather(every, mine)
    table = [[round(float(v), 4) for v in t.cpu().tolist()] for t in every]
    return {name: [row[i] for row in table] for i, name in enumerate(("local", "exchange", "combine",
                                                                      "allgather_alone"))}


def refit_split(torch, dist, program, w, values, offsets, out, offsets_host, world, rank, splits, weight):
    """Time each rank's local phase (rg_run_shard + fix-up + combine, with a
    local stand-in for the exchange, so no rank waits for another) on the
    current split, fit the end weight to the ranks' times
    (sharding.fit_end_weight) and return (weight, fit, new split).  Every
    rank computes the same fit from the all-gathered times."""
    import statistics as st
    local = lambda edges: edges.repeat(world)  # same shape as the gathered records
    times = []
    for i in range(5):
        start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        start.record()
        program.run_sharded(values, offsets, out, total_rows=w.n, world=world, rank=rank, exchange=local,
                            splits=splits)
        end.record()
        torch.cuda.synchronize()
        if i >= 2:
            times.append(start.elapsed_time(end))
    mine = torch.tensor([st.median(times)], dtype=torch.float64, device=values.device)
    every = [torch.empty_like(mine) for _ in range(world)]
    dist.all_gather(every, mine)
    return split_from_rank_times(w.n, offsets_host, world, splits, [float(t.item()) for t in every], weight)


def split_from_rank_times(n, offsets_host, world, splits, rank_ms, weight):
    """The host half of ``refit_split``: rows and segment ends of each
    rank's window under ``splits``, the end weight fitted to the measured
    per-rank times (``weight`` kept when the fit is not possible), and the
    balanced split for it."""
    from ragged.sharding import balanced_split, fit_end_weight, shard_rows, window_ends
    rows = [shard_rows(n, world, r, splits)[1] - shard_rows(n, world, r, splits)[0] for r in range(world)]
    ends = window_ends(offsets_host, world, splits)
    fitted, info = fit_end_weight(rows, ends, rank_ms, weight)
    info = {**info, "model_weight": round(weight, 4), "fitted_weight": round(fitted, 4),
            "rank_ms_before": [round(t, 4) for t in rank_ms]}
    return fitted, info, balanced_split(offsets_host, world, fitted)


def side_configs(torch, args, device, stream, cache, peak) -> dict:
    """c1-c4 on one GPU: each at full size, its first call checked against
    the oracle (whole output), then K calls timed like the main workload
    (L2 flushed between steps when the inputs are smaller than 4x L2)."""
    from ragged import Compiler, ProgramSpec
    l2 = torch.cuda.get_device_properties(device).L2_cache_size
    flush_buffer = torch.empty(2 * l2 // 4, dtype=torch.float32, device=device)
    entries = {}
    for name in SIDE_CONFIGS:
        w = workloads.make(name, scale=args.scale)
        values = workloads.device_values(w, (0, w.n), device)
        offsets_host = w.offsets()
        offsets = torch.from_numpy(offsets_host).to(device)
        out = torch.empty((w.n if w.op == "softmax" else w.b, w.d), dtype=values.dtype, device=device)
        program = Compiler().compile(ProgramSpec(w.op, w.dtype, w.d, w.index), cache)
        max_len = int(w.lengths.max()) if w.b else 0
        holder = {}

        def call():
            holder["r"] = program.run(values, offsets, out, max_len=max_len)

        call()
        torch.cuda.synchronize()
        parity = parity_single(torch, w, values, out, offsets_host)["parity"] if not args.no_parity else "skipped"
        small = values.numel() * values.element_size() < 4 * l2
        with ClockSampler(device.index or 0) as clocks:
            times = time_calls(torch, call, args.steps, args.warmup, stream,
                               (lambda: flush_l2(flush_buffer)) if small else None)
        ms = statistics.median(times)
        gbs = w.algorithmic_bytes() / (ms / 1e3) / 1e9
        report = holder["r"]
        entries[name] = {"op": w.op, "dtype": w.dtype, "D": w.d, "N": w.n, "B": w.b, "offsets": w.index,
                         "us_per_call": round(ms * 1000, 2), "value": round(gbs, 1), "unit": "GB/s",
                         "roofline_frac": round(gbs / peak, 4), "schedule_selected": report.selected,
                         "kernels": list(report.kernel_names), "parity": parity,
                         "l2": "flushed between steps" if small else "inputs larger than L2",
                         "target": "0.70 of peak (D >= 64)" if w.d >= 64 else "none (D < 64)",
                         "clocks": clocks.summary()}
        del values, out, offsets
        torch.cuda.empty_cache()
    return entries


def _native_edge_bytes(w) -> int:
    from ragged import _native
    return _native.shard_edge_bytes(w.op, w.d)


def host_memory_available() -> int:
    try:
        for line in Path("/proc/meminfo").read_text().splitlines():
            if line.startswith("MemAvailable:"):
                return int(line.split()[1]) * 1024
    except OSError:
        pass
    return 0


def e2e_leg(torch, args, w, program, values, offsets_host, out, max_len, select, stream, dist=None, splits=None,
            owners=None, rank=0, world=1, exchange=None) -> dict:
    """Same metric with inputs in pinned host memory; every step copies this
    rank's rows and the offsets in and the rows of out this rank finishes
    back, inside the timed region (max over ranks)."""
    need = values.numel() * values.element_size() + out.numel() * out.element_size() + offsets_host.nbytes
    available = host_memory_available()
    skip = need * world > 0.6 * available
    if dist is not None:
        flag = torch.tensor([1 if skip else 0], device=values.device)
        dist.all_reduce(flag, op=dist.ReduceOp.MAX)
        skip = bool(flag.item())
    if skip:
        return {"value": None, "unit": "GB/s", "h2d_bytes_per_step": need, "d2h_bytes_per_step": None,
                "skipped": f"pinned host buffers ({need * world / 1e9:.1f} GB over all ranks) exceed 60% of "
                           f"MemAvailable ({available / 1e9:.1f} GB)"}
    host_values = torch.empty(values.shape, dtype=values.dtype, pin_memory=True)
    host_values.copy_(values)
    host_offsets = torch.from_numpy(offsets_host).pin_memory()
    if owners is not None:
        mine = np.nonzero(owners == rank)[0]
        first, last = (int(mine[0]), int(mine[-1]) + 1) if mine.size else (0, 0)
    else:
        first, last = 0, out.shape[0]
    host_out = torch.empty((last - first, out.shape[1]), dtype=out.dtype, pin_memory=True)
    dev_offsets = torch.empty_like(host_offsets, device=values.device)

    def step():
        values.copy_(host_values, non_blocking=True)
        dev_offsets.copy_(host_offsets, non_blocking=True)
        if world > 1:
            program.run_sharded(values, dev_offsets, out, total_rows=w.n, world=world, rank=rank, exchange=exchange,
                                splits=splits)
        else:
            program.run(values, dev_offsets, out, select=select, max_len=max_len)
        host_out.copy_(out[first:last], non_blocking=True)

    times = time_calls(torch, step, args.steps, 1, stream, None, dist)
    ms = statistics.mean(times)
    h2d = host_values.numel() * host_values.element_size() + host_offsets.numel() * host_offsets.element_size()
    d2h = host_out.numel() * host_out.element_size()
    return {"value": round(w.algorithmic_bytes() / (ms / 1e3) / 1e9, 3), "unit": "GB/s",
            "h2d_bytes_per_step": int(h2d), "d2h_bytes_per_step": int(d2h), "ms_per_step": round(ms, 3),
            "note": "per rank: its rows and the offsets in, the output rows it finishes out" if world > 1 else
                    "values and offsets in, all output rows out"}


def main() -> None:
    args = parse_args()
    if args.impl == "reference":
        reference_arm(args)
    else:
        ours(args)


if __name__ == "__main__":
    main()
