"""Benchmark: segmented reduction throughput on B200 (one JSON line).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
                    [--workload c5] [--schedule auto] [--no-e2e] [--configs]

A step is one pass of the hot path over one batch: one segmented reduction
of the whole workload (default ``c5``: bf16 sum, D=256, N=200M rows, B=4M
Zipf segments -- the configuration the metric is quoted on at 1/2/4/8
GPUs).  With N GPUs (torchrun, one process per GPU) the rows are split
evenly across ranks (strong scaling: the total work is fixed), each rank
reduces its rows, and the partial sums of segments cut by shard boundaries
are combined over NVLink (NCCL all-gather + a deterministic combine kernel).

value          = algorithmic bytes of the whole job / max-over-ranks device
                 time per step (GB/s), inputs resident in HBM;
e2e            = the same metric through the public API with the inputs in
                 pinned host memory: H2D copy, the call, D2H of the result,
                 every step inside the timed region;
roofline       = the dominant kernel's achieved bandwidth vs the measured
                 copy bandwidth in MEASURED_PEAKS.json;
cpu_baseline   = the CPU oracle port (C, float64, all host threads) on a
                 bounded sample of the same workload (rank 0, N=1 only).

``--impl reference`` times the reference's CPU implementation of the path
(the oracle port; the reference's own GPU path cannot run on sm_100) on the
host cores and prints its line with "impl": "reference".
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


def parse_args():
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
    parser.add_argument("--configs", action="store_true", help="also time c1-c4 on one GPU (extra key)")
    parser.add_argument("--cpu-seconds", type=float, default=12.0, help="target CPU-baseline work")
    return parser.parse_args()


def peak_hbm() -> tuple[float, str]:
    try:
        data = json.loads(PEAKS_FILE.read_text())
        return float(data["hbm_gbs"]), "measured"
    except (OSError, ValueError, KeyError):
        return FALLBACK_HBM_GBS, "fallback"


# --------------------------------------------------------------- clocks ----

class ClockSampler:
    """nvidia-smi samples during the timed region."""

    QUERY = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
             "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
             "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, device: int):
        self.device = device
        self.proc = None

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
        for line in getattr(self, "lines", []):
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


# ------------------------------------------------------------ workload ----

def device_values(torch, w, rows: tuple[int, int], device) -> "torch.Tensor":
    """Values of rows [lo, hi) generated on the device (deterministic per
    row chunk, so every rank builds exactly its slice of one dataset)."""
    lo, hi = rows
    tdtype = torch.float32 if w.dtype == "f32" else torch.bfloat16
    out = torch.empty((hi - lo, w.d), dtype=tdtype, device=device)
    chunk = 1 << 22  # rows per generator chunk
    first = lo // chunk
    for c in range(first, (hi + chunk - 1) // chunk):
        a, b = max(lo, c * chunk), min(hi, (c + 1) * chunk)
        g = torch.Generator(device=device)
        g.manual_seed(1_000_003 * w.value_seed + c)
        block = torch.empty(((c + 1) * chunk - c * chunk, w.d), dtype=tdtype, device=device)
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


def flush_l2(torch, buffer):
    buffer.add_(1)  # writes 2x the L2 (read + write of a buffer > L2)


# ------------------------------------------------------------- CPU leg ----

def cpu_sample(w, seconds: float):
    """(values f32/bf16-as-f32 host array, offsets, bytes) of a leading,
    segment-aligned sample of the workload sized for about ``seconds`` of
    multi-threaded oracle work at a conservative 2 GB/s."""
    target_bytes = int(seconds * 2e9 / 4)  # one call ~ a quarter of the budget
    row_bytes = w.d * w.element_bytes
    target_rows = max(1, min(w.n, target_bytes // row_bytes))
    offsets = w.offsets().astype(np.int64)
    last = int(np.searchsorted(offsets, target_rows, side="right")) - 1
    last = max(1, last)
    sample_offsets = offsets[:last + 1].copy()
    rows = int(sample_offsets[-1])
    if rows == 0:
        last = min(w.b, 1 + int(np.argmax(offsets[1:] > 0)))
        sample_offsets = offsets[:last + 1].copy()
        rows = int(sample_offsets[-1])
    values = w.host_values(slice(0, rows))
    index = np.int32 if w.index == "i32" else np.int64
    return values, sample_offsets.astype(index), rows


def run_cpu_baseline(w, seconds: float) -> dict:
    from oracle import native as coracle  # CPU baseline leg only
    values, offsets, rows = cpu_sample(w, seconds)
    threads = coracle.max_threads()
    b = offsets.size - 1
    s_off = 4 if offsets.dtype == np.int32 else 8
    rows_out = rows if w.op == "softmax" else b
    nbytes = rows * w.d * w.element_bytes + (b + 1) * s_off + rows_out * w.d * w.element_bytes
    coracle.run(w.op, values, offsets, dtype=w.dtype, threads=threads)  # warm-up
    times = []
    deadline = time.perf_counter() + seconds
    while time.perf_counter() < deadline or len(times) < 2:
        t0 = time.perf_counter()
        coracle.run(w.op, values, offsets, dtype=w.dtype, threads=threads)
        times.append(time.perf_counter() - t0)
    best = statistics.median(times)
    return {"value": round(nbytes / best / 1e9, 3), "unit": "GB/s", "cores": threads, "kind": "port",
            "sample": f"leading {rows} rows / {b} segments of {w.name} ({nbytes / 1e9:.2f} GB algorithmic), "
                      f"float64 C oracle, median of {len(times)} calls",
            "seconds_per_call": round(best, 4)}


def reference_arm(args) -> None:
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    w = workloads.make(args.workload, scale=args.scale)
    # Each step is one bounded sample call; the run is sized to a few minutes.
    per_step = max(1.0, min(20.0, 120.0 / max(1, args.steps + args.warmup)))
    base = run_cpu_baseline(w, per_step)
    line = {"impl": "reference", "metric": metric_name(), "value": base["value"], "unit": "GB/s",
            "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": round(base["seconds_per_call"] * 1000, 3), "higher_is_better": True,
            "scaling": "strong", "vs_baseline": None, "dtype": "f64", "data": "synthetic",
            "config": config_dict(w, args, "n/a"),
            "cpu_baseline": {k: base[k] for k in ("value", "unit", "cores", "kind", "sample")},
            "e2e": {"value": base["value"], "unit": "GB/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
            "note": "the reference's GPU path is sm_86/sm_89 MLIR cubins and cannot load on sm_100; its CPU "
                    "implementation of the path (the float64 oracle, restated in C and run on all host threads) "
                    "is timed instead"}
    print(json.dumps(line), flush=True)


def metric_name() -> str:
    return "effective HBM GB/s of segmented reduction (algorithmic bytes / device time per call)"


def config_dict(w, args, flush) -> dict:
    return {"workload": w.name, "op": w.op, "values_dtype": w.dtype, "accumulate": "f32", "D": w.d, "N": w.n,
            "B": w.b, "offsets": w.index, "schedule": args.schedule, "algorithmic_bytes": w.algorithmic_bytes(),
            "parallelism": f"row-sharded x{args.gpus}", "l2": flush, **({"lengths_rule": w.notes["lengths_rule"]}
                                                                      if "lengths_rule" in w.notes else {})}


# ---------------------------------------------------------------- ours ----

def time_calls(torch, fn, steps, warmup, stream, flush=None, dist=None):
    """Per-step device time (ms) with CUDA events on ``stream``, the K steps
    bracketed by a barrier and a synchronize on both sides; with ``dist``
    the per-step times are the maximum over ranks."""
    for _ in range(warmup):
        if flush is not None:
            flush()
        fn()
    torch.cuda.synchronize()
    if dist is not None:
        dist.barrier()
        torch.cuda.synchronize()
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


def ours(args) -> None:
    import torch
    from ragged import ArtifactCache, Compiler, ProgramSpec
    from ragged.sharding import END_WEIGHT, balanced_split, segment_owners, shard_rows, torch_exchange

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
        raise SystemExit("sharded calls compute sum and max; run softmax workloads with --gpus 1")
    offsets_host = w.offsets()
    splits = balanced_split(offsets_host, world, END_WEIGHT) if world > 1 else None
    rows = shard_rows(w.n, world, rank, splits)
    values = device_values(torch, w, rows, device)
    offsets = torch.from_numpy(offsets_host).to(device)
    tdtype = values.dtype
    rows_out = w.n if w.op == "softmax" else w.b
    out = torch.empty((rows_out, w.d), dtype=tdtype, device=device)
    spec = ProgramSpec(w.op, w.dtype, w.d, w.index)
    cache = ArtifactCache(REPO / "_build" / "bench-cache", max_specializations=64)
    program = Compiler().compile(spec, cache)
    max_len = int(w.lengths.max()) if w.b else 0
    select = args.schedule
    stream = torch.cuda.current_stream(device)
    l2 = torch.cuda.get_device_properties(device).L2_cache_size
    input_bytes = values.numel() * values.element_size()
    flush_buffer = None
    flush_note = "inputs larger than L2 (no flush)"
    if input_bytes < 4 * l2:
        flush_buffer = torch.empty(2 * l2 // 4, dtype=torch.float32, device=device)
        flush_note = "L2 flushed between steps (2x L2 buffer rewritten)"

    report_holder = {}
    exchange = torch_exchange() if world > 1 else None

    def step():
        if world > 1:
            report_holder["r"] = program.run_sharded(values, offsets, out, total_rows=w.n, world=world, rank=rank,
                                                     exchange=exchange, splits=splits)
        else:
            report_holder["r"] = program.run(values, offsets, out, select=select, max_len=max_len)

    flush = (lambda: flush_l2(torch, flush_buffer)) if flush_buffer is not None else None
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
            "config": config_dict(w, args, flush_note), "schedule_selected": report.selected,
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
                            "split": f"rows + {END_WEIGHT} x segment ends balanced across ranks",
                            "rank_ms": list(RANK_MS),
                            "collective": "NCCL all-gather of edge records",
                            "edge_bytes_per_rank": _native_edge_bytes(w)}
    if not args.no_e2e:
        owners = segment_owners(offsets_host, world, splits) if w.op != "softmax" else None
        line["e2e"] = e2e_leg(torch, args, w, program, values, offsets_host, out, max_len, select, stream, dist,
                              splits, owners, rank, world, exchange)
    if not args.no_cpu_baseline and rank == 0 and world == 1:
        line["cpu_baseline"] = {k: v for k, v in run_cpu_baseline(w, args.cpu_seconds).items()
                                if k != "seconds_per_call"}
    if rank == 0:
        print(json.dumps(line), flush=True)
    if dist is not None:
        dist.barrier()
        dist.destroy_process_group()


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
