"""Helpers shared by the GPU parity tests.

``execute`` runs one call through the public API (ProgramSpec -> Compiler ->
CompiledProgram.run -> rg_run in libragged_b200.so) with the output placed
inside a guard buffer (rows before and after filled with a sentinel, as the
reference's test/gpu/test_correctness.py:101-111 does) and checks the result
against the CPU oracle with BOTH the reference's tolerance contract and this
build's strict one.
"""
from __future__ import annotations

import functools
import tempfile

import numpy as np

from oracle import reference_port as rp

SENTINEL = -64.0
DISTRIBUTIONS = ("uniform", "long_tail", "bimodal", "burst", "exponential")


def make_lengths(distribution: str, segments: int, total: int, seed: int) -> np.ndarray:
    """Seeded lengths summing to ``total`` (the reference's five length
    families, bench/distributions.py:15-64, restated for tests)."""
    rng = np.random.default_rng(seed)
    if distribution == "uniform":
        weights = np.ones(segments)
    elif distribution == "long_tail":
        weights = np.minimum(rng.pareto(1.3, segments) + 1, 100000.0)
    elif distribution == "bimodal":
        weights = np.where(rng.random(segments) < 0.9, 4.0, 1024.0)
    elif distribution == "exponential":
        weights = rng.exponential(1.0, segments)
    else:
        weights = np.ones(segments)
        width = max(1, segments // 100)
        start = int(rng.integers(segments - width + 1))
        weights[start:start + width] = 16384
    units = np.maximum(1, np.rint(weights * 1024).astype(np.int64))
    share = units / units.sum() * total
    lengths = np.floor(share).astype(np.int64)
    remainder = total - int(lengths.sum())
    lengths[np.argsort(-(share - lengths), kind="stable")[:remainder]] += 1
    return lengths


def offsets_of(lengths, index="i64") -> np.ndarray:
    out = np.zeros(len(lengths) + 1, dtype=np.int64)
    np.cumsum(lengths, out=out[1:])
    return out.astype(np.int32 if index == "i32" else np.int64)


@functools.lru_cache(maxsize=None)
def _cache_dir():
    return tempfile.mkdtemp(prefix="ragged-b200-test-cache-")


@functools.lru_cache(maxsize=512)
def program(op, dtype, d, index, strategy="auto", vectorize=True):
    from ragged import ArtifactCache, Compiler, Optimizations, ProgramSpec
    spec = ProgramSpec(op, dtype, d, index, strategy=strategy, optimizations=Optimizations(vectorize=vectorize))
    return Compiler().compile(spec, ArtifactCache(_cache_dir(), max_specializations=4096))


def prepared(values, dtype):
    values = np.ascontiguousarray(values, dtype=np.float32)
    return rp.quantize_bf16(values) if dtype == "bf16" else values


def run_device(torch, op, dtype, values, offsets, *, select="auto", strategy="auto", stream=None,
               max_len=None, vectorize=True, guard=True):
    """Run through the API; returns (output as float64 numpy, report)."""
    offsets = np.ascontiguousarray(offsets)
    index = "i32" if offsets.dtype == np.int32 else "i64"
    d = values.shape[1]
    prog = program(op, dtype, d, index, strategy, vectorize)
    tdtype = torch.float32 if dtype == "f32" else torch.bfloat16
    rows = values.shape[0] if op == "softmax" else offsets.size - 1
    device_values = torch.from_numpy(np.ascontiguousarray(values, dtype=np.float32)).to("cuda").to(tdtype)
    device_offsets = torch.from_numpy(offsets).to("cuda")
    guard_elems = 64 if guard else 0   # 64 elements: keeps the output 16-byte aligned
    buffer = torch.full((rows * d + 2 * guard_elems,), SENTINEL, device="cuda", dtype=tdtype)
    out = buffer[guard_elems:guard_elems + rows * d].view(rows, d)
    report = prog.run(device_values, device_offsets, out, stream=stream, select=select, max_len=max_len)
    torch.cuda.synchronize()
    result = out.float().cpu().numpy().astype(np.float64)
    if guard:
        flat = buffer.float().cpu().numpy()
        assert np.all(flat[:guard_elems] == SENTINEL) and np.all(flat[guard_elems + rows * d:] == SENTINEL), \
            "write outside the output rows"
    return result, report


def check(actual, values, offsets, op, dtype, reference=None):
    """Both contracts: the reference's assert_matches and check_strict."""
    with np.errstate(all="ignore"):
        if reference is None:
            reference = rp.REFERENCES[op](values, offsets)
        rp.assert_matches(actual, values, offsets, operation=op, input_dtype=dtype, reference=reference)
        rp.check_strict(actual, values, offsets, operation=op, input_dtype=dtype, reference=reference)


def fetcher(tensor):
    """``fetch(lo, hi)`` for oracle.device_check: rows lo..hi of a torch
    tensor as the host array the C oracle reads (f32, or bf16 as raw uint16
    bits), copied a chunk at a time."""
    import torch

    def fetch(lo, hi):
        block = tensor[lo:hi]
        if block.dtype == torch.bfloat16:
            return block.view(torch.int16).cpu().numpy().view(np.uint16)
        return block.float().cpu().numpy()

    return fetch


def host_rows(out, segments=None) -> np.ndarray:
    """Output rows (all, or those of ``segments``) as float64 host values."""
    import torch
    if segments is None:
        return out.float().cpu().numpy().astype(np.float64)
    index = torch.from_numpy(np.asarray(segments, dtype=np.int64)).to(out.device)
    return out.index_select(0, index).float().cpu().numpy().astype(np.float64)
