"""GPU parity at the benchmark configurations' full sizes.

c1-c4 of BASELINE.json run at full size through the public API on every
schedule of their program (the cost model's choice first), values drawn on
the device by the same generator as ``bench.py``; the whole output is
compared with the C float64 oracle (rows streamed from the device in
chunks) under both tolerance contracts.  c5 runs at a tenth of its size
(20M rows, 10 GB): large enough that the row-balanced kernel takes its
virtual CTAs from the claim counter, with its three 5M-row segments chained
across hundreds of virtual CTAs.  A 40M-row segment of f32 D=4 rows makes a
fix-up chain cross thousands of virtual CTAs.
"""
from __future__ import annotations

import functools

import numpy as np
import pytest

from helpers import fetcher, host_rows
from oracle import device_check as dc
from oracle import native

pytestmark = pytest.mark.gpu


@functools.lru_cache(maxsize=None)
def _program(op, dtype, d, index):
    from helpers import program
    return program(op, dtype, d, index)


def _claims(report) -> bool:
    """Whether the row-balanced kernel took virtual CTAs from its claim
    counter: its fix-up runs one CTA per virtual CTA, more than the main
    kernel's resident grid."""
    names = list(report.kernel_names)
    if "rowbalanced" not in names or "rowbalanced_fixup" not in names:
        return False
    main = report.grids[names.index("rowbalanced")][0]
    fixup = report.grids[names.index("rowbalanced_fixup")][0]
    return fixup > main


@functools.lru_cache(maxsize=1)
def _device_cache(name):
    import torch
    from ragged import workloads
    w = workloads.make(name)
    return w, workloads.device_values(w, (0, w.n), torch.device("cuda", 0))


@pytest.mark.parametrize("name", ["c1", "c2_sum", "c2_max", "c3", "c4_sum", "c4_max"])
def test_configuration_full_size(cuda, name):
    w, values = _device_cache(name)
    program = _program(w.op, w.dtype, w.d, w.index)
    offsets_host = w.offsets()
    offsets = cuda.from_numpy(offsets_host).to("cuda")
    max_len = int(w.lengths.max())
    rows = w.n if w.op == "softmax" else w.b
    schedules = ["auto"] + list(program.schedules)
    reference = scale = None
    for select in schedules:
        out = cuda.full((rows, w.d), -64.0, dtype=values.dtype, device="cuda")
        report = program.run(values, offsets, out, select=select, max_len=max_len)
        cuda.cuda.synchronize()
        actual = host_rows(out)
        if w.op == "softmax":
            dc.check_softmax(actual, fetcher(values)(0, w.n), offsets_host, dtype=w.dtype)
            continue
        if reference is None:
            kinds = (w.op, "abssum") if w.op == "sum" else (w.op,)
            parts = dc.segment_partials(fetcher(values), w.n, w.d, offsets_host, np.arange(w.b), kinds=kinds,
                                        dtype=w.dtype)
            reference, scale = parts[0], (parts[1] if w.op == "sum" else None)
        lengths = np.diff(offsets_host.astype(np.int64))
        native.check(actual, w.op, w.dtype, np.concatenate([[0], np.cumsum(lengths)]), reference, scale)
        assert report.selected in program.schedules
    if name == "c2_max":
        assert np.sum(w.lengths == 0) == 2000  # the -inf identity is exercised


def test_c5_tenth_takes_the_claim_counter_path(cuda):
    """bf16 D=256 Zipf sum with three 5M-row segments: the default schedule
    (row-balanced) claims virtual CTAs from the counter; every output row
    is checked (the giant segments chunk by chunk)."""
    from ragged import workloads
    w = workloads.make("c5", scale=0.1)
    values = workloads.device_values(w, (0, w.n), cuda.device("cuda", 0))
    offsets_host = w.offsets()
    program = _program(w.op, w.dtype, w.d, w.index)
    out = cuda.full((w.b, w.d), -64.0, dtype=values.dtype, device="cuda")
    report = program.run(values, cuda.from_numpy(offsets_host).to("cuda"), out, max_len=int(w.lengths.max()))
    cuda.cuda.synchronize()
    assert report.selected == "rowbalanced"
    assert _claims(report), f"expected the claim-counter path: {report.kernel_names} {report.grids}"
    assert int(w.lengths.max()) >= 5_000_000
    dc.check_reduction(host_rows(out), fetcher(values), w.n, offsets_host, np.arange(w.b), op="sum", dtype="bf16")


@pytest.mark.parametrize("op", ["sum", "max"])
@pytest.mark.parametrize("d", [4, 8])
def test_forty_million_row_segment_chains_thousands_of_virtual_ctas(cuda, op, d):
    """64M rows with one 40M-row segment between short ones.  f32 D=8 (two
    16-byte vectors a row, 128 units per CTA): the path is long enough for
    eight virtual CTAs per resident CTA, so the segment's fix-up chain
    crosses thousands of them.  f32 D=4 (one 16-byte packet a row): the
    packed kernel's single wave, the chain crossing most of its CTAs."""
    rng = np.random.default_rng(40)
    short = rng.integers(0, 64, size=200_000)
    giant = 40_000_000
    rest = 64_000_000 - giant - int(short.sum())
    lengths = np.concatenate([short[:100_000], [giant], short[100_000:], [rest]]).astype(np.int64)
    offsets_host = np.concatenate([[0], np.cumsum(lengths)]).astype(np.int64)
    n, b = int(offsets_host[-1]), lengths.size
    g = cuda.Generator(device="cuda")
    g.manual_seed(4040)
    values = cuda.empty((n, d), dtype=cuda.float32, device="cuda").normal_(generator=g)
    if op == "max":
        values[cuda.rand((n, d), generator=g, device="cuda") < 1e-7] = float("nan")
    program = _program(op, "f32", d, "i64")
    out = cuda.full((b, d), -64.0, dtype=cuda.float32, device="cuda")
    report = program.run(values, cuda.from_numpy(offsets_host).to("cuda"), out, select="rowbalanced")
    cuda.cuda.synchronize()
    names = list(report.kernel_names)
    if d == 8:
        assert _claims(report)
        assert report.grids[names.index("rowbalanced_fixup")][0] >= 2000
    else:
        assert "rowbalanced_packed" in names
    dc.check_reduction(host_rows(out), fetcher(values), n, offsets_host, np.arange(b), op=op, dtype="f32")
