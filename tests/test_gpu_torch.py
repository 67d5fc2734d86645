"""PyTorch integration on the GPU: the ``ragged_mlir`` custom ops, NJT
inputs, a torch.compile full graph around a bound program, and CUDA-graph
capture and replay of every schedule (the reference's
test/gpu/test_scheduling.py:151-172 and torch_adapter.py:51-180).  Results
are checked against the CPU oracle with both tolerance contracts.
"""
from __future__ import annotations

import numpy as np
import pytest

from helpers import check, make_lengths, offsets_of, prepared, program

pytestmark = pytest.mark.gpu


def _inputs(torch, dtype, d, segments=300, rows=20_000, seed=41):
    lengths = make_lengths("long_tail", segments, rows, seed=seed)
    lengths[::37] = 0
    offsets = offsets_of(lengths)
    values = prepared(np.random.default_rng(seed).normal(size=(int(offsets[-1]), d)), dtype)
    tdtype = torch.float32 if dtype == "f32" else torch.bfloat16
    return values, offsets, torch.from_numpy(values).to("cuda").to(tdtype), torch.from_numpy(offsets).to("cuda")


def _host(tensor):
    return tensor.float().cpu().numpy().astype(np.float64)


@pytest.mark.parametrize("op", ["sum", "max", "softmax"])
@pytest.mark.parametrize("dtype", ["f32", "bf16"])
def test_custom_ops_match_the_oracle(cuda, op, dtype):
    torch = cuda
    from ragged import torch_adapter
    values, offsets, dv, do = _inputs(torch, dtype, 64)
    prog = program(op, dtype, 64, "i64")
    if op == "softmax":
        out = torch_adapter.segment_softmax(dv, do, program=prog)
    else:
        out = torch_adapter.segment_reduce(dv, do, op, program=prog)
    torch.cuda.synchronize()
    check(_host(out), values, offsets, op, dtype)


@pytest.mark.parametrize("op", ["sum", "max", "softmax"])
def test_njt_inputs(cuda, op):
    torch = cuda
    from ragged import torch_adapter
    values, offsets, dv, do = _inputs(torch, "f32", 32, seed=42)
    nt = torch.nested.nested_tensor_from_jagged(dv, do)
    prog = program(op, "f32", 32, "i64")
    if op == "softmax":
        out = torch_adapter.njt_softmax(nt, program=prog)
        assert out.is_nested and out.offsets().data_ptr() == do.data_ptr()
        out = out.values()
    else:
        out = torch_adapter.njt_reduce(nt, op, program=prog)
    torch.cuda.synchronize()
    check(_host(out), values, offsets, op, "f32")


@pytest.mark.parametrize("op", ["sum", "max", "softmax"])
def test_bound_program_inside_a_compiled_graph(cuda, op):
    """torch.compile(fullgraph=True) around a bound program: the op stays
    opaque in the graph and runs libragged_b200 on the traced producer's
    output (doubling is exact in f32, so the oracle sees the same input)."""
    torch = cuda
    from ragged import torch_adapter
    values, offsets, dv, do = _inputs(torch, "f32", 16, seed=43)
    execute = torch_adapter.bind(program(op, "f32", 16, "i64"))

    def model(v, o):
        return execute(v * 2.0, o)

    out = torch.compile(model, backend="aot_eager", fullgraph=True)(dv, do)
    torch.cuda.synchronize()
    check(_host(out), values * 2.0, offsets, op, "f32")


@pytest.mark.parametrize("op,schedule", [(op, s) for op in ("sum", "max", "softmax")
                                         for s in ("naive", "classified", "rowbalanced")])
def test_cuda_graph_capture_and_replay(cuda, op, schedule):
    """Capture one call per schedule, then replay it on new values written
    into the captured input buffer: counters and scratch are reset inside the
    graph, so every replay is a complete, correct call."""
    torch = cuda
    rng = np.random.default_rng(44)
    lengths = make_lengths("bimodal", 400, 60_000, seed=44)
    offsets = offsets_of(lengths)
    n, d = int(offsets[-1]), 64
    prog = program(op, "f32", d, "i64")
    dv = torch.empty((n, d), device="cuda")
    do = torch.from_numpy(offsets).to("cuda")
    rows = n if op == "softmax" else len(lengths)
    out = torch.empty((rows, d), device="cuda")
    first = rng.normal(size=(n, d)).astype(np.float32)
    dv.copy_(torch.from_numpy(first))
    prog.run(dv, do, out, select=schedule)  # warm-up outside the capture
    torch.cuda.synchronize()
    capture = torch.cuda.Stream()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph, stream=capture):
        report = prog.run(dv, do, out, select=schedule)
    assert report.selected == schedule
    for replay in range(3):
        values = rng.normal(size=(n, d)).astype(np.float32)
        dv.copy_(torch.from_numpy(values))
        out.fill_(-64.0)
        graph.replay()
        torch.cuda.synchronize()
        check(_host(out), values.astype(np.float64), offsets, op, "f32")
    del graph
