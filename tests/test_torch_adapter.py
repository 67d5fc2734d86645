"""PyTorch integration on the host (no GPU): the ``ragged_mlir`` custom ops'
fake (meta) implementations, full-graph torch.compile capture of the opaque
op, NJT component extraction and mode routing.  Restates the reference's
test/python/test_torch_adapter.py; no CUDA kernel runs here.
"""
from __future__ import annotations

from types import SimpleNamespace

import pytest

torch = pytest.importorskip("torch")


@pytest.fixture(scope="module")
def ops():
    from ragged.torch_adapter import register_torch_ops
    return register_torch_ops()


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
@pytest.mark.parametrize("offset_dtype", [torch.int32, torch.int64])
@pytest.mark.parametrize("kind", ["sum", "max"])
def test_meta_reduce_shape(ops, dtype, offset_dtype, kind):
    values = torch.empty((17, 13), dtype=dtype, device="meta")
    offsets = torch.empty((5,), dtype=offset_dtype, device="meta")
    output = ops["segment_reduce"](values, offsets, kind, "shape-only-no-program")
    assert output.shape == (4, 13) and output.dtype == dtype and output.device.type == "meta"


def test_meta_softmax_shape_and_idempotent_registration(ops):
    from ragged.torch_adapter import register_torch_ops
    values = torch.empty((0, 1024), dtype=torch.bfloat16, device="meta")
    offsets = torch.empty((1,), dtype=torch.int64, device="meta")
    assert ops["segment_softmax"](values, offsets, "shape-only-no-program").shape == (0, 1024)
    assert register_torch_ops() == ops


def _capture(function, *args):
    graphs = []

    def backend(graph, _):
        graphs.append(graph)
        return graph.forward

    output = torch.compile(function, backend=backend, fullgraph=True)(*args)
    assert len(graphs) == 1
    return output, graphs[0]


def test_fullgraph_capture_keeps_the_op_opaque(ops):
    def function(values, offsets):
        return torch.ops.ragged_mlir.segment_reduce(values, offsets, "sum", "shape-only-no-program")

    output, graph = _capture(function, torch.empty((17, 13), device="meta"),
                             torch.empty((5,), dtype=torch.int64, device="meta"))
    assert output.shape == (4, 13)
    assert any(node.op == "call_function" and "ragged_mlir.segment_reduce" in str(node.target)
               for node in graph.graph.nodes)


def test_checked_mode_is_a_graph_constant(ops):
    def function(values, offsets):
        return ops["segment_softmax"](values, offsets, "shape-only-no-program", "checked")

    output, graph = _capture(function, torch.empty((6, 4), device="meta"),
                             torch.empty((3,), dtype=torch.int64, device="meta"))
    assert output.shape == (6, 4)
    nodes = [node for node in graph.graph.nodes if "ragged_mlir.segment_softmax" in str(node.target)]
    assert len(nodes) == 1 and nodes[0].args[3] == "checked"


@pytest.mark.parametrize("kind", ["mean", "min"])
def test_fake_rejects_unsupported_reductions(ops, kind):
    from ragged import ValidationError
    with pytest.raises(ValidationError, match="kind"):
        ops["segment_reduce"](torch.empty((3, 4), device="meta"), torch.empty((3,), dtype=torch.int64, device="meta"),
                              kind, "token")


def test_fake_rejects_unknown_modes(ops):
    from ragged import ValidationError
    with pytest.raises(ValidationError, match="mode"):
        ops["segment_softmax"](torch.empty((6, 4), device="meta"), torch.empty((3,), dtype=torch.int64, device="meta"),
                               "token", "unsafe")


def test_njt_components_are_zero_copy():
    from ragged.torch_adapter import jagged_components
    values, offsets = torch.randn(6, 4), torch.tensor([0, 2, 2, 6])
    got_values, got_offsets = jagged_components(torch.nested.nested_tensor_from_jagged(values, offsets))
    assert got_values.data_ptr() == values.data_ptr() and got_offsets.data_ptr() == offsets.data_ptr()


def test_njt_holes_are_rejected():
    from ragged import ValidationError
    from ragged.torch_adapter import jagged_components
    nt = torch.nested.nested_tensor_from_jagged(torch.randn(6, 4), torch.tensor([0, 3, 6]),
                                                lengths=torch.tensor([2, 1]))
    with pytest.raises(ValidationError, match="holes"):
        jagged_components(nt)


def test_njt_ragged_dimension_must_lead():
    from ragged import ValidationError
    from ragged.torch_adapter import jagged_components
    nt = torch.nested.nested_tensor_from_jagged(torch.randn(4, 6), torch.tensor([0, 2, 6]), jagged_dim=2)
    with pytest.raises(ValidationError, match="first non-batch"):
        jagged_components(nt)


def test_dense_tensor_is_not_an_njt():
    from ragged import ValidationError
    from ragged.torch_adapter import jagged_components
    with pytest.raises(ValidationError, match="torch.jagged"):
        jagged_components(torch.randn(2, 3, 4))


@pytest.mark.parametrize("kind", ["sum", "max", "softmax"])
def test_mode_reaches_the_registered_program(monkeypatch, kind):
    """A stub program records the routed keyword arguments; no GPU work."""
    from ragged import ProgramSpec
    from ragged import torch_adapter
    calls = []
    program = SimpleNamespace(spec=ProgramSpec(kind, feature_dim=4),
                              artifact=SimpleNamespace(key=SimpleNamespace(digest="mode-routing-" + kind)),
                              run=lambda values, offsets, out, **kwargs: calls.append(kwargs))
    monkeypatch.setattr(torch_adapter, "_table", torch_adapter.ProgramTable())
    values, offsets = torch.empty((6, 4)), torch.tensor([0, 2, 6])
    if kind == "softmax":
        output = torch_adapter.segment_softmax(values, offsets, program=program, mode="checked")
    else:
        output = torch_adapter.segment_reduce(values, offsets, kind, program=program, mode="checked")
    assert calls == [{"mode": "checked"}]
    assert output.shape == (6 if kind == "softmax" else 2, 4)


def test_bind_routes_through_the_custom_op(monkeypatch):
    from ragged import ProgramSpec
    from ragged import torch_adapter
    calls = []
    program = SimpleNamespace(spec=ProgramSpec("sum", feature_dim=4),
                              artifact=SimpleNamespace(key=SimpleNamespace(digest="bind-routing")),
                              run=lambda values, offsets, out, **kwargs: calls.append((out.shape, kwargs)))
    monkeypatch.setattr(torch_adapter, "_table", torch_adapter.ProgramTable())
    execute = torch_adapter.bind(program)
    assert execute(torch.empty((6, 4)), torch.tensor([0, 2, 6])).shape == (2, 4)
    assert calls == [((2, 4), {"mode": "validated"})]


def test_in_place_specialisation_cannot_back_a_functional_op():
    from ragged import ProgramSpec, ValidationError
    from ragged import torch_adapter
    program = SimpleNamespace(spec=ProgramSpec("softmax", feature_dim=4, alias="inplace"),
                              artifact=SimpleNamespace(key=SimpleNamespace(digest="inplace")))
    with pytest.raises(ValidationError, match="out-of-place"):
        torch_adapter.register_program(program)


@pytest.mark.parametrize("problem", ["bf16", "rank", "broadcast", "noncontiguous", "device", "grad"])
def test_mask_fake_rejects_unsupported_tensor_contract(ops, problem):
    from ragged import ValidationError
    values = torch.empty((6, 4), dtype=torch.bfloat16, device="meta")
    offsets = torch.empty((3,), dtype=torch.int64, device="meta")
    mask = torch.empty((6, 4), device="meta")
    if problem == "bf16":
        mask = mask.to(torch.bfloat16)
    elif problem == "rank":
        mask = torch.empty((24,), device="meta")
    elif problem == "broadcast":
        mask = torch.empty((1, 4), device="meta")
    elif problem == "noncontiguous":
        mask = torch.empty((4, 6), device="meta").t()
    elif problem == "device":
        mask = torch.empty((6, 4))
    else:
        mask.requires_grad_()
    with pytest.raises((ValidationError, RuntimeError)):
        ops["segment_softmax"](values, offsets, "shape-only-no-program", "validated", mask)


def test_masked_softmax_fullgraph_keeps_the_mask_operand(ops):
    class Operation(torch.nn.Module):
        def forward(self, values, offsets, mask):
            return ops["segment_softmax"](values, offsets, "shape-only-no-program", "checked", mask)

    args = (torch.empty((6, 4), dtype=torch.bfloat16, device="meta"), torch.empty((3,), dtype=torch.int64, device="meta"),
            torch.empty((6, 4), device="meta"))
    output, graph = _capture(Operation(), *args)
    assert output.shape == (6, 4) and output.dtype == torch.bfloat16
    nodes = [node for node in graph.graph.nodes if "ragged_mlir.segment_softmax" in str(node.target)]
    assert len(nodes) == 1 and isinstance(nodes[0].args[-1], torch.fx.Node)


def test_njt_mask_routes_the_dense_mask(monkeypatch):
    from ragged import ProgramSpec, ValidationError
    from ragged import torch_adapter
    calls = []
    program = SimpleNamespace(spec=ProgramSpec("softmax", feature_dim=4, mask=True),
                              artifact=SimpleNamespace(key=SimpleNamespace(digest="njt-mask-routing")),
                              run=lambda values, offsets, out, **kwargs: calls.append(kwargs))
    monkeypatch.setattr(torch_adapter, "_table", torch_adapter.ProgramTable())
    values, offsets, mask = torch.empty((6, 4)), torch.tensor([0, 2, 6]), torch.empty((6, 4))
    out = torch_adapter.njt_softmax(torch.nested.nested_tensor_from_jagged(values, offsets), program=program,
                                    mode="checked", mask=mask)
    assert out.values().shape == values.shape and out.offsets().data_ptr() == offsets.data_ptr()
    assert len(calls) == 1 and calls[0]["mask"] is mask and calls[0]["mode"] == "checked"
    with pytest.raises(ValidationError, match="mask presence"):
        torch_adapter.bind(program)(values, offsets)
