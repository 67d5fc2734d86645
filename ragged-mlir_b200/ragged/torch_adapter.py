"""torch integration: two custom operators over compiled programs, and NJT helpers.

Importing ``ragged`` never imports torch; ``register_torch_ops()`` defines
the operators once per process.  Their names and schemas are the
reference's interface (``ragged_mlir::segment_reduce`` and
``ragged_mlir::segment_softmax``, python/ragged/torch_adapter.py:51-86 of
the reference) so graphs written against the reference keep working.
Behind them:

* ``ProgramTable`` maps a string token (the program's artifact digest) to a
  ``CompiledProgram``.  The operators take only the token, which
  torch.compile keeps as a graph constant, so a traced graph holds no Python
  object and the operator stays opaque.
* ``OpContract`` states the operators' tensor contract once; the fake
  (meta) kernels and the real ones share it and share ``output_shape``, so
  shape inference under torch.compile cannot drift from what the real call
  allocates.
* The operators live in a ``torch.library`` fragment: a CPU and a CUDA
  kernel that hand the call to ``CompiledProgram.run`` (which refuses CPU
  tensors: there is no CPU fallback) and a registered fake for tracing.
"""
from __future__ import annotations

from dataclasses import dataclass
import threading
from typing import Any

from .errors import ValidationError
from .runtime import CompiledProgram, _torch

MODES = ("validated", "checked")
REDUCTIONS = ("sum", "max")
SCHEMAS = {
    "segment_reduce": 'segment_reduce(Tensor values, Tensor offsets, str kind, str program, '
                      'str mode="validated") -> Tensor',
    "segment_softmax": 'segment_softmax(Tensor values, Tensor offsets, str program, str mode="validated", '
                       'Tensor? mask=None) -> Tensor',
}


class ProgramTable:
    """Process-wide token -> program map behind the custom operators."""

    def __init__(self):
        self._lock = threading.Lock()
        self._programs: dict[str, CompiledProgram] = {}

    def enter(self, program) -> str:
        if program.spec.alias != "none":
            raise ValidationError("functional custom ops require an out-of-place specialization")
        token = program.artifact.key.digest
        with self._lock:
            self._programs[token] = program
        return token

    def lookup(self, token: str, op: str):
        with self._lock:
            program = self._programs.get(token)
        if program is None:
            raise ValidationError("compiled program token is not registered in this process")
        if program.spec.op != op:
            raise ValidationError("custom op does not match compiled program semantics")
        return program


_table = ProgramTable()
_operators: dict[str, Any] = {}
_define_lock = threading.Lock()
_library = None  # the torch.library fragment; kept alive with the operators


def register_program(program) -> str:
    """Enter ``program`` in the operators' table; returns its token."""
    return _table.enter(program)


@dataclass(frozen=True)
class OpContract:
    """The operators' tensor contract (the reference's docs/abi.md and
    docs/mask-abi.md), checked on fake tensors during tracing; the real
    call's CompiledProgram.run checks the same rules on device tensors."""

    torch: Any

    def mode(self, mode: str) -> None:
        if mode not in MODES:
            raise ValidationError("mode must be validated or checked")

    def kind(self, kind: str) -> None:
        if kind not in REDUCTIONS:
            raise ValidationError("segment_reduce kind must be sum or max")

    def inputs(self, values, offsets) -> None:
        torch = self.torch
        if values.ndim != 2 or offsets.ndim != 1:
            raise ValidationError("expected values[N,D] and offsets[B+1]")
        torch._check(offsets.shape[0] >= 1)
        torch._check(values.shape[1] >= 1)
        torch._check(values.shape[1] <= 1024)
        if values.dtype not in (torch.float32, torch.bfloat16):
            raise ValidationError("values must be f32 or bf16")
        if offsets.dtype not in (torch.int32, torch.int64):
            raise ValidationError("offsets must be i32 or i64")
        if not (values.is_contiguous() and offsets.is_contiguous()):
            raise ValidationError("values and offsets must be contiguous")
        if values.device != offsets.device:
            raise ValidationError("values and offsets must use the same device")

    def mask(self, values, mask) -> None:
        if mask is None:
            return
        if mask.dtype != self.torch.float32:
            raise ValidationError("mask must be f32")
        if tuple(mask.shape) != tuple(values.shape):
            raise ValidationError("mask must have exactly values shape [N,D]; broadcasting is unsupported")
        if not mask.is_contiguous():
            raise ValidationError("mask must be contiguous")
        if mask.device != values.device:
            raise ValidationError("mask must use the values device")
        if mask.requires_grad:
            raise ValidationError("autograd is outside the supported forward-only contract")


def output_shape(op: str, values, offsets) -> tuple:
    """[B, D] for sum and max, [N, D] for softmax."""
    rows = values.shape[0] if op == "softmax" else offsets.shape[0] - 1
    return (rows, values.shape[1])


def _mask_presence(program, mask) -> None:
    if program.spec.mask != (mask is not None):
        raise ValidationError("mask presence must match the compiled specialization")


def _call(values, offsets, token: str, op: str, mode: str, mask=None):
    """The real kernel of both operators: look the program up, allocate the
    output, run it on the current stream."""
    if mode not in MODES:
        raise ValidationError("mode must be validated or checked")
    program = _table.lookup(token, op)
    _mask_presence(program, mask)
    output = values.new_empty(output_shape(op, values, offsets))
    options = {"mode": mode} if mask is None else {"mode": mode, "mask": mask}
    program.run(values, offsets, output, **options)
    return output


def register_torch_ops() -> dict[str, Any]:
    """Define ``ragged_mlir::segment_reduce`` / ``segment_softmax`` (once);
    returns {"segment_reduce": op, "segment_softmax": op}."""
    global _library
    with _define_lock:
        if _operators:
            return dict(_operators)
        torch = _torch()
        contract = OpContract(torch)
        library = torch.library.Library("ragged_mlir", "FRAGMENT")
        for schema in SCHEMAS.values():
            library.define(schema)

        def reduce_kernel(values, offsets, kind, program, mode="validated"):
            contract.kind(kind)
            return _call(values, offsets, program, kind, mode)

        def softmax_kernel(values, offsets, program, mode="validated", mask=None):
            return _call(values, offsets, program, "softmax", mode, mask)

        for key in ("CPU", "CUDA"):
            library.impl("segment_reduce", reduce_kernel, key)
            library.impl("segment_softmax", softmax_kernel, key)

        @torch.library.register_fake("ragged_mlir::segment_reduce", lib=library)
        def reduce_fake(values, offsets, kind, program, mode="validated"):
            contract.mode(mode)
            contract.inputs(values, offsets)
            contract.kind(kind)
            return values.new_empty(output_shape(kind, values, offsets))

        @torch.library.register_fake("ragged_mlir::segment_softmax", lib=library)
        def softmax_fake(values, offsets, program, mode="validated", mask=None):
            contract.mode(mode)
            contract.inputs(values, offsets)
            contract.mask(values, mask)
            return values.new_empty(output_shape("softmax", values, offsets))

        _library = library
        namespace = torch.ops.ragged_mlir
        _operators.update(segment_reduce=namespace.segment_reduce, segment_softmax=namespace.segment_softmax)
        return dict(_operators)


def segment_reduce(values, offsets, kind: str, *, program: CompiledProgram, mode: str = "validated"):
    """Segmented sum or max of ``program`` through the custom operator."""
    return register_torch_ops()["segment_reduce"](values, offsets, kind, register_program(program), mode)


def segment_softmax(values, offsets, *, program: CompiledProgram, mode: str = "validated", mask=None):
    """Segmented softmax of ``program`` through the custom operator."""
    _mask_presence(program, mask)
    return register_torch_ops()["segment_softmax"](values, offsets, register_program(program), mode, mask)


def bind(program: CompiledProgram, *, mode: str = "validated"):
    """A callable ``f(values, offsets[, mask])`` that only invokes the opaque
    operator with this program's token, so torch.compile can capture it in a
    full graph.  The program is registered here, once."""
    if mode not in MODES:
        raise ValidationError("mode must be validated or checked")
    operators = register_torch_ops()
    token = register_program(program)
    if program.spec.op != "softmax":
        reduce_op, kind = operators["segment_reduce"], program.spec.op
        return lambda values, offsets: reduce_op(values, offsets, kind, token, mode)
    softmax_op = operators["segment_softmax"]

    def softmax(values, offsets, mask=None):
        _mask_presence(program, mask)
        return softmax_op(values, offsets, token, mode, mask)

    return softmax


def jagged_components(nt):
    """(values[N, D], offsets[B+1]) of a contiguous ``torch.jagged`` nested
    tensor of shape [B, jagged, D], without copies."""
    torch = _torch()
    if not getattr(nt, "is_nested", False) or nt.layout != torch.jagged:
        raise ValidationError("expected a torch.jagged nested tensor")
    if nt.dim() != 3:
        raise ValidationError("expected NJT shape [B, jagged, D]")
    if nt.lengths() is not None:
        raise ValidationError("NJT with explicit lengths/holes is outside the contiguous offsets contract")
    if nt._ragged_idx != 1:
        raise ValidationError("only the first non-batch NJT dimension may be ragged")
    values, offsets = nt.values(), nt.offsets()
    if values.ndim != 2 or not (values.is_contiguous() and offsets.is_contiguous()):
        raise ValidationError("NJT values[N,D] and offsets must be contiguous")
    return values, offsets


def njt_reduce(nt, kind: str, *, program: CompiledProgram, mode: str = "validated"):
    """Segmented sum or max over the ragged dimension of an NJT: [B, D]."""
    values, offsets = jagged_components(nt)
    return segment_reduce(values, offsets, kind, program=program, mode=mode)


def njt_softmax(nt, *, program: CompiledProgram, mode: str = "validated", mask=None):
    """Softmax over the ragged dimension of an NJT, returned as an NJT on the
    same offsets."""
    values, offsets = jagged_components(nt)
    output = segment_softmax(values, offsets, program=program, mode=mode, mask=mask)
    return _torch().nested.nested_tensor_from_jagged(output, offsets=offsets)
