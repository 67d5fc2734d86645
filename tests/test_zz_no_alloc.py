"""rg_run_noalloc: the row-balanced sum / max for callers that cannot allocate.

Some callers may not allocate device memory at all -- a host that hands its
whole memory budget to its own pool at start-up, or a plugin callback that
is not allowed to allocate -- so rg_run_noalloc keeps its scratch in a
static per-GPU array instead of a caller workspace.  This test calls it
through the C ABI twice in a row (different problems, so the second call
runs on whatever the first left in the shared array) and checks each output
against the existing entry point (rg_run, row-balanced schedule) within the
tolerance the other parity tests use, plus the CPU oracle.  The file sorts
last so that a run stopping at the first failure has run every other test.
"""
from __future__ import annotations

import ctypes

import numpy as np
import pytest

from helpers import check, make_lengths, offsets_of, prepared
from oracle import reference_port as rp

pytestmark = pytest.mark.gpu


def _case(op, dtype, d, index, distribution, seed):
    lengths = make_lengths(distribution, 300, 60_000 if d <= 16 else 12_000, seed=seed)
    lengths[7] = 0
    offsets = offsets_of(lengths, index)
    values = prepared(np.random.default_rng(seed + 1).normal(size=(int(offsets[-1]), d)), dtype)
    return values, offsets


def _device(torch, values, offsets, dtype):
    tdtype = torch.float32 if dtype == "f32" else torch.bfloat16
    return (torch.from_numpy(np.ascontiguousarray(values, dtype=np.float32)).to("cuda").to(tdtype),
            torch.from_numpy(offsets).to("cuda"))


@pytest.mark.parametrize("op,dtype,d,index,distribution", [
    ("sum", "bf16", 256, "i64", "long_tail"),
    ("max", "f32", 128, "i32", "bimodal"),
    ("sum", "f32", 1, "i32", "uniform"),
    ("max", "bf16", 1024, "i64", "burst"),
])
def test_noalloc_matches_rg_run_twice(cuda, op, dtype, d, index, distribution):
    torch = cuda
    from ragged import _native
    lib = _native.library()
    stream = torch.cuda.current_stream().cuda_stream
    for call, seed in enumerate((101, 202)):
        values, offsets = _case(op, dtype, d, index, distribution, seed)
        dv, do = _device(torch, values, offsets, dtype)
        n, b = dv.shape[0], do.numel() - 1
        ops, dts, idx = _native.OPS[op], _native.DTYPES[dtype], _native.INDEX[index]
        # The existing entry point, with a workspace from the caching allocator.
        ws = _native.workspace_bytes(op, dtype, index, d, n, b, "rowbalanced", None)
        scratch = torch.empty(max(ws, 1), dtype=torch.uint8, device="cuda")
        expected = torch.full((b, d), float("nan"), dtype=dv.dtype, device="cuda")
        status = lib.rg_run(ops, dts, idx, d, n, b, dv.data_ptr(), do.data_ptr(), expected.data_ptr(),
                            scratch.data_ptr(), ws, _native.SCHEDULES["rowbalanced"], -1, 0, stream, None)
        assert status == 0, lib.rg_last_error()
        actual = torch.full((b, d), float("nan"), dtype=dv.dtype, device="cuda")
        status = lib.rg_run_noalloc(ops, dts, idx, d, n, b, dv.data_ptr(), do.data_ptr(), actual.data_ptr(), 0,
                                    stream)
        assert status == 0, lib.rg_last_error()
        torch.cuda.synchronize()
        got = actual.float().cpu().numpy().astype(np.float64)
        ref_entry = expected.float().cpu().numpy().astype(np.float64)
        with np.errstate(all="ignore"):
            # Within the tolerance of the parity tests, against rg_run's output ...
            rp.check_strict(got, values, offsets, operation=op, input_dtype=dtype, reference=ref_entry)
            # ... and against the CPU oracle.
            check(got, values, offsets, op, dtype)


def test_noalloc_rejects_softmax_and_bad_arguments(cuda):
    from ragged import _native
    lib = _native.library()
    assert lib.rg_run_noalloc(2, 0, 1, 8, 0, 1, None, None, None, 0, None) == _native.RG_ERR_INVALID_ARGUMENT
    torch = cuda
    values = torch.zeros((4, 8), device="cuda")
    offsets = torch.tensor([0, 4], device="cuda")
    out = torch.empty((4, 8), device="cuda")
    status = lib.rg_run_noalloc(2, 0, 1, 8, 4, 1, values.data_ptr(), offsets.data_ptr(), out.data_ptr(), 0, None)
    assert status == _native.RG_ERR_UNSUPPORTED
