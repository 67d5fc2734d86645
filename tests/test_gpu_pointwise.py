"""The input transform on the GPU: ProgramSpec(scale=...) for every op and
the additive f32 softmax mask (rg_run_pointwise), on every schedule, against
the oracle's masked logits.  Softmax on the classified schedule with staged
rows applies the transform as it loads (fused); every other call goes
through materialised f32 logits, as does every call of a program compiled
with Optimizations(pointwise_fusion=False).  Restates the reference's test/gpu/test_mask.py:
all schedules and widths, f32 mask cancellation, separate roundings,
non-finite and fully masked columns, in place and checked calls, mask
aliasing rules and invalid masks (output untouched), the custom op.
"""
from __future__ import annotations

import functools

import numpy as np
import pytest

from helpers import _cache_dir, check, make_lengths, offsets_of, prepared
from oracle import reference_port as rp

pytestmark = pytest.mark.gpu

SCHEDULES = ("naive", "classified", "rowbalanced")


@functools.lru_cache(maxsize=128)
def pw_program(op, dtype, d, index="i64", mask=False, scale=1.0, inplace=False, fusion=True):
    from ragged import ArtifactCache, Compiler, Optimizations, ProgramSpec
    spec = ProgramSpec(op, dtype, d, index, mask=mask, scale=scale, alias="inplace" if inplace else "none",
                       optimizations=Optimizations(pointwise_fusion=fusion))
    return Compiler().compile(spec, ArtifactCache(_cache_dir(), max_specializations=4096))


def fused_expected(op, dtype, d, select, mask_ptr, inplace_alias=False, fusion=True):
    """Whether rg_run_pointwise takes a fused route for this call: softmax on
    the row-balanced schedule (mask rows aligned to the vector width), or on
    the classified schedule with staged rows and no mask."""
    if not fusion or op != "softmax" or inplace_alias:
        return False
    element = 2 if dtype == "bf16" else 4
    vec = 1
    while 2 * vec * element <= 16 and d % (2 * vec) == 0:
        vec *= 2
    if select == "rowbalanced":
        return mask_ptr is None or mask_ptr % (4 * vec) == 0
    staged = (dtype == "bf16" and d % 8 == 0 and d <= 256) or (dtype == "f32" and d % 4 == 0 and d <= 128)
    return select == "classified" and staged and mask_ptr is None


def run_masked(torch, op, dtype, values, offsets, mask, scale, select, *, inplace=False, mode="validated",
               fusion=True):
    """(result as float64, report); guards around out and mask."""
    d = values.shape[1]
    tdtype = torch.float32 if dtype == "f32" else torch.bfloat16
    index = "i32" if offsets.dtype == np.int32 else "i64"
    rows = values.shape[0] if op == "softmax" else offsets.size - 1
    guard = torch.full((max(rows, values.shape[0]) + 2, d), -64.0, device="cuda", dtype=tdtype)
    device_values = torch.from_numpy(np.ascontiguousarray(values, dtype=np.float32)).to("cuda").to(tdtype)
    if inplace:
        guard[1:1 + values.shape[0]] = device_values
        device_values = guard[1:1 + values.shape[0]]
        out = device_values
    else:
        out = guard[1:1 + rows]
    device_mask = None
    if mask is not None:
        mask_guard = torch.full((values.shape[0] + 2, d), 91.0, device="cuda")
        device_mask = mask_guard[1:-1]
        device_mask.copy_(torch.from_numpy(mask))
    prog = pw_program(op, dtype, d, index, mask is not None, scale, inplace, fusion)
    report = prog.run(device_values, torch.from_numpy(offsets).to("cuda"), out, mask=device_mask, select=select,
                      mode=mode)
    torch.cuda.synchronize()
    assert torch.all(guard[0] == -64).item() and torch.all(guard[1 + (values.shape[0] if inplace else rows):] == -64).item()
    if mask is not None:
        assert torch.all(mask_guard[0] == 91).item() and torch.all(mask_guard[-1] == 91).item()
        np.testing.assert_array_equal(device_mask.cpu().numpy(), mask)
    names = report.kernel_names
    fused = fused_expected(op, dtype, d, report.selected, None if device_mask is None else device_mask.data_ptr(),
                           inplace_alias=False, fusion=fusion)
    assert report.pointwise_materialized == (not fused)
    if fused:
        assert "pointwise_logits" not in names
    else:
        assert names[2 if mode == "checked" else 0] == "pointwise_logits"
        assert (names[-1] == "pointwise_cast") == (dtype == "bf16")
    return out.float().cpu().numpy().astype(np.float64), report


def check_masked(actual, values, offsets, mask, scale, op, dtype):
    logits = rp.masked_logits(values, mask, scale=scale)
    with np.errstate(all="ignore"):
        reference = rp.REFERENCES[op](logits, offsets)
    check(actual, logits, offsets, op, dtype, reference)


@pytest.mark.parametrize("select", SCHEDULES)
@pytest.mark.parametrize("dtype", ["f32", "bf16"])
@pytest.mark.parametrize("d", [1, 7, 128, 1024])
@pytest.mark.parametrize("index", ["i32", "i64"])
def test_mask_and_scale_every_schedule(cuda, select, dtype, d, index):
    lengths = np.array([4097, 0, 1, 33, 300, 32] if d < 1024 else [700, 0, 1, 33, 64], dtype=np.int64)
    offsets = offsets_of(lengths, index)
    rng = np.random.default_rng(951)
    values = prepared(rng.normal(size=(int(offsets[-1]), d)), dtype)
    mask = rng.uniform(-3, 3, size=values.shape).astype(np.float32)
    actual, report = run_masked(cuda, "softmax", dtype, values, offsets, mask, 0.75, select)
    assert report.selected == select
    check_masked(actual, values, offsets, mask, 0.75, "softmax", dtype)


@pytest.mark.parametrize("select", SCHEDULES)
def test_golden_masked_cases(cuda, masked_golden, select):
    for name, case in masked_golden.items():
        offsets = case["offsets"]
        actual, _ = run_masked(cuda, "softmax", case["dtype"], case["values"], offsets, case["mask"], case["scale"],
                               select)
        with np.errstate(all="ignore"):
            rp.assert_matches(actual, case["logits"], offsets, operation="softmax", input_dtype=case["dtype"],
                              reference=case["softmax"])
            rp.check_strict(actual, case["logits"], offsets, operation="softmax", input_dtype=case["dtype"],
                            reference=case["softmax"])


@pytest.mark.parametrize("op", ["sum", "max"])
@pytest.mark.parametrize("select", SCHEDULES)
@pytest.mark.parametrize("dtype,d", [("f32", 1), ("f32", 64), ("bf16", 2), ("bf16", 256)])
def test_scale_for_reductions(cuda, op, select, dtype, d):
    lengths = make_lengths("long_tail", 200, 30_000, seed=81)
    lengths[::17] = 0
    offsets = offsets_of(lengths)
    values = prepared(np.random.default_rng(82).normal(size=(int(offsets[-1]), d)), dtype)
    values[5, 0] = np.nan
    actual, _ = run_masked(cuda, op, dtype, values, offsets, None, -1.5, select)
    check_masked(actual, values, offsets, None, -1.5, op, dtype)


@pytest.mark.parametrize("select", SCHEDULES)
@pytest.mark.parametrize("dtype", ["f32", "bf16"])
def test_inplace_and_checked_with_mask(cuda, select, dtype):
    lengths = np.array([4097, 0, 1, 33, 8193, 32], dtype=np.int64)
    offsets = offsets_of(lengths)
    rng = np.random.default_rng(83)
    values = prepared(rng.normal(size=(int(offsets[-1]), 7)), dtype)
    mask = rng.uniform(-3, 3, size=values.shape).astype(np.float32)
    actual, report = run_masked(cuda, "softmax", dtype, values, offsets, mask, 0.5, select, inplace=True,
                                mode="checked")
    assert report.mode == "checked"
    check_masked(actual, values, offsets, mask, 0.5, "softmax", dtype)


def test_readonly_mask_may_alias_values(cuda):
    torch = cuda
    values = torch.randn((40, 8), device="cuda")
    offsets = torch.tensor([0, 15, 40], device="cuda")
    out = torch.empty_like(values)
    pw_program("softmax", "f32", 8, mask=True).run(values, offsets, out, mask=values)
    torch.cuda.synchronize()
    host = values.cpu().numpy()
    check_masked(out.cpu().numpy().astype(np.float64), host, np.array([0, 15, 40]), host, 1.0, "softmax", "f32")


@pytest.mark.parametrize("overlap", ["out", "partial-out", "inplace-values", "offsets"])
def test_disallowed_mask_aliases_are_rejected_before_writes(cuda, overlap):
    torch = cuda
    from ragged import ValidationError
    base = torch.zeros((21, 8), device="cuda")
    values = torch.randn((20, 8), device="cuda")
    offsets = torch.tensor([0, 10, 20], device="cuda")
    out = base[:20]
    inplace = overlap == "inplace-values"
    mask = {"out": out, "partial-out": base[1:21], "inplace-values": values}.get(overlap)
    if overlap == "offsets":  # offsets stored inside the mask's bytes
        storage = torch.zeros((20 * 8,), dtype=torch.float32, device="cuda")
        mask = storage.view(20, 8)
        offsets = storage[:6].view(torch.int64)
        offsets.copy_(torch.tensor([0, 10, 20], device="cuda"))
    before = (values if inplace else out).clone()
    prog = pw_program("softmax", "f32", 8, mask=True, inplace=inplace)
    with pytest.raises(ValidationError, match="mask must not overlap"):
        prog.run(values, offsets, values if inplace else out, mask=mask)
    torch.cuda.synchronize()
    assert torch.equal(values if inplace else out, before)


@pytest.mark.parametrize("bad", ["missing", "broadcast", "rank", "bf16", "f64", "noncontiguous", "cpu", "unexpected"])
def test_invalid_mask_contract_preserves_output(cuda, bad):
    torch = cuda
    from ragged import RuntimeUnavailable, ValidationError
    values = torch.randn((12, 4), device="cuda")
    offsets = torch.tensor([0, 5, 12], device="cuda")
    out = torch.full_like(values, -64.0)
    mask = torch.zeros_like(values)
    prog = pw_program("softmax", "f32", 4, mask=True)
    if bad == "missing":
        mask = None
    elif bad == "broadcast":
        mask = torch.zeros((1, 4), device="cuda")
    elif bad == "rank":
        mask = torch.zeros((48,), device="cuda")
    elif bad == "bf16":
        mask = mask.to(torch.bfloat16)
    elif bad == "f64":
        mask = mask.double()
    elif bad == "noncontiguous":
        mask = torch.zeros((4, 12), device="cuda").t()
    elif bad == "cpu":
        mask = mask.cpu()
    elif bad == "unexpected":
        prog = pw_program("softmax", "f32", 4)
    with pytest.raises((ValidationError, RuntimeUnavailable)):
        prog.run(values, offsets, out, mask=mask)
    torch.cuda.synchronize()
    assert torch.all(out == -64).item()


@pytest.mark.parametrize("mode", ["validated", "checked"])
def test_mask_through_the_custom_op(cuda, mode):
    torch = cuda
    from ragged import torch_adapter
    values = torch.randn((30, 8), device="cuda")
    offsets = torch.tensor([0, 7, 7, 30], device="cuda")
    mask = torch.where(torch.rand((30, 8), device="cuda") < 0.3, float("-inf"), 0.0).to(torch.float32)
    execute = torch_adapter.bind(pw_program("softmax", "f32", 8, mask=True), mode=mode)
    out = torch.compile(lambda v, o, m: execute(v, o, m), backend="aot_eager", fullgraph=True)(values, offsets, mask)
    torch.cuda.synchronize()
    check_masked(out.cpu().numpy().astype(np.float64), values.cpu().numpy(), np.array([0, 7, 7, 30]),
                 mask.cpu().numpy(), 1.0, "softmax", "f32")


@pytest.mark.parametrize("dtype,d", [("bf16", 128), ("f32", 64), ("bf16", 256)])
def test_fused_and_materialised_routes_both_match(cuda, dtype, d):
    """Masked, scaled softmax on the row-balanced and classified schedules,
    segments of every class (warp, CTA, split normalised in the worker and
    split left to the normalise kernel): each fused route and the
    materialised one match the oracle's masked logits."""
    lengths = np.array([3, 0, 31, 200, 5000, 17, 16000, 1, 90], dtype=np.int64)
    offsets = offsets_of(lengths)
    rng = np.random.default_rng(1909)
    values = prepared(rng.normal(scale=2.0, size=(int(offsets[-1]), d)), dtype)
    mask = np.where(rng.random(values.shape) < 0.2, -np.inf, rng.uniform(-4, 4, size=values.shape)).astype(np.float32)
    mask[offsets[1]:offsets[2] + 40, 3] = -np.inf  # a fully masked column inside a segment
    for select in ("rowbalanced", "classified"):
        for fusion in (True, False):
            actual, report = run_masked(cuda, "softmax", dtype, values, offsets, mask, 0.125, select, fusion=fusion)
            assert report.pointwise_materialized == (not fusion or select == "classified")
            check_masked(actual, values, offsets, mask, 0.125, "softmax", dtype)
    # Scale without a mask: the classified worker scales staged rows itself
    # (a positive scale keeps the packed maximum, a negative one does not).
    values[7, :4] = [np.inf, -np.inf, np.nan, -np.inf]
    for scale in (-0.5, 0.5, 3.0):
        actual, report = run_masked(cuda, "softmax", dtype, values, offsets, None, scale, "classified")
        assert not report.pointwise_materialized
        check_masked(actual, values, offsets, None, scale, "softmax", dtype)
