"""Checked mode on the host (no GPU): the status decoder, the oracle's
offsets_status pinned on the reference's known answers, and the order of the
checked call (validation before any scratch allocation or main launch; only
the execution stream is waited on) with fake torch and native layers.

Restates the reference's test/python/test_checked_contract.py and
test/python/test_runtime_checked.py for this build's runtime.
"""
from __future__ import annotations

from contextlib import contextmanager, nullcontext
from dataclasses import dataclass
from math import prod
from types import SimpleNamespace

import pytest

from oracle import reference_port as rp

I64_MAX = 2**63 - 1


def test_conditions_match_the_oracle_order():
    from ragged.validation import CONDITIONS, STATUS_BYTES
    assert CONDITIONS == rp.CHECK_CONDITIONS and STATUS_BYTES == 56


@pytest.mark.parametrize("slot,index", [(0, 0), (1, 5), (2, 0), (2, 5), (3, 5), (4, 0), (4, 4), (5, 4), (6, 0)])
def test_each_slot_keeps_its_index_domain(slot, index):
    from ragged import ValidationError
    from ragged.validation import CONDITIONS, raise_for_status
    status = [I64_MAX] * 7
    status[slot] = index
    with pytest.raises(ValidationError) as caught:
        raise_for_status(status, b=5)
    assert caught.value.errors == {CONDITIONS[slot]: index}
    assert (caught.value.condition, caught.value.index) == (CONDITIONS[slot], index)


def test_every_condition_survives_decoding_in_protocol_order():
    from ragged import ValidationError
    from ragged.validation import CONDITIONS, raise_for_status
    with pytest.raises(ValidationError) as caught:
        raise_for_status([0, 5, 2, 3, 1, 2, 4], b=5)
    assert caught.value.errors == dict(zip(CONDITIONS, [0, 5, 2, 3, 1, 2, 4]))
    assert list(caught.value.errors) == list(CONDITIONS)
    assert caught.value.condition == "first_nonzero" and caught.value.index == 0
    for condition, index in caught.value.errors.items():
        assert f"{condition} at index {index}" in str(caught.value)


@pytest.mark.parametrize("status", [
    [I64_MAX] * 6, [-1] + [I64_MAX] * 6, [I64_MAX, 4] + [I64_MAX] * 5, [1] + [I64_MAX] * 6,
    [I64_MAX] * 2 + [6] + [I64_MAX] * 4, [I64_MAX] * 4 + [5, I64_MAX, I64_MAX], [True] + [I64_MAX] * 6,
    [I64_MAX] * 6 + [2**63], [I64_MAX] * 6 + [1.0], (I64_MAX,) * 7,
])
def test_corrupt_status_is_never_success(status):
    from ragged import ValidationError
    from ragged.validation import raise_for_status
    with pytest.raises(ValidationError):
        raise_for_status(status, b=5)


@pytest.mark.parametrize("slot", [4, 5, 6])
def test_zero_batch_has_no_segment_index(slot):
    from ragged import ValidationError
    from ragged.validation import raise_for_status
    status = [I64_MAX] * 7
    status[slot] = 0
    with pytest.raises(ValidationError, match="domain"):
        raise_for_status(status, b=0)


def test_all_sentinels_mean_success():
    from ragged.validation import raise_for_status
    raise_for_status([I64_MAX] * 7, b=0)
    raise_for_status([I64_MAX] * 7, b=9)


def test_oracle_status_known_answers():
    """The reference test suite's own expected answers for its checked cases
    (test/gpu/test_checked.py:103-178)."""
    assert rp.offsets_status([1, -2, -3, 11, 10, 0, 1, 7, 6], 8, 4, 4) == dict(
        zip(rp.CHECK_CONDITIONS, [0, 8, 1, 3, 0, 5, 6]))
    for lower in (2, 4097):
        offsets = [0, lower - 1, lower - 1 + 8194]
        assert rp.offsets_status(offsets, offsets[-1], lower, 8193) == {"below_min_len": 0, "above_max_len": 1}
    offsets = [2 * i for i in range(4098)]
    n = offsets[-1]
    offsets[130] = offsets[129] + 1
    offsets[1026] = offsets[1025] + 1
    offsets[2051], offsets[3077], offsets[3001] = -1, -2, n + 1
    assert rp.offsets_status(offsets, n, 2, 2) == {"negative": 2051, "above_n": 3001, "nonmonotone": 2050,
                                                   "below_min_len": 129, "above_max_len": 130}
    for bits in (32, 64):
        low, high = -(1 << (bits - 1)), (1 << (bits - 1)) - 1
        assert rp.offsets_status([0, low, high, 0, 8], 8, 0, 8) == {"negative": 1, "above_n": 2, "nonmonotone": 0}
    assert rp.offsets_status([1], 0) == {"first_nonzero": 0, "final_mismatch": 0, "above_n": 0}
    assert rp.offsets_status([0], 2) == {"final_mismatch": 0}
    assert rp.offsets_status([0, 4, 8], 8) == {}


# ---- the checked call's order, with fake torch and native layers ----------

@pytest.fixture
def host(monkeypatch, tmp_path, native_library):
    import ragged.runtime as runtime
    from ragged import ArtifactCache, Compiler, Hints, ProgramSpec
    from ragged import _native

    @dataclass(frozen=True)
    class Device:
        index: int = 0

    device, log = Device(), []
    state = {"status": [I64_MAX] * 7, "synchronized": False}

    class Stream:
        def __init__(self, handle):
            self.device, self.cuda_stream = device, handle

        def synchronize(self):
            log.append(("synchronize", self.cuda_stream))
            state["synchronized"] = True

    producer, consumer = Stream(101), Stream(202)
    current = [producer]

    @contextmanager
    def stream_context(stream):
        previous, current[0] = current[0], stream
        try:
            yield
        finally:
            current[0] = previous

    sizes = {"i64": 8, "f32": 4, "i32": 4, "bf16": 2, "u8": 1}

    class Tensor:
        requires_grad = False
        is_cuda = True

        def __init__(self, shape, dtype, pointer, where=device):
            self.shape, self.dtype, self.pointer, self.device = shape, dtype, pointer, where
            self.ndim = len(shape)
            self.is_cuda = where != "cpu"

        def is_contiguous(self):
            return True

        def numel(self):
            return prod(self.shape)

        def element_size(self):
            return sizes[self.dtype]

        def data_ptr(self):
            return self.pointer

        def stride(self):
            return (self.shape[1], 1) if self.ndim == 2 else (1,)

        def storage_offset(self):
            return 0

        def record_stream(self, stream):
            assert stream is consumer

        def copy_(self, source, *, non_blocking):
            assert current[0] is consumer and self.device == "cpu" and source.is_cuda and non_blocking
            log.append(("copy", source.numel() * 8))
            return self

        def narrow(self, dim, start, length):
            assert dim == 0 and self.dtype == "u8" and self.ndim == 1 and start + length <= self.shape[0]
            return Tensor((length,), "u8", self.pointer + start, self.device)

        def view(self, dtype):
            assert self.dtype == "u8" and self.shape[0] % sizes[dtype] == 0
            return Tensor((self.shape[0] // sizes[dtype],), dtype, self.pointer, self.device)

        def tolist(self):
            assert self.device == "cpu" and state["synchronized"]
            if self.shape == (1,):  # the device status word read after the call
                log.append(("read_device_word",))
                return [state["device_word"]]
            log.append(("read_host_status",))
            return list(state["status"])

    allocations = []

    def empty(shape, *, dtype, device=device, pin_memory=False):
        assert current[0] is consumer
        assert pin_memory is (device == "cpu")
        tensor = Tensor(tuple(shape), dtype, 0x100000 * (len(allocations) + 1), device)
        allocations.append(tensor)
        log.append(("allocate", device, tuple(shape), dtype))
        return tensor

    fake_torch = SimpleNamespace(
        Tensor=Tensor, float32="f32", bfloat16="bf16", int32="i32", int64="i64", uint8="u8", empty=empty,
        cuda=SimpleNamespace(Stream=Stream, device=lambda _: nullcontext(), get_device_capability=lambda _: (10, 0),
                             current_stream=lambda _: current[0], stream=stream_context,
                             get_device_properties=lambda _: SimpleNamespace(L2_cache_size=126 << 20)))

    def check_offsets(index, n, b, offsets_ptr, min_len, max_len, status_ptr, stream):
        log.append(("launch", "check", index, n, b, min_len, max_len, stream))
        return SimpleNamespace(num_launches=2, kernel_ids=[10, 11], grid=[(1, 1, 1), (max(1, (b + 128) // 128), 1, 1)])

    def run(*args):
        log.append(("launch", "main", args[-2] if len(args) > 1 else None))
        state["synchronized"] = False
        return SimpleNamespace(num_launches=1, kernel_ids=[2], grid=[(4, 1, 1)], d_vector=1, d_tile=1, streams=1,
                               thresholds=[0, 0], status_offset=state.get("status_offset", -1))

    monkeypatch.setattr(runtime, "_torch", lambda: fake_torch)
    monkeypatch.setattr(runtime, "device_l2_mib", lambda _: 126.0, raising=False)
    monkeypatch.setattr(_native, "check_offsets", check_offsets)
    monkeypatch.setattr(_native, "run", run)
    monkeypatch.setattr(_native, "workspace_bytes", lambda *args: 4096)
    monkeypatch.setattr(runtime, "_checked_devices", set())
    spec = ProgramSpec("sum", "f32", 4, "i64", hints=Hints(max_len=32, min_len=1))
    program = Compiler().compile(spec, ArtifactCache(str(tmp_path), max_specializations=16))

    def call(*, b=5, n=10, mode="checked", select="naive"):
        return program.run(Tensor((n, 4), "f32", 1 << 40), Tensor((b + 1,), "i64", 2 << 40),
                           Tensor((b, 4), "f32", 3 << 40), stream=consumer, mode=mode, select=select)

    return SimpleNamespace(call=call, log=log, state=state, allocations=allocations, current=current,
                           producer=producer)


def _kinds(log):
    return [event[0] for event in log]


def test_checked_validates_before_scratch_and_main_launch(host):
    report = host.call(b=128, n=300, select="rowbalanced")
    assert host.current[0] is host.producer
    launches = [event[1] for event in host.log if event[0] == "launch"]
    assert launches == ["check", "main"]
    check = next(event for event in host.log if event[:2] == ("launch", "check"))
    assert check[5:] == (1, 32, 202), "length bounds come from the spec's hints; the execution stream is used"
    read = host.log.index(("read_host_status",))
    main = next(i for i, event in enumerate(host.log) if event[:2] == ("launch", "main"))
    scratch = [i for i, event in enumerate(host.log) if event[0] == "allocate" and event[-1] == "u8"]
    assert read < main and all(i > read for i in scratch)
    assert [event for event in host.log if event[0] == "copy"] == [("copy", 56)]
    assert [event for event in host.log if event[0] == "synchronize"] == [("synchronize", 202)]
    assert report.mode == "checked" and report.validation_workspace_bytes == 56
    assert report.kernel_names[:2] == ("offsets_init", "offsets_check")
    assert report.grids[:2] == ((1, 1, 1), (2, 1, 1))
    assert report.validation_host_ms is not None and report.validation_host_ms >= 0


def test_checked_failure_never_allocates_scratch_or_launches_main(host):
    from ragged import ValidationError
    host.state["status"] = [0, 5, 2, 3, 1, 2, 4]
    with pytest.raises(ValidationError) as caught:
        host.call()
    assert caught.value.condition == "first_nonzero"
    assert [event[1] for event in host.log if event[0] == "launch"] == ["check"]
    assert all(tensor.shape == (7,) for tensor in host.allocations) and len(host.allocations) == 2
    assert host.current[0] is host.producer


def test_validated_mode_reads_nothing_back(host):
    host.state["status"] = [0] * 7  # a bogus status that validated mode must never read
    report = host.call(mode="validated")
    assert [event[1] for event in host.log if event[0] == "launch"] == ["main"]
    assert not {"copy", "synchronize", "read_host_status"} & set(_kinds(host.log))
    assert report.validation_workspace_bytes == 0 and report.validation_host_ms is None


def test_zero_batch_checked_still_validates(host):
    report = host.call(b=0, n=0)
    assert report.classes == () and report.kernel_names == ("offsets_init", "offsets_check")
    assert report.workspace_bytes == 56
    assert [event[1] for event in host.log if event[0] == "launch"] == ["check"]


def test_zero_batch_with_rows_is_reported_by_the_device(host):
    from ragged import ValidationError
    host.state["status"][1] = 0
    with pytest.raises(ValidationError) as caught:
        host.call(b=0, n=1)
    assert caught.value.errors == {"final_mismatch": 0}
    with pytest.raises(ValidationError, match="B=0 requires N=0"):
        host.call(b=0, n=1, mode="validated")


def test_checked_reads_the_device_status_word_after_the_call(host):
    """A schedule that keeps a device status word (the classified worker's
    bounded waits) reports its offset in the scratch; checked mode copies
    the 8-byte word back after the main launch, on the execution stream."""
    host.state["status_offset"] = 16
    host.state["device_word"] = 0
    host.call(select="classified")
    kinds = _kinds(host.log)
    main = next(i for i, event in enumerate(host.log) if event[:2] == ("launch", "main"))
    assert [event for event in host.log if event[0] == "copy"] == [("copy", 56), ("copy", 8)]
    assert kinds.index("read_device_word") > main
    assert [event for event in host.log if event[0] == "synchronize"] == [("synchronize", 202)] * 2


def test_checked_raises_when_a_bounded_wait_gave_up(host):
    host.state["status_offset"] = 16
    host.state["device_word"] = 1
    with pytest.raises(RuntimeError, match="bounded wait"):
        host.call(select="classified")


def test_validated_mode_never_reads_the_device_status_word(host):
    host.state["status_offset"] = 16
    host.state["device_word"] = 1
    host.call(mode="validated", select="classified")
    assert not {"copy", "synchronize", "read_device_word"} & set(_kinds(host.log))
