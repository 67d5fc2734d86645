"""The C ABI library loads and exports what include/ragged_b200.h declares.

No compute call is made here (no GPU in the build container); only entry
points whose argument checks fail before any CUDA call are exercised.
"""
from __future__ import annotations

import ctypes
from pathlib import Path
import re
import subprocess

HEADER = Path(__file__).resolve().parents[1] / "include" / "ragged_b200.h"


def declared_functions() -> set[str]:
    text = HEADER.read_text()
    return set(re.findall(r"^\s*(?:const\s+)?\w+\s+\*?(rg_\w+)\s*\(", text, flags=re.M))


def test_header_declarations_are_exported(native_library):
    from ragged import _native
    names = declared_functions()
    assert names == set(_native.EXPORTED)
    symbols = subprocess.run(["nm", "-D", "--defined-only", str(_native.LIBRARY)], capture_output=True,
                             text=True, check=True).stdout
    exported = {line.split()[-1] for line in symbols.splitlines() if " T " in line}
    assert names <= exported, names - exported
    for name in names:
        assert getattr(native_library, name)


def test_version_and_error_strings(native_library):
    from ragged import _native
    assert "sm_100a" in _native.version()
    assert native_library.rg_error_string(0) == b"success"
    assert native_library.rg_error_string(4) == b"CUDA error"


def test_argument_errors_need_no_device(native_library):
    from ragged import _native
    report = _native.Report()
    # D = 0: rejected before any CUDA call.
    status = native_library.rg_run(0, 0, 1, 0, 0, 1, None, None, None, None, 0, 1, -1, 0, None,
                                   ctypes.byref(report))
    assert status == _native.RG_ERR_INVALID_ARGUMENT
    assert b"D must" in native_library.rg_last_error()
    # B = 0 with N > 0.
    status = native_library.rg_run(0, 0, 1, 4, 3, 0, None, None, None, None, 0, 1, -1, 0, None, None)
    assert status == _native.RG_ERR_INVALID_ARGUMENT
    # i32 offsets with N beyond the i32 range.
    status = native_library.rg_run(0, 0, 0, 4, 2**31, 1, None, None, None, None, 0, 1, -1, 0, None, None)
    assert status == _native.RG_ERR_INVALID_ARGUMENT


def test_missing_library_raises_instead_of_falling_back(monkeypatch, tmp_path):
    """Without libragged_b200.so the package refuses to run: there is no
    CPU implementation to fall back on."""
    import pytest
    from ragged import RuntimeUnavailable, _native
    monkeypatch.setattr(_native, "_lib", None)
    with pytest.raises(RuntimeUnavailable, match="no CPU fallback"):
        _native.library(tmp_path / "libragged_b200.so")


def test_host_tensors_are_refused_not_computed(native_library, tmp_path):
    """run() and run_sharded() with tensors in host memory raise
    RuntimeUnavailable before any launch; nothing is computed on the CPU."""
    import pytest
    torch = pytest.importorskip("torch")
    from ragged import ArtifactCache, Compiler, ProgramSpec, RuntimeUnavailable
    program = Compiler().compile(ProgramSpec("sum", "f32", 4, "i64"), ArtifactCache(tmp_path))
    values, offsets = torch.ones((6, 4)), torch.tensor([0, 2, 6])
    out = torch.full((2, 4), -1.0)
    with pytest.raises(RuntimeUnavailable, match="no CPU execution fallback"):
        program.run(values, offsets, out)
    with pytest.raises(RuntimeUnavailable, match="no CPU execution fallback"):
        program.run_sharded(values, offsets, out, total_rows=6, world=1, rank=0, exchange=lambda edges: edges)
    assert torch.all(out == -1).item()


def test_exchange_result_checks():
    """The all-gather result handed to the combine kernel must be every
    rank's f32 record, contiguous, on the records' device (host logic)."""
    import pytest
    torch = pytest.importorskip("torch")
    from ragged import ValidationError
    from ragged.runtime import _check_gathered
    edges = torch.zeros(16)
    good = torch.zeros(48)
    assert _check_gathered(good, edges, 3, torch) is good
    for bad in (torch.zeros(47), torch.zeros(48, dtype=torch.bfloat16), torch.zeros(96)[::2],
                torch.zeros(48).numpy()):
        with pytest.raises(ValidationError):
            _check_gathered(bad, edges, 3, torch)
