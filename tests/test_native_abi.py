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
