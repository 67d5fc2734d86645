"""Shared pytest configuration.

Markers: ``gpu`` marks tests that need a B200 (they FAIL without one, never
skip).  Everything else runs on CPU (the oracle, host logic, the C ABI's
argument checks and exports, gloo multi-process tests).
"""
from __future__ import annotations

from pathlib import Path
import sys

import numpy as np
import pytest

REPO = Path(__file__).resolve().parents[1]
PACKAGE = REPO / "ragged-mlir_b200"
for path in (str(REPO), str(PACKAGE)):
    if path not in sys.path:
        sys.path.insert(0, path)

GOLDEN = REPO / "tests" / "golden" / "golden.npz"


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a B200 GPU (fails, never skips, without one)")


@pytest.fixture(scope="session")
def masked_golden():
    """name -> dict(values, mask, offsets, logits, softmax, dtype, scale) from
    the reference's oracle/masked.py (tests/golden/make_masked_golden.py)."""
    import json
    path = REPO / "tests" / "golden" / "masked.npz"
    data = np.load(path)
    cases = {}
    for case in json.loads(path.with_suffix(".json").read_text())["cases"]:
        name = case["name"]
        cases[name] = {key: data[f"{name}__{key}"] for key in ("values", "mask", "offsets", "logits", "softmax")}
        cases[name].update(dtype=case["dtype"], scale=case["scale"])
    return cases


@pytest.fixture(scope="session")
def golden():
    """name -> dict(values, offsets, sum, max, softmax, dtype)."""
    import json
    data = np.load(GOLDEN)
    index = json.loads((GOLDEN.with_suffix(".json")).read_text())
    cases = {}
    for case in index["cases"]:
        name = case["name"]
        cases[name] = {key: data[f"{name}__{key}"] for key in ("values", "offsets", "sum", "max", "softmax")}
        cases[name]["dtype"] = case["dtype"]
    return cases


@pytest.fixture(scope="session")
def native_library():
    """Build (if needed) and load libragged_b200.so."""
    sys.path.insert(0, str(PACKAGE))
    import build as package_build  # ragged-mlir_b200/build.py
    package_build.build()
    from ragged import _native
    return _native.library()


@pytest.fixture(scope="session")
def cuda():
    """torch with a B200 device; a missing GPU or library is a failure."""
    import torch
    assert torch.cuda.is_available(), "GPU tests need a CUDA device (no CPU fallback exists)"
    capability = torch.cuda.get_device_capability(0)
    assert capability == (10, 0), f"GPU tests need a B200 (sm_100), found sm_{capability[0]}{capability[1]}"
    from ragged import _native
    _native.library()
    return torch
