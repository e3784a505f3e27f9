"""Test configuration: the `gpu` marker and import paths.

`-m "not gpu"` runs on a CPU-only machine: the oracle against the reference's
golden vectors, host-side logic, and the C-ABI library's exported symbols.
`-m gpu` runs the CUDA path against the oracle on a B200.
"""
from __future__ import annotations

import sys
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parents[1]
for p in (ROOT, ROOT / "tests" / "golden"):
    if str(p) not in sys.path:
        sys.path.insert(0, str(p))


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200, sm_100a)")


@pytest.fixture(scope="session")
def golden():
    import numpy as np
    return np.load(ROOT / "tests" / "golden" / "engram_golden.npz")


@pytest.fixture(scope="session")
def fake1_rows():
    """All rows of the reference's FakeTable(seed=1) (float32 [80000, 160])."""
    import fixtures as FX
    return FX.fake_table_rows(seed=1)
