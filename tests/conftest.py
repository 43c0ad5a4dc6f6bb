"""Test configuration: the `gpu` marker and shared fixtures.

`-m "not gpu"` (CPU, any machine): oracle vs golden fixtures, oracle vs the
reference library when it is built, host logic, and the C-ABI library's
exports.  `-m gpu` (a B200): parity of the CUDA path against the oracle and
the golden fixtures, through the C ABI.
"""
from __future__ import annotations

import sys
from pathlib import Path

import numpy as np
import pytest

ROOT = Path(__file__).resolve().parent.parent
GOLDEN = ROOT / "tests" / "golden"
sys.path.insert(0, str(ROOT))


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200, sm_100a)")


@pytest.fixture(scope="session")
def oracle():
    from oracle.oracle import Oracle
    return Oracle()


@pytest.fixture(scope="session")
def reflib():
    from oracle.oracle import REF_SO, REF_SRC, RefLib
    if not REF_SO.exists() and not REF_SRC.exists():
        pytest.skip("reference library not built here (sources absent)")
    return RefLib()


@pytest.fixture(scope="session")
def cuda():
    import torch
    if not torch.cuda.is_available():
        pytest.fail("gpu test run without a CUDA device")
    import axion_b200
    axion_b200.load()
    return torch.device("cuda", 0)


def golden(name: str):
    p = GOLDEN / name
    return np.load(p) if p.suffix in (".npz", ".npy") else p


def rel_err(y: np.ndarray, ref: np.ndarray, scale: np.ndarray) -> float:
    """max |y - ref| / (sum_k |x_k w_k| + tiny): error normalised by the
    magnitude of the terms summed, so near-cancelling outputs do not give
    false failures."""
    return float(np.max(np.abs(y.astype(np.float64) - ref) / (scale + 1e-30)))
