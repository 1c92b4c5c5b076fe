"""Shared pytest setup.

Markers: ``gpu`` — needs a CUDA device (run with ``-m gpu`` on a B200 box);
everything else runs on a CPU-only host.
"""
from __future__ import annotations

import os
import sys

import numpy as np
import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path.insert(0, ROOT)
sys.path.insert(0, os.path.join(ROOT, "tiny-llm_b200"))
sys.path.insert(0, os.path.join(ROOT, "tests", "golden"))

GOLDEN = os.path.join(ROOT, "tests", "golden", "golden_ref.npz")


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200)")


@pytest.fixture(scope="session")
def golden():
    return np.load(GOLDEN)


@pytest.fixture(scope="session")
def oracle():
    from oracle.oracle import Oracle
    return Oracle()


@pytest.fixture(scope="session")
def reflib():
    from oracle.oracle import RefLib
    if not RefLib.available():
        pytest.skip("reference CPU build (oracle/_ref) not present")
    return RefLib()


@pytest.fixture(scope="session")
def tq():
    """The product library (libtqb200.so) with a visible CUDA device."""
    from tqb200 import lib
    lib.load()
    if lib.device_count() < 1:
        pytest.fail("no CUDA device visible to libtqb200.so")
    return lib


def max_rel(y, ref) -> float:
    """max|y - ref| / max|ref| (benchmarks/bench_kernels.cpp:474-479)."""
    y = np.asarray(y, np.float64)
    ref = np.asarray(ref, np.float64)
    denom = max(np.abs(ref).max(), 1e-30)
    return float(np.abs(y - ref).max() / denom)
