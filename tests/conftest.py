"""Shared fixtures.

* ``-m "not gpu"`` tests: the oracle against the golden fixtures and against
  the reference build, the host logic, and that the C-ABI library loads and
  exports every declared symbol (no device calls).
* ``-m gpu`` tests: parity of the CUDA path (called through the C ABI) with
  the oracle / golden fixtures.
"""
from __future__ import annotations

import os
import sys

import numpy as np
import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
GOLDEN = os.path.join(ROOT, "tests", "golden")
sys.path.insert(0, ROOT)
sys.path.insert(0, os.path.join(ROOT, "oracle"))


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a B200 (sm_100a) GPU")


def _ensure_built():
    from memvanta_b200 import build
    lib = os.path.join(ROOT, "memvanta_b200", "libmemvanta_b200.so")
    if not os.path.exists(lib):
        build.build_lib()
    if not os.path.exists(os.path.join(ROOT, "oracle", "_bin", "libmvoracle.so")):
        build.build_oracle()


_ensure_built()


@pytest.fixture(scope="session")
def oracle():
    from oracle import Oracle
    return Oracle()


@pytest.fixture(scope="session")
def reference():
    from oracle import Reference, ref_available
    if not ref_available():
        pytest.skip("oracle/_ref (the reference build) is not present")
    return Reference()


@pytest.fixture(scope="session")
def golden():
    def load(name):
        return np.load(os.path.join(GOLDEN, name))
    return load


@pytest.fixture(scope="session")
def cuda():
    import torch
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    import memvanta_b200 as mv
    mv.init(0)
    return torch.device("cuda:0")


def rel_err(y, ref):
    """max_i |y_i - ref_i| / max(|ref_i|, rms(ref)) -- the per-output relative
    error the parity bar is stated in (1e-3 Q4_0/Q8_0, 5e-3 Q6_K)."""
    y = np.asarray(y, dtype=np.float64)
    ref = np.asarray(ref, dtype=np.float64)
    rms = np.sqrt(np.mean(ref * ref)) if ref.size else 0.0
    den = np.maximum(np.abs(ref), rms)
    den = np.where(den == 0, 1.0, den)
    return float(np.max(np.abs(y - ref) / den)) if ref.size else 0.0
