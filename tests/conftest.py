"""Test configuration.

Markers:
  gpu -- needs a CUDA device (B200); run with `pytest -m gpu`. Everything else
         runs on a CPU-only host (`pytest -m "not gpu"`).
"""
from __future__ import annotations

import os
import sys

import numpy as np
import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: test needs a CUDA GPU (B200)")


def _cuda_available() -> bool:
    try:
        import torch
        return torch.cuda.is_available()
    except Exception:
        return False


def pytest_collection_modifyitems(config, items):
    if _cuda_available():
        return
    skip = pytest.mark.skip(reason="no CUDA device on this host")
    for item in items:
        if "gpu" in item.keywords:
            item.add_marker(skip)


@pytest.fixture(scope="session")
def oracle():
    import oracle as o
    o.build()
    return o


@pytest.fixture(scope="session")
def qlib():
    """libqmm.so, built in-tree if needed."""
    from machinelearning_b200 import build, _lib
    build.build()
    return _lib.lib()


@pytest.fixture(scope="session")
def golden():
    return np.load(os.path.join(ROOT, "tests", "golden", "golden.npz"))


def assert_close_rel(y, ref, rtol=1e-3, elem_rtol=None):
    """The north-star tolerance: ||y - ref|| / ||ref|| <= rtol (f32 accumulate),
    and per element |y - ref| <= elem_rtol * max(|ref|, rms(ref)) (default
    elem_rtol = rtol; an absolute floor at the output's rms scale, since
    per-element relative error is unstable near zero; the reference's own test
    uses abs 0.05 / rel 3 %, quantize.rs:1195-1202)."""
    elem_rtol = rtol if elem_rtol is None else elem_rtol
    y = np.asarray(y, dtype=np.float64).ravel()
    ref = np.asarray(ref, dtype=np.float64).ravel()
    assert y.shape == ref.shape
    if ref.size == 0:
        return
    assert np.all(np.isfinite(y)), "non-finite output"
    nrm = np.linalg.norm(ref)
    rel = np.linalg.norm(y - ref) / (nrm if nrm > 0 else 1.0)
    assert rel <= rtol, f"norm-wise relative error {rel:.3e} > {rtol}"
    rms = nrm / np.sqrt(ref.size)
    bound = elem_rtol * np.maximum(np.abs(ref), rms) + 1e-30
    worst = np.max(np.abs(y - ref) / bound)
    assert worst <= 1.0, f"per-element error exceeds bound by {worst:.2f}x"
    return rel
