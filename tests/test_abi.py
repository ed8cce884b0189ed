"""C-ABI checks that need no GPU: libqmm.so loads, exports every symbol
include/qmm.h declares, and its host-side argument validation returns the
reference's error kinds (QuantError, kernel/main/src/api/error.rs:5-18)
without touching a device."""
from __future__ import annotations

import ctypes
import os
import re

import numpy as np
import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _declared_symbols():
    hdr = "".join(open(os.path.join(ROOT, "include", h)).read() for h in ("qmm.h", "qmm_tp.h"))
    return sorted(set(re.findall(r"QMM_API\s+[\w\s\*]+?\b(qmm_\w+)\s*\(", hdr)))


def test_header_symbols_exported(qlib):
    from machinelearning_b200 import _lib
    syms = _declared_symbols()
    assert len(syms) >= 25
    for s in syms:
        assert hasattr(qlib, s), f"{s} declared in include/ but not exported"
        assert s in _lib.SIGNATURES, f"{s} has no ctypes signature"
    assert set(_lib.SIGNATURES) == set(syms)


def test_version_and_status_strings(qlib):
    assert qlib.qmm_version() >= 100
    assert qlib.qmm_status_string(0) == b"ok"
    assert qlib.qmm_status_string(1) == b"block alignment"
    assert qlib.qmm_device_count() >= 0


def _host_call(qlib, fn, x, w, m, k, n, y=None):
    y = np.empty(max(m * n, 1), np.float32) if y is None else y
    return getattr(qlib, fn)(x.ctypes.data if x is not None else None, 0 if x is None else x.size,
                             w.ctypes.data if w is not None else None, 0 if w is None else w.size, m, k, n,
                             y.ctypes.data)


@pytest.mark.parametrize("fn", ["qmm_matmul_f32_q8", "qmm_matmul_f32_q8_v2", "qmm_matmul_f32_q4",
                                "qmm_matmul_f32_q4_native", "qmm_matmul_f32_q4_1", "qmm_matmul_f32_q4_1_native"])
def test_block_alignment_error(qlib, fn):
    x = np.ones(33, np.float32)
    w = np.zeros(64, np.uint8)
    assert _host_call(qlib, fn, x, w, 1, 33, 1) == 1


def test_short_weight_is_shape_mismatch(qlib):
    x = np.ones(64, np.float32)
    w = np.zeros(2 * 18 * 4 - 1, np.uint8)  # one byte short of 4 rows x 2 blocks
    assert _host_call(qlib, "qmm_matmul_f32_q4", x, w, 1, 64, 4) == 2


def test_short_input_is_shape_mismatch(qlib):
    x = np.ones(63, np.float32)
    w = np.zeros(2 * 34 * 4, np.uint8)
    assert _host_call(qlib, "qmm_matmul_f32_q8", x, w, 1, 64, 4) == 2


def test_null_pointer_is_invalid_input(qlib):
    w = np.zeros(2 * 34 * 4, np.uint8)
    assert _host_call(qlib, "qmm_matmul_f32_q8", None, w, 1, 64, 4) == 8
    msg = qlib.qmm_last_error_message()
    assert b"null" in msg


def test_unknown_dtype(qlib):
    assert qlib.qmm_dequantize(5, np.zeros(64, np.uint8).ctypes.data, 64, 32,
                               np.zeros(32, np.float32).ctypes.data) == 3


def test_quantize_alignment(qlib):
    x = np.ones(33, np.float32)
    out = np.zeros(64, np.uint8)
    assert qlib.qmm_quantize_q8_0(x.ctypes.data, 33, out.ctypes.data) == 1
    assert qlib.qmm_quantize_q4_0(x.ctypes.data, 33, out.ctypes.data) == 1


def test_workspace_size_rejects_bad_shapes(qlib):
    assert qlib.qmm_workspace_size(8, 0, 1, 16, 33) == 0
    assert qlib.qmm_workspace_size(5, 0, 1, 16, 32) == 0


def test_python_mirror_raises_reference_errors(qlib):
    from machinelearning_b200 import kernel
    with pytest.raises(kernel.BlockAlignment):
        kernel.matmul_f32_q4(np.ones(33, np.float32), np.zeros(18, np.uint8), 1, 33, 1)
    with pytest.raises(kernel.BlockAlignment):
        kernel.quantize_q8_0(np.ones(33, np.float32))
    with pytest.raises(kernel.ShapeMismatch):
        kernel.matmul_f32_q8(np.ones(64, np.float32), np.zeros(10, np.uint8), 1, 64, 4)


def test_selftest_rejects_bad_probe_counts(qlib):
    """Argument checks happen before any device work (runs without a GPU)."""
    from machinelearning_b200 import _lib
    assert qlib.qmm_selftest_bounded_wait(0, None) == _lib.ERR_INVALID_INPUT
    assert qlib.qmm_selftest_bounded_wait((1 << 20) + 1, None) == _lib.ERR_INVALID_INPUT
