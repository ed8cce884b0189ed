"""Python mirror of the reference's quant-kernel crate API, backed by libqmm.so.

Same names, argument meaning and error behaviour as
``llmserve/llmmodel/kernel/main/src/core/quantize.rs`` (crate
``swe-llmmodel-kernel``), so code written against the reference reads the
same here. Every function runs on the GPU through the C ABI; host arrays are
copied in and out. Errors raise the QuantError mirrors (``BlockAlignment``,
``ShapeMismatch``, ``DTypeMismatch``) where the reference returns them; where
the reference would panic on a short slice, ``ShapeMismatch`` is raised.

Block constants: kernel/main/src/api/types.rs:1-23.
"""
from __future__ import annotations

import ctypes

import numpy as np

from . import _lib
from ._lib import ACT_F32, ACT_Q8_0, Q4_0, Q4_1, Q8_0, BlockAlignment, DTypeMismatch, QmmError, ShapeMismatch

Q8_0_BLOCK_SIZE = 32
Q8_0_BLOCK_BYTES = 34
Q4_0_BLOCK_SIZE = 32
Q4_0_BLOCK_BYTES = 18
Q4_1_BLOCK_SIZE = 32
Q4_1_BLOCK_BYTES = 20
TILE_M = 4
TILE_N = 8

__all__ = [
    "Q8_0_BLOCK_SIZE", "Q8_0_BLOCK_BYTES", "Q4_0_BLOCK_SIZE", "Q4_0_BLOCK_BYTES", "Q4_1_BLOCK_SIZE",
    "Q4_1_BLOCK_BYTES", "TILE_M", "TILE_N", "BlockAlignment", "ShapeMismatch", "DTypeMismatch", "QmmError",
    "quantize_q8_0", "quantize_q4_0", "quantize_q4_1", "quantize_row_q8_0", "to_f32",
    "matmul_f32_q8", "matmul_f32_q8_v2", "matmul_f32_q4", "matmul_f32_q4_native", "matmul_f32_q4_1",
    "matmul_f32_q4_1_native", "register_host_weight", "unregister_host_weight",
]


def _f32(x) -> np.ndarray:
    return np.ascontiguousarray(np.asarray(x, dtype=np.float32).ravel())


def _u8(x) -> np.ndarray:
    if isinstance(x, (bytes, bytearray, memoryview)):
        return np.frombuffer(x, dtype=np.uint8)
    return np.ascontiguousarray(np.asarray(x, dtype=np.uint8).ravel())


def _host_matmul(fn, input_data, weight_bytes, m, in_features, out_features) -> np.ndarray:
    x = _f32(input_data)
    w = _u8(weight_bytes)
    y = np.empty(int(m) * int(out_features), dtype=np.float32)
    _lib.check(fn(x.ctypes.data, x.size, w.ctypes.data, w.size, int(m), int(in_features), int(out_features),
                  y.ctypes.data))
    return y


def matmul_f32_q8(input_data, weight_bytes, m, in_features, out_features) -> np.ndarray:
    """F32 input x Q8_0 weights -> F32 [m, out_features] (quantize.rs:297)."""
    return _host_matmul(_lib.lib().qmm_matmul_f32_q8, input_data, weight_bytes, m, in_features, out_features)


def matmul_f32_q8_v2(input_data, weight_bytes, m, in_features, out_features) -> np.ndarray:
    """Integer-domain Q8_0 x Q8_0 path (quantize.rs:429)."""
    return _host_matmul(_lib.lib().qmm_matmul_f32_q8_v2, input_data, weight_bytes, m, in_features, out_features)


def matmul_f32_q4(input_data, weight_bytes, m, in_features, out_features) -> np.ndarray:
    """F32 input x Q4_0 weights (quantize.rs:535)."""
    return _host_matmul(_lib.lib().qmm_matmul_f32_q4, input_data, weight_bytes, m, in_features, out_features)


def matmul_f32_q4_native(input_data, weight_bytes, m, in_features, out_features) -> np.ndarray:
    """Q4_0 x Q8_0-activation integer path (quantize.rs:646)."""
    return _host_matmul(_lib.lib().qmm_matmul_f32_q4_native, input_data, weight_bytes, m, in_features,
                        out_features)


def matmul_f32_q4_1(input_data, weight_bytes, m, in_features, out_features) -> np.ndarray:
    """F32 input x Q4_1 weights (quantize.rs:807)."""
    return _host_matmul(_lib.lib().qmm_matmul_f32_q4_1, input_data, weight_bytes, m, in_features, out_features)


def matmul_f32_q4_1_native(input_data, weight_bytes, m, in_features, out_features) -> np.ndarray:
    """Q4_1 x Q8_0-activation integer path (quantize.rs:938)."""
    return _host_matmul(_lib.lib().qmm_matmul_f32_q4_1_native, input_data, weight_bytes, m, in_features,
                        out_features)


def _quant(fn, data, block_bytes) -> np.ndarray:
    x = _f32(data)
    out = np.empty((x.size // 32) * block_bytes, dtype=np.uint8)
    _lib.check(fn(x.ctypes.data, x.size, out.ctypes.data))
    return out


def quantize_q8_0(data) -> np.ndarray:
    """quantize.rs:15 -- Q8_0 blocks, inverse scale from the un-rounded scale."""
    return _quant(_lib.lib().qmm_quantize_q8_0, data, Q8_0_BLOCK_BYTES)


def quantize_q4_0(data) -> np.ndarray:
    """quantize.rs:124 -- Q4_0 blocks with the reference's interleaved nibble packing."""
    return _quant(_lib.lib().qmm_quantize_q4_0, data, Q4_0_BLOCK_BYTES)


def quantize_q4_1(data) -> np.ndarray:
    """quantize.rs:207."""
    return _quant(_lib.lib().qmm_quantize_q4_1, data, Q4_1_BLOCK_BYTES)


def quantize_row_q8_0(data):
    """quantize.rs:260 -- returns (Q8_0 bytes, f32(f16) scales)."""
    x = _f32(data)
    nb = x.size // 32
    out = np.empty(nb * Q8_0_BLOCK_BYTES, dtype=np.uint8)
    sc = np.empty(nb, dtype=np.float32)
    _lib.check(_lib.lib().qmm_quantize_row_q8_0(x.ctypes.data, x.size, out.ctypes.data, sc.ctypes.data))
    return out, sc


def to_f32(dtype: int, raw, n_elements: int) -> np.ndarray:
    """Tensor::to_f32 for block types (tensor.rs:527-630; Q4_0 in GGML order)."""
    w = _u8(raw)
    out = np.empty(int(n_elements), dtype=np.float32)
    _lib.check(_lib.lib().qmm_dequantize(int(dtype), w.ctypes.data, w.size, int(n_elements), out.ctypes.data))
    return out


_registered: dict[int, np.ndarray] = {}


def register_host_weight(weight_bytes: np.ndarray, dtype: int, n: int, k: int) -> None:
    """Keeps a resident device copy of a host weight buffer for the matmul_* calls above.

    The array is retained here so its address stays valid while registered.
    """
    w = _u8(weight_bytes)
    _lib.check(_lib.lib().qmm_register_host_weight(w.ctypes.data, w.size, int(dtype), int(n), int(k)))
    _registered[w.ctypes.data] = w


def unregister_host_weight(weight_bytes: np.ndarray) -> None:
    w = _u8(weight_bytes)
    _lib.check(_lib.lib().qmm_unregister_host_weight(w.ctypes.data))
    _registered.pop(w.ctypes.data, None)


MATMUL = {
    (Q8_0, False): matmul_f32_q8,
    (Q8_0, True): matmul_f32_q8_v2,
    (Q4_0, False): matmul_f32_q4,
    (Q4_0, True): matmul_f32_q4_native,
    (Q4_1, False): matmul_f32_q4_1,
    (Q4_1, True): matmul_f32_q4_1_native,
}
