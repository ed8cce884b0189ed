"""TEST INFRASTRUCTURE ONLY -- the parity oracle, not part of the product.

numpy/ctypes front end for ``oracle/qmm_oracle.cpp``, a CPU restatement of the
reference's quantized-matmul path (crate ``swe-llmmodel-kernel``:
``llmserve/llmmodel/kernel/main/src/core/{quantize.rs,simd.rs}``). Only
``tests/``, ``__graft_entry__.smoke()`` and the CPU legs of ``bench.py`` may
import this module, and only as the checker / timed CPU baseline. The product
library (``machinelearning_b200``) never calls it.

Function names follow the reference so the parity tests read like its own
tests: ``quantize_q8_0`` (quantize.rs:15), ``quantize_row_q8_0`` (:260),
``quantize_q4_0`` (:124), ``quantize_q4_1`` (:207), ``matmul_f32_q8`` (:297),
``matmul_f32_q8_v2`` (:429), ``matmul_f32_q4`` (:535), ``matmul_f32_q4_native``
(:646), ``matmul_f32_q4_1`` (:807), ``matmul_f32_q4_1_native`` (:938), the
block dots of simd.rs:644-761 and ``to_f32`` (tensor.rs:527-630).
"""
from __future__ import annotations

import ctypes
import os
import subprocess

import numpy as np

_HERE = os.path.dirname(os.path.abspath(__file__))
_LIB_PATH = os.path.join(_HERE, "_build", "libqmm_oracle.so")

Q8_0, Q4_0, Q4_1 = 8, 2, 3  # GGML type ids (gguf/main/src/api/types.rs:8-12)
BLOCK_BYTES = {Q8_0: 34, Q4_0: 18, Q4_1: 20}
QK = 32


class BlockAlignment(ValueError):
    """Mirror of ``QuantError::BlockAlignment`` (kernel/main/src/api/error.rs:13)."""


def build(force: bool = False) -> str:
    """Compile the oracle with its Makefile (g++, OpenMP, -ffp-contract=off)."""
    src = os.path.join(_HERE, "qmm_oracle.cpp")
    if force or not os.path.exists(_LIB_PATH) or os.path.getmtime(_LIB_PATH) < os.path.getmtime(src):
        subprocess.run(["make", "-C", _HERE, "-s"], check=True)
    return _LIB_PATH


_lib = None


def lib() -> ctypes.CDLL:
    global _lib
    if _lib is None:
        if not os.path.exists(_LIB_PATH):
            build()
        L = ctypes.CDLL(_LIB_PATH)
        P = ctypes.c_void_p
        I64 = ctypes.c_int64
        for name in ("orc_matmul_f32_q8", "orc_matmul_f32_q8_v2", "orc_matmul_f32_q4",
                     "orc_matmul_f32_q4_native", "orc_matmul_f32_q4_1", "orc_matmul_f32_q4_1_native"):
            getattr(L, name).argtypes = [P, P, I64, I64, I64, P]
            getattr(L, name).restype = ctypes.c_int
        for name in ("orc_quantize_q8_0", "orc_quantize_q4_0", "orc_quantize_q4_1"):
            getattr(L, name).argtypes = [P, I64, P]
            getattr(L, name).restype = ctypes.c_int
        L.orc_quantize_row_q8_0.argtypes = [P, I64, P, P]
        L.orc_quantize_row_q8_0.restype = None
        L.orc_dequantize.argtypes = [ctypes.c_int, P, I64, P]
        L.orc_dequantize.restype = ctypes.c_int
        L.orc_dequantize_q4_0_interleaved.argtypes = [P, I64, P]
        L.orc_f32_to_f16.argtypes = [ctypes.c_float]
        L.orc_f32_to_f16.restype = ctypes.c_uint16
        L.orc_f16_to_f32.argtypes = [ctypes.c_uint16]
        L.orc_f16_to_f32.restype = ctypes.c_float
        L.orc_f32_to_f16_array.argtypes = [P, I64, P]
        L.orc_f32_to_f16_f16c.argtypes = [P, I64, P]
        L.orc_dot_q8_block.argtypes = [P, P, ctypes.c_float]
        L.orc_dot_q8_block.restype = ctypes.c_float
        L.orc_dot_q4_block.argtypes = [P, P, ctypes.c_float]
        L.orc_dot_q4_block.restype = ctypes.c_float
        L.orc_dot_q8q8_block.argtypes = [P, P]
        L.orc_dot_q8q8_block.restype = ctypes.c_int32
        L.orc_dot_q4q8_block.argtypes = [P, P]
        L.orc_dot_q4q8_block.restype = ctypes.c_int32
        L.orc_dot_q4_1q8_block.argtypes = [P, P, P, P]
        L.orc_set_isa.argtypes = [ctypes.c_int]
        L.orc_set_threads.argtypes = [ctypes.c_int]
        _lib = L
    return _lib


def _ptr(a: np.ndarray) -> int:
    return a.ctypes.data


def _f32(x) -> np.ndarray:
    return np.ascontiguousarray(np.asarray(x, dtype=np.float32))


def _u8(x) -> np.ndarray:
    return np.ascontiguousarray(np.frombuffer(bytes(x), dtype=np.uint8) if isinstance(x, (bytes, bytearray)) else np.asarray(x, dtype=np.uint8))


def set_isa(simd: bool) -> None:
    """True: the reference's runtime dispatch (AVX2+FMA -> AVX2). False: scalar only."""
    lib().orc_set_isa(1 if simd else 0)


def set_threads(n: int) -> None:
    lib().orc_set_threads(int(n))


def threads() -> int:
    return int(lib().orc_get_threads())


def host_has_avx2_fma() -> bool:
    return bool(lib().orc_host_has_avx2_fma())


# ---- f16 ----------------------------------------------------------------------
def f32_to_f16_bits(x) -> np.ndarray:
    x = _f32(x).ravel()
    out = np.empty(x.size, dtype=np.uint16)
    lib().orc_f32_to_f16_array(_ptr(x), x.size, _ptr(out))
    return out


def f32_to_f16_bits_f16c(x) -> np.ndarray:
    x = _f32(x).ravel()
    out = np.empty(x.size, dtype=np.uint16)
    lib().orc_f32_to_f16_f16c(_ptr(x), x.size, _ptr(out))
    return out


# ---- quantizers ---------------------------------------------------------------
def _quant(fn, x, bb):
    x = _f32(x).ravel()
    out = np.zeros((x.size // QK) * bb, dtype=np.uint8)
    if fn(_ptr(x), x.size, _ptr(out)) != 0:
        raise BlockAlignment(f"element count divisible by {QK} required, got {x.size}")
    return out


def quantize_q8_0(x) -> np.ndarray:
    return _quant(lib().orc_quantize_q8_0, x, 34)


def quantize_q4_0(x) -> np.ndarray:
    return _quant(lib().orc_quantize_q4_0, x, 18)


def quantize_q4_1(x) -> np.ndarray:
    return _quant(lib().orc_quantize_q4_1, x, 20)


def quantize_row_q8_0(x):
    """Returns (blocks u8[nb*34], scales f32[nb]) like quantize.rs:260-289."""
    x = _f32(x).ravel()
    nb = x.size // QK
    out = np.zeros(nb * 34, dtype=np.uint8)
    sc = np.zeros(nb, dtype=np.float32)
    lib().orc_quantize_row_q8_0(_ptr(x), x.size, _ptr(out), _ptr(sc))
    return out, sc


def to_f32(dtype: int, w, n_elements: int) -> np.ndarray:
    """Tensor::to_f32 dequantisation (Q4_0 in GGML nibble order)."""
    w = _u8(w)
    out = np.zeros(n_elements, dtype=np.float32)
    rc = lib().orc_dequantize(int(dtype), _ptr(w), n_elements, _ptr(out))
    if rc == 1:
        raise BlockAlignment(f"element count {n_elements} not divisible by 32")
    if rc != 0:
        raise ValueError(f"unsupported dtype {dtype}")
    return out


def dequantize_q4_0_interleaved(w, n_elements: int) -> np.ndarray:
    w = _u8(w)
    out = np.zeros(n_elements, dtype=np.float32)
    lib().orc_dequantize_q4_0_interleaved(_ptr(w), n_elements, _ptr(out))
    return out


# ---- block dots (simd.rs dispatch functions) ----------------------------------
def dot_q8_block(x, q, scale: float) -> float:
    x, q = _f32(x), np.ascontiguousarray(np.asarray(q, dtype=np.int8))
    return float(lib().orc_dot_q8_block(_ptr(x), _ptr(q), ctypes.c_float(scale)))


def dot_q4_block(x, packed, scale: float) -> float:
    x, p = _f32(x), _u8(packed)
    return float(lib().orc_dot_q4_block(_ptr(x), _ptr(p), ctypes.c_float(scale)))


def dot_q8q8_block(a, b) -> int:
    a = np.ascontiguousarray(np.asarray(a, dtype=np.int8))
    b = np.ascontiguousarray(np.asarray(b, dtype=np.int8))
    return int(lib().orc_dot_q8q8_block(_ptr(a), _ptr(b)))


def dot_q4q8_block(packed, q) -> int:
    p, q = _u8(packed), np.ascontiguousarray(np.asarray(q, dtype=np.int8))
    return int(lib().orc_dot_q4q8_block(_ptr(p), _ptr(q)))


def dot_q4_1_q8_block(packed, q):
    p, q = _u8(packed), np.ascontiguousarray(np.asarray(q, dtype=np.int8))
    d, s = ctypes.c_int32(), ctypes.c_int32()
    lib().orc_dot_q4_1q8_block(_ptr(p), _ptr(q), ctypes.addressof(d), ctypes.addressof(s))
    return int(d.value), int(s.value)


# ---- matmuls --------------------------------------------------------------------
def _mm(fn, x, w, m, k, n):
    x = _f32(x).ravel()
    w = _u8(w)
    y = np.zeros(m * n, dtype=np.float32)
    if fn(_ptr(x), _ptr(w), m, k, n, _ptr(y)) != 0:
        raise BlockAlignment(f"in_features {k} not divisible by block size 32")
    return y


def matmul_f32_q8(x, w, m, k, n):
    return _mm(lib().orc_matmul_f32_q8, x, w, m, k, n)


def matmul_f32_q8_v2(x, w, m, k, n):
    return _mm(lib().orc_matmul_f32_q8_v2, x, w, m, k, n)


def matmul_f32_q4(x, w, m, k, n):
    return _mm(lib().orc_matmul_f32_q4, x, w, m, k, n)


def matmul_f32_q4_native(x, w, m, k, n):
    return _mm(lib().orc_matmul_f32_q4_native, x, w, m, k, n)


def matmul_f32_q4_1(x, w, m, k, n):
    return _mm(lib().orc_matmul_f32_q4_1, x, w, m, k, n)


def matmul_f32_q4_1_native(x, w, m, k, n):
    return _mm(lib().orc_matmul_f32_q4_1_native, x, w, m, k, n)


MATMUL = {
    (Q8_0, False): matmul_f32_q8,
    (Q8_0, True): matmul_f32_q8_v2,
    (Q4_0, False): matmul_f32_q4,
    (Q4_0, True): matmul_f32_q4_native,
    (Q4_1, False): matmul_f32_q4_1,
    (Q4_1, True): matmul_f32_q4_1_native,
}


# ---- activations and fused projections (layers crate) ------------------------------
# Element-wise in float32, the reference's operations in its order
# (main/features/tensor/src/core/tensor/math.rs:465-483); numpy's float32
# tanh / exp stand in for Rust's f32 tanh / exp (libm), which round differently
# by an ulp or so.
def gelu(x) -> np.ndarray:
    """math.rs:470-475: 0.5 x (1 + tanh(sqrt(2/pi) (x + 0.044715 x^3)))."""
    x = _f32(x)
    k = np.sqrt(np.float32(2.0) / np.float32(np.pi), dtype=np.float32)
    with np.errstate(over="ignore"):
        return (np.float32(0.5) * x * (np.float32(1.0) + np.tanh(k * (x + np.float32(0.044715) * (x * x * x))))).astype(np.float32)


def silu(x) -> np.ndarray:
    """math.rs:478-483: x * (1 / (1 + exp(-x)))."""
    x = _f32(x)
    with np.errstate(over="ignore"):
        return (x * (np.float32(1.0) / (np.float32(1.0) + np.exp(-x)))).astype(np.float32)


def relu(x) -> np.ndarray:
    """math.rs:465-467: x.max(0)."""
    return np.maximum(_f32(x), np.float32(0.0))


ACTIVATIONS = {0: gelu, 1: silu, 2: relu}


def fuse_rows(*parts) -> np.ndarray:
    """Byte concatenation of weights with equal in_features, as
    Attention::fuse_qkv_weights (layers/main/src/core/attention.rs:306-339) and
    FeedForward::fuse_gate_up_weights (feed_forward.rs:147-187) build the fused
    tensor: the fused matmul's output row is the parts' outputs side by side."""
    return np.concatenate([_u8(p) for p in parts])


def gated_ffn_hidden(act: int, x, gate_w, up_w, dtype: int, m: int, k: int, hidden: int) -> np.ndarray:
    """The hidden activation of FeedForward::forward's gated branch
    (feed_forward.rs:198-231, fused or not: both give the same rows):
    act(matmul(x, gate)) * matmul(x, up) with the f32-activation matmul of the
    weight's type (the fused Linear has use_native_* false)."""
    mm = MATMUL[(dtype, False)]
    g = mm(x, gate_w, m, k, hidden)
    u = mm(x, up_w, m, k, hidden)
    return (ACTIVATIONS[act](g) * u).astype(np.float32)
