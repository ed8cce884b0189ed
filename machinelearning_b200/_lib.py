"""ctypes binding of libqmm.so (the C ABI declared in include/qmm.h and
include/qmm_tp.h).

The library is the product: there is no Python or CPU fallback. Loading fails
loudly when the shared object is missing.
"""
from __future__ import annotations

import ctypes
import os

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "libqmm.so")

# qmm_status
OK = 0
ERR_BLOCK_ALIGNMENT = 1
ERR_SHAPE_MISMATCH = 2
ERR_DTYPE_MISMATCH = 3
ERR_INVALID_DATA = 4
ERR_CUDA = 5
ERR_NCCL = 6
ERR_TIMEOUT = 7
ERR_INVALID_INPUT = 8
ERR_NO_DEVICE = 9

# qmm_dtype (GGML ids)
Q4_0 = 2
Q4_1 = 3
Q8_0 = 8
BLOCK_BYTES = {Q4_0: 18, Q4_1: 20, Q8_0: 34}

# qmm_act
ACT_F32 = 0
ACT_Q8_0 = 1

# activation functions (qmm_gated_forward, qmm_gated_act_dev)
GELU = 0
SILU = 1
RELU = 2

# Every symbol include/qmm.h and include/qmm_tp.h declare, with (restype, argtypes).
_P = ctypes.c_void_p
_SZ = ctypes.c_size_t
_I = ctypes.c_int
_F = ctypes.c_float
_HOST_MM = (_I, [_P, _SZ, _P, _SZ, _SZ, _SZ, _SZ, _P])
SIGNATURES = {
    "qmm_version": (_I, []),
    "qmm_status_string": (ctypes.c_char_p, [_I]),
    "qmm_last_error_message": (ctypes.c_char_p, []),
    "qmm_device_count": (_I, []),
    "qmm_device_error": (_I, [_I, _P]),
    "qmm_device_status": (_I, [_I]),
    "qmm_selftest_bounded_wait": (_I, [ctypes.c_uint, _P]),
    "qmm_launch_count": (ctypes.c_ulonglong, []),
    "qmm_checksum_dev": (_I, [_P, _SZ, _P, _P]),
    "qmm_weight_checksum": (_I, [_P, _P]),
    "qmm_matmul_f32_q8": _HOST_MM,
    "qmm_matmul_f32_q8_v2": _HOST_MM,
    "qmm_matmul_f32_q4": _HOST_MM,
    "qmm_matmul_f32_q4_native": _HOST_MM,
    "qmm_matmul_f32_q4_1": _HOST_MM,
    "qmm_matmul_f32_q4_1_native": _HOST_MM,
    "qmm_quantize_q8_0": (_I, [_P, _SZ, _P]),
    "qmm_quantize_q4_0": (_I, [_P, _SZ, _P]),
    "qmm_quantize_q4_1": (_I, [_P, _SZ, _P]),
    "qmm_quantize_row_q8_0": (_I, [_P, _SZ, _P, _P]),
    "qmm_dequantize": (_I, [_I, _P, _SZ, _SZ, _P]),
    "qmm_register_host_weight": (_I, [_P, _SZ, _I, _SZ, _SZ]),
    "qmm_unregister_host_weight": (_I, [_P]),
    "qmm_weight_create": (_I, [_I, _SZ, _SZ, _P, _SZ, _I, _P]),
    "qmm_weight_create_from_device": (_I, [_I, _SZ, _SZ, _P, _SZ, _I, _P]),
    "qmm_weight_destroy": (_I, [_P]),
    "qmm_weight_info": (_I, [_P, _P, _P, _P, _P, _P]),
    "qmm_linear_forward": (_I, [_P, _P, _SZ, _P, _I, _P]),
    "qmm_linear_forward_host": (_I, [_P, _P, _SZ, _P, _I, _P]),
    "qmm_reserve_workspace": (_I, [_I, _P, _SZ]),
    "qmm_workspace_size": (_SZ, [_I, _I, _SZ, _SZ, _SZ]),
    "qmm_matmul_dev": (_I, [_I, _I, _P, _P, _SZ, _SZ, _SZ, _SZ, _P, _P, _SZ, _P]),
    "qmm_matmul_dev_noalloc": (_I, [_I, _I, _P, _P, _SZ, _SZ, _SZ, _SZ, _P, _P]),
    "qmm_quantize_dev": (_I, [_I, _I, _P, _SZ, _P, _P, _P]),
    "qmm_dequantize_dev": (_I, [_I, _P, _SZ, _SZ, _P, _P]),
    "qmm_gated_act_dev": (_I, [_I, _P, _P, _SZ, _SZ, _SZ, _P, _P]),
    "qmm_weight_fuse_rows": (_I, [_P, _SZ, _P]),
    "qmm_weight_fuse_gate_up": (_I, [_P, _P, _P]),
    "qmm_weight_gate_hidden": (_I, [_P, _P]),
    "qmm_gated_forward": (_I, [_P, _P, _SZ, _P, _I, _P]),
    # decode-step pieces
    "qmm_embed_q8_dev": (_I, [_P, _SZ, _SZ, _P, _SZ, _F, _P, _P]),
    "qmm_rmsnorm_dev": (_I, [_P, _P, _F, _F, _SZ, _SZ, _P, _SZ, _P]),
    "qmm_residual_rmsnorm_dev": (_I, [_P, _P, _P, _P, _F, _F, _SZ, _SZ, _P, _SZ, _P]),
    "qmm_qk_rope_cache_dev": (_I, [_P, _SZ, _I, _I, _I, _P, _P, _F, _F, _P, _P, _P, _I, _P, _P, _P, _P]),
    "qmm_attention_partial_floats": (_SZ, [_SZ, _I, _I, _I]),
    "qmm_attention_decode_dev": (_I, [_P, _P, _P, _SZ, _I, _I, _I, _P, _I, _F, _P, _P, _P]),
    "qmm_attention_decode_fused_dev": (_I, [_P, _SZ, _I, _I, _I, _P, _P, _F, _F, _P, _P, _P, _I, _P, _P, _F, _P, _P,
                                            _P]),
    "qmm_add_int_dev": (_I, [_P, _I, _P]),
    # include/qmm_tp.h
    "qmm_weight_create_row_shard": (_I, [_I, _SZ, _SZ, _P, _SZ, _I, _I, _I, _P]),
    "qmm_tp_available": (_I, []),
    "qmm_tp_unique_id": (_I, [_P]),
    "qmm_tp_init": (_I, [_P, _I, _I, _I, ctypes.c_double, _P]),
    "qmm_tp_destroy": (_I, [_P]),
    "qmm_tp_abort": (_I, [_P]),
    "qmm_tp_rank": (_I, [_P, _P, _P]),
    "qmm_tp_enable_peer": (_I, [_P, _SZ, ctypes.c_double]),
    "qmm_tp_status": (_I, [_P]),
    "qmm_tp_wait": (_I, [_P, _P, ctypes.c_double]),
    "qmm_tp_column_forward": (_I, [_P, _P, _P, _SZ, _P, _I, _P]),
    "qmm_tp_row_forward": (_I, [_P, _P, _P, _SZ, _P, _I, _P]),
    "qmm_tp_all_gather_f32": (_I, [_P, _P, _P, _SZ, _P]),
    "qmm_tp_all_reduce_f32": (_I, [_P, _P, _SZ, _P]),
}
TP_UNIQUE_ID_BYTES = 128


class QmmError(RuntimeError):
    def __init__(self, status: int, message: str):
        super().__init__(f"qmm status {status} ({status_name(status)}): {message}")
        self.status = status


class BlockAlignment(QmmError, ValueError):
    """QuantError::BlockAlignment (kernel/main/src/api/error.rs:13)."""


class ShapeMismatch(QmmError, ValueError):
    """QuantError::ShapeMismatch (kernel/main/src/api/error.rs:10)."""


class DTypeMismatch(QmmError, ValueError):
    """QuantError::DTypeMismatch (kernel/main/src/api/error.rs:7)."""


_STATUS_NAMES = {
    OK: "ok", ERR_BLOCK_ALIGNMENT: "block alignment", ERR_SHAPE_MISMATCH: "shape mismatch",
    ERR_DTYPE_MISMATCH: "dtype mismatch", ERR_INVALID_DATA: "invalid data", ERR_CUDA: "cuda error",
    ERR_NCCL: "nccl error", ERR_TIMEOUT: "timeout", ERR_INVALID_INPUT: "invalid input", ERR_NO_DEVICE: "no device",
}


def status_name(s: int) -> str:
    return _STATUS_NAMES.get(s, "unknown")


_lib = None


def lib() -> ctypes.CDLL:
    """Loads libqmm.so (raises if it has not been built)."""
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            raise ImportError(f"{LIB_PATH} is missing: build it with `python -m machinelearning_b200.build`")
        L = ctypes.CDLL(LIB_PATH)
        for name, (res, args) in SIGNATURES.items():
            fn = getattr(L, name)
            fn.restype = res
            fn.argtypes = args
        _lib = L
    return _lib


def check(status: int) -> None:
    if status == OK:
        return
    msg = lib().qmm_last_error_message()
    msg = msg.decode() if msg else ""
    cls = {ERR_BLOCK_ALIGNMENT: BlockAlignment, ERR_SHAPE_MISMATCH: ShapeMismatch,
           ERR_DTYPE_MISMATCH: DTypeMismatch}.get(status, QmmError)
    raise cls(status, msg)
