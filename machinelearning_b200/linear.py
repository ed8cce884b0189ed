"""Device-resident quantised weights and the ``Linear`` operator.

Mirrors the reference's ``Linear`` (llmserve/llmmodel/layers/main/src/core/linear.rs)
for quantised weights: ``forward`` dispatches on the weight's block type, and
``use_native_q4`` / ``use_native_q8`` select the Q8_0-activation integer path
exactly as the reference's flags do (linear.rs:206-258). Weights live in HBM
as the raw GGUF block bytes (one host-to-device copy, no repacking); the
matmul runs on the caller's current torch CUDA stream. torch supplies device
memory and streams only; all arithmetic is in libqmm.so.
"""
from __future__ import annotations

import ctypes

import numpy as np
import torch

from . import _lib
from ._lib import ACT_F32, ACT_Q8_0, BLOCK_BYTES, Q4_0, Q4_1, Q8_0


class QuantWeight:
    """An [out_features, in_features] block-quantised matrix resident on one GPU."""

    def __init__(self, handle: int, dtype: int, n: int, k: int, device: int):
        self._h = ctypes.c_void_p(handle)
        self.dtype, self.n, self.k, self.device = dtype, n, k, device
        self.gate_hidden = 0  # > 0: a gate/up weight (machinelearning_b200.fused.fuse_gate_up)

    @classmethod
    def from_host(cls, dtype: int, n: int, k: int, data, device: int = 0) -> "QuantWeight":
        buf = np.ascontiguousarray(np.frombuffer(data, dtype=np.uint8) if isinstance(data, (bytes, bytearray, memoryview))
                                   else np.asarray(data, dtype=np.uint8).ravel())
        h = ctypes.c_void_p()
        _lib.check(_lib.lib().qmm_weight_create(int(dtype), int(n), int(k), buf.ctypes.data, buf.size, int(device),
                                                ctypes.byref(h)))
        return cls(h.value, dtype, n, k, device)

    @classmethod
    def from_device(cls, dtype: int, n: int, k: int, t: torch.Tensor) -> "QuantWeight":
        assert t.is_cuda and t.dtype == torch.uint8 and t.is_contiguous()
        h = ctypes.c_void_p()
        _lib.check(_lib.lib().qmm_weight_create_from_device(int(dtype), int(n), int(k), t.data_ptr(), t.numel(),
                                                            t.device.index, ctypes.byref(h)))
        return cls(h.value, dtype, n, k, t.device.index)

    @property
    def handle(self) -> ctypes.c_void_p:
        return self._h

    @property
    def nbytes(self) -> int:
        return self.n * (self.k // 32) * BLOCK_BYTES[self.dtype]

    def device_ptr(self) -> int:
        p = ctypes.c_void_p()
        _lib.check(_lib.lib().qmm_weight_info(self._h, None, None, None, ctypes.byref(p), None))
        return p.value

    def close(self) -> None:
        if self._h is not None and self._h.value:
            _lib.lib().qmm_weight_destroy(self._h)
            self._h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


def _stream_ptr(device: int) -> int:
    return torch.cuda.current_stream(device).cuda_stream


class Linear:
    """y = x W^T + b for a block-quantised W (reference linear.rs:13-31, 206-281)."""

    def __init__(self, weight: QuantWeight, bias: torch.Tensor | None = None):
        self.weight = weight
        self.bias = bias
        self.in_features = weight.k
        self.out_features = weight.n
        self.frozen = False
        self.use_native_q4 = False
        self.use_native_q8 = False

    def is_quantized(self) -> bool:
        return self.weight.dtype in (Q8_0, Q4_0, Q4_1)

    def set_native_q4_matmul(self, enabled: bool) -> None:
        self.use_native_q4 = bool(enabled)

    def set_native_q8_matmul(self, enabled: bool) -> None:
        self.use_native_q8 = bool(enabled)

    def act_mode(self) -> int:
        native = self.use_native_q8 if self.weight.dtype == Q8_0 else self.use_native_q4
        return ACT_Q8_0 if native else ACT_F32

    def forward(self, x: torch.Tensor, out: torch.Tensor | None = None) -> torch.Tensor:
        """x: f32 CUDA tensor [..., in_features] on the weight's device."""
        if x.dtype != torch.float32:
            x = x.float()
        x = x.contiguous()
        if x.shape[-1] != self.in_features:
            raise _lib.ShapeMismatch(_lib.ERR_SHAPE_MISMATCH,
                                     f"last dim {x.shape[-1]} != in_features {self.in_features}")
        m = x.numel() // self.in_features
        shape = (*x.shape[:-1], self.out_features)
        if out is None:
            out = torch.empty(shape, dtype=torch.float32, device=x.device)
        _lib.check(_lib.lib().qmm_linear_forward(self.weight.handle, x.data_ptr(), m, out.data_ptr(),
                                                 self.act_mode(), ctypes.c_void_p(_stream_ptr(self.weight.device))))
        if self.bias is not None:
            out += self.bias
        return out

    __call__ = forward

    def parameter_count(self):
        total = self.in_features * self.out_features + (self.bias.numel() if self.bias is not None else 0)
        return total, (total if self.frozen else 0)


def matmul_dev(dtype: int, act: int, x: torch.Tensor, w: torch.Tensor, n: int, k: int,
               out: torch.Tensor | None = None, workspace: torch.Tensor | None = None) -> torch.Tensor:
    """Caller-managed device matmul over raw weight bytes (qmm_matmul_dev)."""
    m = x.numel() // k
    if out is None:
        out = torch.empty((m, n), dtype=torch.float32, device=x.device)
    ws_bytes = _lib.lib().qmm_workspace_size(int(dtype), int(act), m, n, k)
    if workspace is None or workspace.numel() < ws_bytes:
        workspace = torch.zeros(max(ws_bytes, 256), dtype=torch.uint8, device=x.device)
    _lib.check(_lib.lib().qmm_matmul_dev(int(dtype), int(act), x.data_ptr(), w.data_ptr(), w.numel(), m, k, n,
                                         out.data_ptr(), workspace.data_ptr(), workspace.numel(),
                                         ctypes.c_void_p(_stream_ptr(x.device.index))))
    return out
