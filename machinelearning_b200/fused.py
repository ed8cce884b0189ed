"""Fused projections: QKV and gate+up weights, and the feed-forward block.

Mirrors the reference's fusers in the layers crate:

* ``Attention::fuse_qkv_weights`` (llmserve/llmmodel/layers/main/src/core/
  attention.rs:306-339) and the projection step of ``Attention::forward``
  (attention.rs:349-362): ``QkvProjection``.
* ``FeedForward::fuse_gate_up_weights`` (feed_forward.rs:147-187) and
  ``FeedForward::forward`` (feed_forward.rs:198-251): ``FeedForward``.

The reference fuses by concatenating the Q8_0 bytes of the parts into one
tensor and slicing the fused output. ``fuse_rows`` builds exactly that weight
(for Q4_0 and Q4_1 too). The gate+up fusion here keeps the same rows but
interleaves gate and up in groups of 16 (``qmm_weight_fuse_gate_up``), so the
matmul's epilogue holds each gate value next to its up value and writes
act(gate) * up directly: one launch instead of a matmul, two slices and an
element-wise pass. The result is the one the reference computes for the same
rows (the fused Linear runs the f32-activation matmul, as the reference's does
with ``use_native_*`` false).
"""
from __future__ import annotations

import ctypes
import enum

import torch

from . import _lib
from ._lib import GELU, RELU, SILU
from .linear import Linear, QuantWeight, _stream_ptr


class Activation(enum.IntEnum):
    """layers/main/src/api/types.rs:22-28."""
    Gelu = 0
    Silu = 1
    Relu = 2
    SwiGLU = 3
    GeGLU = 4


_ACT_FN = {Activation.Gelu: GELU, Activation.Silu: SILU, Activation.Relu: RELU,
           Activation.SwiGLU: SILU, Activation.GeGLU: GELU}


def fuse_rows(*parts: QuantWeight) -> QuantWeight:
    """A new weight whose bytes are the parts' bytes in order (qmm_weight_fuse_rows)."""
    if not parts:
        raise ValueError("no parts")
    arr = (ctypes.c_void_p * len(parts))(*[p.handle.value for p in parts])
    h = ctypes.c_void_p()
    _lib.check(_lib.lib().qmm_weight_fuse_rows(arr, len(parts), ctypes.byref(h)))
    return QuantWeight(h.value, parts[0].dtype, sum(p.n for p in parts), parts[0].k, parts[0].device)


def fuse_gate_up(gate: QuantWeight, up: QuantWeight) -> QuantWeight:
    """A gate/up weight for ``gated_forward`` (qmm_weight_fuse_gate_up)."""
    h = ctypes.c_void_p()
    _lib.check(_lib.lib().qmm_weight_fuse_gate_up(gate.handle, up.handle, ctypes.byref(h)))
    hidden = ctypes.c_size_t()
    _lib.check(_lib.lib().qmm_weight_gate_hidden(ctypes.c_void_p(h.value), ctypes.byref(hidden)))
    n = ctypes.c_size_t()
    _lib.check(_lib.lib().qmm_weight_info(ctypes.c_void_p(h.value), None, ctypes.byref(n), None, None, None))
    w = QuantWeight(h.value, gate.dtype, n.value, gate.k, gate.device)
    w.gate_hidden = hidden.value
    return w


def gated_forward(w: QuantWeight, x: torch.Tensor, act_fn: int, out: torch.Tensor | None = None) -> torch.Tensor:
    """act(x . gate^T) * (x . up^T) for a gate/up weight, on the current stream."""
    if x.dtype != torch.float32:
        x = x.float()
    x = x.contiguous()
    if x.shape[-1] != w.k:
        raise _lib.ShapeMismatch(_lib.ERR_SHAPE_MISMATCH, f"last dim {x.shape[-1]} != in_features {w.k}")
    hidden = w.gate_hidden
    m = x.numel() // w.k
    if out is None:
        out = torch.empty((*x.shape[:-1], hidden), dtype=torch.float32, device=x.device)
    _lib.check(_lib.lib().qmm_gated_forward(w.handle, x.data_ptr(), m, out.data_ptr(), int(act_fn),
                                            ctypes.c_void_p(_stream_ptr(w.device))))
    return out


def gated_act(act_fn: int, gate: torch.Tensor, up: torch.Tensor | None, m: int, hidden: int, ld: int,
              out: torch.Tensor | None = None) -> torch.Tensor:
    """out[m][hidden] = act(gate) * up over rows of stride ``ld`` (qmm_gated_act_dev).

    ``gate`` / ``up`` are f32 CUDA tensors whose data pointer is element 0 of
    row 0; ``up`` None applies the activation alone."""
    if out is None:
        out = torch.empty((m, hidden), dtype=torch.float32, device=gate.device)
    _lib.check(_lib.lib().qmm_gated_act_dev(int(act_fn), gate.data_ptr(), up.data_ptr() if up is not None else None,
                                            m, hidden, ld, out.data_ptr(),
                                            ctypes.c_void_p(_stream_ptr(gate.device.index))))
    return out


class QkvProjection:
    """The q/k/v projections of an attention layer, fusable into one matmul."""

    def __init__(self, q_proj: Linear, k_proj: Linear, v_proj: Linear):
        self.q_proj, self.k_proj, self.v_proj = q_proj, k_proj, v_proj
        self.fused_qkv: Linear | None = None
        self.fused_q_dim = 0
        self.fused_kv_dim = 0

    def fuse_qkv_weights(self) -> bool:
        """attention.rs:306-339. False (no-op) if the parts carry biases or
        differ in block type, in_features or device. Q4_0 and Q4_1 fuse too."""
        q, k, v = self.q_proj, self.k_proj, self.v_proj
        if any(p.bias is not None for p in (q, k, v)):
            return False
        if len({p.weight.dtype for p in (q, k, v)}) != 1 or not q.is_quantized():
            return False
        if q.in_features != k.in_features or q.in_features != v.in_features:
            return False
        if len({p.weight.device for p in (q, k, v)}) != 1:
            return False
        self.fused_qkv = Linear(fuse_rows(q.weight, k.weight, v.weight))
        self.fused_qkv.frozen = True
        self.fused_q_dim = q.out_features
        self.fused_kv_dim = k.out_features
        return True

    def forward(self, x: torch.Tensor):
        """(q, k, v) as attention.rs:349-362 computes them."""
        if self.fused_qkv is not None:
            y = self.fused_qkv(x)
            q_end = self.fused_q_dim
            k_end = q_end + self.fused_kv_dim
            v_end = k_end + self.fused_kv_dim
            return (y[..., :q_end].contiguous(), y[..., q_end:k_end].contiguous(),
                    y[..., k_end:v_end].contiguous())
        return self.q_proj(x), self.k_proj(x), self.v_proj(x)

    __call__ = forward


class FeedForward:
    """feed_forward.rs:12-21: up/down projections, an optional gate, an activation."""

    def __init__(self, up_proj: Linear, down_proj: Linear, gate_proj: Linear | None = None,
                 activation: Activation = Activation.Gelu):
        if activation in (Activation.SwiGLU, Activation.GeGLU) and gate_proj is None:
            raise ValueError(f"{activation.name} requires gate_proj")
        self.up_proj, self.down_proj, self.gate_proj = up_proj, down_proj, gate_proj
        self.hidden_dim = up_proj.out_features
        self.activation = Activation(activation)
        self.fused_gate_up: QuantWeight | None = None

    def fuse_gate_up_weights(self) -> bool:
        """feed_forward.rs:147-187. False (no-op) without a gate, with biases,
        or if gate and up differ in block type, shape or device. Q4_0 and Q4_1
        fuse too. The fused weight is the gate/up-interleaved form."""
        g, u = self.gate_proj, self.up_proj
        if g is None or g.bias is not None or u.bias is not None:
            return False
        if g.weight.dtype != u.weight.dtype or not g.is_quantized():
            return False
        if g.in_features != u.in_features or g.out_features != u.out_features or g.weight.device != u.weight.device:
            return False
        self.fused_gate_up = fuse_gate_up(g.weight, u.weight)
        return True

    def hidden(self, x: torch.Tensor) -> torch.Tensor:
        """The activation fed to down_proj (feed_forward.rs:198-251)."""
        fn = _ACT_FN[self.activation]
        m = x.numel() // x.shape[-1]
        if self.activation in (Activation.SwiGLU, Activation.GeGLU):
            if self.fused_gate_up is not None:
                return gated_forward(self.fused_gate_up, x, fn)
            gate = self.gate_proj(x)
            up = self.up_proj(x)
            h = gated_act(fn, gate, up, m, self.hidden_dim, self.hidden_dim)
        else:
            h = gated_act(fn, self.up_proj(x), None, m, self.hidden_dim, self.hidden_dim)
        return h.reshape(*x.shape[:-1], self.hidden_dim)

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        return self.down_proj(self.hidden(x))

    __call__ = forward

    def set_native_q4_matmul(self, enabled: bool) -> None:
        """feed_forward.rs:138-145 (the fused weight keeps the f32 path)."""
        for p in (self.up_proj, self.down_proj, self.gate_proj):
            if p is not None:
                p.set_native_q4_matmul(enabled)

    def set_native_q8_matmul(self, enabled: bool) -> None:
        for p in (self.up_proj, self.down_proj, self.gate_proj):
            if p is not None:
                p.set_native_q8_matmul(enabled)
