"""Fused projections (machinelearning_b200/fused.py): fused QKV weights
(reference Attention::fuse_qkv_weights, layers/main/src/core/attention.rs:306-339),
fused gate+up weights with the activation in the matmul epilogue
(FeedForward::fuse_gate_up_weights / forward, feed_forward.rs:147-251), and the
element-wise activation kernel, checked against the oracle's restatements."""
from __future__ import annotations

import ctypes

import numpy as np
import pytest

from conftest import assert_close_rel

Q4_0, Q4_1, Q8_0 = 2, 3, 8
BB = {Q4_0: 18, Q4_1: 20, Q8_0: 34}
GELU, SILU, RELU = 0, 1, 2
QUANT = {Q4_0: "quantize_q4_0", Q4_1: "quantize_q4_1", Q8_0: "quantize_q8_0"}


# ---- CPU: the oracle's activations and fusion -------------------------------------------------

def test_oracle_activations_match_formulas(oracle):
    x = np.random.default_rng(1).normal(0, 3, 4096).astype(np.float32)
    xd = x.astype(np.float64)
    gelu = 0.5 * xd * (1 + np.tanh(np.sqrt(2 / np.pi) * (xd + 0.044715 * xd ** 3)))
    silu = xd / (1 + np.exp(-xd))
    np.testing.assert_allclose(oracle.gelu(x), gelu, rtol=2e-6, atol=1e-6)
    np.testing.assert_allclose(oracle.silu(x), silu, rtol=2e-6, atol=1e-7)
    assert np.array_equal(oracle.relu(x), np.maximum(x, 0))
    assert oracle.gelu(np.float32([0.0]))[0] == 0 and oracle.silu(np.float32([0.0]))[0] == 0


@pytest.mark.parametrize("dt", [Q8_0, Q4_0, Q4_1])
def test_oracle_fused_rows_are_parts_side_by_side(oracle, dt):
    """The property the reference's fusion rests on: rows are independent, so
    the fused matmul's output is the parts' outputs concatenated, bit for bit."""
    rng = np.random.default_rng(dt)
    k, ns, m = 128, (48, 16, 16), 3
    parts = [getattr(oracle, QUANT[dt])(rng.normal(0, 0.05, n * k).astype(np.float32)) for n in ns]
    x = rng.normal(0, 1, (m, k)).astype(np.float32)
    mm = oracle.MATMUL[(dt, False)]
    fused = mm(x, oracle.fuse_rows(*parts), m, k, sum(ns)).reshape(m, -1)
    sep = np.concatenate([mm(x, p, m, k, n).reshape(m, n) for p, n in zip(parts, ns)], axis=1)
    assert np.array_equal(fused.view(np.uint32), sep.view(np.uint32))


def test_abi_argument_errors(qlib):
    """Validation that returns before touching a device."""
    out = ctypes.c_void_p()
    assert qlib.qmm_weight_fuse_rows(None, 0, ctypes.byref(out)) == 8
    assert qlib.qmm_weight_fuse_gate_up(None, None, ctypes.byref(out)) == 8
    assert qlib.qmm_gated_forward(None, None, 1, None, GELU, None) == 8
    assert qlib.qmm_gated_act_dev(7, None, None, 1, 1, 1, None, None) == 8   # unknown activation
    assert qlib.qmm_gated_act_dev(GELU, None, None, 0, 5, 5, None, None) == 0  # empty: nothing to do
    h = ctypes.c_size_t()
    assert qlib.qmm_weight_gate_hidden(None, ctypes.byref(h)) == 8


# ---- GPU --------------------------------------------------------------------------------------

def _rows(oracle, dt, n, k, rng, scale=0.05):
    return getattr(oracle, QUANT[dt])(rng.normal(0, scale, n * k).astype(np.float32))


def _gemm(dt, m, k, n=2):
    """The f16 tensor-core GEMM (d*q rounded to f16 once): M >= 17 with a
    16-byte row pitch, or 8 mod 16 with N even and M <= 64 (qmm_gemm.cu:
    single_shape_ok). Other decode batches run the exact-split GEMM."""
    rb = (k // 32) * BB[dt]
    return m >= 17 and (rb % 16 == 0 or (rb % 16 == 8 and n % 2 == 0 and m <= 64))


def _gemm_elem(m):
    """Per-element guard of the f16 GEMM: its errors are Gaussian-tailed
    (sigma ~2e-4 of the output rms with exact activations, M <= 128; ~4e-4
    above), so the largest of many outputs reaches ~1e-3 / ~2e-3."""
    return 2e-3 if m <= 128 else 4e-3


def _interleave(gate, up, hidden, k, dt):
    """Host copy of the gate/up layout: groups of 16 rows, gate then up, zero padding."""
    rb = (k // 32) * BB[dt]
    groups = -(-hidden // 16)
    out = np.zeros((groups, 2, 16, rb), np.uint8)
    g = np.zeros((groups * 16, rb), np.uint8)
    u = np.zeros((groups * 16, rb), np.uint8)
    g[:hidden] = gate.reshape(hidden, rb)
    u[:hidden] = up.reshape(hidden, rb)
    out[:, 0] = g.reshape(groups, 16, rb)
    out[:, 1] = u.reshape(groups, 16, rb)
    return out.ravel()


QKV = [  # (dtype, in, q, kv): Gemma-3-1B (4 heads x 256, 1 kv head) and smaller
    (Q8_0, 1152, 1024, 256),
    (Q4_0, 1152, 1024, 256),
    (Q4_1, 1152, 1024, 256),
    (Q8_0, 256, 96, 32),
]


@pytest.mark.gpu
@pytest.mark.parametrize("dt,k,qd,kvd", QKV)
@pytest.mark.parametrize("m", [1, 5, 33])
def test_fused_qkv(oracle, dt, k, qd, kvd, m):
    import torch

    from machinelearning_b200.fused import QkvProjection
    from machinelearning_b200.gguf import checksum
    from machinelearning_b200.linear import Linear, QuantWeight

    rng = np.random.default_rng(k + qd + m)
    ws = [_rows(oracle, dt, n, k, rng) for n in (qd, kvd, kvd)]
    lins = [Linear(QuantWeight.from_host(dt, n, k, w)) for n, w in zip((qd, kvd, kvd), ws)]
    proj = QkvProjection(*lins)
    assert proj.fuse_qkv_weights()
    fw = proj.fused_qkv.weight
    assert (fw.dtype, fw.n, fw.k) == (dt, qd + 2 * kvd, k)
    out = ctypes.c_ulonglong()
    from machinelearning_b200 import _lib
    _lib.check(_lib.lib().qmm_weight_checksum(fw.handle, ctypes.byref(out)))
    assert out.value == checksum(oracle.fuse_rows(*ws).tobytes())  # byte concatenation, nothing repacked
    x = rng.normal(0, 1, (m, k)).astype(np.float32)
    q, kk, v = proj(torch.from_numpy(x).cuda())
    er = _gemm_elem(m) if _gemm(dt, m, k, qd + 2 * kvd) else None
    for got, w, n in zip((q, kk, v), ws, (qd, kvd, kvd)):
        assert tuple(got.shape) == (m, n) and got.is_contiguous()
        assert_close_rel(got.cpu().numpy(), oracle.MATMUL[(dt, False)](x, w, m, k, n), elem_rtol=er)


GATED = [  # (dtype, hidden, in, m, act)
    (Q8_0, 6912, 1152, 1, GELU),    # Gemma-3-1B MLP, decode
    (Q8_0, 6912, 1152, 4, GELU),
    (Q8_0, 6912, 1152, 16, SILU),
    (Q8_0, 6912, 1152, 17, GELU),   # decode-batch GEMM, paired rows (1224-byte pitch)
    (Q8_0, 6912, 1152, 100, GELU),  # decode-batch GEMM, 128-token tile
    (Q4_0, 6912, 1152, 1, SILU),
    (Q4_0, 6912, 1152, 8, GELU),
    (Q4_1, 100, 256, 1, GELU),      # hidden not a multiple of 16: padded group
    (Q4_1, 100, 256, 3, SILU),
    (Q4_1, 100, 256, 20, GELU),     # decode-batch GEMM (160-byte rows), padded group
    (Q8_0, 8, 64, 1, SILU),         # a single partial group
    (Q4_0, 2048, 4096, 32, GELU),   # decode-batch GEMM, 32-token tile
    (Q4_0, 2048, 4096, 200, SILU),  # prefill GEMM, two token tiles
    (Q8_0, 1024, 16384, 1, GELU),   # 35.6 MB: the streaming GEMV
    (Q8_0, 1024, 16384, 9, SILU),
]


@pytest.mark.gpu
@pytest.mark.parametrize("dt,hidden,k,m,act", GATED)
def test_gated_forward(oracle, dt, hidden, k, m, act):
    import torch

    from machinelearning_b200 import _lib
    from machinelearning_b200.fused import fuse_gate_up, gated_act, gated_forward
    from machinelearning_b200.gguf import checksum
    from machinelearning_b200.linear import QuantWeight, matmul_dev

    rng = np.random.default_rng(hidden + k + m)
    gate, up = _rows(oracle, dt, hidden, k, rng), _rows(oracle, dt, hidden, k, rng)
    fw = fuse_gate_up(QuantWeight.from_host(dt, hidden, k, gate), QuantWeight.from_host(dt, hidden, k, up))
    groups = -(-hidden // 16)
    assert fw.gate_hidden == hidden and fw.n == 32 * groups
    out = ctypes.c_ulonglong()
    _lib.check(_lib.lib().qmm_weight_checksum(fw.handle, ctypes.byref(out)))
    layout = _interleave(gate, up, hidden, k, dt)
    assert out.value == checksum(layout.tobytes())
    x = rng.normal(0, 1, (m, k)).astype(np.float32)
    xd = torch.from_numpy(x).cuda()
    h = gated_forward(fw, xd, act)
    torch.cuda.synchronize()
    assert tuple(h.shape) == (m, hidden)
    # against the oracle: act(x . gate) * (x . up)
    ref = oracle.gated_ffn_hidden(act, x, gate, up, dt, m, k, hidden).reshape(m, hidden)
    assert_close_rel(h.cpu().numpy(), ref, rtol=1e-3, elem_rtol=1e-2)
    # the epilogue applies exactly the activation kernel's function to exactly
    # the plain matmul's sums (same kernel plan over the same fused rows)
    wdev = torch.from_numpy(layout).cuda()
    y = matmul_dev(dt, _lib.ACT_F32, xd, wdev, fw.n, k).view(m, groups, 2, 16)
    g = y[:, :, 0, :].reshape(m, -1)[:, :hidden].contiguous()
    u = y[:, :, 1, :].reshape(m, -1)[:, :hidden].contiguous()
    h2 = gated_act(act, g, u, m, hidden, hidden)
    torch.cuda.synchronize()
    assert torch.equal(h.view(torch.int32), h2.view(torch.int32))


@pytest.mark.gpu
@pytest.mark.parametrize("act", [GELU, SILU, RELU])
def test_gated_act_kernel(oracle, act):
    import torch

    from machinelearning_b200.fused import gated_act

    rng = np.random.default_rng(act)
    m, hidden = 7, 1000
    f = rng.normal(0, 4, (m, 2 * hidden)).astype(np.float32)
    f[0, :8] = [0.0, -0.0, 1e-30, -1e-30, 30.0, -30.0, 100.0, -100.0]
    fd = torch.from_numpy(f).cuda()
    # [gate | up] rows of a byte-concatenated fused weight: ld = 2 * hidden
    g, u = f[:, :hidden], f[:, hidden:]
    h = gated_act(act, fd, fd[:, hidden:], m, hidden, 2 * hidden).cpu().numpy()
    ref = oracle.ACTIVATIONS[act](g) * u
    # CUDA's tanhf / expf and the host's differ by an ulp or so; GELU's
    # 1 + tanh(.) cancels for large negative inputs, where one ulp of tanh is
    # an absolute error of about |g| * ulp(1) / 2 on the activation
    tol = 4e-6 * np.abs(ref) + 1.2e-7 * np.abs(g * u) + 1e-30
    assert np.all(np.abs(h - ref) <= tol), np.max(np.abs(h - ref) / tol)
    # ungated: act alone
    a = gated_act(act, fd, None, m, hidden, 2 * hidden).cpu().numpy()
    ra = oracle.ACTIVATIONS[act](g)
    assert np.all(np.abs(a - ra) <= 4e-6 * np.abs(ra) + 1.2e-7 * np.abs(g) + 1e-30)


@pytest.mark.gpu
@pytest.mark.parametrize("dt", [Q8_0, Q4_0])
@pytest.mark.parametrize("activation", ["GeGLU", "SwiGLU", "Gelu"])
def test_feed_forward(oracle, dt, activation):
    """FeedForward::forward, fused and unfused, against the oracle's chain."""
    import torch

    from machinelearning_b200.fused import Activation, FeedForward
    from machinelearning_b200.linear import Linear, QuantWeight

    rng = np.random.default_rng(dt)
    d, hidden, m = 256, 512, 3
    wg, wu, wd = _rows(oracle, dt, hidden, d, rng), _rows(oracle, dt, hidden, d, rng), _rows(oracle, dt, d, hidden, rng)
    act = Activation[activation]
    gated = act in (Activation.GeGLU, Activation.SwiGLU)
    ff = FeedForward(Linear(QuantWeight.from_host(dt, hidden, d, wu)), Linear(QuantWeight.from_host(dt, d, hidden, wd)),
                     Linear(QuantWeight.from_host(dt, hidden, d, wg)) if gated else None, act)
    x = rng.normal(0, 1, (m, d)).astype(np.float32)
    mm = oracle.MATMUL[(dt, False)]
    fn = {Activation.GeGLU: GELU, Activation.SwiGLU: SILU, Activation.Gelu: GELU}[act]
    if gated:
        h_ref = oracle.gated_ffn_hidden(fn, x, wg, wu, dt, m, d, hidden)
    else:
        h_ref = oracle.gelu(mm(x, wu, m, d, hidden))
    y_ref = mm(h_ref, wd, m, hidden, d)
    xd = torch.from_numpy(x).cuda()
    y0 = ff(xd).cpu().numpy()
    assert_close_rel(y0, y_ref, rtol=2e-3, elem_rtol=2e-2)
    assert ff.fuse_gate_up_weights() == gated
    y1 = ff(xd).cpu().numpy()
    assert_close_rel(y1, y_ref, rtol=2e-3, elem_rtol=2e-2)


@pytest.mark.gpu
def test_fuse_errors(oracle):
    import torch

    from machinelearning_b200 import _lib
    from machinelearning_b200.fused import fuse_gate_up, fuse_rows
    from machinelearning_b200.linear import Linear, QuantWeight

    rng = np.random.default_rng(0)
    a = QuantWeight.from_host(Q8_0, 32, 64, _rows(oracle, Q8_0, 32, 64, rng))
    b = QuantWeight.from_host(Q4_0, 32, 64, _rows(oracle, Q4_0, 32, 64, rng))
    c = QuantWeight.from_host(Q8_0, 32, 128, _rows(oracle, Q8_0, 32, 128, rng))
    d = QuantWeight.from_host(Q8_0, 16, 64, _rows(oracle, Q8_0, 16, 64, rng))
    with pytest.raises(_lib.DTypeMismatch):
        fuse_rows(a, b)
    with pytest.raises(_lib.ShapeMismatch):
        fuse_rows(a, c)
    with pytest.raises(_lib.DTypeMismatch):
        fuse_gate_up(a, b)
    with pytest.raises(_lib.ShapeMismatch):
        fuse_gate_up(a, d)
    g = fuse_gate_up(a, a)
    with pytest.raises(_lib.QmmError):
        Linear(g)(torch.zeros(1, 64, device="cuda"))  # a gate/up weight is not a plain Linear
    with pytest.raises(_lib.QmmError):
        fuse_rows(a, g)
