"""Pins the CPU oracle (oracle/qmm_oracle.cpp) before it is trusted as the
parity checker: every known-answer and tolerance test the reference itself
holds for this path, the committed golden vectors (made by an independent
pure-numpy restatement, tests/golden/make_golden.py), and IEEE f16 rounding.

Reference tests restated (paths inside sweengineeringlabs/machinelearning):
  llmserve/llmmodel/kernel/main/src/core/simd.rs:783-883
  llmserve/llmmodel/kernel/main/src/core/quantize.rs:1085-1214
"""
from __future__ import annotations

import numpy as np
import pytest


# ---- simd.rs:787-881 -----------------------------------------------------------------

def test_q8_dot_scalar_vs_dispatch(oracle):
    x = np.arange(32, dtype=np.float32) * np.float32(0.1)
    q = (np.arange(32) - 16).astype(np.int8)
    oracle.set_isa(False)
    s = oracle.dot_q8_block(x, q, 0.5)
    oracle.set_isa(True)
    d = oracle.dot_q8_block(x, q, 0.5)
    assert abs(s - d) < 1e-3


def test_q4_dot_scalar_vs_dispatch(oracle):
    x = np.arange(32, dtype=np.float32) * np.float32(0.1)
    packed = np.array([(((j + 1) % 8 + 8) << 4) | ((j % 8) + 8) for j in range(16)], dtype=np.uint8)
    oracle.set_isa(False)
    s = oracle.dot_q4_block(x, packed, 0.5)
    oracle.set_isa(True)
    d = oracle.dot_q4_block(x, packed, 0.5)
    assert abs(s - d) < 1e-3


def test_q8q8_dot_scalar_vs_dispatch(oracle):
    a = (((np.arange(32) - 16) * 7) & 0xFF).astype(np.uint8).view(np.int8)
    b = (((np.arange(32) * 5) - 60) & 0xFF).astype(np.uint8).view(np.int8)
    oracle.set_isa(False)
    s = oracle.dot_q8q8_block(a, b)
    oracle.set_isa(True)
    assert oracle.dot_q8q8_block(a, b) == s


def test_q8q8_dot_extremes(oracle):
    oracle.set_isa(True)
    mx, mn = np.full(32, 127, np.int8), np.full(32, -128, np.int8)
    assert oracle.dot_q8q8_block(mx, mx) == 32 * 127 * 127 == 516128
    assert oracle.dot_q8q8_block(mn, mn) == 32 * 128 * 128 == 524288
    assert oracle.dot_q8q8_block(mx, mn) == -32 * 127 * 128 == -520192


def test_q4_1_q8_dot_scalar_vs_dispatch(oracle):
    packed = np.array([((j + 1) << 4 | j) & 0xFF for j in range(16)], dtype=np.uint8)
    q = (np.arange(32) - 16).astype(np.int8)
    oracle.set_isa(False)
    s = oracle.dot_q4_1_q8_block(packed, q)
    oracle.set_isa(True)
    assert oracle.dot_q4_1_q8_block(packed, q) == s


def test_q4q8_dot_scalar_vs_dispatch(oracle):
    packed = np.array([((j + 1) << 4 | j) & 0xFF for j in range(16)], dtype=np.uint8)
    q = (np.arange(32) - 16).astype(np.int8)
    oracle.set_isa(False)
    s = oracle.dot_q4q8_block(packed, q)
    oracle.set_isa(True)
    assert oracle.dot_q4q8_block(packed, q) == s
    # independent integer value (GGML order)
    nib = np.array([(int(v) & 0xF) - 8 for v in packed] + [(int(v) >> 4) - 8 for v in packed])
    assert s == int(np.dot(nib, q.astype(np.int64)))


# ---- quantize.rs:1089-1204 -------------------------------------------------------------

def _ramp():
    return ((np.arange(64, dtype=np.float32) - 32.0) / 10.0).astype(np.float32)


def test_q8_roundtrip(oracle):
    x = _ramp()
    d = oracle.to_f32(oracle.Q8_0, oracle.quantize_q8_0(x), 64)
    assert np.all(np.abs(x - d) < 0.05)


def test_q4_roundtrip_interleaved(oracle):
    # the reference's own pairing: quantize_q4_0 + kernel::dequantize_q4_0
    x = _ramp()
    d = oracle.dequantize_q4_0_interleaved(oracle.quantize_q4_0(x), 64)
    assert np.all(np.abs(x - d) < 0.5)


def test_q4_quantizer_vs_matmul_nibble_order(oracle):
    """quantize_q4_0 packs pairs (2i, 2i+1) per byte; every matmul and
    Tensor::to_f32 read (j, j+16). The reference therefore multiplies by a
    permuted weight after quantize_weight_q4_0 -- reproduced, not fixed."""
    x = _ramp()
    w = oracle.quantize_q4_0(x)
    inter = oracle.dequantize_q4_0_interleaved(w, 64)
    ggml = oracle.to_f32(oracle.Q4_0, w, 64)
    perm = np.concatenate([np.arange(0, 32, 2), np.arange(1, 32, 2)])
    for b in range(2):
        np.testing.assert_array_equal(ggml[32 * b:32 * b + 32], inter[32 * b + perm])


def test_q4_1_roundtrip(oracle):
    x = _ramp()
    d = oracle.to_f32(oracle.Q4_1, oracle.quantize_q4_1(x), 64)
    # to_f32 (GGML order) vs interleaved packer: compare as multisets per block
    for b in range(2):
        np.testing.assert_allclose(np.sort(d[32 * b:32 * b + 32]), np.sort(x[32 * b:32 * b + 32]), atol=0.5)


def test_q4_1_roundtrip_constant_block(oracle):
    x = np.full(32, 3.0, np.float32)
    d = oracle.to_f32(oracle.Q4_1, oracle.quantize_q4_1(x), 32)
    assert np.all(np.abs(d - 3.0) < 0.01)


@pytest.mark.parametrize("fn", ["quantize_q8_0", "quantize_q4_0", "quantize_q4_1"])
def test_block_alignment_errors(oracle, fn):
    with pytest.raises(oracle.BlockAlignment):
        getattr(oracle, fn)(np.ones(33, np.float32))


def test_q8_matmul_shape(oracle):
    m, k, n = 2, 64, 32
    x = (np.arange(m * k, dtype=np.float32) * np.float32(0.01)).astype(np.float32)
    w = oracle.quantize_q8_0((np.arange(n * k, dtype=np.float32) * np.float32(0.001)).astype(np.float32))
    assert oracle.matmul_f32_q8(x, w, m, k, n).size == m * n


def test_q8_matmul_v2_matches_v1(oracle):
    m, k, n = 3, 128, 64
    x = (np.sin(np.arange(m * k, dtype=np.float32)) * 0.5).astype(np.float32)
    w = oracle.quantize_q8_0((np.cos(np.arange(n * k, dtype=np.float32)) * 0.3).astype(np.float32))
    v1 = oracle.matmul_f32_q8(x, w, m, k, n)
    v2 = oracle.matmul_f32_q8_v2(x, w, m, k, n)
    ad = np.abs(v1 - v2)
    rd = np.where(np.abs(v1) > 1e-3, ad / np.abs(v1), 0.0)
    assert np.all((ad < 0.05) | (rd < 0.03))


def test_matmul_block_alignment_error(oracle):
    with pytest.raises(oracle.BlockAlignment):
        oracle.matmul_f32_q4(np.ones(33, np.float32), np.zeros(18, np.uint8), 1, 33, 1)


# ---- golden vectors (independent numpy restatement) ---------------------------------------

_KINDS = {"q8": "matmul_f32_q8", "q8_v2": "matmul_f32_q8_v2", "q4": "matmul_f32_q4",
          "q4_native": "matmul_f32_q4_native", "q4_1": "matmul_f32_q4_1", "q4_1_native": "matmul_f32_q4_1_native"}


def test_oracle_matches_golden_matmuls(oracle, golden):
    oracle.set_isa(True)
    assert oracle.host_has_avx2_fma(), "golden order is the AVX2+FMA dispatch path"
    for c in golden["cases"]:
        name, dt, kind, m, k, n = str(c).split(":")
        dt, m, k, n = int(dt), int(m), int(k), int(n)
        y = getattr(oracle, _KINDS[kind])(golden[name + "__x"], golden[name + "__w"], m, k, n)
        np.testing.assert_array_equal(y.view(np.uint32), golden[name + "__y"].view(np.uint32), err_msg=name)
        d = oracle.to_f32(dt, golden[name + "__w"], n * k)
        np.testing.assert_array_equal(d.view(np.uint32), golden[name + "__deq"].view(np.uint32), err_msg=name)


def test_oracle_matches_golden_quantizers(oracle, golden):
    x = golden["edge__x"]
    np.testing.assert_array_equal(oracle.quantize_q8_0(x), golden["edge__q8"])
    q, s = oracle.quantize_row_q8_0(x)
    np.testing.assert_array_equal(q, golden["edge__rowq8"])
    np.testing.assert_array_equal(s.view(np.uint32), golden["edge__rowq8_scales"].view(np.uint32))
    np.testing.assert_array_equal(oracle.quantize_q4_0(x), golden["edge__q4"])
    np.testing.assert_array_equal(oracle.quantize_q4_1(x), golden["edge__q41"])


def test_matmul_thread_count_invariance(oracle):
    rng = np.random.default_rng(3)
    m, k, n = 5, 256, 37
    x = rng.normal(size=m * k).astype(np.float32)
    w = oracle.quantize_q4_0(rng.normal(0, 0.02, n * k).astype(np.float32))
    t0 = oracle.threads()
    oracle.set_threads(1)
    a = oracle.matmul_f32_q4(x, w, m, k, n)
    oracle.set_threads(max(t0, 2))
    b = oracle.matmul_f32_q4(x, w, m, k, n)
    oracle.set_threads(t0)
    np.testing.assert_array_equal(a.view(np.uint32), b.view(np.uint32))


# ---- f16 (the `half` crate's from_f32, not vendored in the reference) --------------------

def test_f16_rne_matches_numpy_and_f16c(oracle):
    rng = np.random.default_rng(0)
    bits = rng.integers(0, 2**32, size=1 << 20, dtype=np.uint64).astype(np.uint32)
    # add every f16 rounding boundary region: halfway points around each f16 value
    h = np.arange(0, 1 << 15, dtype=np.uint32).astype(np.uint16).view(np.float16).astype(np.float32)
    h = h[np.isfinite(h)]
    ulp = np.spacing(h.astype(np.float16)).astype(np.float32)
    mids = np.concatenate([h + ulp / 2, -(h + ulp / 2), np.nextafter(h + ulp / 2, np.float32(np.inf))])
    x = np.concatenate([bits.view(np.float32), mids.astype(np.float32)])
    x = x[~np.isnan(x)]
    sw = oracle.f32_to_f16_bits(x)
    with np.errstate(over="ignore"):
        ref = x.astype(np.float16).view(np.uint16)
    np.testing.assert_array_equal(sw, ref)
    np.testing.assert_array_equal(oracle.f32_to_f16_bits_f16c(x), ref)
