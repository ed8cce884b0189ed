"""Generates tests/golden/golden.npz: small seeded golden vectors for the
quantized-matmul path, computed by an independent pure-numpy restatement of
the reference (NOT by the C++ oracle, which these vectors then pin).

Reference (paths inside sweengineeringlabs/machinelearning):
  llmserve/llmmodel/kernel/main/src/core/quantize.rs  quantizers + matmuls
  llmserve/llmmodel/kernel/main/src/core/simd.rs      x86 AVX2(+FMA) block dots
  main/features/tensor/src/core/tensor/tensor.rs      to_f32 dequantisation

Every float operation below is a numpy float32 scalar/array operation (IEEE
single, round to nearest even, one rounding per operation, no FMA), arranged
in the AVX2 summation order the reference uses on an AVX2+FMA host. f16
conversions use numpy's float16 (IEEE round-to-nearest-even), which is what
the `half` crate implements. Pure Python loops: small shapes only.

    python tests/golden/make_golden.py     # rewrites golden.npz
"""
from __future__ import annotations

import os

import numpy as np

F = np.float32
HERE = os.path.dirname(os.path.abspath(__file__))


def f16(v) -> np.uint16:
    return np.array([v], dtype=np.float32).astype(np.float16).view(np.uint16)[0]


def f16f(bits) -> np.float32:
    return F(np.array([bits], dtype=np.uint16).view(np.float16)[0])


def rnd(v: np.float32) -> float:
    # Rust f32::round: half away from zero
    v = float(v)
    if np.isnan(v):
        return v
    return float(np.sign(v) * np.floor(abs(v) + 0.5)) if abs(v) % 1.0 == 0.5 else float(np.round(v))


def q_i8(v, lo, hi) -> int:
    r = rnd(v)
    if np.isnan(r):
        return 0
    return int(min(max(r, lo), hi))


def amax_of(block) -> np.float32:
    a = F(0.0)
    for v in block:
        av = F(abs(v))
        if not np.isnan(av) and av > a:
            a = av
    return a


def quantize_q8_0(x, rounded_inv=False):
    """quantize.rs:15-48 (rounded_inv=False) / quantize_row_q8_0 :260-289 (True)."""
    x = np.asarray(x, dtype=F)
    out, scales = [], []
    for b in range(x.size // 32):
        blk = x[32 * b:32 * b + 32]
        amax = amax_of(blk)
        scale = F(0.0) if amax == 0 else F(amax / F(127.0))
        h = f16(scale)
        srt = f16f(h)
        sdiv = srt if rounded_inv else scale
        inv = F(0.0) if sdiv == 0 else F(F(1.0) / sdiv)
        out += [int(h) & 0xFF, int(h) >> 8]
        out += [q_i8(F(v * inv), -128, 127) & 0xFF for v in blk]
        scales.append(srt)
    return np.array(out, dtype=np.uint8), np.array(scales, dtype=F)


def quantize_q4_0(x):
    """quantize.rs:124-165 (interleaved nibble packing)."""
    x = np.asarray(x, dtype=F)
    out = []
    for b in range(x.size // 32):
        blk = x[32 * b:32 * b + 32]
        amax = amax_of(blk)
        scale = F(0.0) if amax == 0 else F(amax / F(8.0))
        inv = F(0.0) if scale == 0 else F(F(1.0) / scale)
        h = f16(scale)
        out += [int(h) & 0xFF, int(h) >> 8]
        for i in range(16):
            e = q_i8(F(blk[2 * i] * inv), -8, 7) + 8
            o = q_i8(F(blk[2 * i + 1] * inv), -8, 7) + 8
            out.append(((o << 4) | (e & 0xF)) & 0xFF)
    return np.array(out, dtype=np.uint8)


def quantize_q4_1(x):
    """quantize.rs:207-251."""
    x = np.asarray(x, dtype=F)
    out = []
    for b in range(x.size // 32):
        blk = x[32 * b:32 * b + 32]
        mn, mx = F(np.inf), F(-np.inf)
        for v in blk:
            if not np.isnan(v):
                mn = min(mn, v)
                mx = max(mx, v)
        d = F(F(mx - mn) / F(15.0))
        inv = F(0.0) if d == 0 else F(F(1.0) / d)
        hd, hm = f16(d), f16(mn)
        out += [int(hd) & 0xFF, int(hd) >> 8, int(hm) & 0xFF, int(hm) >> 8]
        for i in range(16):
            e = q_i8(F(F(blk[2 * i] - mn) * inv), 0, 15)
            o = q_i8(F(F(blk[2 * i + 1] - mn) * inv), 0, 15)
            out.append(((o << 4) | (e & 0xF)) & 0xFF)
    return np.array(out, dtype=np.uint8)


def to_f32(dtype, w, n):
    """tensor.rs:527-630."""
    out = np.zeros(n, dtype=F)
    for b in range(n // 32):
        if dtype == 2:
            blk = w[18 * b:18 * b + 18]
            s = f16f(int(blk[0]) | (int(blk[1]) << 8))
            for j in range(16):
                out[32 * b + j] = F(s * F((int(blk[2 + j]) & 0xF) - 8))
                out[32 * b + j + 16] = F(s * F((int(blk[2 + j]) >> 4) - 8))
        elif dtype == 3:
            blk = w[20 * b:20 * b + 20]
            d = f16f(int(blk[0]) | (int(blk[1]) << 8))
            m = f16f(int(blk[2]) | (int(blk[3]) << 8))
            for j in range(16):
                out[32 * b + j] = F(F(d * F(int(blk[4 + j]) & 0xF)) + m)
                out[32 * b + j + 16] = F(F(d * F(int(blk[4 + j]) >> 4)) + m)
        else:
            blk = w[34 * b:34 * b + 34]
            s = f16f(int(blk[0]) | (int(blk[1]) << 8))
            for j in range(32):
                out[32 * b + j] = F(s * F(int(np.int8(blk[2 + j]))))
    return out


def hsum8(v):
    # extract high 128 + add, movehdup + add, movehl + add_ss (simd.rs:125-131)
    s4 = [F(v[i] + v[i + 4]) for i in range(4)]
    s2_0 = F(s4[0] + s4[1])
    s2_2 = F(s4[2] + s4[3])
    return F(s2_0 + s2_2)


def tree4(p):
    # acc_c = chunk c (8 lanes); (a0+a1)+(a2+a3) lane-wise; then hsum8
    lanes = [F(F(p[l] + p[8 + l]) + F(p[16 + l] + p[24 + l])) for l in range(8)]
    return hsum8(lanes)


def dot_q8_block(x, q, scale):
    """simd.rs:87-134 (AVX2+FMA): fma(x, q, +0) per lane, tree, hsum, * scale."""
    p = [F(F(x[i] * F(q[i])) + F(0.0)) for i in range(32)]
    return F(tree4(p) * scale)


def dot_q4_block(x, packed, scale):
    """simd.rs:210-252 (AVX2): GGML-order unpack, mul, tree, hsum, * scale."""
    w = [F((int(packed[j]) & 0xF) - 8) for j in range(16)] + [F((int(packed[j]) >> 4) - 8) for j in range(16)]
    p = [F(x[i] * w[i]) for i in range(32)]
    return F(tree4(p) * scale)


def matmul(kind, x, w, m, k, n):
    x = np.asarray(x, dtype=F).reshape(m, k)
    nb = k // 32
    y = np.zeros((m, n), dtype=F)
    if kind in ("q8_v2",):
        xq, _ = quantize_q8_0(x.ravel(), rounded_inv=False)
    if kind in ("q4_native", "q4_1_native"):
        xq, xs = quantize_q8_0(x.ravel(), rounded_inv=True)
    for r in range(m):
        for c in range(n):
            dot = F(0.0)
            for b in range(nb):
                if kind == "q8":
                    blk = w[(c * nb + b) * 34:(c * nb + b + 1) * 34]
                    s = f16f(int(blk[0]) | (int(blk[1]) << 8))
                    dot = F(dot + dot_q8_block(x[r, 32 * b:32 * b + 32], blk[2:].view(np.int8), s))
                elif kind == "q8_v2":
                    wb = w[(c * nb + b) * 34:(c * nb + b + 1) * 34]
                    ab = xq[(r * nb + b) * 34:(r * nb + b + 1) * 34]
                    a_s = f16f(int(ab[0]) | (int(ab[1]) << 8))
                    w_s = f16f(int(wb[0]) | (int(wb[1]) << 8))
                    idot = int(np.dot(ab[2:].view(np.int8).astype(np.int64), wb[2:].view(np.int8).astype(np.int64)))
                    dot = F(dot + F(F(F(idot) * a_s) * w_s))
                elif kind == "q4":
                    blk = w[(c * nb + b) * 18:(c * nb + b + 1) * 18]
                    s = f16f(int(blk[0]) | (int(blk[1]) << 8))
                    dot = F(dot + dot_q4_block(x[r, 32 * b:32 * b + 32], blk[2:], s))
                elif kind == "q4_native":
                    blk = w[(c * nb + b) * 18:(c * nb + b + 1) * 18]
                    w_s = f16f(int(blk[0]) | (int(blk[1]) << 8))
                    q8 = xq[(r * nb + b) * 34 + 2:(r * nb + b + 1) * 34].view(np.int8).astype(np.int64)
                    nib = np.array([(int(v) & 0xF) - 8 for v in blk[2:]] + [(int(v) >> 4) - 8 for v in blk[2:]])
                    idot = int(np.dot(nib, q8))
                    dot = F(dot + F(F(F(idot) * xs[r * nb + b]) * w_s))
                elif kind == "q4_1":
                    blk = w[(c * nb + b) * 20:(c * nb + b + 1) * 20]
                    d = f16f(int(blk[0]) | (int(blk[1]) << 8))
                    mv = f16f(int(blk[2]) | (int(blk[3]) << 8))
                    xb = x[r, 32 * b:32 * b + 32]
                    bd, xsum = F(0.0), F(0.0)
                    for j in range(16):
                        bd = F(bd + F(xb[j] * F(int(blk[4 + j]) & 0xF)))
                        bd = F(bd + F(xb[j + 16] * F(int(blk[4 + j]) >> 4)))
                        xsum = F(xsum + xb[j])
                        xsum = F(xsum + xb[j + 16])
                    dot = F(dot + F(F(d * bd) + F(mv * xsum)))
                elif kind == "q4_1_native":
                    blk = w[(c * nb + b) * 20:(c * nb + b + 1) * 20]
                    d = f16f(int(blk[0]) | (int(blk[1]) << 8))
                    mv = f16f(int(blk[2]) | (int(blk[3]) << 8))
                    q8 = xq[(r * nb + b) * 34 + 2:(r * nb + b + 1) * 34].view(np.int8).astype(np.int64)
                    nib = np.array([int(v) & 0xF for v in blk[4:]] + [int(v) >> 4 for v in blk[4:]])
                    ud, qs = int(np.dot(nib, q8)), int(q8.sum())
                    dot = F(dot + F(xs[r * nb + b] * F(F(d * F(ud)) + F(mv * F(qs)))))
            y[r, c] = dot
    return y.ravel()


CASES = [  # (name, weight dtype, kind, m, k, n, seed)
    ("q8_m1", 8, "q8", 1, 64, 9, 11),
    ("q8_m5", 8, "q8", 5, 96, 7, 12),
    ("q8v2_m3", 8, "q8_v2", 3, 128, 8, 13),
    ("q4_m1", 2, "q4", 1, 64, 9, 14),
    ("q4_m6", 2, "q4", 6, 96, 5, 15),
    ("q4n_m2", 2, "q4_native", 2, 128, 6, 16),
    ("q41_m2", 3, "q4_1", 2, 64, 7, 17),
    ("q41n_m3", 3, "q4_1_native", 3, 64, 5, 18),
]


def main():
    out = {}
    for name, dt, kind, m, k, n, seed in CASES:
        rng = np.random.default_rng(seed)
        wf = rng.normal(0.0, 0.02, n * k).astype(F)
        x = rng.normal(0.0, 1.0, m * k).astype(F)
        if dt == 8:
            w, _ = quantize_q8_0(wf)
        elif dt == 2:
            w = quantize_q4_0(wf)
        else:
            w = quantize_q4_1(wf)
        out[f"{name}__w"] = w
        out[f"{name}__x"] = x
        out[f"{name}__y"] = matmul(kind, x, w, m, k, n)
        out[f"{name}__deq"] = to_f32(dt, w, n * k)
    # quantiser edge cases: ties, zeros, subnormals, large values
    edge = np.array(
        [0.0] * 32
        + [((i - 16) * 0.5) for i in range(32)]
        + [1e-40 * (i + 1) for i in range(32)]
        + [((-1) ** i) * 1e30 * (i + 1) for i in range(32)]
        + [(i - 32) / 10.0 for i in range(64)],
        dtype=F)
    out["edge__x"] = edge
    out["edge__q8"], _ = quantize_q8_0(edge)
    out["edge__rowq8"], out["edge__rowq8_scales"] = quantize_q8_0(edge, rounded_inv=True)
    out["edge__q4"] = quantize_q4_0(edge)
    out["edge__q41"] = quantize_q4_1(edge)
    out["cases"] = np.array([f"{c[0]}:{c[1]}:{c[2]}:{c[3]}:{c[4]}:{c[5]}" for c in CASES])
    np.savez_compressed(os.path.join(HERE, "golden.npz"), **out)
    print("wrote", os.path.join(HERE, "golden.npz"), len(out), "arrays")


if __name__ == "__main__":
    main()
