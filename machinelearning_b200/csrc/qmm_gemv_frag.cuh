// Register-level building blocks shared by the GEMV kernels (qmm_gemv.cu: the
// streaming kernel; qmm_gemv_resident.cu: the resident small-shape kernel).
//
// A warp works on 32-row weight tiles as two 16-row MMA groups. Per 32-element
// block a lane dequantises its A fragments in registers (f16 magic-number
// trick for f32 activations, raw/offset int8 for Q8_0 activations) and runs
// mma.sync against activation fragments (B) laid out by the x-prep, starting
// from a precomputed accumulator value; per-block scales are applied in f32.
#pragma once

#include <cstdint>

#include "qmm_common.cuh"

namespace qmm {

constexpr int kW = 8;       // warps per CTA
constexpr int kRows = 32;   // weight rows per warp tile (two MMA row groups)
constexpr int kThreads = 32 * kW;
constexpr int kChunk = 8;   // blocks per TMA box along K (16-byte aligned starts)

// kLoaderTma2d:    row pitch % 16 == 0: one [32 rows x kc blocks] TMA tile per stage.
// kLoaderTmaPairs: row pitch % 16 == 8 (e.g. K = 1152), N even: the matrix is
//                  viewed as [N/2][2 * row_bytes] (16-byte pitched); even rows
//                  and odd rows come as two [16 x (kc blocks + pad)] tiles,
//                  the odd ones starting 8 bytes early (skew 8 in shared memory).
// kLoaderCpAsync:  anything else: 16-byte cp.async pieces of each row window.
enum Loader : int { kLoaderTma2d = 0, kLoaderCpAsync = 1, kLoaderTmaPairs = 2 };

// Shared-memory address of row j (0..31) of a stage filled by a TMA loader.
template <int LOADER>
__device__ __forceinline__ const uint8_t* stage_row(const uint8_t* sbase, int j, int pitch) {
    if constexpr (LOADER == kLoaderTmaPairs) return sbase + ((j & 1) * (kRows / 2) + (j >> 1)) * pitch + (j & 1) * 8;
    return sbase + j * pitch;
}

// ---- MMA with a separate accumulator input ------------------------------------------
__device__ __forceinline__ void mma_f16_c(float (&d)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1,
                                          const float (&c)[4]) {
    asm("mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
        "{%10,%11,%12,%13};"
        : "=f"(d[0]), "=f"(d[1]), "=f"(d[2]), "=f"(d[3])
        : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1), "f"(c[0]), "f"(c[1]), "f"(c[2]),
          "f"(c[3]));
}
__device__ __forceinline__ void mma_s8_c(int (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                                         uint32_t b0, uint32_t b1, const int (&c)[4]) {
    asm("mma.sync.aligned.m16n8k32.row.col.s32.s8.s8.s32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
        "{%10,%11,%12,%13};"
        : "=r"(d[0]), "=r"(d[1]), "=r"(d[2]), "=r"(d[3])
        : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1), "r"(c[0]), "r"(c[1]), "r"(c[2]), "r"(c[3]));
}

// Activation fragments of one block for one 8-token tile.
struct XFrag {
    uint4 hi, lo;  // f32 mode: B fragments (hi and lo halves); native: hi.x/.y = s8 B fragment
    uint4 c4;      // accumulator start for this lane's tokens (2t, 2t+1): {c0, c1, c0, c1}
    uint4 s4;      // f32: {s0, s1, sx0, sx1}; native: {xs0, xs1, qsum0, qsum1}
};

// 4 payload bytes at p: AL = known 4-byte aligned (one 32-bit load).
template <bool AL>
__device__ __forceinline__ uint32_t ld_word(const uint8_t* p) {
    if constexpr (AL) return *reinterpret_cast<const uint32_t*>(p);
    return lds_u32_a2(p);
}

// One block of one 16-row group (rows g and g+8 at shared pointers r0/r1).
// AL: the block's payload (the bytes after the f16 header) is 4-byte aligned.
// Lane t covers payload words t and t+4 of each row (elements 4t..4t+3 and
// 16+4t..16+4t+3 for Q8_0; nibble bytes 4t..4t+3 for Q4): per shared load the
// 8 rows x 4 words of a warp fall in distinct banks (row pitch = 4 mod 32 words).
// SPLIT (f32 mode): the hi and lo halves accumulate in two independent chains
// of two MMAs that are added at the end, instead of one chain of four -- half
// the dependent latency, for latency-bound callers.
template <int QT, int NT, bool NATIVE, bool AL, bool SPLIT = false>
__device__ __forceinline__ void consume_group(const uint8_t* r0, const uint8_t* r1, int t, const XFrag (&x)[NT],
                                              float (&acc)[NT][4]) {
    const float d0 = f16_bits_to_f32((uint16_t)lds_u16(r0));
    const float d1 = f16_bits_to_f32((uint16_t)lds_u16(r1));
    float m0 = 0.0f, m1 = 0.0f;
    if constexpr (QT == kQ4_1) {
        m0 = f16_bits_to_f32((uint16_t)lds_u16(r0 + 2));
        m1 = f16_bits_to_f32((uint16_t)lds_u16(r1 + 2));
    }
    constexpr int NOFF = (QT == kQ4_1) ? 4 : 2;
    if constexpr (!NATIVE) {
        uint32_t A0[4], A1[4];  // fragments of the two k16 MMAs of this block
        if constexpr (QT == kQ8_0) {
            const uint32_t u00 = ld_word<AL>(r0 + NOFF + 4 * t) ^ 0x80808080u;
            const uint32_t u01 = ld_word<AL>(r0 + NOFF + 16 + 4 * t) ^ 0x80808080u;
            const uint32_t u10 = ld_word<AL>(r1 + NOFF + 4 * t) ^ 0x80808080u;
            const uint32_t u11 = ld_word<AL>(r1 + NOFF + 16 + 4 * t) ^ 0x80808080u;
            // halves (1024 + (q + 128)) = 1152 + q, exact
            A0[0] = __byte_perm(u00, 0x64646464u, 0x4140);
            A0[1] = __byte_perm(u10, 0x64646464u, 0x4140);
            A0[2] = __byte_perm(u00, 0x64646464u, 0x4342);
            A0[3] = __byte_perm(u10, 0x64646464u, 0x4342);
            A1[0] = __byte_perm(u01, 0x64646464u, 0x4140);
            A1[1] = __byte_perm(u11, 0x64646464u, 0x4140);
            A1[2] = __byte_perm(u01, 0x64646464u, 0x4342);
            A1[3] = __byte_perm(u11, 0x64646464u, 0x4342);
        } else {
            const uint32_t w0 = ld_word<AL>(r0 + NOFF + 4 * t);
            const uint32_t w1 = ld_word<AL>(r1 + NOFF + 4 * t);
            const uint32_t w0s = w0 >> 8, w1s = w1 >> 8;
            // low nibbles -> 1024 + n ; high nibbles -> 1024 + 16 n (activations pre-divided by 16)
            A0[0] = lop3_and_or(w0, 0x000F000Fu, 0x64006400u);
            A0[1] = lop3_and_or(w1, 0x000F000Fu, 0x64006400u);
            A0[2] = lop3_and_or(w0s, 0x000F000Fu, 0x64006400u);
            A0[3] = lop3_and_or(w1s, 0x000F000Fu, 0x64006400u);
            A1[0] = lop3_and_or(w0, 0x00F000F0u, 0x64006400u);
            A1[1] = lop3_and_or(w1, 0x00F000F0u, 0x64006400u);
            A1[2] = lop3_and_or(w0s, 0x00F000F0u, 0x64006400u);
            A1[3] = lop3_and_or(w1s, 0x00F000F0u, 0x64006400u);
        }
#pragma unroll
        for (int nt = 0; nt < NT; ++nt) {
            const float c0[4] = {__uint_as_float(x[nt].c4.x), __uint_as_float(x[nt].c4.y),
                                 __uint_as_float(x[nt].c4.z), __uint_as_float(x[nt].c4.w)};
            float c[4], e[4], f[4], h[4];
            if constexpr (SPLIT) {
                const float z[4] = {0.0f, 0.0f, 0.0f, 0.0f};
                float q[4];
                mma_f16_c(c, A0, x[nt].hi.x, x[nt].hi.y, c0);
                mma_f16_c(f, A0, x[nt].lo.x, x[nt].lo.y, z);
                mma_f16_c(e, A1, x[nt].hi.z, x[nt].hi.w, c);
                mma_f16_c(q, A1, x[nt].lo.z, x[nt].lo.w, f);
#pragma unroll
                for (int i = 0; i < 4; ++i) h[i] = e[i] + q[i];
            } else {
                mma_f16_c(c, A0, x[nt].hi.x, x[nt].hi.y, c0);
                mma_f16_c(e, A1, x[nt].hi.z, x[nt].hi.w, c);
                mma_f16_c(f, A0, x[nt].lo.x, x[nt].lo.y, e);
                mma_f16_c(h, A1, x[nt].lo.z, x[nt].lo.w, f);
            }
            const float s0 = __uint_as_float(x[nt].s4.x), s1 = __uint_as_float(x[nt].s4.y);
            if constexpr (QT == kQ4_1) {
                const float sx0 = __uint_as_float(x[nt].s4.z), sx1 = __uint_as_float(x[nt].s4.w);
                acc[nt][0] = fmaf(s0, fmaf(d0, h[0], m0 * sx0), acc[nt][0]);
                acc[nt][1] = fmaf(s1, fmaf(d0, h[1], m0 * sx1), acc[nt][1]);
                acc[nt][2] = fmaf(s0, fmaf(d1, h[2], m1 * sx0), acc[nt][2]);
                acc[nt][3] = fmaf(s1, fmaf(d1, h[3], m1 * sx1), acc[nt][3]);
            } else {
                acc[nt][0] = fmaf(d0 * s0, h[0], acc[nt][0]);
                acc[nt][1] = fmaf(d0 * s1, h[1], acc[nt][1]);
                acc[nt][2] = fmaf(d1 * s0, h[2], acc[nt][2]);
                acc[nt][3] = fmaf(d1 * s1, h[3], acc[nt][3]);
            }
        }
    } else {
        uint32_t a0, a1, a2, a3;
        if constexpr (QT == kQ8_0) {
            a0 = ld_word<AL>(r0 + NOFF + 4 * t);
            a2 = ld_word<AL>(r0 + NOFF + 16 + 4 * t);
            a1 = ld_word<AL>(r1 + NOFF + 4 * t);
            a3 = ld_word<AL>(r1 + NOFF + 16 + 4 * t);
        } else {
            const uint32_t w0 = ld_word<AL>(r0 + NOFF + 4 * t);
            const uint32_t w1 = ld_word<AL>(r1 + NOFF + 4 * t);
            a0 = w0 & 0x0F0F0F0Fu;
            a1 = w1 & 0x0F0F0F0Fu;
            a2 = (w0 >> 4) & 0x0F0F0F0Fu;
            a3 = (w1 >> 4) & 0x0F0F0F0Fu;
        }
#pragma unroll
        for (int nt = 0; nt < NT; ++nt) {
            const int c0[4] = {(int)x[nt].c4.x, (int)x[nt].c4.y, (int)x[nt].c4.z, (int)x[nt].c4.w};
            int c[4];
            mma_s8_c(c, a0, a1, a2, a3, x[nt].hi.x, x[nt].hi.y, c0);
            const float xs0 = __uint_as_float(x[nt].s4.x), xs1 = __uint_as_float(x[nt].s4.y);
            if constexpr (QT == kQ4_1) {
                const int qs0 = (int)x[nt].s4.z, qs1 = (int)x[nt].s4.w;
                // q8_scales[b] * (d * unsigned_dot + m * q8_sum)   (quantize.rs:1001)
                acc[nt][0] = __fadd_rn(acc[nt][0], __fmul_rn(xs0, __fadd_rn(__fmul_rn(d0, (float)c[0]), __fmul_rn(m0, (float)qs0))));
                acc[nt][1] = __fadd_rn(acc[nt][1], __fmul_rn(xs1, __fadd_rn(__fmul_rn(d0, (float)c[1]), __fmul_rn(m0, (float)qs1))));
                acc[nt][2] = __fadd_rn(acc[nt][2], __fmul_rn(xs0, __fadd_rn(__fmul_rn(d1, (float)c[2]), __fmul_rn(m1, (float)qs0))));
                acc[nt][3] = __fadd_rn(acc[nt][3], __fmul_rn(xs1, __fadd_rn(__fmul_rn(d1, (float)c[3]), __fmul_rn(m1, (float)qs1))));
            } else {
                // (int_dot as f32) * act_scale * w_scale   (quantize.rs:481, 706)
                acc[nt][0] = __fadd_rn(acc[nt][0], __fmul_rn(__fmul_rn((float)c[0], xs0), d0));
                acc[nt][1] = __fadd_rn(acc[nt][1], __fmul_rn(__fmul_rn((float)c[1], xs1), d0));
                acc[nt][2] = __fadd_rn(acc[nt][2], __fmul_rn(__fmul_rn((float)c[2], xs0), d1));
                acc[nt][3] = __fadd_rn(acc[nt][3], __fmul_rn(__fmul_rn((float)c[3], xs1), d1));
            }
        }
    }
}

// Packed form for up to 4 tokens (f32 activations): the 8 MMA columns carry
// (token, half) pairs, column 2m the hi half of token m and column 2m + 1 its
// lo half, so one chain of two MMAs per block covers both halves. Lane (g, t)
// supplies column g (xb: token g >> 1's hi or lo record) and receives token
// t's two halves for rows g and g + 8, added into acc[0] / acc[1]. c: the
// accumulator start of token t's hi column (-corr), s: its scale 2^e, sx:
// its block sum (Q4_1). Same products and per-block terms as consume_group.
template <int QT, bool AL>
__device__ __forceinline__ void consume_group_packed(const uint8_t* r0, const uint8_t* r1, int t, uint4 xb, float c,
                                                     float s, float sx, float (&acc)[2]) {
    const float d0 = f16_bits_to_f32((uint16_t)lds_u16(r0));
    const float d1 = f16_bits_to_f32((uint16_t)lds_u16(r1));
    constexpr int NOFF = (QT == kQ4_1) ? 4 : 2;
    uint32_t A0[4], A1[4];
    if constexpr (QT == kQ8_0) {
        const uint32_t u00 = ld_word<AL>(r0 + NOFF + 4 * t) ^ 0x80808080u;
        const uint32_t u01 = ld_word<AL>(r0 + NOFF + 16 + 4 * t) ^ 0x80808080u;
        const uint32_t u10 = ld_word<AL>(r1 + NOFF + 4 * t) ^ 0x80808080u;
        const uint32_t u11 = ld_word<AL>(r1 + NOFF + 16 + 4 * t) ^ 0x80808080u;
        A0[0] = __byte_perm(u00, 0x64646464u, 0x4140);
        A0[1] = __byte_perm(u10, 0x64646464u, 0x4140);
        A0[2] = __byte_perm(u00, 0x64646464u, 0x4342);
        A0[3] = __byte_perm(u10, 0x64646464u, 0x4342);
        A1[0] = __byte_perm(u01, 0x64646464u, 0x4140);
        A1[1] = __byte_perm(u11, 0x64646464u, 0x4140);
        A1[2] = __byte_perm(u01, 0x64646464u, 0x4342);
        A1[3] = __byte_perm(u11, 0x64646464u, 0x4342);
    } else {
        const uint32_t w0 = ld_word<AL>(r0 + NOFF + 4 * t);
        const uint32_t w1 = ld_word<AL>(r1 + NOFF + 4 * t);
        const uint32_t w0s = w0 >> 8, w1s = w1 >> 8;
        A0[0] = lop3_and_or(w0, 0x000F000Fu, 0x64006400u);
        A0[1] = lop3_and_or(w1, 0x000F000Fu, 0x64006400u);
        A0[2] = lop3_and_or(w0s, 0x000F000Fu, 0x64006400u);
        A0[3] = lop3_and_or(w1s, 0x000F000Fu, 0x64006400u);
        A1[0] = lop3_and_or(w0, 0x00F000F0u, 0x64006400u);
        A1[1] = lop3_and_or(w1, 0x00F000F0u, 0x64006400u);
        A1[2] = lop3_and_or(w0s, 0x00F000F0u, 0x64006400u);
        A1[3] = lop3_and_or(w1s, 0x00F000F0u, 0x64006400u);
    }
    const float c0[4] = {c, 0.0f, c, 0.0f};
    float e[4], h[4];
    mma_f16_c(e, A0, xb.x, xb.y, c0);
    mma_f16_c(h, A1, xb.z, xb.w, e);
    const float v0 = h[0] + h[1], v1 = h[2] + h[3];  // hi + lo, rows g and g + 8
    if constexpr (QT == kQ4_1) {
        const float m0 = f16_bits_to_f32((uint16_t)lds_u16(r0 + 2));
        const float m1 = f16_bits_to_f32((uint16_t)lds_u16(r1 + 2));
        acc[0] = fmaf(s, fmaf(d0, v0, m0 * sx), acc[0]);
        acc[1] = fmaf(s, fmaf(d1, v1, m1 * sx), acc[1]);
    } else {
        acc[0] = fmaf(d0 * s, v0, acc[0]);
        acc[1] = fmaf(d1 * s, v1, acc[1]);
    }
}

// ---- shared loads at a 32-bit address plus a compile-time offset ---------------------
// Volatile (kept in order with the mbarrier waits, which are volatile too) but
// without a memory clobber, so independent arithmetic can move around them.
template <int OFF>
__device__ __forceinline__ uint32_t lds16_at(uint32_t a) {
    uint16_t v;
    asm volatile("ld.shared.u16 %0, [%1+%2];" : "=h"(v) : "r"(a), "n"(OFF));
    return v;
}
template <int OFF>
__device__ __forceinline__ uint32_t lds32_at(uint32_t a) {
    uint32_t v;
    asm volatile("ld.shared.u32 %0, [%1+%2];" : "=r"(v) : "r"(a), "n"(OFF));
    return v;
}
// 4 bytes at a + OFF: AL = 4-byte aligned, else 2-byte aligned (two halves).
template <int OFF, bool AL>
__device__ __forceinline__ uint32_t ldsw_at(uint32_t a) {
    if constexpr (AL) return lds32_at<OFF>(a);
    return __byte_perm(lds16_at<OFF>(a), lds16_at<OFF + 2>(a), 0x5410);
}
// 16 bytes at a + OFF into x when p (x unchanged otherwise).
template <int OFF>
__device__ __forceinline__ void lds128_at_if(uint4& x, uint32_t a, bool p) {
    asm volatile(
        "{\n\t.reg .pred q;\n\tsetp.ne.u32 q, %4, 0;\n\t"
        "@q ld.shared.v4.u32 {%0, %1, %2, %3}, [%5+%6];\n\t}"
        : "+r"(x.x), "+r"(x.y), "+r"(x.z), "+r"(x.w)
        : "r"((uint32_t)p), "r"(a), "n"(OFF));
}

// consume_group_packed on 32-bit shared addresses: rg / rg8 are the stage
// addresses of rows g / g + 8 at the chunk's first block, OFF the block's byte
// offset in the row, rgt / rg8t the same plus the lane's payload word (4t).
template <int QT, bool AL, int OFF>
__device__ __forceinline__ void consume_group_packed_sa(uint32_t rg, uint32_t rg8, uint32_t rgt, uint32_t rg8t,
                                                        uint4 xb, float c, float s, float sx, float (&acc)[2]) {
    const float d0 = f16_bits_to_f32((uint16_t)lds16_at<OFF>(rg));
    const float d1 = f16_bits_to_f32((uint16_t)lds16_at<OFF>(rg8));
    constexpr int NOFF = (QT == kQ4_1) ? 4 : 2;
    uint32_t A0[4], A1[4];
    if constexpr (QT == kQ8_0) {
        const uint32_t u00 = ldsw_at<OFF + NOFF, AL>(rgt) ^ 0x80808080u;
        const uint32_t u01 = ldsw_at<OFF + NOFF + 16, AL>(rgt) ^ 0x80808080u;
        const uint32_t u10 = ldsw_at<OFF + NOFF, AL>(rg8t) ^ 0x80808080u;
        const uint32_t u11 = ldsw_at<OFF + NOFF + 16, AL>(rg8t) ^ 0x80808080u;
        A0[0] = __byte_perm(u00, 0x64646464u, 0x4140);
        A0[1] = __byte_perm(u10, 0x64646464u, 0x4140);
        A0[2] = __byte_perm(u00, 0x64646464u, 0x4342);
        A0[3] = __byte_perm(u10, 0x64646464u, 0x4342);
        A1[0] = __byte_perm(u01, 0x64646464u, 0x4140);
        A1[1] = __byte_perm(u11, 0x64646464u, 0x4140);
        A1[2] = __byte_perm(u01, 0x64646464u, 0x4342);
        A1[3] = __byte_perm(u11, 0x64646464u, 0x4342);
    } else {
        const uint32_t w0 = ldsw_at<OFF + NOFF, AL>(rgt);
        const uint32_t w1 = ldsw_at<OFF + NOFF, AL>(rg8t);
        const uint32_t w0s = w0 >> 8, w1s = w1 >> 8;
        A0[0] = lop3_and_or(w0, 0x000F000Fu, 0x64006400u);
        A0[1] = lop3_and_or(w1, 0x000F000Fu, 0x64006400u);
        A0[2] = lop3_and_or(w0s, 0x000F000Fu, 0x64006400u);
        A0[3] = lop3_and_or(w1s, 0x000F000Fu, 0x64006400u);
        A1[0] = lop3_and_or(w0, 0x00F000F0u, 0x64006400u);
        A1[1] = lop3_and_or(w1, 0x00F000F0u, 0x64006400u);
        A1[2] = lop3_and_or(w0s, 0x00F000F0u, 0x64006400u);
        A1[3] = lop3_and_or(w1s, 0x00F000F0u, 0x64006400u);
    }
    const float c0[4] = {c, 0.0f, c, 0.0f};
    float e[4], h[4];
    mma_f16_c(e, A0, xb.x, xb.y, c0);
    mma_f16_c(h, A1, xb.z, xb.w, e);
    const float v0 = h[0] + h[1], v1 = h[2] + h[3];  // hi + lo, rows g and g + 8
    if constexpr (QT == kQ4_1) {
        const float m0 = f16_bits_to_f32((uint16_t)lds16_at<OFF + 2>(rg));
        const float m1 = f16_bits_to_f32((uint16_t)lds16_at<OFF + 2>(rg8));
        acc[0] = fmaf(s, fmaf(d0, v0, m0 * sx), acc[0]);
        acc[1] = fmaf(s, fmaf(d1, v1, m1 * sx), acc[1]);
    } else {
        acc[0] = fmaf(d0 * s, v0, acc[0]);
        acc[1] = fmaf(d1 * s, v1, acc[1]);
    }
}

}  // namespace qmm
