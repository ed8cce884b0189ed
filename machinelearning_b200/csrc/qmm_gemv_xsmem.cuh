// Device pieces shared by the GEMV kernels that keep their activations in
// shared memory (qmm_gemv_resident.cu, qmm_gemv_band.cu): cluster helpers and
// the in-CTA activation preparation.
#pragma once

#include <cuda_fp16.h>

#include <cstdint>

#include "qmm_common.cuh"
#include "qmm_gemv_frag.cuh"
#include "qmm_kernels.cuh"

namespace qmm {

__device__ __forceinline__ uint32_t cluster_ctarank() {
    uint32_t r;
    asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
    return r;
}
__device__ __forceinline__ uint32_t cluster_id_x() {
    uint32_t r;
    asm volatile("mov.u32 %0, %%clusterid.x;" : "=r"(r));
    return r;
}
// Every thread of every CTA of the cluster: release this CTA's shared-memory
// writes, acquire the others'.
__device__ __forceinline__ void cluster_sync() {
    asm volatile(
        "barrier.cluster.arrive.release.aligned;\n\t"
        "barrier.cluster.wait.acquire.aligned;" ::
            : "memory");
}
// The f32 at the same shared-memory offset as `local` in CTA `rank` of the cluster.
__device__ __forceinline__ float ld_cluster_f32(const float* local, uint32_t rank) {
    uint32_t ra;
    float v;
    asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(ra) : "r"(smem_u32(local)), "r"(rank));
    asm volatile("ld.shared::cluster.f32 %0, [%1];" : "=f"(v) : "r"(ra) : "memory");
    return v;
}

__device__ __forceinline__ uint32_t h2_bits(__half2 h) { return *reinterpret_cast<const uint32_t*>(&h); }

// 2^n as an exact f32 for n in [-127, 127] (2^-127 is subnormal).
__device__ __forceinline__ float exp2_int(int n) {
    return n >= -126 ? __int_as_float((n + 127) << 23) : __int_as_float(0x00400000);
}
// The exponent E with a = f * 2^E, f in [0.5, 1), for finite a > 0 (the
// exponent frexpf returns), read from the bits.
__device__ __forceinline__ int frexp_exponent(float a) {
    const int bits = __float_as_int(a);
    const int biased = bits >> 23;
    if (biased != 0) return biased - 126;
    return (31 - __clz(bits)) - 148;  // subnormal: highest set mantissa bit
}

// One (block, token) task of the activation preparation below, spread over
// LPT consecutive lanes: lane q of the task holds elements [q*32/LPT,
// (q+1)*32/LPT) -- G = 8/LPT groups of four. The block maximum and the
// correction sum use the lanes' local values first and shuffles only for the
// last log2(LPT) levels; the sum keeps the pairwise order
// ((c0+c1)+(c2+c3))+((c4+c5)+(c6+c7)) over the groups for every LPT, so the
// records do not depend on LPT. `live` false: the lanes take part in the
// shuffles (a task's lanes share a warp) but store nothing.
template <int QT, int LPT>
__device__ __forceinline__ void prep_x_task(const float* __restrict__ src, bool al16, uint8_t* rec, uint32_t lo_plane,
                                            uint32_t* r8, int q, bool live) {
    constexpr int G = 8 / LPT;
    float v[4 * G];
    if (al16) {
#pragma unroll
        for (int j = 0; j < G; ++j) {
            const float4 f = reinterpret_cast<const float4*>(src)[q * G + j];
            v[4 * j] = f.x;
            v[4 * j + 1] = f.y;
            v[4 * j + 2] = f.z;
            v[4 * j + 3] = f.w;
        }
    } else {
#pragma unroll
        for (int j = 0; j < 4 * G; ++j) v[j] = src[q * 4 * G + j];
    }
    float am = 0.0f;
#pragma unroll
    for (int j = 0; j < 4 * G; ++j) am = fmaxf(am, fabsf(v[j]));
#pragma unroll
    for (int o = 1; o < LPT; o <<= 1) am = fmaxf(am, __shfl_xor_sync(0xffffffffu, am, o));
    int e = 0;
    if (am > 0.0f && am <= 3.402823466e38f) e = max(-126, min(127, frexp_exponent(am) - 14));
    const float s0 = exp2_int(-e);
    // record order inside each group of four: Q8_0 (0,1,2,3), Q4 (0,2,1,3)
    constexpr int P1 = QT == kQ8_0 ? 1 : 2, P2 = QT == kQ8_0 ? 2 : 1;
    float cg[G], sg[G];
#pragma unroll
    for (int j = 0; j < G; ++j) {
        const int gl = q * G + j;    // group: elements 4gl..4gl+3
        const bool upper = gl >= 4;  // elements 16..31
        // Q4 formats: high-nibble elements meet weights pre-multiplied by 16
        // by the magic trick, so their activations are pre-divided by 16.
        // Multiplying by an exact power of two rounds exactly as ldexpf.
        const float scale = s0 * ((QT != kQ8_0 && upper) ? 0.0625f : 1.0f);
        const float coef = QT == kQ8_0 ? 1152.0f : (QT == kQ4_0 ? (upper ? 1152.0f : 1032.0f) : 1024.0f);
        float vv[4];
        vv[0] = v[4 * j] * scale;
        vv[1] = v[4 * j + P1] * scale;
        vv[2] = v[4 * j + P2] * scale;
        vv[3] = v[4 * j + 3] * scale;
        const __half2 h01 = __floats2half2_rn(vv[0], vv[1]), h23 = __floats2half2_rn(vv[2], vv[3]);
        const float2 f01 = __half22float2(h01), f23 = __half22float2(h23);
        const __half2 l01 = __floats2half2_rn(vv[0] - f01.x, vv[1] - f01.y);
        const __half2 l23 = __floats2half2_rn(vv[2] - f23.x, vv[3] - f23.y);
        const float2 g01 = __half22float2(l01), g23 = __half22float2(l23);
        const float rep[4] = {f01.x + g01.x, f01.y + g01.y, f23.x + g23.x, f23.y + g23.y};
        cg[j] = coef * rep[0] + coef * rep[1] + coef * rep[2] + coef * rep[3];
        sg[j] = QT == kQ4_1 ? (rep[0] + rep[1] + rep[2] + rep[3]) * (upper ? 16.0f : 1.0f) : 0.0f;
        if (live) {
            // 16-byte record r holds groups r and r + 4, in the hi plane and
            // in the lo plane
            uint8_t* rp = rec + 16 * (gl & 3) + (upper ? 8 : 0);
            *reinterpret_cast<uint2*>(rp) = make_uint2(h2_bits(h01), h2_bits(h23));
            *reinterpret_cast<uint2*>(rp + lo_plane) = make_uint2(h2_bits(l01), h2_bits(l23));
        }
    }
#pragma unroll
    for (int w = 1; w < G; w <<= 1)
#pragma unroll
        for (int j = 0; j < G; j += 2 * w) {
            cg[j] = cg[j] + cg[j + w];
            sg[j] = sg[j] + sg[j + w];
        }
    float corr = cg[0], sx = sg[0];
#pragma unroll
    for (int o = 1; o < LPT; o <<= 1) {
        corr += __shfl_xor_sync(0xffffffffu, corr, o);
        if (QT == kQ4_1) sx += __shfl_xor_sync(0xffffffffu, sx, o);
    }
    if (live && q == 0) {
        r8[0] = r8[2] = __float_as_uint(-corr);  // the MMA accumulator starts at -corr
        r8[4] = __float_as_uint(exp2_int(e));
        r8[6] = __float_as_uint(sx);
    }
}

// All tasks (block b, token m) = task b*M + m, nthreads / LPT at a time. A
// warp past the last task leaves; in the last round, lanes past it shadow the
// last task without storing (the shuffles need every lane of the warp).
template <int QT, int LPT>
__device__ __forceinline__ void prep_x_lanes(const float* __restrict__ x, int M, int K, int kb0, int ntask, bool al16,
                                             uint8_t* xf, uint32_t lo_plane, uint32_t* side, int npair, int mstride,
                                             int tid, int nthreads) {
    const int per = nthreads / LPT;
    for (int t0 = 0; t0 < ntask; t0 += per) {
        if (t0 + (tid & ~31) / LPT >= ntask) break;  // warp-uniform
        const int task = t0 + tid / LPT;
        const bool live = task < ntask;
        const int tk = live ? task : ntask - 1;
        const int b = tk / M, m = tk - b * M;
        prep_x_task<QT, LPT>(x + (int64_t)m * K + (int64_t)(kb0 + b) * QK, al16, xf + (uint32_t)(b * mstride + m) * 64,
                             lo_plane, side + (b * npair + (m >> 1)) * 8 + (m & 1), tid % LPT, live);
    }
}

// Activation records for blocks [kb0, kb0 + nbc) of x [M][K] (f32), written
// to shared memory by threads tid = 0..nthreads-1 (a multiple of 32) of the
// CTA. Per (block, token): scale by 2^-e so max|x| lands in [2^13, 2^14),
// split into hi = f16(x') and lo = f16(x' - hi); corr is the magic-number
// bias the MMA adds, s = 2^e, sx = block sum (Q4_1). Layout and element order
// as written by xprep_f32_kernel: xf [nbc][M][4] x 16 B (hi plane; the lo
// plane lo_plane bytes further), side [nbc][npair][8 words] with npair token
// pairs per block (npair >= ceil(M / 2)); tokens M..2*npair-1 get neutral side
// records. mstride >= M: tokens per block in the xf planes (records of tokens
// M..mstride-1 are not written). The caller synchronises before reading them.
// Lanes per task by task count (measured on B200: few tasks want short
// per-lane chains, many tasks fewer shuffles); the records are the same.
template <int QT>
__device__ __forceinline__ void prep_x_smem(const float* __restrict__ x, int M, int K, int kb0, int nbc,
                                            uint8_t* xf, uint32_t lo_plane, uint32_t* side, int npair, int tid,
                                            int nthreads, int mstride = 0) {
    if (mstride < M) mstride = M;
    const int npt = 2 * npair - M;  // padding tokens per block: neutral records
    for (int i = tid; i < nbc * npt; i += nthreads) {
        const int b = i / npt, m = M + i % npt;
        uint32_t* r8 = side + (b * npair + (m >> 1)) * 8 + (m & 1);
        r8[0] = r8[2] = r8[4] = r8[6] = 0u;
    }
    const bool al16 = (reinterpret_cast<uintptr_t>(x) & 15) == 0;  // K * 4 is a multiple of 128
    const int ntask = nbc * M;
    if (ntask <= 32)
        prep_x_lanes<QT, 8>(x, M, K, kb0, ntask, al16, xf, lo_plane, side, npair, mstride, tid, nthreads);
    else if (M == 1 && ntask <= 160)
        prep_x_lanes<QT, 4>(x, M, K, kb0, ntask, al16, xf, lo_plane, side, npair, mstride, tid, nthreads);
    else
        prep_x_lanes<QT, 2>(x, M, K, kb0, ntask, al16, xf, lo_plane, side, npair, mstride, tid, nthreads);
}

}  // namespace qmm
