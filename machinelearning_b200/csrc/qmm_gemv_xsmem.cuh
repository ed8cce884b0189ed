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
template <int QT>
__device__ __forceinline__ void prep_x_smem(const float* __restrict__ x, int M, int K, int kb0, int nbc,
                                            uint8_t* xf, uint32_t lo_plane, uint32_t* side, int npair, int tid,
                                            int nthreads, int mstride = 0) {
    if (mstride < M) mstride = M;
    const int warp = tid >> 5, lane = tid & 31;
    {
        const int npt = 2 * npair - M;  // padding tokens per block: neutral records
        for (int i = tid; i < nbc * npt; i += nthreads) {
            const int b = i / npt, m = M + i % npt;
            uint32_t* r8 = side + (b * npair + (m >> 1)) * 8 + (m & 1);
            r8[0] = r8[2] = r8[4] = r8[6] = 0u;
        }
        const bool x16 = (reinterpret_cast<uintptr_t>(x) & 15) == 0;
        const int ntask = nbc * M;
        const int gl = lane & 7;         // lane in the 8-lane group: elements 4gl..4gl+3
        const bool upper = gl >= 4;      // elements 16..31
        // kPrepUnroll rounds of 32 tasks per pass: their global loads are all
        // in flight together instead of one L2 round trip per round
        constexpr int kPrepUnroll = kResidentPrepUnroll;
        const int kRound = nthreads / 8;
        for (int base = warp * 4; base < ntask; base += kRound * kPrepUnroll) {  // warp-uniform trip count
          float vu[kPrepUnroll][4];
#pragma unroll
          for (int u = 0; u < kPrepUnroll; ++u) {
            const int task = base + u * kRound + (lane >> 3);
            vu[u][0] = vu[u][1] = vu[u][2] = vu[u][3] = 0.0f;
            if (task < ntask) {
                const int b = task / M, m = task % M;
                const float* src = x + (int64_t)m * K + (int64_t)(kb0 + b) * QK + 4 * gl;
                if (x16) {
                    const float4 q = *reinterpret_cast<const float4*>(src);
                    vu[u][0] = q.x;
                    vu[u][1] = q.y;
                    vu[u][2] = q.z;
                    vu[u][3] = q.w;
                } else {
#pragma unroll
                    for (int r = 0; r < 4; ++r) vu[u][r] = src[r];
                }
            }
          }
#pragma unroll
          for (int u = 0; u < kPrepUnroll; ++u) {
            if (base + u * kRound >= ntask) break;  // warp-uniform
            const int task = base + u * kRound + (lane >> 3);
            const bool live = task < ntask;
            const int b = live ? task / M : 0;
            const int m = live ? task % M : 0;
            const float v[4] = {vu[u][0], vu[u][1], vu[u][2], vu[u][3]};
            float am = fmaxf(fmaxf(fabsf(v[0]), fabsf(v[1])), fmaxf(fabsf(v[2]), fabsf(v[3])));
            am = fmaxf(am, __shfl_xor_sync(0xffffffffu, am, 1));
            am = fmaxf(am, __shfl_xor_sync(0xffffffffu, am, 2));
            am = fmaxf(am, __shfl_xor_sync(0xffffffffu, am, 4));
            int e = 0;
            if (am > 0.0f && am <= 3.402823466e38f) e = max(-126, min(127, frexp_exponent(am) - 14));
            // Q4 formats: high-nibble elements meet weights pre-multiplied by 16
            // by the magic trick, so their activations are pre-divided by 16.
            // Multiplying by an exact power of two rounds exactly as ldexpf.
            const float scale = exp2_int(-e) * ((QT != kQ8_0 && upper) ? 0.0625f : 1.0f);
            const float coef = QT == kQ8_0 ? 1152.0f : (QT == kQ4_0 ? (upper ? 1152.0f : 1032.0f) : 1024.0f);
            // record order inside each group of four: Q8_0 (0,1,2,3), Q4 (0,2,1,3)
            constexpr int P1 = QT == kQ8_0 ? 1 : 2, P2 = QT == kQ8_0 ? 2 : 1;
            float vv[4];
            vv[0] = v[0] * scale;
            vv[1] = v[P1] * scale;
            vv[2] = v[P2] * scale;
            vv[3] = v[3] * scale;
            const __half2 h01 = __floats2half2_rn(vv[0], vv[1]), h23 = __floats2half2_rn(vv[2], vv[3]);
            const float2 f01 = __half22float2(h01), f23 = __half22float2(h23);
            const __half2 l01 = __floats2half2_rn(vv[0] - f01.x, vv[1] - f01.y);
            const __half2 l23 = __floats2half2_rn(vv[2] - f23.x, vv[3] - f23.y);
            const float2 g01 = __half22float2(l01), g23 = __half22float2(l23);
            const float rep[4] = {f01.x + g01.x, f01.y + g01.y, f23.x + g23.x, f23.y + g23.y};
            float corr = coef * rep[0] + coef * rep[1] + coef * rep[2] + coef * rep[3];
            float sx = 0.0f;
            if (QT == kQ4_1) sx = (rep[0] + rep[1] + rep[2] + rep[3]) * (upper ? 16.0f : 1.0f);
            corr += __shfl_xor_sync(0xffffffffu, corr, 1);
            corr += __shfl_xor_sync(0xffffffffu, corr, 2);
            corr += __shfl_xor_sync(0xffffffffu, corr, 4);
            if (QT == kQ4_1) {
                sx += __shfl_xor_sync(0xffffffffu, sx, 1);
                sx += __shfl_xor_sync(0xffffffffu, sx, 2);
                sx += __shfl_xor_sync(0xffffffffu, sx, 4);
            }
            if (live) {
                // thread t's 16-byte record holds elements 4t..4t+3 then
                // 16+4t..16+4t+3, in the hi plane and in the lo plane
                uint8_t* rec = xf + ((uint32_t)(b * mstride + m) * 4 + (gl & 3)) * 16 + (upper ? 8 : 0);
                *reinterpret_cast<uint2*>(rec) = make_uint2(h2_bits(h01), h2_bits(h23));
                *reinterpret_cast<uint2*>(rec + lo_plane) = make_uint2(h2_bits(l01), h2_bits(l23));
                if (gl == 0) {
                    uint32_t* r8 = side + (b * npair + (m >> 1)) * 8 + (m & 1);
                    r8[0] = r8[2] = __float_as_uint(-corr);  // the MMA accumulator starts at -corr
                    r8[4] = __float_as_uint(exp2_int(e));
                    r8[6] = __float_as_uint(sx);
                }
            }
          }
        }
    }
}

}  // namespace qmm
