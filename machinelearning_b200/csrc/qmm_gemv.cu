// Decode-time quantised GEMV (M <= 64) for sm_100a.
//
// y[M, N] = x[M, K] . W[N, K]^T with W in raw GGUF block layout (Q4_0, Q4_1 or
// Q8_0 rows of K/32 blocks, exactly as on disk). Replaces the M <= 4 / M > 4
// CPU loops of matmul_f32_q4 / _q4_native / _q8 / _q8_v2 / _q4_1 / _q4_1_native
// (reference llmserve/llmmodel/kernel/main/src/core/quantize.rs:297-1070).
//
// Structure (one CTA per SM, persistent):
//   * warp kW (producer) streams weight tiles -- 16 rows x kc blocks -- from
//     HBM into shared memory with 1-D bulk async copies (TMA), one copy per
//     row (16 lanes issue in parallel), each window widened to 16-byte
//     alignment; completion is counted on an mbarrier in transaction bytes.
//     Every consumer warp owns a ring of kSW stages.
//   * warps 0..kW-1 (consumers) each own 16-row groups. Per 32-element block a
//     warp dequantises its A fragments in registers (f16 magic-number trick for
//     f32 activations, raw/offset int8 for Q8_0 activations) and runs
//     mma.sync against pre-laid-out activation fragments (B), then applies the
//     per-block scales in f32. The tensor pipe does the multiply-adds so the
//     issue slots go to dequantisation.
//   * small N: a row group's K range is split over `ks` warps; the last warp
//     to finish (atomic ticket) sums the partials in a fixed order, so results
//     are deterministic.
//
// Numerics:
//   * f32-activation mode: activations enter the f16 MMA as hi+lo halves of a
//     block-scaled copy (~22 significant bits); weights enter as exact biased
//     integers; products are exact and accumulate in f32. Relative error vs the
//     reference's f32 path is ~1e-5 (bound checked in tests: 1e-3).
//   * Q8_0-activation mode (the reference's *_native / _v2 functions): integer
//     block dots are exact; with ks == 1 (always, for this mode) each output
//     sums the per-block terms in block order with the reference's operation
//     order, so results are bit-identical to the reference.
#include <map>
#include <mutex>
#include <utility>

#include "qmm_common.cuh"
#include "qmm_kernels.cuh"

namespace qmm {

namespace {

constexpr int kW = 4;                 // consumer warps per CTA
constexpr int kSW = 3;                // pipeline stages per consumer warp
constexpr int kThreads = 32 * (kW + 1);
constexpr int kStageTarget = 8192;    // bytes of weights per stage (16 rows)
constexpr uint32_t kMaxIdle = 1u << 24;  // producer polls without progress before giving up

struct Args {
    const uint8_t* w;
    uint64_t w_bytes;
    float* y;
    const void* xa;
    const void* xs;
    const float* xsum;
    float* partial;
    unsigned* counters;
    int M, N, nb, row_bytes, ks, nbu, kc, pitch, units;
    int* err;
};

__device__ __forceinline__ uint4 ldg_nc_u4(const void* p) {
    uint4 r;
    asm volatile("ld.global.nc.v4.u32 {%0,%1,%2,%3}, [%4];"
                 : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w)
                 : "l"(p));
    return r;
}
__device__ __forceinline__ uint2 ldg_nc_u2(const void* p) {
    uint2 r;
    asm volatile("ld.global.nc.v2.u32 {%0,%1}, [%2];" : "=r"(r.x), "=r"(r.y) : "l"(p));
    return r;
}

template <int QT, int NT, bool NATIVE>
__device__ __forceinline__ void consume_block(uint32_t blk0, uint32_t blk1, int b, const Args& a, int g, int t,
                                              float (&acc)[NT][4]) {
    const int Mpad = token_pad(a.M);
    const float d0 = f16_bits_to_f32((uint16_t)lds_u16(blk0));
    const float d1 = f16_bits_to_f32((uint16_t)lds_u16(blk1));
    if constexpr (!NATIVE) {
        uint32_t A0[4], A1[4];  // fragments of the two k16 MMAs of this block
        if constexpr (QT == kQ8_0) {
            const uint32_t u00 = lds_u32_a2(blk0 + 2 + 8 * t) ^ 0x80808080u;
            const uint32_t u01 = lds_u32_a2(blk0 + 6 + 8 * t) ^ 0x80808080u;
            const uint32_t u10 = lds_u32_a2(blk1 + 2 + 8 * t) ^ 0x80808080u;
            const uint32_t u11 = lds_u32_a2(blk1 + 6 + 8 * t) ^ 0x80808080u;
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
            constexpr int NOFF = (QT == kQ4_0) ? 2 : 4;
            const uint32_t w0 = lds_u32_a2(blk0 + NOFF + 4 * t);
            const uint32_t w1 = lds_u32_a2(blk1 + NOFF + 4 * t);
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
        float m0 = 0.0f, m1 = 0.0f;
        if constexpr (QT == kQ4_1) {
            m0 = f16_bits_to_f32((uint16_t)lds_u16(blk0 + 2));
            m1 = f16_bits_to_f32((uint16_t)lds_u16(blk1 + 2));
        }
        const __half* xf = static_cast<const __half*>(a.xa);
        const float2* xcs = static_cast<const float2*>(a.xs);
#pragma unroll
        for (int nt = 0; nt < NT; ++nt) {
            const int m = nt * 8 + g;
            uint4 xh = make_uint4(0, 0, 0, 0), xl = make_uint4(0, 0, 0, 0);
            if (m < a.M) {
                const __half* rec = xf + (((int64_t)b * a.M + m) * 4 + t) * 16;
                xh = ldg_nc_u4(rec);
                xl = ldg_nc_u4(rec + 8);
            }
            const uint4 csr = ldg_nc_u4(xcs + ((int64_t)b * Mpad + nt * 8 + 2 * t));
            const float nc0 = __uint_as_float(csr.x), s0 = __uint_as_float(csr.y);
            const float nc1 = __uint_as_float(csr.z), s1 = __uint_as_float(csr.w);
            float c[4] = {nc0, nc1, nc0, nc1};
            mma_f16_16816(c, A0[0], A0[1], A0[2], A0[3], xh.x, xh.y);
            mma_f16_16816(c, A1[0], A1[1], A1[2], A1[3], xh.z, xh.w);
            mma_f16_16816(c, A0[0], A0[1], A0[2], A0[3], xl.x, xl.y);
            mma_f16_16816(c, A1[0], A1[1], A1[2], A1[3], xl.z, xl.w);
            if constexpr (QT == kQ4_1) {
                const float2 sx = *reinterpret_cast<const float2*>(a.xsum + ((int64_t)b * Mpad + nt * 8 + 2 * t));
                acc[nt][0] = fmaf(s0, fmaf(d0, c[0], m0 * sx.x), acc[nt][0]);
                acc[nt][1] = fmaf(s1, fmaf(d0, c[1], m0 * sx.y), acc[nt][1]);
                acc[nt][2] = fmaf(s0, fmaf(d1, c[2], m1 * sx.x), acc[nt][2]);
                acc[nt][3] = fmaf(s1, fmaf(d1, c[3], m1 * sx.y), acc[nt][3]);
            } else {
                acc[nt][0] = fmaf(d0 * s0, c[0], acc[nt][0]);
                acc[nt][1] = fmaf(d0 * s1, c[1], acc[nt][1]);
                acc[nt][2] = fmaf(d1 * s0, c[2], acc[nt][2]);
                acc[nt][3] = fmaf(d1 * s1, c[3], acc[nt][3]);
            }
        }
    } else {
        uint32_t a0, a1, a2, a3;
        if constexpr (QT == kQ8_0) {
            a0 = lds_u32_a2(blk0 + 2 + 8 * t);
            a2 = lds_u32_a2(blk0 + 6 + 8 * t);
            a1 = lds_u32_a2(blk1 + 2 + 8 * t);
            a3 = lds_u32_a2(blk1 + 6 + 8 * t);
        } else {
            constexpr int NOFF = (QT == kQ4_0) ? 2 : 4;
            const uint32_t w0 = lds_u32_a2(blk0 + NOFF + 4 * t);
            const uint32_t w1 = lds_u32_a2(blk1 + NOFF + 4 * t);
            a0 = w0 & 0x0F0F0F0Fu;
            a1 = w1 & 0x0F0F0F0Fu;
            a2 = (w0 >> 4) & 0x0F0F0F0Fu;
            a3 = (w1 >> 4) & 0x0F0F0F0Fu;
        }
        float m0 = 0.0f, m1 = 0.0f;
        if constexpr (QT == kQ4_1) {
            m0 = f16_bits_to_f32((uint16_t)lds_u16(blk0 + 2));
            m1 = f16_bits_to_f32((uint16_t)lds_u16(blk1 + 2));
        }
        const uint8_t* xq = static_cast<const uint8_t*>(a.xa);
        const int2* xsc = static_cast<const int2*>(a.xs);
#pragma unroll
        for (int nt = 0; nt < NT; ++nt) {
            const int m = nt * 8 + g;
            uint2 bq = make_uint2(0, 0);
            if (m < a.M) bq = ldg_nc_u2(xq + (((int64_t)b * a.M + m) * 4 + t) * 8);
            const uint4 sc = ldg_nc_u4(xsc + ((int64_t)b * Mpad + nt * 8 + 2 * t));
            const float xs0 = __uint_as_float(sc.x), xs1 = __uint_as_float(sc.z);
            const int qs0 = (int)sc.y, qs1 = (int)sc.w;
            int c[4];
            if constexpr (QT == kQ4_0) {  // sum (n - 8) q = sum n q - 8 sum q
                c[0] = -8 * qs0;
                c[1] = -8 * qs1;
                c[2] = -8 * qs0;
                c[3] = -8 * qs1;
            } else {
                c[0] = c[1] = c[2] = c[3] = 0;
            }
            mma_s8_16832(c, a0, a1, a2, a3, bq.x, bq.y);
            if constexpr (QT == kQ4_1) {
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

template <int QT, int NT, bool NATIVE>
__global__ void __launch_bounds__(kThreads, 1) gemv_kernel(const Args a) {
    extern __shared__ __align__(128) uint8_t smem[];
    constexpr int BB = block_bytes(QT);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int stage_bytes = 16 * a.pitch;
    uint64_t* full = reinterpret_cast<uint64_t*>(smem + kW * kSW * stage_bytes);
    uint64_t* empty = full + kW * kSW;
    if (threadIdx.x == 0) {
        for (int i = 0; i < kW * kSW; ++i) {
            mbar_init(&full[i], 1);
            mbar_init(&empty[i], 1);
        }
        fence_mbar_init();
    }
    __syncthreads();
    pdl_launch_dependents();
    pdl_wait();  // activations (and possibly the weights) come from earlier work in the stream
    const int G = gridDim.x * kW;

    if (warp == kW) {
        // ------------------------------- producer ---------------------------------
        int u[kW], c[kW], lt[kW];
#pragma unroll
        for (int w = 0; w < kW; ++w) {
            u[w] = blockIdx.x * kW + w;
            c[w] = 0;
            lt[w] = 0;
        }
        const uint64_t wfl = a.w_bytes & ~uint64_t(15);
        uint32_t idle = 0;
        while (true) {
            bool any = false, issued = false;
#pragma unroll
            for (int w = 0; w < kW; ++w) {
                if (u[w] >= a.units) continue;
                any = true;
                const int slot = lt[w] % kSW;
                if (lt[w] >= kSW && !mbar_test_wait(&empty[w * kSW + slot], ((lt[w] / kSW) - 1) & 1)) continue;
                const int rg = u[w] / a.ks, ksi = u[w] % a.ks;
                const int kb_end = min(a.nb, (ksi + 1) * a.nbu);
                const int kb0 = ksi * a.nbu + c[w] * a.kc;
                const int kb1 = min(kb_end, kb0 + a.kc);
                const int rows = min(16, a.N - rg * 16);
                uint8_t* stage = smem + (w * kSW + slot) * stage_bytes;
                uint64_t* fb = &full[w * kSW + slot];
                uint32_t bytes = 0;
                uint64_t a16 = 0;
                if (lane < rows) {
                    const uint64_t beg = (uint64_t)(rg * 16 + lane) * (uint64_t)a.row_bytes + (uint64_t)kb0 * BB;
                    const uint64_t end = beg + (uint64_t)(kb1 - kb0) * BB;
                    a16 = beg & ~uint64_t(15);
                    uint64_t e16 = (end + 15) & ~uint64_t(15);
                    if (e16 > wfl) {
                        // the last row's window would pass the end of the buffer:
                        // copy the aligned part in bulk and the ragged tail by hand
                        e16 = wfl > a16 ? wfl : a16;
                        uint8_t* dst = stage + lane * a.pitch;
                        for (uint64_t gaddr = e16 > beg ? e16 : beg; gaddr < end; ++gaddr) dst[gaddr - a16] = a.w[gaddr];
                    }
                    bytes = (uint32_t)(e16 - a16);
                }
                uint32_t total = bytes;
#pragma unroll
                for (int o = 16; o > 0; o >>= 1) total += __shfl_xor_sync(0xffffffffu, total, o);
                __syncwarp();
                if (lane == 0) mbar_arrive_expect_tx(fb, total);
                __syncwarp();
                if (bytes) bulk_g2s(stage + lane * a.pitch, a.w + a16, bytes, fb);
                ++lt[w];
                if (kb1 >= kb_end) {
                    c[w] = 0;
                    u[w] += G;
                } else {
                    ++c[w];
                }
                issued = true;
            }
            if (!any) break;
            if (issued) {
                idle = 0;
            } else {
                if (++idle > kMaxIdle) {
                    if (lane == 0 && a.err) atomicExch(a.err, kErrWaitTimeout);
                    break;
                }
                __nanosleep(32);
            }
        }
        // drain: never leave the CTA with copies in flight
#pragma unroll
        for (int w = 0; w < kW; ++w) {
            for (int s = 0; s < kSW; ++s) {
                if (lt[w] > s) {
                    const int i = s + kSW * ((lt[w] - 1 - s) / kSW);
                    mbar_wait_bounded(&full[w * kSW + s], (i / kSW) & 1, a.err);
                }
            }
        }
        return;
    }

    // --------------------------------- consumers ------------------------------------
    const int g = lane >> 2, t = lane & 3;
    int lt = 0;
    bool ok = true;
    for (int u = blockIdx.x * kW + warp; u < a.units && ok; u += G) {
        const int rg = u / a.ks, ksi = u % a.ks;
        const int kb_begin = ksi * a.nbu;
        const int kb_end = min(a.nb, kb_begin + a.nbu);
        float acc[NT][4];
#pragma unroll
        for (int nt = 0; nt < NT; ++nt) acc[nt][0] = acc[nt][1] = acc[nt][2] = acc[nt][3] = 0.0f;
        const int r0 = rg * 16 + g, r1 = r0 + 8;
        for (int kb0 = kb_begin; kb0 < kb_end; kb0 += a.kc) {
            const int kb1 = min(kb_end, kb0 + a.kc);
            const int slot = lt % kSW;
            if (!mbar_wait_bounded(&full[warp * kSW + slot], (lt / kSW) & 1, a.err)) {
                ok = false;
                break;
            }
            const uint32_t sbase = smem_u32(smem + (warp * kSW + slot) * stage_bytes);
            const uint32_t off0 = (uint32_t)(((uint64_t)r0 * a.row_bytes + (uint64_t)kb0 * BB) & 15);
            const uint32_t off1 = (uint32_t)(((uint64_t)r1 * a.row_bytes + (uint64_t)kb0 * BB) & 15);
            const uint32_t base0 = sbase + g * a.pitch + off0;
            const uint32_t base1 = sbase + (g + 8) * a.pitch + off1;
#pragma unroll 2
            for (int b = kb0; b < kb1; ++b) {
                const uint32_t o = (uint32_t)(b - kb0) * BB;
                consume_block<QT, NT, NATIVE>(base0 + o, base1 + o, b, a, g, t, acc);
            }
            __syncwarp();
            if (lane == 0) mbar_arrive(&empty[warp * kSW + slot]);
            ++lt;
        }
        if (!ok) break;
        // ------------------------------- epilogue -------------------------------------
        if (a.ks == 1) {
#pragma unroll
            for (int nt = 0; nt < NT; ++nt) {
                const int m0 = nt * 8 + 2 * t, m1 = m0 + 1;
                if (r0 < a.N) {
                    if (m0 < a.M) a.y[(int64_t)m0 * a.N + r0] = acc[nt][0];
                    if (m1 < a.M) a.y[(int64_t)m1 * a.N + r0] = acc[nt][1];
                }
                if (r1 < a.N) {
                    if (m0 < a.M) a.y[(int64_t)m0 * a.N + r1] = acc[nt][2];
                    if (m1 < a.M) a.y[(int64_t)m1 * a.N + r1] = acc[nt][3];
                }
            }
        } else {
            float* part = a.partial + (int64_t)ksi * a.M * a.N;
#pragma unroll
            for (int nt = 0; nt < NT; ++nt) {
                const int m0 = nt * 8 + 2 * t, m1 = m0 + 1;
                if (r0 < a.N) {
                    if (m0 < a.M) part[(int64_t)m0 * a.N + r0] = acc[nt][0];
                    if (m1 < a.M) part[(int64_t)m1 * a.N + r0] = acc[nt][1];
                }
                if (r1 < a.N) {
                    if (m0 < a.M) part[(int64_t)m0 * a.N + r1] = acc[nt][2];
                    if (m1 < a.M) part[(int64_t)m1 * a.N + r1] = acc[nt][3];
                }
            }
            __threadfence();
            __syncwarp();
            unsigned ticket = 0;
            if (lane == 0) ticket = atomicAdd(&a.counters[rg], 1u);
            ticket = __shfl_sync(0xffffffffu, ticket, 0);
            if (ticket == (unsigned)(a.ks - 1)) {
                __threadfence();
#pragma unroll
                for (int nt = 0; nt < NT; ++nt) {
#pragma unroll
                    for (int e = 0; e < 4; ++e) {
                        const int m = nt * 8 + 2 * t + (e & 1);
                        const int r = (e < 2) ? r0 : r1;
                        if (m < a.M && r < a.N) {
                            float s = 0.0f;
                            for (int k = 0; k < a.ks; ++k) s += __ldcg(a.partial + ((int64_t)k * a.M + m) * a.N + r);
                            a.y[(int64_t)m * a.N + r] = s;
                        }
                    }
                }
                if (lane == 0) a.counters[rg] = 0u;
            }
        }
    }
}

template <int QT, bool NATIVE>
const void* pick_kernel(int nt) {
    switch (nt) {
        case 1: return (const void*)gemv_kernel<QT, 1, NATIVE>;
        case 2: return (const void*)gemv_kernel<QT, 2, NATIVE>;
        case 4: return (const void*)gemv_kernel<QT, 4, NATIVE>;
        default: return (const void*)gemv_kernel<QT, 8, NATIVE>;
    }
}

const void* kernel_for(const GemvPlan& p) {
    if (p.native) {
        if (p.qt == kQ8_0) return pick_kernel<kQ8_0, true>(p.nt);
        if (p.qt == kQ4_0) return pick_kernel<kQ4_0, true>(p.nt);
        return pick_kernel<kQ4_1, true>(p.nt);
    }
    if (p.qt == kQ8_0) return pick_kernel<kQ8_0, false>(p.nt);
    if (p.qt == kQ4_0) return pick_kernel<kQ4_0, false>(p.nt);
    return pick_kernel<kQ4_1, false>(p.nt);
}

size_t align256(size_t v) { return (v + 255) & ~size_t(255); }

// Opt a kernel in to its dynamic shared memory size on the current device,
// once per (device, kernel).
cudaError_t ensure_dynamic_smem(const void* fn, size_t bytes) {
    static std::mutex mu;
    static std::map<std::pair<int, const void*>, size_t> done;
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return e;
    std::lock_guard<std::mutex> lock(mu);
    size_t& have = done[{dev, fn}];
    if (have >= bytes) return cudaSuccess;
    e = cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)bytes);
    if (e == cudaSuccess) have = bytes;
    return e;
}

}  // namespace

bool gemv_plan(int qt, bool native, int M, int N, int K, int num_sms, GemvPlan* p) {
    if (M < 1 || M > 64 || N < 1 || K < QK || K % QK) return false;
    const int bb = block_bytes(qt);
    if (!bb) return false;
    GemvPlan q = {};
    q.qt = qt;
    q.native = native;
    q.M = M;
    q.N = N;
    q.K = K;
    q.nb = K / QK;
    q.row_bytes = q.nb * bb;
    q.nt = token_tiles(M);
    const int groups = (N + 15) / 16;
    const int slots = num_sms * kW;
    int ks = 1;
    if (!native && groups < slots) {
        ks = slots / groups;
        const int max_ks = q.nb / 8 > 1 ? q.nb / 8 : 1;  // keep >= 8 blocks per split
        if (ks > max_ks) ks = max_ks;
        if (ks < 1) ks = 1;
    }
    q.nbu = (q.nb + ks - 1) / ks;
    q.ks = (q.nb + q.nbu - 1) / q.nbu;
    const int kc_max = (kStageTarget / 16 - 32) / bb;
    q.kc = q.nbu < kc_max ? q.nbu : kc_max;
    q.pitch = (int)(((size_t)q.kc * bb + 30 + 15) / 16 * 16);
    q.units = groups * q.ks;
    const int ctas = (q.units + kW - 1) / kW;
    q.grid = ctas < num_sms ? ctas : num_sms;
    q.smem = (size_t)kW * kSW * 16 * q.pitch + 2 * kW * kSW * sizeof(uint64_t);
    *p = q;
    return true;
}

size_t gemv_counters_bytes(const GemvPlan& p) {
    return p.ks > 1 ? align256((size_t)((p.N + 15) / 16) * sizeof(unsigned)) : 0;
}

size_t gemv_workspace_bytes(const GemvPlan& p) {
    const size_t Mpad = (size_t)token_pad(p.M);
    size_t s = 0;
    if (p.native) {
        s += align256((size_t)p.nb * p.M * 32);
        s += align256((size_t)p.nb * Mpad * sizeof(int2));
    } else {
        s += align256((size_t)p.nb * p.M * 128);
        s += align256((size_t)p.nb * Mpad * sizeof(float2));
        if (p.qt == kQ4_1) s += align256((size_t)p.nb * Mpad * sizeof(float));
    }
    if (p.ks > 1) s += align256((size_t)p.ks * p.M * p.N * sizeof(float));
    s += gemv_counters_bytes(p);
    return s;
}

size_t gemv_counters_offset(const GemvPlan& p) { return gemv_workspace_bytes(p) - gemv_counters_bytes(p); }

void gemv_workspace_carve(const GemvPlan& p, void* base, GemvWorkspace* ws) {
    const size_t Mpad = (size_t)token_pad(p.M);
    uint8_t* c = static_cast<uint8_t*>(base);
    *ws = GemvWorkspace{};
    if (p.native) {
        ws->xa = c;
        c += align256((size_t)p.nb * p.M * 32);
        ws->xs = c;
        c += align256((size_t)p.nb * Mpad * sizeof(int2));
    } else {
        ws->xa = c;
        c += align256((size_t)p.nb * p.M * 128);
        ws->xs = c;
        c += align256((size_t)p.nb * Mpad * sizeof(float2));
        if (p.qt == kQ4_1) {
            ws->xsum = reinterpret_cast<float*>(c);
            c += align256((size_t)p.nb * Mpad * sizeof(float));
        }
    }
    if (p.ks > 1) {
        ws->partial = reinterpret_cast<float*>(c);
        c += align256((size_t)p.ks * p.M * p.N * sizeof(float));
        ws->counters = reinterpret_cast<unsigned*>(c);
    }
}

cudaError_t launch_gemv(const GemvPlan& p, const uint8_t* w, const float* x, float* y, const GemvWorkspace& ws,
                        int* err, cudaStream_t st) {
    cudaError_t e;
    const int nzero = ws.counters ? (p.N + 15) / 16 : 0;
    if (p.native) {
        e = launch_xprep_q8(p.qt, x, p.M, p.K, static_cast<uint8_t*>(ws.xa), static_cast<int2*>(ws.xs), ws.counters,
                            nzero, st);
    } else {
        e = launch_xprep_f32(p.qt, x, p.M, p.K, static_cast<__half*>(ws.xa), static_cast<float2*>(ws.xs), ws.xsum,
                             ws.counters, nzero, st);
    }
    if (e != cudaSuccess) return e;
    const void* fn = kernel_for(p);
    e = ensure_dynamic_smem(fn, p.smem);
    if (e != cudaSuccess) return e;
    Args a;
    a.w = w;
    a.w_bytes = (uint64_t)p.N * (uint64_t)p.row_bytes;
    a.y = y;
    a.xa = ws.xa;
    a.xs = ws.xs;
    a.xsum = ws.xsum;
    a.partial = ws.partial;
    a.counters = ws.counters;
    a.M = p.M;
    a.N = p.N;
    a.nb = p.nb;
    a.row_bytes = p.row_bytes;
    a.ks = p.ks;
    a.nbu = p.nbu;
    a.kc = p.kc;
    a.pitch = p.pitch;
    a.units = p.units;
    a.err = err;
    void* args[] = {(void*)&a};
    return launch_pdl_kernel(fn, dim3(p.grid), dim3(kThreads), p.smem, st, args);
}

}  // namespace qmm
