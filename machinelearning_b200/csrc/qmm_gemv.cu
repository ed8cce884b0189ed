// Decode-time quantised GEMV (M <= 64) for sm_100a.
//
// y[M, N] = x[M, K] . W[N, K]^T with W in raw GGUF block layout (Q4_0, Q4_1 or
// Q8_0 rows of K/32 blocks, exactly as on disk). Replaces the M <= 4 / M > 4
// CPU loops of matmul_f32_q4 / _q4_native / _q8 / _q8_v2 / _q4_1 / _q4_1_native
// (reference llmserve/llmmodel/kernel/main/src/core/quantize.rs:297-1070).
//
// Structure (one CTA per SM, persistent):
//   * warp kW (producer) streams weight tiles -- 32 rows x kc blocks -- from
//     HBM into shared memory with 1-D bulk async copies (TMA), one copy per
//     row (the 32 lanes issue in parallel), each window widened to 16-byte
//     alignment; completion is counted on an mbarrier in transaction bytes.
//     Every consumer warp owns a ring of kSW stages.
//   * warps 0..kW-1 (consumers) each own 32-row tiles (two 16-row MMA groups
//     sharing one set of activation fragments). Per 32-element block a warp
//     dequantises its A fragments in registers (f16 magic-number trick for
//     f32 activations, raw/offset int8 for Q8_0 activations), runs mma.sync
//     against the pre-laid-out activation fragments (B, prefetched one block
//     ahead), then applies the per-block scales in f32. The tensor pipe does
//     the multiply-adds so issue slots go to dequantisation.
//   * small N: a tile's K range is split over `ks` warps; the last warp to
//     finish (atomic ticket) sums the partials in a fixed order, so results
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
#include <cuda.h>

#include <map>
#include <mutex>
#include <tuple>
#include <utility>

#include "qmm_common.cuh"
#include "qmm_kernels.cuh"

namespace qmm {

namespace {

constexpr int kW = 8;                    // consumer warps per CTA
constexpr int kSW = 2;                   // pipeline stages per consumer warp
constexpr int kRows = 32;                // weight rows per warp tile (two MMA row groups)
constexpr int kThreads = 32 * (kW + 1);
constexpr int kStageTarget = 10240;      // weight bytes per stage
constexpr uint32_t kMaxIdle = 1u << 24;  // producer polls without progress before giving up

// kLoaderTma2d:    row pitch % 16 == 0: one [32 rows x kc blocks] TMA tile per stage.
// kLoaderTmaPairs: row pitch % 16 == 8 (e.g. K = 1152), N even: the matrix is
//                  viewed as [N/2][2 * row_bytes] (16-byte pitched); even rows
//                  and odd rows come as two [16 x (kc blocks + 16 B)] tiles,
//                  the odd ones starting 8 bytes early (skew 8 in shared memory).
// kLoaderCpAsync:  anything else: 16-byte cp.async pieces of each row window.
enum Loader : int { kLoaderTma2d = 0, kLoaderCpAsync = 1, kLoaderTmaPairs = 2 };

struct Args {
    CUtensorMap tmap;  // weights as a [N rows][row_bytes/4] uint32 tensor (TMA loader only)
    const uint8_t* w;
    uint64_t w_bytes;
    float* y;
    const void* xa;
    const void* xs;
    const float* xsum;
    float* partial;
    unsigned* counters;
    int M, N, nb, row_bytes, ks, nbu, kc, pitch, units, loader;
    int* err;
};

// Activation fragments of one block for one 8-token tile.
struct XFrag {
    uint4 hi, lo;   // f32 mode: B fragments (hi and lo halves); native: hi.x/.y = s8 B fragment
    uint4 cs;       // f32 mode: {-corr0, s0, -corr1, s1}; native: {xs0, qsum0, xs1, qsum1}
    float2 sx;      // Q4_1 f32 mode: per-token block sums
};

// Per-unit activation cursors: record pointers advance by one block per step.
struct XCursor {
    const uint8_t* rec;  // this lane's record of token tile 0 (f32: 32 B, native: 8 B per record)
    const uint4* side;   // cs of token tile 0 (tokens 2t, 2t+1)
    const float2* sx;    // Q4_1 sums
    int64_t rec_step;    // bytes per block
    int side_step;       // uint4 per block
    bool valid[8];       // token nt*8+g < M
};

template <int QT, int NT, bool NATIVE>
__device__ __forceinline__ void load_x(const XCursor& c, int j, XFrag (&x)[NT]) {
    constexpr int kRec = NATIVE ? 8 : 32;
#pragma unroll
    for (int nt = 0; nt < NT; ++nt) {
        const uint8_t* r = c.rec + (int64_t)j * c.rec_step + (int64_t)nt * 8 * 4 * kRec;
        x[nt].hi = make_uint4(0, 0, 0, 0);
        x[nt].lo = make_uint4(0, 0, 0, 0);
        if (c.valid[nt]) {
            if constexpr (NATIVE) {
                const uint2 q = __ldg(reinterpret_cast<const uint2*>(r));
                x[nt].hi.x = q.x;
                x[nt].hi.y = q.y;
            } else {
                x[nt].hi = __ldg(reinterpret_cast<const uint4*>(r));
                x[nt].lo = __ldg(reinterpret_cast<const uint4*>(r) + 1);
            }
        }
        // side arrays are padded to the token tiles, always readable
        x[nt].cs = __ldg(c.side + (int64_t)j * c.side_step + nt * 4);
        if constexpr (QT == kQ4_1 && !NATIVE) x[nt].sx = __ldg(c.sx + (int64_t)j * c.side_step + nt * 4);
    }
}

// One block of one 16-row group (rows g and g+8 at shared pointers r0/r1).
template <int QT, int NT, bool NATIVE>
__device__ __forceinline__ void consume_group(const uint8_t* r0, const uint8_t* r1, int t, const XFrag (&x)[NT],
                                              float (&acc)[NT][4]) {
    const float d0 = f16_bits_to_f32((uint16_t)lds_u16(r0));
    const float d1 = f16_bits_to_f32((uint16_t)lds_u16(r1));
    float m0 = 0.0f, m1 = 0.0f;
    if constexpr (QT == kQ4_1) {
        m0 = f16_bits_to_f32((uint16_t)lds_u16(r0 + 2));
        m1 = f16_bits_to_f32((uint16_t)lds_u16(r1 + 2));
    }
    if constexpr (!NATIVE) {
        uint32_t A0[4], A1[4];  // fragments of the two k16 MMAs of this block
        if constexpr (QT == kQ8_0) {
            const uint32_t u00 = lds_u32_a2(r0 + 2 + 8 * t) ^ 0x80808080u;
            const uint32_t u01 = lds_u32_a2(r0 + 6 + 8 * t) ^ 0x80808080u;
            const uint32_t u10 = lds_u32_a2(r1 + 2 + 8 * t) ^ 0x80808080u;
            const uint32_t u11 = lds_u32_a2(r1 + 6 + 8 * t) ^ 0x80808080u;
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
            const uint32_t w0 = lds_u32_a2(r0 + NOFF + 4 * t);
            const uint32_t w1 = lds_u32_a2(r1 + NOFF + 4 * t);
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
            const float nc0 = __uint_as_float(x[nt].cs.x), s0 = __uint_as_float(x[nt].cs.y);
            const float nc1 = __uint_as_float(x[nt].cs.z), s1 = __uint_as_float(x[nt].cs.w);
            float c[4] = {nc0, nc1, nc0, nc1};
            float e[4] = {0.0f, 0.0f, 0.0f, 0.0f};  // second chain: the lo halves
            mma_f16_16816(c, A0[0], A0[1], A0[2], A0[3], x[nt].hi.x, x[nt].hi.y);
            mma_f16_16816(e, A0[0], A0[1], A0[2], A0[3], x[nt].lo.x, x[nt].lo.y);
            mma_f16_16816(c, A1[0], A1[1], A1[2], A1[3], x[nt].hi.z, x[nt].hi.w);
            mma_f16_16816(e, A1[0], A1[1], A1[2], A1[3], x[nt].lo.z, x[nt].lo.w);
#pragma unroll
            for (int i = 0; i < 4; ++i) c[i] += e[i];
            if constexpr (QT == kQ4_1) {
                acc[nt][0] = fmaf(s0, fmaf(d0, c[0], m0 * x[nt].sx.x), acc[nt][0]);
                acc[nt][1] = fmaf(s1, fmaf(d0, c[1], m0 * x[nt].sx.y), acc[nt][1]);
                acc[nt][2] = fmaf(s0, fmaf(d1, c[2], m1 * x[nt].sx.x), acc[nt][2]);
                acc[nt][3] = fmaf(s1, fmaf(d1, c[3], m1 * x[nt].sx.y), acc[nt][3]);
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
            a0 = lds_u32_a2(r0 + 2 + 8 * t);
            a2 = lds_u32_a2(r0 + 6 + 8 * t);
            a1 = lds_u32_a2(r1 + 2 + 8 * t);
            a3 = lds_u32_a2(r1 + 6 + 8 * t);
        } else {
            constexpr int NOFF = (QT == kQ4_0) ? 2 : 4;
            const uint32_t w0 = lds_u32_a2(r0 + NOFF + 4 * t);
            const uint32_t w1 = lds_u32_a2(r1 + NOFF + 4 * t);
            a0 = w0 & 0x0F0F0F0Fu;
            a1 = w1 & 0x0F0F0F0Fu;
            a2 = (w0 >> 4) & 0x0F0F0F0Fu;
            a3 = (w1 >> 4) & 0x0F0F0F0Fu;
        }
#pragma unroll
        for (int nt = 0; nt < NT; ++nt) {
            const float xs0 = __uint_as_float(x[nt].cs.x), xs1 = __uint_as_float(x[nt].cs.z);
            const int qs0 = (int)x[nt].cs.y, qs1 = (int)x[nt].cs.w;
            int c[4];
            if constexpr (QT == kQ4_0) {  // sum (n - 8) q = sum n q - 8 sum q
                c[0] = -8 * qs0;
                c[1] = -8 * qs1;
                c[2] = -8 * qs0;
                c[3] = -8 * qs1;
            } else {
                c[0] = c[1] = c[2] = c[3] = 0;
            }
            mma_s8_16832(c, a0, a1, a2, a3, x[nt].hi.x, x[nt].hi.y);
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
__global__ void __launch_bounds__(kThreads, 1) gemv_kernel(const __grid_constant__ Args a) {
    extern __shared__ __align__(128) uint8_t smem[];
    constexpr int BB = block_bytes(QT);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int stage_bytes = kRows * a.pitch;
    uint64_t* full = reinterpret_cast<uint64_t*>(smem + kW * kSW * stage_bytes);
    uint64_t* empty = full + kW * kSW;
    if (threadIdx.x == 0) {
        // TMA tiles complete with one arrival + transaction bytes; the cp.async
        // loader arrives once per producer lane plus once for plain tail stores
        const uint32_t full_count = a.loader == kLoaderCpAsync ? 33u : 1u;
        for (int i = 0; i < kW * kSW; ++i) {
            mbar_init(&full[i], full_count);
            mbar_init(&empty[i], 1);
        }
        fence_mbar_init();
    }
    if (a.loader != kLoaderCpAsync && warp == kW && lane == 0) prefetch_tmap(&a.tmap);
    __syncthreads();
    pdl_launch_dependents();
    pdl_wait();  // activations (and possibly the weights) come from earlier work in the stream
    const int G = gridDim.x * kW;

    if (warp == kW) {
        // ------------------------------- producer ---------------------------------
        int u[kW], c[kW], lt[kW];
#pragma unroll
        for (int w = 0; w < kW; ++w) {
            u[w] = w * gridDim.x + blockIdx.x;  // same dealing as the consumers
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
                const int tile = u[w] / a.ks, ksi = u[w] % a.ks;
                const int kb_end = min(a.nb, (ksi + 1) * a.nbu);
                const int kb0 = ksi * a.nbu + c[w] * a.kc;
                const int kb1 = min(kb_end, kb0 + a.kc);
                const int rows = min(kRows, a.N - tile * kRows);
                uint8_t* stage = smem + (w * kSW + slot) * stage_bytes;
                uint64_t* fb = &full[w * kSW + slot];
                if (a.loader == kLoaderTma2d) {
                    // one 2-D tile: 32 rows x kc blocks (rows past N and columns past
                    // the row end are zero-filled by the copy engine)
                    if (lane == 0) {
                        mbar_arrive_expect_tx(fb, (uint32_t)(kRows * a.pitch));
                        tma_load_2d(stage, &a.tmap, kb0 * BB / 4, tile * kRows, fb);
                    }
                } else if (a.loader == kLoaderTmaPairs) {
                    if (lane == 0) {
                        mbar_arrive_expect_tx(fb, (uint32_t)(kRows * a.pitch));
                        tma_load_2d(stage, &a.tmap, kb0 * BB / 4, tile * (kRows / 2), fb);
                        tma_load_2d(stage + (kRows / 2) * a.pitch, &a.tmap, (a.row_bytes + kb0 * BB - 8) / 4,
                                    tile * (kRows / 2), fb);
                    }
                } else {
                    // rows are not 16-byte pitched: the warp copies each row's
                    // window, widened to 16-byte alignment, in 16-byte pieces
                    for (int r = 0; r < rows; ++r) {
                        const uint64_t beg = (uint64_t)(tile * kRows + r) * (uint64_t)a.row_bytes + (uint64_t)kb0 * BB;
                        const uint64_t end = beg + (uint64_t)(kb1 - kb0) * BB;
                        const uint64_t a16 = beg & ~uint64_t(15);
                        uint64_t e16 = (end + 15) & ~uint64_t(15);
                        uint8_t* dst = stage + r * a.pitch;
                        if (e16 > wfl) {
                            // the last row's window would pass the end of the buffer:
                            // the ragged tail is copied with plain loads
                            e16 = wfl > a16 ? wfl : a16;
                            for (uint64_t gaddr = (e16 > beg ? e16 : beg) + lane; gaddr < end; gaddr += 32)
                                dst[gaddr - a16] = a.w[gaddr];
                        }
                        for (uint64_t off = 16u * lane; a16 + off < e16; off += 512) cp_async_16(dst + off, a.w + a16 + off);
                    }
                    cp_async_arrive_noinc(fb);  // 32 arrivals once each lane's copies land
                    __syncwarp();
                    if (lane == 0) mbar_arrive(fb);  // 33rd: orders the plain tail stores
                }
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
    const int Mpad = token_pad(a.M);
    int lt = 0;
    // units are dealt round-robin over CTAs first, so every SM gets work
    for (int u = warp * gridDim.x + blockIdx.x; u < a.units; u += G) {
        const int tile = u / a.ks, ksi = u % a.ks;
        const int kb_begin = ksi * a.nbu;
        const int kb_end = min(a.nb, kb_begin + a.nbu);
        float acc[2][NT][4];
#pragma unroll
        for (int r = 0; r < 2; ++r)
#pragma unroll
            for (int nt = 0; nt < NT; ++nt) acc[r][nt][0] = acc[r][nt][1] = acc[r][nt][2] = acc[r][nt][3] = 0.0f;
        const int row0 = tile * kRows + g;  // this lane's rows: row0 + {0, 8, 16, 24}
        XCursor xc;
        {
            constexpr int kRec = NATIVE ? 8 : 32;
            xc.rec = static_cast<const uint8_t*>(a.xa) + (((int64_t)kb_begin * a.M + g) * 4 + t) * kRec;
            xc.rec_step = (int64_t)a.M * 4 * kRec;
            xc.side = reinterpret_cast<const uint4*>(static_cast<const uint2*>(a.xs) + (int64_t)kb_begin * Mpad + 2 * t);
            xc.sx = reinterpret_cast<const float2*>(a.xsum + (int64_t)kb_begin * Mpad + 2 * t);
            xc.side_step = Mpad / 2;
#pragma unroll
            for (int nt = 0; nt < 8; ++nt) xc.valid[nt] = nt * 8 + g < a.M;
        }
        int chunk_start = kb_begin, chunk_end = kb_begin;
        const uint8_t* rb[4] = {smem, smem, smem, smem};
        bool ok = true;
        // acquire the stage holding block b (when b starts a new chunk)
        auto acquire = [&](int b) {
            if (b != chunk_end) return;
            if (b != kb_begin) {
                __syncwarp();
                if (lane == 0) mbar_arrive(&empty[warp * kSW + (lt % kSW)]);
                ++lt;
            }
            const int slot = lt % kSW;
            if (!mbar_wait_bounded(&full[warp * kSW + slot], (lt / kSW) & 1, a.err)) {
                ok = false;
                return;
            }
            chunk_start = b;
            chunk_end = min(kb_end, b + a.kc);
            const uint8_t* sbase = smem + (warp * kSW + slot) * stage_bytes;
#pragma unroll
            for (int i = 0; i < 4; ++i) {
                const uint64_t gaddr = (uint64_t)(row0 + 8 * i) * a.row_bytes + (uint64_t)b * BB;
                const int j = g + 8 * i;  // row within the tile
                if (a.loader == kLoaderTma2d) {
                    rb[i] = sbase + j * a.pitch;
                } else if (a.loader == kLoaderTmaPairs) {
                    rb[i] = sbase + ((j & 1) * (kRows / 2) + (j >> 1)) * a.pitch + (j & 1) * 8;
                } else {
                    rb[i] = sbase + j * a.pitch + (uint32_t)(gaddr & 15);
                }
            }
        };
        auto consume = [&](int b, const XFrag (&xf)[NT]) {
            const uint32_t o = (uint32_t)(b - chunk_start) * BB;
            consume_group<QT, NT, NATIVE>(rb[0] + o, rb[1] + o, t, xf, acc[0]);
            consume_group<QT, NT, NATIVE>(rb[2] + o, rb[3] + o, t, xf, acc[1]);
        };
        if constexpr (NT <= 2) {
            // activation fragments prefetched one block ahead, ping-pong buffers
            XFrag xa[NT], xb[NT];
            load_x<QT, NT, NATIVE>(xc, 0, xa);
            for (int b = kb_begin; b < kb_end; b += 2) {
                if (b + 1 < kb_end) load_x<QT, NT, NATIVE>(xc, b + 1 - kb_begin, xb);
                acquire(b);
                if (!ok) break;
                consume(b, xa);
                if (b + 1 >= kb_end) break;
                if (b + 2 < kb_end) load_x<QT, NT, NATIVE>(xc, b + 2 - kb_begin, xa);
                acquire(b + 1);
                if (!ok) break;
                consume(b + 1, xb);
            }
        } else {
            // wide token tiles: load in place (prefetching would spill registers)
            XFrag xa[NT];
            for (int b = kb_begin; b < kb_end; ++b) {
                load_x<QT, NT, NATIVE>(xc, b - kb_begin, xa);
                acquire(b);
                if (!ok) break;
                consume(b, xa);
            }
        }
        if (!ok) break;
        __syncwarp();
        if (lane == 0) mbar_arrive(&empty[warp * kSW + (lt % kSW)]);
        ++lt;
        // ------------------------------- epilogue -------------------------------------
        float* dst = a.ks == 1 ? a.y : a.partial + (int64_t)ksi * a.M * a.N;
#pragma unroll
        for (int r = 0; r < 2; ++r) {
            const int ra = row0 + 16 * r, rc = ra + 8;
#pragma unroll
            for (int nt = 0; nt < NT; ++nt) {
                const int m0 = nt * 8 + 2 * t, m1 = m0 + 1;
                if (ra < a.N) {
                    if (m0 < a.M) dst[(int64_t)m0 * a.N + ra] = acc[r][nt][0];
                    if (m1 < a.M) dst[(int64_t)m1 * a.N + ra] = acc[r][nt][1];
                }
                if (rc < a.N) {
                    if (m0 < a.M) dst[(int64_t)m0 * a.N + rc] = acc[r][nt][2];
                    if (m1 < a.M) dst[(int64_t)m1 * a.N + rc] = acc[r][nt][3];
                }
            }
        }
        if (a.ks > 1) {
            __threadfence();
            __syncwarp();
            unsigned ticket = 0;
            if (lane == 0) ticket = atomicAdd(&a.counters[tile], 1u);
            ticket = __shfl_sync(0xffffffffu, ticket, 0);
            if (ticket == (unsigned)(a.ks - 1)) {
                __threadfence();
                // the last split sums all partials of this tile in split order
#pragma unroll
                for (int r = 0; r < 2; ++r) {
#pragma unroll
                    for (int nt = 0; nt < NT; ++nt) {
#pragma unroll
                        for (int e = 0; e < 4; ++e) {
                            const int m = nt * 8 + 2 * t + (e & 1);
                            const int row = row0 + 16 * r + ((e & 2) ? 8 : 0);
                            if (m < a.M && row < a.N) {
                                float s = 0.0f;
                                for (int k = 0; k < a.ks; ++k)
                                    s += __ldcg(a.partial + ((int64_t)k * a.M + m) * a.N + row);
                                a.y[(int64_t)m * a.N + row] = s;
                            }
                        }
                    }
                }
                if (lane == 0) a.counters[tile] = 0u;
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

// cuTensorMapEncodeTiled through the runtime's driver entry point (no -lcuda).
using EncodeTiledFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                   const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                   CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiledFn encode_tiled() {
    static EncodeTiledFn fn = [] {
        void* p = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) != cudaSuccess ||
            q != cudaDriverEntryPointSuccess)
            p = nullptr;
        return reinterpret_cast<EncodeTiledFn>(p);
    }();
    return fn;
}

// Same tensor map, encoded on the stack with no cache (no heap allocation);
// used by the allocation-free entry point.
cudaError_t weight_tensor_map_uncached(const uint8_t* w, const GemvPlan& p, CUtensorMap* out) {
    EncodeTiledFn enc = encode_tiled();
    if (!enc) return cudaErrorNotSupported;
    const int R = p.loader == kLoaderTmaPairs ? 2 : 1;
    const cuuint64_t dims[2] = {(cuuint64_t)(R * p.row_bytes / 4), (cuuint64_t)(p.N / R)};
    const cuuint64_t strides[1] = {(cuuint64_t)(R * p.row_bytes)};
    const cuuint32_t box[2] = {(cuuint32_t)(p.pitch / 4), (cuuint32_t)(kRows / R)};
    const cuuint32_t estr[2] = {1, 1};
    const CUresult r = enc(out, CU_TENSOR_MAP_DATA_TYPE_UINT32, 2, const_cast<uint8_t*>(w), dims, strides, box, estr,
                           CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE,
                           CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    return r == CUDA_SUCCESS ? cudaSuccess : cudaErrorInvalidValue;
}

// The weights viewed as a [N rows][row_bytes / 4] uint32 tensor with a box of
// [kc blocks, 32 rows]. Encoded once per (device, pointer, shape, box).
cudaError_t weight_tensor_map(const uint8_t* w, const GemvPlan& p, CUtensorMap* out) {
    static std::mutex mu;
    static std::map<std::tuple<int, const void*, int, int, int>, CUtensorMap> cache;
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return e;
    const auto key = std::make_tuple(dev, (const void*)w, p.N, p.row_bytes, p.pitch * 4 + p.loader);
    std::lock_guard<std::mutex> lock(mu);
    auto it = cache.find(key);
    if (it != cache.end()) {
        *out = it->second;
        return cudaSuccess;
    }
    EncodeTiledFn enc = encode_tiled();
    if (!enc) return cudaErrorNotSupported;
    // pairs: [N/2][2 * row_bytes / 4] with 16-row boxes (one box per row parity)
    const int R = p.loader == kLoaderTmaPairs ? 2 : 1;
    const cuuint64_t dims[2] = {(cuuint64_t)(R * p.row_bytes / 4), (cuuint64_t)(p.N / R)};
    const cuuint64_t strides[1] = {(cuuint64_t)(R * p.row_bytes)};
    const cuuint32_t box[2] = {(cuuint32_t)(p.pitch / 4), (cuuint32_t)(kRows / R)};
    const cuuint32_t estr[2] = {1, 1};
    CUtensorMap m;
    const CUresult r = enc(&m, CU_TENSOR_MAP_DATA_TYPE_UINT32, 2, const_cast<uint8_t*>(w), dims, strides, box, estr,
                           CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE,
                           CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) return cudaErrorInvalidValue;
    if (cache.size() > 4096) cache.clear();
    cache[key] = m;
    *out = m;
    return cudaSuccess;
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
    const int tiles = (N + kRows - 1) / kRows;
    const int slots = num_sms * kW;
    int ks = 1;
    if (!native && tiles < slots) {
        ks = slots / tiles;
        const int max_ks = q.nb / 8 > 1 ? q.nb / 8 : 1;  // keep >= 8 blocks per split
        if (ks > max_ks) ks = max_ks;
        if (ks < 1) ks = 1;
    }
    // 16-byte row pitch: one 2-D TMA tile per stage (block offsets 8-aligned
    // so every tile starts on a 16-byte boundary); otherwise cp.async windows
    q.loader = (q.row_bytes % 16 == 0)                 ? kLoaderTma2d
               : (q.row_bytes % 16 == 8 && N % 2 == 0) ? kLoaderTmaPairs
                                                       : kLoaderCpAsync;
    if (q.loader != kLoaderCpAsync) {
        const int extra = q.loader == kLoaderTmaPairs ? 16 : 0;  // skew room for the odd rows
        q.nbu = ((q.nb + ks - 1) / ks + 7) / 8 * 8;
        q.ks = (q.nb + q.nbu - 1) / q.nbu;
        int kc = (kStageTarget / kRows) / bb / 8 * 8;
        if (kc < 8) kc = 8;
        if ((kc * bb + extra) / 4 > 256) kc = (1024 - extra) / bb / 8 * 8;  // TMA box inner extent <= 256 elements
        if (kc > q.nbu) kc = q.nbu;
        q.kc = kc;
        q.pitch = kc * bb + extra;  // the tile lands densely
    } else {
        q.nbu = (q.nb + ks - 1) / ks;
        q.ks = (q.nb + q.nbu - 1) / q.nbu;
        const int kc_max = (kStageTarget / kRows - 45) / bb;
        q.kc = q.nbu < kc_max ? q.nbu : kc_max;
        q.pitch = (int)(((size_t)q.kc * bb + 30 + 15) / 16 * 16);
    }
    q.units = tiles * q.ks;
    // units are dealt to CTAs first, so use every SM when there are enough
    q.grid = q.units < num_sms ? q.units : num_sms;
    q.smem = (size_t)kW * kSW * kRows * q.pitch + 2 * kW * kSW * sizeof(uint64_t);
    *p = q;
    return true;
}

size_t gemv_counters_bytes(const GemvPlan& p) {
    return p.ks > 1 ? align256((size_t)((p.N + kRows - 1) / kRows) * sizeof(unsigned)) : 0;
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
                        int* err, cudaStream_t st, bool no_host_alloc) {
    cudaError_t e;
    const int nzero = ws.counters ? (p.N + kRows - 1) / kRows : 0;
    if (p.native) {
        e = launch_xprep_q8(p.qt, x, p.M, p.K, static_cast<uint8_t*>(ws.xa), static_cast<int2*>(ws.xs), ws.counters,
                            nzero, st);
    } else {
        e = launch_xprep_f32(p.qt, x, p.M, p.K, static_cast<__half*>(ws.xa), static_cast<float2*>(ws.xs), ws.xsum,
                             ws.counters, nzero, st);
    }
    if (e != cudaSuccess) return e;
    const void* fn = kernel_for(p);
    // no_host_alloc: set the attribute and encode the tensor map on every call
    // instead of going through the (heap-backed) caches
    e = no_host_alloc ? cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)p.smem)
                      : ensure_dynamic_smem(fn, p.smem);
    if (e != cudaSuccess) return e;
    Args a;
    if (p.loader != kLoaderCpAsync) {
        e = no_host_alloc ? weight_tensor_map_uncached(w, p, &a.tmap) : weight_tensor_map(w, p, &a.tmap);
        if (e != cudaSuccess) return e;
    }
    a.loader = p.loader;
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
