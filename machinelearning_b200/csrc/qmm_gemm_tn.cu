// Decode-batch GEMM for sm_100a: tcgen05 tensor cores, TMEM accumulators,
// exact hi/lo operand split.
//
// y[M, N] = x[M, K] . W[N, K]^T for f32 activations and GGUF block weights
// (Q4_0 / Q4_1 / Q8_0 rows, raw bytes) when M is a decode batch (kGemmMinRows
// .. kGemmTnMaxRows tokens). Replaces the M > 4 row-parallel CPU loops of
// matmul_f32_q4 / _q8 / _q4_1 (reference llmserve/llmmodel/kernel/main/src/
// core/quantize.rs:317-395, 557-630, 807-932) for batched decode.
//
// Shape of the problem: few tokens, many weight rows. So the weights are the
// MMA's M side (128 rows per CTA tile, one TMEM lane each) and the tokens its
// N side (NT = 32, 64 or 128 columns), so no tensor work is padded beyond the
// next multiple of 32 tokens.
//
// Numerics: every operand is split exactly into an f16 high part and an f16
// residual --
//   weights:      w = d*q, wh = f16(d*q), wl = f16(d*q - wh) (fma: the residual
//                 of an 11 x 8-bit product fits an f16 exactly);
//   activations:  x * 2^-e (a power of two per token row, max in [2^14, 2^15)),
//                 xh = f16(.), xl = f16(. - xh);
// and each K step accumulates wh.xh + wl.xh + wh.xl in f32 (the dropped
// wl.xl is 2^-22 of the product). The result matches the reference's f32
// arithmetic to ~1e-6 relative, like the GEMV paths, so a 26-layer decode
// step stays inside the 1e-3 contract (a single f16 rounding per operand,
// ~3e-4 per matmul, compounds past it over the layers).
//
// Two launches per call:
//   1. gemm_tn_xprep: xh, xl [M][K] and the per-row scale.
//   2. gemm_tn_kernel<QT, NT, PAIRED>: one CTA per (128-row weight tile, K
//      slice), eleven warps:
//        warp 0    TMA producer of the xh / xl tiles [NT tokens x 64] per K
//                  step (128-byte swizzle, the canonical K-major UMMA layout);
//        warp 10   TMA producer of raw weight chunks (8 blocks of 128 rows):
//                  one 2-D box when the row pitch is a multiple of 16 bytes;
//                  for 8 mod 16 (K = 1152: 648-byte Q4_0 / 1224-byte Q8_0
//                  rows) the matrix viewed as [N/2][2 * row_bytes] and two
//                  boxes of 64 row pairs (even rows, then odd rows from 8
//                  bytes earlier), so those weights need no padded copy;
//        warp 1    allocates NT TMEM columns; one thread issues
//                  tcgen05.mma.kind::f16 (M 128, N NT, K 16) three times per
//                  16-wide K slice and commits to mbarriers that free the
//                  operand stages;
//        warps 2-9 dequantise (one 32-weight block of one row per thread per K
//                  step, into the swizzled wh and wl tiles), then read the
//                  accumulator back with tcgen05.ld, stage it in shared memory
//                  in weight-row order and store y (or the gate/up
//                  activation) scaled by 2^e.
//      With the paired view, tile row j < 64 is weight row 2j and j >= 64 row
//      2(j - 64) + 1, so every dequantising warp reads rows of one parity
//      (one compile-time byte skew) and writes 32 consecutive tile rows.
//      K slices (grid y) cover runs of whole raw chunks; with more than one,
//      each slice writes its tile to a workspace slab and the last to finish
//      (per-tile ticket) adds the slabs in slice order: deterministic.
// Every wait is bounded (the error word records a timeout; copies in flight
// land before a CTA exits).
#include <cuda.h>
#include <cuda_fp16.h>

#include <cstring>
#include <type_traits>

#include "qmm_common.cuh"
#include "qmm_kernels.cuh"
#include "qmm_tcgen05.cuh"

namespace qmm {

namespace {

using namespace tc;

constexpr int kTnRows = 128;       // weight rows per CTA tile (MMA M, TMEM lanes)
constexpr int kTnBK = 64;          // K per step: one 128-byte swizzle row of f16
constexpr int kTnStepsPerChunk = 4;  // a raw chunk is 8 blocks = 256 elements
constexpr int kTnSR = 2;           // raw chunk stages
constexpr int kTnDqThreads = 256;  // warps 2-9
constexpr int kTnThreads = 64 + kTnDqThreads + 32;
constexpr uint32_t kTnATile = kTnRows * kTnBK * 2;  // 16 KB: one of wh / wl

__host__ __device__ constexpr uint32_t tn_xtile(int NT) { return (uint32_t)NT * kTnBK * 2; }
// Raw chunk row pitch in shared memory (= the TMA box's inner extent): 8
// blocks, an odd number of 16-byte units (conflict-free 16-byte loads by
// consecutive rows); the paired view adds room for the odd rows' 8-byte skew.
__host__ __device__ constexpr int tn_pitch(int qt, bool paired) {
    return paired ? (qt == kQ8_0 ? 304 : (qt == kQ4_0 ? 176 : 208)) : (qt == kQ8_0 ? 272 : (qt == kQ4_0 ? 144 : 176));
}
// Operand ring depths, sized to fill 227 KB with the raw ring.
__host__ __device__ constexpr int tn_sa(int qt, int NT) {
    return NT == 128 ? (qt == kQ8_0 ? 2 : 3) : ((qt == kQ8_0 || (qt == kQ4_1 && NT == 64)) ? 3 : 4);
}
__host__ __device__ constexpr int tn_sx(int qt, int NT) {
    return NT == 32 ? (qt == kQ4_1 ? 5 : 6) : (NT == 64 ? 3 : 2);
}
__host__ __device__ constexpr size_t tn_smem_bytes(int qt, int NT, bool paired) {
    return 1024 + (size_t)tn_sa(qt, NT) * 2 * kTnATile + (size_t)tn_sx(qt, NT) * 2 * tn_xtile(NT) +
           (size_t)kTnSR * kTnRows * tn_pitch(qt, paired) + (2 * tn_sa(qt, NT) + 2 * tn_sx(qt, NT) + 2 * kTnSR + 1) * 8 +
           16;
}
constexpr bool tn_fits(int qt) {
    return tn_smem_bytes(qt, 32, true) <= 232448 && tn_smem_bytes(qt, 64, true) <= 232448 &&
           tn_smem_bytes(qt, 128, true) <= 232448;
}
static_assert(tn_fits(kQ4_0) && tn_fits(kQ4_1) && tn_fits(kQ8_0), "a decode-batch GEMM variant exceeds 227 KB");

struct TArgs {
    CUtensorMap tmap_xh;  // xh [M][K] f16, box [64, NT], 128-byte swizzle
    CUtensorMap tmap_xl;  // xl, same
    CUtensorMap tmap_w;   // raw weights as uint32: [N][row_bytes / 4] box [pitch / 4, 128], or
                          // paired [N / 2][row_bytes / 2] box [pitch / 4, 64]
    const float* xs;      // per-row activation scales 2^e
    float* y;
    int M, N, K, ksteps, row_bytes, weights_immutable;
    int* err;
    int ks, cps;          // K slices (grid y) and raw chunks per slice
    float* partial;       // [ks][M][N] unscaled slice tiles (ks > 1)
    unsigned* counters;   // [tiles] tickets, zero before the launch (ks > 1)
    int gact;             // >= 0: gate/up epilogue (GatedOut), y unused
    float* gout;
    int64_t ghidden;
};

// ---- dequantisation into exact hi / lo f16 pairs ------------------------------------
// q (an exact small integer in f16) times d: hi = f16(q*d), lo = f16(q*d - hi)
// (an fma: the exact residual of the 11-bit x 8-bit product is representable).
__device__ __forceinline__ void hl_pair(__half2 q, __half2 d2, uint32_t& hi, uint32_t& lo) {
    const __half2 h = __hmul2(q, d2);
    hi = h2_u32(h);
    lo = h2_u32(__hfma2(q, d2, __hneg2(h)));
}
// Q4_1 values d*n + m: formed in f32 (d*n exact, one f32 rounding of the sum),
// then split.
__device__ __forceinline__ void hl_pair_f32(float v0, float v1, uint32_t& hi, uint32_t& lo) {
    const __half2 h = __floats2half2_rn(v0, v1);
    const float2 hf = __half22float2(h);
    hi = h2_u32(h);
    lo = h2_u32(__floats2half2_rn(v0 - hf.x, v1 - hf.y));
}

// Q4: the low and high nibbles of bytes (b0, b1) of t = [b0, 0, b1, 0] as
// exact halves 1024 + n.
__device__ __forceinline__ uint32_t lo_nibbles(uint32_t t) { return lop3_and_or(t, 0x000F000Fu, 0x64006400u); }
__device__ __forceinline__ uint32_t hi_nibbles(uint32_t t) { return lop3_and_or(t >> 4, 0x000F000Fu, 0x64006400u); }

template <int P>
__device__ __forceinline__ uint32_t pl_word(const uint32_t* W, int i) {
    if constexpr (P % 4 == 0) return W[P / 4 + i];
    return __byte_perm(W[P / 4 + i], W[P / 4 + i + 1], 0x5432);
}

// One block of one weight row: the block starts OFF bytes into the row's raw
// chunk in shared memory (row base 16-byte aligned; OFF includes the paired
// view's 8-byte skew for odd rows). Its 32 weights become four 16-byte chunks
// of 8 f16 (elements in order) at chunk positions CB..CB+3 of the row's 128
// swizzled bytes, in the wh tile (dh) and the wl tile (dl).
template <int QT, int OFF, int CB>
__device__ __forceinline__ void dequant_block_hl(const uint8_t* row, uint8_t* dh, uint8_t* dl, int r7) {
    constexpr int BB = block_bytes(QT);
    constexpr int U0 = OFF / 16;
    constexpr int ST = OFF - 16 * U0;
    constexpr int NU = (ST + BB + 15) / 16;
    uint32_t W[4 * NU];
    const uint4* src = reinterpret_cast<const uint4*>(row) + U0;
#pragma unroll
    for (int u = 0; u < NU; ++u) {
        const uint4 v = src[u];
        W[4 * u] = v.x;
        W[4 * u + 1] = v.y;
        W[4 * u + 2] = v.z;
        W[4 * u + 3] = v.w;
    }
    const uint32_t hw = W[ST / 4];
    const uint32_t dbits = (ST % 4 == 0) ? (hw & 0xffffu) : (hw >> 16);
    const __half2 d2 = half2_from_bits(dbits);
    uint32_t H[16], L[16];  // pairs of elements 0-1, 2-3, ..., 30-31
    if constexpr (QT == kQ8_0) {
        const __half2 off = __float2half2_rn(1152.0f);
#pragma unroll
        for (int i = 0; i < 8; ++i) {
            const uint32_t u = pl_word<ST + 2>(W, i) ^ 0x80808080u;
            // halves 0x64XX = 1024 + XX = 1152 + q, exact
            hl_pair(__hsub2(as_h2(__byte_perm(u, 0x64646464u, 0x4140)), off), d2, H[2 * i], L[2 * i]);
            hl_pair(__hsub2(as_h2(__byte_perm(u, 0x64646464u, 0x4342)), off), d2, H[2 * i + 1], L[2 * i + 1]);
        }
    } else if constexpr (QT == kQ4_0) {
        const __half2 off = __float2half2_rn(1032.0f);
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            // GGML order: the low nibble of byte j is element j, the high nibble element j + 16
            const uint32_t p = pl_word<ST + 2>(W, i);
            const uint32_t t01 = __byte_perm(p, 0u, 0x4140), t23 = __byte_perm(p, 0u, 0x4342);
            hl_pair(__hsub2(as_h2(lo_nibbles(t01)), off), d2, H[2 * i], L[2 * i]);
            hl_pair(__hsub2(as_h2(lo_nibbles(t23)), off), d2, H[2 * i + 1], L[2 * i + 1]);
            hl_pair(__hsub2(as_h2(hi_nibbles(t01)), off), d2, H[8 + 2 * i], L[8 + 2 * i]);
            hl_pair(__hsub2(as_h2(hi_nibbles(t23)), off), d2, H[8 + 2 * i + 1], L[8 + 2 * i + 1]);
        }
    } else {
        const float d = __half2float(__ushort_as_half((unsigned short)dbits));
        const float m = __half2float(__ushort_as_half((unsigned short)(hw >> 16)));
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            const uint32_t p = pl_word<ST + 4>(W, i);
#pragma unroll
            for (int b = 0; b < 2; ++b) {
                const uint32_t b0 = (p >> (16 * b)) & 0xffu, b1 = (p >> (16 * b + 8)) & 0xffu;
                hl_pair_f32(fmaf(d, (float)(b0 & 15u), m), fmaf(d, (float)(b1 & 15u), m), H[2 * i + b],
                            L[2 * i + b]);
                hl_pair_f32(fmaf(d, (float)(b0 >> 4), m), fmaf(d, (float)(b1 >> 4), m), H[8 + 2 * i + b],
                            L[8 + 2 * i + b]);
            }
        }
    }
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        const uint32_t o = (uint32_t)(((CB + i) ^ r7) << 4);
        *reinterpret_cast<uint4*>(dh + o) = make_uint4(H[4 * i], H[4 * i + 1], H[4 * i + 2], H[4 * i + 3]);
        *reinterpret_cast<uint4*>(dl + o) = make_uint4(L[4 * i], L[4 * i + 1], L[4 * i + 2], L[4 * i + 3]);
    }
}

// Block BLK (0 or 1) of K step KK of a raw chunk, row skew SK (0, or 8 for the
// paired view's odd rows).
template <int QT, int KK, int BLK, int SK>
__device__ __forceinline__ void dequant_kstep_hl(const uint8_t* row, uint8_t* dh, uint8_t* dl, int r7) {
    dequant_block_hl<QT, SK + block_bytes(QT) * (2 * KK + BLK), 4 * BLK>(row, dh, dl, r7);
}

// 16 consecutive TMEM columns of this warp's 32 lanes, one lane per thread.
__device__ __forceinline__ void tmem_ld16(uint32_t taddr, uint32_t (&r)[16]) {
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
          "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
        : "r"(taddr));
    asm volatile("tcgen05.wait::ld.sync.aligned;"
                 : "+r"(r[0]), "+r"(r[1]), "+r"(r[2]), "+r"(r[3]), "+r"(r[4]), "+r"(r[5]), "+r"(r[6]), "+r"(r[7]),
                   "+r"(r[8]), "+r"(r[9]), "+r"(r[10]), "+r"(r[11]), "+r"(r[12]), "+r"(r[13]), "+r"(r[14]),
                   "+r"(r[15])
                 :
                 : "memory");
}

// ---- activation prep: x -> xh, xl (f16) with a power-of-two scale per row ------------
__global__ void gemm_tn_xprep_kernel(const float* __restrict__ x, int M, int K, __half* __restrict__ xh,
                                     __half* __restrict__ xl, float* __restrict__ xs) {
    pdl_launch_dependents();
    pdl_wait();  // x comes from the preceding work in the stream
    __shared__ float red[32];
    const int m = blockIdx.x;
    const float* row = x + (int64_t)m * K;
    const bool v4 = (reinterpret_cast<uintptr_t>(row) & 15) == 0;
    const int n4 = K >> 2;  // K is a multiple of 32
    const float4* r4 = reinterpret_cast<const float4*>(row);
    float am = 0.0f;
    if (v4) {
        for (int k = threadIdx.x; k < n4; k += 4 * blockDim.x) {
            float4 v[4];
#pragma unroll
            for (int u = 0; u < 4; ++u) {
                const int idx = k + u * blockDim.x;
                v[u] = idx < n4 ? r4[idx] : make_float4(0.0f, 0.0f, 0.0f, 0.0f);
            }
#pragma unroll
            for (int u = 0; u < 4; ++u)
                am = fmaxf(am, fmaxf(fmaxf(fabsf(v[u].x), fabsf(v[u].y)), fmaxf(fabsf(v[u].z), fabsf(v[u].w))));
        }
    } else {
        for (int k = threadIdx.x; k < K; k += blockDim.x) am = fmaxf(am, fabsf(row[k]));
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) am = fmaxf(am, __shfl_xor_sync(0xffffffffu, am, o));
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = am;
    __syncthreads();
    if (threadIdx.x < 32) {
        am = threadIdx.x < (blockDim.x >> 5) ? red[threadIdx.x] : 0.0f;
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) am = fmaxf(am, __shfl_xor_sync(0xffffffffu, am, o));
        if (threadIdx.x == 0) red[0] = am;
    }
    __syncthreads();
    am = red[0];
    int e = 0;
    if (am > 0.0f && am <= 3.402823466e38f) {
        const int bits = __float_as_int(am);
        const int E = (bits >> 23) != 0 ? (bits >> 23) - 126 : (31 - __clz(bits)) - 148;  // frexp exponent
        e = max(-126, min(127, E - 15));  // max |x| * 2^-e in [2^14, 2^15)
    }
    const float scale = (-e >= -126) ? __int_as_float((127 - e) << 23) : __int_as_float(0x00400000);
    __half* oh = xh + (int64_t)m * K;
    __half* ol = xl + (int64_t)m * K;
    auto split = [&](float v, __half& h, __half& l) {
        const float s = v * scale;  // exact (power of two, no overflow by the choice of e)
        h = __float2half_rn(s);
        l = __float2half_rn(s - __half2float(h));
    };
    if (v4) {
        for (int k = threadIdx.x; k < n4; k += blockDim.x) {
            const float4 v = r4[k];
            __half h[4], l[4];
            split(v.x, h[0], l[0]);
            split(v.y, h[1], l[1]);
            split(v.z, h[2], l[2]);
            split(v.w, h[3], l[3]);
            uint2 ph, pl;
            memcpy(&ph, h, 8);
            memcpy(&pl, l, 8);
            reinterpret_cast<uint2*>(oh)[k] = ph;
            reinterpret_cast<uint2*>(ol)[k] = pl;
        }
    } else {
        for (int k = threadIdx.x; k < K; k += blockDim.x) split(row[k], oh[k], ol[k]);
    }
    if (threadIdx.x == 0) xs[m] = __int_as_float((e + 127) << 23);
}

// Weight row of tile row j (natural order, or the paired view's even rows
// first, then the odd rows).
template <bool PAIRED>
__device__ __forceinline__ int tile_row(int j) {
    if constexpr (PAIRED) return j < 64 ? 2 * j : 2 * (j - 64) + 1;
    return j;
}

template <int QT, int NT, bool PAIRED>
__global__ void __launch_bounds__(kTnThreads, 1) gemm_tn_kernel(const __grid_constant__ TArgs a) {
    constexpr int SA = tn_sa(QT, NT), SX = tn_sx(QT, NT);
    constexpr int PITCH = tn_pitch(QT, PAIRED);
    constexpr uint32_t kXTile = tn_xtile(NT);
    constexpr uint32_t kTmemCols = NT;  // 32, 64 or 128: a power of two >= 32
    constexpr int YP = kTnRows + 4;     // staging pitch in floats (a token row of the tile)
    static_assert(NT * YP * 4 <= SA * 2 * kTnATile + SX * 2 * kXTile, "staging tile must fit in the operand rings");
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint8_t* sA = smem;                           // [SA][hi, lo] weight tiles
    uint8_t* sX = sA + SA * 2 * kTnATile;         // [SX][hi, lo] activation tiles
    uint8_t* sR = sX + SX * 2 * kXTile;           // [SR] raw chunks
    uint64_t* full_a = reinterpret_cast<uint64_t*>(sR + kTnSR * kTnRows * PITCH);
    uint64_t* empty_a = full_a + SA;
    uint64_t* full_x = empty_a + SA;
    uint64_t* empty_x = full_x + SX;
    uint64_t* rfull = empty_x + SX;
    uint64_t* rempty = rfull + kTnSR;
    uint64_t* acc_full = rempty + kTnSR;
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(acc_full + 1);

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int n0 = blockIdx.x * kTnRows;
    // K slice blockIdx.y: raw chunks [c_begin, c_begin + nchunks)
    const int nchunks_all = (a.ksteps + kTnStepsPerChunk - 1) / kTnStepsPerChunk;
    const int c_begin = (int)blockIdx.y * a.cps;
    const int nchunks = max(1, min(nchunks_all - c_begin, a.cps));  // the planner gives every slice a chunk
    const int steps = min(a.ksteps, (c_begin + nchunks) * kTnStepsPerChunk) - c_begin * kTnStepsPerChunk;

    if (threadIdx.x == 0) {
        for (int s = 0; s < SA; ++s) {
            mbar_init(&full_a[s], kTnDqThreads);
            mbar_init(&empty_a[s], 1);
        }
        for (int s = 0; s < SX; ++s) {
            mbar_init(&full_x[s], 1);
            mbar_init(&empty_x[s], 1);
        }
        for (int r = 0; r < kTnSR; ++r) {
            mbar_init(&rfull[r], 1);
            mbar_init(&rempty[r], kTnDqThreads);
        }
        mbar_init(acc_full, 1);
        fence_mbar_init();
        prefetch_tmap(&a.tmap_xh);
        prefetch_tmap(&a.tmap_xl);
        prefetch_tmap(&a.tmap_w);
    }
    if (warp == 1) {
        tmem_alloc(tmem_slot, kTmemCols);
        tmem_relinquish();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;
    pdl_launch_dependents();

    if (warp == 0) {
        // ----------------------- xh / xl (B operand) TMA producer ------------------------
        if (lane == 0) {
            int issued = 0;
            pdl_wait();  // xh / xl are written by the activation-prep launch
            for (int i = 0; i < steps; ++i) {
                const int s = i % SX;
                if (i >= SX && !mbar_wait_bounded(&empty_x[s], ((i / SX) - 1) & 1, a.err)) break;
                const int kx = (c_begin * kTnStepsPerChunk + i) * kTnBK;
                mbar_arrive_expect_tx(&full_x[s], 2 * kXTile);
                tma_load_2d(sX + (2 * s) * kXTile, &a.tmap_xh, kx, 0, &full_x[s]);
                tma_load_2d(sX + (2 * s + 1) * kXTile, &a.tmap_xl, kx, 0, &full_x[s]);
                ++issued;
            }
            // every copy this thread started has landed before the CTA can exit
            for (int i = (issued > SX ? issued - SX : 0); i < issued; ++i)
                mbar_wait_bounded(&full_x[i % SX], (i / SX) & 1, nullptr);
        }
    } else if (warp == kTnThreads / 32 - 1) {
        // ------------------------- raw weight chunk producer ----------------------------
        if (lane == 0) {
            int r_issued = 0;
            const int BB = block_bytes(QT);
            auto issue_raw = [&](int ci) {
                const int sr = ci % kTnSR;
                const int cb = (c_begin + ci) * 8 * BB;  // byte offset of the chunk in a row
                uint8_t* dst = sR + sr * kTnRows * PITCH;
                mbar_arrive_expect_tx(&rfull[sr], (uint32_t)(kTnRows * PITCH));
                if constexpr (PAIRED) {
                    // even rows 2p at [p][cb], odd rows 2p + 1 from 8 bytes before
                    // their chunk: [p][row_bytes + cb - 8] (16-byte aligned)
                    tma_load_2d(dst, &a.tmap_w, cb / 4, n0 / 2, &rfull[sr]);
                    tma_load_2d(dst + 64 * PITCH, &a.tmap_w, (a.row_bytes + cb - 8) / 4, n0 / 2, &rfull[sr]);
                } else {
                    tma_load_2d(dst, &a.tmap_w, cb / 4, n0, &rfull[sr]);
                }
            };
            // immutable weights: the first chunks may load before the dependency wait
            if (a.weights_immutable)
                for (; r_issued < kTnSR && r_issued < nchunks; ++r_issued) issue_raw(r_issued);
            pdl_wait();
            for (; r_issued < nchunks; ++r_issued) {
                if (r_issued >= kTnSR &&
                    !mbar_wait_bounded(&rempty[r_issued % kTnSR], ((r_issued / kTnSR) - 1) & 1, a.err))
                    break;
                issue_raw(r_issued);
            }
            for (int i = (r_issued > kTnSR ? r_issued - kTnSR : 0); i < r_issued; ++i)
                mbar_wait_bounded(&rfull[i % kTnSR], (i / kTnSR) & 1, nullptr);
        }
    } else if (warp == 1) {
        // ------------------------------- MMA issuer -----------------------------------
        if (lane == 0) {
            pdl_wait();
            constexpr uint32_t idesc = gemm_idesc(NT, kTnRows);
            for (int i = 0; i < steps; ++i) {
                const int sa = i % SA, sx = i % SX;
                if (!mbar_wait_bounded(&full_x[sx], (i / SX) & 1, a.err) ||
                    !mbar_wait_bounded(&full_a[sa], (i / SA) & 1, a.err))
                    break;
                tc_fence_after();
                const uint64_t ah = sw128_desc(smem_u32(sA + (2 * sa) * kTnATile));
                const uint64_t al = sw128_desc(smem_u32(sA + (2 * sa + 1) * kTnATile));
                const uint64_t bh = sw128_desc(smem_u32(sX + (2 * sx) * kXTile));
                const uint64_t bl = sw128_desc(smem_u32(sX + (2 * sx + 1) * kXTile));
#pragma unroll
                for (int k = 0; k < kTnBK / 16; ++k) {  // 32-byte steps inside the swizzle atom
                    mma_f16_ss(tmem, ah + 2 * k, bh + 2 * k, idesc, (i | k) != 0 ? 1u : 0u);
                    mma_f16_ss(tmem, al + 2 * k, bh + 2 * k, idesc, 1u);
                    mma_f16_ss(tmem, ah + 2 * k, bl + 2 * k, idesc, 1u);
                }
                // both stages are free once these MMAs have read them
                mma_commit(&empty_x[sx]);
                mma_commit(&empty_a[sa]);
            }
            mma_commit(acc_full);  // arrives when every MMA above has completed
        }
        __syncwarp();
    } else {
        // --------------------- dequantisers, then the epilogue (warps 2-9) ----------------
        const int d = threadIdx.x - 64;
        const int j = d & (kTnRows - 1);  // tile row
        const int blk = d >> 7;           // which block of the K step (warp-uniform)
        const int r7 = j & 7;
        // paired view: tile rows 64..127 are odd weight rows, 8 bytes into their raw row
        const bool skew = PAIRED && j >= 64;  // warp-uniform
        const int nb = a.K / QK;
        pdl_wait();
        bool ok = true;
        int cur_chunk = 0;  // raw chunk being consumed (within this slice)
        auto step = [&](int i, int sr, auto kk) {  // operand step i, K step KK of raw stage sr
            constexpr int KK = decltype(kk)::value;
            const int s = i % SA;
            if (i >= SA && !mbar_wait_bounded(&empty_a[s], ((i / SA) - 1) & 1, a.err)) return false;
            const uint8_t* rrow = sR + sr * kTnRows * PITCH + j * PITCH;
            const uint32_t off = (uint32_t)((j >> 3) * 1024 + r7 * 128);
            uint8_t* dh = sA + (2 * s) * kTnATile + off;
            uint8_t* dl = sA + (2 * s + 1) * kTnATile + off;
            if (((c_begin + cur_chunk) * kTnStepsPerChunk + KK) * 2 + blk >= nb) {
                // a block past the row end (K not a multiple of the chunk): zeros,
                // whatever bytes the box brought (the next row's, in the paired view)
#pragma unroll
                for (int c = 0; c < 4; ++c) {
                    const uint32_t o = (uint32_t)(((4 * blk + c) ^ r7) << 4);
                    *reinterpret_cast<uint4*>(dh + o) = make_uint4(0, 0, 0, 0);
                    *reinterpret_cast<uint4*>(dl + o) = make_uint4(0, 0, 0, 0);
                }
            } else if (blk == 0) {
                if (skew)
                    dequant_kstep_hl<QT, KK, 0, 8>(rrow, dh, dl, r7);
                else
                    dequant_kstep_hl<QT, KK, 0, 0>(rrow, dh, dl, r7);
            } else {
                if (skew)
                    dequant_kstep_hl<QT, KK, 1, 8>(rrow, dh, dl, r7);
                else
                    dequant_kstep_hl<QT, KK, 1, 0>(rrow, dh, dl, r7);
            }
            fence_proxy_async_smem();  // generic writes -> visible to the tensor core
            mbar_arrive(&full_a[s]);
            return true;
        };
        int i = 0;  // operand steps done
        for (int ci = 0; ci < nchunks && ok; ++ci) {
            const int sr = ci % kTnSR;
            if (!mbar_wait_bounded(&rfull[sr], (ci / kTnSR) & 1, a.err)) break;
            const int nk = min(kTnStepsPerChunk, a.ksteps - (c_begin + ci) * kTnStepsPerChunk);
            cur_chunk = ci;
            ok = step(i, sr, std::integral_constant<int, 0>{});
            if (ok && nk > 1) ok = step(i + 1, sr, std::integral_constant<int, 1>{});
            if (ok && nk > 2) ok = step(i + 2, sr, std::integral_constant<int, 2>{});
            if (ok && nk > 3) ok = step(i + 3, sr, std::integral_constant<int, 3>{});
            i += nk;
            mbar_arrive(&rempty[sr]);  // the chunk is consumed
        }
        // Epilogue: accumulator [128 tile rows][NT tokens] -> staging [token][weight
        // row] in the (idle) weight ring -> y rows, coalesced.
        const bool acc_ok = mbar_wait_bounded(acc_full, 0, a.err);
        tc_fence_after();
        const int q = warp & 3;               // this warp's TMEM lane quarter
        const int half = (warp - 2) >> 2;     // which half of the token columns
        const int jr = q * 32 + lane;         // tile row of this thread
        const int wr = tile_row<PAIRED>(jr);  // its weight row within the tile
        float* ys = reinterpret_cast<float*>(sA);
        constexpr int CH = NT / 2;  // token columns per warp
#pragma unroll
        for (int c0 = 0; c0 < CH; c0 += 16) {
            uint32_t v[16];
            tmem_ld16(tmem + ((uint32_t)(q * 32) << 16) + (uint32_t)(half * CH + c0), v);
#pragma unroll
            for (int c = 0; c < 16; ++c) ys[(half * CH + c0 + c) * YP + wr] = __uint_as_float(v[c]);
        }
        tc_fence_before();
        asm volatile("bar.sync 1, %0;" ::"r"(kTnDqThreads) : "memory");  // the staging tile is complete
        const int et = threadIdx.x - 64;  // 0 .. 255
        const int Mv = min(a.M, NT);
        bool store = acc_ok;
        if (a.ks > 1) {
            // K split: this slice's unscaled tile to the workspace; the last
            // slice of the tile to arrive rebuilds the staging tile as the sum of
            // all slices in slice order, then stores it like an unsplit tile
            float* mine = a.partial + (int64_t)blockIdx.y * a.M * a.N;
            for (int idx = et; idx < Mv * kTnRows; idx += kTnDqThreads) {
                const int m = idx / kTnRows, c = idx % kTnRows;
                if (n0 + c < a.N) mine[(int64_t)m * a.N + n0 + c] = ys[m * YP + c];
            }
            __threadfence();
            asm volatile("bar.sync 1, %0;" ::"r"(kTnDqThreads) : "memory");
            uint32_t* flag = tmem_slot + 1;
            if (et == 0) {
                const unsigned t = atomicAdd(&a.counters[blockIdx.x], 1u);
                *flag = (t == (unsigned)(a.ks - 1)) ? 1u : 0u;
                if (t == (unsigned)(a.ks - 1)) a.counters[blockIdx.x] = 0u;  // left zero for the next call
            }
            asm volatile("bar.sync 1, %0;" ::"r"(kTnDqThreads) : "memory");
            store = store && *flag != 0u;
            if (store) {
                __threadfence();
                for (int idx = et; idx < Mv * kTnRows; idx += kTnDqThreads) {
                    const int m = idx / kTnRows, c = idx % kTnRows;
                    float s = 0.0f;
                    if (n0 + c < a.N)
                        for (int z = 0; z < a.ks; ++z) s += __ldcg(a.partial + ((int64_t)z * a.M + m) * a.N + n0 + c);
                    ys[m * YP + c] = s;
                }
            }
            asm volatile("bar.sync 1, %0;" ::"r"(kTnDqThreads) : "memory");
        }
        if (store) {
            if (a.gact >= 0) {
                // gate/up weight: tile rows [32g, 32g + 16) are gate rows n0 / 2 +
                // 16g + [0, 16), the next 16 the matching up rows
                for (int idx = et; idx < Mv * (kTnRows / 2); idx += kTnDqThreads) {
                    const int m = idx / (kTnRows / 2), h = idx % (kTnRows / 2);
                    const int c = 32 * (h >> 4) + (h & 15);
                    const int64_t gi = (int64_t)(n0 / 2) + h;
                    if (gi < a.ghidden) {
                        const float sc = a.xs[m];
                        a.gout[(int64_t)m * a.ghidden + gi] =
                            gated_value(a.gact, ys[m * YP + c] * sc, ys[m * YP + c + 16] * sc);
                    }
                }
            } else {
                for (int idx = et; idx < Mv * kTnRows; idx += kTnDqThreads) {
                    const int m = idx / kTnRows, c = idx % kTnRows;
                    if (n0 + c < a.N) a.y[(int64_t)m * a.N + n0 + c] = ys[m * YP + c] * a.xs[m];
                }
            }
        }
    }
    __syncthreads();
    if (warp == 1) {
        tc_fence_after();
        tmem_dealloc(tmem, kTmemCols);
    }
}

template <int QT, bool PAIRED>
const void* tn_pick_nt(int nt) {
    if (nt == 32) return (const void*)gemm_tn_kernel<QT, 32, PAIRED>;
    if (nt == 64) return (const void*)gemm_tn_kernel<QT, 64, PAIRED>;
    return (const void*)gemm_tn_kernel<QT, 128, PAIRED>;
}
const void* gemm_tn_kernel_for(int qt, int nt, bool paired) {
    if (qt == kQ8_0) return paired ? tn_pick_nt<kQ8_0, true>(nt) : tn_pick_nt<kQ8_0, false>(nt);
    if (qt == kQ4_0) return paired ? tn_pick_nt<kQ4_0, true>(nt) : tn_pick_nt<kQ4_0, false>(nt);
    return paired ? tn_pick_nt<kQ4_1, true>(nt) : tn_pick_nt<kQ4_1, false>(nt);
}

cudaError_t tn_launch_ex(const void* fn, dim3 grid, dim3 block, size_t smem, cudaStream_t st, void** args) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.dynamicSmemBytes = smem;
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    note_launch();
    return cudaLaunchKernelExC(&cfg, fn, args);
}

size_t al256(size_t v) { return (v + 255) & ~size_t(255); }

int tn_nt(int M) { return M <= 32 ? 32 : (M <= 64 ? 64 : 128); }

// Launch shape: K slices (1, 2, 4 or 8, whole raw chunks each) for the fewest
// rounds of CTAs (one per SM) times (K steps per CTA + a CTA's fixed cost of
// set-up, pipeline fill and epilogue, worth ~24 K steps), with a 3% charge per
// split for the slab round trip.
struct TnPlan {
    int nt, ks, cps;
};
TnPlan tn_plan(int M, int N, int K) {
    TnPlan p{tn_nt(M), 1, 0};
    int sms = 148, dev = 0;
    if (cudaGetDevice(&dev) == cudaSuccess) cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    const int ksteps = (K + kTnBK - 1) / kTnBK;
    const int nch = (ksteps + kTnStepsPerChunk - 1) / kTnStepsPerChunk;
    const long tiles = (N + kTnRows - 1) / kTnRows;
    p.cps = nch;
    double best = -1.0;
    for (int ks = 1; ks <= 8; ks *= 2) {
        const int cps = (nch + ks - 1) / ks;
        if ((nch + cps - 1) / cps != ks) continue;  // every slice gets a chunk
        const long rounds = (tiles * ks + sms - 1) / sms;
        const int steps = min(ksteps, cps * kTnStepsPerChunk);
        const double cost = (double)rounds * (steps + 24.0) * (1.0 + 0.03 * (ks > 1 ? 1 : 0));
        if (best < 0.0 || cost < best) {
            best = cost;
            p.ks = ks;
            p.cps = cps;
        }
    }
    return p;
}

}  // namespace

bool gemm_tn_supported(int qt, bool native, int M, int N, int K) {
    if (native || M < kGemmMinRows || M > kGemmTnMaxRows || N < 1 || K < QK || K % QK) return false;
    const int bb = block_bytes(qt);
    if (!bb) return false;
    const int64_t row_bytes = (int64_t)(K / QK) * bb;
    return row_bytes % 16 == 0 || (row_bytes % 16 == 8 && N % 2 == 0);
}

size_t gemm_tn_workspace_bytes(int M, int N, int K, int qt) {
    (void)qt;
    const TnPlan p = tn_plan(M, N, K);
    size_t b = 2 * al256((size_t)M * K * 2) + al256((size_t)M * 4);
    if (p.ks > 1) b += al256((size_t)p.ks * M * N * 4) + al256((size_t)((N + kTnRows - 1) / kTnRows) * 4);
    return b;
}

cudaError_t launch_gemm_tn(int qt, const uint8_t* w, const float* x, float* y, int M, int N, int K, void* ws,
                           int* err, cudaStream_t st, bool weights_immutable, const GatedOut& g) {
    uint8_t* base = static_cast<uint8_t*>(ws);
    __half* xh = reinterpret_cast<__half*>(base);
    __half* xl = reinterpret_cast<__half*>(base + al256((size_t)M * K * 2));
    float* xs = reinterpret_cast<float*>(base + 2 * al256((size_t)M * K * 2));
    {
        void* args[] = {(void*)&x, (void*)&M, (void*)&K, (void*)&xh, (void*)&xl, (void*)&xs};
        cudaError_t e = tn_launch_ex((const void*)gemm_tn_xprep_kernel, dim3(M), dim3(256), 0, st, args);
        if (e != cudaSuccess) return e;
    }
    const TnPlan p = tn_plan(M, N, K);
    const int row_bytes = (K / QK) * block_bytes(qt);
    const bool paired = row_bytes % 16 != 0;
    const int pitch = tn_pitch(qt, paired);
    TArgs a;
    cudaError_t e = encode_map_2d(&a.tmap_xh, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, xh, (uint64_t)K, (uint64_t)M,
                                  (uint64_t)K * 2, kTnBK, (uint32_t)p.nt, CU_TENSOR_MAP_SWIZZLE_128B);
    if (e == cudaSuccess)
        e = encode_map_2d(&a.tmap_xl, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, xl, (uint64_t)K, (uint64_t)M, (uint64_t)K * 2,
                          kTnBK, (uint32_t)p.nt, CU_TENSOR_MAP_SWIZZLE_128B);
    if (e == cudaSuccess) {
        if (paired)
            e = encode_map_2d(&a.tmap_w, CU_TENSOR_MAP_DATA_TYPE_UINT32, w, (uint64_t)row_bytes / 2, (uint64_t)N / 2,
                              (uint64_t)row_bytes * 2, (uint32_t)pitch / 4, 64, CU_TENSOR_MAP_SWIZZLE_NONE);
        else
            e = encode_map_2d(&a.tmap_w, CU_TENSOR_MAP_DATA_TYPE_UINT32, w, (uint64_t)row_bytes / 4, (uint64_t)N,
                              (uint64_t)row_bytes, (uint32_t)pitch / 4, kTnRows, CU_TENSOR_MAP_SWIZZLE_NONE);
    }
    if (e != cudaSuccess) return e;
    const long tiles = (N + kTnRows - 1) / kTnRows;
    a.ks = p.ks;
    a.cps = p.cps;
    a.partial = nullptr;
    a.counters = nullptr;
    if (p.ks > 1) {
        uint8_t* b = base + 2 * al256((size_t)M * K * 2) + al256((size_t)M * 4);
        a.partial = reinterpret_cast<float*>(b);
        a.counters = reinterpret_cast<unsigned*>(b + al256((size_t)p.ks * M * N * 4));
        e = cudaMemsetAsync(a.counters, 0, (size_t)tiles * 4, st);  // the tickets start from zero
        if (e != cudaSuccess) return e;
    }
    a.xs = xs;
    a.y = y;
    a.M = M;
    a.N = N;
    a.K = K;
    a.ksteps = (K + kTnBK - 1) / kTnBK;
    a.row_bytes = row_bytes;
    a.weights_immutable = weights_immutable ? 1 : 0;
    a.err = err;
    a.gact = g.act;
    a.gout = g.out;
    a.ghidden = g.hidden;
    const void* fn = gemm_tn_kernel_for(qt, p.nt, paired);
    const size_t smem = tn_smem_bytes(qt, p.nt, paired);
    e = ensure_dynamic_smem(fn, smem);
    if (e != cudaSuccess) return e;
    void* args[] = {(void*)&a};
    return tn_launch_ex(fn, dim3((unsigned)tiles, (unsigned)p.ks), dim3(kTnThreads), smem, st, args);
}

}  // namespace qmm
