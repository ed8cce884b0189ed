// Decode-batch GEMM for sm_100a: tcgen05 tensor cores, exact hi/lo operand
// split stacked into a single MMA, stream-K schedule.
//
// y[M, N] = x[M, K] . W[N, K]^T for f32 activations and GGUF block weights
// (Q4_0 / Q4_1 / Q8_0 rows, raw bytes) for the decode batches (17 ..
// kGemmTnMaxRows tokens) the f16 GEMM of qmm_gemm.cu does not take: row
// pitches of 8 mod 16 bytes with odd N or more than 64 tokens. Replaces the
// M > 4 row-parallel CPU loops of
// matmul_f32_q4 / _q8 / _q4_1 (reference llmserve/llmmodel/kernel/main/src/
// core/quantize.rs:317-395, 557-630, 807-932) for batched decode.
//
// Numerics: every operand is split exactly into an f16 high part and an f16
// residual --
//   weights:      w = d*q, wh = f16(d*q), wl = f16(d*q - wh) (an fma: the
//                 residual of an 11 x 8-bit product fits an f16 exactly);
//   activations:  x * 2^-e (a power of two per token row, max in [2^14, 2^15)),
//                 xh = f16(.), xl = f16(. - xh);
// and the four products wh.xh + wl.xh + wh.xl + wl.xl accumulate in f32:
// ~1e-6 relative to the reference's f32 arithmetic, like the GEMV paths.
//
// All four products come from ONE MMA per 16-wide K slice, at the tensor
// core's full width:
//   A (M side) = the activation stack of a tile of NT tokens: per group of G
//                tokens (G = NT / 4), their xh rows then their xl rows, so
//                each TMEM lane quarter holds G tokens' xh and xl results and
//                one shuffle adds them (MMA M = 2 NT: 64 for NT = 32, the
//                accumulator in lanes 0-15 of each quarter; 128 for NT = 64);
//   B (N side) = 128 weight rows as [wh rows | wl rows]: N = 256;
//   D (TMEM)   = 2 NT rows x 256 columns; y[t][n] =
//                (D[xh t][n] + D[xh t][128 + n]) + (D[xl t][n] + D[xl t][128 + n]).
// (Weights on the M side with the tokens on N would pay a full M = 128 MMA
// per 16 K for a 32-wide N: measured 6x slower on B200.)
//
// Schedule: stream-K. The (128-row weight tile, 8-block K chunk) work items
// of a token tile are cut into one contiguous, equal range per persistent CTA
// (grid x; grid y: token tiles); a tile split between CTAs is summed from
// per-CTA partial slabs by the last to finish (a ticket per tile), in K order:
// deterministic.
//
// Two launches per call: gemm_tn_xprep (the activation stacks [2 NT rows per
// token tile][K] f16, the per-row scales), then gemm_tn_kernel<QT, NT, PAIRED>,
// fifteen warps:
//   warp 0     TMA: the stack tile [2 NT rows x 64 k] per K step (128-byte
//              swizzle, the canonical K-major operand layout);
//   warp 14    TMA: raw weight chunks (8 blocks x 128 rows): one 2-D box when
//              the row pitch is a multiple of 16 bytes; for 8 mod 16 (K = 1152:
//              648-byte Q4_0 / 1224-byte Q8_0 rows) the matrix viewed as
//              [N/2][2 * row_bytes] and two boxes of 64 row pairs (even rows,
//              then odd rows from 8 bytes earlier): no padded copy;
//   warp 1     allocates 512 TMEM columns (two accumulators); one thread issues
//              tcgen05.mma.kind::f16 and commits;
//   warps 2-9  dequantise one 32-weight block of one row per thread per K step
//              (ld.shared of the raw bytes, exact hi/lo pairs) into the
//              swizzled B tile: wh at row j, wl at row 128 + j;
//   warps 10-13 epilogue: tcgen05.ld, the hi/lo sums, scale 2^e, store (or
//              the gate/up activation), or the CTA's partial slab.
// With the paired view, tile row j < 64 is weight row 2j and j >= 64 row
// 2(j - 64) + 1 (a dequantising warp reads rows of one parity). Every wait is
// bounded (the error word records a timeout; copies in flight land before a
// CTA exits).
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

constexpr int kTnRows = 128;         // weight rows per tile (the B operand holds wh and wl: N = 256)
constexpr int kTnBK = 64;            // K per step
constexpr int kTnStepsPerChunk = 4;  // a raw chunk is 8 blocks = 256 elements
constexpr int kTnThreads = 15 * 32;
constexpr int kTnDqThreads = 256;    // warps 2-9
constexpr int kTnEpiThreads = 128;   // warps 10-13
constexpr int kTnSB = 2;             // dequantised weight stages (32 KB each)
constexpr uint32_t kTnBTile = 2 * kTnRows * kTnBK * 2;  // 32 KB: wh and wl rows
constexpr int kTnMinChunks = 2;      // work items per CTA at least

__host__ __device__ constexpr uint32_t tn_atile(int NT) { return (uint32_t)(2 * NT) * kTnBK * 2; }
__host__ __device__ constexpr int tn_sa(int NT) { return NT == 32 ? 6 : 4; }
// Raw chunk row pitch in shared memory (= the TMA box's inner extent): 8
// blocks, an odd number of 16-byte units (conflict-free 16-byte loads by
// consecutive rows); the paired view adds room for the odd rows' 8-byte skew.
__host__ __device__ constexpr int tn_pitch(int qt, bool paired) {
    return paired ? (qt == kQ8_0 ? 304 : (qt == kQ4_0 ? 176 : 208)) : (qt == kQ8_0 ? 272 : (qt == kQ4_0 ? 144 : 176));
}
constexpr size_t kTnSmemBudget = 232448 - 1024 - 512;
__host__ __device__ constexpr int tn_sr_raw(int qt, int NT, bool paired) {
    return (int)((kTnSmemBudget - (size_t)tn_sa(NT) * tn_atile(NT) - (size_t)kTnSB * kTnBTile) /
                 ((size_t)kTnRows * tn_pitch(qt, paired)));
}
__host__ __device__ constexpr int tn_sr(int qt, int NT, bool paired) {
    return tn_sr_raw(qt, NT, paired) > 8 ? 8 : tn_sr_raw(qt, NT, paired);
}
__host__ __device__ constexpr size_t tn_smem_bytes(int qt, int NT, bool paired) {
    return 1024 + (size_t)tn_sa(NT) * tn_atile(NT) + (size_t)kTnSB * kTnBTile +
           (size_t)tn_sr(qt, NT, paired) * kTnRows * tn_pitch(qt, paired) +
           (2 * tn_sa(NT) + 2 * kTnSB + 2 * tn_sr(qt, NT, paired) + 4) * 8 + 16;
}
constexpr bool tn_fits(int qt) {
    return tn_sr(qt, 64, true) >= 2 && tn_smem_bytes(qt, 32, true) <= 232448 && tn_smem_bytes(qt, 64, true) <= 232448;
}
static_assert(tn_fits(kQ4_0) && tn_fits(kQ4_1) && tn_fits(kQ8_0), "a decode-batch GEMM variant exceeds 227 KB");

struct TArgs {
    CUtensorMap tmap_x;   // activation stacks [ntok * 2 NT][K] f16, box [64, 2 NT], 128-byte swizzle
    CUtensorMap tmap_w;   // raw weights as uint32: [N][row_bytes / 4] box [pitch / 4, 128], or
                          // paired [N / 2][row_bytes / 2] box [pitch / 4, 64]
    const float* xs;      // per-token activation scales 2^e
    float* y;
    int M, N, K, nb, ksteps, kchunks, tiles, row_bytes, weights_immutable;
    int64_t W;            // work items per token tile: tiles * kchunks
    int* err;
    float* partial;       // [token tiles][grid][2][NT][128] unscaled partial tiles
    unsigned* counters;   // [token tiles][tiles] tickets, zero before the launch
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


// ---- activation prep: x -> the xh / xl stacks, with a power-of-two scale per row --------
// Row of token t in the stack buffer: token tile T = t / NT, t' = t % NT, group
// i = t' / G, r = t' % G (G = NT / 4): T * 2 NT + 2 G i + r (xh) or + G (xl).
// Tokens M .. ntok * NT - 1 get zero rows.
__global__ void gemm_tn_xprep_kernel(const float* __restrict__ x, int M, int K, int NT, __half* __restrict__ xst,
                                     float* __restrict__ xs) {
    pdl_launch_dependents();
    pdl_wait();  // x comes from the preceding work in the stream
    __shared__ float red[32];
    const int t = blockIdx.x;
    const int G = NT / 4;
    const int tt = t % NT, gi = tt / G, r = tt % G;
    const int64_t rh = (int64_t)(t / NT) * 2 * NT + 2 * G * gi + r;
    __half* oh = xst + rh * K;
    __half* ol = xst + (rh + G) * K;
    if (t >= M) {  // padding token: zero rows
        for (int k = threadIdx.x; k < K; k += blockDim.x) {
            oh[k] = __float2half_rn(0.0f);
            ol[k] = __float2half_rn(0.0f);
        }
        return;
    }
    const float* row = x + (int64_t)t * K;
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
    auto split = [&](float v, __half& h, __half& l) {
        const float sv = v * scale;  // exact (power of two, no overflow by the choice of e)
        h = __float2half_rn(sv);
        l = __float2half_rn(sv - __half2float(h));
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
    if (threadIdx.x == 0) xs[t] = __int_as_float((e + 127) << 23);
}

__device__ __forceinline__ uint4 lds128(uint32_t a) {
    uint4 v;
    asm volatile("ld.shared.v4.u32 {%0, %1, %2, %3}, [%4];" : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w) : "r"(a));
    return v;
}

// One block of one weight row into hi / lo f16 pairs H[16], L[16] (pairs of
// elements 0-1, ..., 30-31): the block starts OFF bytes into the row's raw
// chunk at shared address `row` (16-byte aligned; OFF includes the paired
// view's 8-byte skew for odd rows).
template <int QT, int OFF>
__device__ __forceinline__ void dequant_hl(uint32_t row, uint32_t (&H)[16], uint32_t (&L)[16]) {
    constexpr int BB = block_bytes(QT);
    constexpr int U0 = OFF / 16;
    constexpr int ST = OFF - 16 * U0;
    constexpr int NU = (ST + BB + 15) / 16;
    uint32_t W[4 * NU];
#pragma unroll
    for (int u = 0; u < NU; ++u) {
        const uint4 v = lds128(row + 16u * (uint32_t)(U0 + u));
        W[4 * u] = v.x;
        W[4 * u + 1] = v.y;
        W[4 * u + 2] = v.z;
        W[4 * u + 3] = v.w;
    }
    const uint32_t hw = W[ST / 4];
    const uint32_t dbits = (ST % 4 == 0) ? (hw & 0xffffu) : (hw >> 16);
    const __half2 d2 = half2_from_bits(dbits);
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
        const uint32_t mbits = (ST % 4 == 0) ? (hw >> 16) : (W[ST / 4 + 1] & 0xffffu);
        const float m = __half2float(__ushort_as_half((unsigned short)mbits));
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
}

// Block H (0 or 1) of K step KK of a raw chunk, row skew SK.
template <int QT, int KK, int H, int SK>
__device__ __forceinline__ void dequant_step_hl(uint32_t row, uint32_t (&Hv)[16], uint32_t (&Lv)[16]) {
    dequant_hl<QT, SK + block_bytes(QT) * (2 * KK + H)>(row, Hv, Lv);
}

// ---- stream-K bookkeeping (the same in every role) -----------------------------------
// Work item i = (tile i / kchunks, chunk i % kchunks); CTA c owns items
// [floor(c W / G), floor((c + 1) W / G)).
__device__ __forceinline__ int64_t item_begin(int64_t W, int G, int c) { return (W * c) / G; }
__device__ __forceinline__ int item_owner(int64_t W, int G, int64_t i) {
    return (int)(((i + 1) * G + W - 1) / W) - 1;
}


// The weight row of tile row j (natural order, or the paired view's even rows
// first, then the odd rows).
template <bool PAIRED>
__device__ __forceinline__ int tile_row(int j) {
    if constexpr (PAIRED) return j < 64 ? 2 * j : 2 * (j - 64) + 1;
    return j;
}

__device__ __forceinline__ void sts128(uint32_t a, uint32_t x, uint32_t y, uint32_t z, uint32_t w) {
    asm volatile("st.shared.v4.u32 [%0], {%1, %2, %3, %4};" ::"r"(a), "r"(x), "r"(y), "r"(z), "r"(w) : "memory");
}

template <int QT, int NT, bool PAIRED>
__global__ void __launch_bounds__(kTnThreads, 1) gemm_tn_kernel(const __grid_constant__ TArgs a) {
    constexpr int SA = tn_sa(NT), SR = tn_sr(QT, NT, PAIRED);
    constexpr int PITCH = tn_pitch(QT, PAIRED);
    constexpr uint32_t kATile = tn_atile(NT);
    constexpr int MM = 2 * NT;          // MMA M
    constexpr int G = NT / 4;           // tokens per lane quarter
    constexpr uint32_t kDCols = 256;    // accumulator columns (wh | wl)
    extern __shared__ uint8_t smem_raw[];
    // 1024-byte aligned by pointer arithmetic on the shared array (an integer
    // round trip would hide the shared address space: generic loads)
    uint8_t* smem = smem_raw + ((1024u - (smem_u32(smem_raw) & 1023u)) & 1023u);
    uint8_t* sB = smem;                        // [SB] dequantised weight tiles
    uint8_t* sA = sB + kTnSB * kTnBTile;       // [SA] activation stack tiles
    uint8_t* sR = sA + SA * kATile;            // [SR] raw chunks
    uint64_t* full_a = reinterpret_cast<uint64_t*>(sR + SR * kTnRows * PITCH);
    uint64_t* empty_a = full_a + SA;
    uint64_t* full_b = empty_a + SA;
    uint64_t* empty_b = full_b + kTnSB;
    uint64_t* rfull = empty_b + kTnSB;
    uint64_t* rempty = rfull + SR;
    uint64_t* dfull = rempty + SR;   // [2] accumulators written
    uint64_t* dempty = dfull + 2;    // [2] accumulators consumed
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(dempty + 2);

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int Gc = (int)gridDim.x, c = (int)blockIdx.x;
    const int ty = (int)blockIdx.y;  // token tile
    const int64_t w0 = item_begin(a.W, Gc, c), w1 = item_begin(a.W, Gc, c + 1);
    const int kc = a.kchunks;

    if (threadIdx.x == 0) {
        for (int s = 0; s < SA; ++s) {
            mbar_init(&full_a[s], 1);
            mbar_init(&empty_a[s], 1);
        }
        for (int s = 0; s < kTnSB; ++s) {
            mbar_init(&full_b[s], kTnDqThreads);
            mbar_init(&empty_b[s], 1);
        }
        for (int r = 0; r < SR; ++r) {
            mbar_init(&rfull[r], 1);
            mbar_init(&rempty[r], kTnDqThreads);
        }
        for (int t = 0; t < 2; ++t) {
            mbar_init(&dfull[t], 1);
            mbar_init(&dempty[t], 4);
        }
        fence_mbar_init();
        prefetch_tmap(&a.tmap_x);
        prefetch_tmap(&a.tmap_w);
    }
    if (warp == 1) {
        tmem_alloc(tmem_slot, 512);
        tmem_relinquish();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;
    pdl_launch_dependents();
    auto steps_of = [&](int64_t item) {  // K steps of a work item (the last chunk of a row may be short)
        const int ch = (int)(item % kc);
        return min(kTnStepsPerChunk, a.ksteps - ch * kTnStepsPerChunk);
    };

    if (warp == 0) {
        // ---------------------- activation stack (A operand) TMA producer -------------------
        if (lane == 0) {
            pdl_wait();  // the stacks are written by the activation-prep launch
            int i = 0;
            bool ok = true;
            for (int64_t it = w0; it < w1 && ok; ++it) {
                const int ch = (int)(it % kc), nk = steps_of(it);
                for (int kk = 0; kk < nk; ++kk, ++i) {
                    const int s = i % SA;
                    if (i >= SA && !mbar_wait_bounded(&empty_a[s], ((i / SA) - 1) & 1, a.err)) {
                        ok = false;
                        break;
                    }
                    mbar_arrive_expect_tx(&full_a[s], kATile);
                    tma_load_2d(sA + s * kATile, &a.tmap_x, (ch * kTnStepsPerChunk + kk) * kTnBK, ty * MM, &full_a[s]);
                }
            }
            for (int q = (i > SA ? i - SA : 0); q < i; ++q) mbar_wait_bounded(&full_a[q % SA], (q / SA) & 1, nullptr);
        }
    } else if (warp == 14) {
        // ------------------------- raw weight chunk producer ----------------------------
        if (lane == 0) {
            constexpr int BB = block_bytes(QT);
            const int64_t nitems = w1 - w0;
            auto issue_raw = [&](int64_t r) {
                const int64_t it = w0 + r;
                const int sr = (int)(r % SR);
                const int n0 = (int)(it / kc) * kTnRows;
                const int cb = (int)(it % kc) * 8 * BB;  // byte offset of the chunk in a row
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
            int64_t r = 0;
            // immutable weights: the first chunks may load before the dependency wait
            if (a.weights_immutable)
                for (; r < SR && r < nitems; ++r) issue_raw(r);
            pdl_wait();
            for (; r < nitems; ++r) {
                if (r >= SR && !mbar_wait_bounded(&rempty[r % SR], (int)(((r / SR) - 1) & 1), a.err)) break;
                issue_raw(r);
            }
            for (int64_t q = (r > SR ? r - SR : 0); q < r; ++q)
                mbar_wait_bounded(&rfull[q % SR], (int)((q / SR) & 1), nullptr);
        }
    } else if (warp == 1) {
        // ------------------------------- MMA issuer -----------------------------------
        if (lane == 0) {
            pdl_wait();
            constexpr uint32_t idesc = gemm_idesc((int)kDCols, MM);
            int i = 0, g = 0;  // steps, segments
            bool ok = true;
            for (int64_t it = w0; it < w1 && ok; ++g) {
                const int64_t tile = it / kc;
                const int64_t seg_end = min(w1, (tile + 1) * kc);
                const int buf = g & 1;
                const uint32_t dcol = tmem + (uint32_t)(buf * kDCols);
                if (g >= 2 && !mbar_wait_bounded(&dempty[buf], ((g >> 1) - 1) & 1, a.err)) break;
                tc_fence_after();
                bool first = true;
                for (; it < seg_end && ok; ++it) {
                    const int nk = steps_of(it);
                    for (int kk = 0; kk < nk; ++kk, ++i) {
                        const int sa = i % SA, sb = i % kTnSB;
                        if (!mbar_wait_bounded(&full_a[sa], (i / SA) & 1, a.err) ||
                            !mbar_wait_bounded(&full_b[sb], (i / kTnSB) & 1, a.err)) {
                            ok = false;
                            break;
                        }
                        tc_fence_after();
                        const uint64_t ad = sw128_desc(smem_u32(sA + sa * kATile));
                        const uint64_t bd = sw128_desc(smem_u32(sB + sb * kTnBTile));
#pragma unroll
                        for (int k = 0; k < kTnBK / 16; ++k) {  // 32-byte steps inside the swizzle atom
                            mma_f16_ss(dcol, ad + 2 * k, bd + 2 * k, idesc, first ? 0u : 1u);
                            first = false;
                        }
                        // both stages are free once these MMAs have read them
                        mma_commit(&empty_a[sa]);
                        mma_commit(&empty_b[sb]);
                    }
                }
                mma_commit(&dfull[buf]);  // the segment's accumulator is complete
            }
        }
        __syncwarp();
    } else if (warp <= 9) {
        // ----------------------- dequantisers (warps 2-9) -------------------------------
        const int d = threadIdx.x - 64;
        const int j = d & (kTnRows - 1);       // tile row
        const int h = d >> 7;                  // which of a step's two blocks (warp-uniform)
        const bool skew = PAIRED && j >= 64;   // warp-uniform
        const int r7 = j & 7;
        const uint32_t ohi = (uint32_t)((j >> 3) * 1024 + r7 * 128);
        const uint32_t olo = ohi + (uint32_t)(kTnRows / 8) * 1024;  // row 128 + j
        pdl_wait();
        bool ok = true;
        int i = 0;
        int64_t r = 0;
        for (int64_t it = w0; it < w1 && ok; ++it, ++r) {
            const int sr = (int)(r % SR);
            if (!mbar_wait_bounded(&rfull[sr], (int)((r / SR) & 1), a.err)) break;
            const uint32_t row = smem_u32(sR + sr * kTnRows * PITCH + j * PITCH);
            const int ch = (int)(it % kc), nk = steps_of(it);
            for (int kk = 0; kk < nk; ++kk, ++i) {
                const int sb = i % kTnSB;
                if (i >= kTnSB && !mbar_wait_bounded(&empty_b[sb], ((i / kTnSB) - 1) & 1, a.err)) {
                    ok = false;
                    break;
                }
                uint32_t Hv[16], Lv[16];
                if ((ch * kTnStepsPerChunk + kk) * 2 + h >= a.nb) {
                    // a block past the row end (K not a multiple of the chunk): zeros,
                    // whatever bytes the box brought (the next row's, in the paired view)
#pragma unroll
                    for (int e = 0; e < 16; ++e) Hv[e] = Lv[e] = 0u;
                } else {
                    auto deq = [&](auto kkc) {
                        constexpr int KKc = decltype(kkc)::value;
                        if (h == 0) {
                            if (skew) dequant_step_hl<QT, KKc, 0, 8>(row, Hv, Lv);
                            else dequant_step_hl<QT, KKc, 0, 0>(row, Hv, Lv);
                        } else {
                            if (skew) dequant_step_hl<QT, KKc, 1, 8>(row, Hv, Lv);
                            else dequant_step_hl<QT, KKc, 1, 0>(row, Hv, Lv);
                        }
                    };
                    if (kk == 0) deq(std::integral_constant<int, 0>{});
                    else if (kk == 1) deq(std::integral_constant<int, 1>{});
                    else if (kk == 2) deq(std::integral_constant<int, 2>{});
                    else deq(std::integral_constant<int, 3>{});
                }
                const uint32_t tb = smem_u32(sB + sb * kTnBTile);
#pragma unroll
                for (int q4 = 0; q4 < 4; ++q4) {  // 16-byte chunks 4h..4h+3 of the row, swizzled
                    const uint32_t sw = (uint32_t)(((4 * h + q4) ^ r7) << 4);
                    sts128(tb + ohi + sw, Hv[4 * q4], Hv[4 * q4 + 1], Hv[4 * q4 + 2], Hv[4 * q4 + 3]);
                    sts128(tb + olo + sw, Lv[4 * q4], Lv[4 * q4 + 1], Lv[4 * q4 + 2], Lv[4 * q4 + 3]);
                }
                fence_proxy_async_smem();  // generic writes -> visible to the tensor core
                mbar_arrive(&full_b[sb]);
            }
            mbar_arrive(&rempty[sr]);  // the chunk is consumed
        }
    } else {
        // ----------------------------- epilogue (warps 10-13) -----------------------------
        // Lane quarter q holds tokens G q .. G q + G - 1: lanes 0..G-1 their xh rows,
        // lanes G..2G-1 their xl rows (lanes 2G.. unused when NT = 32).
        const int q = warp & 3;
        const bool xh_lane = lane < G;
        const int tok = ty * NT + G * q + (lane & (G - 1));  // token of this lane (valid for lanes < 2G)
        const bool live = xh_lane && tok < a.M;
        const int et = threadIdx.x - 10 * 32;  // 0 .. 127
        const float sc = live ? a.xs[tok] : 0.0f;
        uint32_t* flag = tmem_slot + 1;
        const bool gated = a.gact >= 0;
        pdl_wait();
        int g = 0;
        for (int64_t it = w0; it < w1; ++g) {
            const int64_t tile = it / kc;
            const int64_t seg_end = min(w1, (tile + 1) * kc);
            const int buf = g & 1;
            const int n0 = (int)tile * kTnRows;
            const int cf = item_owner(a.W, Gc, tile * kc), cl = item_owner(a.W, Gc, tile * kc + kc - 1);
            const bool whole = cf == cl;
            it = seg_end;
            if (!mbar_wait_bounded(&dfull[buf], (g >> 1) & 1, a.err)) break;
            tc_fence_after();
            const uint32_t dcol = tmem + ((uint32_t)(q * 32) << 16) + (uint32_t)(buf * kDCols);
            // slot of this CTA's segment: 0 = its first tile, 1 = its last
            const int slot = (tile == w0 / kc) ? 0 : 1;
            const int64_t slab = ((int64_t)ty * Gc + c) * 2;
            float* mine = a.partial + ((slab + slot) * NT) * kTnRows;
            const int tl = tok - ty * NT;  // token within the tile
            bool summer = whole;
            if (!whole) {
#pragma unroll 1
                for (int cb = 0; cb < 4; ++cb) {  // 32 weight rows at a time
                    uint32_t vh[32], vl[32];
                    tmem_ld32(dcol + (uint32_t)(32 * cb), vh);
                    tmem_ld32(dcol + 128u + (uint32_t)(32 * cb), vl);
#pragma unroll
                    for (int e = 0; e < 32; ++e) {
                        float s = __uint_as_float(vh[e]) + __uint_as_float(vl[e]);
                        s += __shfl_xor_sync(0xffffffffu, s, G);  // + the xl row of the same token
                        if (live) mine[(int64_t)tl * kTnRows + 32 * cb + e] = s;
                    }
                }
                __threadfence();
                asm volatile("bar.sync 2, %0;" ::"r"(kTnEpiThreads) : "memory");
                if (et == 0) {
                    unsigned* ctr = a.counters + (int64_t)ty * a.tiles + tile;
                    const unsigned t = atomicAdd(ctr, 1u);
                    const bool last = t == (unsigned)(cl - cf);
                    *flag = last ? 1u : 0u;
                    if (last) *ctr = 0u;  // left zero for the next call
                }
                asm volatile("bar.sync 2, %0;" ::"r"(kTnEpiThreads) : "memory");
                summer = *flag != 0u;
                if (summer) __threadfence();
            }
            if (summer) {
#pragma unroll 1
                for (int cb = 0; cb < 4; ++cb) {
                    float v[32];
                    if (whole) {
                        uint32_t vh[32], vl[32];
                        tmem_ld32(dcol + (uint32_t)(32 * cb), vh);
                        tmem_ld32(dcol + 128u + (uint32_t)(32 * cb), vl);
#pragma unroll
                        for (int e = 0; e < 32; ++e) {
                            float s = __uint_as_float(vh[e]) + __uint_as_float(vl[e]);
                            s += __shfl_xor_sync(0xffffffffu, s, G);
                            v[e] = s;
                        }
                    } else {
                        // the tile's segments in K order: CTAs cf..cl, each its first
                        // (slot 0) or last (slot 1) segment
#pragma unroll
                        for (int e = 0; e < 32; ++e) v[e] = 0.0f;
                        if (live) {
                            for (int cc = cf; cc <= cl; ++cc) {
                                const int sl = (tile == item_begin(a.W, Gc, cc) / kc) ? 0 : 1;
                                const float* p =
                                    a.partial + ((((int64_t)ty * Gc + cc) * 2 + sl) * NT + tl) * kTnRows + 32 * cb;
#pragma unroll
                                for (int e = 0; e < 32; ++e) v[e] = (cc == cf) ? __ldcg(p + e) : v[e] + __ldcg(p + e);
                            }
                        }
                    }
                    if (live) {
                        if (gated) {
                            // weight rows 32 m .. 32 m + 15 are gate rows, the next 16 the
                            // matching up rows: tile row + 16 in natural order, + 8 in the
                            // paired view (both halves of a 32-row group share a parity)
                            constexpr int kUp = PAIRED ? 8 : 16;
                            float* orow = a.gout + (int64_t)tok * a.ghidden;
#pragma unroll
                            for (int e = 0; e < 32; ++e) {
                                const int wrow = n0 + tile_row<PAIRED>(32 * cb + e);
                                if (e + kUp < 32 && (wrow & 31) < 16) {
                                    const int64_t gi = (int64_t)(wrow >> 5) * 16 + (wrow & 31);
                                    if (gi < a.ghidden)
                                        orow[gi] = gated_value(a.gact, v[e] * sc, v[e + (e + kUp < 32 ? kUp : 0)] * sc);
                                }
                            }
                        } else {
                            float* orow = a.y + (int64_t)tok * a.N;
#pragma unroll
                            for (int e = 0; e < 32; ++e) {
                                const int n = n0 + tile_row<PAIRED>(32 * cb + e);
                                if (n < a.N) orow[n] = v[e] * sc;
                            }
                        }
                    }
                }
            }
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(&dempty[buf]);
        }
    }
    __syncthreads();
    if (warp == 1) {
        tc_fence_after();
        tmem_dealloc(tmem, 512);
    }
}

template <int QT, bool PAIRED>
const void* tn_pick_nt(int nt) {
    return nt == 32 ? (const void*)gemm_tn_kernel<QT, 32, PAIRED> : (const void*)gemm_tn_kernel<QT, 64, PAIRED>;
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

int tn_nt(int M) { return M <= 32 ? 32 : 64; }
int tn_ntok(int M) { return (M + tn_nt(M) - 1) / tn_nt(M); }

// Persistent CTAs per token tile: the SMs shared among the token tiles, fewer
// when there are not kTnMinChunks work items each.
int tn_grid(int M, int N, int K) {
    int sms = 148, dev = 0;
    if (cudaGetDevice(&dev) == cudaSuccess) cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    const int per = sms / tn_ntok(M);
    const int64_t tiles = (N + kTnRows - 1) / kTnRows;
    const int64_t kc = ((K / QK) + 7) / 8;
    int64_t g = tiles * kc / kTnMinChunks;
    if (g < 1) g = 1;
    return (int)(g < per ? g : per);
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
    const int nt = tn_nt(M), ntok = tn_ntok(M);
    const size_t grid = (size_t)tn_grid(M, N, K);
    const size_t tiles = (size_t)((N + kTnRows - 1) / kTnRows);
    return al256((size_t)ntok * 2 * nt * K * 2) + al256((size_t)M * 4) + al256((size_t)ntok * grid * 2 * nt * kTnRows * 4) +
           al256((size_t)ntok * tiles * 4);
}

cudaError_t launch_gemm_tn(int qt, const uint8_t* w, const float* x, float* y, int M, int N, int K, void* ws,
                           int* err, cudaStream_t st, bool weights_immutable, const GatedOut& g) {
    const int nt = tn_nt(M), ntok = tn_ntok(M);
    const int grid = tn_grid(M, N, K);
    const int tiles = (N + kTnRows - 1) / kTnRows;
    uint8_t* base = static_cast<uint8_t*>(ws);
    __half* xst = reinterpret_cast<__half*>(base);
    const size_t o1 = al256((size_t)ntok * 2 * nt * K * 2);
    float* xs = reinterpret_cast<float*>(base + o1);
    const size_t o2 = o1 + al256((size_t)M * 4);
    float* partial = reinterpret_cast<float*>(base + o2);
    unsigned* counters =
        reinterpret_cast<unsigned*>(base + o2 + al256((size_t)ntok * grid * 2 * nt * kTnRows * 4));
    {
        // one CTA per token of the tiles: padding tokens get zero rows
        int ntc = nt;
        void* args[] = {(void*)&x, (void*)&M, (void*)&K, (void*)&ntc, (void*)&xst, (void*)&xs};
        cudaLaunchConfig_t cfg = {};
        cfg.gridDim = dim3((unsigned)(ntok * nt));
        cfg.blockDim = dim3(256);
        cfg.stream = st;
        cudaLaunchAttribute attr[1];
        attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
        attr[0].val.programmaticStreamSerializationAllowed = 1;
        cfg.attrs = attr;
        cfg.numAttrs = 1;
        note_launch();
        cudaError_t e = cudaLaunchKernelExC(&cfg, (const void*)gemm_tn_xprep_kernel, args);
        if (e != cudaSuccess) return e;
    }
    const int nb = K / QK;
    const int row_bytes = nb * block_bytes(qt);
    const bool paired = row_bytes % 16 != 0;
    const int pitch = tn_pitch(qt, paired);
    TArgs a;
    cudaError_t e = encode_map_2d(&a.tmap_x, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, xst, (uint64_t)K,
                                  (uint64_t)ntok * 2 * nt, (uint64_t)K * 2, kTnBK, (uint32_t)(2 * nt),
                                  CU_TENSOR_MAP_SWIZZLE_128B);
    if (e == cudaSuccess) {
        if (paired)
            e = encode_map_2d(&a.tmap_w, CU_TENSOR_MAP_DATA_TYPE_UINT32, w, (uint64_t)row_bytes / 2, (uint64_t)N / 2,
                              (uint64_t)row_bytes * 2, (uint32_t)pitch / 4, 64, CU_TENSOR_MAP_SWIZZLE_NONE);
        else
            e = encode_map_2d(&a.tmap_w, CU_TENSOR_MAP_DATA_TYPE_UINT32, w, (uint64_t)row_bytes / 4, (uint64_t)N,
                              (uint64_t)row_bytes, (uint32_t)pitch / 4, kTnRows, CU_TENSOR_MAP_SWIZZLE_NONE);
    }
    if (e != cudaSuccess) return e;
    e = cudaMemsetAsync(counters, 0, (size_t)ntok * tiles * 4, st);  // the tickets start from zero
    if (e != cudaSuccess) return e;
    a.xs = xs;
    a.y = y;
    a.M = M;
    a.N = N;
    a.K = K;
    a.nb = nb;
    a.ksteps = (K + kTnBK - 1) / kTnBK;
    a.kchunks = (nb + 7) / 8;
    a.tiles = tiles;
    a.W = (int64_t)tiles * a.kchunks;
    a.row_bytes = row_bytes;
    a.weights_immutable = weights_immutable ? 1 : 0;
    a.err = err;
    a.partial = partial;
    a.counters = counters;
    a.gact = g.act;
    a.gout = g.out;
    a.ghidden = g.hidden;
    const void* fn = gemm_tn_kernel_for(qt, nt, paired);
    const size_t smem = tn_smem_bytes(qt, nt, paired);
    e = ensure_dynamic_smem(fn, smem);
    if (e != cudaSuccess) return e;
    void* args[] = {(void*)&a};
    return tn_launch_ex(fn, dim3((unsigned)grid, (unsigned)ntok), dim3(kTnThreads), smem, st, args);
}

}  // namespace qmm
