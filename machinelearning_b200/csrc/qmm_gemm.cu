// f16 tensor-core GEMM for sm_100a (prefill and decode batches): tcgen05 with
// TMEM accumulators.
//
// y[M, N] = x[M, K] . W[N, K]^T for f32 activations and GGUF block weights
// (Q4_0 / Q4_1 / Q8_0 rows, raw bytes), M >= kGemmMinRows. Replaces the M > 4
// row-parallel CPU loops of matmul_f32_q4 / _q8 / _q4_1 (reference
// llmserve/llmmodel/kernel/main/src/core/quantize.rs:317-395, 557-630,
// 807-932).
//
// Two launches per call:
//   1. gemm_xprep: each activation row is scaled by a power of two (its max
//      lands in [2^14, 2^15)) and rounded to f16; up to 128 tokens the f16
//      residual of every row is written too, as the rows M .. 2M - 1 of the
//      same token tile (exact activations: D rows m and M + m add).
//   2. gemm_kernel<QT, T, W, H, P>: one CTA per output tile of the token tile
//      (T x 128 rows, or 64 when H: MMA M = 64 for up to 64 stacked rows) by
//      W weight rows (64 .. 224), full K or a K slice:
//        warp 0    TMA producer of the x16 tiles [rows x 64] per K step with
//                  128-byte swizzle (the canonical K-major UMMA layout); the
//                  boxes carry the real rows only, the rest stays zero;
//        last warp TMA producer of raw weight chunks [W rows x 8 blocks]: one
//                  2-D box of the GGUF bytes, or (P: 8-mod-16 row pitches) two
//                  boxes of the paired view [N/2][2 * row_bytes];
//        warp 1    allocates TMEM; one thread issues tcgen05.mma.kind::f16
//                  (M 128 or 64, N W, K 16, both operands read from shared
//                  memory through descriptors) and commits to mbarriers;
//        warps 2.. dequantise: each thread one 32-weight block of one row per
//                  K step (magic-number f16 pairs, one f16 rounding of d*q,
//                  d*(n-8) or d*n+m), written into the swizzled B tile; then
//                  they read the accumulators back with tcgen05.ld into a
//                  staging tile (weight-row order) and write y = acc * row
//                  scale as whole coalesced rows, or the gate/up activation.
//      One dequantised B tile feeds T accumulators: T = 2 for more than 128
//      rows halves the dequantisation per flop. Every wait is bounded (error
//      word on timeout, in-flight copies drained before exit).
//
// Numerics: d*q is rounded to f16 once (unit roundoff 2^-11), products are
// exact and accumulate in f32. Up to 128 tokens the activations are exact
// (hi + residual): ~2e-4 of ||y||; above, they are rounded to f16 too: ~3e-4
// on N(0, 1) activations; both inside the 1e-3 contract (the GEMV paths carry
// activations as f16 hi+lo and exact weights and stay near 1e-5).
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

constexpr int BM = 128;            // tokens per accumulator (MMA M, TMEM lanes)
constexpr int BN = 128;            // weight rows per tile by default (MMA N, TMEM columns); 160 also built
constexpr int BK = 64;             // f16 elements per K step: one 128-byte swizzle row
constexpr int kStepsPerChunk = 4;  // a raw chunk is 8 blocks = 256 elements
// Per weight-tile width W (128 or 160 rows): W / 16 dequantising (then
// epilogue) warps, one (row, block) per thread per K step; 2 + W / 16 + 1 warps
// in all (x16 producer, MMA issuer, dequantisers, raw-chunk producer).
__host__ __device__ constexpr int dq_warps(int W) { return W / 16; }
__host__ __device__ constexpr int dq_threads(int W) { return 2 * W; }
__host__ __device__ constexpr int gemm_threads(int W) { return 64 + dq_threads(W) + 32; }

// Operand rings: the x16 (A) ring is the deeper one -- its TMA loads take
// 1.5-2 us to land under load, and a stage is refilled only once the MMAs
// that read it have completed -- while dequantised weight tiles (B) are ready
// ~0.3 us after their raw chunk is. Sized to fill 227 KB with the raw ring.
__host__ __device__ constexpr int a_stages(int qt, int T, int W = BN) {
    return W > 160 ? (qt == kQ8_0 ? 3 : 4) : (T == 1 ? 6 : (W > BN ? 3 : (qt == kQ8_0 ? 3 : 4)));
}
// Q8_0 at 224 rows: its raw chunks (272-byte rows) leave room for two
// dequantised tiles only.
__host__ __device__ constexpr int b_stages(int qt, int, int W = BN) { return (qt == kQ8_0 && W > 160) ? 2 : 3; }

// Raw chunk row pitch in shared memory (= the TMA box's inner extent): 8
// blocks, padded so consecutive rows sit an odd number of 16-byte units apart
// (conflict-free 16-byte loads by consecutive threads).
__host__ __device__ constexpr int raw_pitch(int qt) { return qt == kQ8_0 ? 272 : (qt == kQ4_0 ? 144 : 176); }
// Row pitches of 8 mod 16 bytes (K = 1152: 648-byte Q4_0 / 1224-byte Q8_0
// rows) are read through a paired view of the weights, [N/2][2 * row_bytes]
// (16-byte pitched): per chunk one box of the even rows and one of the odd
// rows starting 8 bytes early, so no padded copy is needed. The stage holds
// the even rows, then the odd rows (8 bytes of skew each: a wider pitch).
__host__ __device__ constexpr int raw_pitch_p(int qt, bool p) {
    return p ? (qt == kQ8_0 ? 304 : (qt == kQ4_0 ? 176 : 208)) : raw_pitch(qt);
}

struct GArgs {
    CUtensorMap tmap_x;  // x16 [M][K] f16, box [64, 128], 128-byte swizzle
    CUtensorMap tmap_w;  // weights as uint32 [N][row_bytes / 4], box [pitch / 4, 128]
    const float* xs;     // per-row activation scales
    float* y;
    int M, N, K, ksteps, weights_immutable;
    int xrows;           // token rows one x16 box carries (T == 1: rows rounded up to 8; else BM)
    int stack;           // x16 rows [M, 2M) are the f16 residuals of rows [0, M): D rows r and M + r add
    int nb, row_bytes;   // blocks and bytes per weight row
    int* err;
    int ks, cps;         // K slices (blockIdx.z) and raw chunks per slice
    float* partial;      // [ks][M][N] unscaled partial tiles (ks > 1)
    unsigned* counters;  // [tiles] tickets, zero before the launch (ks > 1)
    int gact;        // >= 0: gate/up epilogue (GatedOut), y unused
    float* gout;     // [M][ghidden]
    int64_t ghidden;
    PeerDst peer;    // n > 0: the outputs go to every rank's join buffer instead of y
};

size_t align256(size_t v) { return (v + 255) & ~size_t(255); }

// Half-height token tiles (H: at most 64 tokens, MMA M = 64): x16 stages of
// 8 KB, twice as many of them in the same space. The x16 copies take ~1.5 us
// to land (they queue with the raw chunks' HBM loads) and a stage is refilled
// only when the MMAs that read it complete; twice the copies in flight took
// the 32-token lm_head from 366 to 339 us on B200.
__host__ __device__ constexpr int x_stages(int qt, int T, int W, bool h) { return (h ? 2 : 1) * a_stages(qt, T, W); }
__host__ __device__ constexpr uint32_t x_tile_bytes(bool h) { return (h ? 64u : (uint32_t)BM) * BK * 2; }
__host__ __device__ constexpr size_t gemm_smem_with(int qt, int T, int W, int sr, bool h, bool p = false) {
    return 1024 + (size_t)x_stages(qt, T, W, h) * T * x_tile_bytes(h) + (size_t)b_stages(qt, T, W) * W * BK * 2 +
           (size_t)sr * W * raw_pitch_p(qt, p) +
           (2 * x_stages(qt, T, W, h) + 2 * b_stages(qt, T, W) + 2 * sr + 1) * 8 + 16;
}
// Raw chunk stages: as many as fit (2..6). A chunk is 4 K steps and its TMA
// load takes ~2 us to land under load; the narrower tiles have room to keep
// more of them in flight.
__host__ __device__ constexpr int raw_stages(int qt, int T, int W, bool h = false, bool p = false) {
    int sr = 6;
    while (sr > 2 && gemm_smem_with(qt, T, W, sr, h, p) > 232448) --sr;
    return sr;
}
__host__ __device__ constexpr size_t gemm_smem_bytes(int qt, int T, int W, bool h = false, bool p = false) {
    return gemm_smem_with(qt, T, W, raw_stages(qt, T, W, h, p), h, p);
}
static_assert(gemm_smem_bytes(kQ4_0, 2, 160) <= 232448 && gemm_smem_bytes(kQ4_1, 2, 160) <= 232448 &&
                  gemm_smem_bytes(kQ4_0, 1, 160) <= 232448 && gemm_smem_bytes(kQ4_1, 1, 160) <= 232448 &&
                  gemm_smem_bytes(kQ8_0, 2, BN) <= 232448 && gemm_smem_bytes(kQ4_1, 2, BN) <= 232448 &&
                  gemm_smem_bytes(kQ4_0, 1, 224) <= 232448 && gemm_smem_bytes(kQ4_1, 1, 224) <= 232448 &&
                  gemm_smem_bytes(kQ8_0, 1, 64) <= 232448 && gemm_smem_bytes(kQ8_0, 2, 64) <= 232448 &&
                  gemm_smem_bytes(kQ8_0, 1, 224) <= 232448,
              "a GEMM variant exceeds 227 KB of shared memory");

// Q8_0: 4 int8 -> two f16 pairs d*q (elements in order).
__device__ __forceinline__ void q8_pairs(uint32_t w, __half2 d2, uint32_t& p01, uint32_t& p23) {
    const uint32_t u = w ^ 0x80808080u;
    const __half2 off = __float2half2_rn(1152.0f);
    // halves 0x64XX = 1024 + XX = 1152 + q, exact
    p01 = h2_u32(__hmul2(__hsub2(as_h2(__byte_perm(u, 0x64646464u, 0x4140)), off), d2));
    p23 = h2_u32(__hmul2(__hsub2(as_h2(__byte_perm(u, 0x64646464u, 0x4342)), off), d2));
}
// Q4: the low and high nibbles of bytes (b0, b1) of t = [b0, 0, b1, 0] as
// exact halves 1024 + n.
__device__ __forceinline__ uint32_t lo_nibbles(uint32_t t) { return lop3_and_or(t, 0x000F000Fu, 0x64006400u); }
__device__ __forceinline__ uint32_t hi_nibbles(uint32_t t) { return lop3_and_or(t >> 4, 0x000F000Fu, 0x64006400u); }

template <int QT>
__device__ __forceinline__ uint32_t q4_value(uint32_t h, __half2 d2, __half2 m2) {
    if constexpr (QT == kQ4_0) return h2_u32(__hmul2(__hsub2(as_h2(h), __float2half2_rn(1032.0f)), d2));
    return h2_u32(__hfma2(__hsub2(as_h2(h), __float2half2_rn(1024.0f)), d2, m2));
}

// Payload word i of a block whose payload starts at byte P of the loaded words.
template <int P>
__device__ __forceinline__ uint32_t payload_word(const uint32_t* W, int i) {
    if constexpr (P % 4 == 0) return W[P / 4 + i];
    return __byte_perm(W[P / 4 + i], W[P / 4 + i + 1], 0x5432);
}

// One block of one weight row: the block starts OFF bytes into the row's raw
// chunk (16-byte aligned, in shared memory); its 32 weights become four
// 16-byte chunks of 8 f16 (elements in order) stored at chunk positions
// CB..CB+3 of the row's 128 swizzled bytes at `dst`.
template <int QT, int OFF, int CB>
__device__ __forceinline__ void dequant_block(const uint8_t* row, uint8_t* dst, int r7) {
    constexpr int BB = block_bytes(QT);
    constexpr int U0 = OFF / 16;           // first aligned 16-byte unit
    constexpr int ST = OFF - 16 * U0;      // block start inside the loaded bytes
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
    uint4 c[4];
    if constexpr (QT == kQ8_0) {
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            uint32_t a0, a1, b0, b1;
            q8_pairs(payload_word<ST + 2>(W, 2 * i), d2, a0, a1);
            q8_pairs(payload_word<ST + 2>(W, 2 * i + 1), d2, b0, b1);
            c[i] = make_uint4(a0, a1, b0, b1);  // elements 8i..8i+7
        }
    } else {
        constexpr int NOFF = QT == kQ4_1 ? 4 : 2;
        const __half2 m2 = QT == kQ4_1 ? half2_from_bits(hw >> 16) : __float2half2_rn(0.0f);
        uint32_t lo[8], hi[8];
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            // GGML order: low nibble of byte j is element j, high nibble element j + 16
            const uint32_t p = payload_word<ST + NOFF>(W, i);
            const uint32_t t01 = __byte_perm(p, 0u, 0x4140), t23 = __byte_perm(p, 0u, 0x4342);
            lo[2 * i] = q4_value<QT>(lo_nibbles(t01), d2, m2);
            lo[2 * i + 1] = q4_value<QT>(lo_nibbles(t23), d2, m2);
            hi[2 * i] = q4_value<QT>(hi_nibbles(t01), d2, m2);
            hi[2 * i + 1] = q4_value<QT>(hi_nibbles(t23), d2, m2);
        }
        c[0] = make_uint4(lo[0], lo[1], lo[2], lo[3]);  // elements 0-7
        c[1] = make_uint4(lo[4], lo[5], lo[6], lo[7]);  // 8-15
        c[2] = make_uint4(hi[0], hi[1], hi[2], hi[3]);  // 16-23
        c[3] = make_uint4(hi[4], hi[5], hi[6], hi[7]);  // 24-31
    }
#pragma unroll
    for (int i = 0; i < 4; ++i) *reinterpret_cast<uint4*>(dst + (((CB + i) ^ r7) << 4)) = c[i];
}

// Block BLK (0 or 1) of K step KK of a raw chunk whose row starts SK bytes
// into its shared-memory row (8 for the paired view's odd rows).
template <int QT, int KK, int BLK, int SK = 0>
__device__ __forceinline__ void dequant_kstep(const uint8_t* row, uint8_t* dst, int r7) {
    dequant_block<QT, SK + block_bytes(QT) * (2 * KK + BLK), 4 * BLK>(row, dst, r7);
}
// Zero weights for a block past the row end (the paired view's boxes bring
// the neighbouring row's bytes there, not zero fill).
template <int BLK>
__device__ __forceinline__ void zero_kstep(uint8_t* dst, int r7) {
#pragma unroll
    for (int i = 0; i < 4; ++i) *reinterpret_cast<uint4*>(dst + (((4 * BLK + i) ^ r7) << 4)) = make_uint4(0, 0, 0, 0);
}

// ---- activation prep: x f32 -> x16 f16 with a power-of-two scale per row ---------------
__global__ void gemm_xprep_kernel(const float* __restrict__ x, int M, int K, __half* __restrict__ x16,
                                  float* __restrict__ xs, int stack) {
    pdl_launch_dependents();
    pdl_wait();  // x comes from the preceding work in the stream
    __shared__ float red[32];
    const int m = blockIdx.x;
    const float* row = x + (int64_t)m * K;
    // 16-byte aligned rows: four float4 loads in flight per thread per round
    // (a long row is otherwise one dependent L2 round trip per element:
    // measured 58 us for 32 x 28672)
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
    __half* out = x16 + (int64_t)m * K;
    // stacked: row M + m holds the f16 residual (exact in f32, then rounded:
    // hi + lo carries ~22 significant bits)
    __half* lo = stack ? x16 + (int64_t)(M + m) * K : nullptr;
    if (v4) {
        uint2* o2 = reinterpret_cast<uint2*>(out);  // 4 halves per float4 (rows are 64-byte multiples)
        uint2* l2 = reinterpret_cast<uint2*>(lo);
        for (int k = threadIdx.x; k < n4; k += blockDim.x) {
            const float4 v = r4[k];
            const float a0 = v.x * scale, a1 = v.y * scale, a2 = v.z * scale, a3 = v.w * scale;
            const __half2 h01 = __floats2half2_rn(a0, a1);
            const __half2 h23 = __floats2half2_rn(a2, a3);
            o2[k] = make_uint2(h2_u32(h01), h2_u32(h23));
            if (stack) {
                const float2 f01 = __half22float2(h01), f23 = __half22float2(h23);
                l2[k] = make_uint2(h2_u32(__floats2half2_rn(a0 - f01.x, a1 - f01.y)),
                                   h2_u32(__floats2half2_rn(a2 - f23.x, a3 - f23.y)));
            }
        }
    } else {
        for (int k = threadIdx.x; k < K; k += blockDim.x) {
            const float a0 = row[k] * scale;
            const __half h = __float2half_rn(a0);
            out[k] = h;
            if (stack) lo[k] = __float2half_rn(a0 - __half2float(h));
        }
    }
    if (threadIdx.x == 0) xs[m] = __int_as_float((e + 127) << 23);
}

template <int QT, int T, int W, bool H, bool P>
__global__ void __launch_bounds__(gemm_threads(W), 1) gemm_kernel(const __grid_constant__ GArgs a) {
    static_assert(!H || T == 1, "half-height token tiles come one per CTA");
    static_assert(!P || (T == 1 && W % 64 == 0), "paired view: one token tile, even and odd halves of whole warps");
    constexpr int BMk = H ? 64 : BM;                 // MMA M (token rows of a tile)
    constexpr uint32_t kATile = x_tile_bytes(H);     // x16 stage bytes per token tile
    constexpr int SA = x_stages(QT, T, W, H), SB = b_stages(QT, T, W);
    constexpr int kDqWarps = dq_warps(W), kDqThreads = dq_threads(W);
    constexpr uint32_t kBTile = (uint32_t)W * BK * 2;  // dequantised weight tile bytes
    constexpr uint32_t kTmemCols = T * W <= 128 ? 128 : (T * W <= 256 ? 256 : 512);
    constexpr int PITCH = raw_pitch_p(QT, P);
    constexpr int SR = raw_stages(QT, T, W, H, P);
    extern __shared__ uint8_t smem_raw[];
    // 1024-byte aligned by pointer arithmetic on the shared array (an integer
    // round trip would hide the shared address space: generic loads)
    uint8_t* smem = smem_raw + ((1024u - (smem_u32(smem_raw) & 1023u)) & 1023u);
    uint8_t* sA = smem;                        // [SA][T] x16 tiles
    uint8_t* sB = smem + SA * T * kATile;      // [SB] weight tiles
    uint8_t* sR = sB + SB * kBTile;            // [SR] raw chunks
    uint64_t* full_a = reinterpret_cast<uint64_t*>(sR + SR * W * PITCH);
    uint64_t* empty_a = full_a + SA;
    uint64_t* full_b = empty_a + SA;
    uint64_t* empty_b = full_b + SB;
    uint64_t* rfull = empty_b + SB;
    uint64_t* rempty = rfull + SR;
    uint64_t* acc_full = rempty + SR;
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(acc_full + 1);

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int n0 = blockIdx.x * W, m0 = blockIdx.y * (T * BM);
    // K slice blockIdx.z: raw chunks [c_begin, c_begin + nchunks) of the rows
    const int nchunks_all = (a.ksteps + kStepsPerChunk - 1) / kStepsPerChunk;
    const int c_begin = (int)blockIdx.z * a.cps;
    const int nchunks = max(1, min(nchunks_all - c_begin, a.cps));  // the planner gives every slice a chunk
    const int steps = min(a.ksteps, (c_begin + nchunks) * kStepsPerChunk) - c_begin * kStepsPerChunk;
    // Every CTA starts its K loop at a different raw chunk: CTAs that share a
    // token tile then fetch different x16 tiles at any moment instead of all
    // hitting the same L2 lines (the sum order differs per tile, results stay
    // deterministic).
    const int rot = (int)(blockIdx.x % (unsigned)nchunks);
    auto chunk_of = [&](int ci) { return c_begin + (ci + rot < nchunks ? ci + rot : ci + rot - nchunks); };

    if (threadIdx.x == 0) {
        for (int s = 0; s < SA; ++s) {
            mbar_init(&full_a[s], 1);
            mbar_init(&empty_a[s], 1);
        }
        for (int s = 0; s < SB; ++s) {
            mbar_init(&full_b[s], kDqThreads);
            mbar_init(&empty_b[s], 1);
        }
        for (int r = 0; r < SR; ++r) {
            mbar_init(&rfull[r], 1);
            mbar_init(&rempty[r], kDqThreads);
        }
        mbar_init(acc_full, 1);
        fence_mbar_init();
        prefetch_tmap(&a.tmap_x);
        prefetch_tmap(&a.tmap_w);
    }
    if (warp == 1) {
        tmem_alloc(tmem_slot, kTmemCols);
        tmem_relinquish();
    }
    if (a.xrows < BMk) {
        // Fewer token rows than the MMA is tall (128, or 64 for half-height
        // tiles): the boxes carry the real rows only, and the rows past them
        // stay zero in every stage for the whole launch. Zeroed once here,
        // before any copy lands.
        const uint32_t z0 = (uint32_t)a.xrows * 128u;
        for (int s = 0; s < SA * T; ++s)
            for (uint32_t o = z0 + 16u * threadIdx.x; o < kATile; o += 16u * blockDim.x)
                *reinterpret_cast<uint4*>(sA + (size_t)s * kATile + o) = make_uint4(0, 0, 0, 0);
        fence_proxy_async_smem();  // generic writes -> visible to the tensor core
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;
    pdl_launch_dependents();

    if (warp == 0) {
        // --------------------------- x16 (A) TMA producer ------------------------------
        if (lane == 0) {
            bool ok = true;
            int a_issued = 0;
            pdl_wait();  // x16 is written by the activation-prep launch
            for (int ci = 0; ci < nchunks && ok; ++ci) {
                const int rc = chunk_of(ci);
                const int nk = min(kStepsPerChunk, a.ksteps - rc * kStepsPerChunk);
                for (int kk = 0; kk < nk && ok; ++kk) {
                    const int i = a_issued, s = i % SA;
                    if (i >= SA && !mbar_wait_bounded(&empty_a[s], ((i / SA) - 1) & 1, a.err)) {
                        ok = false;
                        break;
                    }
                    mbar_arrive_expect_tx(&full_a[s], (uint32_t)T * (uint32_t)a.xrows * 128u);
#pragma unroll
                    for (int t = 0; t < T; ++t)
                        tma_load_2d(sA + (s * T + t) * kATile, &a.tmap_x, (rc * kStepsPerChunk + kk) * BK,
                                    m0 + t * BM, &full_a[s]);
                    ++a_issued;
                }
            }
            // every copy this thread started has landed before the CTA can exit
            for (int i = (a_issued > SA ? a_issued - SA : 0); i < a_issued; ++i)
                mbar_wait_bounded(&full_a[i % SA], (i / SA) & 1, nullptr);
        }
    } else if (warp == gemm_threads(W) / 32 - 1) {
        // ------------------------- raw weight chunk producer ----------------------------
        // A thread of its own, so that waiting for a raw slot never holds up
        // the x16 stream.
        if (lane == 0) {
            int r_issued = 0;
            auto issue_raw = [&](int ci) {  // the ci-th chunk of this CTA's sequence
                const int sr = ci % SR;
                const int cb = chunk_of(ci) * 8 * block_bytes(QT);  // byte offset of the chunk in a row
                mbar_arrive_expect_tx(&rfull[sr], (uint32_t)(W * PITCH));
                if constexpr (P) {
                    // even rows 2p at [p][cb]; odd rows 2p + 1 from 8 bytes before
                    // their chunk, [p][row_bytes + cb - 8] (16-byte aligned)
                    tma_load_2d(sR + sr * W * PITCH, &a.tmap_w, cb / 4, n0 / 2, &rfull[sr]);
                    tma_load_2d(sR + sr * W * PITCH + (W / 2) * PITCH, &a.tmap_w, (a.row_bytes + cb - 8) / 4, n0 / 2,
                                &rfull[sr]);
                } else {
                    tma_load_2d(sR + sr * W * PITCH, &a.tmap_w, cb / 4, n0, &rfull[sr]);
                }
            };
            // immutable weights: the first chunks may load before the dependency wait
            if (a.weights_immutable)
                for (; r_issued < SR && r_issued < nchunks; ++r_issued) issue_raw(r_issued);
            pdl_wait();
            for (; r_issued < nchunks; ++r_issued) {
                if (r_issued >= SR && !mbar_wait_bounded(&rempty[r_issued % SR], ((r_issued / SR) - 1) & 1, a.err))
                    break;
                issue_raw(r_issued);
            }
            for (int i = (r_issued > SR ? r_issued - SR : 0); i < r_issued; ++i)
                mbar_wait_bounded(&rfull[i % SR], (i / SR) & 1, nullptr);
        }
    } else if (warp == 1) {
        // ------------------------------- MMA issuer -----------------------------------
        if (lane == 0) {
            pdl_wait();
            for (int i = 0; i < steps; ++i) {  // operand steps in this CTA's chunk order
                const int sa = i % SA, sb = i % SB;
                if (!mbar_wait_bounded(&full_a[sa], (i / SA) & 1, a.err) ||
                    !mbar_wait_bounded(&full_b[sb], (i / SB) & 1, a.err))
                    break;
                tc_fence_after();
                const uint64_t bd = sw128_desc(smem_u32(sB + sb * kBTile));
#pragma unroll
                for (int t = 0; t < T; ++t) {
                    const uint64_t ad = sw128_desc(smem_u32(sA + (sa * T + t) * kATile));
#pragma unroll
                    for (int k = 0; k < BK / 16; ++k)  // 32-byte steps inside the swizzle atom
                        mma_f16_ss(tmem + t * W, ad + 2 * k, bd + 2 * k, gemm_idesc(W, BMk), (i | k) != 0 ? 1u : 0u);
                }
                // both stages are free once these MMAs have read them
                mma_commit(&empty_a[sa]);
                mma_commit(&empty_b[sb]);
            }
            mma_commit(acc_full);  // arrives when every MMA above has completed
        }
        __syncwarp();
    } else {
        // --------------------- dequantisers, then the epilogue (warps 2-9) ----------------
        const int d = threadIdx.x - 64;
        const int row = d % W;  // weight row inside the tile
        const int blk = d / W;  // which block of the K step (warp-uniform: W is a multiple of 32)
        const int r7 = row & 7;
        pdl_wait();
        bool ok = true;
        // paired view: tile rows [W/2, W) are the odd weight rows, 8 bytes
        // into their shared rows (warp-uniform: W/2 is a multiple of 32)
        const bool skew = P && row >= W / 2;
        auto step = [&](int i, int sr, int chunk, auto kk) {  // operand step i, K step KK of raw stage sr
            constexpr int KK = decltype(kk)::value;
            const int s = i % SB;
            if (i >= SB && !mbar_wait_bounded(&empty_b[s], ((i / SB) - 1) & 1, a.err)) return false;
            const uint8_t* rrow = sR + sr * W * PITCH + row * PITCH;
            uint8_t* dst = sB + s * kBTile + (row >> 3) * 1024 + r7 * 128;
            if (P && chunk * 8 + 2 * KK + blk >= a.nb) {
                if (blk == 0) zero_kstep<0>(dst, r7);
                else zero_kstep<1>(dst, r7);
            } else if (skew) {
                if (blk == 0) dequant_kstep<QT, KK, 0, 8>(rrow, dst, r7);
                else dequant_kstep<QT, KK, 1, 8>(rrow, dst, r7);
            } else {
                if (blk == 0) dequant_kstep<QT, KK, 0>(rrow, dst, r7);
                else dequant_kstep<QT, KK, 1>(rrow, dst, r7);
            }
            fence_proxy_async_smem();  // generic writes -> visible to the tensor core
            mbar_arrive(&full_b[s]);
            return true;
        };
        int i = 0;  // operand steps done
        for (int ci = 0; ci < nchunks && ok; ++ci) {
            const int sr = ci % SR;
            if (!mbar_wait_bounded(&rfull[sr], (ci / SR) & 1, a.err)) break;
            const int chunk = chunk_of(ci);
            const int nk = min(kStepsPerChunk, a.ksteps - chunk * kStepsPerChunk);
            ok = step(i, sr, chunk, std::integral_constant<int, 0>{});
            if (ok && nk > 1) ok = step(i + 1, sr, chunk, std::integral_constant<int, 1>{});
            if (ok && nk > 2) ok = step(i + 2, sr, chunk, std::integral_constant<int, 2>{});
            if (ok && nk > 3) ok = step(i + 3, sr, chunk, std::integral_constant<int, 3>{});
            i += nk;
            mbar_arrive(&rempty[sr]);  // the chunk is consumed
        }
        // Epilogue: accumulators -> a padded staging tile in the (now idle)
        // operand rings -> whole output rows, 512 coalesced bytes per warp store.
        const bool acc_ok = mbar_wait_bounded(acc_full, 0, a.err);
        tc_fence_after();
        const int q = warp & 3;  // this warp's TMEM lane quarter
        // the warps of a quarter (2 or 3) split its 32-column blocks
        const int qfirst = 2 + ((q - 2) & 3);
        const int jq = (warp - qfirst) >> 2;
        const int nq = (2 + kDqWarps - qfirst + 3) >> 2;
        constexpr int YP = W + 4;  // staging pitch in floats: 16-byte stores conflict free
        float* ys = reinterpret_cast<float*>(sA);
#pragma unroll
        for (int t = 0; t < T; ++t) {
            // token row inside the tile; an M = 64 accumulator holds row r in
            // TMEM lane 32 (r / 16) + r % 16: the first 16 lanes of each quarter
            const int r = H ? q * 16 + (lane & 15) : t * BM + q * 32 + lane;
            const bool holds = !H || lane < 16;
#pragma unroll 1
            for (int cb = jq; cb < W / 32; cb += nq) {
                uint32_t v[32];
                tmem_ld32(tmem + ((uint32_t)(q * 32) << 16) + (uint32_t)(t * W + cb * 32), v);
                float4* dstp = reinterpret_cast<float4*>(ys + r * YP + cb * 32);
                if (holds && !P) {
#pragma unroll
                    for (int j = 0; j < 8; ++j)
                        dstp[j] = make_float4(__uint_as_float(v[4 * j]), __uint_as_float(v[4 * j + 1]),
                                              __uint_as_float(v[4 * j + 2]), __uint_as_float(v[4 * j + 3]));
                } else if (holds) {
                    // paired view: accumulator column c is weight row 2c (c < W/2)
                    // or 2 (c - W/2) + 1; staged in weight-row order
                    const int c0 = cb * 32;  // all 32 columns in one half (W/2 % 32 == 0)
                    const int base = c0 < W / 2 ? 2 * c0 : 2 * (c0 - W / 2) + 1;
#pragma unroll
                    for (int j = 0; j < 32; ++j) ys[r * YP + base + 2 * j] = __uint_as_float(v[j]);
                }
            }
        }
        tc_fence_before();
        asm volatile("bar.sync 1, %0;" ::"r"(kDqThreads) : "memory");  // the staging tile is complete
        if (a.stack) {
            // stacked activations: token m's products with its hi row (r = m)
            // and its lo row (r = M + m) add
            const int w4 = W / 4;
            for (int idx = threadIdx.x - 64; idx < a.M * w4; idx += kDqThreads) {
                const int r = idx / w4, c4 = idx - r * w4;
                float4* ph = reinterpret_cast<float4*>(ys + r * YP) + c4;
                const float4 l = *(reinterpret_cast<const float4*>(ys + (r + a.M) * YP) + c4);
                const float4 h = *ph;
                *ph = make_float4(h.x + l.x, h.y + l.y, h.z + l.z, h.w + l.w);
            }
            asm volatile("bar.sync 1, %0;" ::"r"(kDqThreads) : "memory");
        }
        bool store = acc_ok;
        if (a.ks > 1) {
            // K split: this slice's unscaled tile to the workspace; the last slice
            // of the tile to arrive rebuilds the staging tile as the sum of all
            // slices in slice order, then stores it like an unsplit tile
            const int et = threadIdx.x - 64;  // 0 .. kDqThreads - 1
            float* mine = a.partial + (int64_t)blockIdx.z * a.M * a.N;
            for (int c4 = lane; c4 < W / 4; c4 += 32)
                for (int r = warp - 2; r < T * BMk; r += kDqWarps) {
                    const int m = m0 + r, n = n0 + 4 * c4;
                    if (m >= a.M) break;
                    const float4 v = *reinterpret_cast<const float4*>(ys + r * YP + 4 * c4);
                    float* pr = mine + (int64_t)m * a.N + n;
#pragma unroll
                    for (int e = 0; e < 4; ++e)
                        if (n + e < a.N) pr[e] = (&v.x)[e];
                }
            __threadfence();
            asm volatile("bar.sync 1, %0;" ::"r"(kDqThreads) : "memory");
            uint32_t* flag = tmem_slot + 1;
            const unsigned tile = blockIdx.y * gridDim.x + blockIdx.x;
            if (et == 0) {
                const unsigned t = atomicAdd(&a.counters[tile], 1u);
                *flag = (t == (unsigned)(a.ks - 1)) ? 1u : 0u;
                if (t == (unsigned)(a.ks - 1)) a.counters[tile] = 0u;  // left zero for the next call
            }
            asm volatile("bar.sync 1, %0;" ::"r"(kDqThreads) : "memory");
            store = store && *flag != 0u;
            if (store) {
                __threadfence();
                for (int c4 = lane; c4 < W / 4; c4 += 32)
                    for (int r = warp - 2; r < T * BMk; r += kDqWarps) {
                        const int m = m0 + r, n = n0 + 4 * c4;
                        if (m >= a.M) break;
                        float acc[4] = {0.0f, 0.0f, 0.0f, 0.0f};
                        for (int q = 0; q < a.ks; ++q) {
                            const float* pq = a.partial + ((int64_t)q * a.M + m) * a.N + n;
#pragma unroll
                            for (int e = 0; e < 4; ++e)
                                if (n + e < a.N) acc[e] += __ldcg(pq + e);
                        }
                        *reinterpret_cast<float4*>(ys + r * YP + 4 * c4) = make_float4(acc[0], acc[1], acc[2], acc[3]);
                    }
            }
            asm volatile("bar.sync 1, %0;" ::"r"(kDqThreads) : "memory");
        }
        if (a.gact >= 0) {
            // gate/up weight: tile columns [32j, 32j + 16) are gate rows
            // n0 / 2 + 16j + [0, 16), the next 16 columns the matching up rows;
            // index li = lane (+32) produces four consecutive outputs
            const bool gvec = ((reinterpret_cast<uintptr_t>(a.gout) & 15) == 0) && (a.ghidden % 4 == 0);
            for (int li = lane; li < W / 8; li += 32)
            for (int r = warp - 2; r < T * BMk && store; r += kDqWarps) {
                const int c = 32 * (li >> 2) + 4 * (li & 3);
                const int64_t i0 = (int64_t)(n0 / 2) + 16 * (li >> 2) + 4 * (li & 3);
                const int m = m0 + r;
                if (m >= a.M) break;
                const float sc = a.xs[m];
                const float4 gv = *reinterpret_cast<const float4*>(ys + r * YP + c);
                const float4 uv = *reinterpret_cast<const float4*>(ys + r * YP + c + 16);
                const float o0 = gated_value(a.gact, gv.x * sc, uv.x * sc);
                const float o1 = gated_value(a.gact, gv.y * sc, uv.y * sc);
                const float o2 = gated_value(a.gact, gv.z * sc, uv.z * sc);
                const float o3 = gated_value(a.gact, gv.w * sc, uv.w * sc);
                float* orow = a.gout + (int64_t)m * a.ghidden + i0;
                if (gvec && i0 + 3 < a.ghidden) {
                    *reinterpret_cast<float4*>(orow) = make_float4(o0, o1, o2, o3);
                } else {
                    if (i0 < a.ghidden) orow[0] = o0;
                    if (i0 + 1 < a.ghidden) orow[1] = o1;
                    if (i0 + 2 < a.ghidden) orow[2] = o2;
                    if (i0 + 3 < a.ghidden) orow[3] = o3;
                }
            }
        }
        const bool vec = ((reinterpret_cast<uintptr_t>(a.y) & 15) == 0) && (a.N % 4 == 0);
        // tensor-parallel join: the tile goes to the same place in every
        // rank's buffer (peer memory over NVLink) instead of y; the launcher
        // offers it only for 16-byte aligned destinations and rows
        const int nout = a.peer.n > 0 ? a.peer.n : 1;
        const int64_t boff = a.peer.n > 0 ? peer_buffer_offset(a.peer) : 0;
        for (int c4 = lane; c4 < W / 4; c4 += 32)
        for (int r = warp - 2; r < T * BMk && store && a.gact < 0; r += kDqWarps) {
            const int n = n0 + 4 * c4;
            const int m = m0 + r;
            if (m >= a.M) break;  // rows are in increasing order
            const float sc = a.xs[m];
            const float4 v = *reinterpret_cast<const float4*>(ys + r * YP + 4 * c4);
            const float4 o = make_float4(v.x * sc, v.y * sc, v.z * sc, v.w * sc);
            for (int q = 0; q < nout; ++q) {
                float* yr = a.peer.n > 0 ? a.peer.dst[q] + boff + (int64_t)m * a.peer.ld + n
                                         : a.y + (int64_t)m * a.N + n;
                if ((vec || a.peer.n > 0) && n + 3 < a.N) {
                    *reinterpret_cast<float4*>(yr) = o;
                } else {
                    if (n < a.N) yr[0] = o.x;
                    if (n + 1 < a.N) yr[1] = o.y;
                    if (n + 2 < a.N) yr[2] = o.z;
                    if (n + 3 < a.N) yr[3] = o.w;
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

template <int QT, bool H>
const void* pick_w(int T, int W, bool p) {
    if constexpr (H) {
        if (p) return W == 64 ? (const void*)gemm_kernel<QT, 1, 64, true, true> : (const void*)gemm_kernel<QT, 1, BN, true, true>;
        if (W == 64) return (const void*)gemm_kernel<QT, 1, 64, true, false>;
        if (W == 224) return (const void*)gemm_kernel<QT, 1, 224, true, false>;
        if constexpr (QT != kQ8_0) {
            if (W == 160) return (const void*)gemm_kernel<QT, 1, 160, true, false>;
        }
        return (const void*)gemm_kernel<QT, 1, BN, true, false>;
    } else {
        if (p) return W == 64 ? (const void*)gemm_kernel<QT, 1, 64, false, true> : (const void*)gemm_kernel<QT, 1, BN, false, true>;
        if (W == 64)
            return T == 1 ? (const void*)gemm_kernel<QT, 1, 64, false, false> : (const void*)gemm_kernel<QT, 2, 64, false, false>;
        if (W == 224) return (const void*)gemm_kernel<QT, 1, 224, false, false>;
        if constexpr (QT != kQ8_0) {
            if (W == 160)
                return T == 1 ? (const void*)gemm_kernel<QT, 1, 160, false, false>
                              : (const void*)gemm_kernel<QT, 2, 160, false, false>;
        }
        return T == 1 ? (const void*)gemm_kernel<QT, 1, BN, false, false> : (const void*)gemm_kernel<QT, 2, BN, false, false>;
    }
}
const void* gemm_kernel_for(int qt, int T, int W, bool h, bool p) {
    if (qt == kQ8_0) return h ? pick_w<kQ8_0, true>(T, W, p) : pick_w<kQ8_0, false>(T, W, p);
    if (qt == kQ4_0) return h ? pick_w<kQ4_0, true>(T, W, p) : pick_w<kQ4_0, false>(T, W, p);
    return h ? pick_w<kQ4_1, true>(T, W, p) : pick_w<kQ4_1, false>(T, W, p);
}

// Weight-tile widths a call may use: 64, 128, 160 and (one token tile) 224
// rows for Q4_0 / Q4_1; 64, 128 and (one token tile, shallower rings) 224 for
// Q8_0 (its raw chunks are twice as wide).
// The paired view (8-mod-16 row pitches) takes one token tile and 64 or 128
// rows (its halves must be whole warps of dequantisers).
bool gemm_width_ok(int qt, int T, int W, bool paired = false) {
    if (paired) return T == 1 && (W == 64 || W == BN);
    if (W == 64 || W == BN || (W == 224 && T == 1)) return true;
    return qt != kQ8_0 && W == 160;
}

cudaError_t launch_ex(const void* fn, dim3 grid, dim3 block, size_t smem, cudaStream_t st, void** args) {
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

}  // namespace

namespace {

// Decode batches (M <= 128) carry their activations exactly: f16 hi rows and
// f16 residual rows stacked in one token tile (2M MMA rows: the half-height
// tile up to 32 tokens, one or two full tiles up to 128), so only the weights'
// f16 rounding of d*q remains (~2e-4 norm-wise instead of ~3e-4). Larger M
// (prefill, tensor-bound) rounds the activations once.
int x_rows(int M) { return M <= 128 ? 2 * M : M; }
bool paired_pitch(int qt, int K) { return ((int64_t)(K / QK) * block_bytes(qt)) % 16 == 8; }
// Shapes the GEMM below can run: 2-D TMA boxes of the raw rows need a row
// pitch that is a multiple of 16 bytes, or 8 mod 16 through the paired view
// (N even, one token tile: up to 64 tokens).
bool single_shape_ok(int qt, int M, int N, int K) {
    if (M < kGemmMinRows || N < 1 || K < QK || K % QK) return false;
    const int bb = block_bytes(qt);
    if (!bb) return false;
    const int64_t rb = (int64_t)(K / QK) * bb;
    if (rb % 16 == 0) return true;
    return rb % 16 == 8 && N % 2 == 0 && x_rows(M) <= BM;
}
// The decode-batch GEMM (qmm_gemm_tn.cu, exact operand split) takes the decode
// batches this GEMM cannot: 8-mod-16 pitches with odd N or 65..128 tokens.
bool route_tn(int qt, int M, int N, int K) {
    if (!gemm_tn_supported(qt, false, M, N, K)) return false;
    return M > kGemmSingleMaxRows || !single_shape_ok(qt, M, N, K);
}
}  // namespace

bool gemm_supported(int qt, bool native, int M, int N, int K) {
    if (native) return gemm_i8_supported(qt, M, N, K);
    return route_tn(qt, M, N, K) || single_shape_ok(qt, M, N, K);
}

namespace {
// Launch shape of a call: token tiles per CTA, weight-tile width, K slices and
// raw chunks per slice. The fewest rounds of CTAs (waves on the SMs) times the
// K steps a CTA runs times the time per K step, which depends little on the
// width (measured on B200: ~0.5 us per K step for W = 64..224 at 32 tokens).
// Config 3: 138 CTAs of 160 rows (one wave) instead of 172 of 128: 95 ->
// 52 us; Llama gate at M = 32: 128 CTAs of 224 rows instead of 224 of 128;
// Llama down at M = 32 (448 K steps): 37 tiles of 224 rows x 4 K slices.
struct GemmPlan {
    int T, W, ks, cps;
};
GemmPlan gemm_plan(int qt, int M, int N, int K, bool paired = false) {
    GemmPlan p{M > BM ? 2 : 1, BN, 1, 0};
    int sms = 148, dev = 0;
    if (cudaGetDevice(&dev) == cudaSuccess) cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    const int ksteps = (K + BK - 1) / BK;
    const int nch = (ksteps + kStepsPerChunk - 1) / kStepsPerChunk;
    p.cps = nch;
    const long gy = (M + p.T * BM - 1) / (p.T * BM);
    double best = -1.0;
    for (const int w : {64, 128, 160, 224}) {
        if (!gemm_width_ok(qt, p.T, w, paired)) continue;
        for (int ks = 1; ks <= 4; ks *= 2) {
            const int cps = (nch + ks - 1) / ks;
            if ((nch + cps - 1) / cps != ks) continue;  // every slice gets a chunk
            const long rounds = ((N + w - 1) / w * gy * ks + sms - 1) / sms;
            const int steps = min(ksteps, cps * kStepsPerChunk);
            // a K split also writes and re-reads its partial tiles: measured on
            // B200, the Llama gate/up weight at 32 tokens ran 198 us split in
            // four (7 rounds of 32 steps) against ~144 us unsplit (2 rounds of 128)
            const double cost = (double)rounds * steps * (300 + w) * (ks > 1 ? 1.15 : 1.0);
            if (best < 0.0 || cost < best) {
                best = cost;
                p.W = w;
                p.ks = ks;
                p.cps = cps;
            }
        }
    }
    return p;
}
size_t x16_bytes(int M, int K) { return align256((size_t)M * K * 2) + align256((size_t)M * 4); }
}  // namespace



size_t gemm_workspace_bytes(int M, int N, int K, int qt, bool native) {
    if (native) return gemm_i8_workspace_bytes(M, N, K, qt);
    if (route_tn(qt, M, N, K)) return gemm_tn_workspace_bytes(M, N, K, qt);
    const int R = x_rows(M);
    const GemmPlan p = gemm_plan(qt, R, N, K, paired_pitch(qt, K));
    size_t b = x16_bytes(R, K);
    if (p.ks > 1) {
        const long tiles = (long)((N + p.W - 1) / p.W) * ((R + p.T * BM - 1) / (p.T * BM));
        b += align256((size_t)p.ks * M * N * 4) + align256((size_t)tiles * 4);
    }
    return b;
}

cudaError_t launch_gemm(int qt, const uint8_t* w, const float* x, float* y, int M, int N, int K, void* ws, int* err,
                        cudaStream_t st, bool weights_immutable, const GatedOut& g, bool native) {
    if (native) return launch_gemm_i8(qt, w, x, y, M, N, K, ws, err, st, weights_immutable);
    if (route_tn(qt, M, N, K))
        return launch_gemm_tn(qt, w, x, y, M, N, K, ws, err, st, weights_immutable, g);
    const int R = x_rows(M);  // x16 rows: hi rows, then (M <= 128) the residual rows
    int stack = R != M ? 1 : 0;
    __half* x16 = static_cast<__half*>(ws);
    float* xs = reinterpret_cast<float*>(static_cast<uint8_t*>(ws) + align256((size_t)R * K * 2));
    {
        void* args[] = {(void*)&x, (void*)&M, (void*)&K, (void*)&x16, (void*)&xs, (void*)&stack};
        cudaError_t e = launch_ex((const void*)gemm_xprep_kernel, dim3(M), dim3(256), 0, st, args);
        if (e != cudaSuccess) return e;
    }
    GArgs a;
    const int row_bytes = (K / QK) * block_bytes(qt);
    const bool paired = paired_pitch(qt, K);
    const GemmPlan gp = gemm_plan(qt, R, N, K, paired);
    // one token tile of fewer than 128 rows: boxes of the real rows only (the
    // kernel keeps the rest of each stage zero); out-of-range boxes would move
    // 128 rows of zero fill per K step
    const bool half = gp.T == 1 && R <= 64;  // MMA M = 64 token tiles
    a.xrows = gp.T == 1 && R < BM ? (R + 7) / 8 * 8 : BM;
    a.stack = stack;
    cudaError_t e = encode_map_2d(&a.tmap_x, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, x16, (uint64_t)K, (uint64_t)R,
                                  (uint64_t)K * 2, BK, (uint32_t)a.xrows, CU_TENSOR_MAP_SWIZZLE_128B);
    if (e != cudaSuccess) return e;
    const int T = gp.T, W = gp.W;
    const long tiles = (long)((N + W - 1) / W) * ((R + T * BM - 1) / (T * BM));
    a.ks = gp.ks;
    a.cps = gp.cps;
    a.partial = nullptr;
    a.counters = nullptr;
    if (gp.ks > 1) {
        uint8_t* b = static_cast<uint8_t*>(ws) + x16_bytes(R, K);
        a.partial = reinterpret_cast<float*>(b);
        a.counters = reinterpret_cast<unsigned*>(b + align256((size_t)gp.ks * M * N * 4));
        e = cudaMemsetAsync(a.counters, 0, (size_t)tiles * 4, st);  // the tickets start from zero
        if (e != cudaSuccess) return e;
    }
    if (paired)  // [N/2][2 * row_bytes]: rows 2p and 2p + 1 side by side, 16-byte pitched
        e = encode_map_2d(&a.tmap_w, CU_TENSOR_MAP_DATA_TYPE_UINT32, w, (uint64_t)row_bytes / 2, (uint64_t)N / 2,
                          (uint64_t)row_bytes * 2, (uint32_t)raw_pitch_p(qt, true) / 4, (uint32_t)W / 2,
                          CU_TENSOR_MAP_SWIZZLE_NONE);
    else
        e = encode_map_2d(&a.tmap_w, CU_TENSOR_MAP_DATA_TYPE_UINT32, w, (uint64_t)row_bytes / 4, (uint64_t)N,
                          (uint64_t)row_bytes, (uint32_t)raw_pitch(qt) / 4, (uint32_t)W, CU_TENSOR_MAP_SWIZZLE_NONE);
    if (e != cudaSuccess) return e;
    a.xs = xs;
    a.y = y;
    a.M = M;
    a.N = N;
    a.K = K;
    a.ksteps = (K + BK - 1) / BK;
    a.weights_immutable = weights_immutable ? 1 : 0;
    a.err = err;
    a.gact = g.act;
    a.gout = g.out;
    a.ghidden = g.hidden;
    a.nb = K / QK;
    a.row_bytes = row_bytes;
    {
        // a join written from the epilogue: float4 stores need 16-byte aligned
        // destinations and rows
        const PeerOut* po = peer_out();
        bool ok = g.act < 0 && po && N % 4 == 0 && po->ld % 4 == 0;
        for (int r = 0; ok && r < po->n; ++r) ok = (reinterpret_cast<uintptr_t>(po->dst[r]) & 15) == 0;
        take_peer_out(a.peer, ok);
    }
    const void* fn = gemm_kernel_for(qt, T, W, half, paired);
    const size_t smem = gemm_smem_bytes(qt, T, W, half, paired);
    e = ensure_dynamic_smem(fn, smem);
    if (e != cudaSuccess) return e;
    void* args[] = {(void*)&a};
    return launch_ex(fn, dim3((N + W - 1) / W, (R + T * BM - 1) / (T * BM), gp.ks), dim3(gemm_threads(W)), smem,
                     st, args);
}

}  // namespace qmm
