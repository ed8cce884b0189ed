// Integer tensor-core GEMM for the Q8_0-activation ("native") modes, sm_100a.
//
// y[M, N] for matmul_f32_q8_v2 / matmul_f32_q4_native / matmul_f32_q4_1_native
// (reference llmserve/llmmodel/kernel/main/src/core/quantize.rs:429-530,
// 646-772, 938-1070) when M >= kGemmMinRows: every token row is quantised to
// Q8_0 by the reference's own quantiser (quantize_q8_0 for Q8_0 weights,
// quantize_row_q8_0 for Q4 weights), every 32-element block dot is an exact
// integer from tcgen05.mma.kind::i8, and each output is the reference's float
// sequence over the blocks in order,
//     Q8_0 / Q4_0:  dot += ((float)int_dot * xs[b]) * ws[b]
//     Q4_1:         dot += xs[b] * (d[b] * (float)unsigned_dot + m[b] * (float)qsum[b])
// so the results are bit-identical to the reference's (no K split: one
// accumulator per output, blocks in order).
//
// Layout: weights on the MMA's M side (128 rows per CTA tile, one TMEM lane
// each), tokens on its N side (NT = 32 or 64 per CTA). A K step is 4 blocks
// (128 bytes of s8 / u8 per row: one 128-byte swizzle row); each block is one
// MMA (K = 32) into its own TMEM columns, so its int32 dot can be scaled on its
// own. Two TMEM buffers of 4 x NT columns let the MMAs of step i + 1 run while
// the epilogue warps consume step i.
//   warp 0     TMA: the step's xq tile [NT tokens x 128 B] (128-byte swizzle) and
//              the blocks' activation scales / corrections [4][NT];
//   warp 14    TMA: raw weight chunks (8 blocks x 128 rows; the paired-row view
//              for 8-mod-16 row pitches, as in the decode-batch GEMM);
//   warp 1     TMEM allocation; one thread issues the 4 MMAs of a step
//              (A = weights, u8 for Q4 nibbles or s8 for Q8_0; B = s8
//              activations; D = s32) and commits;
//   warps 2-5  unpack one weight row per thread per step into the swizzled A
//              tile (Q8_0: the int8 bytes as they are; Q4: nibbles as u8 0..15,
//              the -8 offset of Q4_0 folded into the conversion below) plus
//              the blocks' scales;
//   warps 6-13 the float epilogue: per block, tcgen05.ld of the int32 dots, an
//              exact int-to-float conversion by the 2^23 + 2^22 magic number
//              (Q4_0: the -8 * qsum correction pre-added by the activation
//              prep), then the reference's multiplies and add, each rounded on
//              its own (no contraction into an fma); two warps per TMEM lane
//              quarter, each half of the tokens. Results are staged in shared
//              memory and stored as whole rows.
// Every wait is bounded (the error word records a timeout; copies in flight
// land before a CTA exits).
#include <cuda.h>

#include <cstring>
#include <type_traits>

#include "qmm_common.cuh"
#include "qmm_kernels.cuh"
#include "qmm_tcgen05.cuh"

namespace qmm {

namespace {

using namespace tc;

constexpr int kI8Rows = 128;        // weight rows per tile (MMA M, TMEM lanes)
constexpr int kI8Blocks = 4;        // blocks per K step (128 bytes per row)
constexpr int kI8StepsPerChunk = 2;  // a raw chunk is 8 blocks
constexpr int kI8SR = 2;            // raw chunk stages
constexpr int kI8SA = 4;            // weight stages
constexpr int kI8SX = 4;            // activation stages
constexpr int kI8Threads = 15 * 32;
constexpr int kI8EpiThreads = 256;  // warps 6-13
constexpr uint32_t kI8ATile = kI8Rows * 128;  // 16 KB

__host__ __device__ constexpr int i8_pitch(int qt, bool paired) {
    return paired ? (qt == kQ8_0 ? 304 : (qt == kQ4_0 ? 176 : 208)) : (qt == kQ8_0 ? 272 : (qt == kQ4_0 ? 144 : 176));
}
// Weight stage: the A tile, then the blocks' scales [4][128] (and Q4_1 mins).
__host__ __device__ constexpr uint32_t i8_astage(int qt) {
    return kI8ATile + kI8Blocks * kI8Rows * 4 * (qt == kQ4_1 ? 2 : 1);
}
// Activation stage: the xq tile [NT][128 B], then xs [4][NT] and xc [4][NT].
__host__ __device__ constexpr uint32_t i8_xstage(int NT) { return (uint32_t)NT * 128 + 2 * kI8Blocks * NT * 4; }
__host__ __device__ constexpr size_t i8_smem_bytes(int qt, int NT, bool paired) {
    return 1024 + (size_t)kI8SA * i8_astage(qt) + (size_t)kI8SX * i8_xstage(NT) +
           (size_t)kI8SR * kI8Rows * i8_pitch(qt, paired) + (2 * kI8SA + 2 * kI8SX + 2 * kI8SR + 4) * 8 + 16;
}
static_assert(i8_smem_bytes(kQ8_0, 64, true) <= 232448 && i8_smem_bytes(kQ4_1, 64, true) <= 232448,
              "an integer GEMM variant exceeds 227 KB");
static_assert(i8_astage(kQ8_0) % 1024 == 0 && i8_astage(kQ4_1) % 1024 == 0 && i8_xstage(32) % 1024 == 0 &&
                  i8_xstage(64) % 1024 == 0,
              "stages must keep the swizzled tiles 1024-byte aligned");

struct IArgs {
    CUtensorMap tmap_xq;  // xq [M][K] u8, box [128, NT], 128-byte swizzle
    CUtensorMap tmap_xs;  // xs [nbp][Mp] f32, box [NT, 4]
    CUtensorMap tmap_xc;  // xc [nbp][Mp] 32-bit, box [NT, 4]
    CUtensorMap tmap_w;   // raw weights (plain or paired view), as in the decode-batch GEMM
    float* y;
    int M, N, K, nb, ksteps, row_bytes, weights_immutable;
    int* err;
};

// Instruction descriptor, kind::i8: s32 accumulator, A unsigned (Q4 nibbles)
// or signed (Q8_0), B signed, both K-major, N >> 3 at bit 17, M >> 4 at bit 24.
__host__ __device__ constexpr uint32_t i8_idesc(bool a_signed, int N) {
    return (2u << 4) | ((a_signed ? 1u : 0u) << 7) | (1u << 10) | ((uint32_t)(N >> 3) << 17) |
           ((uint32_t)(kI8Rows >> 4) << 24);
}

__device__ __forceinline__ void mma_i8_ss(uint32_t tmem_d, uint64_t adesc, uint64_t bdesc, uint32_t idesc) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, 0, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::i8 [%0], %1, %2, %3, p;\n\t}" ::"r"(tmem_d),
        "l"(adesc), "l"(bdesc), "r"(idesc)
        : "memory");
}

template <int N>
__device__ __forceinline__ void tmem_ld_cols(uint32_t taddr, uint32_t (&r)[N]);
template <>
__device__ __forceinline__ void tmem_ld_cols<16>(uint32_t taddr, uint32_t (&r)[16]) {
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
template <>
__device__ __forceinline__ void tmem_ld_cols<32>(uint32_t taddr, uint32_t (&r)[32]) {
    tmem_ld32(taddr, r);
}

// ---- f32 pairs (IEEE round to nearest per element) ---------------------------------
__device__ __forceinline__ uint64_t pk(float a, float b) {
    return (uint64_t)__float_as_uint(a) | ((uint64_t)__float_as_uint(b) << 32);
}
__device__ __forceinline__ uint64_t pk_u(uint32_t a, uint32_t b) { return (uint64_t)a | ((uint64_t)b << 32); }
__device__ __forceinline__ uint64_t mul2(uint64_t a, uint64_t b) {
    uint64_t r;
    asm("mul.rn.f32x2 %0, %1, %2;" : "=l"(r) : "l"(a), "l"(b));
    return r;
}
__device__ __forceinline__ uint64_t sub2(uint64_t a, uint64_t b) {
    uint64_t r;
    asm("sub.rn.f32x2 %0, %1, %2;" : "=l"(r) : "l"(a), "l"(b));
    return r;
}
// 0x4B400000 = 2^23 + 2^22: for |v| < 2^22 the float with bits 0x4B400000 + v
// is exactly 12582912 + v.
constexpr uint32_t kMagicBits = 0x4B400000u;
constexpr float kMagic = 12582912.0f;

// ---- weight unpacking ---------------------------------------------------------------
// One block of one weight row, OFF bytes into the row's raw chunk (16-byte
// aligned row base; OFF includes the paired view's skew): its 32 values as
// two 16-byte A-tile chunks (elements 0-15, 16-31) at chunk positions 2B, 2B+1
// of the row's 128 swizzled bytes, and its scale (and Q4_1 min).
template <int QT, int OFF, int B>
__device__ __forceinline__ void unpack_block(const uint8_t* row, uint8_t* dst, int r7, float* ws, float* wm) {
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
    auto word = [&](int byte) -> uint32_t {  // 4 bytes at `byte` (2-byte aligned)
        return (byte % 4 == 0) ? W[byte / 4] : __byte_perm(W[byte / 4], W[byte / 4 + 1], 0x5432);
    };
    const uint32_t hw = W[ST / 4];
    const uint32_t dbits = (ST % 4 == 0) ? (hw & 0xffffu) : (hw >> 16);
    *ws = f16_bits_to_f32((uint16_t)dbits);
    uint4 c0, c1;
    if constexpr (QT == kQ8_0) {
        c0 = make_uint4(word(ST + 2), word(ST + 6), word(ST + 10), word(ST + 14));
        c1 = make_uint4(word(ST + 18), word(ST + 22), word(ST + 26), word(ST + 30));
    } else {
        constexpr int P = ST + (QT == kQ4_1 ? 4 : 2);
        if constexpr (QT == kQ4_1) *wm = f16_bits_to_f32((uint16_t)(ST % 4 == 0 ? (hw >> 16) : (W[ST / 4 + 1] & 0xffffu)));
        const uint32_t p0 = word(P), p1 = word(P + 4), p2 = word(P + 8), p3 = word(P + 12);
        // GGML order: the low nibble of byte j is element j, the high nibble element j + 16
        c0 = make_uint4(p0 & 0x0F0F0F0Fu, p1 & 0x0F0F0F0Fu, p2 & 0x0F0F0F0Fu, p3 & 0x0F0F0F0Fu);
        c1 = make_uint4((p0 >> 4) & 0x0F0F0F0Fu, (p1 >> 4) & 0x0F0F0F0Fu, (p2 >> 4) & 0x0F0F0F0Fu,
                        (p3 >> 4) & 0x0F0F0F0Fu);
    }
    *reinterpret_cast<uint4*>(dst + (((2 * B) ^ r7) << 4)) = c0;
    *reinterpret_cast<uint4*>(dst + (((2 * B + 1) ^ r7) << 4)) = c1;
}

// Block B of K step KK of a raw chunk, row skew SK.
template <int QT, int KK, int B, int SK>
__device__ __forceinline__ void unpack_kstep_block(const uint8_t* row, uint8_t* dst, int r7, float* ws, float* wm) {
    unpack_block<QT, SK + block_bytes(QT) * (kI8Blocks * KK + B), B>(row, dst, r7, ws, wm);
}

template <bool PAIRED>
__device__ __forceinline__ int i8_tile_row(int j) {
    if constexpr (PAIRED) return j < 64 ? 2 * j : 2 * (j - 64) + 1;
    return j;
}

template <int QT, int NT, bool PAIRED>
__global__ void __launch_bounds__(kI8Threads, 1) gemm_i8_kernel(const __grid_constant__ IArgs a) {
    constexpr int PITCH = i8_pitch(QT, PAIRED);
    constexpr uint32_t AST = i8_astage(QT), XST = i8_xstage(NT);
    constexpr uint32_t kTmemCols = 2 * kI8Blocks * NT;  // 256 or 512
    constexpr int CH = NT / 2;                           // token columns per epilogue warp
    constexpr int YP = kI8Rows + 4;                      // staging pitch in floats
    static_assert(NT * YP * 4 <= kI8SA * AST, "staging tile must fit in the weight ring");
    extern __shared__ uint8_t smem_raw[];
    // 1024-byte aligned by pointer arithmetic on the shared array (an integer
    // round trip would hide the shared address space: generic loads)
    uint8_t* smem = smem_raw + ((1024u - (smem_u32(smem_raw) & 1023u)) & 1023u);
    uint8_t* sA = smem;                  // [SA] weight stages
    uint8_t* sX = sA + kI8SA * AST;      // [SX] activation stages
    uint8_t* sR = sX + kI8SX * XST;      // [SR] raw chunks
    uint64_t* full_a = reinterpret_cast<uint64_t*>(sR + kI8SR * kI8Rows * PITCH);
    uint64_t* empty_a = full_a + kI8SA;
    uint64_t* full_x = empty_a + kI8SA;
    uint64_t* empty_x = full_x + kI8SX;
    uint64_t* rfull = empty_x + kI8SX;
    uint64_t* rempty = rfull + kI8SR;
    uint64_t* dfull = rempty + kI8SR;  // [2] TMEM buffers written
    uint64_t* dempty = dfull + 2;      // [2] TMEM buffers consumed
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(dempty + 2);

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int n0 = blockIdx.x * kI8Rows, m0 = blockIdx.y * NT;
    const int steps = a.ksteps;
    const int nchunks = (steps + kI8StepsPerChunk - 1) / kI8StepsPerChunk;

    if (threadIdx.x == 0) {
        for (int s = 0; s < kI8SA; ++s) {
            mbar_init(&full_a[s], 128);
            mbar_init(&empty_a[s], 1 + 8);  // the MMA commit and the 8 epilogue warps
        }
        for (int s = 0; s < kI8SX; ++s) {
            mbar_init(&full_x[s], 1);
            mbar_init(&empty_x[s], 1 + 8);
        }
        for (int r = 0; r < kI8SR; ++r) {
            mbar_init(&rfull[r], 1);
            mbar_init(&rempty[r], 128);
        }
        for (int t = 0; t < 2; ++t) {
            mbar_init(&dfull[t], 1);
            mbar_init(&dempty[t], 8);
        }
        fence_mbar_init();
        prefetch_tmap(&a.tmap_xq);
        prefetch_tmap(&a.tmap_xs);
        prefetch_tmap(&a.tmap_w);
        if (QT != kQ8_0) prefetch_tmap(&a.tmap_xc);
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
        // ---------------------- activation TMA producer ----------------------------------
        if (lane == 0) {
            int issued = 0;
            pdl_wait();  // written by the activation-prep launch
            const uint32_t bytes = (uint32_t)NT * 128 + (uint32_t)kI8Blocks * NT * 4 * (QT == kQ8_0 ? 1 : 2);
            for (int i = 0; i < steps; ++i) {
                const int s = i % kI8SX;
                if (i >= kI8SX && !mbar_wait_bounded(&empty_x[s], ((i / kI8SX) - 1) & 1, a.err)) break;
                uint8_t* st = sX + s * XST;
                mbar_arrive_expect_tx(&full_x[s], bytes);
                tma_load_2d(st, &a.tmap_xq, i * 128, m0, &full_x[s]);
                tma_load_2d(st + NT * 128, &a.tmap_xs, m0, i * kI8Blocks, &full_x[s]);
                if (QT != kQ8_0) tma_load_2d(st + NT * 128 + kI8Blocks * NT * 4, &a.tmap_xc, m0, i * kI8Blocks, &full_x[s]);
                ++issued;
            }
            for (int i = (issued > kI8SX ? issued - kI8SX : 0); i < issued; ++i)
                mbar_wait_bounded(&full_x[i % kI8SX], (i / kI8SX) & 1, nullptr);
        }
    } else if (warp == 14) {
        // ------------------------- raw weight chunk producer ----------------------------
        if (lane == 0) {
            int r_issued = 0;
            constexpr int BB = block_bytes(QT);
            auto issue_raw = [&](int ci) {
                const int sr = ci % kI8SR;
                const int cb = ci * 8 * BB;
                uint8_t* dst = sR + sr * kI8Rows * PITCH;
                mbar_arrive_expect_tx(&rfull[sr], (uint32_t)(kI8Rows * PITCH));
                if constexpr (PAIRED) {
                    tma_load_2d(dst, &a.tmap_w, cb / 4, n0 / 2, &rfull[sr]);
                    tma_load_2d(dst + 64 * PITCH, &a.tmap_w, (a.row_bytes + cb - 8) / 4, n0 / 2, &rfull[sr]);
                } else {
                    tma_load_2d(dst, &a.tmap_w, cb / 4, n0, &rfull[sr]);
                }
            };
            if (a.weights_immutable)
                for (; r_issued < kI8SR && r_issued < nchunks; ++r_issued) issue_raw(r_issued);
            pdl_wait();
            for (; r_issued < nchunks; ++r_issued) {
                if (r_issued >= kI8SR &&
                    !mbar_wait_bounded(&rempty[r_issued % kI8SR], ((r_issued / kI8SR) - 1) & 1, a.err))
                    break;
                issue_raw(r_issued);
            }
            for (int i = (r_issued > kI8SR ? r_issued - kI8SR : 0); i < r_issued; ++i)
                mbar_wait_bounded(&rfull[i % kI8SR], (i / kI8SR) & 1, nullptr);
        }
    } else if (warp == 1) {
        // ------------------------------- MMA issuer -----------------------------------
        if (lane == 0) {
            pdl_wait();
            constexpr uint32_t idesc = i8_idesc(QT == kQ8_0, NT);
            for (int i = 0; i < steps; ++i) {
                const int sa = i % kI8SA, sx = i % kI8SX, tb = i & 1;
                if (!mbar_wait_bounded(&full_x[sx], (i / kI8SX) & 1, a.err) ||
                    !mbar_wait_bounded(&full_a[sa], (i / kI8SA) & 1, a.err) ||
                    (i >= 2 && !mbar_wait_bounded(&dempty[tb], ((i >> 1) - 1) & 1, a.err)))
                    break;
                tc_fence_after();
                const uint64_t ad = sw128_desc(smem_u32(sA + sa * AST));
                const uint64_t bd = sw128_desc(smem_u32(sX + sx * XST));
#pragma unroll
                for (int b = 0; b < kI8Blocks; ++b)  // one block (32 bytes of K) per MMA, each its own columns
                    mma_i8_ss(tmem + (uint32_t)((tb * kI8Blocks + b) * NT), ad + 2 * b, bd + 2 * b, idesc);
                mma_commit(&empty_x[sx]);
                mma_commit(&empty_a[sa]);
                mma_commit(&dfull[tb]);
            }
        }
        __syncwarp();
    } else if (warp <= 5) {
        // ---------------------- weight unpacking (warps 2-5) -----------------------------
        const int j = threadIdx.x - 64;  // tile row
        const int r7 = j & 7;
        const bool skew = PAIRED && j >= 64;  // warp-uniform
        pdl_wait();
        bool ok = true;
        int i = 0;
        for (int ci = 0; ci < nchunks && ok; ++ci) {
            const int sr = ci % kI8SR;
            if (!mbar_wait_bounded(&rfull[sr], (ci / kI8SR) & 1, a.err)) break;
            const uint8_t* rrow = sR + sr * kI8Rows * PITCH + j * PITCH;
            const int nk = min(kI8StepsPerChunk, steps - ci * kI8StepsPerChunk);
            for (int kk = 0; kk < nk && ok; ++kk, ++i) {
                const int s = i % kI8SA;
                if (i >= kI8SA && !mbar_wait_bounded(&empty_a[s], ((i / kI8SA) - 1) & 1, a.err)) {
                    ok = false;
                    break;
                }
                uint8_t* dst = sA + s * AST + (j >> 3) * 1024 + r7 * 128;
                float* ws = reinterpret_cast<float*>(sA + s * AST + kI8ATile);
                float* wm = ws + kI8Blocks * kI8Rows;
                const int nvalid = min(kI8Blocks, a.nb - i * kI8Blocks);  // blocks past the row end are skipped
                auto blocks = [&](auto kkc, auto skc) {
                    constexpr int KKc = decltype(kkc)::value, SKc = decltype(skc)::value;
                    unpack_kstep_block<QT, KKc, 0, SKc>(rrow, dst, r7, ws + 0 * kI8Rows + j, wm + 0 * kI8Rows + j);
                    if (nvalid > 1)
                        unpack_kstep_block<QT, KKc, 1, SKc>(rrow, dst, r7, ws + 1 * kI8Rows + j, wm + 1 * kI8Rows + j);
                    if (nvalid > 2)
                        unpack_kstep_block<QT, KKc, 2, SKc>(rrow, dst, r7, ws + 2 * kI8Rows + j, wm + 2 * kI8Rows + j);
                    if (nvalid > 3)
                        unpack_kstep_block<QT, KKc, 3, SKc>(rrow, dst, r7, ws + 3 * kI8Rows + j, wm + 3 * kI8Rows + j);
                };
                if (kk == 0) {
                    if (skew) blocks(std::integral_constant<int, 0>{}, std::integral_constant<int, 8>{});
                    else blocks(std::integral_constant<int, 0>{}, std::integral_constant<int, 0>{});
                } else {
                    if (skew) blocks(std::integral_constant<int, 1>{}, std::integral_constant<int, 8>{});
                    else blocks(std::integral_constant<int, 1>{}, std::integral_constant<int, 0>{});
                }
                fence_proxy_async_smem();  // generic writes -> visible to the tensor core
                mbar_arrive(&full_a[s]);
            }
            mbar_arrive(&rempty[sr]);
        }
    } else {
        // ------------------------- float epilogue (warps 6-13) ---------------------------
        const int q = warp & 3;               // TMEM lane quarter
        const int half = (warp - 6) >> 2;     // which half of the token columns
        const int j = q * 32 + lane;          // tile row
        const int c0 = half * CH;             // first token column of this warp
        float acc[CH];
#pragma unroll
        for (int c = 0; c < CH; ++c) acc[c] = 0.0f;  // the reference's `let mut dot = 0.0`
        pdl_wait();
        bool ok = true;
        for (int i = 0; i < steps && ok; ++i) {
            const int sa = i % kI8SA, sx = i % kI8SX, tb = i & 1;
            if (!mbar_wait_bounded(&dfull[tb], (i >> 1) & 1, a.err) ||
                !mbar_wait_bounded(&full_x[sx], (i / kI8SX) & 1, a.err) ||
                !mbar_wait_bounded(&full_a[sa], (i / kI8SA) & 1, a.err)) {
                ok = false;
                break;
            }
            tc_fence_after();
            const float* ws = reinterpret_cast<const float*>(sA + sa * AST + kI8ATile);
            const float* xsb = reinterpret_cast<const float*>(sX + sx * XST + NT * 128);
            const uint32_t* xcb = reinterpret_cast<const uint32_t*>(xsb + kI8Blocks * NT);
            const int nvalid = min(kI8Blocks, a.nb - i * kI8Blocks);
            for (int b = 0; b < nvalid; ++b) {  // blocks in order: the reference's sum order
                uint32_t v[CH];
                tmem_ld_cols<CH>(tmem + ((uint32_t)(q * 32) << 16) + (uint32_t)((tb * kI8Blocks + b) * NT + c0), v);
                const float wsj = ws[b * kI8Rows + j];
                const float* xs = xsb + b * NT + c0;
                const uint32_t* xc = xcb + b * NT + c0;
                // The conversion and the first product run on f32 pairs (exact, or
                // a single rounding with no add to fuse with); the last product and
                // the accumulation are scalar __fmul_rn / __fadd_rn, which the
                // compiler never contracts into an fma.
                if constexpr (QT == kQ4_1) {
                    const float wmj = ws[kI8Blocks * kI8Rows + b * kI8Rows + j];
#pragma unroll
                    for (int c = 0; c < CH; c += 2) {
                        const uint64_t fu = sub2(pk_u(v[c] + kMagicBits, v[c + 1] + kMagicBits), pk(kMagic, kMagic));
                        const float f0 = __uint_as_float((uint32_t)fu), f1 = __uint_as_float((uint32_t)(fu >> 32));
                        const float s0 = __fadd_rn(__fmul_rn(wsj, f0), __fmul_rn(wmj, __uint_as_float(xc[c])));
                        const float s1 = __fadd_rn(__fmul_rn(wsj, f1), __fmul_rn(wmj, __uint_as_float(xc[c + 1])));
                        acc[c] = __fadd_rn(acc[c], __fmul_rn(xs[c], s0));
                        acc[c + 1] = __fadd_rn(acc[c + 1], __fmul_rn(xs[c + 1], s1));
                    }
                } else {
#pragma unroll
                    for (int c = 0; c < CH; c += 2) {
                        uint32_t k0 = kMagicBits, k1 = kMagicBits;
                        if constexpr (QT == kQ4_0) {  // 0x4B400000 - 8 * qsum: the -8 offset of the nibbles
                            k0 = xc[c];
                            k1 = xc[c + 1];
                        }
                        const uint64_t f = sub2(pk_u(v[c] + k0, v[c + 1] + k1), pk(kMagic, kMagic));
                        const uint64_t t = mul2(f, *reinterpret_cast<const uint64_t*>(xs + c));
                        acc[c] = __fadd_rn(acc[c], __fmul_rn(__uint_as_float((uint32_t)t), wsj));
                        acc[c + 1] = __fadd_rn(acc[c + 1], __fmul_rn(__uint_as_float((uint32_t)(t >> 32)), wsj));
                    }
                }
            }
            tc_fence_before();
            __syncwarp();
            if (lane == 0) {
                mbar_arrive(&dempty[tb]);
                mbar_arrive(&empty_x[sx]);
                mbar_arrive(&empty_a[sa]);
            }
        }
        // results -> staging [token][weight row] in the (idle) weight ring -> y
        asm volatile("bar.sync 1, %0;" ::"r"(kI8EpiThreads) : "memory");  // every epilogue read of the rings is done
        float* ys = reinterpret_cast<float*>(sA);
        const int wr = i8_tile_row<PAIRED>(j);
#pragma unroll
        for (int c = 0; c < CH; ++c) ys[(c0 + c) * YP + wr] = acc[c];
        asm volatile("bar.sync 1, %0;" ::"r"(kI8EpiThreads) : "memory");
        const int et = threadIdx.x - 6 * 32;
        const int mv = min(NT, a.M - m0);
        if (ok) {
            for (int idx = et; idx < mv * kI8Rows; idx += kI8EpiThreads) {
                const int m = idx / kI8Rows, c = idx % kI8Rows;
                if (n0 + c < a.N) a.y[(int64_t)(m0 + m) * a.N + n0 + c] = ys[m * YP + c];
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
const void* i8_pick_nt(int nt) {
    return nt == 32 ? (const void*)gemm_i8_kernel<QT, 32, PAIRED> : (const void*)gemm_i8_kernel<QT, 64, PAIRED>;
}
const void* gemm_i8_kernel_for(int qt, int nt, bool paired) {
    if (qt == kQ8_0) return paired ? i8_pick_nt<kQ8_0, true>(nt) : i8_pick_nt<kQ8_0, false>(nt);
    if (qt == kQ4_0) return paired ? i8_pick_nt<kQ4_0, true>(nt) : i8_pick_nt<kQ4_0, false>(nt);
    return paired ? i8_pick_nt<kQ4_1, true>(nt) : i8_pick_nt<kQ4_1, false>(nt);
}

size_t al256(size_t v) { return (v + 255) & ~size_t(255); }
int i8_nt(int M) { return M <= 32 ? 32 : 64; }
int round4(int v) { return (v + 3) & ~3; }

}  // namespace

bool gemm_i8_supported(int qt, int M, int N, int K) {
    if (M < kGemmMinRows || N < 1 || K < QK || K % QK) return false;
    const int bb = block_bytes(qt);
    if (!bb) return false;
    const int64_t row_bytes = (int64_t)(K / QK) * bb;
    return row_bytes % 16 == 0 || (row_bytes % 16 == 8 && N % 2 == 0);
}

size_t gemm_i8_workspace_bytes(int M, int N, int K, int qt) {
    (void)N;
    (void)qt;
    const size_t nbp = (size_t)round4(K / QK), mp = (size_t)round4(M);
    return al256((size_t)M * K) + 2 * al256(nbp * mp * 4);
}

cudaError_t launch_gemm_i8(int qt, const uint8_t* w, const float* x, float* y, int M, int N, int K, void* ws,
                           int* err, cudaStream_t st, bool weights_immutable) {
    const int nb = K / QK, nbp = round4(nb), Mp = round4(M);
    uint8_t* base = static_cast<uint8_t*>(ws);
    int8_t* xq = reinterpret_cast<int8_t*>(base);
    float* xs = reinterpret_cast<float*>(base + al256((size_t)M * K));
    uint32_t* xc = reinterpret_cast<uint32_t*>(base + al256((size_t)M * K) + al256((size_t)nbp * Mp * 4));
    cudaError_t e = launch_xprep_i8gemm(qt, x, M, K, Mp, xq, xs, xc, st);
    if (e != cudaSuccess) return e;
    const int nt = i8_nt(M);
    const int row_bytes = nb * block_bytes(qt);
    const bool paired = row_bytes % 16 != 0;
    const int pitch = i8_pitch(qt, paired);
    IArgs a;
    e = encode_map_2d(&a.tmap_xq, CU_TENSOR_MAP_DATA_TYPE_UINT8, xq, (uint64_t)K, (uint64_t)M, (uint64_t)K, 128,
                      (uint32_t)nt, CU_TENSOR_MAP_SWIZZLE_128B);
    if (e == cudaSuccess)
        e = encode_map_2d(&a.tmap_xs, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, xs, (uint64_t)Mp, (uint64_t)nbp, (uint64_t)Mp * 4,
                          (uint32_t)nt, kI8Blocks, CU_TENSOR_MAP_SWIZZLE_NONE);
    if (e == cudaSuccess)
        e = encode_map_2d(&a.tmap_xc, CU_TENSOR_MAP_DATA_TYPE_UINT32, xc, (uint64_t)Mp, (uint64_t)nbp, (uint64_t)Mp * 4,
                          (uint32_t)nt, kI8Blocks, CU_TENSOR_MAP_SWIZZLE_NONE);
    if (e == cudaSuccess) {
        if (paired)
            e = encode_map_2d(&a.tmap_w, CU_TENSOR_MAP_DATA_TYPE_UINT32, w, (uint64_t)row_bytes / 2, (uint64_t)N / 2,
                              (uint64_t)row_bytes * 2, (uint32_t)pitch / 4, 64, CU_TENSOR_MAP_SWIZZLE_NONE);
        else
            e = encode_map_2d(&a.tmap_w, CU_TENSOR_MAP_DATA_TYPE_UINT32, w, (uint64_t)row_bytes / 4, (uint64_t)N,
                              (uint64_t)row_bytes, (uint32_t)pitch / 4, kI8Rows, CU_TENSOR_MAP_SWIZZLE_NONE);
    }
    if (e != cudaSuccess) return e;
    a.y = y;
    a.M = M;
    a.N = N;
    a.K = K;
    a.nb = nb;
    a.ksteps = (nb + kI8Blocks - 1) / kI8Blocks;
    a.row_bytes = row_bytes;
    a.weights_immutable = weights_immutable ? 1 : 0;
    a.err = err;
    const void* fn = gemm_i8_kernel_for(qt, nt, paired);
    const size_t smem = i8_smem_bytes(qt, nt, paired);
    e = ensure_dynamic_smem(fn, smem);
    if (e != cudaSuccess) return e;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3((unsigned)((N + kI8Rows - 1) / kI8Rows), (unsigned)((M + nt - 1) / nt));
    cfg.blockDim = dim3(kI8Threads);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    void* args[] = {(void*)&a};
    note_launch();
    return cudaLaunchKernelExC(&cfg, fn, args);
}

}  // namespace qmm
