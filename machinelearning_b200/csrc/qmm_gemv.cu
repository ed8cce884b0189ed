// Decode-time quantised GEMV (M <= 64) for sm_100a.
//
// y[M, N] = x[M, K] . W[N, K]^T with W in raw GGUF block layout (Q4_0, Q4_1 or
// Q8_0 rows of K/32 blocks, exactly as on disk). Replaces the M <= 4 / M > 4
// CPU loops of matmul_f32_q4 / _q4_native / _q8 / _q8_v2 / _q4_1 / _q4_1_native
// (reference llmserve/llmmodel/kernel/main/src/core/quantize.rs:297-1070).
//
// gemv_plan() sends small decode shapes (f32 activations, M <= 16, weights
// that fit in the SMs' shared memory) to the one-launch resident kernel of
// qmm_gemv_resident.cu; everything else runs here as an x-prep kernel plus the
// streaming GEMV below.
//
// Structure (persistent grid, kW warps per CTA, no dedicated producer):
//   * every warp owns 32-row tiles (two 16-row MMA groups sharing one set of
//     activation fragments) and a ring of kSW shared-memory stages. Lane 0
//     keeps the ring kSW tiles ahead: as soon as the warp has read a stage it
//     refills it with TMA -- one 2-D tensor tile [32 rows x kc blocks] when
//     the row pitch is a multiple of 16 bytes, or two paired-row tiles when it
//     is 8 mod 16 (K = 1152); other pitches use 16-byte cp.async pieces.
//     Completion is counted on per-stage mbarriers.
//   * per 32-element block a lane dequantises its A fragments in registers
//     (f16 magic-number trick for f32 activations, raw/offset int8 for Q8_0
//     activations), runs mma.sync against pre-laid-out activation fragments
//     (B, prefetched one block ahead) starting from a precomputed accumulator
//     value, then applies the per-block scales in f32. The tensor pipe does
//     the multiply-adds, so issue slots go to dequantisation.
//   * stage pitches are chosen so the 8 rows x 4 words a warp reads per shared
//     load land in 32 distinct banks.
//   * small N: a tile's K range is split over `ks` warps in 8-block granules;
//     the last warp to finish (atomic ticket) sums the partials in split
//     order, so results are deterministic.
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
#include <type_traits>
#include <utility>

#include "qmm_common.cuh"
#include "qmm_gemv_frag.cuh"
#include "qmm_kernels.cuh"

namespace qmm {

namespace {

constexpr int kMaxSW = 3;              // pipeline stages per warp (the plan picks 2 or 3)
constexpr size_t kSmemPerSM = 227 * 1024;

struct Args {
    CUtensorMap tmap;  // weights as a [N rows][row_bytes/4] uint32 tensor (TMA loaders)
    const uint8_t* w;
    uint64_t w_bytes;
    float* y;
    const void* xa;
    const uint32_t* side;
    float* partial;
    unsigned* counters;
    int M, N, nb, row_bytes, ks, nbu, kc, pitch, units, weights_immutable, sw;
    int* err;
    int gact;        // >= 0: gate/up epilogue (GatedOut), y unused
    float* gout;     // [M][ghidden]
    int64_t ghidden;
};

// Sequential activation cursor of one unit: each load advances one block.
template <int NT, bool NATIVE>
struct XCursor {
    static constexpr int kRec = NATIVE ? 8 : 32;
    const uint8_t* rec;   // this lane's record of token tile 0 for the next block
    const uint4* side;    // this lane's side record of token tile 0 for the next block
    uint32_t rec_step;    // bytes per block
    uint32_t side_step;   // uint4 per block
    uint32_t valid;       // bit nt: token nt*8+g < M

    __device__ __forceinline__ void load(XFrag (&x)[NT]) {
#pragma unroll
        for (int nt = 0; nt < NT; ++nt) {
            x[nt].hi = make_uint4(0, 0, 0, 0);
            x[nt].lo = make_uint4(0, 0, 0, 0);
            if (valid & (1u << nt)) {
                const uint8_t* r = rec + nt * 8 * 4 * kRec;
                if constexpr (NATIVE) {
                    const uint2 q = __ldg(reinterpret_cast<const uint2*>(r));
                    x[nt].hi.x = q.x;
                    x[nt].hi.y = q.y;
                } else {
                    x[nt].hi = __ldg(reinterpret_cast<const uint4*>(r));
                    x[nt].lo = __ldg(reinterpret_cast<const uint4*>(r) + 1);
                }
            }
            // side records are padded to the token tiles, always readable
            x[nt].c4 = __ldg(side + nt * 8);
            x[nt].s4 = __ldg(side + nt * 8 + 1);
        }
        rec += rec_step;
        side += side_step;
    }
};

// Position of a warp in its tile sequence: unit u, chunk starting at kb0.
struct TileIter {
    int u, kb0, kb_end;
    __device__ __forceinline__ void start(const Args& a, int unit) {
        u = unit;
        if (u < a.units) {
            kb0 = (u % a.ks) * a.nbu;
            kb_end = min(a.nb, kb0 + a.nbu);
        }
    }
    __device__ __forceinline__ bool valid(const Args& a) const { return u < a.units; }
    __device__ __forceinline__ void next(const Args& a, int G) {
        kb0 += a.kc;
        if (kb0 >= kb_end) start(a, u + G);
    }
};

// Fills one stage with the tile at `it`. TMA loaders: lane 0 only. cp.async:
// the whole warp (and it arrives on the barrier from every lane).
template <int QT, int LOADER>
__device__ __forceinline__ void issue_tile(const Args& a, const TileIter& it, uint8_t* stage, uint64_t* fb,
                                           int lane) {
    constexpr int BB = block_bytes(QT);
    const int tile = it.u / a.ks;
    if constexpr (LOADER == kLoaderTma2d) {
        if (lane == 0) {
            mbar_arrive_expect_tx(fb, (uint32_t)(kRows * a.pitch));
            // rows past N and columns past the row end are zero-filled
            tma_load_2d(stage, &a.tmap, it.kb0 * BB / 4, tile * kRows, fb);
        }
    } else if constexpr (LOADER == kLoaderTmaPairs) {
        if (lane == 0) {
            mbar_arrive_expect_tx(fb, (uint32_t)(kRows * a.pitch));
            tma_load_2d(stage, &a.tmap, it.kb0 * BB / 4, tile * (kRows / 2), fb);
            tma_load_2d(stage + (kRows / 2) * a.pitch, &a.tmap, (a.row_bytes + it.kb0 * BB - 8) / 4,
                        tile * (kRows / 2), fb);
        }
    } else {
        const int kb1 = min(it.kb_end, it.kb0 + a.kc);
        const int rows = min(kRows, a.N - tile * kRows);
        const uint64_t wfl = a.w_bytes & ~uint64_t(15);
        for (int r = 0; r < rows; ++r) {
            const uint64_t beg = (uint64_t)(tile * kRows + r) * (uint64_t)a.row_bytes + (uint64_t)it.kb0 * BB;
            const uint64_t end = beg + (uint64_t)(kb1 - it.kb0) * BB;
            const uint64_t a16 = beg & ~uint64_t(15);
            uint64_t e16 = (end + 15) & ~uint64_t(15);
            uint8_t* dst = stage + r * a.pitch;
            if (e16 > wfl) {
                // the last row's window would pass the end of the buffer: the
                // ragged tail is copied with plain loads
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
}

template <int QT, int NT, bool NATIVE, int LOADER>
__global__ void __launch_bounds__(kThreads, 2) gemv_kernel(const __grid_constant__ Args a) {
    extern __shared__ __align__(128) uint8_t smem[];
    constexpr int BB = block_bytes(QT);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int stage_bytes = kRows * a.pitch;
    const int SW = a.sw;  // stages per warp
    uint64_t* full = reinterpret_cast<uint64_t*>(smem + kW * SW * stage_bytes);
    if (threadIdx.x == 0) {
        // TMA tiles complete with one arrival + transaction bytes; the cp.async
        // loader arrives once per lane plus once for plain tail stores
        const uint32_t full_count = LOADER == kLoaderCpAsync ? 33u : 1u;
        for (int i = 0; i < kW * SW; ++i) mbar_init(&full[i], full_count);
        fence_mbar_init();
        if (LOADER != kLoaderCpAsync) prefetch_tmap(&a.tmap);
    }
    __syncthreads();
    pdl_launch_dependents();

    const int G = gridDim.x * kW;
    uint8_t* ring = smem + warp * SW * stage_bytes;
    uint64_t* fbar = full + warp * SW;
    // units are dealt round-robin over CTAs first, so every SM gets work
    const int u_first = warp * gridDim.x + blockIdx.x;

    // Weights a caller declared immutable cannot be written by the preceding
    // work in the stream: start streaming them before the dependency wait.
    if (!a.weights_immutable) pdl_wait();
    TileIter iss;
    iss.start(a, u_first);
    int issued = 0;
    for (int s = 0; s < SW && iss.valid(a); ++s) {
        issue_tile<QT, LOADER>(a, iss, ring + s * stage_bytes, &fbar[s], lane);
        iss.next(a, G);
        ++issued;
    }
    pdl_wait();  // the activations come from the preceding kernel (the x-prep)

    const int g = lane >> 2, t = lane & 3;
    const int Mpad = token_pad(a.M);
    int lt = 0;  // stages consumed
    bool ok = true;
    for (int u = u_first; u < a.units && ok; u += G) {
        const int tile = u / a.ks, ksi = u % a.ks;
        const int kb_begin = ksi * a.nbu;
        const int kb_end = min(a.nb, kb_begin + a.nbu);
        float acc[2][NT][4];
#pragma unroll
        for (int r = 0; r < 2; ++r)
#pragma unroll
            for (int nt = 0; nt < NT; ++nt) acc[r][nt][0] = acc[r][nt][1] = acc[r][nt][2] = acc[r][nt][3] = 0.0f;
        const int row0 = tile * kRows + g;  // this lane's rows: row0 + {0, 8, 16, 24}
        XCursor<NT, NATIVE> xc;
        {
            constexpr int kRec = NATIVE ? 8 : 32;
            xc.rec = static_cast<const uint8_t*>(a.xa) + (((int64_t)kb_begin * a.M + g) * 4 + t) * kRec;
            xc.rec_step = (uint32_t)(a.M * 4 * kRec);
            xc.side = reinterpret_cast<const uint4*>(a.side) + ((int64_t)kb_begin * (Mpad / 2) + t) * 2;
            xc.side_step = (uint32_t)Mpad;  // (Mpad / 2) records of 2 uint4
            xc.valid = 0;
#pragma unroll
            for (int nt = 0; nt < 8; ++nt) xc.valid |= (nt * 8 + g < a.M) ? (1u << nt) : 0u;
        }
        XFrag xa[NT], xb[NT];
        if constexpr (NT <= 2) xc.load(xa);  // prefetched one block ahead below
        for (int cs = kb_begin; cs < kb_end; cs += a.kc) {
            const int ce = min(kb_end, cs + a.kc);
            const int slot = lt % SW;
            if (!mbar_wait_bounded(&fbar[slot], (lt / SW) & 1, a.err)) {
                ok = false;
                break;
            }
            const uint8_t* sbase = ring + slot * stage_bytes;
            const uint8_t* rb[4];
#pragma unroll
            for (int i = 0; i < 4; ++i) {
                const int j = g + 8 * i;  // row within the tile
                if constexpr (LOADER == kLoaderTma2d) {
                    rb[i] = sbase + j * a.pitch;
                } else if constexpr (LOADER == kLoaderTmaPairs) {
                    rb[i] = sbase + ((j & 1) * (kRows / 2) + (j >> 1)) * a.pitch + (j & 1) * 8;
                } else {
                    const uint64_t gaddr = (uint64_t)(row0 + 8 * i) * a.row_bytes + (uint64_t)cs * BB;
                    rb[i] = sbase + j * a.pitch + (uint32_t)(gaddr & 15);
                }
            }
            auto consume = [&](int j, const XFrag (&xf)[NT], auto aligned) {
                constexpr bool AL = decltype(aligned)::value;
                const uint32_t o = (uint32_t)j * BB;
                consume_group<QT, NT, NATIVE, AL>(rb[0] + o, rb[1] + o, t, xf, acc[0]);
                consume_group<QT, NT, NATIVE, AL>(rb[2] + o, rb[3] + o, t, xf, acc[1]);
            };
            // In a dense TMA tile (pitch multiple of 16) Q8_0/Q4_0 payloads sit
            // on 4-byte boundaries for odd block offsets, Q4_1 ones always.
            constexpr bool kTma = LOADER != kLoaderCpAsync;
            using EvenAl = std::integral_constant<bool, kTma && QT == kQ4_1>;
            using OddAl = std::integral_constant<bool, kTma>;
            if constexpr (NT <= 2) {
                int b = cs;
                for (; b + 1 < ce; b += 2) {
                    xc.load(xb);  // block b+1
                    consume(b - cs, xa, EvenAl{});
                    if (b + 2 < kb_end) xc.load(xa);  // block b+2
                    consume(b + 1 - cs, xb, OddAl{});
                }
                if (b < ce) {  // odd chunk length (cp.async loader only)
                    if (b + 1 < kb_end) xc.load(xb);
                    consume(b - cs, xa, std::false_type{});
#pragma unroll
                    for (int nt = 0; nt < NT; ++nt) xa[nt] = xb[nt];
                }
            } else {
                // wide token tiles: load in place (prefetching would spill registers)
                for (int b = cs; b < ce; ++b) {
                    xc.load(xa);
                    consume(b - cs, xa, std::false_type{});
                }
            }
            // stage read: refill it with the tile SW ahead
            __syncwarp();
            ++lt;
            if (iss.valid(a)) {
                fence_proxy_async_smem();
                issue_tile<QT, LOADER>(a, iss, ring + slot * stage_bytes, &fbar[slot], lane);
                iss.next(a, G);
                ++issued;
            }
        }
        if (!ok) break;
        // ------------------------------- epilogue -------------------------------------
        // A gate/up weight (a.gact >= 0): rows row0 + {0, 8} are gate rows
        // tile * 16 + g + {0, 8}, rows row0 + {16, 24} the matching up rows.
        const bool gated = a.gact >= 0;
        if (gated && a.ks == 1) {
#pragma unroll
            for (int nt = 0; nt < NT; ++nt) {
#pragma unroll
                for (int e = 0; e < 4; ++e) {
                    const int m = nt * 8 + 2 * t + (e & 1);
                    const int64_t i = (int64_t)tile * kGateGroup + g + ((e & 2) ? 8 : 0);
                    if (m < a.M && i < a.ghidden)
                        a.gout[(int64_t)m * a.ghidden + i] = gated_value(a.gact, acc[0][nt][e], acc[1][nt][e]);
                }
            }
        }
        float* dst = a.ks == 1 ? a.y : a.partial + (int64_t)ksi * a.M * a.N;
#pragma unroll
        for (int r = 0; r < 2 && !(gated && a.ks == 1); ++r) {
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
                if (gated) {
#pragma unroll
                    for (int nt = 0; nt < NT; ++nt) {
#pragma unroll
                        for (int e = 0; e < 4; ++e) {
                            const int m = nt * 8 + 2 * t + (e & 1);
                            const int row = row0 + ((e & 2) ? 8 : 0);
                            const int64_t i = (int64_t)tile * kGateGroup + g + ((e & 2) ? 8 : 0);
                            if (m < a.M && i < a.ghidden) {
                                float s = 0.0f, su = 0.0f;
                                for (int k = 0; k < a.ks; ++k) {
                                    const float* pk = a.partial + ((int64_t)k * a.M + m) * a.N + row;
                                    s += __ldcg(pk);
                                    su += __ldcg(pk + kGateGroup);
                                }
                                a.gout[(int64_t)m * a.ghidden + i] = gated_value(a.gact, s, su);
                            }
                        }
                    }
                }
#pragma unroll
                for (int r = 0; r < 2 && !gated; ++r) {
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
    if (!ok) {
        // a wait gave up (error word set): let the copies this warp started land
        // before the CTA exits
        for (int i = lt; i < issued; ++i) mbar_wait_bounded(&fbar[i % SW], (i / SW) & 1, nullptr);
    }
}

template <int QT, bool NATIVE, int LOADER>
const void* pick_nt(int nt) {
    switch (nt) {
        case 1: return (const void*)gemv_kernel<QT, 1, NATIVE, LOADER>;
        case 2: return (const void*)gemv_kernel<QT, 2, NATIVE, LOADER>;
        case 4: return (const void*)gemv_kernel<QT, 4, NATIVE, LOADER>;
        default: return (const void*)gemv_kernel<QT, 8, NATIVE, LOADER>;
    }
}

template <int QT, bool NATIVE>
const void* pick_loader(int loader, int nt) {
    if (loader == kLoaderTma2d) return pick_nt<QT, NATIVE, kLoaderTma2d>(nt);
    if (loader == kLoaderTmaPairs) return pick_nt<QT, NATIVE, kLoaderTmaPairs>(nt);
    return pick_nt<QT, NATIVE, kLoaderCpAsync>(nt);
}

const void* kernel_for(const GemvPlan& p) {
    if (p.native) {
        if (p.qt == kQ8_0) return pick_loader<kQ8_0, true>(p.loader, p.nt);
        if (p.qt == kQ4_0) return pick_loader<kQ4_0, true>(p.loader, p.nt);
        return pick_loader<kQ4_1, true>(p.loader, p.nt);
    }
    if (p.qt == kQ8_0) return pick_loader<kQ8_0, false>(p.loader, p.nt);
    if (p.qt == kQ4_0) return pick_loader<kQ4_0, false>(p.loader, p.nt);
    return pick_loader<kQ4_1, false>(p.loader, p.nt);
}

size_t align256(size_t v) { return (v + 255) & ~size_t(255); }

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

// The weights viewed as a [N rows][row_bytes / 4] uint32 tensor with a box of
// [kc blocks, 32 rows] (paired rows: [N/2][2 * row_bytes / 4], 16-row boxes).
// Encoded on the stack, no heap.
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

// Same map, cached per (device, pointer, shape, box).
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
    CUtensorMap m;
    e = weight_tensor_map_uncached(w, p, &m);
    if (e != cudaSuccess) return e;
    if (cache.size() > 4096) cache.clear();
    cache[key] = m;
    *out = m;
    return cudaSuccess;
}

// Row pitch in 32-bit words congruent to 4 mod 8 puts the 8 rows x 4 words of
// one warp-wide shared load in 32 distinct banks.
bool bank_friendly(int pitch_bytes) { return ((pitch_bytes / 4) & 7) == 4; }

// Resident-kernel configuration: clusters of C CTAs splitting K (C a power of
// two, at most 8), tw 32-row tiles per cluster, shared memory within
// kResidentSmemMax, and a grid the device can hold in one wave (the runtime's
// occupancy answer: at most one CTA per SM when it cannot say). Among those,
// the smallest estimated latency in nanoseconds, from B200 timestamps of the
// kernel's phases: ~200 per block per warp (x1.6 for two token tiles), ~500
// plus ~6.5 per (block, token) task for the activation prep, ~1800 for the
// cluster exchange (two cluster barriers and the DSMEM sums), and the CTA's
// weight bytes at ~60 B/ns (the part of the weight fetch the dependency wait
// does not hide).
constexpr size_t kResidentSmemMax = 200 * 1024;

bool resident_plan(GemvPlan& q, int num_sms) {
    if (q.native || q.M > 16 || q.loader == kLoaderCpAsync || q.kc != kChunk) return false;
    const int T = (q.N + kRows - 1) / kRows;
    const int G = (q.nb + kChunk - 1) / kChunk;
    double best = 0.0;
    bool found = false;
    for (int C = 1; C <= kMaxResidentCluster && C <= G; C *= 2) {
        const int gpc = (G + C - 1) / C;
        const int nbc = q.nb < gpc * kChunk ? q.nb : gpc * kChunk;
        for (int tw = 1; tw <= kW; tw *= 2) {
            const long clusters = (T + tw - 1) / tw;
            const size_t smem = resident_layout(tw, gpc, q.pitch, q.M).total;
            if (smem > kResidentSmemMax) continue;
            const int cap = resident_capacity(q.qt, q.loader, q.nt, C, smem);
            if (clusters > (cap > 0 ? (long)cap : (long)(num_sms / C))) continue;
            const int wpt = kW / tw;
            const int bpw = (nbc + wpt - 1) / wpt;
            const double wbytes = (double)tw * gpc * kRows * q.pitch;
            const double cost = bpw * 200.0 * (q.nt > 1 ? 1.6 : 1.0) + (500.0 + 6.5 * nbc * q.M) +
                                (C > 1 ? 1800.0 : 0.0) + wbytes / 60.0;
            if (!found || cost < best) {
                found = true;
                best = cost;
                q.cluster = C;
                q.tw = tw;
                q.gpc = gpc;
                q.grid = (int)(clusters * C);
                q.smem = smem;
            }
        }
    }
    if (!found) return false;
    q.kind = kGemvResident;
    q.ks = 1;
    q.nbu = q.nb;
    q.sw = 0;
    q.units = 0;
    return true;
}

// The band kernel (M = 1, f32 activations, 16-byte row pitch), for weights
// the resident kernel cannot hold. K is cut into ks slices of whole chunks of
// kc = kBandWarps * band_bpw blocks (a multiple of 8: 16-byte aligned TMA
// coordinates); a chunk is one 2-D box of 32 rows, its width padded to a row
// pitch of 4 mod 8 words (B200, measured: 32-row boxes of 0.6 to 1 KB rows
// stream at ~5.5-5.8 TB/s through a 4-6 stage ring, 288-byte rows at ~3.8).
// The activations of a slice live in shared memory; the ring takes what they
// and the partial tiles leave (3 to 8 stages). Among the fitting choices: the
// shortest stream per CTA (its tiles times its slice's boxes), then the
// smaller ks (fewer partial sums in global memory).
constexpr size_t kBandSmemMax = 227 * 1024;
constexpr int kBandMaxM = 1;  // token counts routed here (band_kernel_m)

bool band_plan(GemvPlan& q, int num_sms) {
    if (q.native || q.M > kBandMaxM || q.row_bytes % 16 != 0) return false;
    const int bb = block_bytes(q.qt);
    const int kc = kBandWarps * band_bpw(q.qt);
    const int mt = band_mt(q.M);
    int pitch = kc * bb;
    if (((pitch / 4) & 7) != 4) pitch += 16;
    if (pitch > 1024) return false;
    const int tiles = (q.N + kRows - 1) / kRows;
    double best = 0.0;
    bool found = false;
    for (int ks = 1; ks <= 8; ks *= 2) {
        const int nq = ((q.nb + ks - 1) / ks + kc - 1) / kc;  // chunks per slice
        const int nbs = nq * kc;
        if (ks > 1 && (long)nbs * (ks - 1) >= q.nb) continue;  // a slice without blocks
        const size_t fixed = band_layout(0, pitch, nbs, mt, kBandWarps).total;
        if (fixed + 3 * 32 * (size_t)pitch > kBandSmemMax) continue;
        int S = (int)((kBandSmemMax - fixed) / (32 * (size_t)pitch));
        if (S > 8) S = 8;
        const size_t smem = band_layout(S, pitch, nbs, mt, kBandWarps).total;
        int cap = band_capacity(q.qt, q.M, smem);
        if (cap <= 0) cap = num_sms;
        long grid = cap < (long)tiles * ks ? cap : (long)tiles * ks;
        grid -= grid % ks;
        if (grid < ks) continue;
        const long per_slice = grid / ks;
        const long rounds = (tiles + per_slice - 1) / per_slice;
        // shallow rings lose bandwidth (measured: 3 stages ~13% below 6)
        const double depth = S >= 5 ? 1.0 : (S == 4 ? 1.05 : 1.13);
        const double cost = (double)rounds * nq * 32.0 * pitch * depth * (ks > 1 ? 1.02 : 1.0);
        if (!found || cost < best) {
            found = true;
            best = cost;
            q.ks = ks;
            q.nbu = nbs;
            q.sw = S;
            q.smem = smem;
            q.grid = (int)grid;
        }
    }
    if (!found) return false;
    q.kind = kGemvBand;
    q.kc = kc;
    q.pitch = pitch;
    q.tw = kBandWarps;
    q.cluster = 1;
    q.loader = kLoaderTma2d;
    q.units = 0;
    return true;
}

}  // namespace

cudaError_t encode_map_2d(CUtensorMap* out, CUtensorMapDataType dtype, const void* base, uint64_t dim0,
                          uint64_t dim1, uint64_t row_stride_bytes, uint32_t box0, uint32_t box1,
                          CUtensorMapSwizzle swizzle) {
    EncodeTiledFn enc = encode_tiled();
    if (!enc) return cudaErrorNotSupported;
    const cuuint64_t dims[2] = {(cuuint64_t)dim0, (cuuint64_t)dim1};
    const cuuint64_t strides[1] = {(cuuint64_t)row_stride_bytes};
    const cuuint32_t box[2] = {box0, box1};
    const cuuint32_t estr[2] = {1, 1};
    const CUresult r = enc(out, dtype, 2, const_cast<void*>(base), dims, strides, box, estr,
                           CU_TENSOR_MAP_INTERLEAVE_NONE, swizzle, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                           CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    return r == CUDA_SUCCESS ? cudaSuccess : cudaErrorInvalidValue;
}

cudaError_t set_max_dynamic_smem(const void* fn) {
    int dev = 0, optin = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e == cudaSuccess) e = cudaDeviceGetAttribute(&optin, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev);
    cudaFuncAttributes fa;
    if (e == cudaSuccess) e = cudaFuncGetAttributes(&fa, fn);
    if (e != cudaSuccess) return e;
    return cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, optin - (int)fa.sharedSizeBytes);
}

cudaError_t ensure_dynamic_smem(const void* fn, size_t bytes) {
    static std::mutex mu;
    static std::map<std::pair<int, const void*>, bool> done;
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return e;
    std::lock_guard<std::mutex> lock(mu);
    bool& d = done[{dev, fn}];
    if (!d) {
        e = set_max_dynamic_smem(fn);
        if (e != cudaSuccess) return e;
        d = true;
    }
    (void)bytes;  // larger than the device allows: the launch reports it
    return cudaSuccess;
}

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
    q.loader = (q.row_bytes % 16 == 0)                 ? kLoaderTma2d
               : (q.row_bytes % 16 == 8 && N % 2 == 0) ? kLoaderTmaPairs
                                                       : kLoaderCpAsync;
    if (q.loader != kLoaderCpAsync) {
        // chunks of 8 blocks (16-byte aligned starts); the stage pitch is made
        // bank friendly: Tma2d by the chunk size (8 blocks for Q8_0/Q4_0), the
        // paired loader by the pad after the chunk (16 or 32 bytes)
        q.kc = 8;
        if (q.loader == kLoaderTmaPairs) {
            q.pitch = q.kc * bb + 16;
            if (!bank_friendly(q.pitch)) q.pitch += 16;
        } else {
            q.pitch = q.kc * bb;
        }
    } else {
        const int kc_max = 8;
        q.kc = kc_max;
        q.pitch = (int)(((size_t)q.kc * bb + 30 + 15) / 16 * 16);
    }
    if (resident_plan(q, num_sms)) {
        *p = q;
        return true;
    }
    {
        GemvPlan b = q;
        if (band_plan(b, num_sms)) {
            *p = b;
            return true;
        }
    }
    q.kind = kGemvStreaming;
    // Shared memory and L1 share one array per SM. The activation fragments are
    // read through L1 by every warp, so leave room for them when they fit
    // (measured: a deeper ring that starves L1 costs up to 40%); then take the
    // most warps (two CTAs per SM), then the deepest ring that fits.
    auto smem_for = [&](int sw) { return (size_t)kW * sw * kRows * q.pitch + (size_t)kW * sw * sizeof(uint64_t); };
    const size_t x_bytes = (size_t)q.nb * ((size_t)M * (native ? 32 : 128) + (size_t)token_pad(M) * 16);
    const size_t l1_keep = x_bytes <= 96 * 1024 ? x_bytes : 32 * 1024;
    const size_t budget = kSmemPerSM - l1_keep - 8 * 1024;
    int ctas_per_sm = 0;
    q.sw = 2;
    for (int cps = 2; cps >= 1 && !ctas_per_sm; --cps) {
        for (int sw = kMaxSW; sw >= 2; --sw) {
            if ((smem_for(sw) + 1024) * cps <= budget) {
                ctas_per_sm = cps;
                q.sw = sw;
                break;
            }
        }
    }
    if (!ctas_per_sm) ctas_per_sm = 1;  // a 2-stage ring always fits the hardware limit
    q.smem = smem_for(q.sw);
    const int slots = num_sms * ctas_per_sm * kW;
    // Split K across warps when there are fewer tiles than warp slots (the
    // Q8_0-activation mode keeps whole rows per warp: that is what makes its
    // results bit-identical to the reference's block-order sums).
    int want = 1;
    if (!native && tiles < slots) want = slots / tiles;
    const int granules = (q.nb + q.kc - 1) / q.kc;  // whole chunks per split
    int ks = want < granules ? want : granules;
    if (ks < 1) ks = 1;
    q.nbu = q.kc * ((granules + ks - 1) / ks);
    q.ks = (q.nb + q.nbu - 1) / q.nbu;
    q.units = tiles * q.ks;
    // units are dealt to CTAs first, so use every SM when there are enough
    const int max_ctas = num_sms * ctas_per_sm;
    q.grid = q.units < max_ctas ? q.units : max_ctas;
    q.weights_immutable = false;
    *p = q;
    return true;
}

size_t gemv_workspace_bytes(const GemvPlan& p) {
    if (p.kind == kGemvResident) return 0;  // everything lives in shared memory
    if (p.kind == kGemvBand)  // slice partials and tickets when K is split
        return p.ks > 1 ? align256((size_t)p.ks * p.M * p.N * sizeof(float)) +
                              align256((size_t)((p.N + kRows - 1) / kRows) * sizeof(unsigned))
                        : 0;
    const size_t Mpad = (size_t)token_pad(p.M);
    size_t s = align256((size_t)p.nb * p.M * (p.native ? 32 : 128));
    s += align256((size_t)p.nb * Mpad * 16);  // side records: (Mpad/2) x 32 B per block
    if (p.ks > 1) {
        s += align256((size_t)p.ks * p.M * p.N * sizeof(float));
        s += align256((size_t)((p.N + kRows - 1) / kRows) * sizeof(unsigned));
    }
    return s;
}

void gemv_workspace_carve(const GemvPlan& p, void* base, GemvWorkspace* ws) {
    const size_t Mpad = (size_t)token_pad(p.M);
    uint8_t* c = static_cast<uint8_t*>(base);
    *ws = GemvWorkspace{};
    if (p.kind == kGemvResident) return;
    if (p.kind == kGemvBand) {
        if (p.ks > 1) {
            ws->partial = reinterpret_cast<float*>(c);
            ws->counters = reinterpret_cast<unsigned*>(c + align256((size_t)p.ks * p.M * p.N * sizeof(float)));
        }
        return;
    }
    ws->xa = c;
    c += align256((size_t)p.nb * p.M * (p.native ? 32 : 128));
    ws->side = reinterpret_cast<uint32_t*>(c);
    c += align256((size_t)p.nb * Mpad * 16);
    if (p.ks > 1) {
        ws->partial = reinterpret_cast<float*>(c);
        c += align256((size_t)p.ks * p.M * p.N * sizeof(float));
        ws->counters = reinterpret_cast<unsigned*>(c);
    }
}

cudaError_t launch_gemv(const GemvPlan& p, const uint8_t* w, const float* x, float* y, const GemvWorkspace& ws,
                        int* err, cudaStream_t st, bool no_host_alloc, const GatedOut& g) {
    cudaError_t e;
    if (p.kind == kGemvBand) {
        CUtensorMap tmap;
        e = no_host_alloc ? weight_tensor_map_uncached(w, p, &tmap) : weight_tensor_map(w, p, &tmap);
        if (e != cudaSuccess) return e;
        return launch_gemv_band(p, tmap, x, y, ws, err, st, no_host_alloc, g);
    }
    if (p.kind == kGemvResident) {
        CUtensorMap tmap;
        e = no_host_alloc ? weight_tensor_map_uncached(w, p, &tmap) : weight_tensor_map(w, p, &tmap);
        if (e != cudaSuccess) return e;
        return launch_gemv_resident(p, tmap, x, y, err, st, no_host_alloc, g);
    }
    const int nzero = ws.counters ? (p.N + kRows - 1) / kRows : 0;
    if (p.native) {
        e = launch_xprep_q8(p.qt, x, p.M, p.K, static_cast<uint8_t*>(ws.xa), ws.side, ws.counters, nzero, st);
    } else {
        e = launch_xprep_f32(p.qt, x, p.M, p.K, static_cast<__half*>(ws.xa), ws.side, ws.counters, nzero, st);
    }
    if (e != cudaSuccess) return e;
    const void* fn = kernel_for(p);
    // no_host_alloc: set the attribute and encode the tensor map on every call
    // instead of going through the (heap-backed) caches
    e = no_host_alloc ? set_max_dynamic_smem(fn) : ensure_dynamic_smem(fn, p.smem);
    if (e != cudaSuccess) return e;
    Args a;
    if (p.loader != kLoaderCpAsync) {
        e = no_host_alloc ? weight_tensor_map_uncached(w, p, &a.tmap) : weight_tensor_map(w, p, &a.tmap);
        if (e != cudaSuccess) return e;
    }
    a.weights_immutable = p.weights_immutable ? 1 : 0;
    a.sw = p.sw;
    a.w = w;
    a.w_bytes = (uint64_t)p.N * (uint64_t)p.row_bytes;
    a.y = y;
    a.xa = ws.xa;
    a.side = ws.side;
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
    a.gact = g.act;
    a.gout = g.out;
    a.ghidden = g.hidden;
    void* args[] = {(void*)&a};
    return launch_pdl_kernel(fn, dim3(p.grid), dim3(kThreads), p.smem, st, args);
}

}  // namespace qmm
