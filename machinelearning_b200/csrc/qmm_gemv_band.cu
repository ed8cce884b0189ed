// Band GEMV: decode shapes (f32 activations, M <= 8) whose weights are too
// large for the resident kernel (tens of MB to GB: Llama-70B projections,
// vocabulary heads). Bandwidth-bound; the layout is built for HBM streaming:
//   * the K blocks are cut into ks slices; CTA c works on slice c % ks of the
//     32-row tiles c / ks, c / ks + grid / ks, ..., so its activations are
//     prepared once, in shared memory, for the whole launch.
//   * warp 0 streams the slice of each tile through an S-stage shared-memory
//     ring in chunks of kc blocks, one 2-D TMA box of 32 rows per stage (one
//     bulk-tensor operation per ~18-32 KB: per-row copies cap the ring far
//     below HBM bandwidth). The box is up to 16 bytes wider than the chunk so
//     the row pitch in shared memory is 4 mod 8 words (conflict-free reads);
//     the extra bytes belong to the next chunk and come from L2.
//   * W consumer warps split every chunk by blocks (dequantisation and MMAs
//     are consume_group() from qmm_gemv_frag.cuh, as in the other GEMVs) and
//     keep their 32-row partial tile in registers until the slice is done;
//     they hand it to the reducer warp through a double-buffered slot.
//   * the reducer warp sums the W partials in warp order. With ks == 1 it
//     stores the tile; otherwise it writes the slice's partial tile to global
//     memory and the last slice to arrive (a ticket per tile) adds the ks
//     partials in slice order and stores. Results are deterministic.
// Every wait is bounded (the error word records a timeout); a CTA leaves only
// after the copies it issued have landed.
#include <cuda.h>

#include <mutex>
#include <type_traits>

#include "qmm_common.cuh"
#include "qmm_gemv_frag.cuh"
#include "qmm_gemv_xsmem.cuh"
#include "qmm_kernels.cuh"

namespace qmm {

namespace {

struct BArgs {
    CUtensorMap tmap;  // weights as uint32 [N][row_bytes / 4], box [pitch / 4, 32]
    const float* x;
    float* y;
    float* partial;      // [ks][M][N] (ks > 1)
    unsigned* counters;  // [tiles], zero on entry (ks > 1); left zero
    int M, N, K, nb;
    int ks;     // K slices
    int nbs;    // blocks per slice (the last slice may be shorter)
    int kc;     // blocks per chunk
    int pitch;  // shared-memory row pitch of a stage (= box width in bytes)
    int S;      // ring stages
    int tiles;  // ceil(N / 32)
    int weights_immutable;
    int* err;
    int gact;  // >= 0: gate/up epilogue (GatedOut), y unused
    float* gout;
    int64_t ghidden;
    PeerDst peer;  // n > 0: the outputs go to every rank's join buffer instead of y
};

template <int W>
struct BandThreads {
    static constexpr int kConsumers = 32 * W;
    static constexpr int kTotal = 32 * (W + 2);  // producer, consumers, reducer
};

// Blocks JB..BPW-1 of a consumer warp's share of a chunk (compile-time
// offsets: every shared load is [register + immediate]).
struct BandLane {
    uint32_t rg, rg8, rg16, rg24;      // rows g, g+8, g+16, g+24 at the warp's first block
    uint32_t rgt, rg8t, rg16t, rg24t;  // the same plus the lane's payload word
    uint32_t xa;                       // the lane's activation record (column g) at that block
    uint32_t sa;                       // the lane's token terms at that block
};
template <int QT, int MT, int BPW, int JB>
__device__ __forceinline__ void band_blocks(const BandLane& l, bool xvalid, float (&acc)[2][2]) {
    if constexpr (JB < BPW) {
        constexpr int BB = block_bytes(QT);
        constexpr int NP = (MT + 1) / 2;
        constexpr int OFF = JB * BB, XO = JB * MT * 64, SO = JB * NP * 32;
        // chunks start 16-byte aligned and an even number of blocks into the
        // row: payloads of odd blocks are 4-byte aligned (Q8_0, Q4_0), Q4_1
        // payloads always are
        constexpr bool AL = QT == kQ4_1 || (JB & 1);
        uint4 xb = make_uint4(0, 0, 0, 0);
        lds128_at_if<XO>(xb, l.xa, xvalid);
        const float cs = __uint_as_float(lds32_at<SO>(l.sa));
        const float ss = __uint_as_float(lds32_at<SO + 16>(l.sa));
        const float sx = QT == kQ4_1 ? __uint_as_float(lds32_at<SO + 24>(l.sa)) : 0.0f;
        consume_group_packed_sa<QT, AL, OFF>(l.rg, l.rg8, l.rgt, l.rg8t, xb, cs, ss, sx, acc[0]);
        consume_group_packed_sa<QT, AL, OFF>(l.rg16, l.rg24, l.rg16t, l.rg24t, xb, cs, ss, sx, acc[1]);
        band_blocks<QT, MT, BPW, JB + 1>(l, xvalid, acc);
    }
}

template <int QT, int MT>
__global__ void __launch_bounds__(BandThreads<kBandWarps>::kTotal, 1)
    gemv_band_kernel(const __grid_constant__ BArgs a) {
    constexpr int W = kBandWarps;
    constexpr int BPW = band_bpw(QT);  // blocks per consumer warp per chunk (even)
    constexpr int KC = W * BPW;         // blocks per chunk
    constexpr int NP = (MT + 1) / 2;    // token pairs of the side records
    extern __shared__ __align__(128) uint8_t smem[];
    constexpr int BB = block_bytes(QT);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const BandLayout L = band_layout(a.S, a.pitch, a.nbs, MT, W);
    uint64_t* bars = reinterpret_cast<uint64_t*>(smem + L.bar);
    uint64_t* full = bars;
    uint64_t* empty = bars + a.S;
    uint64_t* rfull = bars + 2 * a.S;
    uint64_t* rempty = rfull + 2;
    const int ks = a.ks;
    const int slice = (int)blockIdx.x % ks;
    const int tstep = (int)gridDim.x / ks;                 // CTAs per slice
    const int tfirst = (int)blockIdx.x / ks;
    const int kb0 = slice * a.nbs;                          // this CTA's first block
    const int nbc = max(0, min(a.nb - kb0, a.nbs));         // its blocks
    const int nch = (nbc + KC - 1) / KC;                    // chunks per tile
    const int ntile = a.tiles > tfirst ? (a.tiles - tfirst + tstep - 1) / tstep : 0;  // its tiles

    if (threadIdx.x == 0) {
        for (int i = 0; i < a.S; ++i) {
            mbar_init(&full[i], 1);
            mbar_init(&empty[i], W);
        }
        for (int i = 0; i < 2; ++i) {
            mbar_init(&rfull[i], W);
            mbar_init(&rempty[i], 1);
        }
        fence_mbar_init();
        prefetch_tmap(&a.tmap);
    }
    __syncthreads();
    pdl_launch_dependents();

    if (warp == 0) {
        // ---------------- producer: one 32-row box per stage ------------------------------
        if (lane == 0) {
            if (a.weights_immutable == 0) pdl_wait();
            const int total = ntile * nch;
            const uint32_t stage_bytes = 32u * (uint32_t)a.pitch;
            int i = 0;
            for (; i < total; ++i) {
                const int s = i % a.S;
                if (i >= a.S && !mbar_wait_bounded(&empty[s], ((i / a.S) - 1) & 1, a.err)) break;
                const int tile = tfirst + (i / nch) * tstep;
                const int cb0 = kb0 + (i % nch) * KC;
                // rows past N and columns past the row end are zero-filled and counted
                mbar_arrive_expect_tx(&full[s], stage_bytes);
                tma_load_2d(smem + L.ring + (uint32_t)s * stage_bytes, &a.tmap, cb0 * BB / 4, tile * 32, &full[s]);
            }
            // before the CTA may leave: every issued copy has landed
            for (int q = max(0, i - a.S); q < i; ++q) mbar_wait_bounded(&full[q % a.S], (q / a.S) & 1, nullptr);
        }
    } else if (warp <= W) {
        // ---------------- consumers ---------------------------------------------------------
        const int cw = warp - 1;
        const int ctid = threadIdx.x - 32;
        // activation records: zero first (tokens M..MT-1 and the blocks of a
        // chunk past the slice contribute exactly zero), then fill
        {
            uint4* z = reinterpret_cast<uint4*>(smem + L.xf);
            const int nz = (int)((L.part - L.xf) / 16);
            for (int i = ctid; i < nz; i += BandThreads<W>::kConsumers) z[i] = make_uint4(0, 0, 0, 0);
        }
        asm volatile("bar.sync 1, %0;" ::"r"(BandThreads<W>::kConsumers) : "memory");
        pdl_wait();  // x comes from the preceding work in the stream
        const uint32_t lo_plane = (uint32_t)a.nbs * MT * 64u;
        prep_x_smem<QT>(a.x, a.M, a.K, kb0, nbc, smem + L.xf, lo_plane, reinterpret_cast<uint32_t*>(smem + L.side), NP,
                        ctid, BandThreads<W>::kConsumers, MT);
        asm volatile("bar.sync 1, %0;" ::"r"(BandThreads<W>::kConsumers) : "memory");
        const int g = lane >> 2, t = lane & 3;
        // lane (g, t) supplies MMA column g (token g / 2, hi or lo half) and
        // receives token t (lanes past M read token M - 1's terms: not stored)
        const int tp = min(t, a.M - 1);
        const bool xvalid = g < 2 * a.M;
        const uint32_t xl = smem_u32(smem + L.xf) + ((uint32_t)((cw * BPW) * MT + (g >> 1)) * 4 + t) * 16 +
                            ((g & 1) ? lo_plane : 0u);
        const uint32_t sl = smem_u32(smem + L.side) + (((cw * BPW) * NP + (tp >> 1)) * 8 + (tp & 1)) * 4;
        const uint32_t ring0 = smem_u32(smem + L.ring) + (uint32_t)(g * a.pitch) + (uint32_t)(cw * BPW * BB);
        float* part = reinterpret_cast<float*>(smem + L.part);
        bool ok = true;
        int i = 0;  // chunks consumed
        for (int j = 0; j < ntile && ok; ++j) {
            float acc[2][2] = {{0.0f, 0.0f}, {0.0f, 0.0f}};  // [row group][rows g, g + 8] for token t
            for (int c = 0; c < nch; ++c, ++i) {
                const int s = i % a.S;
                if (!mbar_wait_bounded(&full[s], (i / a.S) & 1, a.err)) {
                    ok = false;
                    break;
                }
                BandLane l;
                l.rg = ring0 + (uint32_t)s * 32u * (uint32_t)a.pitch;
                l.rg8 = l.rg + 8u * (uint32_t)a.pitch;
                l.rg16 = l.rg + 16u * (uint32_t)a.pitch;
                l.rg24 = l.rg + 24u * (uint32_t)a.pitch;
                l.rgt = l.rg + 4u * t;
                l.rg8t = l.rg8 + 4u * t;
                l.rg16t = l.rg16 + 4u * t;
                l.rg24t = l.rg24 + 4u * t;
                l.xa = xl + (uint32_t)(c * KC) * MT * 64u;
                l.sa = sl + (uint32_t)(c * KC) * NP * 32u;
                band_blocks<QT, MT, BPW, 0>(l, xvalid, acc);
                __syncwarp();
                if (lane == 0) mbar_arrive(&empty[s]);
            }
            if (!ok) break;
            const int slot = j & 1;
            if (j >= 2 && !mbar_wait_bounded(&rempty[slot], ((j >> 1) - 1) & 1, a.err)) break;
            // lane (g, t): token t of rows g, g + 8, g + 16, g + 24
            float* pw = part + ((size_t)slot * W + cw) * 32 * 8;
#pragma unroll
            for (int r = 0; r < 2; ++r) {
                pw[(16 * r + g) * 8 + t] = acc[r][0];
                pw[(16 * r + g + 8) * 8 + t] = acc[r][1];
            }
            __syncwarp();
            if (lane == 0) mbar_arrive(&rfull[slot]);
        }
    } else {
        // ---------------- reducer: warp sums, slice sums, stores --------------------------------
        const float* part = reinterpret_cast<const float*>(smem + L.part);
        const bool gated = a.gact >= 0;
        const int row = lane;
        for (int j = 0; j < ntile; ++j) {
            const int slot = j & 1;
            const int tile = tfirst + j * tstep;
            const int n = tile * 32 + row;
            if (!mbar_wait_bounded(&rfull[slot], (j >> 1) & 1, a.err)) break;
            float v[8];
#pragma unroll
            for (int m = 0; m < 8; ++m) v[m] = 0.0f;
            for (int q = 0; q < W; ++q) {
                const float4* pp = reinterpret_cast<const float4*>(part + (((size_t)slot * W + q) * 32 + row) * 8);
                const float4 p0 = pp[0], p1 = pp[1];
                v[0] += p0.x;
                v[1] += p0.y;
                v[2] += p0.z;
                v[3] += p0.w;
                v[4] += p1.x;
                v[5] += p1.y;
                v[6] += p1.z;
                v[7] += p1.w;
            }
            __syncwarp();
            if (lane == 0) mbar_arrive(&rempty[slot]);
            if (ks > 1) {
                // this slice's partial tile to global memory; the last slice of
                // the tile to arrive adds all of them in slice order
#pragma unroll
                for (int m = 0; m < 8; ++m)
                    if (m < a.M && n < a.N) a.partial[((int64_t)slice * a.M + m) * a.N + n] = v[m];
                __threadfence();
                __syncwarp();
                unsigned ticket = 0;
                if (lane == 0) ticket = atomicAdd(&a.counters[tile], 1u);
                ticket = __shfl_sync(0xffffffffu, ticket, 0);
                if (ticket != (unsigned)(ks - 1)) continue;
                __threadfence();
#pragma unroll
                for (int m = 0; m < 8; ++m) {
                    float s = 0.0f;
                    if (m < a.M && n < a.N)
                        for (int q = 0; q < ks; ++q)
                            s += q == slice ? v[m] : __ldcg(a.partial + ((int64_t)q * a.M + m) * a.N + n);
                    v[m] = s;
                }
                if (lane == 0) a.counters[tile] = 0u;
            }
            if (gated) {
                // rows 0..15 are gate rows tile*16 + row, rows 16..31 the matching up rows
#pragma unroll
                for (int m = 0; m < 8; ++m) {
                    const float up = __shfl_down_sync(0xffffffffu, v[m], 16);
                    const int64_t gi = (int64_t)tile * kGateGroup + row;
                    if (m < a.M && row < kGateGroup && gi < a.ghidden)
                        a.gout[(int64_t)m * a.ghidden + gi] = gated_value(a.gact, v[m], up);
                }
            } else if (a.peer.n > 0) {
                // tensor-parallel join: the same row of every rank's buffer
                // (peer memory over NVLink), coalesced 128-byte warp stores
                const int64_t boff = peer_buffer_offset(a.peer);
#pragma unroll
                for (int r = 0; r < kMaxPeers; ++r)
                    if (r < a.peer.n) {
                        float* d = a.peer.dst[r] + boff;
#pragma unroll
                        for (int m = 0; m < 8; ++m)
                            if (m < a.M && n < a.N) d[(int64_t)m * a.peer.ld + n] = v[m];
                    }
            } else {
#pragma unroll
                for (int m = 0; m < 8; ++m)
                    if (m < a.M && n < a.N) a.y[(int64_t)m * a.N + n] = v[m];
            }
        }
    }
}

// One token (decode at batch 1); the kernel is written for up to 4 (MT), the
// planner routes M = 1 only (measured: no gain over the streaming kernel yet
// for 2 to 4 tokens).
template <int QT>
const void* band_kernel_m(int M) {
    (void)M;
    return (const void*)gemv_band_kernel<QT, 1>;
}

const void* band_kernel_for(int qt, int M) {
    if (qt == kQ8_0) return band_kernel_m<kQ8_0>(M);
    if (qt == kQ4_0) return band_kernel_m<kQ4_0>(M);
    return band_kernel_m<kQ4_1>(M);
}

}  // namespace

int band_threads() { return BandThreads<kBandWarps>::kTotal; }

int band_capacity(int qt, int M, size_t smem) {
    const void* fn = band_kernel_for(qt, M);
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess) return 0;
    struct Entry {
        int dev;
        const void* fn;
        size_t smem;
        int cap;
    };
    static std::mutex mu;
    static Entry cache[256];
    static int used = 0;
    std::lock_guard<std::mutex> lock(mu);
    for (int i = 0; i < used; ++i) {
        const Entry& e = cache[i];
        if (e.dev == dev && e.fn == fn && e.smem == smem) return e.cap;
    }
    int cap = 0;
    // raised directly (not through ensure_dynamic_smem's map): this query runs
    // inside the allocation-free entry point too, and its answer is cached here
    if (set_max_dynamic_smem(fn) == cudaSuccess) {
        int per_sm = 0, sms = 0;
        if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, fn, band_threads(), smem) == cudaSuccess &&
            cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev) == cudaSuccess)
            cap = per_sm * sms;
    }
    cudaGetLastError();  // a failed query must not surface as the next launch's error
    if (used < 256) cache[used++] = Entry{dev, fn, smem, cap};
    return cap;
}

cudaError_t launch_gemv_band(const GemvPlan& p, const CUtensorMap& tmap, const float* x, float* y,
                             const GemvWorkspace& ws, int* err, cudaStream_t st, bool no_host_alloc,
                             const GatedOut& g) {
    const void* fn = band_kernel_for(p.qt, p.M);
    cudaError_t e = no_host_alloc ? set_max_dynamic_smem(fn) : ensure_dynamic_smem(fn, p.smem);
    if (e != cudaSuccess) return e;
    const int tiles = (p.N + kRows - 1) / kRows;
    if (p.ks > 1) {
        // the tickets start from zero (the kernel leaves them zero again)
        e = cudaMemsetAsync(ws.counters, 0, (size_t)tiles * sizeof(unsigned), st);
        if (e != cudaSuccess) return e;
    }
    BArgs a;
    a.tmap = tmap;
    a.x = x;
    a.y = y;
    a.partial = ws.partial;
    a.counters = ws.counters;
    a.M = p.M;
    a.N = p.N;
    a.K = p.K;
    a.nb = p.nb;
    a.ks = p.ks;
    a.nbs = p.nbu;
    a.kc = p.kc;
    a.pitch = p.pitch;
    a.S = p.sw;
    a.tiles = tiles;
    a.weights_immutable = p.weights_immutable ? 1 : 0;
    a.err = err;
    a.gact = g.act;
    a.gout = g.out;
    a.ghidden = g.hidden;
    take_peer_out(a.peer, g.act < 0 && !no_host_alloc);
    void* args[] = {(void*)&a};
    return launch_pdl_kernel(fn, dim3(p.grid), dim3(band_threads()), p.smem, st, args);
}

}  // namespace qmm
