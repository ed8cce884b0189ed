// Resident small-shape GEMV (f32 activations, M <= 16) for sm_100a.
//
// Decode GEMVs with a few MB of weights (the Gemma-3-1B projections: 0.3 to
// 8.5 MB) are latency-bound: HBM delivers their weights in about a
// microsecond, while a separate activation-prep launch, activation loads at
// L2 latency and a split-K fix-up through global atomics each cost more. This
// kernel is one launch per call and keeps everything on chip:
//   * the grid is made of clusters of `cluster` CTAs; a cluster owns `tw`
//     consecutive 32-row tiles, and CTA rank r of the cluster owns the K
//     granules [r*gpc, (r+1)*gpc) of 8 blocks (TMA boxes start 16-byte aligned).
//   * thread 0 loads the CTA's whole weight share with 2-D TMA boxes onto one
//     mbarrier -- before the programmatic-dependency wait when the weights are
//     immutable, so the loads overlap the preceding kernel in the stream.
//   * after the wait the CTA splits its activation blocks into the f16 hi/lo
//     records the streaming path's x-prep kernel writes (qmm_quant.cu), here in
//     shared memory, with one 8-lane group per (block, token).
//   * each warp takes a contiguous block range of one tile (8 / tw warps per
//     tile) and writes its partial 32-row x 8-token tile to shared memory; the
//     CTA sums the warp partials in warp order, and for cluster > 1 the CTAs
//     sum the cluster's partials in rank order through distributed shared
//     memory. No global workspace and no atomics: results are deterministic.
// The per-block arithmetic (dequantisation, MMA, scales) is consume_group()
// from qmm_gemv_frag.cuh, shared with the streaming kernel.
#include <cuda.h>

#include <mutex>
#include <type_traits>

#include "qmm_common.cuh"
#include "qmm_gemv_frag.cuh"
#include "qmm_gemv_xsmem.cuh"
#include "qmm_kernels.cuh"

namespace qmm {

namespace {

struct RArgs {
    CUtensorMap tmap;  // weights as in the streaming kernel (same box)
    const float* x;
    float* y;
    int M, N, K, nb, row_bytes, pitch, cluster, tw, gpc, weights_immutable;
    int* err;
    int gact;        // >= 0: gate/up epilogue (GatedOut), y unused
    float* gout;     // [M][ghidden]
    int64_t ghidden;
};

template <int QT, int NT, int LOADER>
__global__ void __launch_bounds__(kThreads, 2) gemv_resident_kernel(const __grid_constant__ RArgs a) {
    extern __shared__ __align__(128) uint8_t smem[];
    constexpr int BB = block_bytes(QT);
    constexpr int MP = 8 * NT;  // tokens padded to the MMA tiles
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const ResidentLayout L = resident_layout(a.tw, a.gpc, a.pitch, a.M);
    uint64_t* bar = reinterpret_cast<uint64_t*>(smem + L.bar);
    const int rank = (int)cluster_ctarank();
    const int tile0 = (int)cluster_id_x() * a.tw;
    const int G = (a.nb + kChunk - 1) / kChunk;
    const int g0 = rank * a.gpc;
    const int ng = max(0, min(a.gpc, G - g0));           // granules held by this CTA
    const int kb0 = g0 * kChunk;                          // its first block
    const int nbc = max(0, min(a.nb - kb0, ng * kChunk));  // its blocks
    const int ntl = min(a.tw, (a.N + kRows - 1) / kRows - tile0);  // its tiles (>= 1)

    if (threadIdx.x == 0) {
        mbar_init(bar, 1);
        fence_mbar_init();
        prefetch_tmap(&a.tmap);
    }
    __syncthreads();
    pdl_launch_dependents();

    // Rows past N and columns past the row end are zero-filled by TMA and
    // still counted as transaction bytes.
    auto issue = [&]() {
        if (threadIdx.x != 0 || ng == 0) return;
        mbar_arrive_expect_tx(bar, (uint32_t)(ntl * ng * kRows * a.pitch));
        for (int tl = 0; tl < ntl; ++tl) {
            const int tile = tile0 + tl;
            for (int gi = 0; gi < ng; ++gi) {
                uint8_t* st = smem + L.stages + (uint32_t)(tl * a.gpc + gi) * kRows * a.pitch;
                const int kb = kb0 + gi * kChunk;
                if constexpr (LOADER == kLoaderTmaPairs) {
                    tma_load_2d(st, &a.tmap, kb * BB / 4, tile * (kRows / 2), bar);
                    tma_load_2d(st + (kRows / 2) * a.pitch, &a.tmap, (a.row_bytes + kb * BB - 8) / 4,
                                tile * (kRows / 2), bar);
                } else {
                    tma_load_2d(st, &a.tmap, kb * BB / 4, tile * kRows, bar);
                }
            }
        }
    };
    if (a.weights_immutable) issue();
    pdl_wait();  // x (and mutable weights) come from preceding work in the stream
    if (!a.weights_immutable) issue();

    // ---- activation records for blocks [kb0, kb0 + nbc) -----------------------------
    // Per (block, token): scale by 2^-e so max|x| lands in [2^13, 2^14), split
    // into hi = f16(x') and lo = f16(x' - hi); corr is the magic-number bias
    // the MMA adds, s = 2^e, sx = block sum (Q4_1). Layout and element order
    // as written by xprep_f32_kernel.
    const uint32_t lo_plane = (uint32_t)a.gpc * kChunk * a.M * 64;  // bytes from the hi to the lo plane
    prep_x_smem<QT>(a.x, a.M, a.K, kb0, nbc, smem + L.xf, lo_plane, reinterpret_cast<uint32_t*>(smem + L.side),
                    MP / 2, threadIdx.x, kThreads);
    __syncthreads();
    bool ok = true;
    if (ng > 0) {
        ok = mbar_wait_bounded(bar, 0, a.err);
        // gave up (error word set): let the copies land before the CTA moves on
        if (!ok) mbar_wait_bounded(bar, 0, nullptr);
    }

    // ---- per-warp partial tiles ---------------------------------------------------------
    const int wpt = kW / a.tw;  // warps per tile
    const int tl = warp / wpt, sub = warp % wpt;
    const int g = lane >> 2, t = lane & 3;
    float acc[2][NT][4];
#pragma unroll
    for (int r = 0; r < 2; ++r)
#pragma unroll
        for (int nt = 0; nt < NT; ++nt) acc[r][nt][0] = acc[r][nt][1] = acc[r][nt][2] = acc[r][nt][3] = 0.0f;
    if (ok && tl < ntl) {
        const int b_begin = nbc * sub / wpt, b_end = nbc * (sub + 1) / wpt;
        const uint8_t* xfb = smem + L.xf;
        const uint4* sd = reinterpret_cast<const uint4*>(smem + L.side);
        const uint8_t* tbase = smem + L.stages + (uint32_t)(tl * a.gpc) * kRows * a.pitch;
        // one block: activation fragments from the hi/lo planes (16 bytes per
        // lane, consecutive lanes consecutive records: no bank conflicts), then
        // both 16-row groups with the short MMA chains
        auto block = [&](int b, auto aligned) {
            constexpr bool AL = decltype(aligned)::value;
            XFrag xr[NT];
#pragma unroll
            for (int nt = 0; nt < NT; ++nt) {
                const int m = nt * 8 + g;
                if (m < a.M) {
                    const uint8_t* p = xfb + ((uint32_t)(b * a.M + m) * 4 + t) * 16;
                    xr[nt].hi = *reinterpret_cast<const uint4*>(p);
                    xr[nt].lo = *reinterpret_cast<const uint4*>(p + lo_plane);
                } else {
                    xr[nt].hi = make_uint4(0, 0, 0, 0);
                    xr[nt].lo = make_uint4(0, 0, 0, 0);
                }
                xr[nt].c4 = sd[(b * (MP / 2) + nt * 4 + t) * 2];
                xr[nt].s4 = sd[(b * (MP / 2) + nt * 4 + t) * 2 + 1];
            }
            const uint8_t* sbase = tbase + (uint32_t)(b >> 3) * kRows * a.pitch;
            const uint32_t o = (uint32_t)(b & 7) * BB;
            consume_group<QT, NT, false, AL, true>(stage_row<LOADER>(sbase, g, a.pitch) + o,
                                                   stage_row<LOADER>(sbase, g + 8, a.pitch) + o, t, xr, acc[0]);
            consume_group<QT, NT, false, AL, true>(stage_row<LOADER>(sbase, g + 16, a.pitch) + o,
                                                   stage_row<LOADER>(sbase, g + 24, a.pitch) + o, t, xr, acc[1]);
        };
        // payloads of odd blocks in a 16-byte aligned box are 4-byte aligned
        // (Q8_0, Q4_0); Q4_1 payloads always are. Blocks go in (even, odd)
        // pairs so both alignments are static and the two blocks interleave.
        using EvenAl = std::integral_constant<bool, QT == kQ4_1>;
        using OddAl = std::true_type;
        int b = b_begin;
        if (b < b_end && (b & 1)) block(b++, OddAl{});
        for (; b + 1 < b_end; b += 2) {
            block(b, EvenAl{});
            block(b + 1, OddAl{});
        }
        if (b < b_end) block(b, EvenAl{});
    }
    float* part = reinterpret_cast<float*>(smem + L.part);  // [kW][NT][32 rows][8 tokens]
#pragma unroll
    for (int r = 0; r < 2; ++r) {
#pragma unroll
        for (int nt = 0; nt < NT; ++nt) {
            float* p0 = part + ((warp * NT + nt) * kRows + 16 * r + g) * 8 + 2 * t;
            *reinterpret_cast<float2*>(p0) = make_float2(acc[r][nt][0], acc[r][nt][1]);
            *reinterpret_cast<float2*>(p0 + 64) = make_float2(acc[r][nt][2], acc[r][nt][3]);  // row + 8
        }
    }
    __syncthreads();

    // ---- CTA sums (warp order), then cluster sums (rank order) -------------------------
    // A gate/up weight (a.gact >= 0) holds gate rows in the first kGateGroup
    // rows of each tile and the matching up rows in the rest: one thread sums
    // both and writes act(gate) * up.
    float* cpart = reinterpret_cast<float*>(smem + L.cpart);  // [tw][MP][32 rows]
    const bool gated = a.gact >= 0;
    const int orows = gated ? kGateGroup : kRows;
    const int nout = ntl * a.M * orows;  // row fastest: coalesced stores of y
    auto store = [&](int tl2, int m, int row, float s, float su) {
        if (gated) {
            const int64_t i = (int64_t)(tile0 + tl2) * kGateGroup + row;
            if (i < a.ghidden) a.gout[(int64_t)m * a.ghidden + i] = gated_value(a.gact, s, su);
        } else {
            const int n = (tile0 + tl2) * kRows + row;
            if (n < a.N) a.y[(int64_t)m * a.N + n] = s;
        }
    };
    const int osh = gated ? 4 : 5;  // log2(orows)
    for (int o = threadIdx.x; o < nout; o += kThreads) {
        const int row = o & (orows - 1), mt = o >> osh;
        const int tl2 = mt / a.M, m = mt - tl2 * a.M;
        // the warps' partials: all loads first, then the sum in warp order
        const float* pp = part + ((tl2 * wpt * NT + (m >> 3)) * kRows + row) * 8 + (m & 7);
        float pv[kW], pu[kW];
#pragma unroll
        for (int q = 0; q < kW; ++q) {
            pv[q] = q < wpt ? pp[q * NT * kRows * 8] : 0.0f;
            pu[q] = (gated && q < wpt) ? pp[q * NT * kRows * 8 + kGateGroup * 8] : 0.0f;
        }
        float s = 0.0f, su = 0.0f;
#pragma unroll
        for (int q = 0; q < kW; ++q) {
            if (q < wpt) {
                s += pv[q];
                su += pu[q];
            }
        }
        if (a.cluster == 1) {
            store(tl2, m, row, s, su);
        } else {
            cpart[(tl2 * MP + m) * kRows + row] = s;
            if (gated) cpart[(tl2 * MP + m) * kRows + row + kGateGroup] = su;
        }
    }
    if (a.cluster > 1) {
        cluster_sync();
        for (int o = rank * kThreads + threadIdx.x; o < nout; o += a.cluster * kThreads) {
            const int row = o & (orows - 1), mt = o >> osh;
            const int tl2 = mt / a.M, m = mt - tl2 * a.M;
            const float* src = cpart + (tl2 * MP + m) * kRows + row;
            // the cluster's partials (at most kMaxResidentCluster): all remote
            // loads in flight together, then the sum in rank order
            float cv[kMaxResidentCluster], cu[kMaxResidentCluster];
#pragma unroll
            for (int q = 0; q < kMaxResidentCluster; ++q) {
                cv[q] = q < a.cluster ? ld_cluster_f32(src, (uint32_t)q) : 0.0f;
                cu[q] = (gated && q < a.cluster) ? ld_cluster_f32(src + kGateGroup, (uint32_t)q) : 0.0f;
            }
            float s = 0.0f, su = 0.0f;
#pragma unroll
            for (int q = 0; q < kMaxResidentCluster; ++q) {
                if (q < a.cluster) {
                    s += cv[q];
                    su += cu[q];
                }
            }
            store(tl2, m, row, s, su);
        }
        cluster_sync();  // no CTA leaves while its partials may still be read
    }
}

template <int QT, int LOADER>
const void* pick_nt(int nt) {
    return nt == 1 ? (const void*)gemv_resident_kernel<QT, 1, LOADER> : (const void*)gemv_resident_kernel<QT, 2, LOADER>;
}

template <int QT>
const void* pick_loader(int loader, int nt) {
    return loader == kLoaderTmaPairs ? pick_nt<QT, kLoaderTmaPairs>(nt) : pick_nt<QT, kLoaderTma2d>(nt);
}

const void* resident_kernel_for(const GemvPlan& p) {
    if (p.qt == kQ8_0) return pick_loader<kQ8_0>(p.loader, p.nt);
    if (p.qt == kQ4_0) return pick_loader<kQ4_0>(p.loader, p.nt);
    return pick_loader<kQ4_1>(p.loader, p.nt);
}

}  // namespace

int resident_capacity(int qt, int loader, int nt, int cluster, size_t smem) {
    GemvPlan p = {};
    p.qt = qt;
    p.loader = loader;
    p.nt = nt;
    const void* fn = resident_kernel_for(p);
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess) return 0;
    struct Entry {
        int dev;
        const void* fn;
        int cluster;
        size_t smem;
        int cap;
    };
    static std::mutex mu;
    static Entry cache[256];
    static int used = 0;
    std::lock_guard<std::mutex> lock(mu);
    for (int i = 0; i < used; ++i) {
        const Entry& e = cache[i];
        if (e.dev == dev && e.fn == fn && e.cluster == cluster && e.smem == smem) return e.cap;
    }
    int cap = 0;
    // raised directly (not through ensure_dynamic_smem's map): this query runs
    // inside the allocation-free entry point too, and its answer is cached here
    if (set_max_dynamic_smem(fn) == cudaSuccess) {
        if (cluster == 1) {
            int per_sm = 0, sms = 0;
            if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, fn, kThreads, smem) == cudaSuccess &&
                cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev) == cudaSuccess)
                cap = per_sm * sms;
        } else {
            cudaLaunchConfig_t cfg = {};
            cfg.gridDim = dim3(cluster * 32);
            cfg.blockDim = dim3(kThreads);
            cfg.dynamicSmemBytes = smem;
            cudaLaunchAttribute attr[1];
            attr[0].id = cudaLaunchAttributeClusterDimension;
            attr[0].val.clusterDim.x = (unsigned)cluster;
            attr[0].val.clusterDim.y = 1;
            attr[0].val.clusterDim.z = 1;
            cfg.attrs = attr;
            cfg.numAttrs = 1;
            if (cudaOccupancyMaxActiveClusters(&cap, fn, &cfg) != cudaSuccess) cap = 0;
        }
    }
    cudaGetLastError();  // a failed query must not surface as the next launch's error
    if (used < 256) cache[used++] = Entry{dev, fn, cluster, smem, cap};
    return cap;
}

cudaError_t launch_gemv_resident(const GemvPlan& p, const CUtensorMap& tmap, const float* x, float* y, int* err,
                                 cudaStream_t st, bool no_host_alloc, const GatedOut& g) {
    if (p.native || p.nt > 2 || p.loader == kLoaderCpAsync) return cudaErrorInvalidValue;
    const void* fn = resident_kernel_for(p);
    cudaError_t e = no_host_alloc ? set_max_dynamic_smem(fn) : ensure_dynamic_smem(fn, p.smem);
    if (e != cudaSuccess) return e;
    RArgs a;
    a.tmap = tmap;
    a.x = x;
    a.y = y;
    a.M = p.M;
    a.N = p.N;
    a.K = p.K;
    a.nb = p.nb;
    a.row_bytes = p.row_bytes;
    a.pitch = p.pitch;
    a.cluster = p.cluster;
    a.tw = p.tw;
    a.gpc = p.gpc;
    a.weights_immutable = p.weights_immutable ? 1 : 0;
    a.err = err;
    a.gact = g.act;
    a.gout = g.out;
    a.ghidden = g.hidden;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(p.grid);
    cfg.blockDim = dim3(kThreads);
    cfg.dynamicSmemBytes = p.smem;
    cfg.stream = st;
    cudaLaunchAttribute attr[2];
    int na = 0;
    attr[na].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[na].val.programmaticStreamSerializationAllowed = 1;
    ++na;
    if (p.cluster > 1) {
        attr[na].id = cudaLaunchAttributeClusterDimension;
        attr[na].val.clusterDim.x = (unsigned)p.cluster;
        attr[na].val.clusterDim.y = 1;
        attr[na].val.clusterDim.z = 1;
        ++na;
    }
    cfg.attrs = attr;
    cfg.numAttrs = na;
    void* args[] = {(void*)&a};
    note_launch();
    return cudaLaunchKernelExC(&cfg, fn, args);
}

}  // namespace qmm
