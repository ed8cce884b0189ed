// Internal launch interface between the C-ABI layer (qmm_api.cu) and the
// kernels. Not installed; the public interface is include/qmm.h.
#pragma once

#include <cuda.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <cstdint>

namespace qmm {

// Rows of a gate/up weight are interleaved in groups of kGateGroup: fused
// rows [2G*j, 2G*j + G) are gate rows [G*j, G*j + G) and the next G rows the
// matching up rows, so every 32-row output tile holds whole pairs.
constexpr int kGateGroup = 16;

// Epilogue of a gate/up matmul: instead of y, out[m][i] = act(y[m][gate i]) *
// y[m][up i] for i < hidden (act 0 GELU, 1 SiLU). act < 0: plain y.
struct GatedOut {
    int act = -1;
    float* out = nullptr;
    int64_t hidden = 0;
};

// Output of a tensor-parallel join written from the producing kernel's own
// epilogue (qmm_tp.cu): while a request is set on the calling thread, a
// launcher that supports it (the band GEMV and the f16 GEMM, plain outputs)
// stores element (m, n) at dst[r] + b * pstride + m * ld + n for every rank r
// -- peer memory over NVLink, this rank's own buffer among them -- instead of
// y, and sets `taken`; b = (*epoch + 1) & 1 is the join's buffer, read on the
// device so that a captured step replays correctly. Other kernels write y
// and leave it unset.
constexpr int kMaxPeers = 8;
struct PeerOut {
    float* dst[kMaxPeers] = {};
    int n = 0;
    int64_t ld = 0;
    int64_t pstride = 0;
    const unsigned long long* epoch = nullptr;
    bool taken = false;
};
PeerOut* peer_out();  // this thread's request (null: none)
void set_peer_out(PeerOut* p);
// Kernel-side copy of a request (plain data for __grid_constant__ arguments).
struct PeerDst {
    float* dst[kMaxPeers];
    int n;
    int64_t ld;
    int64_t pstride;
    const unsigned long long* epoch;
};
// Element offset of the join's buffer (device side; the preceding join has
// completed before any epilogue runs: stream order / programmatic wait).
__device__ __forceinline__ int64_t peer_buffer_offset(const PeerDst& p) {
    return (int64_t)((__ldcg(p.epoch) + 1ull) & 1ull) * p.pstride;
}
// Takes this thread's request when the launch can honour it (row-contiguous
// [M][N] output, 16-byte aligned rows for vector stores): fills `out`, marks
// the request taken. Otherwise `out.n` = 0.
void take_peer_out(PeerDst& out, bool supported);

// ---- quantisers / dequantiser (qmm_quant.cu) -----------------------------------
cudaError_t launch_quantize_q8_0(const float* x, int64_t n, uint8_t* out, float* scales, bool rounded_inv,
                                 cudaStream_t st);
cudaError_t launch_quantize_q4_0(const float* x, int64_t n, uint8_t* out, cudaStream_t st);
cudaError_t launch_quantize_q4_1(const float* x, int64_t n, uint8_t* out, cudaStream_t st);
cudaError_t launch_dequantize(int qt, const uint8_t* w, int64_t n, float* out, cudaStream_t st);
// Adds the position-weighted checksum of [p, p + len) into *acc (p 4-byte aligned).
cudaError_t launch_checksum(const uint8_t* p, uint64_t len, unsigned long long* acc, cudaStream_t st);
// out[m][i] = act(gate[m*ld + i]) * up[m*ld + i] (up null: act alone);
// kind 0 = tanh GELU, 1 = SiLU, 2 = ReLU.
cudaError_t launch_gated_act(int kind, const float* gate, const float* up, int64_t m, int64_t hidden, int64_t ld,
                             float* out, cudaStream_t st);

// ---- decode-step pieces around the matmuls (qmm_decode.cu) ----------------------
cudaError_t launch_embed_q8(const uint8_t* emb, int hidden, const int* tokens, int batch, int vocab, float scale,
                            float* x, cudaStream_t st);
cudaError_t launch_rmsnorm(const float* x, const float* w, float offset, float eps, int rows, int dim, float* y, int ldy,
                           cudaStream_t st);
cudaError_t launch_residual_norm(float* x, const float* branch, const float* w_post, const float* w_next, float offset,
                                 float eps, int rows, int dim, float* h, int ldh, cudaStream_t st);
cudaError_t launch_qk_rope_cache(const float* qkv, int batch, int nq, int nkv, int hd, const float* qn_w,
                                 const float* kn_w, float offset, float eps, const float* cos_t, const float* sin_t,
                                 const int* pos_dev, int ctx, float* q_out, float* k_cache, float* v_cache,
                                 cudaStream_t st);
size_t attn_partial_floats(int batch, int nq, int hd, int ctx);
cudaError_t launch_attention(const float* q, const float* k_cache, const float* v_cache, int batch, int nq, int nkv,
                             int hd, const int* pos_dev, int ctx, float inv_scale, float* part, float* out,
                             cudaStream_t st);
cudaError_t launch_attention_fused(const float* qkv, int batch, int nq, int nkv, int hd, const float* qn_w,
                                   const float* kn_w, float offset, float eps, const float* cos_t, const float* sin_t,
                                   const int* pos_dev, int ctx, float* k_cache, float* v_cache, float inv_scale,
                                   float* part, float* out, cudaStream_t st);
cudaError_t launch_add_int(int* p, int v, cudaStream_t st);

// ---- GEMV activation preparation (qmm_quant.cu) ----------------------------------
// f32 mode:   xf [nb][M][4][16 halves];  native: xq [nb][M][4][8 bytes]
// both:       side [nb][token_pad(M)/2][8 words] (see the kernels)
// Both also zero `nzero` words at `zero` (the GEMV's split-K tickets).
cudaError_t launch_xprep_f32(int qt, const float* x, int M, int K, __half* xf, uint32_t* side, unsigned* zero,
                             int nzero, cudaStream_t st);
cudaError_t launch_xprep_q8(int qt, const float* x, int M, int K, uint8_t* xq, uint32_t* side, unsigned* zero,
                           int nzero, cudaStream_t st);
cudaError_t launch_pdl_kernel(const void* fn, dim3 grid, dim3 block, size_t smem, cudaStream_t st, void** args);

// ---- GEMV (qmm_gemv.cu, qmm_gemv_resident.cu) --------------------------------------
// kGemvStreaming: x-prep kernel, then a persistent GEMV streaming weight tiles
//                 through per-warp shared-memory rings (any shape, M <= 64).
// kGemvResident:  one kernel per call for small decode shapes: every CTA loads
//                 its whole share of the weights into shared memory, prepares
//                 the activations itself, and K splits are summed on chip
//                 (warps through shared memory, cluster CTAs through DSMEM).
// kGemvBand:      decode shapes (M <= 8, f32 activations) too large to keep on
//                 chip: each CTA owns a K slice of a run of 32-row tiles with
//                 its activations prepared in shared memory, streams the
//                 weights through a deep ring of wide TMA boxes, and slices are
//                 summed in slice order by the last to finish (qmm_gemv_band.cu).
enum GemvKind : int { kGemvStreaming = 0, kGemvResident = 1, kGemvBand = 2 };

struct GemvPlan {
    int kind;        // GemvKind
    int qt;          // kQ4_0 / kQ4_1 / kQ8_0
    bool native;     // Q8_0-quantised activations (int8 MMA) instead of f32 activations
    int M, N, K;     // y[M,N] = x[M,K] . W[N,K]^T
    int nb;          // K / 32
    int row_bytes;   // nb * block bytes
    int nt;          // token tiles of 8 (1, 2, 4 or 8)
    int ks;          // streaming: K splits per 32-row tile
    int nbu;         // streaming: blocks per K split
    int kc;          // blocks per pipeline stage / TMA box
    int pitch;       // shared-memory bytes per row slot of a stage
    int loader;      // 0: 2-D TMA tile; 1: cp.async windows; 2: paired-row 2-D TMA tiles
    int sw;          // streaming: shared-memory stages per warp
    int units;       // streaming: tiles * ks
    int cluster;     // resident: CTAs per thread-block cluster (they split K)
    int tw;          // resident: 32-row tiles per cluster
    int gpc;         // resident: 8-block granules of K per CTA
    int grid;        // CTAs
    size_t smem;     // dynamic shared memory per CTA
    bool weights_immutable;  // weights are not written by earlier work in the stream:
                             // the GEMV may start fetching them before its dependency wait
};

// Shared-memory layout of the resident kernel (byte offsets), used by the
// planner and the kernel alike. M <= 16 tokens, padded to mp = 8 or 16.
struct ResidentLayout {
    uint32_t stages, xf, side, part, cpart, bar, total;
};
__host__ __device__ inline ResidentLayout resident_layout(int tw, int gpc, int pitch, int M) {
    const uint32_t mp = M <= 8 ? 8u : 16u;
    const uint32_t blocks = (uint32_t)gpc * 8u;
    ResidentLayout L;
    uint32_t o = 0;
    L.stages = o;  // [tw][gpc] stages of 32 rows x pitch
    o += (uint32_t)tw * (uint32_t)gpc * 32u * (uint32_t)pitch;
    o = (o + 127u) & ~127u;
    L.xf = o;  // hi plane [blocks][M][4] x 16 B, then the lo plane
    o += blocks * (uint32_t)M * 128u;
    L.side = o;  // [blocks][mp / 2] x 32 B side records
    o += blocks * (mp / 2u) * 32u;
    L.part = o;  // [8 warps][mp / 8][32 rows][8 tokens] f32 warp partials
    o += 8u * mp * 32u * 4u;
    L.cpart = o;  // [tw][mp][32 rows] f32 CTA partials (read by the cluster)
    o += (uint32_t)tw * mp * 32u * 4u;
    L.bar = o;  // one mbarrier
    o += 16u;
    L.total = o;
    return L;
}

// Band kernel geometry: consumer warps per CTA and blocks per warp per chunk
// (even: payload alignment then follows the block index); a chunk (one TMA
// box of 32 rows) is kBandWarps * band_bpw(qt) blocks: 48 Q4_0 / Q4_1 (880 /
// 976-byte rows), 24 Q8_0 (816-byte rows).
constexpr int kBandWarps = 12;
__host__ __device__ constexpr int band_bpw(int qt) { return qt == 8 ? 2 : 4; }
// Token capacity of the band kernel variant for M tokens (M <= 4).
__host__ __device__ constexpr int band_mt(int M) { return M <= 1 ? 1 : (M == 2 ? 2 : 4); }

// Shared-memory layout of the band kernel (byte offsets), host and device:
// S ring stages of 32 rows x pitch, activations of nbs blocks x M tokens
// (M: the variant's token capacity; side records for ceil(M / 2) token
// pairs), W consumer warps.
struct BandLayout {
    uint32_t ring, xf, side, part, bar, total;
};
__host__ __device__ inline BandLayout band_layout(int S, int pitch, int nbs, int M, int W) {
    BandLayout L;
    uint32_t o = 0;
    L.ring = o;  // [S][32 rows][pitch]
    o += (uint32_t)S * 32u * (uint32_t)pitch;
    o = (o + 127u) & ~127u;
    L.xf = o;  // hi plane [nbs][M][4] x 16 B, then the lo plane
    o += (uint32_t)nbs * (uint32_t)M * 128u;
    L.side = o;  // [nbs][ceil(M / 2) pairs] x 32 B
    o += (uint32_t)nbs * (uint32_t)((M + 1) / 2) * 32u;
    L.part = o;  // [2 slots][W warps][32 rows][8 tokens] f32
    o += 2u * (uint32_t)W * 32u * 8u * 4u;
    L.bar = o;  // full[S], empty[S], rfull[2], rempty[2]
    o += (uint32_t)(2 * S + 4) * 8u;
    L.total = o;
    return L;
}

// Fills a plan for the given problem on a device with `num_sms` SMs. Returns
// false if the shape is not handled by the GEMV kernel (M > 64).
bool gemv_plan(int qt, bool native, int M, int N, int K, int num_sms, GemvPlan* p);

// Workspace layout shared by the xprep and GEMV launches.
struct GemvWorkspace {
    void* xa;            // xf (f32 mode) or xq (native)
    uint32_t* side;      // per-(block, token pair) records
    float* partial;      // [ks][M][N] when ks > 1
    unsigned* counters;  // [tiles] when ks > 1; cleared by the xprep kernel of every call
};
size_t gemv_workspace_bytes(const GemvPlan& p);
// Carves `base` (256-byte aligned) into the pieces.
void gemv_workspace_carve(const GemvPlan& p, void* base, GemvWorkspace* ws);

// no_host_alloc: skip the host-side caches (for the allocation-free entry point).
// g: optional gate/up epilogue (y may then be null).
cudaError_t launch_gemv(const GemvPlan& p, const uint8_t* w, const float* x, float* y, const GemvWorkspace& ws,
                        int* err, cudaStream_t st, bool no_host_alloc = false, const GatedOut& g = GatedOut());

// The band kernel (launch_gemv dispatches kGemvBand plans to it; tmap: the
// weights with a [pitch / 4, 32] box), threads per CTA, and how many of its
// CTAs (the variant for M tokens) with `smem` bytes fit on the current device
// at once (0: unknown).
cudaError_t launch_gemv_band(const GemvPlan& p, const CUtensorMap& tmap, const float* x, float* y,
                             const GemvWorkspace& ws, int* err, cudaStream_t st, bool no_host_alloc,
                             const GatedOut& g);
int band_threads();
int band_capacity(int qt, int M, size_t smem);

// The resident kernel (launch_gemv dispatches to it for kGemvResident plans).
cudaError_t launch_gemv_resident(const GemvPlan& p, const CUtensorMap& tmap, const float* x, float* y, int* err,
                                 cudaStream_t st, bool no_host_alloc, const GatedOut& g);

// Activation-prep tasks ((block, token) pairs) a resident CTA handles per pass:
// 32 eight-lane groups x this many rounds, loads of a pass in flight together.
constexpr int kResidentPrepUnroll = 8;
// Largest cluster the resident-kernel planner uses (CTAs summed through DSMEM).
constexpr int kMaxResidentCluster = 8;

// How many resident-kernel clusters of `cluster` CTAs (CTAs, for cluster 1)
// with `smem` bytes of shared memory can be resident on the current device at
// once; 0 if the runtime cannot say. Cached per (device, kernel, cluster,
// smem) in a fixed table (no heap use).
int resident_capacity(int qt, int loader, int nt, int cluster, size_t smem);

// Opts a kernel in to dynamic shared memory on the current device: the limit
// is raised once to the device maximum and never lowered, so occupancy
// queries and launches with any size up to it cannot undo one another
// (ensure_dynamic_smem caches per device and kernel; set_max_dynamic_smem
// does the same without the cache's heap use).
cudaError_t ensure_dynamic_smem(const void* fn, size_t bytes);
cudaError_t set_max_dynamic_smem(const void* fn);

// A 2-D TMA tensor map (dim0 innermost, in elements; zero fill out of bounds).
cudaError_t encode_map_2d(CUtensorMap* out, CUtensorMapDataType dtype, const void* base, uint64_t dim0,
                          uint64_t dim1, uint64_t row_stride_bytes, uint32_t box0, uint32_t box1,
                          CUtensorMapSwizzle swizzle);

// ---- prefill GEMM (qmm_gemm.cu): tcgen05 tensor cores, f32 activations ------------------
// y[M,N] = x[M,K] . W[N,K]^T for f32-activation calls with M >= kGemmMinRows
// and a weight row pitch that is a multiple of 16 bytes.
constexpr int kGemmMinRows = 17;
bool gemm_supported(int qt, bool native, int M, int N, int K);
// x16 activations and scales, plus K-slice partials and tickets when the call's
// plan splits K (planned per device the same way at launch).
// native: Q8_0-quantised activations (the integer GEMM of qmm_gemm_i8.cu).
size_t gemm_workspace_bytes(int M, int N, int K, int qt, bool native = false);
// ws: gemm_workspace_bytes(M, N, K, qt, native) bytes, 256-byte aligned.
cudaError_t launch_gemm(int qt, const uint8_t* w, const float* x, float* y, int M, int N, int K, void* ws,
                        int* err, cudaStream_t st, bool weights_immutable, const GatedOut& g = GatedOut(),
                        bool native = false);

// ---- decode-batch GEMM (qmm_gemm_tn.cu): tcgen05, exact hi/lo split of both
// operands (~1e-6 relative). Capable of f32-activation calls with
// kGemmMinRows <= M <= kGemmTnMaxRows and a row pitch of 0 or 8 mod 16 bytes
// (N even for the latter); routed only the decode batches the f16 GEMM
// (qmm_gemm.cu) cannot take: 8-mod-16 pitches with odd N or more than 64
// tokens. The f16 GEMM takes every other call of up to kGemmSingleMaxRows
// tokens: exact activations (f16 hi and residual rows stacked in the token
// tile) and d*q rounded to f16 once, ~2e-4 norm-wise, at a fraction of the
// exact split's cost (Gemma decode batch 64 on B200: lm_head 418 -> 226 us,
// down 152 -> 39 us).
constexpr int kGemmTnMaxRows = 128;
constexpr int kGemmSingleMaxRows = 128;
bool gemm_tn_supported(int qt, bool native, int M, int N, int K);
size_t gemm_tn_workspace_bytes(int M, int N, int K, int qt);
cudaError_t launch_gemm_tn(int qt, const uint8_t* w, const float* x, float* y, int M, int N, int K, void* ws,
                           int* err, cudaStream_t st, bool weights_immutable, const GatedOut& g = GatedOut());

// ---- integer GEMM for the Q8_0-activation modes (qmm_gemm_i8.cu): tcgen05
// kind::i8, one MMA per 32-element block, the reference's per-block float
// sequence in the epilogue (bit-identical). M >= kGemmMinRows, row pitch 0
// or 8 mod 16 bytes (N even for the latter).
bool gemm_i8_supported(int qt, int M, int N, int K);
size_t gemm_i8_workspace_bytes(int M, int N, int K, int qt);
cudaError_t launch_gemm_i8(int qt, const uint8_t* w, const float* x, float* y, int M, int N, int K, void* ws,
                           int* err, cudaStream_t st, bool weights_immutable);
// Activation prep of the integer GEMM (qmm_quant.cu): xq [M][K] s8, xs / xc
// [nbp][Mp] (see the kernel).
cudaError_t launch_xprep_i8gemm(int qt, const float* x, int M, int K, int Mp, int8_t* xq, float* xs, uint32_t* xc,
                                cudaStream_t st);

int* device_error_word(int device);

// Launch accounting (qmm_launch_count): every launch site calls note_launch().
void note_launch();

}  // namespace qmm
