// Internal launch interface between the C-ABI layer (qmm_api.cu) and the
// kernels. Not installed; the public interface is include/qmm.h.
#pragma once

#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <cstdint>

namespace qmm {

// ---- quantisers / dequantiser (qmm_quant.cu) -----------------------------------
cudaError_t launch_quantize_q8_0(const float* x, int64_t n, uint8_t* out, float* scales, bool rounded_inv,
                                 cudaStream_t st);
cudaError_t launch_quantize_q4_0(const float* x, int64_t n, uint8_t* out, cudaStream_t st);
cudaError_t launch_quantize_q4_1(const float* x, int64_t n, uint8_t* out, cudaStream_t st);
cudaError_t launch_dequantize(int qt, const uint8_t* w, int64_t n, float* out, cudaStream_t st);

// ---- GEMV activation preparation (qmm_quant.cu) ----------------------------------
// f32 mode:   xf  [nb][M][4][16 halves], xcs [nb][token_pad(M)] float2, xsum [nb][token_pad(M)] (Q4_1 only)
// native:     xq  [nb][M][4][8 bytes],   xsc [nb][token_pad(M)] int2
// Both also zero `nzero` words at `zero` (the GEMV's split-K tickets).
cudaError_t launch_xprep_f32(int qt, const float* x, int M, int K, __half* xf, float2* xcs, float* xsum,
                             unsigned* zero, int nzero, cudaStream_t st);
cudaError_t launch_xprep_q8(int qt, const float* x, int M, int K, uint8_t* xq, int2* xsc, unsigned* zero, int nzero,
                           cudaStream_t st);
cudaError_t launch_pdl_kernel(const void* fn, dim3 grid, dim3 block, size_t smem, cudaStream_t st, void** args);

// ---- GEMV (qmm_gemv.cu) ---------------------------------------------------------
struct GemvPlan {
    int qt;          // kQ4_0 / kQ4_1 / kQ8_0
    bool native;     // Q8_0-quantised activations (int8 MMA) instead of f32 activations
    int M, N, K;     // y[M,N] = x[M,K] . W[N,K]^T
    int nb;          // K / 32
    int row_bytes;   // nb * block bytes
    int nt;          // token tiles of 8 (1, 2, 4 or 8)
    int ks;          // K splits per 16-row group
    int nbu;         // blocks per K split
    int kc;          // blocks per pipeline stage
    int pitch;       // shared-memory bytes per row slot of a stage
    int loader;      // 0: one 2-D TMA tile per stage (16-byte row pitch); 1: cp.async windows
    int units;       // row groups * ks
    int grid;        // CTAs
    size_t smem;     // dynamic shared memory per CTA
};

// Fills a plan for the given problem on a device with `num_sms` SMs. Returns
// false if the shape is not handled by the GEMV kernel (M > 64).
bool gemv_plan(int qt, bool native, int M, int N, int K, int num_sms, GemvPlan* p);

// Workspace layout shared by the xprep and GEMV launches.
struct GemvWorkspace {
    void* xa;          // xf (f32 mode) or xq (native)
    void* xs;          // xcs (float2) or xsc (int2)
    float* xsum;       // Q4_1 f32 mode only
    float* partial;    // [ks][M][N] when ks > 1
    unsigned* counters;  // [row groups] when ks > 1; zero before first use, self-resetting
};
size_t gemv_workspace_bytes(const GemvPlan& p);
// Carves `base` (256-byte aligned) into the pieces. Counters are at the end.
void gemv_workspace_carve(const GemvPlan& p, void* base, GemvWorkspace* ws);
size_t gemv_counters_offset(const GemvPlan& p);
size_t gemv_counters_bytes(const GemvPlan& p);

// no_host_alloc: skip the host-side caches (for the allocation-free entry point).
cudaError_t launch_gemv(const GemvPlan& p, const uint8_t* w, const float* x, float* y, const GemvWorkspace& ws,
                        int* err, cudaStream_t st, bool no_host_alloc = false);

int* device_error_word(int device);

}  // namespace qmm
