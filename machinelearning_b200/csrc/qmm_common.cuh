// Shared device helpers for the B200 (sm_100a) quantized-matmul library.
//
// Block formats (reference: llmserve/llmmodel/kernel/main/src/api/types.rs:1-23,
// GGML type ids from llmserve/llmmodel/gguf/main/src/api/types.rs:8-12):
//   Q8_0  id 8  34 B  [f16 d LE][32 x i8 q]          value = d * q
//   Q4_0  id 2  18 B  [f16 d LE][16 B nibbles]        value = d * (nib - 8)
//   Q4_1  id 3  20 B  [f16 d LE][f16 m LE][16 B nib]  value = d * nib + m
// Nibble order is GGML's: the low nibble of byte j is element j, the high
// nibble is element j + 16 (reference simd.rs:30-52, tensor.rs:545-555).
#pragma once

#include <cstdint>
#include <cuda_fp16.h>
#include <cuda_runtime.h>

namespace qmm {

constexpr int QK = 32;
constexpr int Q8_0_BYTES = 34;
constexpr int Q4_0_BYTES = 18;
constexpr int Q4_1_BYTES = 20;

enum QType : int { kQ4_0 = 2, kQ4_1 = 3, kQ8_0 = 8 };

__host__ __device__ constexpr int block_bytes(int qt) {
    return qt == kQ8_0 ? Q8_0_BYTES : (qt == kQ4_0 ? Q4_0_BYTES : (qt == kQ4_1 ? Q4_1_BYTES : 0));
}

// GEMV token tiles are 8 wide and come in counts of 1, 2, 4 or 8 (M <= 64);
// per-token side arrays are padded to the tile count the kernel reads.
__host__ __device__ constexpr int token_tiles(int M) { return M <= 8 ? 1 : (M <= 16 ? 2 : (M <= 32 ? 4 : 8)); }
__host__ __device__ constexpr int token_pad(int M) { return 8 * token_tiles(M); }

// Error word written by kernels whose bounded waits ran out (device global,
// one per loaded module per device). Read and cleared by qmm_device_error().
enum DeviceError : int { kErrNone = 0, kErrWaitTimeout = 1, kErrBadLaunch = 2 };

// ---- f16 helpers -------------------------------------------------------------
__device__ __forceinline__ float f16_bits_to_f32(uint16_t h) {
    return __half2float(__ushort_as_half(h));
}
__device__ __forceinline__ uint16_t f32_to_f16_bits_rn(float f) {
    return __half_as_ushort(__float2half_rn(f));
}

// ---- shared-memory addressing ------------------------------------------------
__device__ __forceinline__ uint32_t smem_u32(const void* p) {
    return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

// ---- mbarrier ----------------------------------------------------------------
__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}
__device__ __forceinline__ void fence_mbar_init() {
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}
__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
    asm volatile(
        "{\n\t.reg .b64 st;\n\t"
        "mbarrier.arrive.release.cta.shared::cta.b64 st, [%0];\n\t}" ::"r"(smem_u32(bar))
        : "memory");
}
__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
    asm volatile(
        "{\n\t.reg .b64 st;\n\t"
        "mbarrier.arrive.expect_tx.release.cta.shared::cta.b64 st, [%0], %1;\n\t}" ::"r"(smem_u32(bar)),
        "r"(bytes)
        : "memory");
}
// One probe of the phase with the given parity: the thread may be suspended
// for at most ~20 ns while the phase is incomplete (a short hint: hand-offs
// between warps are latency critical, and the default suspension measured
// ~20% slower in the GEMM pipeline).
__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.acquire.cta.shared::cta.b64 p, [%1], %2, 20;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(smem_u32(bar)), "r"(parity)
        : "memory");
    return ok != 0;
}
__device__ __forceinline__ bool mbar_test_wait(uint64_t* bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.test_wait.parity.acquire.cta.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(smem_u32(bar)), "r"(parity)
        : "memory");
    return ok != 0;
}

// Bounded wait: every spin in this library gives up after a fixed number of
// probes (each try_wait already suspends for a hardware-chosen interval), sets
// the device error word and reports failure, so a logic error can never hang a
// GPU. The limit is orders of magnitude above any legitimate wait.
constexpr uint32_t kMaxWaitProbes = 1u << 20;

__device__ __forceinline__ bool mbar_wait_bounded(uint64_t* bar, uint32_t parity, int* err) {
    for (uint32_t i = 0; i < kMaxWaitProbes; ++i) {
        if (mbar_try_wait(bar, parity)) return true;
    }
    if (err) atomicExch(err, kErrWaitTimeout);
    return false;
}

// ---- bulk async copy (TMA, 1-D) ------------------------------------------------
// dst/src 16-byte aligned, bytes a multiple of 16; completion is counted on the
// mbarrier as transaction bytes.
__device__ __forceinline__ void bulk_g2s(void* dst_smem, const void* src_gmem, uint32_t bytes, uint64_t* bar) {
    asm volatile(
        "cp.async.bulk.shared::cta.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
            smem_u32(dst_smem)),
        "l"(src_gmem), "r"(bytes), "r"(smem_u32(bar))
        : "memory");
}

// ---- tiled tensor copy (TMA, 2-D, no multicast) ----------------------------------
// Box lands densely in shared memory (row pitch = box inner bytes). Rows or
// columns outside the tensor are zero-filled and still counted as bytes.
__device__ __forceinline__ void tma_load_2d(void* dst_smem, const void* tmap, int x, int y, uint64_t* bar) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], "
        "[%4];" ::"r"(smem_u32(dst_smem)),
        "l"(tmap), "r"(x), "r"(y), "r"(smem_u32(bar))
        : "memory");
}
__device__ __forceinline__ void prefetch_tmap(const void* tmap) {
    asm volatile("prefetch.tensormap [%0];" ::"l"(tmap) : "memory");
}

// ---- 16-byte asynchronous copies (LDGSTS) tracked by an mbarrier --------------------
__device__ __forceinline__ void cp_async_16(void* dst_smem, const void* src_gmem) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(smem_u32(dst_smem)), "l"(src_gmem) : "memory");
}
// Arrive on `bar` once every cp.async this thread issued so far has landed
// (the arrival is one of the barrier's expected arrivals).
__device__ __forceinline__ void cp_async_arrive_noinc(uint64_t* bar) {
    asm volatile("cp.async.mbarrier.arrive.noinc.shared::cta.b64 [%0];" ::"r"(smem_u32(bar)) : "memory");
}

// Orders this thread's earlier generic-proxy shared-memory accesses before its
// later async-proxy ones (a TMA write into a buffer that was just read).
__device__ __forceinline__ void fence_proxy_async_smem() {
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

// ---- programmatic dependent launch ----------------------------------------------
// wait: block until the preceding grid in the stream has completed and its
// memory is visible. launch_dependents: allow the next grid to start launching.
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void pdl_launch_dependents() {
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}

// ---- activations ------------------------------------------------------------------
// The reference's element-wise activations in f32, the same operations in the
// same order: kind 0 tanh-approximated GELU (reference
// main/features/tensor/src/core/tensor/math.rs:470-475), 1 SiLU (:478-483),
// 2 ReLU (:465-467).
__device__ __forceinline__ float act_value(int kind, float g) {
    if (kind == 0) {
        const float k = sqrtf(2.0f / 3.14159265358979323846f);
        return 0.5f * g * (1.0f + tanhf(k * (g + 0.044715f * (g * g * g))));
    }
    if (kind == 1) return g * (1.0f / (1.0f + expf(-g)));
    return fmaxf(g, 0.0f);
}
// act(g) * u: the gated forms (GeGLU, SwiGLU) of feed_forward.rs:198-231.
__device__ __forceinline__ float gated_value(int kind, float g, float u) { return act_value(kind, g) * u; }

// ---- shared loads ----------------------------------------------------------------
// Plain C++ loads (not asm volatile) so the compiler can schedule them; they
// stay after an mbarrier wait because the wait's asm clobbers "memory".
__device__ __forceinline__ uint32_t lds_u16(const uint8_t* p) { return *reinterpret_cast<const uint16_t*>(p); }
// 4 bytes from a 2-byte-aligned shared address.
__device__ __forceinline__ uint32_t lds_u32_a2(const uint8_t* p) {
    const uint16_t* q = reinterpret_cast<const uint16_t*>(p);
    return __byte_perm((uint32_t)q[0], (uint32_t)q[1], 0x5410);
}

// ---- tensor-core fragments (mma.sync, register operands) ----------------------
// Not volatile: pure functions of their register operands, free to be
// interleaved with independent work.
// D(16x8 f32) = A(16x16 f16, row) * B(16x8 f16, col) + D
__device__ __forceinline__ void mma_f16_16816(float (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                                              uint32_t b0, uint32_t b1) {
    asm("mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
        "{%0,%1,%2,%3};"
        : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
        : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}
// D(16x8 s32) = A(16x32 s8, row) * B(32x8 s8, col) + D  (exact integer sums)
__device__ __forceinline__ void mma_s8_16832(int (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                                             uint32_t b0, uint32_t b1) {
    asm("mma.sync.aligned.m16n8k32.row.col.s32.s8.s8.s32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
        "{%0,%1,%2,%3};"
        : "+r"(d[0]), "+r"(d[1]), "+r"(d[2]), "+r"(d[3])
        : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

// ---- magic-number dequantisation to f16 pairs -----------------------------------
// (w & 0x000F000F) | 0x6400_6400 yields the halves (1024 + n0, 1024 + n4) for
// the nibbles at bits [3:0] and [19:16]; with mask 0x00F000F0 the nibbles at
// [7:4]/[23:20] give (1024 + 16 n). Both are exact in f16.
__device__ __forceinline__ uint32_t lop3_and_or(uint32_t a, uint32_t mask, uint32_t bias) {
    uint32_t r;
    // (a & b) | c  -> LUT 0xEA
    asm("lop3.b32 %0, %1, %2, %3, 0xEA;" : "=r"(r) : "r"(a), "r"(mask), "r"(bias));
    return r;
}

}  // namespace qmm
