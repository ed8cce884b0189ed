// Block quantisers, dequantisers and GEMV activation preparation (sm_100a).
//
// Every quantiser here reproduces the reference's arithmetic bit for bit:
//   - IEEE division for amax/127, amax/8, (max-min)/15 and 1/scale (no fast math),
//   - x * inv with a single rounding (no FMA contraction: __fmul_rn),
//   - round half away from zero (roundf, Rust f32::round), clamp, saturating cast,
//   - f16 scales by round-to-nearest-even (__float2half_rn; the `half` crate).
// Reference: llmserve/llmmodel/kernel/main/src/core/quantize.rs:15-289 and
// main/features/tensor/src/core/tensor/tensor.rs:527-630.
#include "qmm_common.cuh"
#include "qmm_kernels.cuh"

namespace qmm {

namespace {

__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
    return v;
}
__device__ __forceinline__ float warp_min(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v = fminf(v, __shfl_xor_sync(0xffffffffu, v, o));
    return v;
}
__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v = __fadd_rn(v, __shfl_xor_sync(0xffffffffu, v, o));
    return v;
}
__device__ __forceinline__ int warp_sum_i(int v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}

// Rust `(v).round().clamp(lo, hi) as i8` (NaN -> 0).
__device__ __forceinline__ int round_clamp(float v, float lo, float hi) {
    float r = roundf(v);
    if (isnan(r)) return 0;
    r = fminf(fmaxf(r, lo), hi);
    return (int)r;
}

// Q8_0 block quantisation of the 32 values held one per lane. `rounded_inv`
// selects quantize_row_q8_0 (inv = 1/f32(f16(scale)), quantize.rs:272-276)
// instead of quantize_q8_0 (inv = 1/scale, quantize.rs:32-34).
struct Q8Block {
    int q;            // this lane's quant
    uint16_t d_bits;  // f16 scale
    float d_rt;       // f32(f16(scale))
};
__device__ __forceinline__ Q8Block q8_block_lane(float x, bool rounded_inv) {
    const float amax = warp_max(fabsf(x));
    const float scale = (amax == 0.0f) ? 0.0f : __fdiv_rn(amax, 127.0f);
    const uint16_t h = f32_to_f16_bits_rn(scale);
    const float srt = f16_bits_to_f32(h);
    const float sdiv = rounded_inv ? srt : scale;
    const float inv = (sdiv == 0.0f) ? 0.0f : __fdiv_rn(1.0f, sdiv);
    Q8Block r;
    r.q = round_clamp(__fmul_rn(x, inv), -128.0f, 127.0f);
    r.d_bits = h;
    r.d_rt = srt;
    return r;
}

// ---- weight / activation quantisers (one warp per 32-element block) --------------

__global__ void quantize_q8_0_kernel(const float* __restrict__ x, int64_t nblocks, uint8_t* __restrict__ out,
                                     float* __restrict__ scales, int rounded_inv) {
    const int lane = threadIdx.x & 31;
    const int64_t warps = (int64_t)gridDim.x * (blockDim.x >> 5);
    for (int64_t b = (int64_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5); b < nblocks; b += warps) {
        const Q8Block r = q8_block_lane(x[b * QK + lane], rounded_inv != 0);
        uint8_t* o = out + b * Q8_0_BYTES;
        o[2 + lane] = (uint8_t)(int8_t)r.q;
        if (lane == 0) {
            o[0] = (uint8_t)(r.d_bits & 0xff);
            o[1] = (uint8_t)(r.d_bits >> 8);
            if (scales) scales[b] = r.d_rt;
        }
    }
}

// quantize.rs:124-165: interleaved packing (element 2i low nibble, 2i+1 high).
__global__ void quantize_q4_0_kernel(const float* __restrict__ x, int64_t nblocks, uint8_t* __restrict__ out) {
    const int lane = threadIdx.x & 31;
    const int64_t warps = (int64_t)gridDim.x * (blockDim.x >> 5);
    for (int64_t b = (int64_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5); b < nblocks; b += warps) {
        const float v = x[b * QK + lane];
        const float amax = warp_max(fabsf(v));
        const float scale = (amax == 0.0f) ? 0.0f : __fdiv_rn(amax, 8.0f);
        const float inv = (scale == 0.0f) ? 0.0f : __fdiv_rn(1.0f, scale);
        const int q = round_clamp(__fmul_rn(v, inv), -8.0f, 7.0f) + 8;
        // lanes 0-1 write the f16 scale, lanes 2-17 one packed byte each
        const uint32_t h = f32_to_f16_bits_rn(scale);
        const int j = (lane - 2) & 15;
        const int qe = __shfl_sync(0xffffffffu, q, 2 * j);
        const int qo = __shfl_sync(0xffffffffu, q, 2 * j + 1);
        const uint32_t byte = lane == 0 ? (h & 0xffu) : (lane == 1 ? (h >> 8) : (uint32_t)(((qo & 0xf) << 4) | (qe & 0xf)));
        if (lane < Q4_0_BYTES) out[b * Q4_0_BYTES + lane] = (uint8_t)byte;
    }
}

// quantize.rs:207-251
__global__ void quantize_q4_1_kernel(const float* __restrict__ x, int64_t nblocks, uint8_t* __restrict__ out) {
    const int lane = threadIdx.x & 31;
    const int64_t warps = (int64_t)gridDim.x * (blockDim.x >> 5);
    for (int64_t b = (int64_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5); b < nblocks; b += warps) {
        const float v = x[b * QK + lane];
        const float mn = warp_min(v), mx = warp_max(v);
        const float d = __fdiv_rn(__fsub_rn(mx, mn), 15.0f);
        const float inv = (d == 0.0f) ? 0.0f : __fdiv_rn(1.0f, d);
        float r = roundf(__fmul_rn(__fsub_rn(v, mn), inv));
        const int q = isnan(r) ? 0 : (int)fminf(fmaxf(r, 0.0f), 15.0f);
        // lanes 0-3 write d and m (f16 LE), lanes 4-19 one packed byte each
        const uint32_t hdm = f32_to_f16_bits_rn(d) | ((uint32_t)f32_to_f16_bits_rn(mn) << 16);
        const int j = (lane - 4) & 15;
        const int qe = __shfl_sync(0xffffffffu, q, 2 * j);
        const int qo = __shfl_sync(0xffffffffu, q, 2 * j + 1);
        const uint32_t byte = lane < 4 ? ((hdm >> (8 * lane)) & 0xffu) : (uint32_t)(((qo & 0xf) << 4) | (qe & 0xf));
        if (lane < Q4_1_BYTES) out[b * Q4_1_BYTES + lane] = (uint8_t)byte;
    }
}

// Tensor::to_f32 (tensor.rs:527-630): one thread per output element.
__global__ void dequantize_kernel(int qt, const uint8_t* __restrict__ w, int64_t n, float* __restrict__ out) {
    const int64_t stride = (int64_t)gridDim.x * blockDim.x;
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += stride) {
        const int64_t b = i / QK;
        const int e = (int)(i % QK);
        float v;
        if (qt == kQ4_0) {
            const uint8_t* blk = w + b * Q4_0_BYTES;
            const float s = f16_bits_to_f32((uint16_t)(blk[0] | (blk[1] << 8)));
            const uint8_t byte = blk[2 + (e & 15)];
            const int nib = (e < 16) ? (byte & 0xf) : (byte >> 4);
            v = __fmul_rn(s, (float)(nib - 8));
        } else if (qt == kQ4_1) {
            const uint8_t* blk = w + b * Q4_1_BYTES;
            const float d = f16_bits_to_f32((uint16_t)(blk[0] | (blk[1] << 8)));
            const float m = f16_bits_to_f32((uint16_t)(blk[2] | (blk[3] << 8)));
            const uint8_t byte = blk[4 + (e & 15)];
            const int nib = (e < 16) ? (byte & 0xf) : (byte >> 4);
            v = __fadd_rn(__fmul_rn(d, (float)nib), m);
        } else {
            const uint8_t* blk = w + b * Q8_0_BYTES;
            const float s = f16_bits_to_f32((uint16_t)(blk[0] | (blk[1] << 8)));
            v = __fmul_rn(s, (float)(int8_t)blk[2 + e]);
        }
        out[i] = v;
    }
}

// out[m][i] = act(gate[m * ld + i]) * up[m * ld + i] (up null: act alone), the
// activation step of the reference's FeedForward::forward
// (layers/main/src/core/feed_forward.rs:198-251).
__global__ void gated_act_kernel(int kind, const float* __restrict__ gate, const float* __restrict__ up, int64_t m,
                                 int64_t hidden, int64_t ld, float* __restrict__ out) {
    pdl_launch_dependents();
    pdl_wait();  // gate / up are written by the matmul before this launch
    const int64_t total = m * hidden;
    const int64_t stride = (int64_t)gridDim.x * blockDim.x;
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < total; i += stride) {
        const int64_t o = (i / hidden) * ld + i % hidden;
        const float a = act_value(kind, gate[o]);
        out[i] = up ? a * up[o] : a;
    }
}

// Position-weighted checksum of a byte range: sum over its little-endian
// 32-bit words w_i (tail zero-padded) of w_i * (2i + 1) mod 2^64, added into
// *acc. Addition mod 2^64 is order independent, so the atomics give one
// deterministic value. `p` is 4-byte aligned.
__global__ void checksum_kernel(const uint8_t* __restrict__ p, uint64_t len, unsigned long long* acc) {
    const uint64_t nfull = len / 4;
    const uint32_t* w = reinterpret_cast<const uint32_t*>(p);
    unsigned long long s = 0;
    const uint64_t stride = (uint64_t)gridDim.x * blockDim.x;
    for (uint64_t i = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x; i < nfull; i += stride)
        s += (unsigned long long)w[i] * (2ull * i + 1ull);
    if (blockIdx.x == 0 && threadIdx.x == 0 && (len & 3)) {
        uint32_t last = 0;
        for (uint64_t b = nfull * 4; b < len; ++b) last |= (uint32_t)p[b] << (8 * (b - nfull * 4));
        s += (unsigned long long)last * (2ull * nfull + 1ull);
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
    if ((threadIdx.x & 31) == 0) atomicAdd(acc, s);
}

// ---- GEMV activation preparation ---------------------------------------------------
//
// f32-activation mode: the GEMV feeds x to f16 tensor-core MMAs. Per (token,
// block) the 32 values are scaled by 2^-e so that max|x| lands in [2^13, 2^14)
// (exact, power of two), then split into hi = f16(x') and lo = f16(x' - hi),
// which together carry ~22 significant bits. The MMA sees weights biased by
// the f16 magic-number trick; `corr` is the bias contribution to subtract, and
// `s` = 2^e restores the scale. Layouts (see qmm_kernels.cuh):
//   xf   [nb][M][4 t] x {hi: 4 x half2, lo: 4 x half2}    (32 B per record)
//   side [nb][token_pad(M)/2 pairs] x 8 words
//        {-corr0, -corr1, -corr0, -corr1, s0, s1, sx0, sx1}
//   (the first four are the MMA accumulator's initial value as the GEMV lane
//   holding tokens (2p, 2p+1) needs it; sx = block sum, Q4_1 only).
// The element order inside a record is the K permutation the GEMV's A
// fragments use (K order inside a block is free in a dot product as long as
// both operands follow it).
template <int QT>
__global__ void xprep_f32_kernel(const float* __restrict__ x, int M, int K, int Mpad, __half* __restrict__ xf,
                                 uint32_t* __restrict__ side, unsigned* __restrict__ zero, int nzero) {
    // let the next kernel (the GEMV) launch and start streaming its weights;
    // this kernel writes nothing before the wait below
    pdl_launch_dependents();
    pdl_wait();  // x may be produced by the preceding kernel in the stream
    const int lane = threadIdx.x & 31;
    for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < nzero; i += gridDim.x * blockDim.x) zero[i] = 0u;
    const int nb = K / QK;
    const int64_t total = (int64_t)nb * Mpad;
    const int64_t warps = (int64_t)gridDim.x * (blockDim.x >> 5);
    for (int64_t idx = (int64_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5); idx < total; idx += warps) {
        const int b = (int)(idx / Mpad);
        const int m = (int)(idx % Mpad);
        uint32_t* rec8 = side + ((int64_t)b * (Mpad / 2) + (m >> 1)) * 8 + (m & 1);
        if (m >= M) {  // padding tokens: neutral corr/scale
            if (lane == 0) rec8[0] = rec8[2] = rec8[4] = rec8[6] = 0u;
            continue;
        }
        const float v = x[(int64_t)m * K + (int64_t)b * QK + lane];
        const float amax = warp_max(fabsf(v));
        int e = 0;
        if (amax > 0.0f && isfinite(amax)) {
            int E;
            frexpf(amax, &E);  // amax = f * 2^E, f in [0.5, 1)
            e = E - 14;
            e = max(-126, min(127, e));
        }
        const float xs = ldexpf(v, -e);  // exact unless subnormal
        const bool q4 = (QT != kQ8_0);
        // Q4 formats: high-nibble elements (16..31) meet weights pre-multiplied
        // by 16 by the magic trick, so their activations are pre-divided by 16.
        const float vv = (q4 && lane >= 16) ? xs * 0.0625f : xs;
        const __half hi = __float2half_rn(vv);
        const __half lo = __float2half_rn(vv - __half2float(hi));
        const float rep = __half2float(hi) + __half2float(lo);
        float c;
        if (QT == kQ8_0) {
            c = 1152.0f * rep;                       // A = 1152 + q
        } else if (QT == kQ4_0) {
            c = (lane < 16) ? 1032.0f * rep : 1152.0f * rep;  // 1024+n-8 ; (1024+16n)/16... see kernels
        } else {
            c = (lane < 16) ? 1024.0f * rep : 1024.0f * rep;  // Q4_1: remove the 1024 / 64*16 bias only
        }
        const float corr = warp_sum(c);
        float sx = 0.0f;
        if (QT == kQ4_1) sx = warp_sum((lane < 16) ? rep : 16.0f * rep);
        // destination half index inside the 16-half record of thread t: thread t
        // covers elements 4t..4t+3 (first MMA) and 16+4t..16+4t+3 (second MMA)
        const int j = lane & 15;
        const int t = j >> 2;
        const int r = j & 3;
        int idx8;
        if (QT == kQ8_0) {
            idx8 = (lane >> 4) * 4 + r;  // byte order: (q0,q1) then (q2,q3)
        } else {
            idx8 = (lane >> 4) * 4 + (r & 1) * 2 + (r >> 1);  // nibble pairs (n0,n2) then (n1,n3)
        }
        __half* rec = xf + (((int64_t)b * M + m) * 4 + t) * 16;
        rec[idx8] = hi;
        rec[8 + idx8] = lo;
        if (lane == 0) {
            rec8[0] = rec8[2] = __float_as_uint(-corr);  // MMA accumulator starts at -corr
            rec8[4] = __float_as_uint(ldexpf(1.0f, e));
            rec8[6] = __float_as_uint(sx);
        }
    }
}

// Q8_0-activation ("native") mode: each (token, block) is quantised exactly as
// the reference does before its integer dots -- quantize_q8_0 for Q8_0 weights
// (matmul_f32_q8_v2, quantize.rs:451) and quantize_row_q8_0 for Q4_0/Q4_1
// weights (quantize.rs:674-676) -- and laid out for the s8 MMA:
//   xq   [nb][M][4 t] x 8 bytes {b0, b1}
//   side [nb][token_pad(M)/2 pairs] x 8 words
//        {c0, c1, c0, c1, xs0, xs1, qsum0, qsum1}
//   c = -8 * qsum for Q4_0 (sum (n - 8) q = sum n q - 8 sum q), else 0: the s32
//   MMA accumulator's initial value; xs = f32(f16(scale)) as float bits.
template <int QT>
__global__ void xprep_q8_kernel(const float* __restrict__ x, int M, int K, int Mpad, uint8_t* __restrict__ xq,
                                uint32_t* __restrict__ side, unsigned* __restrict__ zero, int nzero) {
    pdl_launch_dependents();  // see xprep_f32_kernel
    pdl_wait();
    const int lane = threadIdx.x & 31;
    for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < nzero; i += gridDim.x * blockDim.x) zero[i] = 0u;
    const int nb = K / QK;
    const int64_t total = (int64_t)nb * Mpad;
    const int64_t warps = (int64_t)gridDim.x * (blockDim.x >> 5);
    for (int64_t idx = (int64_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5); idx < total; idx += warps) {
        const int b = (int)(idx / Mpad);
        const int m = (int)(idx % Mpad);
        uint32_t* rec8 = side + ((int64_t)b * (Mpad / 2) + (m >> 1)) * 8 + (m & 1);
        if (m >= M) {
            if (lane == 0) rec8[0] = rec8[2] = rec8[4] = rec8[6] = 0u;
            continue;
        }
        const float v = x[(int64_t)m * K + (int64_t)b * QK + lane];
        const Q8Block r = q8_block_lane(v, QT != kQ8_0);
        const int qsum = warp_sum_i(r.q);
        // thread t: q[4t..4t+3] then q[16+4t..16+4t+3] (the s8 MMA's k order)
        const int j = lane & 15;
        const int t = j >> 2;
        const int off = (lane >> 4) * 4 + (j & 3);
        xq[(((int64_t)b * M + m) * 4 + t) * 8 + off] = (uint8_t)(int8_t)r.q;
        if (lane == 0) {
            rec8[0] = rec8[2] = (uint32_t)(QT == kQ4_0 ? -8 * qsum : 0);
            rec8[4] = __float_as_uint(r.d_rt);
            rec8[6] = (uint32_t)qsum;
        }
    }
}

// Q8_0-activation mode for the integer tensor-core GEMM (qmm_gemm_i8.cu): each
// (token, block) quantised exactly as the reference does before its integer
// dots (quantize_q8_0 for Q8_0 weights, quantize_row_q8_0 for Q4 weights), laid
// out for TMA:
//   xq  [M][K] s8, row-major (the K-major B operand);
//   xs  [nbp][Mp] f32 = f32(f16(scale)), block-major (a tile's tokens contiguous);
//   xc  [nbp][Mp] 32-bit: Q4_0 the integer 0x4B400000 - 8 * qsum (added to a
//       block dot it gives the float bits of 2^23 + 2^22 + (dot - 8 qsum): an
//       exact int-to-float conversion by one subtraction); Q4_1 (float)qsum;
//       Q8_0 unused.
// Mp = M rounded up to 4 (16-byte rows), nbp = K/32 rounded up to 4.
template <int QT>
__global__ void xprep_i8gemm_kernel(const float* __restrict__ x, int M, int K, int Mp, int8_t* __restrict__ xq,
                                    float* __restrict__ xs, uint32_t* __restrict__ xc) {
    pdl_launch_dependents();
    pdl_wait();  // x may be produced by the preceding kernel in the stream
    const int lane = threadIdx.x & 31;
    const int nb = K / QK;
    const int64_t total = (int64_t)nb * M;
    const int64_t warps = (int64_t)gridDim.x * (blockDim.x >> 5);
    for (int64_t idx = (int64_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5); idx < total; idx += warps) {
        const int m = (int)(idx / nb);
        const int b = (int)(idx % nb);
        const float v = x[(int64_t)m * K + (int64_t)b * QK + lane];
        const Q8Block r = q8_block_lane(v, QT != kQ8_0);
        xq[(int64_t)m * K + (int64_t)b * QK + lane] = (int8_t)r.q;
        const int qsum = warp_sum_i(r.q);
        if (lane == 0) {
            xs[(int64_t)b * Mp + m] = r.d_rt;
            if (QT == kQ4_0) xc[(int64_t)b * Mp + m] = 0x4B400000u - (uint32_t)(8 * qsum);
            if (QT == kQ4_1) xc[(int64_t)b * Mp + m] = __float_as_uint((float)qsum);
        }
    }
}

}  // namespace

// ---- launchers ---------------------------------------------------------------------

static int grid_for_warps(int64_t warps_needed, int warps_per_cta) {
    int64_t g = (warps_needed + warps_per_cta - 1) / warps_per_cta;
    if (g < 1) g = 1;
    if (g > 148 * 16) g = 148 * 16;
    return (int)g;
}

cudaError_t launch_quantize_q8_0(const float* x, int64_t n, uint8_t* out, float* scales, bool rounded_inv,
                                 cudaStream_t st) {
    const int64_t nb = n / QK;
    if (nb == 0) return cudaSuccess;
    quantize_q8_0_kernel<<<grid_for_warps(nb, 8), 256, 0, st>>>(x, nb, out, scales, rounded_inv ? 1 : 0);
    note_launch();
    return cudaGetLastError();
}
cudaError_t launch_quantize_q4_0(const float* x, int64_t n, uint8_t* out, cudaStream_t st) {
    const int64_t nb = n / QK;
    if (nb == 0) return cudaSuccess;
    quantize_q4_0_kernel<<<grid_for_warps(nb, 8), 256, 0, st>>>(x, nb, out);
    note_launch();
    return cudaGetLastError();
}
cudaError_t launch_quantize_q4_1(const float* x, int64_t n, uint8_t* out, cudaStream_t st) {
    const int64_t nb = n / QK;
    if (nb == 0) return cudaSuccess;
    quantize_q4_1_kernel<<<grid_for_warps(nb, 8), 256, 0, st>>>(x, nb, out);
    note_launch();
    return cudaGetLastError();
}
cudaError_t launch_gated_act(int kind, const float* gate, const float* up, int64_t m, int64_t hidden, int64_t ld,
                             float* out, cudaStream_t st) {
    if (m * hidden == 0) return cudaSuccess;
    int64_t g = (m * hidden + 255) / 256;
    if (g > 148 * 8) g = 148 * 8;
    void* args[] = {(void*)&kind, (void*)&gate, (void*)&up, (void*)&m, (void*)&hidden, (void*)&ld, (void*)&out};
    return launch_pdl_kernel((const void*)gated_act_kernel, dim3((unsigned)g), dim3(256), 0, st, args);
}

cudaError_t launch_checksum(const uint8_t* p, uint64_t len, unsigned long long* acc, cudaStream_t st) {
    uint64_t g = (len / 4 + 255) / 256;
    if (g < 1) g = 1;
    if (g > 148 * 16) g = 148 * 16;
    checksum_kernel<<<(int)g, 256, 0, st>>>(p, len, acc);
    note_launch();
    return cudaGetLastError();
}

cudaError_t launch_dequantize(int qt, const uint8_t* w, int64_t n, float* out, cudaStream_t st) {
    if (n == 0) return cudaSuccess;
    int64_t g = (n + 255) / 256;
    if (g > 148 * 32) g = 148 * 32;
    dequantize_kernel<<<(int)g, 256, 0, st>>>(qt, w, n, out);
    note_launch();
    return cudaGetLastError();
}

static cudaError_t launch_pdl(const void* fn, dim3 grid, dim3 block, size_t smem, cudaStream_t st, void** args) {
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

cudaError_t launch_xprep_f32(int qt, const float* x, int M, int K, __half* xf, uint32_t* side, unsigned* zero,
                             int nzero, cudaStream_t st) {
    const int Mpad = token_pad(M);
    const int64_t warps = (int64_t)(K / QK) * Mpad;
    dim3 grid(grid_for_warps(warps, 8)), block(256);
    void* args[] = {(void*)&x,    (void*)&M,    (void*)&K,     (void*)&Mpad, (void*)&xf,
                    (void*)&side, (void*)&zero, (void*)&nzero};
    const void* fn = qt == kQ8_0 ? (const void*)xprep_f32_kernel<kQ8_0>
                                 : (qt == kQ4_0 ? (const void*)xprep_f32_kernel<kQ4_0>
                                                : (const void*)xprep_f32_kernel<kQ4_1>);
    return launch_pdl(fn, grid, block, 0, st, args);
}

cudaError_t launch_xprep_q8(int qt, const float* x, int M, int K, uint8_t* xq, uint32_t* side, unsigned* zero,
                           int nzero, cudaStream_t st) {
    const int Mpad = token_pad(M);
    const int64_t warps = (int64_t)(K / QK) * Mpad;
    dim3 grid(grid_for_warps(warps, 8)), block(256);
    void* args[] = {(void*)&x, (void*)&M, (void*)&K, (void*)&Mpad, (void*)&xq, (void*)&side, (void*)&zero, (void*)&nzero};
    const void* fn = qt == kQ8_0 ? (const void*)xprep_q8_kernel<kQ8_0>
                                 : (qt == kQ4_0 ? (const void*)xprep_q8_kernel<kQ4_0>
                                                : (const void*)xprep_q8_kernel<kQ4_1>);
    return launch_pdl(fn, grid, block, 0, st, args);
}

cudaError_t launch_pdl_kernel(const void* fn, dim3 grid, dim3 block, size_t smem, cudaStream_t st, void** args) {
    return launch_pdl(fn, grid, block, smem, st, args);
}

cudaError_t launch_xprep_i8gemm(int qt, const float* x, int M, int K, int Mp, int8_t* xq, float* xs, uint32_t* xc,
                                cudaStream_t st) {
    const int64_t total = (int64_t)(K / QK) * M;
    const int grid = grid_for_warps(total, 8);
    void* args[] = {(void*)&x, (void*)&M, (void*)&K, (void*)&Mp, (void*)&xq, (void*)&xs, (void*)&xc};
    const void* fn = qt == kQ8_0 ? (const void*)xprep_i8gemm_kernel<kQ8_0>
                                 : (qt == kQ4_0 ? (const void*)xprep_i8gemm_kernel<kQ4_0>
                                                : (const void*)xprep_i8gemm_kernel<kQ4_1>);
    return launch_pdl_kernel(fn, dim3(grid), dim3(256), 0, st, args);
}

}  // namespace qmm
