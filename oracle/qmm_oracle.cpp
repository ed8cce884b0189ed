// TEST INFRASTRUCTURE ONLY -- NOT PART OF THE PRODUCT.
//
// CPU restatement of the reference's quantized-matmul path
// (sweengineeringlabs/machinelearning, crate swe-llmmodel-kernel), used as the
// parity checker for the CUDA kernels and as the timed CPU baseline. Only
// tests/, __graft_entry__.smoke() and bench.py's CPU legs may load this.
//
// Files restated (paths inside the reference project):
//   llmserve/llmmodel/kernel/main/src/api/types.rs      block constants
//   llmserve/llmmodel/kernel/main/src/core/quantize.rs  quantizers, dequantizers, matmuls
//   llmserve/llmmodel/kernel/main/src/core/simd.rs      per-block dot products + dispatch
//   main/features/tensor/src/core/tensor/tensor.rs      Tensor::to_f32 dequant (GGML order)
//
// The x86 block dots use the same intrinsic sequence as the reference's AVX2
// (+FMA) functions, so the floating-point summation order -- and therefore
// every output bit -- is the one the reference produces on an AVX2+FMA host.
// Build with -ffp-contract=off: Rust never fuses a multiply and an add, and
// neither may this file outside the explicit _mm256_fmadd_ps the reference uses.
//
// The f16 conversions restate IEEE-754 binary16 round-to-nearest-even, which is
// what the `half` crate (2.7.1, not vendored in the reference) implements in
// both its F16C and its software paths.

#include <immintrin.h>
#include <cmath>
#include <cstdint>
#include <cstring>
#include <vector>
#include <omp.h>

namespace {

// ---- block constants: kernel/main/src/api/types.rs:1-23 ---------------------
constexpr int QK = 32;            // elements per block (Q8_0 / Q4_0 / Q4_1)
constexpr int Q8_0_BYTES = 34;    // f16 d + 32 x i8
constexpr int Q4_0_BYTES = 18;    // f16 d + 16 nibble bytes
constexpr int Q4_1_BYTES = 20;    // f16 d + f16 m + 16 nibble bytes
constexpr int TILE_N = 8;

// ---- IEEE binary16 <-> binary32 ---------------------------------------------
uint16_t f32_to_f16(float f) {
    uint32_t x;
    std::memcpy(&x, &f, 4);
    const uint32_t sign = (x >> 16) & 0x8000u;
    const uint32_t exp = (x >> 23) & 0xffu;
    uint32_t man = x & 0x7fffffu;
    if (exp == 0xffu) {                       // inf / nan
        if (man == 0) return (uint16_t)(sign | 0x7c00u);
        return (uint16_t)(sign | 0x7e00u | (man >> 13));
    }
    const int e = (int)exp - 127 + 15;        // rebiased exponent
    if (e >= 0x1f) return (uint16_t)(sign | 0x7c00u);  // overflow -> inf
    if (e <= 0) {                             // subnormal half (or zero)
        if (e < -10) return (uint16_t)sign;   // below half of the smallest subnormal
        man |= 0x800000u;                     // implicit bit
        const int shift = 14 - e;             // 14..24
        uint32_t h = man >> shift;
        const uint32_t rem = man & ((1u << shift) - 1u);
        const uint32_t half = 1u << (shift - 1);
        if (rem > half || (rem == half && (h & 1u))) h += 1u;
        return (uint16_t)(sign | h);
    }
    uint32_t h = ((uint32_t)e << 10) | (man >> 13);
    const uint32_t rem = man & 0x1fffu;
    if (rem > 0x1000u || (rem == 0x1000u && (h & 1u))) h += 1u;  // may carry into exp (ok)
    return (uint16_t)(sign | h);
}

float f16_to_f32(uint16_t h) {
    const uint32_t sign = ((uint32_t)h & 0x8000u) << 16;
    const uint32_t exp = ((uint32_t)h >> 10) & 0x1fu;
    uint32_t man = (uint32_t)h & 0x3ffu;
    uint32_t x;
    if (exp == 0) {
        if (man == 0) {
            x = sign;
        } else {                              // subnormal: normalise
            int e = -1;
            do { man <<= 1; ++e; } while ((man & 0x400u) == 0);
            x = sign | ((uint32_t)(127 - 15 - e) << 23) | ((man & 0x3ffu) << 13);
        }
    } else if (exp == 0x1fu) {
        x = sign | 0x7f800000u | (man << 13);
    } else {
        x = sign | ((exp + 127 - 15) << 23) | (man << 13);
    }
    float f;
    std::memcpy(&f, &x, 4);
    return f;
}

inline float load_f16(const uint8_t* p) { return f16_to_f32((uint16_t)(p[0] | (p[1] << 8))); }
inline void store_f16(uint8_t* p, float v) {
    const uint16_t h = f32_to_f16(v);
    p[0] = (uint8_t)(h & 0xff);
    p[1] = (uint8_t)(h >> 8);
}

// Rust `f32::max` / `f32::min` return the non-NaN operand (IEEE maxNum/minNum).
inline float rmax(float a, float b) { return std::fmax(a, b); }
inline float rmin(float a, float b) { return std::fmin(a, b); }

// Rust `(v).round().clamp(lo, hi) as i8`: round half away from zero, clamp,
// saturating cast (NaN -> 0).
inline int8_t round_clamp_i8(float v, float lo, float hi) {
    float r = std::round(v);
    if (std::isnan(r)) return 0;
    if (r < lo) r = lo;
    if (r > hi) r = hi;
    return (int8_t)(int)r;
}

// ---- quantizers: kernel/main/src/core/quantize.rs -----------------------------

// quantize.rs:15-48 (and the allocation-free twin :54-89). inv_scale uses the
// un-rounded f32 scale.
void quantize_q8_0_block(const float* x, uint8_t* out) {
    float amax = 0.0f;
    for (int i = 0; i < QK; ++i) amax = rmax(amax, std::fabs(x[i]));
    const float scale = (amax == 0.0f) ? 0.0f : amax / 127.0f;
    const float inv = (scale == 0.0f) ? 0.0f : 1.0f / scale;
    store_f16(out, scale);
    for (int i = 0; i < QK; ++i) out[2 + i] = (uint8_t)round_clamp_i8(x[i] * inv, -128.0f, 127.0f);
}

// quantize.rs:260-289. inv_scale uses the f16-round-tripped scale, and the
// round-tripped scale is also returned for the caller.
float quantize_row_q8_0_block(const float* x, uint8_t* out) {
    float amax = 0.0f;
    for (int i = 0; i < QK; ++i) amax = rmax(amax, std::fabs(x[i]));
    const float scale = (amax == 0.0f) ? 0.0f : amax / 127.0f;
    const uint16_t h = f32_to_f16(scale);
    const float scale_rt = f16_to_f32(h);
    const float inv = (scale_rt == 0.0f) ? 0.0f : 1.0f / scale_rt;
    out[0] = (uint8_t)(h & 0xff);
    out[1] = (uint8_t)(h >> 8);
    for (int i = 0; i < QK; ++i) out[2 + i] = (uint8_t)round_clamp_i8(x[i] * inv, -128.0f, 127.0f);
    return scale_rt;
}

// quantize.rs:124-165. Packs element 2i in the low nibble and 2i+1 in the high
// nibble of byte i (the "interleaved" order the reference's quantizer writes).
void quantize_q4_0_block(const float* x, uint8_t* out) {
    float amax = 0.0f;
    for (int i = 0; i < QK; ++i) amax = rmax(amax, std::fabs(x[i]));
    const float scale = (amax == 0.0f) ? 0.0f : amax / 8.0f;
    const float inv = (scale == 0.0f) ? 0.0f : 1.0f / scale;
    store_f16(out, scale);
    for (int i = 0; i < 16; ++i) {
        const int8_t e = round_clamp_i8(x[2 * i] * inv, -8.0f, 7.0f);
        const int8_t o = round_clamp_i8(x[2 * i + 1] * inv, -8.0f, 7.0f);
        const uint8_t eu = (uint8_t)(e + 8), ou = (uint8_t)(o + 8);
        out[2 + i] = (uint8_t)((ou << 4) | (eu & 0x0f));
    }
}

// quantize.rs:207-251.
void quantize_q4_1_block(const float* x, uint8_t* out) {
    float mn = INFINITY, mx = -INFINITY;
    for (int i = 0; i < QK; ++i) { mn = rmin(mn, x[i]); mx = rmax(mx, x[i]); }
    const float d = (mx - mn) / 15.0f;
    const float inv = (d == 0.0f) ? 0.0f : 1.0f / d;
    store_f16(out, d);
    store_f16(out + 2, mn);
    for (int i = 0; i < 16; ++i) {
        float ve = std::round((x[2 * i] - mn) * inv);
        float vo = std::round((x[2 * i + 1] - mn) * inv);
        // clamp(0,15) as u8 (NaN -> 0)
        auto cu = [](float v) -> uint8_t {
            if (std::isnan(v)) return 0;
            if (v < 0.0f) v = 0.0f;
            if (v > 15.0f) v = 15.0f;
            return (uint8_t)(int)v;
        };
        out[4 + i] = (uint8_t)((cu(vo) << 4) | (cu(ve) & 0x0f));
    }
}

// ---- per-block dots: kernel/main/src/core/simd.rs ----------------------------

// simd.rs:12-18
float dot_q8_scalar(const float* x, const int8_t* q, float s) {
    float sum = 0.0f;
    for (int i = 0; i < 32; ++i) sum += x[i] * (float)q[i];
    return sum * s;
}
// simd.rs:21-27
int32_t dot_q8q8_scalar(const int8_t* a, const int8_t* b) {
    int32_t s = 0;
    for (int i = 0; i < 32; ++i) s += (int32_t)a[i] * (int32_t)b[i];
    return s;
}
// simd.rs:30-40 (GGML order: low nibble of byte j is element j, high is j+16)
float dot_q4_scalar(const float* x, const uint8_t* p, float s) {
    float sum = 0.0f;
    for (int j = 0; j < 16; ++j) {
        const int lo = (p[j] & 0x0f) - 8, hi = ((p[j] >> 4) & 0x0f) - 8;
        sum += x[j] * (float)lo;
        sum += x[j + 16] * (float)hi;
    }
    return sum * s;
}
// simd.rs:43-52
int32_t dot_q4q8_scalar(const uint8_t* p, const int8_t* q) {
    int32_t s = 0;
    for (int j = 0; j < 16; ++j) {
        s += ((p[j] & 0x0f) - 8) * (int32_t)q[j];
        s += (((p[j] >> 4) & 0x0f) - 8) * (int32_t)q[j + 16];
    }
    return s;
}
// simd.rs:59-71
void dot_q4_1q8_scalar(const uint8_t* p, const int8_t* q, int32_t* dot, int32_t* qsum) {
    int32_t d = 0, s = 0;
    for (int j = 0; j < 16; ++j) {
        d += (p[j] & 0x0f) * (int32_t)q[j];
        d += ((p[j] >> 4) & 0x0f) * (int32_t)q[j + 16];
        s += q[j];
        s += q[j + 16];
    }
    *dot = d;
    *qsum = s;
}

// 8-lane -> 1 horizontal sum used by every f32 AVX2 dot in simd.rs
// (extract high 128, add, movehdup, add, movehl, add_ss).
__attribute__((target("avx2"))) inline float hsum256(__m256 v) {
    const __m128 lo = _mm256_castps256_ps128(v);
    const __m128 hi = _mm256_extractf128_ps(v, 1);
    const __m128 s4 = _mm_add_ps(lo, hi);
    const __m128 s2 = _mm_add_ps(s4, _mm_movehdup_ps(s4));
    return _mm_cvtss_f32(_mm_add_ss(s2, _mm_movehl_ps(s2, s2)));
}

// 8 x i32 horizontal sum, shuffle form (simd.rs:168-177).
__attribute__((target("avx2"))) inline int32_t hsum_i32_shuffle(__m256i v) {
    __m128i s = _mm_add_epi32(_mm256_castsi256_si128(v), _mm256_extracti128_si256(v, 1));
    s = _mm_add_epi32(s, _mm_shuffle_epi32(s, 0xB1));
    s = _mm_add_epi32(s, _mm_shuffle_epi32(s, 0x4E));
    return _mm_cvtsi128_si32(s);
}
// 8 x i32 horizontal sum, byte-shift form (simd.rs:271-278).
__attribute__((target("avx2"))) inline int32_t hsum_i32_srli(__m256i v) {
    __m128i s = _mm_add_epi32(_mm256_castsi256_si128(v), _mm256_extracti128_si256(v, 1));
    s = _mm_add_epi32(s, _mm_srli_si128(s, 8));
    s = _mm_add_epi32(s, _mm_srli_si128(s, 4));
    return _mm_cvtsi128_si32(s);
}

// simd.rs:87-134: four independent FMA accumulators, one per 8-lane chunk,
// then (a0+a1)+(a2+a3) and the horizontal sum, times the block scale.
__attribute__((target("avx2,fma"))) float dot_q8_avx2_fma(const float* x, const int8_t* q, float s) {
    __m256 acc[4];
    for (int c = 0; c < 4; ++c) {
        const __m256 xv = _mm256_loadu_ps(x + 8 * c);
        const __m128i q8 = _mm_loadl_epi64((const __m128i*)(q + 8 * c));
        const __m256 qv = _mm256_cvtepi32_ps(_mm256_cvtepi8_epi32(q8));
        acc[c] = _mm256_fmadd_ps(xv, qv, _mm256_setzero_ps());
    }
    const __m256 t = _mm256_add_ps(_mm256_add_ps(acc[0], acc[1]), _mm256_add_ps(acc[2], acc[3]));
    return hsum256(t) * s;
}

// simd.rs:183-208: single accumulator, mul then add (hosts without FMA).
__attribute__((target("avx2"))) float dot_q8_avx2(const float* x, const int8_t* q, float s) {
    __m256 acc = _mm256_setzero_ps();
    for (int c = 0; c < 4; ++c) {
        const __m256 xv = _mm256_loadu_ps(x + 8 * c);
        const __m128i q8 = _mm_loadl_epi64((const __m128i*)(q + 8 * c));
        const __m256 qv = _mm256_cvtepi32_ps(_mm256_cvtepi8_epi32(q8));
        acc = _mm256_add_ps(acc, _mm256_mul_ps(xv, qv));
    }
    return hsum256(acc) * s;
}

// simd.rs:151-178: sign-extend to i16, madd, add halves, shuffle-reduce.
__attribute__((target("avx2"))) int32_t dot_q8q8_avx2(const int8_t* a, const int8_t* b) {
    const __m256i av = _mm256_loadu_si256((const __m256i*)a);
    const __m256i bv = _mm256_loadu_si256((const __m256i*)b);
    const __m256i lo = _mm256_madd_epi16(_mm256_cvtepi8_epi16(_mm256_castsi256_si128(av)),
                                         _mm256_cvtepi8_epi16(_mm256_castsi256_si128(bv)));
    const __m256i hi = _mm256_madd_epi16(_mm256_cvtepi8_epi16(_mm256_extracti128_si256(av, 1)),
                                         _mm256_cvtepi8_epi16(_mm256_extracti128_si256(bv, 1)));
    return hsum_i32_shuffle(_mm256_add_epi32(lo, hi));
}

// simd.rs:210-252: scalar nibble unpack (GGML order) into a stack array, four
// product vectors (mul, no FMA), (p0+p1)+(p2+p3), horizontal sum, times scale.
__attribute__((target("avx2"))) float dot_q4_avx2(const float* x, const uint8_t* p, float s) {
    alignas(32) float w[32];
    for (int j = 0; j < 16; ++j) {
        w[j] = (float)((p[j] & 0x0f) - 8);
        w[j + 16] = (float)(((p[j] >> 4) & 0x0f) - 8);
    }
    __m256 prod[4];
    for (int c = 0; c < 4; ++c) prod[c] = _mm256_mul_ps(_mm256_loadu_ps(x + 8 * c), _mm256_loadu_ps(w + 8 * c));
    const __m256 t = _mm256_add_ps(_mm256_add_ps(prod[0], prod[1]), _mm256_add_ps(prod[2], prod[3]));
    return hsum256(t) * s;
}

// simd.rs:254-294: maddubs(unsigned nibbles, q8) - 8 * sum(q8).
__attribute__((target("avx2"))) int32_t dot_q4q8_avx2(const uint8_t* p, const int8_t* q) {
    const __m128i packed = _mm_loadu_si128((const __m128i*)p);
    const __m128i m = _mm_set1_epi8(0x0f);
    const __m256i nib = _mm256_set_m128i(_mm_and_si128(_mm_srli_epi16(packed, 4), m), _mm_and_si128(packed, m));
    const __m256i qv = _mm256_loadu_si256((const __m256i*)q);
    const __m256i one16 = _mm256_set1_epi16(1);
    const int32_t biased = hsum_i32_srli(_mm256_madd_epi16(_mm256_maddubs_epi16(nib, qv), one16));
    const int32_t qsum = hsum_i32_srli(_mm256_madd_epi16(_mm256_maddubs_epi16(_mm256_set1_epi8(1), qv), one16));
    return biased - 8 * qsum;
}

// simd.rs:296-339
__attribute__((target("avx2"))) void dot_q4_1q8_avx2(const uint8_t* p, const int8_t* q, int32_t* dot, int32_t* qsum) {
    const __m128i packed = _mm_loadu_si128((const __m128i*)p);
    const __m128i m = _mm_set1_epi8(0x0f);
    const __m256i nib = _mm256_set_m128i(_mm_and_si128(_mm_srli_epi16(packed, 4), m), _mm_and_si128(packed, m));
    const __m256i qv = _mm256_loadu_si256((const __m256i*)q);
    const __m256i one16 = _mm256_set1_epi16(1);
    *dot = hsum_i32_srli(_mm256_madd_epi16(_mm256_maddubs_epi16(nib, qv), one16));
    *qsum = hsum_i32_srli(_mm256_madd_epi16(_mm256_maddubs_epi16(_mm256_set1_epi8(1), qv), one16));
}

// ---- runtime dispatch: simd.rs:644-761 ----------------------------------------
// The oracle can be pinned to the scalar functions (isa = 0) for the
// dispatch-vs-scalar known-answer tests; isa = 1 follows the reference's own
// detection order (AVX2+FMA, then AVX2, then the portable code).
int g_isa = 1;

inline bool has_avx2() { return __builtin_cpu_supports("avx2"); }
inline bool has_fma() { return __builtin_cpu_supports("fma"); }

inline float dot_q8(const float* x, const int8_t* q, float s) {
    if (g_isa) {
        if (has_avx2() && has_fma()) return dot_q8_avx2_fma(x, q, s);
        if (has_avx2()) return dot_q8_avx2(x, q, s);
    }
    return dot_q8_scalar(x, q, s);
}
inline int32_t dot_q8q8(const int8_t* a, const int8_t* b) {
    if (g_isa && has_avx2()) return dot_q8q8_avx2(a, b);
    return dot_q8q8_scalar(a, b);
}
inline float dot_q4(const float* x, const uint8_t* p, float s) {
    if (g_isa && has_avx2()) return dot_q4_avx2(x, p, s);
    return dot_q4_scalar(x, p, s);
}
inline int32_t dot_q4q8(const uint8_t* p, const int8_t* q) {
    if (g_isa && has_avx2()) return dot_q4q8_avx2(p, q);
    return dot_q4q8_scalar(p, q);
}
inline void dot_q4_1q8(const uint8_t* p, const int8_t* q, int32_t* d, int32_t* s) {
    if (g_isa && has_avx2()) { dot_q4_1q8_avx2(p, q, d, s); return; }
    dot_q4_1q8_scalar(p, q, d, s);
}

// ---- matmul drivers ---------------------------------------------------------
// Every y[m, n] is produced by one thread walking the K blocks in order, so the
// value does not depend on the thread count or the chunking. The chunking
// below mirrors the reference's rayon split: output columns for m <= 4
// (quantize.rs:317-355), output rows in TILE_N column tiles for m > 4
// (quantize.rs:356-395).
template <class ColFn>
void drive(int64_t m, int64_t n, float* y, ColFn col) {
    if (m <= 4) {
        const int nt = omp_get_max_threads();
        int64_t chunk = n / nt;
        if (chunk < TILE_N) chunk = TILE_N;
        const int64_t nchunks = (n + chunk - 1) / chunk;
        for (int64_t r = 0; r < m; ++r) {
#pragma omp parallel for schedule(static)
            for (int64_t c = 0; c < nchunks; ++c) {
                const int64_t c0 = c * chunk, c1 = (c0 + chunk < n) ? c0 + chunk : n;
                for (int64_t j = c0; j < c1; ++j) y[r * n + j] = col(r, j);
            }
        }
    } else {
#pragma omp parallel for schedule(static)
        for (int64_t r = 0; r < m; ++r) {
            for (int64_t j0 = 0; j0 < n; j0 += TILE_N) {
                const int64_t j1 = (j0 + TILE_N < n) ? j0 + TILE_N : n;
                for (int64_t j = j0; j < j1; ++j) y[r * n + j] = col(r, j);
            }
        }
    }
}

}  // namespace

extern "C" {

// Status codes shared with the product library: 0 ok, 1 block alignment.
enum { ORC_OK = 0, ORC_BLOCK_ALIGNMENT = 1 };

void orc_set_isa(int isa) { g_isa = isa; }
int orc_get_isa(void) { return g_isa; }
int orc_host_has_avx2_fma(void) { return has_avx2() && has_fma(); }
void orc_set_threads(int n) { if (n > 0) omp_set_num_threads(n); }
int orc_get_threads(void) { return omp_get_max_threads(); }

uint16_t orc_f32_to_f16(float f) { return f32_to_f16(f); }
float orc_f16_to_f32(uint16_t h) { return f16_to_f32(h); }
void orc_f32_to_f16_array(const float* x, int64_t n, uint16_t* out) {
    for (int64_t i = 0; i < n; ++i) out[i] = f32_to_f16(x[i]);
}
// Hardware F16C conversion (round-to-nearest-even), the path `half` takes on
// hosts with F16C; used to cross-check the software restatement.
__attribute__((target("f16c"))) void orc_f32_to_f16_f16c(const float* x, int64_t n, uint16_t* out) {
    for (int64_t i = 0; i < n; ++i) {
        const __m128i h = _mm_cvtps_ph(_mm_set_ss(x[i]), _MM_FROUND_TO_NEAREST_INT);
        out[i] = (uint16_t)_mm_extract_epi16(h, 0);
    }
}

int orc_quantize_q8_0(const float* x, int64_t n, uint8_t* out) {
    if (n % QK) return ORC_BLOCK_ALIGNMENT;
    for (int64_t b = 0; b < n / QK; ++b) quantize_q8_0_block(x + b * QK, out + b * Q8_0_BYTES);
    return ORC_OK;
}
// Debug-asserted only in the reference; the caller guarantees n % 32 == 0.
void orc_quantize_row_q8_0(const float* x, int64_t n, uint8_t* out, float* scales) {
    for (int64_t b = 0; b < n / QK; ++b) scales[b] = quantize_row_q8_0_block(x + b * QK, out + b * Q8_0_BYTES);
}
int orc_quantize_q4_0(const float* x, int64_t n, uint8_t* out) {
    if (n % QK) return ORC_BLOCK_ALIGNMENT;
    for (int64_t b = 0; b < n / QK; ++b) quantize_q4_0_block(x + b * QK, out + b * Q4_0_BYTES);
    return ORC_OK;
}
int orc_quantize_q4_1(const float* x, int64_t n, uint8_t* out) {
    if (n % QK) return ORC_BLOCK_ALIGNMENT;
    for (int64_t b = 0; b < n / QK; ++b) quantize_q4_1_block(x + b * QK, out + b * Q4_1_BYTES);
    return ORC_OK;
}

// Tensor::to_f32 (tensor.rs:527-561 Q4_0 in GGML order, :563-598 Q4_1,
// :600-630 Q8_0). dtype ids follow GGML: 2 Q4_0, 3 Q4_1, 8 Q8_0.
int orc_dequantize(int dtype, const uint8_t* w, int64_t n, float* out) {
    if (n % QK) return ORC_BLOCK_ALIGNMENT;
    const int64_t nb = n / QK;
    for (int64_t b = 0; b < nb; ++b) {
        float* o = out + b * QK;
        if (dtype == 2) {
            const uint8_t* blk = w + b * Q4_0_BYTES;
            const float s = load_f16(blk);
            for (int j = 0; j < 16; ++j) {
                o[j] = s * (float)((blk[2 + j] & 0x0f) - 8);
                o[j + 16] = s * (float)(((blk[2 + j] >> 4) & 0x0f) - 8);
            }
        } else if (dtype == 3) {
            const uint8_t* blk = w + b * Q4_1_BYTES;
            const float d = load_f16(blk), mm = load_f16(blk + 2);
            for (int j = 0; j < 16; ++j) {
                o[j] = d * (float)(blk[4 + j] & 0x0f) + mm;
                o[j + 16] = d * (float)((blk[4 + j] >> 4) & 0x0f) + mm;
            }
        } else if (dtype == 8) {
            const uint8_t* blk = w + b * Q8_0_BYTES;
            const float s = load_f16(blk);
            for (int j = 0; j < 32; ++j) o[j] = s * (float)(int8_t)blk[2 + j];
        } else {
            return 3;  // dtype mismatch
        }
    }
    return ORC_OK;
}

// kernel::dequantize_q4_0 (quantize.rs:168-197): the interleaved unpack that
// pairs with quantize_q4_0. Not used by any matmul in the reference.
void orc_dequantize_q4_0_interleaved(const uint8_t* w, int64_t n, float* out) {
    for (int64_t b = 0; b < n / QK; ++b) {
        const uint8_t* blk = w + b * Q4_0_BYTES;
        const float s = load_f16(blk);
        for (int i = 0; i < 16; ++i) {
            out[b * QK + 2 * i] = (float)((blk[2 + i] & 0x0f) - 8) * s;
            out[b * QK + 2 * i + 1] = (float)(((blk[2 + i] >> 4) & 0x0f) - 8) * s;
        }
    }
}

// Block-dot entry points for the known-answer tests (simd.rs:783-883).
float orc_dot_q8_block(const float* x, const int8_t* q, float s) { return dot_q8(x, q, s); }
int32_t orc_dot_q8q8_block(const int8_t* a, const int8_t* b) { return dot_q8q8(a, b); }
float orc_dot_q4_block(const float* x, const uint8_t* p, float s) { return dot_q4(x, p, s); }
int32_t orc_dot_q4q8_block(const uint8_t* p, const int8_t* q) { return dot_q4q8(p, q); }
void orc_dot_q4_1q8_block(const uint8_t* p, const int8_t* q, int32_t* d, int32_t* s) { dot_q4_1q8(p, q, d, s); }

// matmul_f32_q8 (quantize.rs:297-409)
int orc_matmul_f32_q8(const float* x, const uint8_t* w, int64_t m, int64_t k, int64_t n, float* y) {
    if (k % QK) return ORC_BLOCK_ALIGNMENT;
    const int64_t nb = k / QK, rb = nb * Q8_0_BYTES;
    drive(m, n, y, [&](int64_t r, int64_t c) {
        const float* xr = x + r * k;
        const uint8_t* wr = w + c * rb;
        float dot = 0.0f;
        for (int64_t b = 0; b < nb; ++b)
            dot += dot_q8(xr + b * QK, (const int8_t*)(wr + b * Q8_0_BYTES + 2), load_f16(wr + b * Q8_0_BYTES));
        return dot;
    });
    return ORC_OK;
}

// matmul_f32_q8_v2 (quantize.rs:429-530): activations through quantize_q8_0.
int orc_matmul_f32_q8_v2(const float* x, const uint8_t* w, int64_t m, int64_t k, int64_t n, float* y) {
    if (k % QK) return ORC_BLOCK_ALIGNMENT;
    const int64_t nb = k / QK, rb = nb * Q8_0_BYTES;
    std::vector<uint8_t> xq((size_t)(m * rb));
    for (int64_t b = 0; b < m * nb; ++b) quantize_q8_0_block(x + b * QK, xq.data() + b * Q8_0_BYTES);
    drive(m, n, y, [&](int64_t r, int64_t c) {
        const uint8_t* ar = xq.data() + r * rb;
        const uint8_t* wr = w + c * rb;
        float dot = 0.0f;
        for (int64_t b = 0; b < nb; ++b) {
            const float as = load_f16(ar + b * Q8_0_BYTES), ws = load_f16(wr + b * Q8_0_BYTES);
            const int32_t id = dot_q8q8((const int8_t*)(ar + b * Q8_0_BYTES + 2), (const int8_t*)(wr + b * Q8_0_BYTES + 2));
            dot += (float)id * as * ws;
        }
        return dot;
    });
    return ORC_OK;
}

// matmul_f32_q4 (quantize.rs:535-640)
int orc_matmul_f32_q4(const float* x, const uint8_t* w, int64_t m, int64_t k, int64_t n, float* y) {
    if (k % QK) return ORC_BLOCK_ALIGNMENT;
    const int64_t nb = k / QK, rb = nb * Q4_0_BYTES;
    drive(m, n, y, [&](int64_t r, int64_t c) {
        const float* xr = x + r * k;
        const uint8_t* wr = w + c * rb;
        float dot = 0.0f;
        for (int64_t b = 0; b < nb; ++b)
            dot += dot_q4(xr + b * QK, wr + b * Q4_0_BYTES + 2, load_f16(wr + b * Q4_0_BYTES));
        return dot;
    });
    return ORC_OK;
}

// Activation rows through quantize_row_q8_0 (rounded-scale variant), shared by
// the two *_native Q4 matmuls (quantize.rs:674-676, 721-723).
static void quantize_rows_rounded(const float* x, int64_t m, int64_t k, std::vector<uint8_t>& q, std::vector<float>& sc) {
    const int64_t nb = k / QK;
    q.assign((size_t)(m * nb * Q8_0_BYTES), 0);
    sc.assign((size_t)(m * nb), 0.0f);
    for (int64_t b = 0; b < m * nb; ++b) sc[b] = quantize_row_q8_0_block(x + b * QK, q.data() + b * Q8_0_BYTES);
}

// matmul_f32_q4_native (quantize.rs:646-772)
int orc_matmul_f32_q4_native(const float* x, const uint8_t* w, int64_t m, int64_t k, int64_t n, float* y) {
    if (k % QK) return ORC_BLOCK_ALIGNMENT;
    const int64_t nb = k / QK, rb = nb * Q4_0_BYTES;
    std::vector<uint8_t> xq;
    std::vector<float> xs;
    quantize_rows_rounded(x, m, k, xq, xs);
    drive(m, n, y, [&](int64_t r, int64_t c) {
        const uint8_t* wr = w + c * rb;
        float dot = 0.0f;
        for (int64_t b = 0; b < nb; ++b) {
            const float ws = load_f16(wr + b * Q4_0_BYTES);
            const int32_t id = dot_q4q8(wr + b * Q4_0_BYTES + 2, (const int8_t*)(xq.data() + (r * nb + b) * Q8_0_BYTES + 2));
            dot += (float)id * xs[r * nb + b] * ws;
        }
        return dot;
    });
    return ORC_OK;
}

// matmul_f32_q4_1 (quantize.rs:807-932): the reference computes this one with
// plain scalar loops, no SIMD dispatch.
int orc_matmul_f32_q4_1(const float* x, const uint8_t* w, int64_t m, int64_t k, int64_t n, float* y) {
    if (k % QK) return ORC_BLOCK_ALIGNMENT;
    const int64_t nb = k / QK, rb = nb * Q4_1_BYTES;
    drive(m, n, y, [&](int64_t r, int64_t c) {
        const float* xr = x + r * k;
        const uint8_t* wr = w + c * rb;
        float dot = 0.0f;
        for (int64_t b = 0; b < nb; ++b) {
            const uint8_t* blk = wr + b * Q4_1_BYTES;
            const float d = load_f16(blk), mv = load_f16(blk + 2);
            const float* xb = xr + b * QK;
            float bd = 0.0f, xsum = 0.0f;
            for (int j = 0; j < 16; ++j) {
                const float lo = (float)(blk[4 + j] & 0x0f), hi = (float)((blk[4 + j] >> 4) & 0x0f);
                bd += xb[j] * lo;
                bd += xb[j + 16] * hi;
                xsum += xb[j];
                xsum += xb[j + 16];
            }
            dot += d * bd + mv * xsum;
        }
        return dot;
    });
    return ORC_OK;
}

// matmul_f32_q4_1_native (quantize.rs:938-1070)
int orc_matmul_f32_q4_1_native(const float* x, const uint8_t* w, int64_t m, int64_t k, int64_t n, float* y) {
    if (k % QK) return ORC_BLOCK_ALIGNMENT;
    const int64_t nb = k / QK, rb = nb * Q4_1_BYTES;
    std::vector<uint8_t> xq;
    std::vector<float> xs;
    quantize_rows_rounded(x, m, k, xq, xs);
    drive(m, n, y, [&](int64_t r, int64_t c) {
        const uint8_t* wr = w + c * rb;
        float dot = 0.0f;
        for (int64_t b = 0; b < nb; ++b) {
            const uint8_t* blk = wr + b * Q4_1_BYTES;
            const float d = load_f16(blk), mv = load_f16(blk + 2);
            int32_t ud, qs;
            dot_q4_1q8(blk + 4, (const int8_t*)(xq.data() + (r * nb + b) * Q8_0_BYTES + 2), &ud, &qs);
            dot += xs[r * nb + b] * (d * (float)ud + mv * (float)qs);
        }
        return dot;
    });
    return ORC_OK;
}

}  // extern "C"
