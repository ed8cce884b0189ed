/*
 * qmm.h -- C ABI of the B200 (sm_100a) quantized-matmul library (libqmm.so).
 *
 * Drop-in device path for the quantized-matmul hot path of
 * sweengineeringlabs/machinelearning (crate swe-llmmodel-kernel, called from
 * Linear::forward). Every entry point is `extern "C"`, takes plain pointers and
 * sizes, returns a qmm_status, never throws, never aborts the process, and
 * frees only what it allocated (conventions of the reference's FFI crate,
 * llminference/main/features/inference/ffi/main/src/lib.rs:12-40).
 *
 * Reference files cited below are paths inside the reference project.
 *
 * Weights are the raw GGUF / quantizer block bytes, uploaded unchanged:
 *   Q8_0 (id 8)  34 B / 32 values  [f16 d][32 x i8]            d*q
 *   Q4_0 (id 2)  18 B / 32 values  [f16 d][16 nibble bytes]    d*(n-8)
 *   Q4_1 (id 3)  20 B / 32 values  [f16 d][f16 m][16 nibble bytes]  d*n+m
 * Nibble order is GGML's (low nibble of byte j = element j, high = j+16), the
 * order every reference matmul reads (simd.rs:30-52).
 */
#ifndef QMM_H
#define QMM_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define QMM_API __attribute__((visibility("default")))

/* Status codes. 1-4 mirror QuantError (kernel/main/src/api/error.rs:5-18). */
typedef enum qmm_status {
    QMM_OK = 0,
    QMM_ERR_BLOCK_ALIGNMENT = 1, /* in_features (or element count) not a multiple of 32 */
    QMM_ERR_SHAPE_MISMATCH = 2,  /* a buffer is shorter than the shape needs (the reference panics) */
    QMM_ERR_DTYPE_MISMATCH = 3,  /* unknown or unsupported block type */
    QMM_ERR_INVALID_DATA = 4,
    QMM_ERR_CUDA = 5,            /* a CUDA call failed; see qmm_last_error_message() */
    QMM_ERR_NCCL = 6,
    QMM_ERR_TIMEOUT = 7,         /* a bounded device-side wait gave up (see qmm_device_error) */
    QMM_ERR_INVALID_INPUT = 8,   /* null pointer, misaligned pointer, bad enum */
    QMM_ERR_NO_DEVICE = 9        /* no CUDA device / the library's kernels cannot run here */
} qmm_status;

/* Block types (GGML ids, gguf/main/src/api/types.rs:8-12). */
typedef enum qmm_dtype { QMM_Q4_0 = 2, QMM_Q4_1 = 3, QMM_Q8_0 = 8 } qmm_dtype;

/* Activation handling, the reference's Linear flags (linear.rs:24-29):
 *   QMM_ACT_F32  : f32 activations x dequantised weights   (matmul_f32_q4 / _q8 / _q4_1)
 *   QMM_ACT_Q8_0 : activations quantised to Q8_0, integer block dots
 *                  (matmul_f32_q4_native / _q8_v2 / _q4_1_native; use_native_q4/q8 = true).
 *                  Q8_0 weights use quantize_q8_0 (quantize.rs:451), Q4 weights use
 *                  quantize_row_q8_0 (quantize.rs:676), exactly as the reference. */
typedef enum qmm_act { QMM_ACT_F32 = 0, QMM_ACT_Q8_0 = 1 } qmm_act;

QMM_API int qmm_version(void);
QMM_API const char* qmm_status_string(int status);
/* Detail of the last failing call on this host thread ("" if none). */
QMM_API const char* qmm_last_error_message(void);
/* Number of CUDA devices the library can use (0 on a host without GPUs). */
QMM_API int qmm_device_count(void);
/* Reads and clears the device-side error word of `device` (0 = none, 1 = a
 * bounded wait timed out). Synchronises the device. */
QMM_API int qmm_device_error(int device, int* out_error);
/* The same check as a status: synchronises `device`, reads and clears its
 * error word, and returns QMM_OK, or QMM_ERR_TIMEOUT when a bounded wait of a
 * kernel gave up since the last check (the reference's FFI turns every
 * failure into a code, ffi/main/src/lib.rs:15-21). */
QMM_API int qmm_device_status(int device);
/* Launches, on `stream`, one wait on a shared-memory barrier that nothing
 * completes, bounded to `probes` probes (1..2^20) instead of the library's
 * 2^20, after which the kernel records a timeout in the error word and
 * returns, as every wait of the hot path does. For testing the timeout path
 * without hanging or faulting a GPU: qmm_device_status then reports
 * QMM_ERR_TIMEOUT and the context stays usable. No counterpart in the
 * reference (a CPU library). */
QMM_API int qmm_selftest_bounded_wait(unsigned probes, void* stream);
/* Number of kernel launches this library has issued in this process (stream
 * captures included), for launch accounting in benchmarks. No counterpart in
 * the reference (a CPU library). */
QMM_API unsigned long long qmm_launch_count(void);

/* ------------------------------------------------------------------------
 * Reference-signature host entry points. Host buffers in, host buffers out,
 * exactly the arguments of the Rust functions they replace; `output` holds
 * m*out_features floats. Each call runs on the current CUDA device and
 * synchronises. If `weight_bytes` was registered with
 * qmm_register_host_weight(), its resident device copy is used; otherwise the
 * weights are copied to the device for this call.
 * ------------------------------------------------------------------------ */
/* matmul_f32_q8 (quantize.rs:297-303) */
QMM_API int qmm_matmul_f32_q8(const float* input_data, size_t input_len, const uint8_t* weight_bytes,
                              size_t weight_len, size_t m, size_t in_features, size_t out_features,
                              float* output);
/* matmul_f32_q8_v2 (quantize.rs:429-435) */
QMM_API int qmm_matmul_f32_q8_v2(const float* input_data, size_t input_len, const uint8_t* weight_bytes,
                                 size_t weight_len, size_t m, size_t in_features, size_t out_features,
                                 float* output);
/* matmul_f32_q4 (quantize.rs:535-541) */
QMM_API int qmm_matmul_f32_q4(const float* input_data, size_t input_len, const uint8_t* weight_bytes,
                              size_t weight_len, size_t m, size_t in_features, size_t out_features,
                              float* output);
/* matmul_f32_q4_native (quantize.rs:646-652) */
QMM_API int qmm_matmul_f32_q4_native(const float* input_data, size_t input_len, const uint8_t* weight_bytes,
                                     size_t weight_len, size_t m, size_t in_features, size_t out_features,
                                     float* output);
/* matmul_f32_q4_1 (quantize.rs:807-813) */
QMM_API int qmm_matmul_f32_q4_1(const float* input_data, size_t input_len, const uint8_t* weight_bytes,
                                size_t weight_len, size_t m, size_t in_features, size_t out_features,
                                float* output);
/* matmul_f32_q4_1_native (quantize.rs:938-944) */
QMM_API int qmm_matmul_f32_q4_1_native(const float* input_data, size_t input_len, const uint8_t* weight_bytes,
                                       size_t weight_len, size_t m, size_t in_features, size_t out_features,
                                       float* output);

/* quantize_q8_0 (quantize.rs:15-48): n % 32 == 0, out holds n/32*34 bytes. */
QMM_API int qmm_quantize_q8_0(const float* data, size_t n, uint8_t* out);
/* quantize_q4_0 (quantize.rs:124-165, interleaved nibble packing as the reference writes it). */
QMM_API int qmm_quantize_q4_0(const float* data, size_t n, uint8_t* out);
/* quantize_q4_1 (quantize.rs:207-251). */
QMM_API int qmm_quantize_q4_1(const float* data, size_t n, uint8_t* out);
/* quantize_row_q8_0 (quantize.rs:260-289): also writes the f32(f16) scales (n/32 floats). */
QMM_API int qmm_quantize_row_q8_0(const float* input, size_t n, uint8_t* out, float* scales);
/* Tensor::to_f32 for block types (tensor.rs:527-630; Q4_0 in GGML order). */
QMM_API int qmm_dequantize(int dtype, const uint8_t* raw, size_t raw_len, size_t n_elements, float* out);

/* Registers a host weight buffer (e.g. an mmap'd GGUF tensor, tensor.rs:405-414)
 * whose bytes are uploaded once to the current device and reused by the
 * reference-signature calls above for as long as it stays registered. The
 * caller must not change those bytes while registered. */
QMM_API int qmm_register_host_weight(const uint8_t* weight_bytes, size_t weight_len, int dtype, size_t n, size_t k);
QMM_API int qmm_unregister_host_weight(const uint8_t* weight_bytes);

/* ------------------------------------------------------------------------
 * Device API (the hot path). Pointers ending in _dev are device pointers;
 * `stream` is a cudaStream_t (NULL = legacy default stream). Calls are
 * asynchronous on `stream` and do not synchronise.
 * ------------------------------------------------------------------------ */
typedef struct qmm_weight qmm_weight;

/* Uploads an [n, k] block matrix (n rows of k/32 blocks, the GGUF layout) to
 * `device` with one host-to-device copy, byte for byte, no repacking. */
QMM_API int qmm_weight_create(int dtype, size_t n, size_t k, const uint8_t* host_bytes, size_t len, int device,
                              qmm_weight** out);
/* Same, from bytes already on `device` (device-to-device copy). */
QMM_API int qmm_weight_create_from_device(int dtype, size_t n, size_t k, const uint8_t* dev_bytes, size_t len,
                                          int device, qmm_weight** out);
QMM_API int qmm_weight_destroy(qmm_weight* w);
QMM_API int qmm_weight_info(const qmm_weight* w, int* dtype, size_t* n, size_t* k, const uint8_t** dev_bytes,
                            int* device);

/* Activation functions (qmm_gated_forward: GELU and SiLU; qmm_gated_act_dev:
 * all three). */
#define QMM_GELU 0
#define QMM_SILU 1
#define QMM_RELU 2

/* Fused projections (reference: Attention::fuse_qkv_weights,
 * llmserve/llmmodel/layers/main/src/core/attention.rs:306-339, and
 * FeedForward::fuse_gate_up_weights, feed_forward.rs:147-187).
 *
 * qmm_weight_fuse_rows: a new weight whose bytes are the parts' bytes
 * concatenated in order (rows = sum of the parts' rows), as the reference's
 * fused QKV / gate+up tensors are; y of the fused weight is the parts' outputs
 * side by side. Parts: same block type (Q8_0, Q4_0 or Q4_1; the reference fuses
 * Q8_0 only), same in_features, same device. The parts stay valid.
 *
 * qmm_weight_fuse_gate_up: a gate/up weight for qmm_gated_forward. Same rules,
 * plus gate and up of equal shape [hidden, k]. Its rows interleave gate and up
 * in groups of 16 (rows 32j..32j+15 = gate rows 16j.., rows 32j+16..32j+31 = up
 * rows 16j..), zero rows padding hidden to a multiple of 16, so one output tile
 * of the matmul holds matching gate and up values. qmm_linear_forward rejects
 * it; qmm_weight_gate_hidden reports hidden (0 for an ordinary weight).
 *
 * qmm_gated_forward: out_dev[m][hidden] = act(x . gate^T) * (x . up^T), act =
 * QMM_GELU or QMM_SILU, the activation applied in the matmul's epilogue (one
 * launch for decode shapes). The matmul is the f32-activation form for every
 * block type, as the reference's fused Linear (use_native_* false). */
QMM_API int qmm_weight_fuse_rows(const qmm_weight* const* parts, size_t count, qmm_weight** out);
QMM_API int qmm_weight_fuse_gate_up(const qmm_weight* gate, const qmm_weight* up, qmm_weight** out);
QMM_API int qmm_weight_gate_hidden(const qmm_weight* w, size_t* hidden);
QMM_API int qmm_gated_forward(const qmm_weight* w, const float* x_dev, size_t m, float* out_dev, int act_fn,
                              void* stream);

/* 64-bit position-weighted checksum of device bytes: the sum over their
 * little-endian 32-bit words w_i (the tail zero-padded) of w_i * (2i + 1),
 * modulo 2^64 -- for verifying that an upload (a GGUF tensor's file range,
 * reference gguf/main/src/core/parser.rs:501-576) arrived byte for byte.
 * Synchronous. qmm_checksum_dev: data_dev 4-byte aligned, on the current
 * device. No counterpart in the reference (its mmap path has no device copy
 * to verify). */
QMM_API int qmm_checksum_dev(const void* data_dev, size_t len, void* stream, unsigned long long* out);
QMM_API int qmm_weight_checksum(const qmm_weight* w, unsigned long long* out);

/* y_dev[m, n] = x_dev[m, k] . W^T on the weight's device, workspace managed by
 * the library (one buffer per device and stream, grown on demand with
 * cudaMalloc; grow it with qmm_reserve_workspace before capturing a graph). */
QMM_API int qmm_linear_forward(const qmm_weight* w, const float* x_dev, size_t m, float* y_dev, int act,
                               void* stream);
/* Host-buffer variant of qmm_linear_forward: copies x in and y out on `stream`
 * (pinned buffers make the copies asynchronous) and synchronises the stream. */
QMM_API int qmm_linear_forward_host(const qmm_weight* w, const float* x_host, size_t m, float* y_host, int act,
                                    void* stream);
QMM_API int qmm_reserve_workspace(int device, void* stream, size_t bytes);

/* Fully caller-managed form: raw device weight bytes and a caller workspace of
 * at least qmm_workspace_size() bytes (256-byte aligned, not shared by
 * concurrent calls). w_dev must be 16-byte aligned. */
QMM_API size_t qmm_workspace_size(int dtype, int act, size_t m, size_t n, size_t k);
QMM_API int qmm_matmul_dev(int dtype, int act, const float* x_dev, const uint8_t* w_dev, size_t w_len, size_t m,
                           size_t k, size_t n, float* y_dev, void* workspace_dev, size_t workspace_bytes,
                           void* stream);

/* Allocation-free form of qmm_matmul_dev (no counterpart in the reference, which
 * has no device code). For callers that may not allocate device memory: a
 * plugin whose host framework owns the device memory pool, or a serving loop
 * that cannot take cudaMalloc's implicit device-wide synchronisation. The
 * workspace is a fixed 4 MiB device array inside the library
 * (QMM_NOALLOC_SCRATCH_BYTES; held by every device that loads the library until
 * the process exits); shapes whose workspace does not fit are rejected with
 * QMM_ERR_INVALID_INPUT. The first call on a device, with that device current,
 * looks the array's address up (make it before any stream capture). The array
 * is shared: calls that overlap on the GPU race, so keep them ordered (one
 * stream, or explicit synchronisation). It runs the GEMV kernels only (rows
 * in chunks of at most 64): calls with 17 or more rows of f32 activations,
 * which qmm_matmul_dev sends to the tensor-core GEMM, are slower here.
 * Arguments as qmm_matmul_dev. */
#define QMM_NOALLOC_SCRATCH_BYTES (4u << 20)
QMM_API int qmm_matmul_dev_noalloc(int dtype, int act, const float* x_dev, const uint8_t* w_dev, size_t w_len,
                                   size_t m, size_t k, size_t n, float* y_dev, void* stream);

/* Device quantisers, bit-identical to the reference's:
 *   variant 0: quantize_q8_0   (unrounded inverse scale), dtype QMM_Q8_0
 *   variant 1: quantize_row_q8_0 (f16-rounded inverse scale), dtype QMM_Q8_0; scales_dev optional
 *   dtype QMM_Q4_0 / QMM_Q4_1: quantize_q4_0 / quantize_q4_1 (variant ignored). */
QMM_API int qmm_quantize_dev(int dtype, int variant, const float* x_dev, size_t n, uint8_t* out_dev,
                             float* scales_dev, void* stream);
/* Device dequantiser with Tensor::to_f32 semantics. */
QMM_API int qmm_dequantize_dev(int dtype, const uint8_t* w_dev, size_t w_len, size_t n_elements, float* out_dev,
                               void* stream);

/* Element-wise activation step of FeedForward::forward (reference
 * layers/main/src/core/feed_forward.rs:198-251), for gate and up produced by
 * separate matmuls or by one matmul over qmm_weight_fuse_rows(gate, up):
 * out_dev[m][hidden] = act(gate_dev[i * ld + j]) * up_dev[i * ld + j], in f32,
 * act = QMM_GELU (tanh approximation), QMM_SILU or QMM_RELU; up_dev may be null
 * (the ungated activations: out = act(gate)). ld >= hidden is the row stride of
 * gate and up in elements (2 * hidden for the [gate | up] output of a fused
 * weight, with up_dev = gate_dev + hidden). Launched with programmatic
 * dependent launch, so it overlaps the tail of the matmul before it. */
QMM_API int qmm_gated_act_dev(int act_fn, const float* gate_dev, const float* up_dev, size_t m, size_t hidden,
                              size_t ld, float* out_dev, void* stream);

/* ---- Decode-step pieces around the matmuls (device pointers, stream-ordered).
 * A Gemma-3 decode step is these plus the matmuls above (fused QKV, fused
 * gate/up with the GeGLU epilogue, o, down, lm_head). The reference runs them
 * on f32 host tensors; each entry cites the Rust code it replaces.
 * The decode position is read from device memory (pos_dev) so a captured step
 * can be replayed while qmm_add_int_dev advances it. */

/* x[b] = scale * dequant(emb row tokens[b]) from a Q8_0 [vocab][hidden] tied
 * embedding; token ids are clamped to [0, vocab). Replaces TokenEmbedding::
 * forward + mul_scalar(embedding_scale) (model/main/src/core/forward.rs:122-127). */
QMM_API int qmm_embed_q8_dev(const uint8_t* emb_dev, size_t vocab, size_t hidden, const int* tokens_dev,
                             size_t batch, float scale, float* x_dev, void* stream);
/* y = x / sqrt(mean(x^2) + eps) * (w + offset) per row; y rows ld_y floats
 * apart (0: dim; wider rows keep their tail). Replaces RMSNorm::forward
 * (layers/main/src/core/rms_norm.rs:66-85, tensor math.rs:334-380). */
QMM_API int qmm_rmsnorm_dev(const float* x_dev, const float* w_dev, float offset, float eps, size_t rows, size_t dim,
                            float* y_dev, size_t ld_y, void* stream);
/* x += rmsnorm(branch, w_post); then (w_next non-null) h = rmsnorm(x, w_next),
 * h rows ld_h floats apart (0: dim): a sandwich post-norm and residual add
 * fused with the next pre-norm (layers/main/src/core/transformer_block.rs:424-449). */
QMM_API int qmm_residual_rmsnorm_dev(float* x_dev, const float* branch_dev, const float* w_post_dev,
                                     const float* w_next_dev, float offset, float eps, size_t rows, size_t dim,
                                     float* h_dev, size_t ld_h, void* stream);
/* From fused q|k|v rows [batch][(n_heads + 2 n_kv_heads) head_dim]: per-head
 * RMSNorm of q and k, half-split RoPE with cos/sin tables [ctx][head_dim/2]
 * at position *pos_dev; q into q_out [batch][n_heads][head_dim], k and v into
 * the caches [batch][n_kv_heads][ctx][head_dim] at that position. head_dim a
 * multiple of 64, at most 256 (layers/main/src/core/attention.rs:505-540,
 * rope.rs:7-130). */
QMM_API int qmm_qk_rope_cache_dev(const float* qkv_dev, size_t batch, int n_heads, int n_kv_heads, int head_dim,
                                  const float* q_norm_dev, const float* k_norm_dev, float offset, float eps,
                                  const float* cos_dev, const float* sin_dev, const int* pos_dev, int ctx,
                                  float* q_out_dev, float* k_cache_dev, float* v_cache_dev, void* stream);
/* Floats of the partial-result buffer qmm_attention_decode_dev needs. */
QMM_API size_t qmm_attention_partial_floats(size_t batch, int n_heads, int head_dim, int ctx);
/* Single-token attention over cache positions 0..*pos_dev: scores q.k *
 * inv_scale, softmax, weighted sum of v; grouped-query heads share their kv
 * head. out [batch][n_heads * head_dim]. At most 8 heads and head_dim 256
 * (layers/main/src/core/attention.rs:545-600, decode: no mask). */
QMM_API int qmm_attention_decode_dev(const float* q_dev, const float* k_cache_dev, const float* v_cache_dev,
                                     size_t batch, int n_heads, int n_kv_heads, int head_dim, const int* pos_dev,
                                     int ctx, float inv_scale, float* partial_dev, float* out_dev, void* stream);
/* qmm_qk_rope_cache_dev and qmm_attention_decode_dev in one pass (one launch
 * fewer per layer): every attention CTA normalises and rotates the q heads
 * itself; the one holding the position writes k and v to the caches. Same
 * arguments and limits (context at most 2048). */
QMM_API int qmm_attention_decode_fused_dev(const float* qkv_dev, size_t batch, int n_heads, int n_kv_heads,
                                           int head_dim, const float* q_norm_dev, const float* k_norm_dev, float offset,
                                           float eps, const float* cos_dev, const float* sin_dev, const int* pos_dev,
                                           int ctx, float* k_cache_dev, float* v_cache_dev, float inv_scale,
                                           float* partial_dev, float* out_dev, void* stream);
/* *p_dev += value, stream-ordered (advances a captured step's position). */
QMM_API int qmm_add_int_dev(int* p_dev, int value, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* QMM_H */
