/* Tensor-parallel quantised linears over NCCL (libqmm.so).
 *
 * The reference has no distributed code: every output of its quantised
 * matmul is an independent dot product over whole 32-weight blocks
 * (llmserve/llmmodel/kernel/main/src/core/quantize.rs:458-484), which is what
 * makes these shardings valid. The entry points extend the C-ABI of
 * include/qmm.h under the reference FFI crate's conventions
 * (llminference/main/features/inference/ffi/main/src/lib.rs:12-21): status
 * codes instead of panics, null checks on every pointer, opaque handles, the
 * library frees what it allocates.
 *
 * NCCL is loaded at run time (dlopen of libnccl.so.2, or the path in the
 * QMM_NCCL_LIBRARY environment variable), so libqmm.so itself has no link
 * dependency on it; a process that already holds an NCCL (PyTorch's) gets
 * that one. Communicators are created non-blocking: every wait on NCCL is a
 * host-side poll of ncclCommGetAsyncError with a time limit, and a failure or
 * a limit that runs out aborts the communicator (ncclCommAbort) and returns
 * QMM_ERR_NCCL or QMM_ERR_TIMEOUT. After that the handle only accepts
 * qmm_tp_destroy; every other call returns QMM_ERR_NCCL.
 *
 * Shardings (rank r of W):
 *   column-parallel (q / k / v / gate / up / lm_head): output rows
 *     [r*N/W, (r+1)*N/W), a contiguous byte range of the GGUF tensor
 *     (qmm_weight_create on host_bytes + r*N/W*row_bytes). The join is an
 *     all-gather; outputs are bit-identical to one GPU.
 *   row-parallel (o / down): blocks [r*nb/W, (r+1)*nb/W) of every row
 *     (qmm_weight_create_row_shard: one strided copy, blocks byte-for-byte).
 *     The join is an all-reduce (sum): results agree within f32 rounding.
 *   Megatron pairing: column-parallel gate/up shards fused with
 *     qmm_weight_fuse_gate_up, qmm_gated_forward on the shard, then
 *     qmm_tp_row_forward on the local hidden slice: one all-reduce per FFN.
 */
#ifndef QMM_TP_H
#define QMM_TP_H

#include <stddef.h>
#include <stdint.h>

#include "qmm.h"

#ifdef __cplusplus
extern "C" {
#endif

#define QMM_TP_UNIQUE_ID_BYTES 128 /* sizeof(ncclUniqueId) */

typedef struct qmm_tp_comm qmm_tp_comm;

/* 1 when an NCCL library can be loaded (0 otherwise; never an error). */
QMM_API int qmm_tp_available(void);

/* ncclGetUniqueId on the calling process (rank 0), to be sent to every rank. */
QMM_API int qmm_tp_unique_id(uint8_t out[QMM_TP_UNIQUE_ID_BYTES]);

/* Joins communicator `id` as `rank` of `world` on CUDA device `device` (-1:
 * the calling thread's current device). Non-blocking init, polled until it
 * completes or `timeout_s` seconds pass (then: abort, QMM_ERR_TIMEOUT). */
QMM_API int qmm_tp_init(const uint8_t id[QMM_TP_UNIQUE_ID_BYTES], int world, int rank, int device,
                        double timeout_s, qmm_tp_comm** out);

/* Frees the handle (ncclCommDestroy, or nothing more after an abort).
 * Null is a no-op. */
QMM_API int qmm_tp_destroy(qmm_tp_comm* comm);

/* ncclCommAbort: ends in-flight collectives of this communicator. */
QMM_API int qmm_tp_abort(qmm_tp_comm* comm);

QMM_API int qmm_tp_rank(const qmm_tp_comm* comm, int* rank, int* world);

/* Joins over peer memory instead of NCCL collectives (collective; every rank
 * calls it once, after qmm_tp_init). Each rank allocates a flag array and two
 * join buffers of `bytes` each and maps every other rank's through CUDA IPC
 * (NVLink peer access; the handles travel through the communicator). From
 * then on, qmm_tp_column_forward / qmm_tp_row_forward whose joined result fits
 * in `bytes` write it straight into every rank's buffer -- from the producing
 * kernel's own epilogue where that kernel supports it (the band GEMV and the
 * f16 tensor-core GEMM), else by a copy kernel -- and one join kernel per call
 * stores this rank's epoch into every peer's flags (release, system scope),
 * waits for every peer's (acquire; bounded by the communicator's time limit)
 * and reads the buffer out into y: a copy (column), or the sum over ranks in
 * rank order (row; every rank then holds identical bits). Calls that do not
 * fit, or that run under stream capture, join through NCCL as before. A
 * join waits at most `join_timeout_s` seconds for a peer's signal (<= 0: the
 * communicator's time limit); one whose wait runs out records it on the
 * device, and the next qmm_tp_wait returns QMM_ERR_TIMEOUT and aborts the
 * communicator. At most 8 ranks. */
QMM_API int qmm_tp_enable_peer(qmm_tp_comm* comm, size_t bytes, double join_timeout_s);

/* One poll of ncclCommGetAsyncError: QMM_OK, or (after an abort)
 * QMM_ERR_NCCL with the NCCL error string in qmm_last_error_message(). */
QMM_API int qmm_tp_status(qmm_tp_comm* comm);

/* Waits for everything enqueued on `stream` (cudaStream_t; null = legacy
 * stream), polling the communicator's error state, for at most `timeout_s`
 * seconds: QMM_OK, QMM_ERR_NCCL (aborted) or QMM_ERR_TIMEOUT (aborted). */
QMM_API int qmm_tp_wait(qmm_tp_comm* comm, void* stream, double timeout_s);

/* Blocks [rank*nb/world, (rank+1)*nb/world) of every row of an [n][k]
 * tensor (nb = k/32 divisible by world) as a weight of n rows and k/world
 * columns: one strided host-to-device copy, blocks byte-for-byte. */
QMM_API int qmm_weight_create_row_shard(int dtype, size_t n, size_t k, const uint8_t* host_bytes, size_t len,
                                        int rank, int world, int device, qmm_weight** out);

/* Column-parallel forward: y_dev [m][world * shard->n] on every rank from
 * x_dev [m][shard->k] (the full activations) and this rank's output rows.
 * The local product runs through qmm_linear_forward, then one all-gather
 * (m > 1: into a rank-major buffer and a reorder kernel). Enqueued on
 * `stream`; completion and errors through qmm_tp_wait / qmm_tp_status. */
QMM_API int qmm_tp_column_forward(qmm_tp_comm* comm, const qmm_weight* shard, const float* x_dev, size_t m,
                                  float* y_dev, int act, void* stream);

/* Row-parallel forward: y_dev [m][shard->n], the sum over ranks, from this
 * rank's K slice x_local_dev [m][shard->k] (columns [rank*K/world, ...) of the
 * full activations, or a Megatron-paired hidden slice). One all-reduce. */
QMM_API int qmm_tp_row_forward(qmm_tp_comm* comm, const qmm_weight* shard, const float* x_local_dev, size_t m,
                               float* y_dev, int act, void* stream);

/* An in-place all-gather / all-reduce (sum) of f32 buffers on `stream`, for
 * callers that join their own products (count = elements per rank). */
QMM_API int qmm_tp_all_gather_f32(qmm_tp_comm* comm, const float* send_dev, float* recv_dev, size_t count,
                                  void* stream);
QMM_API int qmm_tp_all_reduce_f32(qmm_tp_comm* comm, float* buf_dev, size_t count, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* QMM_TP_H */
