// Tensor-parallel C ABI of libqmm.so (declared in include/qmm_tp.h): NCCL
// communicators with host-side time limits, and the column-/row-parallel
// quantised linears on top of the single-GPU entry points of include/qmm.h.
//
// NCCL is resolved with dlopen at the first use, so the library links no NCCL
// and a process that already loaded one (PyTorch's libnccl.so.2) shares it.
// Every communicator is created non-blocking (ncclConfig_t.blocking = 0):
// nothing here ever blocks inside NCCL. Waits are host polls of
// ncclCommGetAsyncError (and cudaStreamQuery) with a time limit; an NCCL error
// or a limit that runs out aborts the communicator (ncclCommAbort, which also
// ends its kernels still in flight) and returns QMM_ERR_NCCL / QMM_ERR_TIMEOUT,
// the reference FFI's "errors become codes" convention
// (llminference/main/features/inference/ffi/main/src/lib.rs:12-21).
#include <dlfcn.h>
#include <nccl.h>

#include <algorithm>
#include <atomic>
#include <chrono>
#include <cstdlib>
#include <cstring>
#include <mutex>
#include <string>
#include <thread>
#include <vector>

#include "../../include/qmm.h"
#include "../../include/qmm_tp.h"
#include "qmm_common.cuh"
#include "qmm_kernels.cuh"

namespace qmm {
int set_last_error(int status, const std::string& msg);
void note_launch();
}  // namespace qmm

static_assert(sizeof(ncclUniqueId) == QMM_TP_UNIQUE_ID_BYTES, "unique id size");

namespace {

using Clock = std::chrono::steady_clock;

int fail(int status, const std::string& msg) { return qmm::set_last_error(status, msg); }

// ---- NCCL entry points, resolved at run time ---------------------------------------
struct NcclApi {
    bool ok = false;
    std::string why;
    ncclResult_t (*GetUniqueId)(ncclUniqueId*) = nullptr;
    ncclResult_t (*CommInitRankConfig)(ncclComm_t*, int, ncclUniqueId, int, ncclConfig_t*) = nullptr;
    ncclResult_t (*CommGetAsyncError)(ncclComm_t, ncclResult_t*) = nullptr;
    ncclResult_t (*CommAbort)(ncclComm_t) = nullptr;
    ncclResult_t (*CommFinalize)(ncclComm_t) = nullptr;
    ncclResult_t (*CommDestroy)(ncclComm_t) = nullptr;
    ncclResult_t (*AllGather)(const void*, void*, size_t, ncclDataType_t, ncclComm_t, cudaStream_t) = nullptr;
    ncclResult_t (*AllReduce)(const void*, void*, size_t, ncclDataType_t, ncclRedOp_t, ncclComm_t,
                              cudaStream_t) = nullptr;
    const char* (*GetErrorString)(ncclResult_t) = nullptr;
};

template <class F>
bool bind(void* h, const char* name, F& fn) {
    fn = reinterpret_cast<F>(dlsym(h, name));
    return fn != nullptr;
}

NcclApi load_nccl() {
    NcclApi a;
    const char* env = std::getenv("QMM_NCCL_LIBRARY");
    void* h = nullptr;
    if (env && *env) {
        h = dlopen(env, RTLD_NOW | RTLD_LOCAL);
    } else {
        h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_LOCAL);
        if (!h) h = dlopen("libnccl.so", RTLD_NOW | RTLD_LOCAL);
    }
    if (!h) {
        const char* e = dlerror();
        a.why = std::string("cannot load NCCL: ") + (e ? e : "unknown");
        return a;
    }
    bool ok = bind(h, "ncclGetUniqueId", a.GetUniqueId) && bind(h, "ncclCommInitRankConfig", a.CommInitRankConfig) &&
              bind(h, "ncclCommGetAsyncError", a.CommGetAsyncError) && bind(h, "ncclCommAbort", a.CommAbort) &&
              bind(h, "ncclCommFinalize", a.CommFinalize) && bind(h, "ncclCommDestroy", a.CommDestroy) &&
              bind(h, "ncclAllGather", a.AllGather) && bind(h, "ncclAllReduce", a.AllReduce) &&
              bind(h, "ncclGetErrorString", a.GetErrorString);
    if (!ok) {
        a.why = "the NCCL library lacks a needed entry point";
        return a;
    }
    a.ok = true;
    return a;
}

const NcclApi& nccl() {
    static const NcclApi api = load_nccl();
    return api;
}

std::string nccl_str(ncclResult_t r) {
    const char* s = nccl().GetErrorString ? nccl().GetErrorString(r) : nullptr;
    return s ? s : ("NCCL error " + std::to_string((int)r));
}

double seconds_since(Clock::time_point t0) {
    return std::chrono::duration<double>(Clock::now() - t0).count();
}

// Pause between polls: yield for the first 2 ms of a wait (a collective's
// enqueue on a non-blocking communicator settles in tens of microseconds, and a
// sleeping poll would add the timer's granularity to every call), then sleep.
void poll_pause(Clock::time_point t0) {
    if (seconds_since(t0) < 2e-3) std::this_thread::yield();
    else std::this_thread::sleep_for(std::chrono::microseconds(100));
}

struct DevGuard {
    int prev = -1;
    bool ok = true;
    explicit DevGuard(int dev) {
        if (dev < 0) return;
        if (cudaGetDevice(&prev) != cudaSuccess) prev = -1;
        if (dev != prev) ok = cudaSetDevice(dev) == cudaSuccess;
    }
    ~DevGuard() {
        int cur = -1;
        if (prev >= 0 && cudaGetDevice(&cur) == cudaSuccess && cur != prev) cudaSetDevice(prev);
    }
};

// Rank-major [world][m][nl] -> [m][world * nl].
__global__ void tp_reorder_kernel(const float* __restrict__ g, float* __restrict__ y, int m, int nl, int world) {
    const int64_t total = (int64_t)m * nl * world;
    const int64_t row = (int64_t)nl * world;
    for (int64_t o = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; o < total; o += (int64_t)gridDim.x * blockDim.x) {
        const int64_t i = o / row, c = o - i * row;
        const int64_t r = c / nl, j = c - r * nl;
        y[o] = g[(r * m + i) * nl + j];
    }
}

// ---- joins over peer memory (qmm_tp_enable_peer) ------------------------------------
// Every rank owns one allocation, mapped into every other rank's address space
// (CUDA IPC over NVLink): [flags: one u64 per rank][error word][epoch][ticket]
// [buffer 0][buffer 1]. The epoch lives on the device: the join kernel reads
// it, and the last of its CTAs advances it, so a captured sequence of joins
// replays correctly. A join of epoch e writes rank s's part into buffer e % 2
// of every rank --
// from the producing kernel's epilogue (band GEMV, f16 GEMM) or, for other
// kernels, tp_push_kernel -- then tp_join_kernel stores e into flags[s] of
// every peer (release, system scope), waits until its own flags[r] >= e for
// every peer r (acquire, bounded by a time limit), and reads its buffer out
// into y (column: a copy; row: the sum over ranks in rank order, so every rank
// holds the same bits). Two buffers suffice: a rank writes epoch e + 1 only
// after it saw every peer's flag e, which each peer stores after it has read
// out its epoch e - 1 buffer (stream order).
constexpr size_t kFlagsOff = 0, kErrOff = 64, kEpochOff = 128, kTicketOff = 192, kBufOff = 256;

__device__ __forceinline__ uint64_t ld_acquire_sys(const uint64_t* p) {
    uint64_t v;
    asm volatile("ld.acquire.sys.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
    return v;
}
__device__ __forceinline__ void st_release_sys(uint64_t* p, uint64_t v) {
    asm volatile("st.release.sys.global.u64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}
__device__ __forceinline__ uint64_t global_ns() {
    uint64_t t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}

// Copies this rank's [rows][cols] result into every rank's buffer (row stride ld).
struct PushArgs {
    qmm::PeerDst to;
    const float* src;
    int64_t rows, cols;
};
__global__ void tp_push_kernel(const __grid_constant__ PushArgs a) {
    const int64_t total = a.rows * a.cols;
    const int64_t boff = qmm::peer_buffer_offset(a.to);
    for (int64_t o = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; o < total; o += (int64_t)gridDim.x * blockDim.x) {
        const int64_t i = o / a.cols, j = o - i * a.cols;
        const float v = a.src[o];
#pragma unroll
        for (int r = 0; r < qmm::kMaxPeers; ++r)
            if (r < a.to.n) a.to.dst[r][boff + i * a.to.ld + j] = v;
    }
}

struct JoinArgs {
    uint64_t* signal[qmm::kMaxPeers];  // &flags[rank] in rank r's allocation (null for this rank)
    const uint64_t* flags;             // this rank's flags
    int* errw;                         // this rank's error word
    unsigned long long* epoch;         // this rank's epoch (joins completed)
    unsigned* ticket;                  // CTAs done, zero between joins
    const float* buf;                  // this rank's buffer 0 (buffer 1 at + pstride)
    int64_t pstride;
    float* y;
    int64_t count;  // elements of y (row join: also of each rank's slot)
    long long limit_ns;
    int world, rank, reduce, vec4;
};
__global__ void tp_join_kernel(const __grid_constant__ JoinArgs a) {
    // every CTA reads the epoch before the last one to finish advances it
    const uint64_t e = __ldcg(a.epoch) + 1ull;
    // everything this rank wrote for the epoch precedes this kernel in stream
    // order; the release below publishes it to the peers
    if (blockIdx.x == 0 && threadIdx.x < (unsigned)a.world && (int)threadIdx.x != a.rank) {
        __threadfence_system();
        st_release_sys(a.signal[threadIdx.x], e);
    }
    __shared__ int ok;
    if (threadIdx.x == 0) {
        int good = 1;
        const uint64_t t0 = global_ns();
        for (int r = 0; r < a.world && good; ++r) {
            if (r == a.rank) continue;
            while (ld_acquire_sys(a.flags + r) < e) {
                if ((long long)(global_ns() - t0) > a.limit_ns) {
                    good = 0;
                    atomicExch(a.errw, 1);
                    break;
                }
                __nanosleep(128);
            }
        }
        ok = good;
    }
    __syncthreads();
    const int64_t stride = (int64_t)gridDim.x * blockDim.x;
    const int64_t t = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    const float* buf = a.buf + (int64_t)(e & 1ull) * a.pstride;
    if (!ok) {
        // y is left as it was; the host reads the error word
    } else if (a.vec4) {
        const float4* b4 = reinterpret_cast<const float4*>(buf);
        float4* y4 = reinterpret_cast<float4*>(a.y);
        const int64_t n4 = a.count / 4;
        for (int64_t i = t; i < n4; i += stride) {
            float4 s = __ldcg(b4 + i);
            for (int r = 1; a.reduce && r < a.world; ++r) {
                const float4 v = __ldcg(b4 + r * n4 + i);
                s.x += v.x;
                s.y += v.y;
                s.z += v.z;
                s.w += v.w;
            }
            y4[i] = s;
        }
    } else {
        for (int64_t i = t; i < a.count; i += stride) {
            float s = __ldcg(buf + i);
            for (int r = 1; a.reduce && r < a.world; ++r) s += __ldcg(buf + r * a.count + i);
            a.y[i] = s;
        }
    }
    // the last CTA to finish advances the epoch (and leaves the ticket zero)
    __syncthreads();
    if (threadIdx.x == 0) {
        __threadfence();
        if (atomicAdd(a.ticket, 1u) == gridDim.x - 1) {
            *a.ticket = 0u;
            *a.epoch = e;
            __threadfence();
        }
    }
}

}  // namespace

struct qmm_tp_comm {
    ncclComm_t comm = nullptr;
    int rank = 0, world = 1, device = 0;
    double timeout_s = 60.0;
    std::atomic<int> aborted{0};
    std::mutex mu;  // guards the gather buffer
    float* gbuf = nullptr;
    size_t gbytes = 0;
    // joins over peer memory
    uint8_t* xmem = nullptr;                   // this rank's allocation
    uint8_t* pmem[qmm::kMaxPeers] = {};        // every rank's allocation as mapped here (own included)
    size_t cap = 0;                            // bytes per buffer
    double join_timeout_s = 60.0;              // a join's wait for the peers' signals
    bool peer_on = false;
};

namespace {

void abort_comm(qmm_tp_comm* c) {
    int expected = 0;
    if (c->comm && c->aborted.compare_exchange_strong(expected, 1)) nccl().CommAbort(c->comm);
}

// Polls the communicator until it leaves ncclInProgress (non-blocking init,
// finalize, or an enqueue that returned ncclInProgress). Aborts on error or
// when `limit_s` runs out.
int settle(qmm_tp_comm* c, double limit_s, const char* what) {
    const auto t0 = Clock::now();
    for (;;) {
        ncclResult_t st = ncclInProgress;
        const ncclResult_t r = nccl().CommGetAsyncError(c->comm, &st);
        if (r != ncclSuccess) {
            abort_comm(c);
            return fail(QMM_ERR_NCCL, std::string(what) + ": ncclCommGetAsyncError: " + nccl_str(r));
        }
        if (st == ncclSuccess) return QMM_OK;
        if (st != ncclInProgress) {
            abort_comm(c);
            return fail(QMM_ERR_NCCL, std::string(what) + ": " + nccl_str(st));
        }
        if (seconds_since(t0) > limit_s) {
            abort_comm(c);
            return fail(QMM_ERR_TIMEOUT, std::string(what) + " did not complete within " + std::to_string(limit_s) +
                                             " s; communicator aborted");
        }
        poll_pause(t0);
    }
}

// Result of an enqueue on a non-blocking communicator.
int enqueued(qmm_tp_comm* c, ncclResult_t r, const char* what) {
    if (r == ncclSuccess) return QMM_OK;
    if (r == ncclInProgress) return settle(c, c->timeout_s, what);
    abort_comm(c);
    return fail(QMM_ERR_NCCL, std::string(what) + ": " + nccl_str(r));
}

int usable(const qmm_tp_comm* c) {
    if (!c) return fail(QMM_ERR_INVALID_INPUT, "null communicator");
    if (c->aborted.load()) return fail(QMM_ERR_NCCL, "communicator was aborted");
    return QMM_OK;
}

int gather_buffer(qmm_tp_comm* c, size_t bytes, cudaStream_t st, float** out) {
    std::lock_guard<std::mutex> lock(c->mu);
    if (c->gbytes < bytes) {
        cudaStreamCaptureStatus cs = cudaStreamCaptureStatusNone;
        if (cudaStreamIsCapturing(st, &cs) == cudaSuccess && cs != cudaStreamCaptureStatusNone)
            return fail(QMM_ERR_INVALID_INPUT, "gather buffer must grow during stream capture; run once uncaptured");
        if (c->gbuf) {
            cudaStreamSynchronize(st);
            cudaFree(c->gbuf);
            c->gbuf = nullptr;
            c->gbytes = 0;
        }
        const cudaError_t e = cudaMalloc(&c->gbuf, bytes);
        if (e != cudaSuccess) {
            cudaGetLastError();
            return fail(QMM_ERR_CUDA, std::string("gather buffer: ") + cudaGetErrorString(e));
        }
        c->gbytes = bytes;
    }
    *out = c->gbuf;
    return QMM_OK;
}

size_t align256(size_t v) { return (v + 255) & ~size_t(255); }

void release_peer(qmm_tp_comm* c) {
    for (int r = 0; r < qmm::kMaxPeers; ++r) {
        if (c->pmem[r] && r != c->rank) cudaIpcCloseMemHandle(c->pmem[r]);
        c->pmem[r] = nullptr;
    }
    if (c->xmem) cudaFree(c->xmem);
    c->xmem = nullptr;
    c->peer_on = false;
    cudaGetLastError();
}

// The join of one column- or row-parallel forward over peer memory. Returns
// -1 when the join cannot take this call (not enabled, or too large for the
// buffers), so the caller joins through NCCL instead.
int peer_forward(qmm_tp_comm* c, const qmm_weight* shard, const float* x, size_t m, float* y, int act,
                 cudaStream_t st, bool column, size_t cols) {
    if (!c->peer_on) return -1;
    const size_t W = (size_t)c->world;
    const size_t count = column ? m * W * cols : m * cols;
    const size_t need = (column ? count : W * count) * sizeof(float);
    if (need > c->cap) return -1;
    float* own = reinterpret_cast<float*>(c->xmem + kBufOff);  // buffer 0; buffer 1 at + cap
    const unsigned long long* epoch = reinterpret_cast<const unsigned long long*>(c->xmem + kEpochOff);
    qmm::PeerOut po;
    po.n = c->world;
    po.ld = column ? (int64_t)(W * cols) : (int64_t)cols;
    po.pstride = (int64_t)(c->cap / sizeof(float));
    po.epoch = epoch;
    const size_t part = column ? (size_t)c->rank * cols : (size_t)c->rank * m * cols;  // this rank's place
    for (int r = 0; r < c->world; ++r) po.dst[r] = reinterpret_cast<float*>(c->pmem[r] + kBufOff) + part;
    // where a kernel that cannot write the join itself leaves the result:
    // contiguous [m][cols] (not in the join buffers: their index is on the device)
    float* ylocal = nullptr;
    {
        int rc = gather_buffer(c, m * cols * sizeof(float), st, &ylocal);
        if (rc) return rc;
    }
    qmm::set_peer_out(&po);
    int rc = qmm_linear_forward(shard, x, m, ylocal, act, st);
    qmm::set_peer_out(nullptr);
    if (rc) return rc;
    if (!po.taken) {
        PushArgs pa;
        for (int r = 0; r < qmm::kMaxPeers; ++r) pa.to.dst[r] = po.dst[r];
        pa.to.n = c->world;
        pa.to.ld = po.ld;
        pa.to.pstride = po.pstride;
        pa.to.epoch = epoch;
        pa.src = ylocal;
        pa.rows = (int64_t)m;
        pa.cols = (int64_t)cols;
        const int64_t total = pa.rows * pa.cols;
        const int blocks = (int)std::min<int64_t>((total + 255) / 256, 148 * 4);
        qmm::note_launch();
        tp_push_kernel<<<blocks, 256, 0, st>>>(pa);
        const cudaError_t e1 = cudaGetLastError();
        if (e1 != cudaSuccess) {
            abort_comm(c);
            return fail(QMM_ERR_CUDA, std::string("tp_push_kernel: ") + cudaGetErrorString(e1));
        }
    }
    JoinArgs j;
    for (int r = 0; r < qmm::kMaxPeers; ++r)
        j.signal[r] = (r < c->world && r != c->rank)
                          ? reinterpret_cast<uint64_t*>(c->pmem[r] + kFlagsOff) + c->rank
                          : nullptr;
    j.flags = reinterpret_cast<const uint64_t*>(c->xmem + kFlagsOff);
    j.errw = reinterpret_cast<int*>(c->xmem + kErrOff);
    j.epoch = reinterpret_cast<unsigned long long*>(c->xmem + kEpochOff);
    j.ticket = reinterpret_cast<unsigned*>(c->xmem + kTicketOff);
    j.buf = own;
    j.pstride = po.pstride;
    j.y = y;
    j.count = (int64_t)count;
    j.limit_ns = (long long)(c->join_timeout_s * 1e9);
    j.world = c->world;
    j.rank = c->rank;
    j.reduce = column ? 0 : 1;
    j.vec4 = (count % 4 == 0 && (reinterpret_cast<uintptr_t>(y) & 15) == 0) ? 1 : 0;
    const int64_t items = j.vec4 ? (int64_t)count / 4 : (int64_t)count;
    const int blocks = (int)std::max<int64_t>(1, std::min<int64_t>((items + 255) / 256, 148 * 2));
    qmm::note_launch();
    tp_join_kernel<<<blocks, 256, 0, st>>>(j);
    const cudaError_t e2 = cudaGetLastError();
    if (e2 != cudaSuccess) {
        abort_comm(c);
        return fail(QMM_ERR_CUDA, std::string("tp_join_kernel: ") + cudaGetErrorString(e2));
    }
    return QMM_OK;
}

}  // namespace

extern "C" {

QMM_API int qmm_tp_available(void) { return nccl().ok ? 1 : 0; }

QMM_API int qmm_tp_unique_id(uint8_t out[QMM_TP_UNIQUE_ID_BYTES]) {
    if (!out) return fail(QMM_ERR_INVALID_INPUT, "null pointer");
    if (!nccl().ok) return fail(QMM_ERR_NCCL, nccl().why);
    ncclUniqueId id;
    const ncclResult_t r = nccl().GetUniqueId(&id);
    if (r != ncclSuccess) return fail(QMM_ERR_NCCL, "ncclGetUniqueId: " + nccl_str(r));
    std::memcpy(out, id.internal, QMM_TP_UNIQUE_ID_BYTES);
    return QMM_OK;
}

QMM_API int qmm_tp_init(const uint8_t id[QMM_TP_UNIQUE_ID_BYTES], int world, int rank, int device, double timeout_s,
                        qmm_tp_comm** out) {
    if (!id || !out) return fail(QMM_ERR_INVALID_INPUT, "null pointer");
    *out = nullptr;
    if (world < 1 || rank < 0 || rank >= world) return fail(QMM_ERR_INVALID_INPUT, "bad rank / world");
    if (!(timeout_s > 0.0)) return fail(QMM_ERR_INVALID_INPUT, "timeout must be positive");
    if (!nccl().ok) return fail(QMM_ERR_NCCL, nccl().why);
    DevGuard guard(device);
    if (!guard.ok) return fail(QMM_ERR_CUDA, "cudaSetDevice failed");
    int dev = device;
    if (dev < 0 && cudaGetDevice(&dev) != cudaSuccess) {
        cudaGetLastError();
        dev = -1;  // no CUDA context: only a stand-in NCCL can get further
    }
    ncclUniqueId uid;
    std::memcpy(uid.internal, id, QMM_TP_UNIQUE_ID_BYTES);
    ncclConfig_t cfg = NCCL_CONFIG_INITIALIZER;
    cfg.blocking = 0;
    qmm_tp_comm* c = new qmm_tp_comm;
    c->rank = rank;
    c->world = world;
    c->device = dev;
    c->timeout_s = timeout_s;
    const ncclResult_t r = nccl().CommInitRankConfig(&c->comm, world, uid, rank, &cfg);
    if (r != ncclSuccess && r != ncclInProgress) {
        if (c->comm) nccl().CommAbort(c->comm);
        delete c;
        return fail(QMM_ERR_NCCL, "ncclCommInitRankConfig: " + nccl_str(r));
    }
    const int rc = settle(c, timeout_s, "communicator init");
    if (rc) {
        delete c;  // settle() aborted it
        return rc;
    }
    *out = c;
    return QMM_OK;
}

QMM_API int qmm_tp_abort(qmm_tp_comm* c) {
    if (!c) return fail(QMM_ERR_INVALID_INPUT, "null communicator");
    abort_comm(c);
    return QMM_OK;
}

QMM_API int qmm_tp_destroy(qmm_tp_comm* c) {
    if (!c) return QMM_OK;
    int rc = QMM_OK;
    {
        DevGuard guard(c->device);
        if (!c->aborted.load() && c->comm) {
            // finalize flushes outstanding work; bounded like every other wait
            ncclResult_t r = nccl().CommFinalize(c->comm);
            if (r == ncclSuccess || r == ncclInProgress) rc = settle(c, c->timeout_s, "communicator finalize");
            else {
                abort_comm(c);
                rc = fail(QMM_ERR_NCCL, "ncclCommFinalize: " + nccl_str(r));
            }
            if (!c->aborted.load()) nccl().CommDestroy(c->comm);
        }
        if (c->gbuf) cudaFree(c->gbuf);
        release_peer(c);
    }
    delete c;
    return rc;
}

QMM_API int qmm_tp_rank(const qmm_tp_comm* c, int* rank, int* world) {
    if (!c) return fail(QMM_ERR_INVALID_INPUT, "null communicator");
    if (rank) *rank = c->rank;
    if (world) *world = c->world;
    return QMM_OK;
}

QMM_API int qmm_tp_enable_peer(qmm_tp_comm* c, size_t bytes, double join_timeout_s) {
    int rc = usable(c);
    if (rc) return rc;
    if (bytes == 0) return fail(QMM_ERR_INVALID_INPUT, "join buffers must not be empty");
    if (c->world > qmm::kMaxPeers) return fail(QMM_ERR_INVALID_INPUT, "peer joins take at most 8 ranks");
    if (c->peer_on) return fail(QMM_ERR_INVALID_INPUT, "peer joins are already enabled");
    DevGuard guard(c->device);
    if (!guard.ok) return fail(QMM_ERR_CUDA, "cudaSetDevice failed");
    c->cap = align256(bytes);
    c->join_timeout_s = join_timeout_s > 0.0 ? join_timeout_s : c->timeout_s;
    const size_t total = kBufOff + 2 * c->cap;
    auto cuda_err = [&](cudaError_t e, const char* what) {
        cudaGetLastError();
        release_peer(c);
        return fail(QMM_ERR_CUDA, std::string(what) + ": " + cudaGetErrorString(e));
    };
    cudaError_t e = cudaMalloc(&c->xmem, total);
    if (e != cudaSuccess) {
        c->xmem = nullptr;
        return cuda_err(e, "join buffers");
    }
    // zeroed before this rank's handle leaves: no peer can write earlier
    e = cudaMemset(c->xmem, 0, total);
    if (e == cudaSuccess) e = cudaDeviceSynchronize();
    if (e != cudaSuccess) return cuda_err(e, "join buffers");
    c->pmem[c->rank] = c->xmem;
    if (c->world == 1) {
        c->peer_on = true;
        return QMM_OK;
    }
    cudaIpcMemHandle_t mine;
    e = cudaIpcGetMemHandle(&mine, c->xmem);
    if (e != cudaSuccess) return cuda_err(e, "cudaIpcGetMemHandle");
    static_assert(sizeof(cudaIpcMemHandle_t) == 64, "IPC handle size");
    const size_t hb = sizeof(cudaIpcMemHandle_t);
    uint8_t* dh = nullptr;
    cudaStream_t s = nullptr;
    e = cudaMalloc(&dh, hb * (size_t)c->world);
    if (e == cudaSuccess) e = cudaMemcpy(dh + hb * (size_t)c->rank, &mine, hb, cudaMemcpyHostToDevice);
    if (e == cudaSuccess) e = cudaStreamCreateWithFlags(&s, cudaStreamNonBlocking);
    if (e != cudaSuccess) {
        if (dh) cudaFree(dh);
        return cuda_err(e, "handle exchange");
    }
    // the handles travel through the communicator itself (bounded like every wait)
    rc = enqueued(c, nccl().AllGather(dh + hb * (size_t)c->rank, dh, hb, ncclUint8, c->comm, s), "ncclAllGather");
    if (!rc) rc = qmm_tp_wait(c, s, c->timeout_s);
    std::vector<cudaIpcMemHandle_t> all((size_t)c->world);
    if (!rc) {
        e = cudaMemcpy(all.data(), dh, hb * (size_t)c->world, cudaMemcpyDeviceToHost);
        if (e != cudaSuccess) rc = fail(QMM_ERR_CUDA, std::string("handle exchange: ") + cudaGetErrorString(e));
    }
    cudaStreamDestroy(s);
    cudaFree(dh);
    if (rc) {
        release_peer(c);
        return rc;
    }
    for (int r = 0; r < c->world; ++r) {
        if (r == c->rank) continue;
        void* p = nullptr;
        e = cudaIpcOpenMemHandle(&p, all[(size_t)r], cudaIpcMemLazyEnablePeerAccess);
        if (e != cudaSuccess) return cuda_err(e, "cudaIpcOpenMemHandle");
        c->pmem[r] = static_cast<uint8_t*>(p);
    }
    c->peer_on = true;
    return QMM_OK;
}

QMM_API int qmm_tp_status(qmm_tp_comm* c) {
    int rc = usable(c);
    if (rc) return rc;
    ncclResult_t st = ncclSuccess;
    const ncclResult_t r = nccl().CommGetAsyncError(c->comm, &st);
    if (r != ncclSuccess || (st != ncclSuccess && st != ncclInProgress)) {
        abort_comm(c);
        return fail(QMM_ERR_NCCL, "communicator error: " + nccl_str(r != ncclSuccess ? r : st));
    }
    return QMM_OK;
}

QMM_API int qmm_tp_wait(qmm_tp_comm* c, void* stream, double timeout_s) {
    int rc = usable(c);
    if (rc) return rc;
    if (!(timeout_s > 0.0)) return fail(QMM_ERR_INVALID_INPUT, "timeout must be positive");
    DevGuard guard(c->device);
    if (!guard.ok) return fail(QMM_ERR_CUDA, "cudaSetDevice failed");
    const cudaStream_t st = (cudaStream_t)stream;
    const auto t0 = Clock::now();
    auto drain = [&]() {
        // after an abort NCCL's kernels exit; let the stream run dry (bounded)
        const auto t1 = Clock::now();
        while (cudaStreamQuery(st) == cudaErrorNotReady && seconds_since(t1) < 10.0)
            std::this_thread::sleep_for(std::chrono::microseconds(200));
        cudaGetLastError();
    };
    for (;;) {
        ncclResult_t as = ncclSuccess;
        const ncclResult_t r = nccl().CommGetAsyncError(c->comm, &as);
        if (r != ncclSuccess || (as != ncclSuccess && as != ncclInProgress)) {
            abort_comm(c);
            drain();
            return fail(QMM_ERR_NCCL, "communicator error: " + nccl_str(r != ncclSuccess ? r : as));
        }
        const cudaError_t q = cudaStreamQuery(st);
        if (q == cudaSuccess) {
            // (captured joins replay without passing through here: with joins
            // over peer memory enabled, every wait reads the error word)
            if (!c->peer_on) return QMM_OK;
            // a join's bounded wait for a peer's signal records its time-out here
            int ew = 0;
            cudaError_t ce = cudaMemcpyAsync(&ew, c->xmem + kErrOff, sizeof(int), cudaMemcpyDeviceToHost, st);
            if (ce == cudaSuccess) ce = cudaStreamSynchronize(st);
            if (ce != cudaSuccess) {
                cudaGetLastError();
                return fail(QMM_ERR_CUDA, std::string("join error word: ") + cudaGetErrorString(ce));
            }
            if (ew != 0) {
                abort_comm(c);
                return fail(QMM_ERR_TIMEOUT, "peer join: a peer's signal did not arrive within " +
                                                 std::to_string(c->join_timeout_s) + " s; communicator aborted");
            }
            return QMM_OK;
        }
        if (q != cudaErrorNotReady) {
            cudaGetLastError();
            return fail(QMM_ERR_CUDA, std::string("cudaStreamQuery: ") + cudaGetErrorString(q));
        }
        if (seconds_since(t0) > timeout_s) {
            abort_comm(c);
            drain();
            return fail(QMM_ERR_TIMEOUT, "stream work did not finish within " + std::to_string(timeout_s) +
                                             " s; communicator aborted");
        }
        poll_pause(t0);
    }
}

QMM_API int qmm_tp_all_gather_f32(qmm_tp_comm* c, const float* send, float* recv, size_t count, void* stream) {
    int rc = usable(c);
    if (rc) return rc;
    if (!send || !recv) return fail(QMM_ERR_INVALID_INPUT, "null pointer");
    if (count == 0) return QMM_OK;
    DevGuard guard(c->device);
    if (!guard.ok) return fail(QMM_ERR_CUDA, "cudaSetDevice failed");
    return enqueued(c, nccl().AllGather(send, recv, count, ncclFloat32, c->comm, (cudaStream_t)stream),
                    "ncclAllGather");
}

QMM_API int qmm_tp_all_reduce_f32(qmm_tp_comm* c, float* buf, size_t count, void* stream) {
    int rc = usable(c);
    if (rc) return rc;
    if (!buf) return fail(QMM_ERR_INVALID_INPUT, "null pointer");
    if (count == 0) return QMM_OK;
    DevGuard guard(c->device);
    if (!guard.ok) return fail(QMM_ERR_CUDA, "cudaSetDevice failed");
    return enqueued(c, nccl().AllReduce(buf, buf, count, ncclFloat32, ncclSum, c->comm, (cudaStream_t)stream),
                    "ncclAllReduce");
}

QMM_API int qmm_tp_column_forward(qmm_tp_comm* c, const qmm_weight* shard, const float* x, size_t m, float* y,
                                  int act, void* stream) {
    int rc = usable(c);
    if (rc) return rc;
    if (!shard || !x || !y) return fail(QMM_ERR_INVALID_INPUT, "null pointer");
    size_t nl = 0;
    int wdev = -1;
    rc = qmm_weight_info(shard, nullptr, &nl, nullptr, nullptr, &wdev);
    if (rc) return rc;
    if (wdev != c->device) return fail(QMM_ERR_INVALID_INPUT, "shard lives on another device than the communicator");
    if (m == 0) return QMM_OK;
    DevGuard guard(c->device);
    if (!guard.ok) return fail(QMM_ERR_CUDA, "cudaSetDevice failed");
    const cudaStream_t st = (cudaStream_t)stream;
    if (c->world == 1) return qmm_linear_forward(shard, x, m, y, act, stream);
    rc = peer_forward(c, shard, x, m, y, act, st, /*column=*/true, nl);
    if (rc != -1) return rc;
    if (m == 1) {
        // [1][world * nl] is already rank-major: gather in place
        float* slot = y + (size_t)c->rank * nl;
        rc = qmm_linear_forward(shard, x, m, slot, act, stream);
        if (rc) return rc;
        return enqueued(c, nccl().AllGather(slot, y, nl, ncclFloat32, c->comm, st), "ncclAllGather");
    }
    if (m * nl * (size_t)c->world > (size_t)INT32_MAX) return fail(QMM_ERR_INVALID_INPUT, "output too large");
    float* g = nullptr;
    rc = gather_buffer(c, m * nl * (size_t)c->world * sizeof(float), st, &g);
    if (rc) return rc;
    float* local = g + (size_t)c->rank * m * nl;
    rc = qmm_linear_forward(shard, x, m, local, act, stream);
    if (rc) return rc;
    rc = enqueued(c, nccl().AllGather(local, g, m * nl, ncclFloat32, c->comm, st), "ncclAllGather");
    if (rc) return rc;
    const int64_t total = (int64_t)m * nl * c->world;
    const int blocks = (int)std::min<int64_t>((total + 255) / 256, 148 * 8);
    qmm::note_launch();
    tp_reorder_kernel<<<blocks, 256, 0, st>>>(g, y, (int)m, (int)nl, c->world);
    const cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) return fail(QMM_ERR_CUDA, std::string("tp_reorder_kernel: ") + cudaGetErrorString(e));
    return QMM_OK;
}

QMM_API int qmm_tp_row_forward(qmm_tp_comm* c, const qmm_weight* shard, const float* x_local, size_t m, float* y,
                               int act, void* stream) {
    int rc = usable(c);
    if (rc) return rc;
    if (!shard || !x_local || !y) return fail(QMM_ERR_INVALID_INPUT, "null pointer");
    size_t n = 0;
    int wdev = -1;
    rc = qmm_weight_info(shard, nullptr, &n, nullptr, nullptr, &wdev);
    if (rc) return rc;
    if (wdev != c->device) return fail(QMM_ERR_INVALID_INPUT, "shard lives on another device than the communicator");
    if (m == 0) return QMM_OK;
    DevGuard guard(c->device);
    if (!guard.ok) return fail(QMM_ERR_CUDA, "cudaSetDevice failed");
    if (c->world > 1) {
        rc = peer_forward(c, shard, x_local, m, y, act, (cudaStream_t)stream, /*column=*/false, n);
        if (rc != -1) return rc;
    }
    rc = qmm_linear_forward(shard, x_local, m, y, act, stream);
    if (rc || c->world == 1) return rc;
    return enqueued(c, nccl().AllReduce(y, y, m * n, ncclFloat32, ncclSum, c->comm, (cudaStream_t)stream),
                    "ncclAllReduce");
}

}  // extern "C"
