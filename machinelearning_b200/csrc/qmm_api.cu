// C ABI of libqmm.so (declared in include/qmm.h).
//
// Conventions follow the reference's FFI crate
// (llminference/main/features/inference/ffi/main/src/lib.rs:12-40): status
// codes instead of panics/exceptions, null checks on every pointer, the library
// frees what it allocates, concurrent calls are allowed (shared state is behind
// mutexes; per-stream workspaces keep concurrent streams apart).
#include <atomic>
#include <cstdio>
#include <cstring>
#include <map>
#include <mutex>
#include <string>
#include <utility>
#include <vector>

#include "../../include/qmm.h"
#include "../../include/qmm_tp.h"
#include "qmm_common.cuh"
#include "qmm_kernels.cuh"

namespace qmm {
static std::atomic<unsigned long long> g_launches{0};
void note_launch() { g_launches.fetch_add(1, std::memory_order_relaxed); }
static unsigned long long launch_count() { return g_launches.load(std::memory_order_relaxed); }
}  // namespace qmm

using namespace qmm;

// Device-side error word (one per device context). Kernels receive its address.
__device__ int g_qmm_device_error = 0;

// Accumulator of qmm_checksum_dev (one per device context).
__device__ unsigned long long g_qmm_checksum_acc = 0;

// Scratch for qmm_matmul_dev_noalloc: a fixed, file-scope device array, so that
// entry point never allocates. Every device that loads the library holds these
// 4 MiB until the process exits. Host code must not use the symbol itself as a
// device address; qmm_matmul_dev_noalloc looks the address up per device.
constexpr size_t kNoAllocScratchBytes = size_t(4) << 20;
static __device__ __align__(256) uint8_t g_qmm_noalloc_scratch[kNoAllocScratchBytes];

// Self-test of the bounded-wait path (qmm_selftest_bounded_wait): one thread
// waits on a freshly initialised mbarrier that nothing ever completes, with
// the library's own probe loop cut to `probes`, then records the timeout in
// the error word exactly as a kernel of the hot path would, and returns. It
// cannot hang: the loop is bounded and no other thread waits on it.
__global__ void selftest_wait_kernel(uint32_t probes, int* err) {
    __shared__ __align__(8) uint64_t bar;
    if (threadIdx.x != 0) return;
    qmm::mbar_init(&bar, 1);
    qmm::fence_mbar_init();
    bool done = false;
    for (uint32_t i = 0; i < probes && !done; ++i) done = qmm::mbar_try_wait(&bar, 0);
    if (!done && err) atomicExch(err, qmm::kErrWaitTimeout);
}

namespace {

thread_local std::string t_last_error;

int fail(int status, const std::string& msg) {
    t_last_error = msg;
    return status;
}
}  // namespace

namespace qmm {
int set_last_error(int status, const std::string& msg) { return fail(status, msg); }
}  // namespace qmm

namespace {
int cuda_fail(cudaError_t e, const char* where) {
    cudaGetLastError();  // clear sticky-free errors so later calls are not poisoned
    return fail(QMM_ERR_CUDA, std::string(where) + ": " + cudaGetErrorString(e));
}
#define QMM_CUDA(call)                                  \
    do {                                                \
        cudaError_t _e = (call);                        \
        if (_e != cudaSuccess) return cuda_fail(_e, #call); \
    } while (0)

struct DeviceGuard {
    int prev = -1;
    bool ok = true;
    explicit DeviceGuard(int dev) {
        if (cudaGetDevice(&prev) != cudaSuccess) prev = -1;
        if (dev >= 0 && dev != prev) ok = cudaSetDevice(dev) == cudaSuccess;
    }
    ~DeviceGuard() {
        int cur = -1;
        if (prev >= 0 && cudaGetDevice(&cur) == cudaSuccess && cur != prev) cudaSetDevice(prev);
    }
};

bool valid_dtype(int dt) { return dt == QMM_Q4_0 || dt == QMM_Q4_1 || dt == QMM_Q8_0; }

int num_sms(int dev) {
    static std::mutex mu;
    static std::map<int, int> cache;
    std::lock_guard<std::mutex> lock(mu);
    auto it = cache.find(dev);
    if (it != cache.end()) return it->second;
    int v = 0;
    if (cudaDeviceGetAttribute(&v, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || v <= 0) v = 148;
    cache[dev] = v;
    return v;
}

int current_device() {
    int d = 0;
    if (cudaGetDevice(&d) != cudaSuccess) return -1;
    return d;
}

// ---- per-(device, stream) workspaces ---------------------------------------------
struct Buffer {
    void* ptr = nullptr;
    size_t bytes = 0;
};
std::mutex g_ws_mu;
std::map<std::pair<int, void*>, Buffer> g_ws;
std::map<std::pair<int, void*>, Buffer> g_io;  // host-entry staging (qmm_linear_forward_host)

int get_workspace(int dev, void* stream, size_t need, void** out) {
    std::lock_guard<std::mutex> lock(g_ws_mu);
    Buffer& b = g_ws[{dev, stream}];
    if (b.bytes < need) {
        cudaStreamCaptureStatus cs = cudaStreamCaptureStatusNone;
        if (cudaStreamIsCapturing((cudaStream_t)stream, &cs) == cudaSuccess && cs != cudaStreamCaptureStatusNone)
            return fail(QMM_ERR_INVALID_INPUT,
                        "workspace must grow during stream capture; call qmm_reserve_workspace first");
        if (b.ptr) {
            cudaStreamSynchronize((cudaStream_t)stream);
            cudaFree(b.ptr);
            b.ptr = nullptr;
            b.bytes = 0;
        }
        size_t want = need < (1u << 20) ? (1u << 20) : need;
        QMM_CUDA(cudaMalloc(&b.ptr, want));
        QMM_CUDA(cudaMemset(b.ptr, 0, want));
        b.bytes = want;
    }
    *out = b.ptr;
    return QMM_OK;
}

// ---- shape helpers ----------------------------------------------------------------
constexpr size_t kMaxGemvRows = 64;

size_t row_bytes_of(int dt, size_t k) { return (k / QK) * (size_t)block_bytes(dt); }

int check_shape(int dt, size_t m, size_t k, size_t n, size_t w_len) {
    if (!valid_dtype(dt)) return fail(QMM_ERR_DTYPE_MISMATCH, "unsupported block type id");
    if (k % QK) return fail(QMM_ERR_BLOCK_ALIGNMENT, "in_features not divisible by block size 32");
    if (k == 0 || n > (size_t)INT32_MAX || k > (size_t)INT32_MAX || m > (size_t)INT32_MAX)
        return fail(QMM_ERR_SHAPE_MISMATCH, "shape out of range");
    if (w_len < n * row_bytes_of(dt, k)) return fail(QMM_ERR_SHAPE_MISMATCH, "weight buffer shorter than n*k/32 blocks");
    return QMM_OK;
}

size_t workspace_for(int dt, int act, size_t m, size_t n, size_t k, int dev) {
    if (m == 0 || n == 0) return 0;
    if (gemm_supported(dt, act == QMM_ACT_Q8_0, (int)m, (int)n, (int)k))
        return gemm_workspace_bytes((int)m, (int)n, (int)k, dt, act == QMM_ACT_Q8_0);
    const size_t rows = m < kMaxGemvRows ? m : kMaxGemvRows;
    GemvPlan p;
    if (!gemv_plan(dt, act == QMM_ACT_Q8_0, (int)rows, (int)n, (int)k, num_sms(dev), &p)) return 0;
    return gemv_workspace_bytes(p);
}

// The device matmul: GEMV in chunks of <= 64 activation rows.
// immutable_w: the weights are library-owned (a qmm_weight, complete before
// any call), so the GEMV may fetch them before waiting on preceding kernels.
// g: optional gate/up epilogue (y then unused; g.out advances with the rows).
int run_matmul(int dt, int act, const float* x, const uint8_t* w, size_t m, size_t k, size_t n, float* y,
               void* ws, size_t ws_bytes, cudaStream_t st, bool immutable_w = false,
               const GatedOut& g = GatedOut()) {
    if (m == 0 || n == 0) return QMM_OK;
    const int dev = current_device();
    if (dev < 0) return fail(QMM_ERR_NO_DEVICE, "no CUDA device");
    int* err = device_error_word(dev);
    // prefill-sized M: one tensor-core GEMM over all rows
    if (gemm_supported(dt, act == QMM_ACT_Q8_0, (int)m, (int)n, (int)k)) {
        const bool native = act == QMM_ACT_Q8_0;
        if (gemm_workspace_bytes((int)m, (int)n, (int)k, dt, native) > ws_bytes)
            return fail(QMM_ERR_INVALID_INPUT, "workspace too small");
        cudaError_t e = launch_gemm(dt, w, x, y, (int)m, (int)n, (int)k, ws, err, st, immutable_w, g, native);
        if (e != cudaSuccess) return cuda_fail(e, "launch_gemm");
        return QMM_OK;
    }
    // a join written by the kernel itself addresses whole [M][N] outputs: not
    // offered to a GEMV that runs in row chunks
    struct HidePeer {
        PeerOut* saved = nullptr;
        explicit HidePeer(bool hide) {
            if (hide) {
                saved = peer_out();
                set_peer_out(nullptr);
            }
        }
        ~HidePeer() {
            if (saved) set_peer_out(saved);
        }
    } hide(m > kMaxGemvRows);
    for (size_t r0 = 0; r0 < m; r0 += kMaxGemvRows) {
        const size_t rows = (m - r0) < kMaxGemvRows ? (m - r0) : kMaxGemvRows;
        GemvPlan p;
        if (!gemv_plan(dt, act == QMM_ACT_Q8_0, (int)rows, (int)n, (int)k, num_sms(dev), &p))
            return fail(QMM_ERR_SHAPE_MISMATCH, "shape not supported");
        if (gemv_workspace_bytes(p) > ws_bytes) return fail(QMM_ERR_INVALID_INPUT, "workspace too small");
        p.weights_immutable = immutable_w;
        GemvWorkspace w_s;
        gemv_workspace_carve(p, ws, &w_s);
        GatedOut gr = g;
        if (gr.act >= 0) gr.out += (int64_t)r0 * gr.hidden;
        cudaError_t e = launch_gemv(p, w, x + r0 * k, y ? y + r0 * n : nullptr, w_s, err, st, false, gr);
        if (e != cudaSuccess) return cuda_fail(e, "launch_gemv");
    }
    return QMM_OK;
}

}  // namespace

namespace qmm {
int* device_error_word(int device) {
    static std::mutex mu;
    static std::map<int, int*> cache;
    std::lock_guard<std::mutex> lock(mu);
    auto it = cache.find(device);
    if (it != cache.end()) return it->second;
    void* p = nullptr;
    if (cudaGetSymbolAddress(&p, g_qmm_device_error) != cudaSuccess) {
        cudaGetLastError();
        return nullptr;
    }
    cache[device] = static_cast<int*>(p);
    return static_cast<int*>(p);
}

namespace {
thread_local PeerOut* t_peer_out = nullptr;
}
PeerOut* peer_out() { return t_peer_out; }
void set_peer_out(PeerOut* p) { t_peer_out = p; }
void take_peer_out(PeerDst& out, bool supported) {
    out.n = 0;
    PeerOut* p = t_peer_out;
    if (!p || !supported || p->taken || p->n < 1 || p->n > kMaxPeers) return;
    for (int r = 0; r < kMaxPeers; ++r) out.dst[r] = r < p->n ? p->dst[r] : nullptr;
    out.n = p->n;
    out.ld = p->ld;
    out.pstride = p->pstride;
    out.epoch = p->epoch;
    p->taken = true;
}
}  // namespace qmm

struct qmm_weight {
    int dtype;
    size_t n, k;
    int device;
    uint8_t* dev;
    size_t len;
    size_t gate_hidden;  // > 0: a gate/up weight (rows interleaved in kGateGroup groups)
};

namespace {
std::mutex g_reg_mu;
std::map<const uint8_t*, qmm_weight*> g_registered;

int weight_create_impl(int dtype, size_t n, size_t k, const uint8_t* src, size_t len, int device, bool from_device,
                       qmm_weight** out) {
    if (!out || !src) return fail(QMM_ERR_INVALID_INPUT, "null pointer");
    *out = nullptr;
    int rc = check_shape(dtype, 0, k, n, len);
    if (rc) return rc;
    int ndev = 0;
    if (cudaGetDeviceCount(&ndev) != cudaSuccess || ndev == 0) {
        cudaGetLastError();
        return fail(QMM_ERR_NO_DEVICE, "no CUDA device");
    }
    if (device < 0 || device >= ndev) return fail(QMM_ERR_INVALID_INPUT, "bad device index");
    DeviceGuard guard(device);
    if (!guard.ok) return fail(QMM_ERR_CUDA, "cudaSetDevice failed");
    const size_t bytes = n * row_bytes_of(dtype, k);
    uint8_t* d = nullptr;
    QMM_CUDA(cudaMalloc(&d, (bytes + 15) & ~size_t(15)));
    cudaError_t e = cudaMemcpy(d, src, bytes, from_device ? cudaMemcpyDeviceToDevice : cudaMemcpyHostToDevice);
    // a device-to-device cudaMemcpy may still be running when it returns: the
    // handle's bytes must be final before any kernel may read them
    if (e == cudaSuccess) e = cudaDeviceSynchronize();
    if (e != cudaSuccess) {
        cudaFree(d);
        return cuda_fail(e, "weight upload");
    }
    qmm_weight* w = new qmm_weight{dtype, n, k, device, d, bytes, 0};
    *out = w;
    return QMM_OK;
}

// A new device weight of `rows` rows whose bytes are written by `fill`
// (device-to-device copies on the legacy stream), synchronised before return.
template <class F>
int weight_build(int dtype, size_t rows, size_t k, int device, size_t gate_hidden, F&& fill, qmm_weight** out) {
    DeviceGuard guard(device);
    if (!guard.ok) return fail(QMM_ERR_CUDA, "cudaSetDevice failed");
    const size_t bytes = rows * row_bytes_of(dtype, k);
    uint8_t* d = nullptr;
    QMM_CUDA(cudaMalloc(&d, (bytes + 15) & ~size_t(15)));
    cudaError_t e = fill(d);
    if (e == cudaSuccess) e = cudaDeviceSynchronize();
    if (e != cudaSuccess) {
        cudaFree(d);
        return cuda_fail(e, "weight fuse");
    }
    *out = new qmm_weight{dtype, rows, k, device, d, bytes, gate_hidden};
    return QMM_OK;
}

int act_for(bool native) { return native ? QMM_ACT_Q8_0 : QMM_ACT_F32; }

// Shared body of the reference-signature host calls.
int host_matmul(int dt, bool native, const float* x, size_t x_len, const uint8_t* w, size_t w_len, size_t m, size_t k,
                size_t n, float* y) {
    if (!x || !w || !y) return fail(QMM_ERR_INVALID_INPUT, "null pointer");
    int rc = check_shape(dt, m, k, n, w_len);
    if (rc) return rc;
    if (x_len < m * k) return fail(QMM_ERR_SHAPE_MISMATCH, "input shorter than m*in_features");
    if (m == 0 || n == 0) return QMM_OK;
    const int dev = current_device();
    if (dev < 0) return fail(QMM_ERR_NO_DEVICE, "no CUDA device");
    const qmm_weight* reg = nullptr;
    {
        std::lock_guard<std::mutex> lock(g_reg_mu);
        auto it = g_registered.find(w);
        if (it != g_registered.end() && it->second->dtype == dt && it->second->n == n && it->second->k == k &&
            it->second->device == dev)
            reg = it->second;
    }
    const size_t wb = n * row_bytes_of(dt, k);
    const size_t ws = workspace_for(dt, act_for(native), m, n, k, dev);
    auto al = [](size_t v) { return (v + 255) & ~size_t(255); };
    const size_t need = al(m * k * 4) + al(m * n * 4) + (reg ? 0 : al(wb)) + al(ws);
    // a per-thread scratch so concurrent host calls never share device buffers
    thread_local std::map<int, Buffer> scratch;
    Buffer& b = scratch[dev];
    if (b.bytes < need) {
        if (b.ptr) cudaFree(b.ptr);
        b.ptr = nullptr;
        b.bytes = 0;
        QMM_CUDA(cudaMalloc(&b.ptr, need));
        QMM_CUDA(cudaMemset(b.ptr, 0, need));
        b.bytes = need;
    }
    uint8_t* base = static_cast<uint8_t*>(b.ptr);
    float* xd = reinterpret_cast<float*>(base);
    float* yd = reinterpret_cast<float*>(base + al(m * k * 4));
    uint8_t* wd = base + al(m * k * 4) + al(m * n * 4);
    void* wsd = wd + (reg ? 0 : al(wb));
    const uint8_t* wuse = reg ? reg->dev : wd;
    cudaStream_t st = nullptr;
    QMM_CUDA(cudaMemcpyAsync(xd, x, m * k * 4, cudaMemcpyHostToDevice, st));
    if (!reg) QMM_CUDA(cudaMemcpyAsync(wd, w, wb, cudaMemcpyHostToDevice, st));
    rc = run_matmul(dt, act_for(native), xd, wuse, m, k, n, yd, wsd, ws, st, /*immutable_w=*/reg != nullptr);
    if (rc) return rc;
    QMM_CUDA(cudaMemcpyAsync(y, yd, m * n * 4, cudaMemcpyDeviceToHost, st));
    QMM_CUDA(cudaStreamSynchronize(st));
    return QMM_OK;
}

int host_quantize(int dt, int variant, const float* x, size_t n, uint8_t* out, float* scales) {
    if (!x || !out) return fail(QMM_ERR_INVALID_INPUT, "null pointer");
    if (n % QK) return fail(QMM_ERR_BLOCK_ALIGNMENT, "element count not divisible by 32");
    if (n == 0) return QMM_OK;
    const size_t nb = n / QK, ob = nb * block_bytes(dt);
    float* xd = nullptr;
    uint8_t* od = nullptr;
    float* sd = nullptr;
    QMM_CUDA(cudaMalloc(&xd, n * 4));
    cudaError_t e = cudaMalloc(&od, ob);
    if (e == cudaSuccess && scales) e = cudaMalloc(&sd, nb * 4);
    if (e == cudaSuccess) e = cudaMemcpy(xd, x, n * 4, cudaMemcpyHostToDevice);
    if (e == cudaSuccess) {
        if (dt == QMM_Q8_0) e = launch_quantize_q8_0(xd, (int64_t)n, od, sd, variant == 1, nullptr);
        else if (dt == QMM_Q4_0) e = launch_quantize_q4_0(xd, (int64_t)n, od, nullptr);
        else e = launch_quantize_q4_1(xd, (int64_t)n, od, nullptr);
    }
    if (e == cudaSuccess) e = cudaMemcpy(out, od, ob, cudaMemcpyDeviceToHost);
    if (e == cudaSuccess && scales) e = cudaMemcpy(scales, sd, nb * 4, cudaMemcpyDeviceToHost);
    cudaFree(xd);
    cudaFree(od);
    if (sd) cudaFree(sd);
    if (e != cudaSuccess) return cuda_fail(e, "quantize");
    return QMM_OK;
}

}  // namespace

extern "C" {

QMM_API int qmm_version(void) { return 100; }

QMM_API const char* qmm_status_string(int s) {
    switch (s) {
        case QMM_OK: return "ok";
        case QMM_ERR_BLOCK_ALIGNMENT: return "block alignment";
        case QMM_ERR_SHAPE_MISMATCH: return "shape mismatch";
        case QMM_ERR_DTYPE_MISMATCH: return "dtype mismatch";
        case QMM_ERR_INVALID_DATA: return "invalid data";
        case QMM_ERR_CUDA: return "cuda error";
        case QMM_ERR_NCCL: return "nccl error";
        case QMM_ERR_TIMEOUT: return "timeout";
        case QMM_ERR_INVALID_INPUT: return "invalid input";
        case QMM_ERR_NO_DEVICE: return "no device";
        default: return "unknown status";
    }
}

QMM_API const char* qmm_last_error_message(void) { return t_last_error.c_str(); }

QMM_API int qmm_device_count(void) {
    int n = 0;
    if (cudaGetDeviceCount(&n) != cudaSuccess) {
        cudaGetLastError();
        return 0;
    }
    return n;
}

QMM_API unsigned long long qmm_launch_count(void) { return qmm::launch_count(); }

QMM_API int qmm_device_error(int device, int* out_error) {
    if (!out_error) return fail(QMM_ERR_INVALID_INPUT, "null pointer");
    DeviceGuard guard(device);
    if (!guard.ok) return fail(QMM_ERR_INVALID_INPUT, "bad device");
    int* p = device_error_word(device);
    if (!p) return fail(QMM_ERR_CUDA, "device error word unavailable");
    QMM_CUDA(cudaDeviceSynchronize());
    int v = 0;
    QMM_CUDA(cudaMemcpy(&v, p, sizeof(int), cudaMemcpyDeviceToHost));
    const int zero = 0;
    QMM_CUDA(cudaMemcpy(p, &zero, sizeof(int), cudaMemcpyHostToDevice));
    *out_error = v;
    return QMM_OK;
}

QMM_API int qmm_device_status(int device) {
    int v = 0;
    int rc = qmm_device_error(device, &v);
    if (rc) return rc;
    if (v == kErrWaitTimeout) return fail(QMM_ERR_TIMEOUT, "a bounded device-side wait timed out");
    if (v != kErrNone) return fail(QMM_ERR_CUDA, "device error word " + std::to_string(v));
    return QMM_OK;
}

QMM_API int qmm_selftest_bounded_wait(unsigned probes, void* stream) {
    if (probes == 0 || probes > kMaxWaitProbes) return fail(QMM_ERR_INVALID_INPUT, "probes outside 1..2^20");
    const int dev = current_device();
    if (dev < 0) return fail(QMM_ERR_NO_DEVICE, "no CUDA device");
    int* err = device_error_word(dev);
    if (!err) return fail(QMM_ERR_CUDA, "device error word unavailable");
    selftest_wait_kernel<<<1, 32, 0, (cudaStream_t)stream>>>(probes, err);
    note_launch();
    QMM_CUDA(cudaGetLastError());
    return QMM_OK;
}

#define QMM_HOST_MATMUL(name, dt, native)                                                                    \
    QMM_API int name(const float* input_data, size_t input_len, const uint8_t* weight_bytes, size_t weight_len, \
                     size_t m, size_t in_features, size_t out_features, float* output) {                       \
        return host_matmul(dt, native, input_data, input_len, weight_bytes, weight_len, m, in_features,       \
                           out_features, output);                                                              \
    }
QMM_HOST_MATMUL(qmm_matmul_f32_q8, QMM_Q8_0, false)
QMM_HOST_MATMUL(qmm_matmul_f32_q8_v2, QMM_Q8_0, true)
QMM_HOST_MATMUL(qmm_matmul_f32_q4, QMM_Q4_0, false)
QMM_HOST_MATMUL(qmm_matmul_f32_q4_native, QMM_Q4_0, true)
QMM_HOST_MATMUL(qmm_matmul_f32_q4_1, QMM_Q4_1, false)
QMM_HOST_MATMUL(qmm_matmul_f32_q4_1_native, QMM_Q4_1, true)
#undef QMM_HOST_MATMUL

QMM_API int qmm_quantize_q8_0(const float* data, size_t n, uint8_t* out) {
    return host_quantize(QMM_Q8_0, 0, data, n, out, nullptr);
}
QMM_API int qmm_quantize_q4_0(const float* data, size_t n, uint8_t* out) {
    return host_quantize(QMM_Q4_0, 0, data, n, out, nullptr);
}
QMM_API int qmm_quantize_q4_1(const float* data, size_t n, uint8_t* out) {
    return host_quantize(QMM_Q4_1, 0, data, n, out, nullptr);
}
QMM_API int qmm_quantize_row_q8_0(const float* input, size_t n, uint8_t* out, float* scales) {
    if (!scales) return fail(QMM_ERR_INVALID_INPUT, "null pointer");
    return host_quantize(QMM_Q8_0, 1, input, n, out, scales);
}

QMM_API int qmm_dequantize(int dtype, const uint8_t* raw, size_t raw_len, size_t n_elements, float* out) {
    if (!raw || !out) return fail(QMM_ERR_INVALID_INPUT, "null pointer");
    if (!valid_dtype(dtype)) return fail(QMM_ERR_DTYPE_MISMATCH, "unsupported block type id");
    if (n_elements % QK) return fail(QMM_ERR_BLOCK_ALIGNMENT, "element count not divisible by 32");
    const size_t bytes = n_elements / QK * block_bytes(dtype);
    if (raw_len < bytes) return fail(QMM_ERR_SHAPE_MISMATCH, "raw buffer shorter than the element count needs");
    if (n_elements == 0) return QMM_OK;
    uint8_t* wd = nullptr;
    float* od = nullptr;
    QMM_CUDA(cudaMalloc(&wd, bytes));
    cudaError_t e = cudaMalloc(&od, n_elements * 4);
    if (e == cudaSuccess) e = cudaMemcpy(wd, raw, bytes, cudaMemcpyHostToDevice);
    if (e == cudaSuccess) e = launch_dequantize(dtype, wd, (int64_t)n_elements, od, nullptr);
    if (e == cudaSuccess) e = cudaMemcpy(out, od, n_elements * 4, cudaMemcpyDeviceToHost);
    cudaFree(wd);
    cudaFree(od);
    if (e != cudaSuccess) return cuda_fail(e, "dequantize");
    return QMM_OK;
}

QMM_API int qmm_register_host_weight(const uint8_t* weight_bytes, size_t weight_len, int dtype, size_t n, size_t k) {
    if (!weight_bytes) return fail(QMM_ERR_INVALID_INPUT, "null pointer");
    const int dev = current_device();
    if (dev < 0) return fail(QMM_ERR_NO_DEVICE, "no CUDA device");
    qmm_weight* w = nullptr;
    int rc = weight_create_impl(dtype, n, k, weight_bytes, weight_len, dev, false, &w);
    if (rc) return rc;
    std::lock_guard<std::mutex> lock(g_reg_mu);
    auto it = g_registered.find(weight_bytes);
    if (it != g_registered.end()) qmm_weight_destroy(it->second);
    g_registered[weight_bytes] = w;
    return QMM_OK;
}

QMM_API int qmm_unregister_host_weight(const uint8_t* weight_bytes) {
    std::lock_guard<std::mutex> lock(g_reg_mu);
    auto it = g_registered.find(weight_bytes);
    if (it == g_registered.end()) return fail(QMM_ERR_INVALID_INPUT, "not registered");
    qmm_weight_destroy(it->second);
    g_registered.erase(it);
    return QMM_OK;
}

QMM_API int qmm_weight_create(int dtype, size_t n, size_t k, const uint8_t* host_bytes, size_t len, int device,
                              qmm_weight** out) {
    return weight_create_impl(dtype, n, k, host_bytes, len, device, false, out);
}

QMM_API int qmm_weight_create_from_device(int dtype, size_t n, size_t k, const uint8_t* dev_bytes, size_t len,
                                          int device, qmm_weight** out) {
    return weight_create_impl(dtype, n, k, dev_bytes, len, device, true, out);
}

QMM_API int qmm_weight_create_row_shard(int dtype, size_t n, size_t k, const uint8_t* host_bytes, size_t len,
                                        int rank, int world, int device, qmm_weight** out) {
    if (!out || !host_bytes) return fail(QMM_ERR_INVALID_INPUT, "null pointer");
    *out = nullptr;
    int rc = check_shape(dtype, 0, k, n, len);
    if (rc) return rc;
    if (world < 1 || rank < 0 || rank >= world) return fail(QMM_ERR_INVALID_INPUT, "bad rank / world");
    const size_t nb = k / QK;
    if (nb % (size_t)world) return fail(QMM_ERR_SHAPE_MISMATCH, "k/32 blocks do not split evenly over the ranks");
    int ndev = 0;
    if (cudaGetDeviceCount(&ndev) != cudaSuccess || ndev == 0) {
        cudaGetLastError();
        return fail(QMM_ERR_NO_DEVICE, "no CUDA device");
    }
    if (device < 0 || device >= ndev) return fail(QMM_ERR_INVALID_INPUT, "bad device index");
    const size_t bb = (size_t)block_bytes(dtype), row = nb * bb, local = row / (size_t)world;
    const uint8_t* src = host_bytes + (size_t)rank * local;
    return weight_build(dtype, n, k / (size_t)world, device, 0,
                        [&](uint8_t* d) { return cudaMemcpy2D(d, local, src, row, local, n, cudaMemcpyHostToDevice); },
                        out);
}

QMM_API int qmm_weight_fuse_rows(const qmm_weight* const* parts, size_t count, qmm_weight** out) {
    if (!out || !parts || count == 0) return fail(QMM_ERR_INVALID_INPUT, "null pointer or no parts");
    *out = nullptr;
    size_t rows = 0;
    for (size_t i = 0; i < count; ++i) {
        const qmm_weight* p = parts[i];
        if (!p) return fail(QMM_ERR_INVALID_INPUT, "null part");
        if (p->gate_hidden) return fail(QMM_ERR_INVALID_INPUT, "part is a gate/up weight");
        if (p->dtype != parts[0]->dtype) return fail(QMM_ERR_DTYPE_MISMATCH, "parts differ in block type");
        if (p->k != parts[0]->k) return fail(QMM_ERR_SHAPE_MISMATCH, "parts differ in in_features");
        if (p->device != parts[0]->device) return fail(QMM_ERR_INVALID_INPUT, "parts on different devices");
        rows += p->n;
    }
    if (rows > (size_t)INT32_MAX) return fail(QMM_ERR_SHAPE_MISMATCH, "shape out of range");
    const int dt = parts[0]->dtype;
    const size_t k = parts[0]->k;
    return weight_build(dt, rows, k, parts[0]->device, 0, [&](uint8_t* d) {
        size_t off = 0;
        for (size_t i = 0; i < count; ++i) {
            const size_t b = parts[i]->n * row_bytes_of(dt, k);
            cudaError_t e = cudaMemcpyAsync(d + off, parts[i]->dev, b, cudaMemcpyDeviceToDevice, 0);
            if (e != cudaSuccess) return e;
            off += b;
        }
        return cudaSuccess;
    }, out);
}

QMM_API int qmm_weight_fuse_gate_up(const qmm_weight* gate, const qmm_weight* up, qmm_weight** out) {
    if (!out || !gate || !up) return fail(QMM_ERR_INVALID_INPUT, "null pointer");
    *out = nullptr;
    if (gate->gate_hidden || up->gate_hidden) return fail(QMM_ERR_INVALID_INPUT, "part is a gate/up weight");
    if (gate->dtype != up->dtype) return fail(QMM_ERR_DTYPE_MISMATCH, "gate and up differ in block type");
    if (gate->k != up->k || gate->n != up->n) return fail(QMM_ERR_SHAPE_MISMATCH, "gate and up differ in shape");
    if (gate->device != up->device) return fail(QMM_ERR_INVALID_INPUT, "gate and up on different devices");
    const size_t hidden = gate->n, G = kGateGroup;
    if (hidden == 0) return fail(QMM_ERR_SHAPE_MISMATCH, "empty gate");
    const size_t groups = (hidden + G - 1) / G;
    if (2 * G * groups > (size_t)INT32_MAX) return fail(QMM_ERR_SHAPE_MISMATCH, "shape out of range");
    const size_t rb = row_bytes_of(gate->dtype, gate->k);
    return weight_build(gate->dtype, 2 * G * groups, gate->k, gate->device, hidden, [&](uint8_t* d) {
        // rows padded to whole groups with zero blocks (d = 0: every product 0)
        cudaError_t e = cudaMemsetAsync(d, 0, 2 * G * groups * rb, 0);
        const size_t full = hidden / G, tail = hidden % G;
        const qmm_weight* src[2] = {gate, up};
        for (int h = 0; h < 2 && e == cudaSuccess; ++h) {
            if (full)  // group j of this half -> fused rows [2Gj + hG, 2Gj + hG + G)
                e = cudaMemcpy2DAsync(d + h * G * rb, 2 * G * rb, src[h]->dev, G * rb, G * rb, full,
                                      cudaMemcpyDeviceToDevice, 0);
            if (e == cudaSuccess && tail)
                e = cudaMemcpyAsync(d + (2 * G * full + h * G) * rb, src[h]->dev + full * G * rb, tail * rb,
                                    cudaMemcpyDeviceToDevice, 0);
        }
        return e;
    }, out);
}

QMM_API int qmm_weight_gate_hidden(const qmm_weight* w, size_t* hidden) {
    if (!w || !hidden) return fail(QMM_ERR_INVALID_INPUT, "null pointer");
    *hidden = w->gate_hidden;
    return QMM_OK;
}

QMM_API int qmm_gated_forward(const qmm_weight* w, const float* x_dev, size_t m, float* out_dev, int act_fn,
                              void* stream) {
    if (!w || !x_dev || !out_dev) return fail(QMM_ERR_INVALID_INPUT, "null pointer");
    if (!w->gate_hidden) return fail(QMM_ERR_INVALID_INPUT, "not a gate/up weight");
    if (act_fn != QMM_GELU && act_fn != QMM_SILU) return fail(QMM_ERR_INVALID_INPUT, "unknown activation");
    if (m == 0) return QMM_OK;
    if (m > (size_t)INT32_MAX) return fail(QMM_ERR_SHAPE_MISMATCH, "shape out of range");
    DeviceGuard guard(w->device);
    if (!guard.ok) return fail(QMM_ERR_CUDA, "cudaSetDevice failed");
    const size_t need = workspace_for(w->dtype, QMM_ACT_F32, m, w->n, w->k, w->device);
    void* ws = nullptr;
    int rc = get_workspace(w->device, stream, need, &ws);
    if (rc) return rc;
    GatedOut g;
    g.act = act_fn;
    g.out = out_dev;
    g.hidden = (int64_t)w->gate_hidden;
    return run_matmul(w->dtype, QMM_ACT_F32, x_dev, w->dev, m, w->k, w->n, nullptr, ws, need, (cudaStream_t)stream,
                      /*immutable_w=*/true, g);
}

QMM_API int qmm_weight_destroy(qmm_weight* w) {
    if (!w) return QMM_OK;
    {
        DeviceGuard guard(w->device);
        cudaFree(w->dev);
    }
    delete w;
    return QMM_OK;
}

QMM_API int qmm_weight_info(const qmm_weight* w, int* dtype, size_t* n, size_t* k, const uint8_t** dev_bytes,
                            int* device) {
    if (!w) return fail(QMM_ERR_INVALID_INPUT, "null pointer");
    if (dtype) *dtype = w->dtype;
    if (n) *n = w->n;
    if (k) *k = w->k;
    if (dev_bytes) *dev_bytes = w->dev;
    if (device) *device = w->device;
    return QMM_OK;
}

QMM_API int qmm_checksum_dev(const void* data_dev, size_t len, void* stream, unsigned long long* out) {
    if (!out || (!data_dev && len)) return fail(QMM_ERR_INVALID_INPUT, "null pointer");
    if ((uintptr_t)data_dev & 3) return fail(QMM_ERR_INVALID_INPUT, "misaligned pointer (4 B)");
    if (current_device() < 0) return fail(QMM_ERR_NO_DEVICE, "no CUDA device");
    cudaStream_t st = (cudaStream_t)stream;
    // one accumulator per device (the module's __device__ variable); calls are serialised
    static std::mutex mu;
    std::lock_guard<std::mutex> lock(mu);
    void* acc = nullptr;
    QMM_CUDA(cudaGetSymbolAddress(&acc, g_qmm_checksum_acc));
    QMM_CUDA(cudaMemsetAsync(acc, 0, sizeof(unsigned long long), st));
    if (len) QMM_CUDA(launch_checksum(static_cast<const uint8_t*>(data_dev), len, static_cast<unsigned long long*>(acc), st));
    unsigned long long v = 0;
    QMM_CUDA(cudaMemcpyAsync(&v, acc, sizeof v, cudaMemcpyDeviceToHost, st));
    QMM_CUDA(cudaStreamSynchronize(st));
    *out = v;
    return QMM_OK;
}

QMM_API int qmm_weight_checksum(const qmm_weight* w, unsigned long long* out) {
    if (!w || !out) return fail(QMM_ERR_INVALID_INPUT, "null pointer");
    DeviceGuard guard(w->device);
    if (!guard.ok) return fail(QMM_ERR_CUDA, "cudaSetDevice failed");
    return qmm_checksum_dev(w->dev, w->len, nullptr, out);
}

QMM_API size_t qmm_workspace_size(int dtype, int act, size_t m, size_t n, size_t k) {
    if (!valid_dtype(dtype) || k % QK || k == 0) return 0;
    const int dev = current_device();
    if (dev < 0) return 0;
    return workspace_for(dtype, act, m, n, k, dev);
}

QMM_API int qmm_reserve_workspace(int device, void* stream, size_t bytes) {
    DeviceGuard guard(device);
    if (!guard.ok) return fail(QMM_ERR_INVALID_INPUT, "bad device");
    void* p = nullptr;
    return get_workspace(device, stream, bytes, &p);
}

QMM_API int qmm_matmul_dev(int dtype, int act, const float* x_dev, const uint8_t* w_dev, size_t w_len, size_t m,
                           size_t k, size_t n, float* y_dev, void* workspace_dev, size_t workspace_bytes,
                           void* stream) {
    if (act != QMM_ACT_F32 && act != QMM_ACT_Q8_0) return fail(QMM_ERR_INVALID_INPUT, "bad activation mode");
    int rc = check_shape(dtype, m, k, n, w_len);
    if (rc) return rc;
    if (m == 0 || n == 0) return QMM_OK;
    if (!x_dev || !w_dev || !y_dev || !workspace_dev) return fail(QMM_ERR_INVALID_INPUT, "null pointer");
    if (((uintptr_t)w_dev & 15) || ((uintptr_t)x_dev & 3) || ((uintptr_t)y_dev & 3) || ((uintptr_t)workspace_dev & 255))
        return fail(QMM_ERR_INVALID_INPUT, "misaligned pointer (w 16 B, x/y 4 B, workspace 256 B)");
    return run_matmul(dtype, act, x_dev, w_dev, m, k, n, y_dev, workspace_dev, workspace_bytes,
                      (cudaStream_t)stream);
}

QMM_API int qmm_linear_forward(const qmm_weight* w, const float* x_dev, size_t m, float* y_dev, int act,
                               void* stream) {
    if (!w || !x_dev || !y_dev) return fail(QMM_ERR_INVALID_INPUT, "null pointer");
    if (w->gate_hidden) return fail(QMM_ERR_INVALID_INPUT, "gate/up weight: use qmm_gated_forward");
    if (act != QMM_ACT_F32 && act != QMM_ACT_Q8_0) return fail(QMM_ERR_INVALID_INPUT, "bad activation mode");
    if (m == 0) return QMM_OK;
    DeviceGuard guard(w->device);
    if (!guard.ok) return fail(QMM_ERR_CUDA, "cudaSetDevice failed");
    const size_t need = workspace_for(w->dtype, act, m, w->n, w->k, w->device);
    void* ws = nullptr;
    int rc = get_workspace(w->device, stream, need, &ws);
    if (rc) return rc;
    return run_matmul(w->dtype, act, x_dev, w->dev, m, w->k, w->n, y_dev, ws, need, (cudaStream_t)stream,
                      /*immutable_w=*/true);
}

QMM_API int qmm_linear_forward_host(const qmm_weight* w, const float* x_host, size_t m, float* y_host, int act,
                                    void* stream) {
    if (!w || !x_host || !y_host) return fail(QMM_ERR_INVALID_INPUT, "null pointer");
    if (w->gate_hidden) return fail(QMM_ERR_INVALID_INPUT, "gate/up weight: use qmm_gated_forward");
    if (act != QMM_ACT_F32 && act != QMM_ACT_Q8_0) return fail(QMM_ERR_INVALID_INPUT, "bad activation mode");
    if (m == 0) return QMM_OK;
    DeviceGuard guard(w->device);
    if (!guard.ok) return fail(QMM_ERR_CUDA, "cudaSetDevice failed");
    auto al = [](size_t v) { return (v + 255) & ~size_t(255); };
    const size_t ws_need = workspace_for(w->dtype, act, m, w->n, w->k, w->device);
    const size_t io = al(m * w->k * 4) + al(m * w->n * 4);
    void* ws = nullptr;
    int rc = get_workspace(w->device, stream, ws_need, &ws);
    if (rc) return rc;
    // staging buffers for x/y live apart from the compute workspace, so a
    // graph captured with qmm_linear_forward on this stream keeps its addresses
    void* iob = nullptr;
    {
        std::lock_guard<std::mutex> lock(g_ws_mu);
        Buffer& b = g_io[{w->device, stream}];
        if (b.bytes < io) {
            if (b.ptr) {
                cudaStreamSynchronize((cudaStream_t)stream);
                cudaFree(b.ptr);
                b.ptr = nullptr;
                b.bytes = 0;
            }
            QMM_CUDA(cudaMalloc(&b.ptr, io));
            b.bytes = io;
        }
        iob = b.ptr;
    }
    uint8_t* base = static_cast<uint8_t*>(iob);
    float* xd = reinterpret_cast<float*>(base);
    float* yd = reinterpret_cast<float*>(base + al(m * w->k * 4));
    cudaStream_t st = (cudaStream_t)stream;
    QMM_CUDA(cudaMemcpyAsync(xd, x_host, m * w->k * 4, cudaMemcpyHostToDevice, st));
    rc = run_matmul(w->dtype, act, xd, w->dev, m, w->k, w->n, yd, ws, ws_need, st, /*immutable_w=*/true);
    if (rc) return rc;
    QMM_CUDA(cudaMemcpyAsync(y_host, yd, m * w->n * 4, cudaMemcpyDeviceToHost, st));
    QMM_CUDA(cudaStreamSynchronize(st));
    return QMM_OK;
}

// Allocation-free matmul: the same kernels as qmm_matmul_dev, with the
// workspace taken from the library's fixed device array instead of the
// caller. For callers that may not allocate device memory (a plugin whose
// host framework owns the device memory pool, or a serving loop that cannot
// afford cudaMalloc's implicit device-wide synchronisation).
//  * Set-up: the first call on a device (with that device current) looks up
//    the array's device address with cudaGetSymbolAddress; make that first
//    call before any stream capture. Later calls only read the cached address.
//  * Limit: the plan's workspace must fit in 4 MiB (QMM_NOALLOC_SCRATCH_BYTES);
//    larger shapes return QMM_ERR_INVALID_INPUT.
//  * The array is shared by every call in the process and keeps the last
//    call's contents. The parts that must start at zero (the split-K tickets)
//    are cleared by each call's first kernel; everything else is overwritten
//    before it is read. Calls that overlap on the GPU (different streams, or
//    different host threads without ordering) race on it.
//  * Calls no cudaMalloc/cudaFree and no heap-allocating routine: the tensor
//    map is encoded on the stack each call, and the planner's occupancy
//    answers live in fixed-size tables (filled by the first call per kernel
//    and shared-memory size, which also raises that kernel's shared-memory
//    limit -- another reason to make the first calls before any capture).
//  * Runs the GEMV kernels only (M in chunks of at most 64 rows): calls with
//    17 or more f32-activation rows, which qmm_matmul_dev sends to the
//    tensor-core GEMM when the row pitch allows, are slower here.
namespace {
constexpr int kNoAllocMaxDevices = 64;
std::mutex g_noalloc_mu;
void* g_noalloc_addr[kNoAllocMaxDevices] = {};
int* g_noalloc_err[kNoAllocMaxDevices] = {};
}  // namespace

QMM_API int qmm_matmul_dev_noalloc(int dtype, int act, const float* x_dev, const uint8_t* w_dev, size_t w_len,
                                   size_t m, size_t k, size_t n, float* y_dev, void* stream) {
    if (act != QMM_ACT_F32 && act != QMM_ACT_Q8_0) return fail(QMM_ERR_INVALID_INPUT, "bad activation mode");
    int rc = check_shape(dtype, m, k, n, w_len);
    if (rc) return rc;
    if (m == 0 || n == 0) return QMM_OK;
    if (!x_dev || !w_dev || !y_dev) return fail(QMM_ERR_INVALID_INPUT, "null pointer");
    if (((uintptr_t)w_dev & 15) || ((uintptr_t)x_dev & 3) || ((uintptr_t)y_dev & 3))
        return fail(QMM_ERR_INVALID_INPUT, "misaligned pointer (w 16 B, x/y 4 B)");
    int dev = -1;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0) return fail(QMM_ERR_NO_DEVICE, "no CUDA device");
    if (dev >= kNoAllocMaxDevices) return fail(QMM_ERR_INVALID_INPUT, "device index beyond the no-alloc table");
    void* scratch = nullptr;
    int* err = nullptr;
    {
        std::lock_guard<std::mutex> lock(g_noalloc_mu);
        if (!g_noalloc_addr[dev]) {  // one-time set-up on this device
            void* p = nullptr;
            cudaError_t e = cudaGetSymbolAddress(&p, g_qmm_noalloc_scratch);
            if (e != cudaSuccess) return cuda_fail(e, "cudaGetSymbolAddress(no-alloc scratch)");
            void* q = nullptr;
            e = cudaGetSymbolAddress(&q, g_qmm_device_error);
            if (e != cudaSuccess) return cuda_fail(e, "cudaGetSymbolAddress(error word)");
            g_noalloc_err[dev] = static_cast<int*>(q);
            g_noalloc_addr[dev] = p;
        }
        scratch = g_noalloc_addr[dev];
        err = g_noalloc_err[dev];
    }
    int sms = 0;
    if (cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || sms <= 0) sms = 148;
    for (size_t r0 = 0; r0 < m; r0 += kMaxGemvRows) {
        const size_t rows = (m - r0) < kMaxGemvRows ? (m - r0) : kMaxGemvRows;
        GemvPlan p;
        if (!gemv_plan(dtype, act == QMM_ACT_Q8_0, (int)rows, (int)n, (int)k, sms, &p))
            return fail(QMM_ERR_SHAPE_MISMATCH, "shape not supported");
        const size_t need = gemv_workspace_bytes(p);
        if (need > kNoAllocScratchBytes) {
            char msg[160];
            snprintf(msg, sizeof msg, "workspace of %zu bytes exceeds the no-alloc scratch limit of %zu bytes", need,
                     kNoAllocScratchBytes);
            return fail(QMM_ERR_INVALID_INPUT, msg);
        }
        GemvWorkspace w_s;
        gemv_workspace_carve(p, scratch, &w_s);
        cudaError_t e = launch_gemv(p, w_dev, x_dev + r0 * k, y_dev + r0 * n, w_s, err, (cudaStream_t)stream,
                                    /*no_host_alloc=*/true);
        if (e != cudaSuccess) return cuda_fail(e, "launch_gemv (no-alloc)");
    }
    return QMM_OK;
}

QMM_API int qmm_quantize_dev(int dtype, int variant, const float* x_dev, size_t n, uint8_t* out_dev,
                             float* scales_dev, void* stream) {
    if (!x_dev || !out_dev) return fail(QMM_ERR_INVALID_INPUT, "null pointer");
    if (!valid_dtype(dtype)) return fail(QMM_ERR_DTYPE_MISMATCH, "unsupported block type id");
    if (n % QK) return fail(QMM_ERR_BLOCK_ALIGNMENT, "element count not divisible by 32");
    cudaError_t e;
    if (dtype == QMM_Q8_0) e = launch_quantize_q8_0(x_dev, (int64_t)n, out_dev, scales_dev, variant == 1, (cudaStream_t)stream);
    else if (dtype == QMM_Q4_0) e = launch_quantize_q4_0(x_dev, (int64_t)n, out_dev, (cudaStream_t)stream);
    else e = launch_quantize_q4_1(x_dev, (int64_t)n, out_dev, (cudaStream_t)stream);
    if (e != cudaSuccess) return cuda_fail(e, "quantize");
    return QMM_OK;
}

QMM_API int qmm_dequantize_dev(int dtype, const uint8_t* w_dev, size_t w_len, size_t n_elements, float* out_dev,
                               void* stream) {
    if (!w_dev || !out_dev) return fail(QMM_ERR_INVALID_INPUT, "null pointer");
    if (!valid_dtype(dtype)) return fail(QMM_ERR_DTYPE_MISMATCH, "unsupported block type id");
    if (n_elements % QK) return fail(QMM_ERR_BLOCK_ALIGNMENT, "element count not divisible by 32");
    if (w_len < n_elements / QK * block_bytes(dtype)) return fail(QMM_ERR_SHAPE_MISMATCH, "buffer too short");
    cudaError_t e = launch_dequantize(dtype, w_dev, (int64_t)n_elements, out_dev, (cudaStream_t)stream);
    if (e != cudaSuccess) return cuda_fail(e, "dequantize");
    return QMM_OK;
}

QMM_API int qmm_gated_act_dev(int act_fn, const float* gate_dev, const float* up_dev, size_t m, size_t hidden,
                              size_t ld, float* out_dev, void* stream) {
    if (act_fn != QMM_GELU && act_fn != QMM_SILU && act_fn != QMM_RELU)
        return fail(QMM_ERR_INVALID_INPUT, "unknown activation");
    if (m * hidden == 0) return QMM_OK;
    if (!gate_dev || !out_dev) return fail(QMM_ERR_INVALID_INPUT, "null pointer");
    if (ld < hidden) return fail(QMM_ERR_SHAPE_MISMATCH, "row stride below hidden");
    cudaError_t e = launch_gated_act(act_fn, gate_dev, up_dev, (int64_t)m, (int64_t)hidden, (int64_t)ld, out_dev,
                                     (cudaStream_t)stream);
    if (e != cudaSuccess) return cuda_fail(e, "gated activation");
    return QMM_OK;
}

}  // extern "C"

// ---- decode-step pieces (device pointers, stream-ordered) ------------------------
namespace {
bool dims_ok(size_t v) { return v > 0 && v <= (size_t)INT32_MAX; }
}  // namespace

QMM_API int qmm_embed_q8_dev(const uint8_t* emb_dev, size_t vocab, size_t hidden, const int* tokens_dev,
                             size_t batch, float scale, float* x_dev, void* stream) {
    if (!emb_dev || !tokens_dev || !x_dev) return fail(QMM_ERR_INVALID_INPUT, "null pointer");
    if (hidden % QK) return fail(QMM_ERR_BLOCK_ALIGNMENT, "hidden size not divisible by 32");
    if (!dims_ok(vocab) || !dims_ok(hidden) || batch > (size_t)INT32_MAX)
        return fail(QMM_ERR_SHAPE_MISMATCH, "shape out of range");
    cudaError_t e = launch_embed_q8(emb_dev, (int)hidden, tokens_dev, (int)batch, (int)vocab, scale, x_dev,
                                    (cudaStream_t)stream);
    return e == cudaSuccess ? QMM_OK : cuda_fail(e, "embed");
}

QMM_API int qmm_rmsnorm_dev(const float* x_dev, const float* w_dev, float offset, float eps, size_t rows, size_t dim,
                            float* y_dev, size_t ld_y, void* stream) {
    if (!x_dev || !w_dev || !y_dev) return fail(QMM_ERR_INVALID_INPUT, "null pointer");
    if (!dims_ok(dim) || rows > (size_t)INT32_MAX || ld_y > (size_t)INT32_MAX || (ld_y && ld_y < dim))
        return fail(QMM_ERR_SHAPE_MISMATCH, "shape out of range");
    cudaError_t e = launch_rmsnorm(x_dev, w_dev, offset, eps, (int)rows, (int)dim, y_dev, (int)ld_y,
                                   (cudaStream_t)stream);
    return e == cudaSuccess ? QMM_OK : cuda_fail(e, "rmsnorm");
}

QMM_API int qmm_residual_rmsnorm_dev(float* x_dev, const float* branch_dev, const float* w_post_dev,
                                     const float* w_next_dev, float offset, float eps, size_t rows, size_t dim,
                                     float* h_dev, size_t ld_h, void* stream) {
    if (!x_dev || !branch_dev || !w_post_dev || (w_next_dev && !h_dev))
        return fail(QMM_ERR_INVALID_INPUT, "null pointer");
    if (!dims_ok(dim) || rows > (size_t)INT32_MAX || ld_h > (size_t)INT32_MAX || (ld_h && ld_h < dim))
        return fail(QMM_ERR_SHAPE_MISMATCH, "shape out of range");
    cudaError_t e = launch_residual_norm(x_dev, branch_dev, w_post_dev, w_next_dev, offset, eps, (int)rows, (int)dim,
                                         h_dev, (int)ld_h, (cudaStream_t)stream);
    return e == cudaSuccess ? QMM_OK : cuda_fail(e, "residual rmsnorm");
}

QMM_API int qmm_qk_rope_cache_dev(const float* qkv_dev, size_t batch, int n_heads, int n_kv_heads, int head_dim,
                                  const float* q_norm_dev, const float* k_norm_dev, float offset, float eps,
                                  const float* cos_dev, const float* sin_dev, const int* pos_dev, int ctx,
                                  float* q_out_dev, float* k_cache_dev, float* v_cache_dev, void* stream) {
    if (!qkv_dev || !q_norm_dev || !k_norm_dev || !cos_dev || !sin_dev || !pos_dev || !q_out_dev || !k_cache_dev ||
        !v_cache_dev)
        return fail(QMM_ERR_INVALID_INPUT, "null pointer");
    if (n_heads <= 0 || n_kv_heads <= 0 || n_heads % n_kv_heads || head_dim <= 0 || head_dim % 64 ||
        head_dim > 256 || ctx <= 0 || batch > (size_t)INT32_MAX)
        return fail(QMM_ERR_SHAPE_MISMATCH, "heads, head_dim (a multiple of 64, at most 256) or context out of range");
    cudaError_t e = launch_qk_rope_cache(qkv_dev, (int)batch, n_heads, n_kv_heads, head_dim, q_norm_dev, k_norm_dev,
                                         offset, eps, cos_dev, sin_dev, pos_dev, ctx, q_out_dev, k_cache_dev,
                                         v_cache_dev, (cudaStream_t)stream);
    return e == cudaSuccess ? QMM_OK : cuda_fail(e, "qk rope cache");
}

QMM_API size_t qmm_attention_partial_floats(size_t batch, int n_heads, int head_dim, int ctx) {
    if (batch > (size_t)INT32_MAX || n_heads <= 0 || head_dim <= 0 || ctx <= 0) return 0;
    return attn_partial_floats((int)batch, n_heads, head_dim, ctx);
}

QMM_API int qmm_attention_decode_dev(const float* q_dev, const float* k_cache_dev, const float* v_cache_dev,
                                     size_t batch, int n_heads, int n_kv_heads, int head_dim, const int* pos_dev,
                                     int ctx, float inv_scale, float* partial_dev, float* out_dev, void* stream) {
    if (!q_dev || !k_cache_dev || !v_cache_dev || !pos_dev || !partial_dev || !out_dev)
        return fail(QMM_ERR_INVALID_INPUT, "null pointer");
    if (n_heads <= 0 || n_heads > 8 || n_kv_heads <= 0 || n_heads % n_kv_heads || head_dim <= 0 || head_dim > 256 ||
        ctx <= 0 || batch > (size_t)INT32_MAX)
        return fail(QMM_ERR_SHAPE_MISMATCH, "heads (at most 8), head_dim (at most 256) or context out of range");
    cudaError_t e = launch_attention(q_dev, k_cache_dev, v_cache_dev, (int)batch, n_heads, n_kv_heads, head_dim,
                                     pos_dev, ctx, inv_scale, partial_dev, out_dev, (cudaStream_t)stream);
    return e == cudaSuccess ? QMM_OK : cuda_fail(e, "attention");
}

QMM_API int qmm_attention_decode_fused_dev(const float* qkv_dev, size_t batch, int n_heads, int n_kv_heads,
                                           int head_dim, const float* q_norm_dev, const float* k_norm_dev, float offset,
                                           float eps, const float* cos_dev, const float* sin_dev, const int* pos_dev,
                                           int ctx, float* k_cache_dev, float* v_cache_dev, float inv_scale,
                                           float* partial_dev, float* out_dev, void* stream) {
    if (!qkv_dev || !q_norm_dev || !k_norm_dev || !cos_dev || !sin_dev || !pos_dev || !k_cache_dev || !v_cache_dev ||
        !partial_dev || !out_dev)
        return fail(QMM_ERR_INVALID_INPUT, "null pointer");
    if (n_heads <= 0 || n_heads > 8 || n_kv_heads <= 0 || n_heads % n_kv_heads || head_dim <= 0 || head_dim % 64 ||
        head_dim > 256 || ctx <= 0 || ctx > 64 * 32 || batch > (size_t)INT32_MAX)
        return fail(QMM_ERR_SHAPE_MISMATCH,
                    "heads (at most 8), head_dim (a multiple of 64, at most 256) or context (at most 2048) out of range");
    cudaError_t e = launch_attention_fused(qkv_dev, (int)batch, n_heads, n_kv_heads, head_dim, q_norm_dev, k_norm_dev,
                                           offset, eps, cos_dev, sin_dev, pos_dev, ctx, k_cache_dev, v_cache_dev,
                                           inv_scale, partial_dev, out_dev, (cudaStream_t)stream);
    return e == cudaSuccess ? QMM_OK : cuda_fail(e, "fused attention");
}

QMM_API int qmm_add_int_dev(int* p_dev, int value, void* stream) {
    if (!p_dev) return fail(QMM_ERR_INVALID_INPUT, "null pointer");
    cudaError_t e = launch_add_int(p_dev, value, (cudaStream_t)stream);
    return e == cudaSuccess ? QMM_OK : cuda_fail(e, "add int");
}
