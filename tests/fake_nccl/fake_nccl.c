/* A stand-in for libnccl.so.2 for the CPU tests of libqmm.so's tensor-parallel
 * C ABI (include/qmm_tp.h): it implements the entry points the library
 * resolves, with no GPU work, and fails in the way the test selects with
 * fake_nccl_set_mode(). Counters record what the library called.
 *
 * Modes: 0 healthy; 1 init never completes (ncclInProgress forever);
 * 2 init fails asynchronously (ncclSystemError); 3 healthy init, then the
 * communicator reports ncclRemoteError (a peer failed); 4 healthy init, then
 * collectives stay in progress forever (a peer that never joins). */
#include <stdlib.h>
#include <string.h>

typedef struct { char internal[128]; } ncclUniqueId;
typedef struct { int dummy; } fake_comm;
enum { ok = 0, sys_err = 2, remote_err = 6, in_progress = 7 };

static int g_mode = 0;
int fake_nccl_aborts = 0, fake_nccl_destroys = 0, fake_nccl_finalizes = 0, fake_nccl_collectives = 0;
static int g_async = ok;

void fake_nccl_set_mode(int m) {
    g_mode = m;
    fake_nccl_aborts = fake_nccl_destroys = fake_nccl_finalizes = fake_nccl_collectives = 0;
    g_async = ok;
}

int ncclGetUniqueId(ncclUniqueId* id) {
    memset(id->internal, 0x5a, sizeof id->internal);
    return ok;
}
int ncclCommInitRankConfig(void** comm, int nranks, ncclUniqueId id, int rank, void* config) {
    (void)nranks; (void)id; (void)rank; (void)config;
    *comm = calloc(1, sizeof(fake_comm));
    g_async = (g_mode == 1 || g_mode == 2) ? in_progress : ok;
    return in_progress;
}
int ncclCommGetAsyncError(void* comm, int* st) {
    (void)comm;
    if (g_mode == 2 && g_async == in_progress) g_async = sys_err;
    if (g_mode == 3 && fake_nccl_collectives > 0) g_async = remote_err;
    *st = g_async;
    return ok;
}
int ncclCommAbort(void* comm) { fake_nccl_aborts++; free(comm); return ok; }
int ncclCommFinalize(void* comm) { (void)comm; fake_nccl_finalizes++; return ok; }
int ncclCommDestroy(void* comm) { fake_nccl_destroys++; free(comm); return ok; }
static int collective(void) {
    fake_nccl_collectives++;
    if (g_mode == 4) { g_async = in_progress; return in_progress; }
    return ok;
}
int ncclAllGather(const void* s, void* r, size_t n, int t, void* c, void* st) {
    (void)s; (void)r; (void)n; (void)t; (void)c; (void)st;
    return collective();
}
int ncclAllReduce(const void* s, void* r, size_t n, int t, int op, void* c, void* st) {
    (void)s; (void)r; (void)n; (void)t; (void)op; (void)c; (void)st;
    return collective();
}
const char* ncclGetErrorString(int r) {
    return r == sys_err ? "fake: system error" : r == remote_err ? "fake: remote process exited or there was a network error" : "fake";
}
