/* A stand-in for libnccl.so.2 used by tests/test_tp_watchdog.py: it exports
 * the NCCL entry points libnxq resolves at run time (tp.cu) and lets the test
 * choose what they return, so the TP layer's failure handling (asynchronous
 * errors, failed enqueues, a collective that never finishes) runs on a CPU
 * without a GPU or a real communicator.  Return codes follow nccl.h:
 * 0 success, 1 unhandled CUDA error, 6 remote error, 7 in progress. */
#include <stdio.h>
#include <string.h>

typedef struct { char internal[128]; } ncclUniqueId;
typedef void* ncclComm_t;

static int g_async = 0;        /* what ncclCommGetAsyncError reports */
static int g_allreduce_rc = 0; /* what ncclAllReduce returns */
static int g_calls[6];         /* init, destroy, abort, allreduce, get_async, unique_id */
static int g_comm_obj;

void fake_set(int async_err, int allreduce_rc) { g_async = async_err; g_allreduce_rc = allreduce_rc; }
int fake_calls(int which) { return (which >= 0 && which < 6) ? g_calls[which] : -1; }
void fake_reset(void) { memset(g_calls, 0, sizeof g_calls); g_async = 0; g_allreduce_rc = 0; }

int ncclGetUniqueId(ncclUniqueId* id) { memset(id, 7, sizeof *id); g_calls[5]++; return 0; }
int ncclCommInitRank(ncclComm_t* comm, int nranks, ncclUniqueId id, int rank) {
    (void)nranks; (void)id; (void)rank;
    *comm = &g_comm_obj;
    g_calls[0]++;
    return 0;
}
int ncclCommDestroy(ncclComm_t comm) { (void)comm; g_calls[1]++; return 0; }
int ncclCommAbort(ncclComm_t comm) { (void)comm; g_calls[2]++; return 0; }
int ncclCommGetAsyncError(ncclComm_t comm, int* err) { (void)comm; *err = g_async; g_calls[4]++; return 0; }
int ncclAllReduce(const void* s, void* r, size_t n, int dt, int op, ncclComm_t comm, void* stream) {
    (void)s; (void)r; (void)n; (void)dt; (void)op; (void)comm; (void)stream;
    g_calls[3]++;
    return g_allreduce_rc;
}
int ncclAllGather(const void* s, void* r, size_t n, int dt, ncclComm_t comm, void* stream) {
    (void)s; (void)r; (void)n; (void)dt; (void)comm; (void)stream;
    return 0;
}
const char* ncclGetErrorString(int r) {
    static char buf[64];
    snprintf(buf, sizeof buf, "fake nccl error %d", r);
    return buf;
}
