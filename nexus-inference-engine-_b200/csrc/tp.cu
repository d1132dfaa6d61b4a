// Tensor parallelism over NCCL (NVLink 5 / NVSwitch): the north-star split of
// one projection across the GPUs of a box.  The reference runs on one device
// only and has no counterpart; the split rules are
//   COL (QKV, gate, up):  rank r owns output rows [r*N/T, (r+1)*N/T); no exchange.
//   ROW (O, down):        rank r owns reduction columns [r*K/T, (r+1)*K/T);
//                         the fp32 partial outputs are summed by ncclAllReduce.
//
// NCCL is resolved at run time (dlopen of libnccl.so.2, preferring the copy
// already loaded into the process, e.g. by torch.distributed; NXQ_NCCL_LIB
// names another library), so libnxq.so has no link-time NCCL dependency and
// the single-GPU entry points work without it.
//
// Failure detection.  The reference has a single device and silently
// zero-fills on failure (compute_dispatch.cpp:174-176).  Here a collective
// whose peer has died never completes on its own, so nxq_tp_wait polls the
// stream and ncclCommGetAsyncError until the work is done, NCCL reports an
// error, or a deadline passes; in the last two cases it aborts the
// communicator (ncclCommAbort ends the NCCL kernels still waiting) and every
// later TP call fails with NXQ_ERR_STATE until nxq_tp_shutdown and a new
// nxq_tp_init.  Every TP call also checks for an asynchronous error first.
#include <dlfcn.h>
#include <nccl.h>

#include <atomic>
#include <chrono>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <mutex>
#include <thread>
#include <vector>

#include "nxq_internal.h"
#include "qmm_mma.h"
#include "tp_p2p.h"

namespace nxq {
int qmatmul_dispatch(const Weight* w, const void* x, int x_dtype, void* y, int y_dtype, int64_t M,
                     cudaStream_t st);
}

using namespace nxq;

namespace {

struct NcclApi {
    void* lib = nullptr;
    ncclResult_t (*GetUniqueId)(ncclUniqueId*) = nullptr;
    ncclResult_t (*CommInitRank)(ncclComm_t*, int, ncclUniqueId, int) = nullptr;
    ncclResult_t (*CommDestroy)(ncclComm_t) = nullptr;
    ncclResult_t (*CommAbort)(ncclComm_t) = nullptr;
    ncclResult_t (*CommGetAsyncError)(ncclComm_t, ncclResult_t*) = nullptr;
    ncclResult_t (*AllReduce)(const void*, void*, size_t, ncclDataType_t, ncclRedOp_t, ncclComm_t,
                              cudaStream_t) = nullptr;
    ncclResult_t (*AllGather)(const void*, void*, size_t, ncclDataType_t, ncclComm_t, cudaStream_t) = nullptr;
    const char* (*GetErrorString)(ncclResult_t) = nullptr;
};

NcclApi g_nccl;
std::mutex g_tp_mu;
ncclComm_t g_comm = nullptr;
int g_rank = -1, g_world = 0;
bool g_dead = false;  // the communicator was aborted: TP calls fail until shutdown + init
char g_dead_why[256] = "";
std::atomic<bool> g_hook_stream_pending{false};  // NXQ_HOOK_TP_STREAM_PENDING

// The peer-memory allreduce (tp_p2p.cu): this rank's symmetric buffer, the
// peers' buffers mapped through CUDA IPC, and the launch parameters.
// A device buffer on every rank, mapped into every other rank through CUDA
// IPC (handles exchanged once through the communicator): `at[q]` addresses
// rank q's buffer from this rank (the own one locally).
struct SymBuf {
    void* base = nullptr;
    void* peer[kP2PMaxWorld] = {};
    void* at[kP2PMaxWorld] = {};
};

struct P2PState {
    bool on = false;
    SymBuf buf;
    P2PParams tmpl{};
};
P2PState g_p2p;
constexpr int64_t kP2PCap = 1 << 21;  // floats per data half: allreduces up to 8 MB use peer memory

// The fused row split: the decode GEMV exchanges partial tiles itself.
struct TpxState {
    bool on = false;
    SymBuf buf;
    TpExchange tmpl{};
};
TpxState g_tpx;

int load_nccl() {
    if (g_nccl.lib) return NXQ_OK;
    void* h = nullptr;
    const char* forced = getenv("NXQ_NCCL_LIB");
    if (forced && forced[0]) {
        h = dlopen(forced, RTLD_NOW | RTLD_LOCAL);
        if (!h) return fail(NXQ_ERR_NCCL, "cannot load NXQ_NCCL_LIB=%s: %s", forced, dlerror());
    }
    if (!h) h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_NOLOAD);
    if (!h) h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_GLOBAL);
    if (!h) h = dlopen("libnccl.so", RTLD_NOW | RTLD_GLOBAL);
    if (!h) return fail(NXQ_ERR_NCCL, "cannot load libnccl.so.2: %s", dlerror());
#define NXQ_SYM(field, name)                                                          \
    g_nccl.field = reinterpret_cast<decltype(g_nccl.field)>(dlsym(h, name));          \
    if (!g_nccl.field) return fail(NXQ_ERR_NCCL, "libnccl is missing %s", name);
    NXQ_SYM(GetUniqueId, "ncclGetUniqueId")
    NXQ_SYM(CommInitRank, "ncclCommInitRank")
    NXQ_SYM(CommDestroy, "ncclCommDestroy")
    NXQ_SYM(CommAbort, "ncclCommAbort")
    NXQ_SYM(CommGetAsyncError, "ncclCommGetAsyncError")
    NXQ_SYM(AllReduce, "ncclAllReduce")
    NXQ_SYM(AllGather, "ncclAllGather")
    NXQ_SYM(GetErrorString, "ncclGetErrorString")
#undef NXQ_SYM
    g_nccl.lib = h;
    return NXQ_OK;
}

int nccl_fail(ncclResult_t r, const char* what) {
    return fail(NXQ_ERR_NCCL, "%s: %s", what, g_nccl.GetErrorString ? g_nccl.GetErrorString(r) : "?");
}

// Aborts the communicator (caller holds g_tp_mu); later TP calls fail.
int abort_comm(int status, const char* why) {
    if (g_comm && !g_dead) g_nccl.CommAbort(g_comm);
    g_dead = true;
    snprintf(g_dead_why, sizeof g_dead_why, "%s", why);
    return fail(status, "%s; the TP communicator was aborted (nxq_tp_shutdown, then nxq_tp_init, to rejoin)", why);
}

// A usable communicator with no pending asynchronous error (caller holds
// g_tp_mu); aborts it when NCCL reports one.
int check_comm() {
    if (!g_comm) return fail(NXQ_ERR_STATE, "nxq_tp_init has not been called");
    if (g_dead) return fail(NXQ_ERR_STATE, "the TP communicator was aborted earlier (%s)", g_dead_why);
    ncclResult_t async_err = ncclSuccess;
    ncclResult_t r = g_nccl.CommGetAsyncError(g_comm, &async_err);
    if (r != ncclSuccess) return abort_comm(NXQ_ERR_NCCL, "ncclCommGetAsyncError failed");
    if (async_err != ncclSuccess && async_err != ncclInProgress) {
        char why[200];
        snprintf(why, sizeof why, "NCCL reported an asynchronous error: %s", g_nccl.GetErrorString(async_err));
        return abort_comm(NXQ_ERR_NCCL, why);
    }
    return NXQ_OK;
}

void sym_unmap(SymBuf* sb) {
    for (int r = 0; r < kP2PMaxWorld; ++r)
        if (sb->peer[r]) cudaIpcCloseMemHandle(sb->peer[r]);
    if (sb->base) cudaFree(sb->base);
    *sb = SymBuf{};
}

// Every rank's element is 1 after a ncclMin over ranks of `mine` (1 = ok).
bool all_ranks_ok(bool mine) {
    uint8_t* d = nullptr;
    uint8_t v = mine ? 1 : 0, all = 0;
    if (cudaMalloc(&d, 1) != cudaSuccess) {
        cudaGetLastError();
        return false;  // in practice every rank fails the same tiny allocation
    }
    cudaMemcpy(d, &v, 1, cudaMemcpyHostToDevice);
    if (g_nccl.AllReduce(d, d, 1, ncclUint8, ncclMin, g_comm, 0) == ncclSuccess && cudaStreamSynchronize(0) == cudaSuccess)
        cudaMemcpy(&all, d, 1, cudaMemcpyDeviceToHost);
    cudaFree(d);
    return all == 1;
}

// Allocates `bytes` (zeroed) on every rank and maps every peer's buffer;
// collective over the communicator (caller holds g_tp_mu).  Either every rank
// succeeds or none keeps anything.
bool sym_map(size_t bytes, SymBuf* sb) {
    *sb = SymBuf{};
    bool ok = cudaMalloc(&sb->base, bytes) == cudaSuccess && cudaMemset(sb->base, 0, bytes) == cudaSuccess &&
              cudaDeviceSynchronize() == cudaSuccess;
    cudaIpcMemHandle_t mine{};
    ok = ok && cudaIpcGetMemHandle(&mine, sb->base) == cudaSuccess;
    // Every rank takes part in the exchange, whatever happened above (a rank
    // that failed sends a zero handle and all of them then give up).
    const size_t hb = sizeof(cudaIpcMemHandle_t);
    uint8_t* dh = nullptr;
    if (cudaMalloc(&dh, (size_t)g_world * hb) != cudaSuccess) {
        cudaGetLastError();
        sym_unmap(sb);
        return false;
    }
    cudaMemcpy(dh + (size_t)g_rank * hb, &mine, hb, cudaMemcpyHostToDevice);
    std::vector<cudaIpcMemHandle_t> hs((size_t)g_world);
    bool got = g_nccl.AllGather(dh + (size_t)g_rank * hb, dh, hb, ncclUint8, g_comm, 0) == ncclSuccess &&
               cudaStreamSynchronize(0) == cudaSuccess &&
               cudaMemcpy(hs.data(), dh, g_world * hb, cudaMemcpyDeviceToHost) == cudaSuccess;
    cudaFree(dh);
    if (!all_ranks_ok(ok && got)) {
        cudaGetLastError();
        sym_unmap(sb);
        return false;
    }
    for (int q = 0; q < g_world && ok; ++q) {
        if (q == g_rank) {
            sb->at[q] = sb->base;
            continue;
        }
        ok = cudaIpcOpenMemHandle(&sb->peer[q], hs[q], cudaIpcMemLazyEnablePeerAccess) == cudaSuccess;
        sb->at[q] = sb->peer[q];
    }
    // Whether every rank could map every peer decides for all of them.
    if (!all_ranks_ok(ok)) {
        cudaGetLastError();
        sym_unmap(sb);
        return false;
    }
    return true;
}

// The peer-memory allreduce, when NXQ_TP_ALLREDUCE=p2p asks for it.  It is
// not the default: on two B200 it took 16-19 us per call for 16 KB - 2 MB
// against NCCL's 12 us (measured in a CUDA graph of the benchmark's calls).
// Any failure leaves it off; the allreduce then runs on NCCL.
void p2p_setup() {
    if (!sym_map(p2p_bytes(g_world, kP2PCap), &g_p2p.buf)) return;
    P2PParams& t = g_p2p.tmpl;
    t.rank = g_rank;
    t.world = g_world;
    t.cap = kP2PCap;
    for (int q = 0; q < g_world; ++q) {
        t.data[q] = static_cast<float*>(g_p2p.buf.at[q]);
        t.flags[q] = reinterpret_cast<unsigned long long*>(static_cast<char*>(g_p2p.buf.at[q]) +
                                                           2 * kP2PCap * sizeof(float));
    }
    t.ctl = t.flags[g_rank] + (size_t)g_world * kP2PBlocks;
    g_p2p.on = true;
}

// The fused row split (the default): decode-size row-split calls exchange
// their partial tiles inside the GEMV launch; other calls use NCCL.
void tpx_setup() {
    if (!sym_map(tpx_bytes(g_world), &g_tpx.buf)) return;
    TpExchange& t = g_tpx.tmpl;
    t.on = 1;
    t.rank = g_rank;
    t.world = g_world;
    // NXQ_TP_EXCHANGE=owner: the owner exchange (an all-to-all's volume grows
    // with the world, the owner exchange's stays under twice the output, at
    // the cost of a second hop).  Opt-in: verified on two GPUs, not yet
    // measured at 4 or 8 ranks, where the all-to-all default was measured.
    const char* ex = getenv("NXQ_TP_EXCHANGE");
    t.owner = ex && strcmp(ex, "owner") == 0 ? 1 : 0;
    for (int q = 0; q < g_world; ++q) t.recv[q] = static_cast<unsigned long long*>(g_tpx.buf.at[q]);
    t.ctl = t.recv[g_rank] + (size_t)2 * g_world * kTpxSlotWords;
    g_tpx.on = true;
}

// NXQ_TP_ALLREDUCE: unset or "fused" (the default) = decode-size row splits
// exchange their tiles inside the GEMV launch; "p2p" = the peer-memory
// allreduce kernel; "nccl" = NCCL only.  Measured on two B200 (config-2 down
// shard, graphs of 16 calls, us per call at M = 1 / 8 / 32): fused 13.0 /
// 13.4 / 23.7, GEMV + NCCL allreduce 19.6 / 21.1 / 28.7.
void peer_setup() {
    const char* env = getenv("NXQ_TP_ALLREDUCE");
    if (g_world < 2 || g_world > kP2PMaxWorld) return;
    if (env && strcmp(env, "p2p") == 0) p2p_setup();
    if (!env || strcmp(env, "fused") == 0) tpx_setup();
}

// All ranks' queued work is done before any rank unmaps or frees its buffers
// (a peer's kernel may still read or write them): a device synchronize and a
// one-byte NCCL allreduce as a barrier.
void peer_shutdown() {
    if (!g_p2p.buf.base && !g_tpx.buf.base) return;
    cudaDeviceSynchronize();
    if (!g_dead) all_ranks_ok(true);
    sym_unmap(&g_p2p.buf);
    sym_unmap(&g_tpx.buf);
    g_p2p = P2PState{};
    g_tpx = TpxState{};
}

int check_weight_ptr(nxq_weight_t h, const Weight** out) {
    size_t bytes = 0;
    int rc = nxq_weight_info(h, nullptr, nullptr, nullptr, nullptr, &bytes);
    if (rc) return rc;
    *out = reinterpret_cast<const Weight*>(h);
    return NXQ_OK;
}

}  // namespace

extern "C" {

NXQ_API int nxq_tp_unique_id_size(void) { return (int)sizeof(ncclUniqueId); }

NXQ_API int nxq_tp_unique_id(void* out, size_t n) {
    if (!out || n < sizeof(ncclUniqueId)) return fail(NXQ_ERR_ARG, "buffer smaller than %zu", sizeof(ncclUniqueId));
    int rc = load_nccl();
    if (rc) return rc;
    ncclUniqueId id;
    ncclResult_t r = g_nccl.GetUniqueId(&id);
    if (r != ncclSuccess) return nccl_fail(r, "ncclGetUniqueId");
    memcpy(out, &id, sizeof id);
    return NXQ_OK;
}

NXQ_API int nxq_tp_init(int rank, int world, const void* unique_id, size_t n) {
    if (!unique_id || n < sizeof(ncclUniqueId)) return fail(NXQ_ERR_ARG, "bad unique id");
    if (world < 1 || rank < 0 || rank >= world) return fail(NXQ_ERR_ARG, "rank %d of %d", rank, world);
    std::lock_guard<std::mutex> lk(g_tp_mu);
    if (g_comm) return fail(NXQ_ERR_STATE, "TP group already initialised");
    int rc = load_nccl();
    if (rc) return rc;
    ncclUniqueId id;
    memcpy(&id, unique_id, sizeof id);
    ncclResult_t r = g_nccl.CommInitRank(&g_comm, world, id, rank);
    if (r != ncclSuccess) {
        g_comm = nullptr;
        return nccl_fail(r, "ncclCommInitRank");
    }
    g_rank = rank;
    g_world = world;
    g_dead = false;
    g_dead_why[0] = 0;
    peer_setup();
    return NXQ_OK;
}

NXQ_API int nxq_tp_p2p_enabled(int* on) {
    if (!on) return fail(NXQ_ERR_ARG, "null argument");
    std::lock_guard<std::mutex> lk(g_tp_mu);
    *on = g_p2p.on ? 1 : g_tpx.on ? 2 : 0;
    return NXQ_OK;
}

NXQ_API int nxq_tp_shutdown(void) {
    std::lock_guard<std::mutex> lk(g_tp_mu);
    if (!g_comm) return NXQ_OK;
    peer_shutdown();
    ncclResult_t r = ncclSuccess;
    if (!g_dead) {
        ncclResult_t async_err = ncclSuccess;
        g_nccl.CommGetAsyncError(g_comm, &async_err);
        // A communicator with a pending error cannot be destroyed cleanly.
        r = async_err == ncclSuccess ? g_nccl.CommDestroy(g_comm) : g_nccl.CommAbort(g_comm);
    }
    g_comm = nullptr;
    g_rank = -1;
    g_world = 0;
    g_dead = false;
    if (r != ncclSuccess) return nccl_fail(r, "ncclCommDestroy");
    return NXQ_OK;
}

NXQ_API int nxq_tp_allreduce_f32(float* buf_dev, int64_t count, void* stream) {
    if (!buf_dev || count < 0) return fail(NXQ_ERR_ARG, "bad buffer");
    std::lock_guard<std::mutex> lk(g_tp_mu);
    if (int rc = check_comm()) return rc;
    if (count == 0) return NXQ_OK;
    if (g_p2p.on && count <= kP2PCap) {
        P2PParams p = g_p2p.tmpl;
        p.buf = buf_dev;
        p.count = count;
        p.status = context_status();
        cudaError_t e = launch_p2p_allreduce(p, (cudaStream_t)stream);
        if (e != cudaSuccess) return cuda_fail(e, "peer-memory allreduce launch");
        return NXQ_OK;
    }
    ncclResult_t r = g_nccl.AllReduce(buf_dev, buf_dev, (size_t)count, ncclFloat32, ncclSum, g_comm,
                                      (cudaStream_t)stream);
    if (r != ncclSuccess) {
        // A collective that failed to enqueue on this rank leaves the others
        // waiting for it: abort rather than leave the group half-entered.
        char why[200];
        snprintf(why, sizeof why, "ncclAllReduce failed: %s", g_nccl.GetErrorString(r));
        return abort_comm(NXQ_ERR_NCCL, why);
    }
    return NXQ_OK;
}

NXQ_API int nxq_tp_wait(void* stream, int64_t timeout_ms) {
    if (timeout_ms < 0) return fail(NXQ_ERR_ARG, "negative timeout");
    using clk = std::chrono::steady_clock;
    const auto deadline = clk::now() + std::chrono::milliseconds(timeout_ms);
    for (int polls = 0;; ++polls) {
        {
            std::lock_guard<std::mutex> lk(g_tp_mu);
            if (int rc = check_comm()) return rc;
            cudaError_t q = g_hook_stream_pending.load() ? cudaErrorNotReady : cudaStreamQuery((cudaStream_t)stream);
            if (q == cudaSuccess) return NXQ_OK;
            if (q != cudaErrorNotReady) {
                cudaGetLastError();
                char why[200];
                snprintf(why, sizeof why, "the TP stream failed: %s", cudaGetErrorName(q));
                return abort_comm(NXQ_ERR_CUDA, why);
            }
            if (clk::now() >= deadline) {
                char why[200];
                snprintf(why, sizeof why, "TP work on the stream did not finish within %lld ms (a peer may have "
                         "left)", (long long)timeout_ms);
                return abort_comm(NXQ_ERR_TIMEOUT, why);
            }
        }
        std::this_thread::sleep_for(std::chrono::microseconds(polls < 100 ? 20 : 1000));
    }
}

NXQ_API int nxq_tp_test_hook(int hook, int on) {
    if (hook != NXQ_HOOK_TP_STREAM_PENDING) return fail(NXQ_ERR_ARG, "unknown TP test hook %d", hook);
    g_hook_stream_pending.store(on != 0);
    return NXQ_OK;
}

NXQ_API int nxq_tp_qmatmul(nxq_weight_t shard, const void* x_dev, int x_dtype, void* y_dev,
                           int y_dtype, int64_t M, int split, void* stream) {
    const Weight* w = nullptr;
    int rc = check_weight_ptr(shard, &w);
    if (rc) return rc;
    if (split != NXQ_SPLIT_COL && split != NXQ_SPLIT_ROW) return fail(NXQ_ERR_ARG, "bad split");
    {
        std::lock_guard<std::mutex> lk(g_tp_mu);
        if (int crc = check_comm()) return crc;
    }
    if (split == NXQ_SPLIT_ROW && y_dtype != NXQ_F32)
        return fail(NXQ_ERR_ARG, "ROW split produces fp32 partial sums; y_dtype must be NXQ_F32");
    if (split == NXQ_SPLIT_ROW && g_tpx.on && M > 0 && x_dev && y_dev &&
        (x_dtype == NXQ_F32 || x_dtype == NXQ_F16 || x_dtype == NXQ_BF16)) {
        if ((rc = context_ready())) return rc;
        rc = mma_qmatmul_tp(w, x_dev, x_dtype, static_cast<float*>(y_dev), M, (cudaStream_t)stream, g_tpx.tmpl);
        if (rc != NXQ_ERR_UNSUPPORTED) return rc;
    }
    rc = nxq_qmatmul(shard, x_dev, x_dtype, y_dev, y_dtype, M, stream);
    if (rc || split == NXQ_SPLIT_COL) return rc;
    return nxq_tp_allreduce_f32((float*)y_dev, M * w->shape.N, stream);
}

}  // extern "C"
