// The C ABI of libnxq.so (include/nxq.h): context, HBM weight residency,
// dispatch to the kernels, and the synchronous host-buffer drop-in.
//
// Reference counterparts:
//   ComputeDispatch::init_gpu / gemm_int4 / clear_buffer_cache
//       nexus/src/compute/compute_dispatch.cpp:47, :142-176, :853-860
//   MetalBackend::wrap_pointer / gemm_int4_gpu / buffer caches
//       nexus/src/compute/metal/metal_backend.mm:814-834, :274-303
#include <cuda_runtime.h>
#if defined(__x86_64__)
#include <immintrin.h>
#endif

#include <atomic>
#include <chrono>
#include <cstddef>
#include <cstdio>
#include <cstring>
#include <mutex>
#include <vector>
#include <unordered_set>

#include "nxq_internal.h"
#include "qmm_gemm.h"
#include "qmm_mma.h"
#include "stream_scratch.h"

namespace nxq {

namespace {

thread_local char g_err[512] = "";

struct Context {
    bool ready = false;
    int device = -1;
    int sm_count = 0;
    int cc_major = 0, cc_minor = 0;
    size_t smem_optin = 0;
    cudaStream_t host_stream = nullptr;  // registration
    DeviceStatus* status = nullptr;  // error word and wait settings (device memory)
    unsigned int* flag_host = nullptr;  // mapped pinned word kernels set on an error
    std::mutex mu;                   // registration, teardown
    std::unordered_set<Weight*> live;
    unsigned generation = 0;         // bumped by every nxq_init: host-call contexts of an old one are stale
};

Context g_ctx;
std::mutex g_init_mu;

// One per calling thread for nxq_qmatmul_host: its own stream and device
// buffers, so concurrent host calls neither share buffers nor take a global
// lock; the buffers grow on the thread's first calls and stay.  All of them
// are freed by nxq_shutdown.
struct HostCall {
    unsigned generation = 0;
    cudaStream_t st = nullptr;
    cudaEvent_t done = nullptr;  // recorded after the output copy; the call spins on it
    void* dx = nullptr;
    size_t dx_bytes = 0;
    void* dy = nullptr;
    size_t dy_bytes = 0;
};
std::mutex g_hostcall_mu;
std::vector<HostCall*> g_hostcalls;
thread_local HostCall* t_hostcall = nullptr;

int host_call_context(HostCall** out) {
    HostCall* hc = t_hostcall;
    if (!hc || hc->generation != g_ctx.generation) {
        hc = new (std::nothrow) HostCall();
        if (!hc) return fail(NXQ_ERR_NOMEM, "host allocation failed");
        hc->generation = g_ctx.generation;
        cudaError_t e = cudaStreamCreateWithFlags(&hc->st, cudaStreamNonBlocking);
        if (e != cudaSuccess) {
            delete hc;
            return cuda_fail(e, "cudaStreamCreate (host-call stream)");
        }
        if ((e = cudaEventCreateWithFlags(&hc->done, cudaEventDisableTiming)) != cudaSuccess) {
            cudaStreamDestroy(hc->st);
            delete hc;
            return cuda_fail(e, "cudaEventCreate (host-call event)");
        }
        std::lock_guard<std::mutex> lk(g_hostcall_mu);
        g_hostcalls.push_back(hc);
        t_hostcall = hc;
    }
    *out = hc;
    return NXQ_OK;
}

// Waits for `ev` by polling it, falling back to a blocking wait after 2 ms.
// A decode call completes in tens of microseconds, sooner than a blocking
// synchronize wakes its thread (measured on a B200 host: a 512 KB copy and
// its wait took 30 us polling, 39 us with a stream synchronize).
cudaError_t wait_spinning(cudaEvent_t ev) {
    const auto t0 = std::chrono::steady_clock::now();
    for (;;) {
        const cudaError_t q = cudaEventQuery(ev);
        if (q != cudaErrorNotReady) return q;
        if (std::chrono::steady_clock::now() - t0 > std::chrono::milliseconds(2)) return cudaEventSynchronize(ev);
#if defined(__x86_64__)
        _mm_pause();
#endif
    }
}

int check_ready() {
    if (!g_ctx.ready) return fail(NXQ_ERR_STATE, "nxq_init has not been called");
    int dev = -1;
    if (cudaGetDevice(&dev) != cudaSuccess || dev != g_ctx.device) {
        cudaError_t e = cudaSetDevice(g_ctx.device);
        if (e != cudaSuccess) return cuda_fail(e, "cudaSetDevice");
    }
    return NXQ_OK;
}

int check_weight(nxq_weight_t h, Weight** out) {
    Weight* w = reinterpret_cast<Weight*>(h);
    if (!w) return fail(NXQ_ERR_ARG, "null weight handle");
    std::lock_guard<std::mutex> lk(g_ctx.mu);
    if (!g_ctx.live.count(w) || w->magic != kWeightMagic)
        return fail(NXQ_ERR_ARG, "weight handle is not live (released or foreign)");
    *out = w;
    return NXQ_OK;
}

bool dtype_ok(int d) { return d == NXQ_F32 || d == NXQ_F16 || d == NXQ_BF16; }
size_t dtype_size(int d) { return d == NXQ_F32 ? 4 : 2; }

int grow(void** buf, size_t* have, size_t need) {
    if (*have >= need) return NXQ_OK;
    if (*buf) cudaFree(*buf);
    *buf = nullptr;
    *have = 0;
    cudaError_t e = cudaMalloc(buf, need);
    if (e != cudaSuccess) return cuda_fail(e, "cudaMalloc (host-call buffers)");
    *have = need;
    return NXQ_OK;
}

// Reads the device status word after a synchronize: a bounded wait that
// gave up (NXQ_ERR_TIMEOUT), or an activation too large for f16
// (NXQ_ERR_RANGE).  The word is cleared once reported.
int report_status(const DeviceStatus& st) {
    if (!st.code) return NXQ_OK;
    // Clear the error (code and where); the settings after it stay.
    cudaMemset(g_ctx.status, 0, 2 * sizeof(unsigned));
    if (st.code == kStatusRange) {
        static const char* const what[] = {"?", "the f16 conversion of fp32/bf16 activations",
                                           "the RMSNorm prologue", "the decode GEMV's activation staging"};
        return fail(NXQ_ERR_RANGE,
                    "an activation of magnitude >= 65520 reached %s: it is outside the f16 range the "
                    "tensor-core kernels compute in (results of that call are not finite)",
                    what[st.where < 4 ? st.where : 0]);
    }
    scratch_reset_counters();
    return fail(NXQ_ERR_TIMEOUT, "device-side bounded wait expired (code %u at %u)", st.code, st.where);
}

int check_device_status() {
    DeviceStatus st{};
    cudaError_t e = cudaMemcpy(&st, g_ctx.status, sizeof st, cudaMemcpyDeviceToHost);
    if (e != cudaSuccess) return cuda_fail(e, "read device status");
    if (st.code) *reinterpret_cast<volatile unsigned int*>(g_ctx.flag_host) = 0u;
    return report_status(st);
}

// After a synchronize: the device status only when a kernel flagged an error.
int check_host_flag() {
    if (!*reinterpret_cast<volatile unsigned int*>(g_ctx.flag_host)) return NXQ_OK;
    return check_device_status();
}

// Registers N rows of K from GGUF blocks.  `src` is host (is_host) or device
// memory; rows are `src_row_blocks` blocks long in the source and blocks
// [blk0, blk0 + K/QK) of each are kept (a column slice for ROW sharding).
int register_impl(const void* src, bool is_host, int type, int64_t N, int64_t K,
                  int64_t src_row_blocks, int64_t blk0, cudaStream_t st, nxq_weight_t* out) {
    TiledShape s;
    if (!make_tiled_shape(type, N, K, &s)) {
        Geometry g;
        if (!geometry_of(type, &g)) return fail(NXQ_ERR_CODEC, "unsupported block type %d", type);
        return fail(NXQ_ERR_SHAPE, "bad shape N=%lld K=%lld for block of %d elements",
                    (long long)N, (long long)K, g.qk);
    }
    Weight* w = new (std::nothrow) Weight();
    if (!w) return fail(NXQ_ERR_NOMEM, "host allocation failed");
    w->magic = kWeightMagic;
    w->device = g_ctx.device;
    w->shape = s;
    w->packed_bytes = (size_t)N * (size_t)(K / s.g.qk) * (size_t)s.g.bb;
    w->dev_bytes = (size_t)s.total_bytes() + kTailPad;
    cudaError_t e = cudaMalloc(&w->dev, w->dev_bytes);
    if (e != cudaSuccess) {
        delete w;
        return cuda_fail(e, "cudaMalloc (weight)");
    }
    auto bail = [&](int status) {
        cudaFree(w->dev);
        delete w;
        return status;
    };
    if ((e = cudaMemsetAsync(w->dev, 0, w->dev_bytes, st)) != cudaSuccess)
        return bail(cuda_fail(e, "cudaMemsetAsync (weight)"));

    const size_t slice_bytes = (size_t)(K / s.g.qk) * s.g.bb;
    const size_t src_pitch = (size_t)src_row_blocks * s.g.bb;
    if (!is_host) {
        // Device source: repack straight from it.
        e = launch_repack((const uint8_t*)src, w->dev, s, 0, N, blk0, src_row_blocks, st);
        if (e != cudaSuccess) return bail(cuda_fail(e, "repack launch"));
    } else {
        // Host source: stage up to ~256 MB of rows at a time.
        int64_t rows_per = (int64_t)((256u << 20) / slice_bytes);
        if (rows_per < 1) rows_per = 1;
        if (rows_per > N) rows_per = N;
        uint8_t* stage = nullptr;
        if ((e = cudaMalloc(&stage, (size_t)rows_per * slice_bytes)) != cudaSuccess)
            return bail(cuda_fail(e, "cudaMalloc (staging)"));
        for (int64_t r0 = 0; r0 < N && e == cudaSuccess; r0 += rows_per) {
            int64_t nr = N - r0 < rows_per ? N - r0 : rows_per;
            const uint8_t* hsrc = (const uint8_t*)src + (size_t)r0 * src_pitch + (size_t)blk0 * s.g.bb;
            e = cudaMemcpy2DAsync(stage, slice_bytes, hsrc, src_pitch, slice_bytes, (size_t)nr,
                                  cudaMemcpyHostToDevice, st);
            if (e == cudaSuccess)
                e = launch_repack(stage, w->dev, s, r0, nr, 0, K / s.g.qk, st);
            // The staging buffer is reused: finish this pass before the next copy.
            if (e == cudaSuccess) e = cudaStreamSynchronize(st);
        }
        cudaFree(stage);
        if (e != cudaSuccess) return bail(cuda_fail(e, "weight upload/repack"));
    }
    if ((e = cudaStreamSynchronize(st)) != cudaSuccess) return bail(cuda_fail(e, "weight registration"));
    {
        std::lock_guard<std::mutex> lk(g_ctx.mu);
        g_ctx.live.insert(w);
    }
    *out = reinterpret_cast<nxq_weight_t>(w);
    return NXQ_OK;
}

}  // namespace

int fail(int status, const char* fmt, ...) {
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(g_err, sizeof g_err, fmt, ap);
    va_end(ap);
    return status;
}

int cuda_fail(cudaError_t e, const char* what) {
    return fail(NXQ_ERR_CUDA, "%s: %s (%s)", what, cudaGetErrorName(e), cudaGetErrorString(e));
}

namespace {
std::atomic<uint64_t> g_launches{0};
}

void note_launches(unsigned n) { g_launches.fetch_add(n, std::memory_order_relaxed); }

const char* type_name(int type) {
    switch (type) {
        case T_Q4_0: return "Q4_0";
        case T_Q4_1: return "Q4_1";
        case T_Q8_0: return "Q8_0";
        case T_Q2_K: return "Q2_K";
        case T_Q3_K: return "Q3_K";
        case T_Q4_K: return "Q4_K";
        case T_Q5_K: return "Q5_K";
        case T_Q6_K: return "Q6_K";
        case T_I4G32: return "I4G32";
        case T_I4G64: return "I4G64";
        case T_I4G128: return "I4G128";
        case T_I4G256: return "I4G256";
        case T_NXF_I8: return "NXF_I8";
        case T_NXF_F16: return "NXF_F16";
        case T_NXF_F32: return "NXF_F32";
        default: return "?";
    }
}

int context_sm_count() { return g_ctx.sm_count; }
DeviceStatus* context_status() { return g_ctx.status; }
int context_ready() { return check_ready(); }

// Runs y = x W^T on `st` through the best kernel for (type, M, dtypes).
int qmatmul_dispatch(const Weight* w, const void* x, int x_dtype, void* y, int y_dtype, int64_t M,
                     cudaStream_t st) {
    const TiledShape& s = w->shape;
    if (M == 0) return NXQ_OK;
    if (mma_supported(s, M)) {
        int rc = mma_qmatmul(w, x, x_dtype, y, y_dtype, M, st);
        if (rc != NXQ_ERR_UNSUPPORTED) return rc;
    }
    if (gemm_supported(s, M)) {
        int rc = gemm_qmatmul(w, x, x_dtype, y, y_dtype, M, st);
        if (rc != NXQ_ERR_UNSUPPORTED) return rc;
    }
    int splits = simt_pick_splits(s, M, g_ctx.sm_count);
    float* partials = nullptr;
    cudaError_t e;
    if (splits > 1) {
        e = cudaMallocAsync((void**)&partials, (size_t)splits * M * s.N * sizeof(float), st);
        if (e != cudaSuccess) return cuda_fail(e, "cudaMallocAsync (split partials)");
    }
    e = launch_qmm_simt(w->dev, s, x, x_dtype, y, y_dtype, M, partials, splits, st);
    if (partials) cudaFreeAsync(partials, st);
    if (e != cudaSuccess) return cuda_fail(e, "qmm_simt launch");
    return NXQ_OK;
}

}  // namespace nxq

using namespace nxq;

extern "C" {

NXQ_API int nxq_abi_version(void) { return NXQ_ABI_VERSION; }

NXQ_API int nxq_last_error(char* buf, size_t n) {
    if (!buf || n == 0) return NXQ_ERR_ARG;
    snprintf(buf, n, "%s", g_err);
    return NXQ_OK;
}

NXQ_API int nxq_block_geometry(int type, int* block_elems, int* block_bytes) {
    Geometry g;
    if (!geometry_of(type, &g)) return fail(NXQ_ERR_CODEC, "unsupported block type %d", type);
    if (block_elems) *block_elems = g.qk;
    if (block_bytes) *block_bytes = g.bb;
    return NXQ_OK;
}

NXQ_API int nxq_init(int device) {
    std::lock_guard<std::mutex> lk(g_init_mu);
    if (g_ctx.ready) {
        if (device == g_ctx.device) return NXQ_OK;
        return fail(NXQ_ERR_STATE, "nxq already initialised on device %d", g_ctx.device);
    }
    int count = 0;
    cudaError_t e = cudaGetDeviceCount(&count);
    if (e != cudaSuccess || count == 0)
        return fail(NXQ_ERR_UNSUPPORTED, "no CUDA device available (%s)",
                    e == cudaSuccess ? "0 devices" : cudaGetErrorString(e));
    if (device < 0 || device >= count) return fail(NXQ_ERR_ARG, "device %d out of range", device);
    NXQ_CUDA(cudaSetDevice(device));
    cudaDeviceProp p;
    NXQ_CUDA(cudaGetDeviceProperties(&p, device));
    if (p.major != 10)
        return fail(NXQ_ERR_UNSUPPORTED, "device %d is sm_%d%d; libnxq is built for sm_100a only",
                    device, p.major, p.minor);
    g_ctx.device = device;
    g_ctx.sm_count = p.multiProcessorCount;
    g_ctx.cc_major = p.major;
    g_ctx.cc_minor = p.minor;
    g_ctx.smem_optin = p.sharedMemPerBlockOptin;
    NXQ_CUDA(cudaStreamCreateWithFlags(&g_ctx.host_stream, cudaStreamNonBlocking));
    NXQ_CUDA(cudaMalloc(&g_ctx.status, sizeof(DeviceStatus)));
    NXQ_CUDA(cudaHostAlloc(&g_ctx.flag_host, sizeof(unsigned int), cudaHostAllocMapped));
    *g_ctx.flag_host = 0u;
    {
        DeviceStatus init{};
        init.wait_cycles = kDefaultWaitCycles;
        NXQ_CUDA(cudaHostGetDevicePointer((void**)&init.host_flag, g_ctx.flag_host, 0));
        NXQ_CUDA(cudaMemcpy(g_ctx.status, &init, sizeof init, cudaMemcpyHostToDevice));
    }
    ++g_ctx.generation;
    // Keep stream-ordered scratch in the pool between calls instead of
    // returning it to the driver after every synchronize.
    cudaMemPool_t pool;
    if (cudaDeviceGetDefaultMemPool(&pool, device) == cudaSuccess) {
        uint64_t keep = 1ull << 30;
        cudaMemPoolSetAttribute(pool, cudaMemPoolAttrReleaseThreshold, &keep);
    }
    int rc = mma_init(device);
    if (rc != NXQ_OK) return rc;
    if ((rc = gemm_init(device)) != NXQ_OK) return rc;
    g_ctx.ready = true;
    return NXQ_OK;
}

NXQ_API int nxq_shutdown(void) {
    std::lock_guard<std::mutex> lk(g_init_mu);
    if (!g_ctx.ready) return NXQ_OK;
    cudaSetDevice(g_ctx.device);
    cudaDeviceSynchronize();
    {
        std::lock_guard<std::mutex> lk2(g_ctx.mu);
        for (Weight* w : g_ctx.live) {
            w->magic = 0;
            cudaFree(w->dev);
            delete w;
        }
        g_ctx.live.clear();
    }
    {
        std::lock_guard<std::mutex> lk2(g_hostcall_mu);
        for (HostCall* hc : g_hostcalls) {
            if (hc->dx) cudaFree(hc->dx);
            if (hc->dy) cudaFree(hc->dy);
            if (hc->st) cudaStreamDestroy(hc->st);
            if (hc->done) cudaEventDestroy(hc->done);
            hc->dx = hc->dy = nullptr;
            hc->st = nullptr;
            hc->done = nullptr;
            hc->generation = 0;  // the owning thread makes a new one on its next call
        }
        g_hostcalls.clear();  // the structs themselves stay with their threads' pointers
    }
    if (g_ctx.status) cudaFree(g_ctx.status);
    g_ctx.status = nullptr;
    if (g_ctx.flag_host) cudaFreeHost(g_ctx.flag_host);
    g_ctx.flag_host = nullptr;
    if (g_ctx.host_stream) cudaStreamDestroy(g_ctx.host_stream);
    g_ctx.host_stream = nullptr;
    g_ctx.ready = false;
    g_ctx.device = -1;
    return NXQ_OK;
}

NXQ_API int nxq_weight_register(const void* host_blocks, size_t bytes, int type, int64_t N,
                                int64_t K, nxq_weight_t* out) {
    if (!host_blocks || !out) return fail(NXQ_ERR_ARG, "null argument");
    int rc = check_ready();
    if (rc) return rc;
    Geometry g;
    if (!geometry_of(type, &g)) return fail(NXQ_ERR_CODEC, "unsupported block type %d", type);
    if (N <= 0 || K <= 0 || K % g.qk)
        return fail(NXQ_ERR_SHAPE, "bad shape N=%lld K=%lld (K must be a positive multiple of %d)",
                    (long long)N, (long long)K, g.qk);
    if (bytes != (size_t)N * (size_t)(K / g.qk) * (size_t)g.bb)
        return fail(NXQ_ERR_SHAPE, "bytes=%zu but N*(K/%d)*%d = %zu", bytes, g.qk, g.bb,
                    (size_t)N * (size_t)(K / g.qk) * (size_t)g.bb);
    std::lock_guard<std::mutex> lk(g_init_mu);
    return register_impl(host_blocks, true, type, N, K, K / g.qk, 0, g_ctx.host_stream, out);
}

NXQ_API int nxq_weight_register_device(const void* dev_blocks, size_t bytes, int type, int64_t N,
                                       int64_t K, void* stream, nxq_weight_t* out) {
    if (!dev_blocks || !out) return fail(NXQ_ERR_ARG, "null argument");
    int rc = check_ready();
    if (rc) return rc;
    Geometry g;
    if (!geometry_of(type, &g)) return fail(NXQ_ERR_CODEC, "unsupported block type %d", type);
    if (N <= 0 || K <= 0 || K % g.qk)
        return fail(NXQ_ERR_SHAPE, "bad shape N=%lld K=%lld", (long long)N, (long long)K);
    if (bytes != (size_t)N * (size_t)(K / g.qk) * (size_t)g.bb)
        return fail(NXQ_ERR_SHAPE, "bytes=%zu does not match N*(K/QK)*block_bytes", bytes);
    std::lock_guard<std::mutex> lk(g_init_mu);
    return register_impl(dev_blocks, false, type, N, K, K / g.qk, 0, (cudaStream_t)stream, out);
}

// Validates a TP shard request; fills the slice geometry.
static int shard_geometry(size_t bytes, int type, int64_t N, int64_t K, int split, int rank,
                          int world, Geometry* g, int64_t* n_loc, int64_t* k_loc) {
    if (!geometry_of(type, g)) return fail(NXQ_ERR_CODEC, "unsupported block type %d", type);
    if (world < 1 || rank < 0 || rank >= world) return fail(NXQ_ERR_ARG, "rank %d of %d", rank, world);
    if (N <= 0 || K <= 0 || K % g->qk) return fail(NXQ_ERR_SHAPE, "bad shape");
    if (bytes != (size_t)N * (size_t)(K / g->qk) * (size_t)g->bb)
        return fail(NXQ_ERR_SHAPE, "bytes does not match N*(K/QK)*block_bytes");
    if (split == NXQ_SPLIT_COL) {
        if (N % world) return fail(NXQ_ERR_SHAPE, "N=%lld not divisible by %d", (long long)N, world);
        *n_loc = N / world;
        *k_loc = K;
        return NXQ_OK;
    }
    if (split == NXQ_SPLIT_ROW) {
        if (K % world || (K / world) % g->qk)
            return fail(NXQ_ERR_SHAPE, "K=%lld / %d is not a multiple of the %d-element block",
                        (long long)K, world, g->qk);
        *n_loc = N;
        *k_loc = K / world;
        return NXQ_OK;
    }
    return fail(NXQ_ERR_ARG, "split must be NXQ_SPLIT_COL or NXQ_SPLIT_ROW");
}

NXQ_API int nxq_shard_extract(const void* host_blocks, size_t bytes, int type, int64_t N,
                              int64_t K, int split, int rank, int world, void* out,
                              size_t out_bytes) {
    if (!host_blocks || !out) return fail(NXQ_ERR_ARG, "null argument");
    Geometry g;
    int64_t n_loc = 0, k_loc = 0;
    int rc = shard_geometry(bytes, type, N, K, split, rank, world, &g, &n_loc, &k_loc);
    if (rc) return rc;
    const size_t row_bytes = (size_t)(K / g.qk) * g.bb;
    const size_t slice = (size_t)(k_loc / g.qk) * g.bb;
    if (out_bytes != (size_t)n_loc * slice)
        return fail(NXQ_ERR_SHAPE, "out_bytes=%zu, shard needs %zu", out_bytes, (size_t)n_loc * slice);
    const uint8_t* src = (const uint8_t*)host_blocks;
    uint8_t* dst = (uint8_t*)out;
    if (split == NXQ_SPLIT_COL) {
        memcpy(dst, src + (size_t)rank * n_loc * row_bytes, (size_t)n_loc * row_bytes);
    } else {
        for (int64_t n = 0; n < N; ++n)
            memcpy(dst + (size_t)n * slice, src + (size_t)n * row_bytes + (size_t)rank * slice, slice);
    }
    return NXQ_OK;
}

NXQ_API int nxq_weight_register_shard(const void* host_blocks, size_t bytes, int type, int64_t N,
                                      int64_t K, int split, int rank, int world,
                                      nxq_weight_t* out) {
    if (!host_blocks || !out) return fail(NXQ_ERR_ARG, "null argument");
    int rc = check_ready();
    if (rc) return rc;
    Geometry g;
    int64_t n_loc = 0, k_loc = 0;
    if ((rc = shard_geometry(bytes, type, N, K, split, rank, world, &g, &n_loc, &k_loc))) return rc;
    const int64_t row_blocks = K / g.qk;
    std::lock_guard<std::mutex> lk(g_init_mu);
    if (split == NXQ_SPLIT_COL) {
        const uint8_t* src = (const uint8_t*)host_blocks + (size_t)rank * n_loc * row_blocks * g.bb;
        return register_impl(src, true, type, n_loc, K, row_blocks, 0, g_ctx.host_stream, out);
    }
    return register_impl(host_blocks, true, type, N, k_loc, row_blocks, rank * (k_loc / g.qk),
                         g_ctx.host_stream, out);
}

NXQ_API int nxq_weight_release(nxq_weight_t h) {
    Weight* w = nullptr;
    int rc = check_weight(h, &w);
    if (rc) return rc;
    rc = check_ready();
    if (rc) return rc;
    std::lock_guard<std::mutex> lk(g_ctx.mu);
    g_ctx.live.erase(w);
    w->magic = 0;
    // Work queued on other streams may still read the weight.
    cudaDeviceSynchronize();
    cudaFree(w->dev);
    delete w;
    return NXQ_OK;
}

NXQ_API int nxq_weight_info(nxq_weight_t h, int* type, int64_t* N, int64_t* K, size_t* packed_bytes,
                            size_t* device_bytes) {
    Weight* w = nullptr;
    int rc = check_weight(h, &w);
    if (rc) return rc;
    if (type) *type = w->shape.type;
    if (N) *N = w->shape.N;
    if (K) *K = w->shape.K;
    if (packed_bytes) *packed_bytes = w->packed_bytes;
    if (device_bytes) *device_bytes = w->dev_bytes;
    return NXQ_OK;
}

NXQ_API int nxq_dequant(nxq_weight_t h, float* y_dev, void* stream) {
    Weight* w = nullptr;
    int rc = check_weight(h, &w);
    if (rc) return rc;
    if (!y_dev) return fail(NXQ_ERR_ARG, "null output");
    if ((uintptr_t)y_dev % 16) return fail(NXQ_ERR_ARG, "output must be 16-byte aligned");
    if ((rc = check_ready())) return rc;
    cudaError_t e = launch_dequant(w->dev, w->shape, y_dev, (cudaStream_t)stream);
    if (e != cudaSuccess) return cuda_fail(e, "dequant launch");
    return NXQ_OK;
}

NXQ_API int nxq_qmatmul(nxq_weight_t h, const void* x_dev, int x_dtype, void* y_dev, int y_dtype,
                        int64_t M, void* stream) {
    Weight* w = nullptr;
    int rc = check_weight(h, &w);
    if (rc) return rc;
    if (M < 0) return fail(NXQ_ERR_ARG, "M=%lld", (long long)M);
    if (M > 0 && (!x_dev || !y_dev)) return fail(NXQ_ERR_ARG, "null activation or output");
    if (!dtype_ok(x_dtype) || !dtype_ok(y_dtype)) return fail(NXQ_ERR_ARG, "bad dtype");
    if ((rc = check_ready())) return rc;
    return qmatmul_dispatch(w, x_dev, x_dtype, y_dev, y_dtype, M, (cudaStream_t)stream);
}

NXQ_API int nxq_qmatmul_grouped(const nxq_weight_t* hs, int count, const void* const* x_dev, int x_dtype,
                                void* const* y_dev, int y_dtype, const int64_t* M, void* stream) {
    if (count < 0 || (count > 0 && (!hs || !x_dev || !y_dev || !M))) return fail(NXQ_ERR_ARG, "grouped: bad arrays");
    if (!dtype_ok(x_dtype) || !dtype_ok(y_dtype)) return fail(NXQ_ERR_ARG, "bad dtype");
    std::vector<Weight*> ws((size_t)count);
    for (int i = 0; i < count; ++i) {
        if (int rc = check_weight(hs[i], &ws[i])) return rc;
        if (M[i] < 0) return fail(NXQ_ERR_ARG, "grouped: M[%d]=%lld", i, (long long)M[i]);
        if (M[i] > 0 && (!x_dev[i] || !y_dev[i])) return fail(NXQ_ERR_ARG, "grouped: null activation or output %d", i);
    }
    if (int rc = check_ready()) return rc;
    cudaStream_t st = (cudaStream_t)stream;
    int rc = mma_qmatmul_grouped(ws.data(), count, x_dev, x_dtype, y_dev, y_dtype, M, st);
    if (rc != NXQ_ERR_UNSUPPORTED) return rc;
    // Mixed block types, prefill batch sizes or activations that need a
    // conversion pass: the items one after another on the same stream.
    for (int i = 0; i < count; ++i)
        if ((rc = qmatmul_dispatch(ws[i], x_dev[i], x_dtype, y_dev[i], y_dtype, M[i], st))) return rc;
    return NXQ_OK;
}

NXQ_API int nxq_qmatmul_swiglu(nxq_weight_t hg, nxq_weight_t hu, const void* x_dev, int x_dtype, void* h_dev,
                               int h_dtype, int64_t M, void* stream) {
    Weight *wg = nullptr, *wu = nullptr;
    int rc = check_weight(hg, &wg);
    if (rc || (rc = check_weight(hu, &wu))) return rc;
    if (wg->shape.N != wu->shape.N || wg->shape.K != wu->shape.K)
        return fail(NXQ_ERR_SHAPE, "swiglu: gate [%lld][%lld] and up [%lld][%lld] differ", (long long)wg->shape.N,
                    (long long)wg->shape.K, (long long)wu->shape.N, (long long)wu->shape.K);
    if (M < 0) return fail(NXQ_ERR_ARG, "M=%lld", (long long)M);
    if (M == 0) return NXQ_OK;
    if (!x_dev || !h_dev) return fail(NXQ_ERR_ARG, "null activation or output");
    if (!dtype_ok(x_dtype) || !dtype_ok(h_dtype)) return fail(NXQ_ERR_ARG, "bad dtype");
    if ((rc = check_ready())) return rc;
    cudaStream_t st = (cudaStream_t)stream;
    rc = mma_qmatmul_swiglu(wg, wu, x_dev, x_dtype, h_dev, h_dtype, M, st);
    if (rc != NXQ_ERR_UNSUPPORTED) return rc;
    // Gate and up into fp32 intermediates (one grouped launch where it can
    // be), then h = silu(g) * u.
    const int64_t mn = M * wg->shape.N;
    StreamScratch* sc = nullptr;
    if ((rc = scratch_for(st, 0, 0, 0, &sc, (size_t)(2 * mn)))) return rc;
    float* gu[2] = {sc->epi, sc->epi + mn};
    const Weight* ws[2] = {wg, wu};
    const void* xs[2] = {x_dev, x_dev};
    const int64_t Ms[2] = {M, M};
    rc = mma_qmatmul_grouped(ws, 2, xs, x_dtype, reinterpret_cast<void* const*>(gu), NXQ_F32, Ms, st);
    if (rc == NXQ_ERR_UNSUPPORTED) {
        if ((rc = qmatmul_dispatch(wg, x_dev, x_dtype, gu[0], NXQ_F32, M, st))) return rc;
        rc = qmatmul_dispatch(wu, x_dev, x_dtype, gu[1], NXQ_F32, M, st);
    }
    if (rc) return rc;
    cudaError_t e = launch_swiglu(gu[0], gu[1], h_dev, h_dtype, mn, st);
    return e == cudaSuccess ? NXQ_OK : cuda_fail(e, "swiglu launch");
}

NXQ_API int nxq_rmsnorm_qmatmul(const nxq_weight_t* hs, int count, const void* x_dev, int x_dtype,
                                const float* norm_dev, float eps, void* const* y_dev, int y_dtype, int64_t M,
                                void* stream) {
    if (count < 1 || !hs || !y_dev) return fail(NXQ_ERR_ARG, "rmsnorm_qmatmul: bad arrays");
    if (M < 0 || !(eps >= 0.0f)) return fail(NXQ_ERR_ARG, "rmsnorm_qmatmul: M=%lld eps=%g", (long long)M, (double)eps);
    if (!dtype_ok(x_dtype) || !dtype_ok(y_dtype)) return fail(NXQ_ERR_ARG, "bad dtype");
    std::vector<Weight*> ws((size_t)count);
    for (int i = 0; i < count; ++i) {
        if (int rc = check_weight(hs[i], &ws[i])) return rc;
        if (ws[i]->shape.K != ws[0]->shape.K)
            return fail(NXQ_ERR_SHAPE, "rmsnorm_qmatmul: weight %d has K=%lld, weight 0 K=%lld", i,
                        (long long)ws[i]->shape.K, (long long)ws[0]->shape.K);
        if (M > 0 && !y_dev[i]) return fail(NXQ_ERR_ARG, "rmsnorm_qmatmul: null output %d", i);
    }
    if (M == 0) return NXQ_OK;
    if (!x_dev || !norm_dev) return fail(NXQ_ERR_ARG, "rmsnorm_qmatmul: null activation or norm weight");
    if (int rc = check_ready()) return rc;
    cudaStream_t st = (cudaStream_t)stream;
    const int64_t K = ws[0]->shape.K;
    StreamScratch* sc = nullptr;
    int rc = scratch_for(st, 0, 0, (size_t)(M * K), &sc);
    if (rc) return rc;
    cudaError_t e = launch_rmsnorm_to_half(x_dev, x_dtype, norm_dev, eps, sc->xh, M, K, st);
    if (e != cudaSuccess) return cuda_fail(e, "rmsnorm launch");
    std::vector<const void*> xs((size_t)count, sc->xh);
    std::vector<int64_t> Ms((size_t)count, M);
    rc = mma_qmatmul_grouped(ws.data(), count, xs.data(), NXQ_F16, y_dev, y_dtype, Ms.data(), st);
    if (rc != NXQ_ERR_UNSUPPORTED) return rc;
    for (int i = 0; i < count; ++i)
        if ((rc = qmatmul_dispatch(ws[i], sc->xh, NXQ_F16, y_dev[i], y_dtype, M, st))) return rc;
    return NXQ_OK;
}

NXQ_API int nxq_qmatmul_residual(nxq_weight_t h, const void* x_dev, int x_dtype, const float* res_dev, void* y_dev,
                                 int y_dtype, int64_t M, void* stream) {
    Weight* w = nullptr;
    int rc = check_weight(h, &w);
    if (rc) return rc;
    if (M < 0) return fail(NXQ_ERR_ARG, "M=%lld", (long long)M);
    if (M == 0) return NXQ_OK;
    if (!x_dev || !y_dev || !res_dev) return fail(NXQ_ERR_ARG, "null activation, residual or output");
    if (!dtype_ok(x_dtype) || !dtype_ok(y_dtype)) return fail(NXQ_ERR_ARG, "bad dtype");
    if ((rc = check_ready())) return rc;
    cudaStream_t st = (cudaStream_t)stream;
    if (mma_supported(w->shape, M)) {
        rc = mma_qmatmul(w, x_dev, x_dtype, y_dev, y_dtype, M, st, res_dev);
        if (rc != NXQ_ERR_UNSUPPORTED) return rc;
    }
    // Other kernels: the product into an fp32 intermediate, then y = it + res
    // (y may be the residual buffer itself).
    const int64_t mn = M * w->shape.N;
    StreamScratch* sc = nullptr;
    if ((rc = scratch_for(st, 0, 0, 0, &sc, (size_t)mn))) return rc;
    if ((rc = qmatmul_dispatch(w, x_dev, x_dtype, sc->epi, NXQ_F32, M, st))) return rc;
    cudaError_t e = launch_add_residual(sc->epi, res_dev, y_dev, y_dtype, mn, st);
    return e == cudaSuccess ? NXQ_OK : cuda_fail(e, "residual add launch");
}

NXQ_API int nxq_qmatmul_noalloc(nxq_weight_t h, const void* x_dev, int x_dtype, void* y_dev, int y_dtype,
                                int64_t M, void* stream) {
    Weight* w = nullptr;
    int rc = check_weight(h, &w);
    if (rc) return rc;
    if (M < 0) return fail(NXQ_ERR_ARG, "M=%lld", (long long)M);
    if (M == 0) return NXQ_OK;
    if (!x_dev || !y_dev) return fail(NXQ_ERR_ARG, "null activation or output");
    if (!dtype_ok(x_dtype) || !dtype_ok(y_dtype)) return fail(NXQ_ERR_ARG, "bad dtype");
    if ((rc = check_ready())) return rc;
    return launch_qmm_simt_noalloc(w->dev, w->shape, x_dev, x_dtype, y_dev, y_dtype, M, g_ctx.sm_count,
                                   (cudaStream_t)stream);
}

NXQ_API int nxq_qmatmul_host(nxq_weight_t h, const float* x_host, float* y_host, int64_t M) {
    Weight* w = nullptr;
    int rc = check_weight(h, &w);
    if (rc) return rc;
    if (M < 0) return fail(NXQ_ERR_ARG, "M=%lld", (long long)M);
    if (M == 0) return NXQ_OK;
    if (!x_host || !y_host) return fail(NXQ_ERR_ARG, "null activation or output");
    if ((rc = check_ready())) return rc;
    HostCall* hc = nullptr;
    if ((rc = host_call_context(&hc))) return rc;
    const size_t xb = (size_t)M * w->shape.K * sizeof(float);
    const size_t yb = (size_t)M * w->shape.N * sizeof(float);
    if ((rc = grow(&hc->dx, &hc->dx_bytes, xb))) return rc;
    if ((rc = grow(&hc->dy, &hc->dy_bytes, yb))) return rc;
    cudaStream_t st = hc->st;
    NXQ_CUDA(cudaMemcpyAsync(hc->dx, x_host, xb, cudaMemcpyHostToDevice, st));
    rc = qmatmul_dispatch(w, hc->dx, NXQ_F32, hc->dy, NXQ_F32, M, st);
    if (rc) return rc;
    NXQ_CUDA(cudaMemcpyAsync(y_host, hc->dy, yb, cudaMemcpyDeviceToHost, st));
    NXQ_CUDA(cudaEventRecord(hc->done, st));
    NXQ_CUDA(wait_spinning(hc->done));
    // A kernel that raised an error also set the mapped host flag: no device
    // read on the normal path.
    return check_host_flag();
}

NXQ_API int nxq_qmatmul_kernel_name(nxq_weight_t h, int64_t M, int x_dtype, int y_dtype, char* buf,
                                    size_t n) {
    Weight* w = nullptr;
    int rc = check_weight(h, &w);
    if (rc) return rc;
    if (!buf || n == 0) return fail(NXQ_ERR_ARG, "null buffer");
    if (M < 1 || !dtype_ok(x_dtype) || !dtype_ok(y_dtype)) return fail(NXQ_ERR_ARG, "bad M or dtype");
    if (mma_supported(w->shape, M)) {
        mma_kernel_name(w->shape, M, buf, n);
        return NXQ_OK;
    }
    if (gemm_supported(w->shape, M)) {
        gemm_kernel_name(w->shape, M, buf, n);
        return NXQ_OK;
    }
    snprintf(buf, n, "simt<%s,mb%d>", type_name(w->shape.type), simt_rows_per_pass(M));
    return NXQ_OK;
}

NXQ_API int nxq_launch_count(uint64_t* out) {
    if (!out) return fail(NXQ_ERR_ARG, "null argument");
    *out = g_launches.load(std::memory_order_relaxed);
    return NXQ_OK;
}

NXQ_API int nxq_set_wait_limit(uint64_t microseconds) {
    int rc = check_ready();
    if (rc) return rc;
    if (microseconds > 60ull * 1000 * 1000) return fail(NXQ_ERR_ARG, "wait limit above 60 s");
    // Converted at 2 cycles per ns (the SM clock is at most 1965 MHz, so the
    // wait lasts at least this long).
    const long long cycles = microseconds ? (long long)microseconds * 2000 : kDefaultWaitCycles;
    cudaDeviceSynchronize();
    NXQ_CUDA(cudaMemcpy(reinterpret_cast<char*>(g_ctx.status) + offsetof(DeviceStatus, wait_cycles), &cycles,
                        sizeof cycles, cudaMemcpyHostToDevice));
    return NXQ_OK;
}

NXQ_API int nxq_test_hook(int hook, int on) {
    int rc = check_ready();
    if (rc) return rc;
    unsigned bit = 0;
    switch (hook) {
        case NXQ_HOOK_STREAMK_SKIP_COUNT: bit = kHookStreamKSkipCount; break;
        default: return fail(NXQ_ERR_ARG, "unknown test hook %d", hook);
    }
    cudaDeviceSynchronize();
    unsigned hooks = 0;
    char* at = reinterpret_cast<char*>(g_ctx.status) + offsetof(DeviceStatus, hooks);
    NXQ_CUDA(cudaMemcpy(&hooks, at, sizeof hooks, cudaMemcpyDeviceToHost));
    hooks = on ? (hooks | bit) : (hooks & ~bit);
    NXQ_CUDA(cudaMemcpy(at, &hooks, sizeof hooks, cudaMemcpyHostToDevice));
    return NXQ_OK;
}

NXQ_API int nxq_stream_sync(void* stream) {
    int rc = check_ready();
    if (rc) return rc;
    NXQ_CUDA(cudaStreamSynchronize((cudaStream_t)stream));
    return check_host_flag();
}

}  // extern "C"
