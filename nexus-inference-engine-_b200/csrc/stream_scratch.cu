// Per-stream scratch shared by the matmul kernels (stream_scratch.h).
#include "stream_scratch.h"

#include <cuda_bf16.h>

#include <list>
#include <mutex>

namespace nxq {

namespace {

// Rounds fp32 / bf16 activations to f16; a finite value beyond the f16
// range is reported in the status word (kStatusRange, where = 1).
__global__ void to_half_kernel(const void* __restrict__ x, int dt, __half* __restrict__ out, int64_t n,
                               DeviceStatus* status) {
    bool over = false;
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x) {
        float v;
        if (dt == NXQ_F32)
            v = reinterpret_cast<const float*>(x)[i];
        else if (dt == NXQ_BF16)
            v = __bfloat162float(reinterpret_cast<const __nv_bfloat16*>(x)[i]);
        else
            v = __half2float(reinterpret_cast<const __half*>(x)[i]);
        over |= f16_overflows(v);
        out[i] = __float2half_rn(v);
    }
    if (over) raise_range(status, 1u);
}

std::mutex g_scratch_mu;
// Entries are never moved, so pointers handed out stay valid.
std::list<StreamScratch> g_scratch;

}  // namespace

int scratch_for(cudaStream_t st, size_t ws_floats, size_t n_counters, size_t xh_elems, StreamScratch** out,
                size_t epi_floats) {
    std::lock_guard<std::mutex> lk(g_scratch_mu);
    StreamScratch* sc = nullptr;
    for (auto& e : g_scratch)
        if (e.st == st) sc = &e;
    if (!sc) {
        g_scratch.push_back(StreamScratch{});
        sc = &g_scratch.back();
        sc->st = st;
    }
    const bool grow = sc->ws_floats < ws_floats || sc->n_counters < n_counters || sc->xh_elems < xh_elems ||
                      sc->epi_floats < epi_floats;
    if (grow) {
        cudaStreamCaptureStatus cs = cudaStreamCaptureStatusNone;
        if (cudaStreamIsCapturing(st, &cs) == cudaSuccess && cs != cudaStreamCaptureStatusNone)
            return fail(NXQ_ERR_STATE,
                        "scratch for this stream must grow, which cannot happen during graph capture: "
                        "run the largest call once on this stream before capturing");
        // The old buffers may still be in use by work queued on this stream.
        cudaError_t e = cudaStreamSynchronize(st);
        if (e != cudaSuccess) return cuda_fail(e, "scratch grow sync");
        if (sc->ws_floats < ws_floats) {
            cudaFree(sc->ws);
            sc->ws = nullptr;
            sc->ws_floats = 0;
            if ((e = cudaMalloc(&sc->ws, ws_floats * sizeof(float))) != cudaSuccess)
                return cuda_fail(e, "cudaMalloc (split-K workspace)");
            sc->ws_floats = ws_floats;
        }
        if (sc->n_counters < n_counters) {
            cudaFree(sc->counters);
            sc->counters = nullptr;
            sc->n_counters = 0;
            if ((e = cudaMalloc(&sc->counters, n_counters * sizeof(unsigned))) != cudaSuccess)
                return cuda_fail(e, "cudaMalloc (tile counters)");
            if ((e = cudaMemset(sc->counters, 0, n_counters * sizeof(unsigned))) != cudaSuccess)
                return cuda_fail(e, "cudaMemset (tile counters)");
            sc->n_counters = n_counters;
        }
        if (sc->xh_elems < xh_elems) {
            cudaFree(sc->xh);
            sc->xh = nullptr;
            sc->xh_elems = 0;
            if ((e = cudaMalloc(&sc->xh, xh_elems * sizeof(__half))) != cudaSuccess)
                return cuda_fail(e, "cudaMalloc (f16 activations)");
            sc->xh_elems = xh_elems;
        }
        if (sc->epi_floats < epi_floats) {
            cudaFree(sc->epi);
            sc->epi = nullptr;
            sc->epi_floats = 0;
            if ((e = cudaMalloc(&sc->epi, epi_floats * sizeof(float))) != cudaSuccess)
                return cuda_fail(e, "cudaMalloc (epilogue intermediates)");
            sc->epi_floats = epi_floats;
        }
    }
    *out = sc;
    return NXQ_OK;
}

void scratch_reset_counters() {
    std::lock_guard<std::mutex> lk(g_scratch_mu);
    for (auto& e : g_scratch)
        if (e.counters) cudaMemset(e.counters, 0, e.n_counters * sizeof(unsigned));
    cudaDeviceSynchronize();
}

int scratch_try(cudaStream_t st, size_t ws_floats, size_t n_counters, StreamScratch** out) {
    *out = nullptr;
    {
        std::lock_guard<std::mutex> lk(g_scratch_mu);
        for (auto& e : g_scratch)
            if (e.st == st && e.ws_floats >= ws_floats && e.n_counters >= n_counters) {
                *out = &e;
                return NXQ_OK;
            }
    }
    cudaStreamCaptureStatus cs = cudaStreamCaptureStatusNone;
    if (cudaStreamIsCapturing(st, &cs) == cudaSuccess && cs != cudaStreamCaptureStatusNone) return NXQ_OK;
    return scratch_for(st, ws_floats, n_counters, 0, out);
}

namespace {

__device__ __forceinline__ void store_as(void* p, int dt, int64_t i, float v) {
    if (dt == NXQ_F32)
        reinterpret_cast<float*>(p)[i] = v;
    else if (dt == NXQ_F16)
        reinterpret_cast<__half*>(p)[i] = __float2half_rn(v);
    else
        reinterpret_cast<__nv_bfloat16*>(p)[i] = __float2bfloat16_rn(v);
}

__global__ void swiglu_kernel(const float* __restrict__ g, const float* __restrict__ u, void* __restrict__ h, int dt,
                              int64_t n) {
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x) {
        const float a = g[i];
        store_as(h, dt, i, a / (1.0f + expf(-a)) * u[i]);
    }
}

__global__ void add_residual_kernel(const float* __restrict__ a, const float* res, void* y, int dt, int64_t n) {
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x)
        store_as(y, dt, i, a[i] + res[i]);
}

__device__ __forceinline__ float load_as(const void* p, int dt, int64_t i) {
    if (dt == NXQ_F32) return reinterpret_cast<const float*>(p)[i];
    if (dt == NXQ_F16) return __half2float(reinterpret_cast<const __half*>(p)[i]);
    return __bfloat162float(reinterpret_cast<const __nv_bfloat16*>(p)[i]);
}

constexpr int kNormThreads = 512;

// One CTA per row: sum of squares (per-thread partials, then warps, then the
// CTA), r = rsqrtf(sum / K + eps), then the scaled row.
__global__ void __launch_bounds__(kNormThreads) rmsnorm_to_half_kernel(const void* __restrict__ x, int dt,
                                                                     const float* __restrict__ w, float eps,
                                                                     __half* __restrict__ out, int64_t K,
                                                                     DeviceStatus* status) {
    __shared__ float part[kNormThreads / 32];
    __shared__ float r_s;
    const int64_t row = blockIdx.x;
    float ss = 0.0f;
    for (int64_t i = threadIdx.x; i < K; i += kNormThreads) {
        const float v = load_as(x, dt, row * K + i);
        ss = fmaf(v, v, ss);
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xFFFFFFFFu, ss, o);
    if ((threadIdx.x & 31) == 0) part[threadIdx.x >> 5] = ss;
    __syncthreads();
    if (threadIdx.x < 32) {
        float t = threadIdx.x < kNormThreads / 32 ? part[threadIdx.x] : 0.0f;
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) t += __shfl_xor_sync(0xFFFFFFFFu, t, o);
        if (threadIdx.x == 0) r_s = rsqrtf(t / (float)K + eps);
    }
    __syncthreads();
    const float r = r_s;
    bool over = false;
    for (int64_t i = threadIdx.x; i < K; i += kNormThreads) {
        const float v = load_as(x, dt, row * K + i) * r * w[i];
        over |= f16_overflows(v);
        out[row * K + i] = __float2half_rn(v);
    }
    if (over) raise_range(status, 2u);
}

unsigned elementwise_grid(int64_t n) {
    int64_t g = (n + 255) / 256;
    return (unsigned)(g > 4096 ? 4096 : g < 1 ? 1 : g);
}

}  // namespace

cudaError_t launch_swiglu(const float* g, const float* u, void* h, int h_dtype, int64_t n, cudaStream_t st) {
    swiglu_kernel<<<elementwise_grid(n), 256, 0, st>>>(g, u, h, h_dtype, n);
    note_launches(1);
    return cudaGetLastError();
}

cudaError_t launch_rmsnorm_to_half(const void* x, int x_dtype, const float* w, float eps, __half* out, int64_t M,
                                   int64_t K, cudaStream_t st) {
    rmsnorm_to_half_kernel<<<(unsigned)M, kNormThreads, 0, st>>>(x, x_dtype, w, eps, out, K, context_status());
    note_launches(1);
    return cudaGetLastError();
}

cudaError_t launch_add_residual(const float* a, const float* res, void* y, int y_dtype, int64_t n, cudaStream_t st) {
    add_residual_kernel<<<elementwise_grid(n), 256, 0, st>>>(a, res, y, y_dtype, n);
    note_launches(1);
    return cudaGetLastError();
}

cudaError_t launch_to_half(const void* x, int dtype, __half* out, int64_t n, cudaStream_t st) {
    int64_t g = (n + 255) / 256;
    if (g > 4096) g = 4096;
    if (g < 1) g = 1;
    to_half_kernel<<<(unsigned)g, 256, 0, st>>>(x, dtype, out, n, context_status());
    note_launches(1);
    return cudaGetLastError();
}

}  // namespace nxq
