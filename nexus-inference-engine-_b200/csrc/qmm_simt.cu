// CUDA-core fused dequant-matmul over the tiled residency layout.
//
// Every weight is decoded with the exact fp32 decoder (formats.cuh decode8, the
// reference's values bit for bit) and multiplied in fp32, so this path carries
// no rounding beyond fp32 accumulation.  It serves every block type and any M,
// and is the path for the block types and shapes the tensor-core kernels do
// not take.  Thread r of a CTA owns weight row r of a 128-row tile, the same
// row-per-thread ownership the tensor-core kernels use.
#include "nxq_internal.h"

#include <cuda_bf16.h>

#include <mutex>

namespace nxq {

namespace {

constexpr int kMaxMB = 32;  // activation rows per CTA pass, at most


__device__ __forceinline__ float load_act(const void* x, int dtype, int64_t i) {
    switch (dtype) {
        case NXQ_F16: return __half2float(reinterpret_cast<const __half*>(x)[i]);
        case NXQ_BF16: return __bfloat162float(reinterpret_cast<const __nv_bfloat16*>(x)[i]);
        default: return reinterpret_cast<const float*>(x)[i];
    }
}

__device__ __forceinline__ void store_out(void* y, int dtype, int64_t i, float v) {
    switch (dtype) {
        case NXQ_F16: reinterpret_cast<__half*>(y)[i] = __float2half_rn(v); break;
        case NXQ_BF16: reinterpret_cast<__nv_bfloat16*>(y)[i] = __float2bfloat16_rn(v); break;
        default: reinterpret_cast<float*>(y)[i] = v;
    }
}

// grid = (tiles, splits, token blocks of this launch); block = 128 threads.
// Token block z of the launch covers rows m_base + z MB .. + MB - 1.
template <int MB>
__global__ void __launch_bounds__(TILE_ROWS) qmm_simt_kernel(
    const uint8_t* __restrict__ tiled, TiledShape s, const void* __restrict__ x, int x_dtype,
    void* __restrict__ y, int y_dtype, int64_t M, float* __restrict__ partials, int splits, int64_t m_base) {
    __shared__ float xs[MB][CHUNK_K];
    const int r = threadIdx.x;
    const int64_t tile = blockIdx.x;
    const int split = blockIdx.y;
    const int64_t m0 = m_base + (int64_t)blockIdx.z * MB;
    const int mb = (int)(M - m0 < MB ? M - m0 : MB);
    const int64_t n = tile * TILE_ROWS + r;
    const int64_t c_begin = s.chunks * split / splits;
    const int64_t c_end = s.chunks * (split + 1) / splits;

    float acc[MB];
#pragma unroll
    for (int m = 0; m < MB; ++m) acc[m] = 0.0f;

    for (int64_t c = c_begin; c < c_end; ++c) {
        const int64_t k0 = c * CHUNK_K;
        __syncthreads();
        for (int i = r; i < MB * CHUNK_K; i += TILE_ROWS) {
            int m = i / CHUNK_K, kk = i % CHUNK_K;
            float v = 0.0f;
            if (m < mb && k0 + kk < s.K) v = load_act(x, x_dtype, (m0 + m) * s.K + k0 + kk);
            xs[m][kk] = v;
        }
        __syncthreads();
        const uint8_t* chunk = tiled + s.chunk_offset(tile, c);
        const int kmax = (int)(s.K - k0 < CHUNK_K ? s.K - k0 : CHUNK_K);
        for (int e0 = 0; e0 < kmax; e0 += 8) {
            float w[8];
            decode8(s.type, chunk, r, e0, w);
#pragma unroll
            for (int m = 0; m < MB; ++m) {
                float a = acc[m];
#pragma unroll
                for (int i = 0; i < 8; ++i) a = fmaf(w[i], xs[m][e0 + i], a);
                acc[m] = a;
            }
        }
    }
    if (n >= s.N) return;
    for (int m = 0; m < mb; ++m) {
        if (splits == 1)
            store_out(y, y_dtype, (m0 + m) * s.N + n, acc[m]);
        else
            partials[((int64_t)split * M + m0 + m) * s.N + n] = acc[m];
    }
}

// y[i] = sum over splits of partials[split][i], in split order.
__global__ void reduce_splits_kernel(const float* __restrict__ partials, int splits, int64_t count,
                                     void* __restrict__ y, int y_dtype) {
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < count;
         i += (int64_t)gridDim.x * blockDim.x) {
        float a = 0.0f;
        for (int sp = 0; sp < splits; ++sp) a += partials[(int64_t)sp * count + i];
        store_out(y, y_dtype, i, a);
    }
}

}  // namespace

int simt_rows_per_pass(int64_t M) { return M <= 1 ? 1 : M <= 4 ? 4 : M <= 8 ? 8 : M <= 16 ? 16 : 32; }

int simt_pick_splits(const TiledShape& s, int64_t M, int sm_count) {
    const int mb = simt_rows_per_pass(M);
    int64_t ctas = s.tiles * ((M + mb - 1) / mb);
    int64_t want = (2LL * sm_count + ctas - 1) / ctas;
    if (want < 1) want = 1;
    if (want > s.chunks) want = s.chunks;
    if (want > 64) want = 64;
    return (int)want;
}

cudaError_t launch_qmm_simt(const uint8_t* tiled, const TiledShape& s, const void* x, int x_dtype,
                            void* y, int y_dtype, int64_t M, float* partials, int splits,
                            cudaStream_t st) {
    if (splits < 1) splits = 1;
    const int mb = simt_rows_per_pass(M);
    // The grid's z extent is at most 65535: more token blocks than that run
    // as several launches, each starting at its own first token.
    const int64_t zblocks = (M + mb - 1) / mb;
    cudaError_t e = cudaSuccess;
    for (int64_t z0 = 0; z0 < zblocks && e == cudaSuccess; z0 += 65535) {
        const int64_t zn = zblocks - z0 < 65535 ? zblocks - z0 : 65535;
        dim3 grid((unsigned)s.tiles, (unsigned)splits, (unsigned)zn);
        const int64_t m_base = z0 * mb;
        switch (mb) {
#define NXQ_SIMT_CASE(MB)                                                                       \
    case MB:                                                                                    \
        qmm_simt_kernel<MB><<<grid, TILE_ROWS, 0, st>>>(tiled, s, x, x_dtype, y, y_dtype, M,     \
                                                        partials, splits, m_base);              \
        break;
            NXQ_SIMT_CASE(1)
            NXQ_SIMT_CASE(4)
            NXQ_SIMT_CASE(8)
            NXQ_SIMT_CASE(16)
            NXQ_SIMT_CASE(kMaxMB)
#undef NXQ_SIMT_CASE
        }
        e = cudaGetLastError();
        note_launches(1);
    }
    if (e != cudaSuccess || splits == 1) return e;
    int64_t count = M * s.N;
    int64_t g = (count + 255) / 256;
    if (g > 65535 * 8) g = 65535 * 8;
    reduce_splits_kernel<<<(unsigned)g, 256, 0, st>>>(partials, splits, count, y, y_dtype);
    note_launches(1);
    return cudaGetLastError();
}

// ---------------------------------------------------------------------------
// Allocation-free variant (nxq_qmatmul_noalloc).
//
// Some callers cannot allocate GPU memory while they run: code inside a
// custom allocator or memory-pool callback, real-time loops that forbid
// cudaMalloc's implicit device synchronization, and hosts whose GPU memory
// is fully reserved up front.  For them the split-K partial sums of the
// kernel above live in this fixed array instead of a per-call buffer.  Every
// GPU that loads the library holds it (kNoAllocScratchFloats floats, 8 MiB)
// until the process exits.  All calls share it, so calls that can overlap on
// the GPU (different streams) race and must be serialized by the caller.
// Nothing in it has to start at zero: every split writes all of its M x N
// partials before the reduction reads them.
// ---------------------------------------------------------------------------
static __device__ __align__(256) float g_noalloc_partials[kNoAllocScratchFloats];

namespace {
std::mutex g_noalloc_mu;
float* g_noalloc_ptr[64] = {};  // device address of g_noalloc_partials, per device
}  // namespace

int launch_qmm_simt_noalloc(const uint8_t* tiled, const TiledShape& s, const void* x, int x_dtype, void* y,
                            int y_dtype, int64_t M, int sm_count, cudaStream_t st) {
    int dev = -1;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return cuda_fail(e, "cudaGetDevice");
    if (dev < 0 || dev >= 64) return fail(NXQ_ERR_ARG, "device index %d out of range", dev);
    const int64_t outputs = M * s.N;
    if (outputs > (int64_t)kNoAllocScratchFloats)
        return fail(NXQ_ERR_SHAPE,
                    "nxq_qmatmul_noalloc: M*N = %lld exceeds its fixed scratch of %lld fp32 values",
                    (long long)outputs, (long long)kNoAllocScratchFloats);
    float* ptr = nullptr;
    {
        // First call on this device: resolve the array's device address (the
        // host-side symbol is only a stand-in and must not reach a kernel).
        std::lock_guard<std::mutex> lk(g_noalloc_mu);
        if (!g_noalloc_ptr[dev]) {
            void* p = nullptr;
            e = cudaGetSymbolAddress(&p, g_noalloc_partials);
            if (e != cudaSuccess) return cuda_fail(e, "cudaGetSymbolAddress (no-alloc scratch)");
            g_noalloc_ptr[dev] = static_cast<float*>(p);
        }
        ptr = g_noalloc_ptr[dev];
    }
    int splits = simt_pick_splits(s, M, sm_count);
    const int64_t fit = (int64_t)kNoAllocScratchFloats / (outputs > 0 ? outputs : 1);
    if (splits > fit) splits = (int)fit;
    if (splits < 1) splits = 1;
    e = launch_qmm_simt(tiled, s, x, x_dtype, y, y_dtype, M, ptr, splits, st);
    if (e != cudaSuccess) return cuda_fail(e, "qmm_simt (no-alloc) launch");
    return NXQ_OK;
}

}  // namespace nxq
