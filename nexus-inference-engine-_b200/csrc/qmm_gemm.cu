// Tensor-core prefill GEMM (M > 32 tokens) on tcgen05 / TMEM, sm_100a.
//
// y[M][N] = x[M][K] * W^T for Q4_0, Q8_0, Q4_K and Q3_K weights.  The
// reference has no batched quantized GEMM at all (its prefill runs token by
// token through gemm_int4, hybrid_model.cpp:608-633, and its fp32 fallback is
// the Metal gemm_f32_tiled, gemm_dequant.metal:77-119); this kernel is the
// prefill path for batches of more than 32 tokens.
//
// Work: a persistent grid of one CTA per SM walks (weight tile, token tile)
// work tiles of 128 weight rows x 256 tokens.  Per 64-element k-step:
//   warp 26      producer: the packed tile-chunk (256 k) by one 1-D bulk copy
//                per chunk, up to four chunks ahead (Rings)
//   warp 0       producer: the 256 x 64 f16 activation box by TMA (128-byte
//                swizzle, no multicast), four k-steps ahead
//   warps 2-17   four dequant warpgroups: thread r decodes row r's 32-element
//                group to f16 and writes it to TMEM with tcgen05.st - the
//                MMA's A operand; a k-step's two groups go to two warpgroups,
//                alternate k-steps to the other two
//   warp 1       one thread issues 4 x tcgen05.mma.kind::f16 M=128 N=256 K=16
//                (A from TMEM, B from shared memory) into a 256-column fp32
//                accumulator in TMEM
//   warps 18-25  epilogue: tcgen05.ld of the accumulator (two warps per lane
//                quadrant), conversion, store
// (Measured: two N=128 mma per K=16 into accumulator halves handed back
// separately, so the next tile starts while the second half drains, ran 18 %
// slower than one N=256 mma.)
// Every wait is bounded (sm100_ptx.cuh).
//
// Numerics as the decode kernels: weights rounded once to f16, activations
// in f16 (bf16/fp32 inputs are converted first), exact products, fp32
// accumulation; the output is rounded to the requested dtype.
#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>

#include <cstdio>

#include "dq_f16.cuh"
#include "qmm_gemm.h"
#include "sm100_ptx.cuh"
#include "stream_scratch.h"

namespace nxq {

namespace {

constexpr int kDeqGroups = 4;  // dequant warpgroups
constexpr int kEpiWarps = 8;   // two per TMEM lane quadrant
constexpr int kWarpProducer = 0, kWarpMma = 1, kWarpDeq0 = 2, kWarpEpi0 = 2 + 4 * kDeqGroups;
constexpr int kWarpWProducer = kWarpEpi0 + kEpiWarps;  // issues the tile-chunk copies
constexpr int kThreads = 32 * (kWarpWProducer + 1);
constexpr int kNT = 256;              // tokens per work tile (MMA N)
constexpr int kKS = 64;               // reduction elements per k-step (one swizzle atom)
constexpr int kStepsPerChunk = CHUNK_K / kKS;
constexpr int kAStages = 4;           // TMEM A buffers of 32 columns (measured: 8 gain nothing)
constexpr int kBarBytes = 512;        // mbarriers, TMEM address, abort flag
constexpr uint32_t kColD = 256;       // accumulator: columns 256..511
constexpr uint32_t kTmemCols = 512;
constexpr int kXBytes = kNT * kKS * 2;  // 32 KB per k-step

// Tile-chunk ring depth: as many stages (up to 4) as fit next to the x ring.
// Ring depths: four activation stages (measured: a fifth, in place of a
// tile-chunk stage, gains nothing), then as many tile-chunk stages (up to 4)
// as fit.
template <int TYPE>
struct Rings {
    static constexpr int WB = dq::Group<TYPE>::kStage;
    static constexpr int kBudget = 227 * 1024 - 1024 - kBarBytes;
    static constexpr int kX = 4;
    static constexpr int fit = (kBudget - kX * kXBytes) / WB;
    static constexpr int kW = fit > 4 ? 4 : fit;
    static_assert(kW >= 2, "tile-chunk ring too shallow");
};

struct GemmParams {
    const uint8_t* w;
    TiledShape s;
    int64_t M;
    void* y;
    int y_dtype;
    int m_tiles;
    int tiles;
    DeviceStatus* status;
};

template <typename T>
__device__ __forceinline__ T from_f32(float v);
template <>
__device__ __forceinline__ float from_f32<float>(float v) { return v; }
template <>
__device__ __forceinline__ __half from_f32<__half>(float v) { return __float2half_rn(v); }
template <>
__device__ __forceinline__ __nv_bfloat16 from_f32<__nv_bfloat16>(float v) { return __float2bfloat16_rn(v); }

// y[m0 + j][n] = v[j] for j < cnt (element offset `off` = m0 * N + n).
template <typename T>
__device__ __forceinline__ void store_col(void* y, int64_t off, int64_t N, int cnt, const uint32_t (&v)[32]) {
    T* q = reinterpret_cast<T*>(y) + off;
    if (cnt == 32) {
#pragma unroll
        for (int j = 0; j < 32; ++j, q += N) *q = from_f32<T>(__uint_as_float(v[j]));
    } else {
#pragma unroll
        for (int j = 0; j < 32; ++j, q += N)
            if (j < cnt) *q = from_f32<T>(__uint_as_float(v[j]));
    }
}

__device__ __forceinline__ bool warp_wait(uint64_t* bar, uint32_t parity, const ptx::WaitCtl& c, unsigned where) {
    int ok = 0;
    if ((threadIdx.x & 31) == 0) ok = ptx::mbar_wait(bar, parity, c, where) ? 1 : 0;
    return __shfl_sync(0xFFFFFFFFu, ok, 0) != 0;
}

template <int TYPE, int S>
__device__ __forceinline__ void dq_step(const uint8_t* stage, int r, int h, uint32_t taddr) {
    uint32_t o[16];
    if (h == 0)
        dq::Group<TYPE>::template decode<2 * S>(stage, r, o);
    else
        dq::Group<TYPE>::template decode<2 * S + 1>(stage, r, o);
    ptx::tmem_st16(taddr, o);
}

template <int TYPE>
__global__ void __launch_bounds__(kThreads, 1) tc_gemm_kernel(const GemmParams p, const __grid_constant__ CUtensorMap xmap) {
    constexpr int WB = dq::Group<TYPE>::kStage;
    constexpr int kXStages = Rings<TYPE>::kX, kWStages = Rings<TYPE>::kW;
    static_assert((2 * kXStages + 2 * kWStages + 2 * kAStages + 3) * 8 + 8 <= kBarBytes, "barrier area too small");
    static_assert(kAStages * 32 <= (int)kColD, "A stages overlap the accumulator");
    constexpr uint32_t IDESC = ptx::idesc_f16_f32(128, kNT);

    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = smem_raw + ((1024 - (ptx::smem_addr(smem_raw) & 1023)) & 1023);
    uint8_t* xs = smem;                                  // kXStages x 32 KB
    uint8_t* ws = smem + kXStages * kXBytes;             // kWStages x WB
    uint64_t* bars = reinterpret_cast<uint64_t*>(ws + kWStages * WB);
    uint64_t* x_full = bars;
    uint64_t* x_empty = x_full + kXStages;
    uint64_t* w_full = x_empty + kXStages;
    uint64_t* w_empty = w_full + kWStages;
    uint64_t* a_full = w_empty + kWStages;
    uint64_t* a_empty = a_full + kAStages;
    uint64_t* d_full = a_empty + kAStages;
    uint64_t* d_empty = d_full + 1;
    uint64_t* drain = d_empty + 1;
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(drain + 1);
    volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const ptx::WaitCtl ctl{abort_flag, p.status};
    if (threadIdx.x == 0) {
        for (int i = 0; i < kXStages; ++i) {
            ptx::mbar_init(&x_full[i], 1);
            ptx::mbar_init(&x_empty[i], 1);
        }
        for (int i = 0; i < kWStages; ++i) {
            ptx::mbar_init(&w_full[i], 1);
            ptx::mbar_init(&w_empty[i], 4 * kDeqGroups);
        }
        for (int i = 0; i < kAStages; ++i) {
            ptx::mbar_init(&a_full[i], 8);
            ptx::mbar_init(&a_empty[i], 1);
        }
        ptx::mbar_init(d_full, 1);
        ptx::mbar_init(d_empty, kEpiWarps);
        ptx::mbar_init(drain, 1);
        *abort_flag = 0;
        ptx::fence_mbar_init();
    }
    if (warp == kWarpProducer) {
        ptx::tmem_alloc(tmem_slot, kTmemCols);
        ptx::tmem_relinquish();
    }
    ptx::tc_fence_before();
    __syncthreads();
    ptx::tc_fence_after();
    const uint32_t tmem = *tmem_slot;

    const int chunks = (int)p.s.chunks;
    const int G = gridDim.x;

    if (warp == kWarpWProducer) {
        if (lane == 0) {
            uint32_t qw = 0;
            bool ok = true;
            for (int tile = blockIdx.x; tile < p.tiles && ok; tile += G) {
                const int wt = tile / p.m_tiles;
                for (int c = 0; c < chunks && ok; ++c, ++qw) {
                    const int sw = qw % kWStages;
                    if (qw >= kWStages && !(ok = ptx::mbar_wait(&w_empty[sw], ((qw / kWStages) & 1) ^ 1u, ctl, 11)))
                        break;
                    ptx::mbar_arrive_expect_tx(&w_full[sw], WB);
                    ptx::bulk_g2s(ws + sw * WB, p.w + p.s.chunk_offset(wt, c), WB, &w_full[sw]);
                }
            }
            // Do not leave with copies in flight (bounded, ignoring the abort flag).
            for (uint32_t k = qw >= kWStages ? qw - kWStages : 0; k < qw; ++k) {
                const long long t0 = clock64();
                while (!ptx::mbar_try_wait(&w_full[k % kWStages], (k / kWStages) & 1) && clock64() - t0 < ptx::kWaitCycles) {
                }
            }
        }
    } else if (warp == kWarpProducer) {
        if (lane == 0) {
            ptx::prefetch_tmap(&xmap);
            uint32_t qx = 0;
            bool ok = true;
            for (int tile = blockIdx.x; tile < p.tiles && ok; tile += G) {
                const int wt = tile / p.m_tiles, mt = tile - wt * p.m_tiles;
                (void)wt;
                for (int c = 0; c < chunks && ok; ++c) {
                    for (int st = 0; st < kStepsPerChunk; ++st, ++qx) {
                        const int sx = qx % kXStages;
                        if (qx >= kXStages &&
                            !(ok = ptx::mbar_wait(&x_empty[sx], ((qx / kXStages) & 1) ^ 1u, ctl, 12)))
                            break;
                        ptx::mbar_arrive_expect_tx(&x_full[sx], kXBytes);
                        ptx::tma_load_2d(xs + sx * kXBytes, &xmap, c * CHUNK_K + st * kKS, mt * kNT, &x_full[sx]);
                    }
                }
            }
            // Do not leave with copies in flight (bounded, ignoring the abort flag).
            for (uint32_t k = qx >= kXStages ? qx - kXStages : 0; k < qx; ++k) {
                const long long t0 = clock64();
                while (!ptx::mbar_try_wait(&x_full[k % kXStages], (k / kXStages) & 1) && clock64() - t0 < ptx::kWaitCycles) {
                }
            }
        }
    } else if (warp == kWarpMma) {
        if (lane == 0) {
            uint32_t qx = 0, qa = 0, nt = 0;
            bool ok = true;
            for (int tile = blockIdx.x; tile < p.tiles && ok; tile += G, ++nt) {
                if (nt > 0 && !(ok = ptx::mbar_wait(d_empty, (nt - 1) & 1, ctl, 13))) break;
                ptx::tc_fence_after();
                for (int c = 0; c < chunks && ok; ++c) {
                    for (int st = 0; st < kStepsPerChunk; ++st, ++qx, ++qa) {
                        const int sx = qx % kXStages, sa = qa % kAStages;
                        if (!(ok = ptx::mbar_wait(&x_full[sx], (qx / kXStages) & 1, ctl, 14))) break;
                        if (!(ok = ptx::mbar_wait(&a_full[sa], (qa / kAStages) & 1, ctl, 15))) break;
                        ptx::tc_fence_after();
                        const uint32_t xb = ptx::smem_addr(xs + sx * kXBytes);
#pragma unroll
                        for (int kk = 0; kk < kKS / 16; ++kk)
                            ptx::mma_ts_f16(tmem + kColD, tmem + sa * 32 + kk * 8, ptx::desc_sw128_kmajor(xb + kk * 32),
                                            IDESC, (c == 0 && st == 0 && kk == 0) ? 0u : 1u);
                        ptx::mma_commit(&x_empty[sx]);
                        ptx::mma_commit(&a_empty[sa]);
                    }
                }
                if (ok) ptx::mma_commit(d_full);
            }
            ptx::mma_commit(drain);
            const long long t0 = clock64();
            while (!ptx::mbar_try_wait(drain, 0) && clock64() - t0 < ptx::kWaitCycles) {
            }
        }
    } else if (warp < kWarpEpi0) {
        // Warpgroup wg takes k-steps of parity wg/2, group 2*step + wg%2.
        const int wg = (warp - kWarpDeq0) >> 2, quad = warp & 3, r = quad * 32 + lane;
        const int h = wg & 1, par = wg >> 1;
        uint32_t qw = 0, qa = 0;
        bool ok = true;
        for (int tile = blockIdx.x; tile < p.tiles && ok; tile += G) {
            for (int c = 0; c < chunks && ok; ++c, ++qw) {
                const int sw = qw % kWStages;
                if (!(ok = warp_wait(&w_full[sw], (qw / kWStages) & 1, ctl, 16))) break;
                const uint8_t* stage = ws + sw * WB;
#pragma unroll
                for (int st = 0; st < kStepsPerChunk; ++st, ++qa) {
                    if ((st & 1) != par) continue;
                    const int sa = qa % kAStages;
                    if (qa >= kAStages && !(ok = warp_wait(&a_empty[sa], ((qa / kAStages) & 1) ^ 1u, ctl, 17))) break;
                    ptx::tc_fence_after();
                    const uint32_t taddr = tmem + ((uint32_t)(quad * 32) << 16) + sa * 32 + 16 * h;
                    if (st == 0) dq_step<TYPE, 0>(stage, r, h, taddr);
                    if (st == 1) dq_step<TYPE, 1>(stage, r, h, taddr);
                    if (st == 2) dq_step<TYPE, 2>(stage, r, h, taddr);
                    if (st == 3) dq_step<TYPE, 3>(stage, r, h, taddr);
                    ptx::tmem_wait_st();
                    ptx::tc_fence_before();
                    __syncwarp();
                    if (lane == 0) ptx::mbar_arrive(&a_full[sa]);
                }
                __syncwarp();
                if (ok && lane == 0) ptx::mbar_arrive(&w_empty[sw]);
            }
        }
    } else {
        // Epilogue: warp (quad, sub) reads TMEM lanes 32 quad .. (its lane
        // quadrant) = weight row n, and token columns 128 sub .. 128 sub + 127.
        const int ew = warp - kWarpEpi0, quad = warp & 3, r = quad * 32 + lane, sub = ew >> 2;
        const int64_t M = p.M, N = p.s.N;
        uint32_t nt = 0;
        for (int tile = blockIdx.x; tile < p.tiles; tile += G, ++nt) {
            if (!warp_wait(d_full, nt & 1, ctl, 18)) break;
            ptx::tc_fence_after();
            const int wt = tile / p.m_tiles, mt = tile - wt * p.m_tiles;
            const int64_t n = (int64_t)wt * TILE_ROWS + r;
#pragma unroll 1
            for (int cb = 0; cb < 4; ++cb) {
                uint32_t v[32];
                const int c0 = sub * (kNT / 2) + 32 * cb;  // token column in the tile
                const uint32_t ta = tmem + ((uint32_t)(quad * 32) << 16) + kColD + c0;
                ptx::tmem_ld16(ta, *reinterpret_cast<uint32_t(*)[16]>(&v[0]));
                ptx::tmem_ld16(ta + 16, *reinterpret_cast<uint32_t(*)[16]>(&v[16]));
                ptx::tmem_wait_ld();
                const int64_t m0 = (int64_t)mt * kNT + c0;
                const int cnt = M - m0 >= 32 ? 32 : (int)(M - m0);
                if (n < N && cnt > 0) {
                    if (p.y_dtype == NXQ_BF16)
                        store_col<__nv_bfloat16>(p.y, m0 * N + n, N, cnt, v);
                    else if (p.y_dtype == NXQ_F16)
                        store_col<__half>(p.y, m0 * N + n, N, cnt, v);
                    else
                        store_col<float>(p.y, m0 * N + n, N, cnt, v);
                }
            }
            ptx::tc_fence_before();
            __syncwarp();
            if (lane == 0) ptx::mbar_arrive(d_empty);
        }
    }

    ptx::tc_fence_before();
    __syncthreads();
    if (warp == kWarpProducer) {
        ptx::tc_fence_after();
        ptx::tmem_dealloc(tmem, kTmemCols);
    }
}

using EncodeTiledFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                   const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                   CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);
EncodeTiledFn g_encode = nullptr;
bool g_gemm_enabled = true;

template <int TYPE>
size_t smem_bytes() {
    return 1024 + (size_t)Rings<TYPE>::kX * kXBytes + (size_t)Rings<TYPE>::kW * dq::Group<TYPE>::kStage + kBarBytes;
}

template <int TYPE>
int set_attr() {
    cudaError_t e = cudaFuncSetAttribute(tc_gemm_kernel<TYPE>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         (int)smem_bytes<TYPE>());
    if (e != cudaSuccess) return cuda_fail(e, "cudaFuncSetAttribute (tc_gemm)");
    return NXQ_OK;
}

template <int TYPE>
int launch(const Weight* w, const CUtensorMap& tmap, void* y, int y_dtype, int64_t M, cudaStream_t st) {
    GemmParams p;
    p.w = w->dev;
    p.s = w->shape;
    p.M = M;
    p.y = y;
    p.y_dtype = y_dtype;
    p.m_tiles = (int)((M + kNT - 1) / kNT);
    p.tiles = (int)(w->shape.tiles * p.m_tiles);
    p.status = context_status();
    int grid = context_sm_count();
    if (grid > p.tiles) grid = p.tiles;
    tc_gemm_kernel<TYPE><<<grid, kThreads, smem_bytes<TYPE>(), st>>>(p, tmap);
    cudaError_t e = cudaGetLastError();
    note_launches(1);
    if (e != cudaSuccess) return cuda_fail(e, "tc_gemm launch");
    return NXQ_OK;
}

// NXF INT8 weights are tiled as Q8_0 records and run on its kernel.
bool type_ok(int type) {
    return type == T_Q4_K || type == T_Q4_0 || type == T_Q8_0 || type == T_Q3_K || type == T_Q6_K ||
           type == T_Q5_K || type == T_Q4_1 || type == T_Q2_K || is_i4g(type) || type == T_NXF_I8;
}

}  // namespace

int gemm_init(int) {
    const char* env = getenv("NXQ_PREFILL_KERNEL");
    g_gemm_enabled = !(env && env[0] == 's');  // "simt" selects the CUDA-core kernel
    if (!g_gemm_enabled) return NXQ_OK;
    // The activation boxes are TMA copies described by a tensor map, which
    // only the driver can encode.  Without that entry point the tensor-core
    // GEMM cannot run; prefill would silently fall to the CUDA-core kernel,
    // so initialisation fails instead (NXQ_PREFILL_KERNEL=simt asks for the
    // CUDA-core kernel explicitly).
    void* fn = nullptr;
    cudaDriverEntryPointQueryResult q;
    cudaError_t e = cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &fn, cudaEnableDefault, &q);
    if (e != cudaSuccess || q != cudaDriverEntryPointSuccess || !fn)
        return fail(NXQ_ERR_UNSUPPORTED,
                    "the driver does not provide cuTensorMapEncodeTiled (%s, query result %d): the tcgen05 "
                    "prefill GEMM cannot run; set NXQ_PREFILL_KERNEL=simt to use the CUDA-core kernel",
                    e == cudaSuccess ? "no error" : cudaGetErrorName(e), (int)q);
    g_encode = reinterpret_cast<EncodeTiledFn>(fn);
    int rc;
    if ((rc = set_attr<T_Q4_K>()) || (rc = set_attr<T_Q4_0>()) || (rc = set_attr<T_Q8_0>()) ||
        (rc = set_attr<T_Q3_K>()) || (rc = set_attr<T_I4G128>()) || (rc = set_attr<T_Q6_K>()) ||
        (rc = set_attr<T_Q5_K>()) || (rc = set_attr<T_Q4_1>()) || (rc = set_attr<T_Q2_K>()) ||
        (rc = set_attr<T_I4G32>()) || (rc = set_attr<T_I4G64>()) || (rc = set_attr<T_I4G256>()))
        return rc;
    return NXQ_OK;
}

bool gemm_supported(const TiledShape& s, int64_t M) { return g_gemm_enabled && type_ok(s.type) && M > 32; }

void gemm_kernel_name(const TiledShape& s, int64_t, char* buf, size_t n) {
    snprintf(buf, n, "tc_gemm<%s,n%d>", type_name(s.type), kNT);
}

int gemm_qmatmul(const Weight* w, const void* x, int x_dtype, void* y, int y_dtype, int64_t M, cudaStream_t st) {
    const TiledShape& s = w->shape;
    if (!gemm_supported(s, M)) return NXQ_ERR_UNSUPPORTED;
    const bool direct = x_dtype == NXQ_F16 && ((uintptr_t)x % 16) == 0;
    const void* xh = x;
    if (!direct) {
        StreamScratch* sc = nullptr;
        int rc = scratch_for(st, 0, 0, (size_t)(M * s.K), &sc);
        if (rc) return rc;
        cudaError_t e = launch_to_half(x, x_dtype, sc->xh, M * s.K, st);
        if (e != cudaSuccess) return cuda_fail(e, "to_half launch");
        xh = sc->xh;
    }
    // Activations [M][K] f16; box 64 (k) x 256 (tokens), 128-byte swizzle; rows
    // beyond M and columns beyond K read as zero.
    CUtensorMap tmap;
    cuuint64_t dims[2] = {(cuuint64_t)s.K, (cuuint64_t)M};
    cuuint64_t strides[1] = {(cuuint64_t)s.K * 2};
    cuuint32_t box[2] = {(cuuint32_t)kKS, (cuuint32_t)kNT};
    cuuint32_t estr[2] = {1, 1};
    CUresult cr = g_encode(&tmap, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, const_cast<void*>(xh), dims, strides, box, estr,
                           CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                           CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (cr != CUDA_SUCCESS) return fail(NXQ_ERR_CUDA, "cuTensorMapEncodeTiled failed (%d)", (int)cr);
    switch (s.type) {
        case T_Q4_K: return launch<T_Q4_K>(w, tmap, y, y_dtype, M, st);
        case T_Q4_0: return launch<T_Q4_0>(w, tmap, y, y_dtype, M, st);
        case T_Q8_0:
        case T_NXF_I8: return launch<T_Q8_0>(w, tmap, y, y_dtype, M, st);
        case T_Q3_K: return launch<T_Q3_K>(w, tmap, y, y_dtype, M, st);
        case T_I4G128: return launch<T_I4G128>(w, tmap, y, y_dtype, M, st);
        case T_Q6_K: return launch<T_Q6_K>(w, tmap, y, y_dtype, M, st);
        case T_Q5_K: return launch<T_Q5_K>(w, tmap, y, y_dtype, M, st);
        case T_Q4_1: return launch<T_Q4_1>(w, tmap, y, y_dtype, M, st);
        case T_Q2_K: return launch<T_Q2_K>(w, tmap, y, y_dtype, M, st);
        case T_I4G32: return launch<T_I4G32>(w, tmap, y, y_dtype, M, st);
        case T_I4G64: return launch<T_I4G64>(w, tmap, y, y_dtype, M, st);
        case T_I4G256: return launch<T_I4G256>(w, tmap, y, y_dtype, M, st);
        default: return NXQ_ERR_UNSUPPORTED;
    }
}

}  // namespace nxq
