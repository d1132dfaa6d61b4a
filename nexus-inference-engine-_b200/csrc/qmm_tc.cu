// Tensor-core dequant-fused quantized matmul for sm_100a (tcgen05 / TMEM).
//
// Replaces the reference's Metal GEMV kernels (gemv_int4_nr8.metal:31-87,
// gemv_q3k.metal:33-98; dispatched from metal_backend.mm:607-642) for the
// GGUF block types Q4_0, Q8_0, Q4_K and Q3_K, decode batches M <= 32.
//
// Work decomposition.  The weight is stored tiled (formats.cuh): a "unit" is
// one tile-chunk, 128 weight rows x 256 reduction elements, contiguous in HBM.
// A persistent grid of G CTAs (one per SM) splits the U = tiles x chunks units
// into G contiguous ranges (stream-K), so every CTA streams one contiguous
// byte range and the load is balanced to within one unit.  A tile whose
// chunks are spread over several CTAs is finished by whichever of them
// arrives last: each writes its fp32 partial to a workspace slot, and the
// last (an atomic counter per tile, self-resetting) sums all partials in CTA
// order, so results are deterministic.
//
// Per CTA, warp-specialized (448 threads):
//   warp 0       producer: 1-D bulk copy of the packed tile-chunk and four 2-D
//                TMA loads of the activation chunk (f16, 128-byte swizzle)
//                into an S-stage shared-memory ring (no multicast)
//   warp 1       MMA: 16 x tcgen05.mma.kind::f16 per unit, M=128 weight rows,
//                N = NT tokens (16 or 32), K = 16; A from TMEM, B from shared
//                memory; fp32 accumulators in TMEM (double-buffered per tile)
//   warps 2-9    dequant: two warpgroups, one per 128-element half of the
//                chunk; thread r owns weight row r, decodes its packed bytes
//                to f16 in registers and writes them with tcgen05.st into
//                the TMEM A buffer (double-buffered)
//   warps 10-13  epilogue: tcgen05.ld of the accumulator, output in the
//                requested dtype, or split-K partial + fixup
//
// Numerics: weights are rounded once to f16 after an exact-range f16 decode
// (relative error <= 2^-11 per weight); products are exact and accumulate in
// fp32.  Activations enter as f16 (bf16/fp32 inputs are rounded to f16).
#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>

#include <cstdio>
#include <cstdlib>
#include <mutex>
#include <vector>

#include "qmm_tc.h"
#include "dq_f16.cuh"
#include "sm100_ptx.cuh"
#include "stream_scratch.h"

namespace nxq {

namespace {

constexpr int kThreads = 448;
constexpr int kWarpProducer = 0;
constexpr int kWarpMma = 1;
constexpr int kWarpDeq0 = 2;   // 2..9
constexpr int kWarpEpi0 = 10;  // 10..13
constexpr uint32_t kTmemCols = 512;
// TMEM columns: A (dequantized weights) double buffer, then D (accumulators).
__host__ __device__ constexpr uint32_t col_a(int b) { return b ? 128u : 0u; }
__host__ __device__ constexpr uint32_t col_d(int b) { return b ? 384u : 256u; }
constexpr int kMaxNT = 32;

// ---------------------------------------------------------------------------
// Per-format dequantization of one row's 128-element half of a tile-chunk into
// 64 TMEM columns (16-bit pairs: element 2c in the low half, 2c+1 high).
// `rec` points at the row's record in the shared-memory stage.
// ---------------------------------------------------------------------------

// Fmt<TYPE>::dq<H>: half H of a row's chunk (groups 4H..4H+3) into 64 TMEM columns.
template <int TYPE>
struct Fmt {
    static constexpr int kStageBytes = dq::Group<TYPE>::kStage;
    template <int H>
    __device__ static void dq(const uint8_t* s, int r, uint32_t t) {
        uint32_t o[16];
        dq::Group<TYPE>::template decode<4 * H + 0>(s, r, o);
        ptx::tmem_st16(t + 0, o);
        dq::Group<TYPE>::template decode<4 * H + 1>(s, r, o);
        ptx::tmem_st16(t + 16, o);
        dq::Group<TYPE>::template decode<4 * H + 2>(s, r, o);
        ptx::tmem_st16(t + 32, o);
        dq::Group<TYPE>::template decode<4 * H + 3>(s, r, o);
        ptx::tmem_st16(t + 48, o);
    }
};

// ---------------------------------------------------------------------------

struct TcParams {
    const uint8_t* w;
    TiledShape s;
    int64_t M;
    void* y;
    int y_dtype;
    float* ws;            // [grid][2][NT][128] split-K partials
    unsigned* counters;   // [tiles], zero between calls
    DeviceStatus* status;
    int64_t units;        // tiles * chunks
    int grid;
    int stages;
};

__device__ __forceinline__ int64_t unit_begin(int64_t c, int64_t U, int64_t G) { return c * U / G; }
// The CTA whose range holds unit u.
__device__ __forceinline__ int64_t owner_of(int64_t u, int64_t U, int64_t G) {
    return ((u + 1) * G + U - 1) / U - 1;
}

__device__ __forceinline__ void store_y(void* y, int dt, int64_t i, float v) {
    if (dt == NXQ_F32)
        reinterpret_cast<float*>(y)[i] = v;
    else if (dt == NXQ_F16)
        reinterpret_cast<__half*>(y)[i] = __float2half_rn(v);
    else
        reinterpret_cast<__nv_bfloat16*>(y)[i] = __float2bfloat16_rn(v);
}

// Warp-uniform bounded wait: lane 0 polls, the verdict is broadcast.
__device__ __forceinline__ bool warp_wait(uint64_t* bar, uint32_t parity, const ptx::WaitCtl& c,
                                          unsigned where) {
    int ok = 0;
    if ((threadIdx.x & 31) == 0) ok = ptx::mbar_wait(bar, parity, c, where) ? 1 : 0;
    return __shfl_sync(0xFFFFFFFFu, ok, 0) != 0;
}

__device__ __forceinline__ void epi_bar() { asm volatile("bar.sync 1, 128;" ::: "memory"); }

template <int TYPE, int NT>
__global__ void __launch_bounds__(kThreads, 1)
    tc_gemv_kernel(const TcParams p, const __grid_constant__ CUtensorMap xmap) {
    constexpr int WB = Fmt<TYPE>::kStageBytes;
    constexpr int XB = 4 * NT * 128;  // four 64-element swizzle atoms of NT rows
    constexpr uint32_t IDESC = ptx::idesc_f16_f32(128, NT);
    const int S = p.stages;

    extern __shared__ uint8_t smem_raw[];
    // 1024-byte alignment for the swizzled activation tiles.
    uint8_t* smem = smem_raw + ((1024 - (ptx::smem_addr(smem_raw) & 1023)) & 1023);
    uint8_t* xs = smem;                       // S x XB
    uint8_t* wst = smem + (size_t)S * XB;     // S x WB
    uint64_t* bars = reinterpret_cast<uint64_t*>(wst + (size_t)S * WB);
    uint64_t* full = bars;                    // [S]
    uint64_t* empty = bars + S;               // [S]
    uint64_t* a_full = bars + 2 * S;          // [2]
    uint64_t* a_empty = a_full + 2;           // [2]
    uint64_t* acc_full = a_empty + 2;         // [2]
    uint64_t* acc_empty = acc_full + 2;       // [2]
    uint64_t* drain = acc_empty + 2;          // [1]
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(drain + 1);
    volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
    volatile int* last_flag = abort_flag + 1;
    volatile int* epi_ok = abort_flag + 2;

    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;
    const ptx::WaitCtl ctl{abort_flag, p.status};

    if (threadIdx.x == 0) {
        for (int i = 0; i < S; ++i) {
            ptx::mbar_init(&full[i], 1);
            ptx::mbar_init(&empty[i], 8 + 1);
        }
        for (int i = 0; i < 2; ++i) {
            ptx::mbar_init(&a_full[i], 8);
            ptx::mbar_init(&a_empty[i], 1);
            ptx::mbar_init(&acc_full[i], 1);
            ptx::mbar_init(&acc_empty[i], 4);
        }
        ptx::mbar_init(drain, 1);
        *abort_flag = 0;
        *last_flag = 0;
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

    const int64_t U = p.units, G = p.grid;
    const int64_t chunks = p.s.chunks;
    const int64_t u0 = unit_begin(blockIdx.x, U, G);
    const int64_t u1 = unit_begin(blockIdx.x + 1, U, G);

    if (warp == kWarpProducer) {
        if (lane == 0) {
            ptx::prefetch_tmap(&xmap);
            int64_t i = 0;
            for (int64_t u = u0; u < u1; ++u, ++i) {
                const int st = (int)(i % S);
                const uint32_t ph = (uint32_t)((i / S) & 1);
                if (i >= S && !ptx::mbar_wait(&empty[st], ph ^ 1u, ctl, 1)) break;
                const int64_t t = u / chunks, kc = u % chunks;
                ptx::mbar_arrive_expect_tx(&full[st], WB + XB);
                ptx::bulk_g2s(wst + (size_t)st * WB, p.w + p.s.chunk_offset(t, kc), WB, &full[st]);
#pragma unroll
                for (int a = 0; a < 4; ++a)
                    ptx::tma_load_2d(xs + (size_t)st * XB + a * NT * 128, &xmap, (int)(kc * CHUNK_K + a * 64), 0,
                                     &full[st]);
            }
            // Whatever happened, do not leave with copies in flight: wait for the
            // latest load issued into every stage (bounded, ignoring the abort flag).
            const int64_t issued = i;
            for (int64_t k = issued - S < 0 ? 0 : issued - S; k < issued; ++k) {
                const int st = (int)(k % S);
                const uint32_t ph = (uint32_t)((k / S) & 1);
                const long long t0 = clock64();
                while (!ptx::mbar_try_wait(&full[st], ph) && clock64() - t0 < ptx::kWaitCycles) {
                }
            }
        }
    } else if (warp == kWarpMma) {
        if (lane == 0) {
            int64_t i = 0, tile_i = 0;
            for (int64_t u = u0; u < u1; ++u, ++i) {
                const int st = (int)(i % S);
                const uint32_t ph = (uint32_t)((i / S) & 1);
                const int ab = (int)(i & 1);
                const uint32_t aph = (uint32_t)((i >> 1) & 1);
                const int64_t kc = u % chunks;
                const bool first = (u == u0) || kc == 0;
                const bool last = (u == u1 - 1) || kc == chunks - 1;
                const int acc = (int)(tile_i & 1);
                if (first && tile_i >= 2) {
                    if (!ptx::mbar_wait(&acc_empty[acc], (uint32_t)(((tile_i >> 1) & 1) ^ 1), ctl, 2)) break;
                }
                if (!ptx::mbar_wait(&full[st], ph, ctl, 3)) break;
                if (!ptx::mbar_wait(&a_full[ab], aph, ctl, 4)) break;
                ptx::tc_fence_after();
                const uint32_t dcol = tmem + col_d(acc);
                const uint32_t acol = tmem + col_a(ab);
                const uint32_t xb = ptx::smem_addr(xs + (size_t)st * XB);
#pragma unroll
                for (int kk = 0; kk < CHUNK_K / 16; ++kk) {
                    const uint64_t desc = ptx::desc_sw128_kmajor(xb + (kk >> 2) * NT * 128 + (kk & 3) * 32);
                    ptx::mma_ts_f16(dcol, acol + kk * 8, desc, IDESC, (first && kk == 0) ? 0u : 1u);
                }
                ptx::mma_commit(&a_empty[ab]);
                ptx::mma_commit(&empty[st]);
                if (last) {
                    ptx::mma_commit(&acc_full[acc]);
                    ++tile_i;
                }
            }
            // No MMA may still be running when TMEM is released.
            ptx::mma_commit(drain);
            const long long t0 = clock64();
            while (!ptx::mbar_try_wait(drain, 0) && clock64() - t0 < ptx::kWaitCycles) {
            }
        }
    } else if (warp < kWarpEpi0) {
        // Dequant warpgroups: h = which 128-element half of the chunk.
        const int h = (warp - kWarpDeq0) >> 2;
        const int quad = warp & 3;
        const int r = quad * 32 + lane;
        int64_t i = 0;
        for (int64_t u = u0; u < u1; ++u, ++i) {
            const int st = (int)(i % S);
            const uint32_t ph = (uint32_t)((i / S) & 1);
            const int ab = (int)(i & 1);
            const uint32_t aph = (uint32_t)((i >> 1) & 1);
            if (!warp_wait(&full[st], ph, ctl, 5)) break;
            if (i >= 2 && !warp_wait(&a_empty[ab], aph ^ 1u, ctl, 6)) break;
            ptx::tc_fence_after();
            const uint32_t taddr = tmem + ((uint32_t)(quad * 32) << 16) + col_a(ab) + 64 * h;
            const uint8_t* stage = wst + (size_t)st * WB;
            if (h == 0)
                Fmt<TYPE>::template dq<0>(stage, r, taddr);
            else
                Fmt<TYPE>::template dq<1>(stage, r, taddr);
            ptx::tmem_wait_st();
            ptx::tc_fence_before();
            __syncwarp();
            if (lane == 0) {
                ptx::mbar_arrive(&a_full[ab]);
                ptx::mbar_arrive(&empty[st]);
            }
        }
    } else {
        // Epilogue warpgroup.
        const int quad = warp & 3;
        const int r = quad * 32 + lane;
        const int et = threadIdx.x - kWarpEpi0 * 32;  // 0..127
        const int64_t M = p.M, N = p.s.N;
        int64_t tile_i = 0;
        int64_t u = u0;
        while (u < u1) {
            const int64_t t = u / chunks;
            const int64_t kc0 = u % chunks;
            const int64_t tile_end = (t + 1) * chunks;
            const int64_t seg_end = u1 < tile_end ? u1 : tile_end;
            const bool whole = (kc0 == 0) && (seg_end == tile_end);
            const int acc = (int)(tile_i & 1);
            // One thread waits and the verdict is shared through a named
            // barrier, so all 128 epilogue threads always take the same path.
            if (et == 0) *epi_ok = ptx::mbar_wait(&acc_full[acc], (uint32_t)((tile_i >> 1) & 1), ctl, 7) ? 1 : 0;
            epi_bar();
            if (!*epi_ok) break;
            ptx::tc_fence_after();
            uint32_t v[NT];
#pragma unroll
            for (int c = 0; c < NT / 16; ++c)
                ptx::tmem_ld16(tmem + ((uint32_t)(quad * 32) << 16) + col_d(acc) + 16 * c,
                               *reinterpret_cast<uint32_t(*)[16]>(&v[16 * c]));
            ptx::tmem_wait_ld();
            ptx::tc_fence_before();
            __syncwarp();
            if (lane == 0) ptx::mbar_arrive(&acc_empty[acc]);

            const int64_t n = t * TILE_ROWS + r;
            if (whole) {
                if (n < N) {
#pragma unroll
                    for (int m = 0; m < NT; ++m)
                        if (m < M) store_y(p.y, p.y_dtype, m * N + n, __uint_as_float(v[m]));
                }
            } else {
                // Split-K tile: publish the partial, the last contributor sums.
                const int64_t c = blockIdx.x;
                const int slot = (unit_begin(c, U, G) / chunks == t) ? 0 : 1;
                float* mine = p.ws + ((size_t)c * 2 + slot) * (NT * TILE_ROWS);
#pragma unroll
                for (int m = 0; m < NT; ++m) mine[m * TILE_ROWS + r] = __uint_as_float(v[m]);
                __threadfence();
                epi_bar();
                const int64_t cf = owner_of(t * chunks, U, G);
                const int64_t cl = owner_of(tile_end - 1, U, G);
                if (et == 0) {
                    const unsigned old = atomicAdd(&p.counters[t], 1u);
                    *last_flag = (old == (unsigned)(cl - cf)) ? 1 : 0;
                }
                epi_bar();
                if (*last_flag) {
                    __threadfence();
                    // Sum the contributors in CTA order; the NT loads of one
                    // contributor are independent, so they are all in flight.
                    float a[NT];
#pragma unroll
                    for (int m = 0; m < NT; ++m) a[m] = 0.0f;
                    for (int64_t c2 = cf; c2 <= cl; ++c2) {
                        const int s2 = (unit_begin(c2, U, G) / chunks == t) ? 0 : 1;
                        const float* src = p.ws + ((size_t)c2 * 2 + s2) * (NT * TILE_ROWS) + r;
#pragma unroll
                        for (int m = 0; m < NT; ++m)
                            if (m < M) a[m] += __ldcg(src + m * TILE_ROWS);
                    }
                    if (n < N) {
#pragma unroll
                        for (int m = 0; m < NT; ++m)
                            if (m < M) store_y(p.y, p.y_dtype, m * N + n, a[m]);
                    }
                    if (et == 0) p.counters[t] = 0u;
                }
                epi_bar();
            }
            ++tile_i;
            u = seg_end;
        }
    }

    ptx::tc_fence_before();
    __syncthreads();
    if (warp == kWarpProducer) {
        ptx::tc_fence_after();
        ptx::tmem_dealloc(tmem, kTmemCols);
    }
}

// ---------------------------------------------------------------------------
// Host side
// ---------------------------------------------------------------------------

using EncodeTiledFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                   const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                   CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);
EncodeTiledFn g_encode = nullptr;
bool g_tc_enabled = true;
size_t g_smem_limit = 0;

template <int TYPE>
constexpr int stage_bytes() {
    return Fmt<TYPE>::kStageBytes;
}

int stages_for(int wb, int xb) {
    const size_t fixed = 1024 + 256;  // alignment slack + barriers and flags (<= 2*8+9 words + 16 B)
    int s = (int)((g_smem_limit - fixed) / (size_t)(wb + xb));
    if (s > 8) s = 8;
    return s;
}

size_t smem_for(int s, int wb, int xb) { return 1024 + (size_t)s * (wb + xb) + 256; }

template <int TYPE, int NT>
int set_attr() {
    const int wb = Fmt<TYPE>::kStageBytes, xb = 4 * NT * 128;
    const int s = stages_for(wb, xb);
    if (s < 2) return fail(NXQ_ERR_UNSUPPORTED, "not enough shared memory for the tensor-core kernel");
    cudaError_t e = cudaFuncSetAttribute(tc_gemv_kernel<TYPE, NT>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         (int)smem_for(s, wb, xb));
    if (e != cudaSuccess) return cuda_fail(e, "cudaFuncSetAttribute (tc_gemv)");
    return NXQ_OK;
}

template <int TYPE, int NT>
int launch_tc(const Weight* w, const CUtensorMap& tmap, void* y, int y_dtype, int64_t M, StreamScratch* sc,
              int grid, cudaStream_t st) {
    const int wb = Fmt<TYPE>::kStageBytes, xb = 4 * NT * 128;
    TcParams p;
    p.w = w->dev;
    p.s = w->shape;
    p.M = M;
    p.y = y;
    p.y_dtype = y_dtype;
    p.ws = sc->ws;
    p.counters = sc->counters;
    p.status = context_status();
    p.units = w->shape.tiles * w->shape.chunks;
    p.grid = grid;
    p.stages = stages_for(wb, xb);
    tc_gemv_kernel<TYPE, NT><<<grid, kThreads, smem_for(p.stages, wb, xb), st>>>(p, tmap);
    cudaError_t e = cudaGetLastError();
    note_launches(1);
    if (e != cudaSuccess) return cuda_fail(e, "tc_gemv launch");
    return NXQ_OK;
}

bool type_has_tc(int type) { return type == T_Q4_K || type == T_Q4_0 || type == T_Q8_0 || type == T_Q3_K; }

}  // namespace

int tc_init(int device) {
    const char* env = getenv("NXQ_DECODE_KERNEL");
    g_tc_enabled = !(env && env[0] == 's');  // "simt" selects the CUDA-core kernel
    cudaDeviceProp prop;
    cudaError_t e = cudaGetDeviceProperties(&prop, device);
    if (e != cudaSuccess) return cuda_fail(e, "cudaGetDeviceProperties");
    g_smem_limit = prop.sharedMemPerBlockOptin;
    void* fn = nullptr;
    cudaDriverEntryPointQueryResult q;
    e = cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &fn, cudaEnableDefault, &q);
    if (e != cudaSuccess || q != cudaDriverEntryPointSuccess || !fn) {
        g_tc_enabled = false;
        return fail(NXQ_ERR_CUDA, "cuTensorMapEncodeTiled is not available from the driver");
    }
    g_encode = reinterpret_cast<EncodeTiledFn>(fn);
    int rc;
#define NXQ_ATTR(T)                                  \
    if ((rc = set_attr<T, 16>()) != NXQ_OK) return rc; \
    if ((rc = set_attr<T, 32>()) != NXQ_OK) return rc;
    NXQ_ATTR(T_Q4_K)
    NXQ_ATTR(T_Q4_0)
    NXQ_ATTR(T_Q8_0)
    NXQ_ATTR(T_Q3_K)
#undef NXQ_ATTR
    return NXQ_OK;
}

bool tc_supported(const TiledShape& s, int64_t M, int, int) {
    return g_tc_enabled && type_has_tc(s.type) && M >= 1 && M <= kMaxNT;
}

void tc_kernel_name(const TiledShape& s, int64_t M, char* buf, size_t n) {
    snprintf(buf, n, "tc_gemv<%s,n%d>", type_name(s.type), M <= 16 ? 16 : 32);
}

int tc_qmatmul(const Weight* w, const void* x, int x_dtype, void* y, int y_dtype, int64_t M, cudaStream_t st) {
    const TiledShape& s = w->shape;
    if (!tc_supported(s, M, x_dtype, y_dtype)) return NXQ_ERR_UNSUPPORTED;
    const int NT = M <= 16 ? 16 : 32;
    const int64_t units = s.tiles * s.chunks;
    int grid = context_sm_count();
    if (grid > units) grid = (int)units;
    const bool direct = x_dtype == NXQ_F16 && ((uintptr_t)x % 16) == 0;
    StreamScratch* sc = nullptr;
    int rc = scratch_for(st, (size_t)grid * 2 * kMaxNT * TILE_ROWS, (size_t)s.tiles,
                         direct ? 0 : (size_t)(M * s.K), &sc);
    if (rc) return rc;
    const void* xh = x;
    if (!direct) {
        cudaError_t e = launch_to_half(x, x_dtype, sc->xh, M * s.K, st);
        if (e != cudaSuccess) return cuda_fail(e, "to_half launch");
        xh = sc->xh;
    }
    // Activation tensor map: [M][K] f16, box 64 x NT, 128-byte swizzle; rows
    // beyond M and columns beyond K read as zero.
    CUtensorMap tmap;
    cuuint64_t dims[2] = {(cuuint64_t)s.K, (cuuint64_t)M};
    cuuint64_t strides[1] = {(cuuint64_t)s.K * 2};
    cuuint32_t box[2] = {64, (cuuint32_t)NT};
    cuuint32_t estr[2] = {1, 1};
    CUresult cr = g_encode(&tmap, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, const_cast<void*>(xh), dims, strides, box,
                           estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                           CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (cr != CUDA_SUCCESS) return fail(NXQ_ERR_CUDA, "cuTensorMapEncodeTiled failed (%d)", (int)cr);
#define NXQ_CASE(T)                                                                        \
    case T:                                                                                \
        return NT == 16 ? launch_tc<T, 16>(w, tmap, y, y_dtype, M, sc, grid, st)           \
                        : launch_tc<T, 32>(w, tmap, y, y_dtype, M, sc, grid, st);
    switch (s.type) {
        NXQ_CASE(T_Q4_K)
        NXQ_CASE(T_Q4_0)
        NXQ_CASE(T_Q8_0)
        NXQ_CASE(T_Q3_K)
        default:
            return NXQ_ERR_UNSUPPORTED;
    }
#undef NXQ_CASE
}

}  // namespace nxq
