// Internal declarations shared by the C-ABI layer and the kernel files.
#pragma once
#include <cuda_runtime.h>

#include <cstdarg>
#include <cstddef>
#include <cstdint>

#include "../../include/nxq.h"
#include "formats.cuh"

namespace nxq {

// A registered, HBM-resident weight (the nxq_weight_t handle).
struct Weight {
    uint32_t magic;       // kWeightMagic while live; guards stale handles
    int device;
    TiledShape shape;
    uint8_t* dev = nullptr;   // tiled copy (shape.total_bytes() + kTailPad)
    size_t dev_bytes = 0;
    size_t packed_bytes = 0;  // N * K/QK * block_bytes (the algorithmic bytes)
};
constexpr uint32_t kWeightMagic = 0x4E58514Bu;  // "NXQK"
constexpr size_t kTailPad = 256;                 // slack after the last tile-chunk

// Records `msg` as the calling thread's last error and returns `status`.
int fail(int status, const char* fmt, ...);
// Maps a CUDA error to NXQ_ERR_CUDA with the call site in the message.
int cuda_fail(cudaError_t e, const char* what);

#define NXQ_CUDA(call)                                          \
    do {                                                        \
        cudaError_t e_ = (call);                                \
        if (e_ != cudaSuccess) return ::nxq::cuda_fail(e_, #call); \
    } while (0)

// Device-side error word of the context: 0 = ok, else the first error a
// kernel raised (kStatusTimeout: a bounded wait ran out; kStatusRange: a
// finite activation was too large for f16).  `where` says which wait or
// conversion.  Read by the host after a synchronize (nxq_stream_sync,
// nxq_qmatmul_host).
// The same device allocation also holds the settings kernels read on their
// slow paths: the limit of a bounded wait on another CTA's progress (in SM
// clock cycles; nxq_set_wait_limit) and test hooks (nxq_test_hook).  Drain
// waits (letting a CTA's own copies land before it exits) always use the
// fixed kDrainWaitCycles.
// host_flag is a word of mapped pinned host memory that a kernel raising an
// error also sets, so a host call learns of an error without a device read.
struct DeviceStatus {
    unsigned int code;
    unsigned int where;
    long long wait_cycles;
    unsigned int hooks;  // kHook* bits
    unsigned int pad;
    unsigned int* host_flag;
};
constexpr unsigned kStatusTimeout = 1u;
constexpr unsigned kStatusRange = 2u;
constexpr long long kDefaultWaitCycles = 4000000000LL;  // ~2 s at 2 GHz
constexpr long long kDrainWaitCycles = 4000000000LL;
// Test hook: CTAs of a stream-K launch that publish a partial sum for a tile
// another CTA finishes do not count themselves in, so that CTA's bounded wait
// for the counts runs out (a lost arrival, made on purpose and bounded).
constexpr unsigned kHookStreamKSkipCount = 1u;

// True when a finite v rounds to an infinite f16 (|v| >= 65520): the
// tensor-core kernels compute in f16, so such an activation would turn a
// finite result into inf or NaN.
__device__ __forceinline__ bool f16_overflows(float v) {
    const float a = fabsf(v);
    return a >= 65520.0f && a <= 3.402823466e38f;
}
// Sets the host-visible error flag (mapped pinned memory, written over the bus).
__device__ __forceinline__ void raise_host_flag(DeviceStatus* st) {
    unsigned int* f = st->host_flag;
    if (f) {
        *reinterpret_cast<volatile unsigned int*>(f) = 1u;
        __threadfence_system();
    }
}
// Records a range error (first error wins; `where` names the conversion).
__device__ __forceinline__ void raise_range(DeviceStatus* st, unsigned where) {
    if (st && atomicCAS(&st->code, 0u, kStatusRange) == 0u) {
        st->where = where;
        raise_host_flag(st);
    }
}

// The context's device status word and SM count (nxq_api.cu).
DeviceStatus* context_status();
// NXQ_OK once nxq_init has run, with the context's device made current on the
// calling thread; else the status (and message) the C ABI returns.
int context_ready();
int context_sm_count();

// Process-wide count of kernels launched by the library (nxq_launch_count).
void note_launches(unsigned n);

// ---- kernel launchers (return cudaError_t of the launch) -------------------
cudaError_t launch_repack(const uint8_t* src, uint8_t* dst, const TiledShape& s,
                          int64_t row0, int64_t rows, int64_t blk0, int64_t src_row_blocks,
                          cudaStream_t st);
cudaError_t launch_dequant(const uint8_t* tiled, const TiledShape& s, float* y, cudaStream_t st);

// CUDA-core fused dequant-GEMV/GEMM with exact fp32 decode; any M (chunked by 32).
// `partials` must hold splits * M * N floats when splits > 1.
cudaError_t launch_qmm_simt(const uint8_t* tiled, const TiledShape& s, const void* x, int x_dtype,
                            void* y, int y_dtype, int64_t M, float* partials, int splits,
                            cudaStream_t st);
int simt_pick_splits(const TiledShape& s, int64_t M, int sm_count);
// The CUDA-core kernel with its split-K partials in a fixed device array
// (no allocation); M * N must not exceed kNoAllocScratchFloats.
constexpr int64_t kNoAllocScratchFloats = 2 * 1024 * 1024;  // 8 MiB of fp32
int launch_qmm_simt_noalloc(const uint8_t* tiled, const TiledShape& s, const void* x, int x_dtype, void* y,
                            int y_dtype, int64_t M, int sm_count, cudaStream_t st);
int simt_rows_per_pass(int64_t M);
const char* type_name(int type);

}  // namespace nxq
