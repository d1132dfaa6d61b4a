// Per-stream scratch shared by the matmul kernels: split-K workspace, tile
// counters (zero between calls; the kernels reset what they use) and an f16
// copy of the activations for inputs that are not f16.  Calls on one stream
// are ordered, so they can share one set; calls on different streams get
// different sets.
#pragma once
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include "nxq_internal.h"

namespace nxq {

struct StreamScratch {
    cudaStream_t st = nullptr;
    float* ws = nullptr;
    size_t ws_floats = 0;
    unsigned* counters = nullptr;
    size_t n_counters = 0;
    __half* xh = nullptr;
    size_t xh_elems = 0;
    float* epi = nullptr;  // fp32 intermediates of epilogues that run as their own kernel
    size_t epi_floats = 0;
};

// Scratch of `st`, grown to at least the given sizes.  Growing synchronizes the
// stream and is refused while the stream is being captured into a graph.
int scratch_for(cudaStream_t st, size_t ws_floats, size_t n_counters, size_t xh_elems, StreamScratch** out,
                size_t epi_floats = 0);

// Zeroes every stream's tile counters: after a kernel gave up a bounded wait,
// counts it left behind must not carry into the next launch (device idle).
void scratch_reset_counters();

// As scratch_for, except that a scratch which would have to grow while `st` is
// being captured is not an error: *out is then null and nothing is recorded.
int scratch_try(cudaStream_t st, size_t ws_floats, size_t n_counters, StreamScratch** out);

// out[i] = (half)x[i] for an f32/bf16/f16 array of n elements.
cudaError_t launch_to_half(const void* x, int dtype, __half* out, int64_t n, cudaStream_t st);

// h[i] = silu(g[i]) * u[i] = g[i] / (1 + exp(-g[i])) * u[i] in fp32, stored as h_dtype.
cudaError_t launch_swiglu(const float* g, const float* u, void* h, int h_dtype, int64_t n, cudaStream_t st);

// RMSNorm of each of the M rows of x [M][K] (f32/bf16/f16): out = f16(x * r * w)
// with r = 1 / sqrt(sum(x^2) / K + eps), all in fp32; one CTA per row.
cudaError_t launch_rmsnorm_to_half(const void* x, int x_dtype, const float* w, float eps, __half* out, int64_t M,
                                   int64_t K, cudaStream_t st);

// y[i] = a[i] + res[i] in fp32, stored as y_dtype (y may be res).
cudaError_t launch_add_residual(const float* a, const float* res, void* y, int y_dtype, int64_t n, cudaStream_t st);

}  // namespace nxq
