// Tensor-core (tcgen05) prefill GEMM for M > 32 tokens.
#pragma once
#include "nxq_internal.h"

namespace nxq {

int context_sm_count();
DeviceStatus* context_status();

// Kernel attributes and driver entry points; NXQ_PREFILL_KERNEL=simt selects
// the CUDA-core kernel instead (for comparisons).
int gemm_init(int device);
bool gemm_supported(const TiledShape& s, int64_t M);
void gemm_kernel_name(const TiledShape& s, int64_t M, char* buf, size_t n);
// y = x W^T; NXQ_ERR_UNSUPPORTED to decline.
int gemm_qmatmul(const Weight* w, const void* x, int x_dtype, void* y, int y_dtype, int64_t M, cudaStream_t st);

}  // namespace nxq
