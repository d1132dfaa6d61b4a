// Tensor-core (tcgen05 / TMEM) dequant-fused matmul kernels for sm_100a.
#pragma once
#include "nxq_internal.h"

namespace nxq {

int context_sm_count();
DeviceStatus* context_status();

// One-time per-device set-up (kernel attributes, driver entry points).
int tc_init(int device);
// True when the tensor-core kernels take this (block type, M, dtypes).
bool tc_supported(const TiledShape& s, int64_t M, int x_dtype, int y_dtype);
// Kernel name for nxq_qmatmul_kernel_name (valid when tc_supported).
void tc_kernel_name(const TiledShape& s, int64_t M, char* buf, size_t n);
// Launches y = x W^T on the tensor-core path; NXQ_ERR_UNSUPPORTED to decline.
int tc_qmatmul(const Weight* w, const void* x, int x_dtype, void* y, int y_dtype, int64_t M,
               cudaStream_t st);

}  // namespace nxq
