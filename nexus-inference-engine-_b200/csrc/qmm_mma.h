// Register-fragment (mma.sync) dequant-fused GEMV for decode batches M <= 32.
#pragma once
#include "nxq_internal.h"

namespace nxq {

int context_sm_count();
DeviceStatus* context_status();

// Kernel attributes; reads NXQ_DECODE_KERNEL ("simt" selects the exact
// CUDA-core kernel instead, for comparisons).
int mma_init(int device);
bool mma_supported(const TiledShape& s, int64_t M);
void mma_kernel_name(const TiledShape& s, int64_t M, char* buf, size_t n);
// y = x W^T (+ res, fp32 [M][N], if given); NXQ_ERR_UNSUPPORTED to decline.
int mma_qmatmul(const Weight* w, const void* x, int x_dtype, void* y, int y_dtype, int64_t M, cudaStream_t st,
                const float* res = nullptr);
// h = silu(x Wg^T) * (x Wu^T) in one launch (each CTA takes a tile of both
// weights); NXQ_ERR_UNSUPPORTED (nothing launched) unless the weights match,
// M <= 32, x is read as it is and the weight has tiles for half the SMs.
int mma_qmatmul_swiglu(const Weight* wg, const Weight* wu, const void* x, int x_dtype, void* h, int h_dtype,
                       int64_t M, cudaStream_t st);
// y_i = x_i W_i^T for n weights of one block type in as few launches as
// possible (16 weights each); items with M_i = 0 are skipped.
// NXQ_ERR_UNSUPPORTED (nothing launched) unless every item has 1 <= M_i <= 32
// and activations the kernel reads as they are.
int mma_qmatmul_grouped(const Weight* const* w, int n, const void* const* x, int x_dtype, void* const* y,
                        int y_dtype, const int64_t* M, cudaStream_t st);
// Row-split tensor parallelism in one launch: y (fp32 [M][N], every rank) =
// the sum over ranks of x_r W_r^T, each rank's partial tiles pushed into the
// others' exchange buffers over peer memory as they finish (tp_p2p.h).
// NXQ_ERR_UNSUPPORTED (the caller then multiplies and allreduces) when the
// shape or the split does not fit the exchange.
struct TpExchange;
int mma_qmatmul_tp(const Weight* w, const void* x, int x_dtype, float* y, int64_t M, cudaStream_t st,
                   const TpExchange& tp);

}  // namespace nxq
