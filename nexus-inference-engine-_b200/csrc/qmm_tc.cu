// Tensor-core dequant-fused matmul (tcgen05 / TMEM, sm_100a).
#include "qmm_tc.h"

namespace nxq {

int tc_init(int) { return NXQ_OK; }

bool tc_supported(const TiledShape&, int64_t, int, int) { return false; }

void tc_kernel_name(const TiledShape&, int64_t, char* buf, size_t n) {
    if (n) buf[0] = 0;
}

int tc_qmatmul(const Weight*, const void*, int, void*, int, int64_t, cudaStream_t) {
    return NXQ_ERR_UNSUPPORTED;
}

}  // namespace nxq
