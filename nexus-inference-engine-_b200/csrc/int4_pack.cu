// NXF INT4 group weights (quant/gptq.cpp:9-70) into NXQ_TYPE_I4G<gs> blocks
// (host code only).
//
// The reference keeps the codec as three arrays - packed codes, fp32 scales,
// fp32 zeros per group of group_size elements - and reads them in two orders:
// quant/gptq.cpp's flat order over the tensor (element i is nibble i, low
// nibble first; group i / group_size) and the GEMV shader's K-major order
// (gemm_dequant.metal:29-70: codes [K/2][N], scales and zeros
// [K/group_size][N]).  Packing gathers, for every row n and group j along K,
// one block [scale][zero][group_size/2 code bytes in the flat order], so the
// weight registers like any GGUF block type and decodes as
// (float(q) - zero) * scale with the reference's fp32 values.
#include <cstring>
#include <vector>

#include "nxq_internal.h"

using nxq::fail;

namespace {

bool gs_ok(int gs) { return gs == 32 || gs == 64 || gs == 128 || gs == 256; }

}  // namespace

extern "C" {

NXQ_API int nxq_int4_pack(const uint8_t* codes, const float* scales, const float* zeros, int64_t N, int64_t K,
                          int group_size, int layout, void* out, size_t out_bytes) {
    if (!codes || !scales || !out) return fail(NXQ_ERR_ARG, "int4_pack: null argument");
    if (!gs_ok(group_size)) return fail(NXQ_ERR_CODEC, "int4_pack: group size %d (32, 64, 128 or 256)", group_size);
    if (layout != NXQ_INT4_ROWS && layout != NXQ_INT4_KMAJOR) return fail(NXQ_ERR_ARG, "int4_pack: layout %d", layout);
    if (N <= 0 || K <= 0 || K % group_size)
        return fail(NXQ_ERR_SHAPE, "int4_pack: N=%lld K=%lld (K a multiple of %d)", (long long)N, (long long)K,
                    group_size);
    const int64_t gpr = K / group_size, bb = 8 + group_size / 2;
    if (out_bytes != (size_t)(N * gpr * bb))
        return fail(NXQ_ERR_SHAPE, "int4_pack: out_bytes=%zu, need %lld", out_bytes, (long long)(N * gpr * bb));
    uint8_t* o = static_cast<uint8_t*>(out);
    for (int64_t n = 0; n < N; ++n)
        for (int64_t j = 0; j < gpr; ++j) {
            uint8_t* blk = o + (n * gpr + j) * bb;
            const int64_t gi = layout == NXQ_INT4_ROWS ? n * gpr + j : j * N + n;
            const float z = zeros ? zeros[gi] : 0.0f;
            std::memcpy(blk, &scales[gi], 4);
            std::memcpy(blk + 4, &z, 4);
            uint8_t* q = blk + 8;
            const int64_t k0 = j * group_size;
            if (layout == NXQ_INT4_ROWS) {
                // The group's elements are consecutive in the flat order, and
                // K and group_size are even, so its nibbles are whole bytes.
                std::memcpy(q, codes + (n * K + k0) / 2, (size_t)group_size / 2);
            } else {
                for (int i = 0; i < group_size; i += 2) q[i / 2] = codes[((k0 + i) / 2) * N + n];
            }
        }
    return NXQ_OK;
}

NXQ_API int nxq_weight_register_int4(const uint8_t* codes, const float* scales, const float* zeros, int64_t N,
                                     int64_t K, int group_size, int layout, nxq_weight_t* out) {
    if (!out) return fail(NXQ_ERR_ARG, "register_int4: null output");
    if (!gs_ok(group_size)) return fail(NXQ_ERR_CODEC, "register_int4: group size %d", group_size);
    if (N <= 0 || K <= 0 || K % group_size) return fail(NXQ_ERR_SHAPE, "register_int4: N=%lld K=%lld", (long long)N, (long long)K);
    const size_t bytes = (size_t)N * (size_t)(K / group_size) * (size_t)(8 + group_size / 2);
    std::vector<uint8_t> blocks;
    try {
        blocks.resize(bytes);
    } catch (const std::bad_alloc&) {
        return fail(NXQ_ERR_NOMEM, "register_int4: %zu bytes of host memory", bytes);
    }
    if (int rc = nxq_int4_pack(codes, scales, zeros, N, K, group_size, layout, blocks.data(), bytes)) return rc;
    return nxq_weight_register(blocks.data(), bytes, 100 + group_size / 32, N, K, out);
}

}  // extern "C"
