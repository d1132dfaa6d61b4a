// Residency layout kernels: GGUF row-major blocks -> tiled HBM copy, and the
// exact fp32 decode of a tiled copy (the device counterpart of
// dequant_gguf_to_fp32, nexus/src/import/gguf_importer.cpp:958-1000).
#include "nxq_internal.h"

namespace nxq {

// One warp per (row, block): the lanes copy the block's byte segments to their
// tiled positions (consecutive lanes, consecutive bytes) and, for Q4_0 / Q4_K,
// write the code bytes in the tiled order.  `src` holds `rows` rows of
// `src_row_blocks` blocks; blocks [blk0, blk0 + K/QK) of each source row become
// row (row0 + i) of the weight.  (The offsets let a tensor-parallel rank take a
// column slice of each row.)
__global__ void repack_kernel(const uint8_t* __restrict__ src, uint8_t* __restrict__ dst,
                              TiledShape s, int64_t row0, int64_t rows, int64_t blk0,
                              int64_t src_row_blocks) {
    const int64_t kb = s.K / s.g.qk;  // blocks per destination row
    const int64_t total = rows * kb;
    const int per_chunk = CHUNK_K / s.g.qk;
    const int lane = threadIdx.x & 31;
    const int64_t nwarps = (int64_t)gridDim.x * (blockDim.x >> 5);
    for (int64_t idx = (blockIdx.x * (int64_t)blockDim.x + threadIdx.x) >> 5; idx < total; idx += nwarps) {
        const int64_t i = idx / kb, b = idx - (idx / kb) * kb;
        const int64_t n = row0 + i;
        const uint8_t* blk = src + (i * src_row_blocks + blk0 + b) * s.g.bb;
        const int64_t tile = n / TILE_ROWS, r = n % TILE_ROWS;
        const int64_t chunk = b / per_chunk, j = b % per_chunk;
        uint8_t* base = dst + s.chunk_offset(tile, chunk);
        Segment seg[3];
        const int ns = block_segments(s.type, (int)r, (int)j, seg);
        if (s.type == T_NXF_I8) {
            // The Q8_0 record's scale field: fl16(1/127) for every block.
            if (lane == 0) {
                base[r * 272 + 2 * j] = (uint8_t)(kNxfI8ScaleHalf & 0xFF);
                base[r * 272 + 2 * j + 1] = (uint8_t)(kNxfI8ScaleHalf >> 8);
            }
        } else if (s.type == T_NXF_F16) {
            // One half per lane; subnormals become (signed) zero, as the
            // reference's FP16 decode reads them.
            uint32_t h = (uint32_t)blk[2 * lane] | ((uint32_t)blk[2 * lane + 1] << 8);
            if ((h & 0x7C00u) == 0) h &= 0x8000u;
            base[seg[0].dst + 2 * lane] = (uint8_t)(h & 0xFF);
            base[seg[0].dst + 2 * lane + 1] = (uint8_t)(h >> 8);
            continue;
        }
        // Bytes [c0, c1) of the block are 4-bit codes stored in the tiled order;
        // Q3_K's first 96 bytes (hmask, qs), Q6_K's first 192 (ql, qh), Q5_K's
        // last 160 (qh, qs) and Q2_K's qs are regrouped (q3/q6/q5/q2_tiled_byte).
        const int c0 = s.type == T_Q4_0 ? 2 : s.type == T_Q4_1 ? 4 : s.type == T_Q4_K ? 16 : is_i4g(s.type) ? 8 : s.g.bb;
        const int c1 = s.type == T_Q4_0 ? 18 : s.type == T_Q4_1 ? 20 : s.type == T_Q4_K ? 144 : s.g.bb;
        for (int q = 0; q < ns; ++q)
            for (int t = lane; t < seg[q].len; t += 32) {
                const int sb = seg[q].src + t;
                uint8_t v;
                if (sb >= c0 && sb < c1) {
                    const int g = (sb - c0) >> 4;
                    v = q4_tiled_byte(s.type, blk + c0 + 16 * g, (sb - c0) & 15);
                } else if (s.type == T_Q3_K && sb < 96) {
                    v = q3_tiled_byte(blk, sb);
                } else if (s.type == T_Q6_K && sb < 192) {
                    v = q6_tiled_byte(blk, sb);
                } else if (s.type == T_Q5_K && sb >= 16) {
                    v = q5_tiled_byte(blk, sb - 16);
                } else if (s.type == T_Q2_K && sb >= 16 && sb < 80) {
                    v = q2_tiled_byte(blk, sb);
                } else {
                    v = blk[sb];
                }
                base[seg[q].dst + t] = v;
            }
    }
}

cudaError_t launch_repack(const uint8_t* src, uint8_t* dst, const TiledShape& s, int64_t row0,
                          int64_t rows, int64_t blk0, int64_t src_row_blocks, cudaStream_t st) {
    const int64_t total = rows * (s.K / s.g.qk);  // blocks, one warp each
    int64_t grid = (total + 7) / 8;
    if (grid > 148 * 64) grid = 148 * 64;
    if (grid < 1) grid = 1;
    repack_kernel<<<(unsigned)grid, 256, 0, st>>>(src, dst, s, row0, rows, blk0, src_row_blocks);
    note_launches(1);
    return cudaGetLastError();
}

// One thread per 8 consecutive output elements; consecutive threads write
// consecutive 32-byte runs of y[n][k].
__global__ void dequant_kernel(const uint8_t* __restrict__ tiled, TiledShape s, float* __restrict__ y) {
    const int64_t groups_per_row = s.K / 8;
    const int64_t total = s.N * groups_per_row;
    for (int64_t idx = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; idx < total;
         idx += (int64_t)gridDim.x * blockDim.x) {
        int64_t n = idx / groups_per_row;
        int64_t k = (idx % groups_per_row) * 8;
        const uint8_t* chunk = tiled + s.chunk_offset(n / TILE_ROWS, k / CHUNK_K);
        float v[8];
        decode8(s.type, chunk, (int)(n % TILE_ROWS), (int)(k % CHUNK_K), v);
        float4* o = reinterpret_cast<float4*>(y + n * s.K + k);
        o[0] = make_float4(v[0], v[1], v[2], v[3]);
        o[1] = make_float4(v[4], v[5], v[6], v[7]);
    }
}

cudaError_t launch_dequant(const uint8_t* tiled, const TiledShape& s, float* y, cudaStream_t st) {
    int64_t total = s.N * (s.K / 8);
    int64_t grid = (total + 255) / 256;
    if (grid > 65535 * 16) grid = 65535 * 16;
    if (grid < 1) grid = 1;
    dequant_kernel<<<(unsigned)grid, 256, 0, st>>>(tiled, s, y);
    note_launches(1);
    return cudaGetLastError();
}

}  // namespace nxq
