// Block formats and the HBM residency layout.
//
// Block semantics follow nexus/src/import/gguf_importer.cpp (decoders at
// :679-954); the byte offsets of every field are the reference's.  What changes
// is where those bytes sit in HBM.  The reference wraps mmap'd GGUF/NXF chunks
// as GPU buffers (metal_backend.mm:814-834); here registration re-tiles the
// blocks once so that every kernel streams contiguous, 16-byte aligned tiles:
//
//   tile      = 128 consecutive weight rows (TILE_ROWS)
//   chunk     = 256 consecutive reduction elements (CHUNK_K)
//   tile-chunk = TILE_ROWS x CHUNK_K weights = TILE_ROWS "row records" of
//                crb bytes (crb = (CHUNK_K / QK) * block_bytes); stored
//                contiguously at ((tile * chunks_per_row) + chunk) * TILE_ROWS * crb.
//
// Inside a tile-chunk each format keeps a row's bytes in "planes" so a thread
// that owns row r reads 16-byte aligned words (see place_block() below).
// Rows beyond N and blocks beyond K are zero bytes, which every format decodes
// to zero.  Decoding the tiled copy gives exactly the values of decoding the
// GGUF bytes.  Scales and most codes are copied byte for byte; the
// transformations are the order of the 4-bit codes of Q4_0 and Q4_K inside
// each 32-element group (q4_code_pos) and of the 2-bit codes and high-mask
// bits of Q3_K (q3_lo_pos, q3_hi_pos), chosen so that one or two AND/OR
// operations of a 32-bit code word yield two consecutive elements as an f16
// pair.
#pragma once
#include <cstdint>
#include <cuda_fp16.h>

namespace nxq {

constexpr int TILE_ROWS = 128;
constexpr int CHUNK_K = 256;

enum BlockType : int {
    T_Q4_0 = 2, T_Q4_1 = 3, T_Q8_0 = 8, T_Q2_K = 10, T_Q3_K = 11,
    T_Q4_K = 12, T_Q5_K = 13, T_Q6_K = 14,
    // NXF INT4 with one fp32 scale and zero per group of gs elements along K
    // (quant/gptq.cpp:9-27: w = (q - zero) * scale), as blocks of one group:
    // [scale f32][zero f32][gs/2 code bytes, element 2i low / 2i+1 high nibble
    // of byte i].  Ids outside the GGUF range: 100 + gs / 32.
    T_I4G32 = 101, T_I4G64 = 102, T_I4G128 = 104, T_I4G256 = 108,
    // NXF chunks decoded by the reference's engine at load time
    // (hybrid_model.cpp:190-255), as blocks of 32 consecutive elements along
    // K of the chunk's flat [N][K] array:
    //   T_NXF_I8   Codec::INT8, 32 int8 codes, w = (float)q / 127
    //   T_NXF_F16  Codec::FP16, 32 IEEE halves, subnormals read as zero
    //   T_NXF_F32  Codec::FP32 (and any chunk of 4 bytes per element), 32 floats
    T_NXF_I8 = 120, T_NXF_F16 = 121, T_NXF_F32 = 122
};

__host__ __device__ constexpr bool is_nxf_flat(int type) {
    return type == T_NXF_I8 || type == T_NXF_F16 || type == T_NXF_F32;
}
// The f16 value of 1/127 (0x2008 = 0.0078735...): the scale every tiled
// T_NXF_I8 block carries so the tensor-core kernels read it as Q8_0.
constexpr uint16_t kNxfI8ScaleHalf = 0x2008;

__host__ __device__ constexpr bool is_i4g(int type) {
    return type == T_I4G32 || type == T_I4G64 || type == T_I4G128 || type == T_I4G256;
}
// Group size of an I4G type; the header of its tiled row record (one 8-byte
// scale/zero pair per block of the chunk, padded to 16 bytes).
__host__ __device__ constexpr int i4g_gs(int type) { return 32 * (type - 100); }
__host__ __device__ constexpr int i4g_hdr(int type) { return ((8 * (CHUNK_K / i4g_gs(type))) + 15) & ~15; }

struct Geometry {
    int qk;    // elements per block
    int bb;    // bytes per block
    int crb;   // bytes per row record (one row of one tile-chunk)
};

__host__ __device__ inline bool geometry_of(int type, Geometry* g) {
    int qk = 0, bb = 0;
    switch (type) {
        case T_Q4_0: qk = 32; bb = 18; break;
        case T_Q4_1: qk = 32; bb = 20; break;
        case T_Q8_0: qk = 32; bb = 34; break;
        case T_Q2_K: qk = 256; bb = 84; break;
        case T_Q3_K: qk = 256; bb = 110; break;
        case T_Q4_K: qk = 256; bb = 144; break;
        case T_Q5_K: qk = 256; bb = 176; break;
        case T_Q6_K: qk = 256; bb = 210; break;
        case T_I4G32: case T_I4G64: case T_I4G128: case T_I4G256:
            qk = i4g_gs(type);
            bb = 8 + qk / 2;
            break;
        case T_NXF_I8: qk = 32; bb = 32; break;
        case T_NXF_F16: qk = 32; bb = 64; break;
        case T_NXF_F32: qk = 32; bb = 128; break;
        default: return false;
    }
    g->qk = qk;
    g->bb = bb;
    // T_NXF_I8 rows are tiled as Q8_0 records (a constant f16 scale per block).
    g->crb = is_i4g(type) ? i4g_hdr(type) + CHUNK_K / 2 : type == T_NXF_I8 ? 272 : (CHUNK_K / qk) * bb;
    return true;
}

// Tiled-copy geometry of one registered weight.
struct TiledShape {
    int type;
    int64_t N, K;
    int64_t tiles;            // ceil(N / TILE_ROWS)
    int64_t chunks;           // ceil(K / CHUNK_K) per row
    int64_t tile_chunk_bytes; // TILE_ROWS * crb
    Geometry g;
    __host__ __device__ int64_t chunk_offset(int64_t tile, int64_t chunk) const {
        return (tile * chunks + chunk) * tile_chunk_bytes;
    }
    __host__ __device__ int64_t total_bytes() const { return tiles * chunks * tile_chunk_bytes; }
};

inline bool make_tiled_shape(int type, int64_t N, int64_t K, TiledShape* s) {
    Geometry g;
    if (!geometry_of(type, &g) || N <= 0 || K <= 0 || K % g.qk) return false;
    s->type = type;
    s->N = N;
    s->K = K;
    s->g = g;
    s->tiles = (N + TILE_ROWS - 1) / TILE_ROWS;
    s->chunks = (K + CHUNK_K - 1) / CHUNK_K;
    s->tile_chunk_bytes = (int64_t)TILE_ROWS * g.crb;
    return true;
}

// ---------------------------------------------------------------------------
// Byte placement of one GGUF block inside a tile-chunk.
//   r = row within the tile (0..127), j = block index within the row record
//   (0..CHUNK_K/QK-1).  Each format lists (source offset, length, destination)
//   segments; planes are laid out so per-row records are 16-byte aligned where
//   the kernels read them with vector loads.
//
//   Q4_0  record 144 B: [d x8 : 16 B][codes x8 : 8 x 16 B, tiled code order]
//   Q4_1  record 160 B: [(d,m) x8 : 32 B][codes x8 : 8 x 16 B, tiled code order]
//   Q8_0  record 272 B: [d x8 : 16 B][codes x8 : 8 x 32 B]
//   Q4_K  record 144 B: the block itself (d, dmin, scales[12], qs[128]), qs in
//         tiled code order
//   Q5_K  record 176 B: [d, dmin, scales[12]][low nibbles: 8 groups x 16 B,
//         tiled code order][high bits: 8 groups x 4 B, see q5_hi_bit]
//   Q3_K  plane A 128 x 96 B (hmask + qs regrouped: 8 x [L0 L1 H], see
//         q3_lo_pos); plane B 128 x 14 B (scales[12], d)
//   Q2_K  plane A 128 x 80 B (scales[16], qs regrouped: 8 x [L0 L1], see
//         q2_tiled_byte); plane B 128 x 4 B (dmin, d)
//   Q6_K  plane A 128 x 192 B (ql, qh regrouped: 8 x [L0 L1 L2 L3 H0 H1], see
//         q6_lo_bit); plane B 128 x 16 B (scales); plane C 128 x 2 B (d)
//   I4G   record H + 128 B: [(scale, zero) x 256/gs, padded to H = 16..64 B]
//         [codes: 8 groups of 32 elements x 16 B, tiled code order]
//   NXF_I8  record 272 B as Q8_0: [fl16(1/127) x8][codes x8 of 32 B]
//   NXF_F16 record 512 B: the halves in order (subnormals written as zero)
//   NXF_F32 record 1024 B: the floats in order
// ---------------------------------------------------------------------------
struct Segment {
    int src, len;
    int64_t dst;
};

__host__ __device__ inline int block_segments(int type, int r, int j, Segment* s) {
    const int R = TILE_ROWS;
    switch (type) {
        case T_Q4_0:
            s[0] = {0, 2, (int64_t)r * 144 + 2 * j};
            s[1] = {2, 16, (int64_t)r * 144 + 16 + 16 * j};
            return 2;
        case T_Q4_1:
            s[0] = {0, 4, (int64_t)r * 160 + 4 * j};
            s[1] = {4, 16, (int64_t)r * 160 + 32 + 16 * j};
            return 2;
        case T_Q8_0:
            s[0] = {0, 2, (int64_t)r * 272 + 2 * j};
            s[1] = {2, 32, (int64_t)r * 272 + 16 + 32 * j};
            return 2;
        case T_Q4_K:
            s[0] = {0, 144, (int64_t)r * 144};
            return 1;
        case T_Q5_K:
            s[0] = {0, 176, (int64_t)r * 176};
            return 1;
        case T_Q3_K:
            s[0] = {0, 96, (int64_t)r * 96};
            s[1] = {96, 14, (int64_t)R * 96 + r * 14};
            return 2;
        case T_Q2_K:
            s[0] = {0, 80, (int64_t)r * 80};
            s[1] = {80, 4, (int64_t)R * 80 + r * 4};
            return 2;
        case T_Q6_K:
            s[0] = {0, 192, (int64_t)r * 192};
            s[1] = {192, 16, (int64_t)R * 192 + r * 16};
            s[2] = {208, 2, (int64_t)R * 208 + r * 2};
            return 3;
        case T_I4G32: case T_I4G64: case T_I4G128: case T_I4G256: {
            const int gs = i4g_gs(type), crb = i4g_hdr(type) + CHUNK_K / 2;
            s[0] = {0, 8, (int64_t)r * crb + 8 * j};
            s[1] = {8, gs / 2, (int64_t)r * crb + i4g_hdr(type) + (gs / 2) * j};
            return 2;
        }
        case T_NXF_I8:  // the scale field is not in the source (repack_kernel writes it)
            s[0] = {0, 32, (int64_t)r * 272 + 16 + 32 * j};
            return 1;
        case T_NXF_F16:
            s[0] = {0, 64, (int64_t)r * 512 + 64 * j};
            return 1;
        case T_NXF_F32:
            s[0] = {0, 128, (int64_t)r * 1024 + 128 * j};
            return 1;
        default:
            return 0;
    }
}

// ---------------------------------------------------------------------------
// 4-bit code order of Q4_0 / Q4_K in the tiled copy.  A 32-element group (a
// Q4_0 block; a Q4_K sub-block) keeps its 16 code bytes, as four 32-bit
// little-endian words; element e of the group sits in word e/8 at bit
// 16*(e&1) + 4*((e&7)>>1).  So word w holds elements 8w..8w+7 with the pairs
// (8w, 8w+1), (8w+2, 8w+3) in bits {0-3, 16-19} and {4-7, 20-23}, and the next
// two pairs in the same places of w >> 8.
// Where the GGUF block holds element e of a group:
//   Q4_0  byte e % 16, high nibble iff e >= 16   (gguf_importer.cpp:687-690)
//   Q4_1  the same                                (gguf_importer.cpp:707-712)
//   Q4_K  byte e / 2,  high nibble iff e is odd  (gguf_importer.cpp:864-868)
//   I4G   byte e / 2,  high nibble iff e is odd  (quant/gptq.cpp:11-24)
// ---------------------------------------------------------------------------
__host__ __device__ inline void q4_code_pos(int e, int* byte, int* shift) {
    const int i = e & 7;
    *byte = 4 * (e >> 3) + 2 * (i & 1) + (i >> 2);
    *shift = 4 * ((i >> 1) & 1);
}

__host__ __device__ inline int q4_gguf_code(int type, const uint8_t* g, int e) {
    if (type == T_Q4_0 || type == T_Q4_1) return e < 16 ? (g[e] & 15) : (g[e - 16] >> 4);
    return (e & 1) ? (g[e >> 1] >> 4) : (g[e >> 1] & 15);
}

// Byte `ob` (0..15) of a 32-element group in the tiled order: byte 4w + k
// holds elements 8w + {0,4,1,5}[k] (low nibble) and 8w + {2,6,3,7}[k] (high),
// the inverse of q4_code_pos.
__host__ __device__ inline uint8_t q4_tiled_byte(int type, const uint8_t* gguf, int ob) {
    const int w = ob >> 2, k = ob & 3;
    const int lo = 8 * w + ((k & 1) << 2) + (k >> 1), hi = lo + 2;
    return (uint8_t)(q4_gguf_code(type, gguf, lo) | (q4_gguf_code(type, gguf, hi) << 4));
}

// ---------------------------------------------------------------------------
// Q3_K code order in the tiled copy.  Each 32-element group (two 16-element
// scale groups) becomes three 32-bit words [L0][L1][H], the 12 bytes that the
// GGUF block spends on it (8 of qs, 4 of hmask).  L0 holds the 2-bit low codes
// of elements 0..15, L1 of 16..31: element e at bit 2*(e>>1) + 16*(e&1) of its
// word, so the pair (2i, 2i+1) sits in bits {2i, 2i+1} and {16+2i, 17+2i}.  H
// holds the 32 high bits: for a pair k = i&3 of the low byte half (i < 4) the
// high bits sit 2 above the code ({2k+2, 2k+18}), for i >= 4 one more (read
// through H >> 1); the bits of L1's elements are those positions plus 8
// (mod 32, read through a rotate by 8).  So a pair is (L & mask | magic) |
// (H' & mask') with a magic number whose unit is the code's lowest bit.
// Where the GGUF block holds element j (gguf_importer.cpp:809-827):
//   low code  (qs[j/4] >> 2(j%4)) & 3   (qs at block offset 32)
//   high bit  (hmask[j/8] >> (j%8)) & 1 (hmask at block offset 0)
// ---------------------------------------------------------------------------
__host__ __device__ inline int q3_lo_pos(int e16) { return 2 * (e16 >> 1) + 16 * (e16 & 1); }
__host__ __device__ inline int q3_hi_pos(int e32) {
    const int e = e32 & 15, i = e >> 1;
    const int p = 2 * (i & 3) + 2 + (i >> 2) + 16 * (e & 1);
    return e32 < 16 ? p : (p + 8) & 31;
}

// Byte `ob` (0..95) of the tiled Q3_K plane-A record of one GGUF block.
__host__ __device__ inline uint8_t q3_tiled_byte(const uint8_t* blk, int ob) {
    const int G = ob / 12, wb = ob % 12, word = wb >> 2;
    uint32_t v = 0;
    for (int bit = 0; bit < 8; ++bit) {
        const int p = 8 * (wb & 3) + bit;
        uint32_t b;
        if (word < 2) {
            // p = 2i + 16s + f: element 2i + s of the word, bit f of its code
            const int s = p >> 4, i = (p & 15) >> 1, f = p & 1;
            const int j = 32 * G + 16 * word + 2 * i + s;
            b = (blk[32 + (j >> 2)] >> (2 * (j & 3) + f)) & 1u;
        } else {
            // invert q3_hi_pos: positions with (p & 15) in [2, 9] belong to L0
            const bool low = ((p & 15) >= 2) && ((p & 15) <= 9);
            const int pa = low ? p : ((p - 8) & 31);
            const int s = pa >> 4, q = (pa & 15) - 2;  // q = 2k + (i >> 2)
            const int i = 4 * (q & 1) + (q >> 1);
            const int j = 32 * G + (low ? 0 : 16) + 2 * i + s;
            b = (blk[j >> 3] >> (j & 7)) & 1u;
        }
        v |= b << bit;
    }
    return (uint8_t)v;
}

// Q2_K code order in the tiled copy: the 2-bit codes (block offset 16, element
// j at bits 2(j%4) of byte j/4, gguf_importer.cpp:756-786) regrouped per 32
// elements as Q3_K's low codes: words L0 (elements 0..15) and L1 (16..31),
// element e at bit q3_lo_pos(e % 16).  Byte `ob` (16..79) of plane A.
__host__ __device__ inline uint8_t q2_tiled_byte(const uint8_t* blk, int ob) {
    const int G = (ob - 16) >> 3, wb = (ob - 16) & 7, word = wb >> 2;
    uint32_t v = 0;
    for (int bit = 0; bit < 8; ++bit) {
        const int p = 8 * (wb & 3) + bit, s = p >> 4, i = (p & 15) >> 1, f = p & 1;
        const int j = 32 * G + 16 * word + 2 * i + s;
        v |= (uint32_t)((blk[16 + (j >> 2)] >> (2 * (j & 3) + f)) & 1) << bit;
    }
    return (uint8_t)v;
}

__device__ __forceinline__ int q2_tiled_code(const uint8_t* rec, int e) {
    const int G = e >> 5, e32 = e & 31;
    const uint32_t w = *reinterpret_cast<const uint32_t*>(rec + 16 + 8 * G + 4 * (e32 >> 4));
    return (int)((w >> q3_lo_pos(e32 & 15)) & 3u);
}

__device__ __forceinline__ int q3_tiled_code(const uint8_t* rec, int e) {
    const int G = e >> 5, e32 = e & 31;
    const uint32_t* w = reinterpret_cast<const uint32_t*>(rec + 12 * G);
    const uint32_t lo = (w[e32 >> 4] >> q3_lo_pos(e32 & 15)) & 3u;
    const uint32_t hb = (w[2] >> q3_hi_pos(e32)) & 1u;
    return (int)(lo | (hb << 2));
}

// ---------------------------------------------------------------------------
// Q6_K code order in the tiled copy.  Each 32-element group becomes six 32-bit
// words [L0 L1 L2 L3][H0 H1], the 24 bytes the block spends on it (16 of ql,
// 8 of qh).  L_w holds the low 4 bits of elements 8w..8w+7 in the 4-bit order
// of Q4_0 / Q4_K: element 8w+i at bit 4k + 16s (k = i/2, s = i%2).  H_{w/2}
// holds their high 2 bits at bit ((4 + 4k + 16s) mod 32) + 2 (w % 2): right
// above the low nibble of pairs k = 0, 1 (after a rotate by 2 (w % 2)) and of
// pairs k = 2, 3 of L_w >> 8 (after a rotate by 8 + 2 (w % 2)).  So a pair is
// (L & mask | magic) | (H' & mask') with magic 1024 (k even) or 64 (k odd).
// Where the block holds element j (NEXUS Q6_K, gguf_importer.cpp:924-954):
//   low 4 bits  (ql[j/2] >> 4(j%2)) & 15     (ql at block offset 0)
//   high 2 bits (qh[j/4] >> 2(j%4)) & 3      (qh at block offset 128)
// ---------------------------------------------------------------------------
__host__ __device__ inline int q6_lo_bit(int e32) {
    const int i = e32 & 7;
    return 4 * (i >> 1) + 16 * (i & 1);
}
__host__ __device__ inline int q6_hi_bit(int e32) {
    const int i = e32 & 7;
    return ((4 + 4 * (i >> 1) + 16 * (i & 1)) & 31) + 2 * ((e32 >> 3) & 1);
}

// Byte `ob` (0..191) of the tiled Q6_K plane-A record of one block.
__host__ __device__ inline uint8_t q6_tiled_byte(const uint8_t* blk, int ob) {
    const int G = ob / 24, wb = ob % 24, word = wb >> 2;
    uint32_t v = 0;
    for (int bit = 0; bit < 8; ++bit) {
        const int p = 8 * (wb & 3) + bit;
        uint32_t b;
        if (word < 4) {  // p = 4k + 16s + f: bit f of the low nibble of element 8 word + 2k + s
            const int s = p >> 4, k = (p & 15) >> 2, f = p & 3;
            const int j = 32 * G + 8 * word + 2 * k + s;
            b = (blk[j >> 1] >> (4 * (j & 1) + f)) & 1u;
        } else {  // p = ((4 + 4k + 16s) mod 32) + 2h + f: bit f of the high bits of L word 2 (word - 4) + h
            const int f = p & 1, h = (p >> 1) & 1;
            const int u = (p - 2 * h - f - 4) & 31;
            const int k = (u >> 2) & 3, s = u >> 4;
            const int j = 32 * G + 8 * (2 * (word - 4) + h) + 2 * k + s;
            b = (blk[128 + (j >> 2)] >> (2 * (j & 3) + f)) & 1u;
        }
        v |= b << bit;
    }
    return (uint8_t)v;
}

// ---------------------------------------------------------------------------
// Q5_K code order in the tiled copy.  After the 16-byte header, group G keeps
// its low nibbles as four 32-bit words L_w at 16 + 16G (the 4-bit order,
// element 8w+i at bit 4k + 16s) and its 32 high bits as one word H at 144 +
// 4G, element 8w+i at bit ((4 + 4k + 16s) mod 32) + w: rotated by w (pairs
// k = 0, 1 of L_w) or 8 + w (pairs 2, 3 of L_w >> 8) each high bit sits right
// above its nibble, so a pair is (L & mask | magic) | (H' & mask').
// Where the block holds element j (gguf_importer.cpp:878-915):
//   low 4 bits  (qs[j/2] >> 4(j%2)) & 15     (qs at block offset 48)
//   high bit    (qh[j/8] >> (j%8)) & 1       (qh at block offset 16)
// ---------------------------------------------------------------------------
__host__ __device__ inline int q5_hi_bit(int e32) {
    const int i = e32 & 7;
    return ((4 + 4 * (i >> 1) + 16 * (i & 1)) & 31) + (e32 >> 3);
}

// Byte `ob` (0..159) of the tiled Q5_K code planes (record offset 16 + ob).
__host__ __device__ inline uint8_t q5_tiled_byte(const uint8_t* blk, int ob) {
    uint32_t v = 0;
    if (ob < 128) {  // low nibbles: bit p = 4k + 16s + f of word (ob % 16) / 4 of group ob / 16
        const int G = ob >> 4, wb = ob & 15, word = wb >> 2;
        for (int bit = 0; bit < 8; ++bit) {
            const int p = 8 * (wb & 3) + bit, s = p >> 4, k = (p & 15) >> 2, f = p & 3;
            const int j = 32 * G + 8 * word + 2 * k + s;
            v |= (uint32_t)((blk[48 + (j >> 1)] >> (4 * (j & 1) + f)) & 1) << bit;
        }
    } else {  // high bits: bit p = ((4 + 4k + 16s) mod 32) + w of group (ob - 128) / 4
        const int G = (ob - 128) >> 2, wb = (ob - 128) & 3;
        for (int bit = 0; bit < 8; ++bit) {
            const int p = 8 * wb + bit, w = p & 3, u = (p - w - 4) & 31;
            const int j = 32 * G + 8 * w + 2 * ((u >> 2) & 3) + (u >> 4);
            v |= (uint32_t)((blk[16 + (j >> 3)] >> (j & 7)) & 1) << bit;
        }
    }
    return (uint8_t)v;
}

// Code of element e (0..255) of a tiled Q5_K record.
__device__ __forceinline__ int q5_tiled_code(const uint8_t* rec, int e) {
    const int G = e >> 5, e32 = e & 31;
    const uint32_t l = *reinterpret_cast<const uint32_t*>(rec + 16 + 16 * G + 4 * (e32 >> 3));
    const uint32_t h = *reinterpret_cast<const uint32_t*>(rec + 144 + 4 * G);
    return (int)(((l >> q6_lo_bit(e32)) & 15u) | (((h >> q5_hi_bit(e32)) & 1u) << 4));
}

__device__ __forceinline__ int q6_tiled_code(const uint8_t* rec, int e) {
    const int G = e >> 5, e32 = e & 31;
    const uint32_t* w = reinterpret_cast<const uint32_t*>(rec + 24 * G);
    const uint32_t lo = (w[e32 >> 3] >> q6_lo_bit(e32)) & 15u;
    const uint32_t hi = (w[4 + (e32 >> 4)] >> q6_hi_bit(e32)) & 3u;
    return (int)(lo | (hi << 4));
}

__device__ __forceinline__ int q4_tiled_code(const uint8_t* g, int e) {
    int byte, shift;
    q4_code_pos(e, &byte, &shift);
    return (g[byte] >> shift) & 15;
}

// ---------------------------------------------------------------------------
// Exact device decode.  Every multiply/subtract is an explicit round-to-nearest
// fp32 intrinsic, in the reference's evaluation order, so nvcc cannot contract
// them into FMAs and the decoded bits equal the reference's.
// ---------------------------------------------------------------------------

// IEEE half -> float keeping subnormals and NaN payloads (gguf_importer.cpp:202-237).
__device__ __forceinline__ float half_bits_to_float(uint32_t h) {
    uint32_t sign = (h & 0x8000u) << 16;
    uint32_t e = (h >> 10) & 31u;
    uint32_t f = h & 1023u;
    if (e == 0) {
        // f * 2^-24 is exact in fp32.
        float mag = __fmul_rn((float)f, 5.9604644775390625e-08f);
        return __uint_as_float(__float_as_uint(mag) | sign);
    }
    if (e == 31) return __uint_as_float(sign | 0x7F800000u | (f << 13));
    return __uint_as_float(sign | ((e + 112u) << 23) | (f << 13));
}

__device__ __forceinline__ uint32_t rd16(const uint8_t* p) { return (uint32_t)p[0] | ((uint32_t)p[1] << 8); }

// The shared 6-bit scale/min unpack of Q4_K/Q5_K (gguf_importer.cpp:856-861).
__device__ __forceinline__ void kquant_scale_min(const uint8_t* sc, int g, int* s, int* m) {
    if (g < 4) {
        *s = sc[g] & 63;
        *m = (sc[g] >> 6) | ((sc[g + 8] & 15) << 2);
    } else {
        *s = sc[g] & 63;
        *m = (sc[g] >> 6) | ((sc[g + 4] >> 4) << 2);
    }
}

// Decode 8 consecutive elements [e0, e0+8) (e0 % 8 == 0, e0 < CHUNK_K) of row r
// of one tile-chunk into out[].  Values are bit-identical to the reference.
__device__ inline void decode8(int type, const uint8_t* chunk, int r, int e0, float* out) {
    const int R = TILE_ROWS;
    switch (type) {
        case T_Q4_0: {  // :679-695
            const uint8_t* rec = chunk + (int64_t)r * 144;
            int j = e0 >> 5, w = e0 & 31;
            float d = half_bits_to_float(rd16(rec + 2 * j));
            const uint8_t* q = rec + 16 + 16 * j;
            for (int i = 0; i < 8; ++i) out[i] = __fmul_rn((float)(q4_tiled_code(q, w + i) - 8), d);
            break;
        }
        case T_Q4_1: {  // :699-717
            const uint8_t* rec = chunk + (int64_t)r * 160;
            int j = e0 >> 5, w = e0 & 31;
            float d = half_bits_to_float(rd16(rec + 4 * j));
            float m = half_bits_to_float(rd16(rec + 4 * j + 2));
            const uint8_t* q = rec + 32 + 16 * j;
            for (int i = 0; i < 8; ++i) out[i] = __fadd_rn(__fmul_rn((float)q4_tiled_code(q, w + i), d), m);
            break;
        }
        case T_Q8_0: {  // :721-733
            const uint8_t* rec = chunk + (int64_t)r * 272;
            int j = e0 >> 5, w = e0 & 31;
            float d = half_bits_to_float(rd16(rec + 2 * j));
            const int8_t* q = (const int8_t*)(rec + 16 + 32 * j);
            for (int i = 0; i < 8; ++i) out[i] = __fmul_rn((float)q[w + i], d);
            break;
        }
        case T_Q2_K: {  // :756-786
            const uint8_t* rec = chunk + (int64_t)r * 80;
            const uint8_t* tail = chunk + (int64_t)R * 80 + r * 4;
            float dmin = half_bits_to_float(rd16(tail));
            float d = half_bits_to_float(rd16(tail + 2));
            int g = e0 >> 4;
            float s = __fmul_rn(d, (float)(rec[g] & 15));
            float m = __fmul_rn(dmin, (float)(rec[g] >> 4));
            for (int i = 0; i < 8; ++i) out[i] = __fsub_rn(__fmul_rn(s, (float)q2_tiled_code(rec, e0 + i)), m);
            break;
        }
        case T_Q3_K: {  // :791-833
            const uint8_t* rec = chunk + (int64_t)r * 96;
            const uint8_t* tail = chunk + (int64_t)R * 96 + r * 14;
            float d = half_bits_to_float(rd16(tail + 12));
            int g = e0 >> 4;
            int i8 = g & 7;
            int hi = tail[8 + i8 / 2] >> (4 * (i8 & 1));
            int sc = g < 8 ? ((tail[i8] & 15) | ((hi & 3) << 4))
                           : ((tail[i8] >> 4) | (((hi >> 2) & 3) << 4));
            sc -= 32;
            float ds = __fmul_rn(d, (float)sc);
            for (int i = 0; i < 8; ++i) out[i] = __fmul_rn(ds, __fsub_rn((float)q3_tiled_code(rec, e0 + i), 4.0f));
            break;
        }
        case T_Q4_K: {  // :838-873
            const uint8_t* rec = chunk + (int64_t)r * 144;
            float d = half_bits_to_float(rd16(rec));
            float dmin = half_bits_to_float(rd16(rec + 2));
            int s, m;
            kquant_scale_min(rec + 4, e0 >> 5, &s, &m);
            float ds = __fmul_rn(d, (float)s);
            float dm = __fmul_rn(dmin, (float)m);
            const uint8_t* q = rec + 16 + 16 * (e0 >> 5);
            for (int i = 0; i < 8; ++i)
                out[i] = __fsub_rn(__fmul_rn(ds, (float)q4_tiled_code(q, (e0 & 31) + i)), dm);
            break;
        }
        case T_Q5_K: {  // :878-915
            const uint8_t* rec = chunk + (int64_t)r * 176;
            float d = half_bits_to_float(rd16(rec));
            float dmin = half_bits_to_float(rd16(rec + 2));
            int s, m;
            kquant_scale_min(rec + 4, e0 >> 5, &s, &m);
            float ds = __fmul_rn(d, (float)s);
            float dm = __fmul_rn(dmin, (float)m);
            for (int i = 0; i < 8; ++i) out[i] = __fsub_rn(__fmul_rn(ds, (float)q5_tiled_code(rec, e0 + i)), dm);
            break;
        }
        case T_I4G32: case T_I4G64: case T_I4G128: case T_I4G256: {  // quant/gptq.cpp:9-27
            const uint8_t* rec = chunk + (int64_t)r * (i4g_hdr(type) + CHUNK_K / 2);
            const int j = e0 / i4g_gs(type);
            const float scale = __uint_as_float((uint32_t)rec[8 * j] | ((uint32_t)rec[8 * j + 1] << 8) |
                                                ((uint32_t)rec[8 * j + 2] << 16) | ((uint32_t)rec[8 * j + 3] << 24));
            const float zero = __uint_as_float((uint32_t)rec[8 * j + 4] | ((uint32_t)rec[8 * j + 5] << 8) |
                                               ((uint32_t)rec[8 * j + 6] << 16) | ((uint32_t)rec[8 * j + 7] << 24));
            const uint8_t* q = rec + i4g_hdr(type) + 16 * (e0 >> 5);
            for (int i = 0; i < 8; ++i)
                out[i] = __fmul_rn(__fsub_rn((float)q4_tiled_code(q, (e0 & 31) + i), zero), scale);
            break;
        }
        case T_NXF_I8: {  // hybrid_model.cpp:248-255: (float)i8 / 127.0f
            const int8_t* q = (const int8_t*)(chunk + (int64_t)r * 272 + 16 + 32 * (e0 >> 5) + (e0 & 31));
            for (int i = 0; i < 8; ++i) out[i] = __fdiv_rn((float)q[i], 127.0f);
            break;
        }
        case T_NXF_F16: {  // hybrid_model.cpp:192-210: subnormals to zero, Inf/NaN keep the mantissa
            const uint8_t* h = chunk + (int64_t)r * 512 + 2 * e0;
            for (int i = 0; i < 8; ++i) {
                const uint32_t b = rd16(h + 2 * i), sign = (b & 0x8000u) << 16, e = (b >> 10) & 31u, m = b & 1023u;
                out[i] = __uint_as_float(e == 0 ? sign : e == 31 ? (sign | 0x7F800000u | (m << 13))
                                                                 : (sign | ((e + 112u) << 23) | (m << 13)));
            }
            break;
        }
        case T_NXF_F32: {  // hybrid_model.cpp:165-176: the chunk's floats as they are
            const float* f = reinterpret_cast<const float*>(chunk + (int64_t)r * 1024) + e0;
            for (int i = 0; i < 8; ++i) out[i] = f[i];
            break;
        }
        case T_Q6_K: {  // :924-954
            const uint8_t* rec = chunk + (int64_t)r * 192;
            const int8_t* scl = (const int8_t*)(chunk + (int64_t)R * 192 + r * 16);
            float d = half_bits_to_float(rd16(chunk + (int64_t)R * 208 + r * 2));
            float ds = __fmul_rn(d, (float)scl[e0 >> 4]);
            for (int i = 0; i < 8; ++i) out[i] = __fmul_rn(ds, __fsub_rn((float)q6_tiled_code(rec, e0 + i), 32.0f));
            break;
        }
        default:
            for (int i = 0; i < 8; ++i) out[i] = 0.0f;
    }
}

}  // namespace nxq
