// Register-fragment dequant-fused GEMV for decode batches (M <= 32), sm_100a.
//
// Replaces the reference's Metal decode GEMV (gemv_int4_nr8.metal:31-87,
// gemv_q3k.metal:33-98; dispatched by ComputeDispatch::gemm_int4 ->
// MetalBackend::gemv_int4_nr8, metal_backend.mm:607-642) for every GGUF
// block type of the reference (Q4_0, Q4_1, Q8_0, Q2_K .. Q6_K) and the NXF
// INT4 group format.
//
// Why mma.sync and not tcgen05 here: a tcgen05.mma with M=128, K=16 costs
// ~60 cycles for any N <= 128 (measured on this B200), so feeding dequantized
// weights as its 128-row operand caps a GEMV at ~34 weights/cycle/SM.  The
// warp-level mma.sync.m16n8k16 takes its operands straight from the registers
// the dequantization writes, at 2 cycles/instruction/SM (measured), and the
// kernel is bound by the instructions that unpack the codes.  So the design
// minimises instructions per weight:
//   - weights are the mma's 16-row A operand (256 weights per mma; the tokens
//     are its 8 columns, 1..4 n8 tiles for M <= 8/16/32, all reusing the same
//     dequantized fragments);
//   - the tiled 4-bit code order (formats.cuh, q4_code_pos) makes each pair
//     of consecutive elements one AND/OR of a code word, then one f16
//     subtract of the magic number and one f16 FMA with the scale and offset;
//   - the activations are staged in their natural order, 8 elements per
//     16-byte piece, in lane order so the fragment loads are conflict-free.
//
// Decomposition: the weight is stored tiled (formats.cuh: 128-row tiles x
// 256-k chunks, each tile-chunk contiguous, a tile's chunks in order).  A
// unit is one tile-chunk, one bulk copy.  One CTA per SM, each taking a run
// of consecutive units: whole tiles, a run that crosses tile boundaries
// (stream-K; a tile shared by several CTAs is finished by the one holding its
// first units, from the others' partial sums in global memory), or, in a
// cluster of C CTAs, 1/C of one tile's chunks (partial sums meeting in the
// leader's shared memory).  (Measured: cutting the rows finer than tiles, so
// that every SM gets the same share, was slower - a unit that straddles two
// tiles costs more than the balance gains.)
//
// Per consumer group, 8 warps; warp w owns rows 16w..16w+15 of the tile.  Lane
// (g, t) (g = lane/4, t = lane%4) holds rows 16w+g and 16w+8+g, and the mma's
// k-slots {2t, 2t+1, 2t+8, 2t+9} of k-step j map to chunk elements
// 64t + 4j + {0, 1, 2, 3}, for x and W alike: every lane decodes one private
// 64-element slice of two rows, exactly the sub-blocks whose scales it alone
// needs.  Units are staged into an S-deep shared-memory ring: the window's
// row records byte for byte by bulk copies, and x by cp.async as 16-byte
// pieces x[token][64t + 8m .. 64t + 8m + 7] at piece index (n8 tile, m, lane).
//
// Numerics: each weight is formed in f16 as fl16(q * fl16(d*sc) + fl16(-dmin*m))
// (Q4_K; the other types analogously), products are exact and accumulate in
// fp32; activations enter as f16.
#include <cuda_bf16.h>
#include <cuda_fp16.h>

#include <cstdio>
#include <cstdlib>
#include <cstring>

#include "dq_f16.cuh"
#include "qmm_mma.h"
#include "sm100_ptx.cuh"
#include "stream_scratch.h"
#include "tp_p2p.h"

namespace nxq {

namespace {

constexpr int kWarps = 8;
constexpr int kThreads = kWarps * 32;
constexpr int kMaxMT = 32;

using dq::h2u;
using dq::u2h;

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
    return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}
template <int N>
__device__ __forceinline__ void cp_wait() {
    asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}

// C[16 rows][8 tokens] += A[16 rows][16 k] * B[16 k][8 tokens]; f16 in, fp32 accumulate.
__device__ __forceinline__ void mma16816(float (&c)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                                         uint32_t b0, uint32_t b1) {
    asm("mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
        "{%0,%1,%2,%3};"
        : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
        : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

__device__ __forceinline__ uint32_t word_of(const uint4& v, int i) {
    return i == 0 ? v.x : i == 1 ? v.y : i == 2 ? v.z : v.w;
}

// ---------------------------------------------------------------------------
// Per-format lane decoders.  load() reads the lane's 64-element slice (chunk
// elements 64t .. 64t+63) of row `row` of a staged tile-chunk and its scales;
// pairs(m, p) returns elements 8m .. 8m+7 of the slice as four f16 pairs
// (2i, 2i+1), i = 0..3.
// ---------------------------------------------------------------------------
template <int TYPE>
struct Lane;

// Q4_K / Q5_K header hd = (d, dmin, scales[12]): the f16 scale and offset
// pairs of sub-blocks 2t, 2t+1.  Scale bytes 2t, 2t+1 hold the 6-bit scale
// and the low 2 bits of the min, nibbles of bytes 8 + 2(t&1) + {0,1} the high
// 4 bits of the min.  (scale, min) pairs become exact f16 integers by the
// magic number; one f16 multiply by (d, d) / (-dmin, -dmin) then rounds d*sc
// and -dmin*m once each, as fp32 math followed by one rounding would.
__device__ __forceinline__ void kquant_lane_scales(const uint4& hd, int t, __half2 (&s2)[2], __half2 (&o2)[2]) {
    const uint32_t v = __byte_perm(((t < 2 ? hd.y : hd.z) >> (16 * (t & 1))), 0u, 0x4140u);
    const uint32_t e = __byte_perm(((hd.w >> (16 * (t & 1))) >> (4 * (t >> 1))), 0u, 0x4140u);
    const __half2 magic = u2h(0x64006400u);
    const __half2 sc = __hsub2(u2h((v & 0x003F003Fu) | 0x64006400u), magic);
    const __half2 mn = __hsub2(u2h(((v >> 6) & 0x00030003u) | ((e & 0x000F000Fu) << 2) | 0x64006400u), magic);
    const uint32_t sp = h2u(__hmul2(sc, u2h(__byte_perm(hd.x, 0u, 0x1010u))));
    const uint32_t op = h2u(__hmul2(mn, u2h(__byte_perm(hd.x, 0u, 0x3232u) ^ 0x80008000u)));
    s2[0] = u2h(__byte_perm(sp, 0u, 0x1010u));
    s2[1] = u2h(__byte_perm(sp, 0u, 0x3232u));
    o2[0] = u2h(__byte_perm(op, 0u, 0x1010u));
    o2[1] = u2h(__byte_perm(op, 0u, 0x3232u));
}

// Q4_K (gguf_importer.cpp:838-873): record = block (d, dmin, scales[12], qs[128]);
// the slice is sub-blocks 2t, 2t+1 = code bytes 32t .. 32t+31.
template <>
struct Lane<T_Q4_K> {
    static constexpr int kStage = TILE_ROWS * 144;
    uint4 q0, q1;
    __half2 s2[2], o2[2];
    __device__ __forceinline__ void load(const uint8_t* st, int row, int t) {
        const uint8_t* rec = st + row * 144;
        const uint4 hd = *reinterpret_cast<const uint4*>(rec);
        q0 = *reinterpret_cast<const uint4*>(rec + 16 + 32 * t);
        q1 = *reinterpret_cast<const uint4*>(rec + 32 + 32 * t);
        kquant_lane_scales(hd, t, s2, o2);
    }
    __device__ __forceinline__ void pairs(int m, uint32_t (&p)[4]) const {
        dq::q4_word_pairs(word_of(m < 4 ? q0 : q1, m & 3), s2[m >> 2], o2[m >> 2], p);
    }
};

// Q5_K (gguf_importer.cpp:878-915): record = [d, dmin, scales[12]][L words of
// 8 groups][H words] (formats.cuh, q5_hi_bit); the slice is sub-blocks 2t,
// 2t+1: L words at 16 + 32t, H words at 144 + 8t.
template <>
struct Lane<T_Q5_K> {
    static constexpr int kStage = TILE_ROWS * 176;
    uint4 q0, q1;
    uint2 hh;
    __half2 s2[2], o2[2];
    __device__ __forceinline__ void load(const uint8_t* st, int row, int t) {
        const uint8_t* rec = st + row * 176;
        const uint4 hd = *reinterpret_cast<const uint4*>(rec);
        q0 = *reinterpret_cast<const uint4*>(rec + 16 + 32 * t);
        q1 = *reinterpret_cast<const uint4*>(rec + 32 + 32 * t);
        hh = *reinterpret_cast<const uint2*>(rec + 144 + 8 * t);
        kquant_lane_scales(hd, t, s2, o2);
    }
    __device__ __forceinline__ void pairs(int m, uint32_t (&p)[4]) const {
        const uint32_t l = word_of(m < 4 ? q0 : q1, m & 3), h = m < 4 ? hh.x : hh.y;
        switch (m & 3) {
            case 0: dq::q5_word_pairs<0>(l, h, s2[m >> 2], o2[m >> 2], p); break;
            case 1: dq::q5_word_pairs<1>(l, h, s2[m >> 2], o2[m >> 2], p); break;
            case 2: dq::q5_word_pairs<2>(l, h, s2[m >> 2], o2[m >> 2], p); break;
            default: dq::q5_word_pairs<3>(l, h, s2[m >> 2], o2[m >> 2], p); break;
        }
    }
};

// Q6_K (gguf_importer.cpp:924-954): plane A = 8 x [L0 L1 L2 L3 H0 H1] per row
// (formats.cuh, q6_lo_bit); the slice (elements 64t .. 64t+63) is groups 2t,
// 2t+1 = 48 bytes at r*192 + 48t, with scales 4t .. 4t+3 (16 elements each)
// and d.  Weights fl16((q - 32) * fl16(d * sc)).
template <>
struct Lane<T_Q6_K> {
    static constexpr int kStage = TILE_ROWS * 210;
    uint32_t L[8], H[4];
    __half2 s2[4];
    __device__ __forceinline__ void load(const uint8_t* st, int row, int t) {
        const uint4* rec = reinterpret_cast<const uint4*>(st + row * 192 + 48 * t);
        const uint4 a = rec[0], b = rec[1], c = rec[2];
        L[0] = a.x; L[1] = a.y; L[2] = a.z; L[3] = a.w;
        H[0] = b.x; H[1] = b.y;
        L[4] = b.z; L[5] = b.w; L[6] = c.x; L[7] = c.y;
        H[2] = c.z; H[3] = c.w;
        const uint32_t sc = *reinterpret_cast<const uint32_t*>(st + TILE_ROWS * 192 + row * 16 + 4 * t);
        const float d = __half2float(__ushort_as_half(*reinterpret_cast<const uint16_t*>(st + TILE_ROWS * 208 + row * 2)));
#pragma unroll
        for (int i = 0; i < 4; ++i) s2[i] = __float2half2_rn(d * (float)(int8_t)(sc >> (8 * i)));
    }
    // Elements 8m .. 8m+7 of the slice: group m >> 2, L word m & 3, scale m >> 1.
    __device__ __forceinline__ void pairs(int m, uint32_t (&p)[4]) const {
        const int g = m >> 2, wl = m & 3;
        if (wl & 1)
            dq::q6_word_pairs<2>(L[4 * g + wl], H[2 * g + (wl >> 1)], s2[m >> 1], p);
        else
            dq::q6_word_pairs<0>(L[4 * g + wl], H[2 * g + (wl >> 1)], s2[m >> 1], p);
    }
};

// NXF INT4 groups (quant/gptq.cpp:9-27): record = [(scale, zero) per group of
// the chunk, padded to H bytes][codes x8 of 16 B]; sub-blocks 2t, 2t+1 of the
// slice lie in groups 64t / gs and (64t + 32) / gs.  Weights
// fl16(q * fl16(scale) + fl16(-(zero * scale))).
template <int TYPE>
struct LaneI4G {
    static constexpr int GS = i4g_gs(TYPE), H = i4g_hdr(TYPE), REC = H + CHUNK_K / 2;
    static constexpr int kStage = TILE_ROWS * REC;
    uint4 q0, q1;
    __half2 s2[2], o2[2];
    __device__ __forceinline__ void load(const uint8_t* st, int row, int t) {
        const uint8_t* rec = st + row * REC;
        q0 = *reinterpret_cast<const uint4*>(rec + H + 32 * t);
        q1 = *reinterpret_cast<const uint4*>(rec + H + 16 + 32 * t);
#pragma unroll
        for (int h = 0; h < 2; ++h) {
            const float2 sz = *reinterpret_cast<const float2*>(rec + 8 * ((64 * t + 32 * h) / GS));
            s2[h] = __float2half2_rn(sz.x);
            o2[h] = __float2half2_rn(-(sz.y * sz.x));
        }
    }
    __device__ __forceinline__ void pairs(int m, uint32_t (&p)[4]) const {
        dq::q4_word_pairs(word_of(m < 4 ? q0 : q1, m & 3), s2[m >> 2], o2[m >> 2], p);
    }
};
template <>
struct Lane<T_I4G32> : LaneI4G<T_I4G32> {};
template <>
struct Lane<T_I4G64> : LaneI4G<T_I4G64> {};
template <>
struct Lane<T_I4G128> : LaneI4G<T_I4G128> {};
template <>
struct Lane<T_I4G256> : LaneI4G<T_I4G256> {};

// Q4_0 (gguf_importer.cpp:679-695): record = [d x8][codes x8 of 16 B]; the
// slice is blocks 2t, 2t+1.
template <>
struct Lane<T_Q4_0> {
    static constexpr int kStage = TILE_ROWS * 144;
    uint4 q0, q1;
    __half2 s2[2], o2[2];
    __device__ __forceinline__ void load(const uint8_t* st, int row, int t) {
        const uint8_t* rec = st + row * 144;
        const uint32_t dw = *reinterpret_cast<const uint32_t*>(rec + 4 * t);
        q0 = *reinterpret_cast<const uint4*>(rec + 16 + 32 * t);
        q1 = *reinterpret_cast<const uint4*>(rec + 32 + 32 * t);
        const __half2 neg8 = u2h(0xC800C800u);
        s2[0] = u2h((dw & 0xFFFFu) | (dw << 16));
        s2[1] = u2h((dw >> 16) | (dw & 0xFFFF0000u));
        o2[0] = __hmul2(s2[0], neg8);  // exact
        o2[1] = __hmul2(s2[1], neg8);
    }
    __device__ __forceinline__ void pairs(int m, uint32_t (&p)[4]) const {
        dq::q4_word_pairs(word_of(m < 4 ? q0 : q1, m & 3), s2[m >> 2], o2[m >> 2], p);
    }
};

// Q4_1 (gguf_importer.cpp:699-717): record = [(d, m) x8][codes x8 of 16 B];
// the slice is blocks 2t, 2t+1; weights fl16(q * d + m).
template <>
struct Lane<T_Q4_1> {
    static constexpr int kStage = TILE_ROWS * 160;
    uint4 q0, q1;
    __half2 s2[2], o2[2];
    __device__ __forceinline__ void load(const uint8_t* st, int row, int t) {
        const uint8_t* rec = st + row * 160;
        const uint2 dm = *reinterpret_cast<const uint2*>(rec + 8 * t);
        q0 = *reinterpret_cast<const uint4*>(rec + 32 + 32 * t);
        q1 = *reinterpret_cast<const uint4*>(rec + 48 + 32 * t);
        s2[0] = u2h((dm.x & 0xFFFFu) | (dm.x << 16));
        o2[0] = u2h((dm.x >> 16) | (dm.x & 0xFFFF0000u));
        s2[1] = u2h((dm.y & 0xFFFFu) | (dm.y << 16));
        o2[1] = u2h((dm.y >> 16) | (dm.y & 0xFFFF0000u));
    }
    __device__ __forceinline__ void pairs(int m, uint32_t (&p)[4]) const {
        dq::q4_word_pairs(word_of(m < 4 ? q0 : q1, m & 3), s2[m >> 2], o2[m >> 2], p);
    }
};

// Q2_K (gguf_importer.cpp:756-786): plane A = [scales[16]][8 x [L0 L1]] per
// row (formats.cuh, q2_tiled_byte), plane B = (dmin, d); the slice (elements
// 64t .. 64t+63) is code words 4t .. 4t+3 with scale bytes 4t .. 4t+3.
template <>
struct Lane<T_Q2_K> {
    static constexpr int kStage = TILE_ROWS * 84;
    uint4 q;
    __half2 s2[4], o2[4];
    __device__ __forceinline__ void load(const uint8_t* st, int row, int t) {
        const uint8_t* rec = st + row * 80;
        q = *reinterpret_cast<const uint4*>(rec + 16 + 16 * t);
        const uint32_t sc = *reinterpret_cast<const uint32_t*>(rec + 4 * t);
        const uint32_t dd = *reinterpret_cast<const uint32_t*>(st + TILE_ROWS * 80 + row * 4);
        const float dmin = __half2float(__ushort_as_half((unsigned short)(dd & 0xFFFFu)));
        const float d = __half2float(__ushort_as_half((unsigned short)(dd >> 16)));
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            const uint32_t b = (sc >> (8 * i)) & 0xFFu;
            s2[i] = __float2half2_rn(d * (float)(b & 15u));
            o2[i] = __float2half2_rn(-(dmin * (float)(b >> 4)));
        }
    }
    // Elements 8m .. 8m+7: code word m >> 1 (low or high byte of each half),
    // scale group m >> 1.
    __device__ __forceinline__ void pairs(int m, uint32_t (&p)[4]) const {
        const uint32_t l = word_of(q, m >> 1);
        dq::q2_half_pairs((m & 1) ? l >> 8 : l, s2[m >> 1], o2[m >> 1], p);
    }
};

// Q8_0 (gguf_importer.cpp:721-733): record = [d x8][codes x8 of 32 B]; the
// slice is blocks 2t, 2t+1 = code bytes 64t .. 64t+63.
template <>
struct Lane<T_Q8_0> {
    static constexpr int kStage = TILE_ROWS * 272;
    uint4 c[4];
    __half2 s2[2];
    __device__ __forceinline__ void load(const uint8_t* st, int row, int t) {
        const uint8_t* rec = st + row * 272;
        const uint32_t dw = *reinterpret_cast<const uint32_t*>(rec + 4 * t);
        const uint4* cv = reinterpret_cast<const uint4*>(rec + 16 + 64 * t);
#pragma unroll
        for (int i = 0; i < 4; ++i) c[i] = cv[i];
        s2[0] = u2h((dw & 0xFFFFu) | (dw << 16));
        s2[1] = u2h((dw >> 16) | (dw & 0xFFFF0000u));
    }
    __device__ __forceinline__ void pairs(int m, uint32_t (&p)[4]) const {
        // Signed byte b -> f16 1152 + b via (b ^ 0x80) in the mantissa of 1024.
        const __half2 bias = u2h(0x64806480u);
        const uint32_t w0 = word_of(c[m >> 1], 2 * (m & 1)), w1 = word_of(c[m >> 1], 2 * (m & 1) + 1);
        const __half2 s = s2[m >> 2];
        p[0] = h2u(__hmul2(__hsub2(u2h(__byte_perm(w0, 0u, 0x4140u) ^ 0x64806480u), bias), s));
        p[1] = h2u(__hmul2(__hsub2(u2h(__byte_perm(w0, 0u, 0x4342u) ^ 0x64806480u), bias), s));
        p[2] = h2u(__hmul2(__hsub2(u2h(__byte_perm(w1, 0u, 0x4140u) ^ 0x64806480u), bias), s));
        p[3] = h2u(__hmul2(__hsub2(u2h(__byte_perm(w1, 0u, 0x4342u) ^ 0x64806480u), bias), s));
    }
};

// Q3_K (gguf_importer.cpp:791-833): plane A = 8 x [L0 L1 H] per row (tiled
// code order, formats.cuh q3_lo_pos), plane B = [scales 12][d] at 128*96 +
// row*14.  The slice's elements are groups 2t, 2t+1 = bytes 24t .. 24t+23 of
// the row's plane-A record, in four 16-element scale groups.
template <>
struct Lane<T_Q3_K> {
    static constexpr int kStage = TILE_ROWS * 110;
    uint32_t L[4], H[2], Hr[2];  // L0, L1 of group 2t, then of 2t+1; their high-bit words
    __half2 s2[4];
    __device__ __forceinline__ void load(const uint8_t* st, int row, int t) {
        const uint8_t* rec = st + row * 96 + 24 * t;
        const uint2 a = *reinterpret_cast<const uint2*>(rec);
        const uint2 b = *reinterpret_cast<const uint2*>(rec + 8);
        const uint2 c = *reinterpret_cast<const uint2*>(rec + 16);
        L[0] = a.x;
        L[1] = a.y;
        H[0] = b.x;
        L[2] = b.y;
        L[3] = c.x;
        H[1] = c.y;
        Hr[0] = __funnelshift_r(H[0], H[0], 8);
        Hr[1] = __funnelshift_r(H[1], H[1], 8);
        const uint16_t* tl = reinterpret_cast<const uint16_t*>(st + TILE_ROWS * 96 + row * 14);
        // Groups G = 4t + gg (gg = 0..3): i8 = G & 7 = 4(t&1) + gg; the low 4
        // bits of the 6-bit scale are nibble (t >> 1) of scale byte i8, the
        // high 2 bits are bits 2(t >> 1) + {0,1} of nibble (gg & 1) of byte
        // 8 + 2(t&1) + (gg >> 1).  (scale - 32) * d as one f16 rounding of the
        // exact product, through exact f16 integers.
        const uint32_t lo4 = ((t & 1) ? (tl[2] | ((uint32_t)tl[3] << 16)) : (tl[0] | ((uint32_t)tl[1] << 16)));
        const uint32_t hi2 = (uint32_t)tl[4 + (t & 1)];  // bytes 8 + 2(t&1), +1
        const uint32_t sh = 4 * (t >> 1), hs = 2 * (t >> 1);
        const __half2 d2 = u2h(__byte_perm((uint32_t)tl[6], 0u, 0x1010u));
        const __half2 bias = u2h(0x64206420u);  // 1056 = magic + 32
#pragma unroll
        for (int pr = 0; pr < 2; ++pr) {  // groups gg = 2pr, 2pr+1
            const uint32_t l = (__byte_perm(lo4, 0u, 0x4040u | ((2 * pr + 1) << 8) | (2 * pr)) >> sh) & 0x000F000Fu;
            const uint32_t hb = (hi2 >> (8 * pr)) & 0xFFu;  // byte for gg = 2pr, 2pr+1: nibbles 0, 1
            const uint32_t h = (((hb >> hs) & 3u) | ((((hb >> 4) >> hs) & 3u) << 16)) << 4;
            const uint32_t sp = h2u(__hmul2(__hsub2(u2h(l | h | 0x64006400u), bias), d2));
            s2[2 * pr] = u2h(__byte_perm(sp, 0u, 0x1010u));
            s2[2 * pr + 1] = u2h(__byte_perm(sp, 0u, 0x3232u));
        }
    }
    // Elements 8m .. 8m+7 of the slice: group m >> 2, L word (m & 3) >> 1,
    // pairs 4((m & 3) & 1) .. +3 of that word.
    __device__ __forceinline__ void pairs(int m, uint32_t (&p)[4]) const {
        const int g = m >> 2, j = (m & 3) >> 1;
        uint32_t l = L[2 * g + j], h = j ? Hr[g] : H[g];
        if (m & 1) {
            l >>= 8;
            h >>= 1;
        }
        const __half2 s = s2[m >> 1];
        p[0] = dq::q3_pair<0>(l, h, s);
        p[1] = dq::q3_pair<1>(l, h, s);
        p[2] = dq::q3_pair<2>(l, h, s);
        p[3] = dq::q3_pair<3>(l, h, s);
    }
};

// Cluster-wide barrier over all threads of all CTAs of the cluster.
__device__ __forceinline__ void cluster_sync() {
    asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}
// Address of the same shared-memory location in CTA `rank` of the cluster.
__device__ __forceinline__ uint32_t cluster_addr(const void* p, uint32_t rank) {
    uint32_t r;
    asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(smem_u32(p)), "r"(rank));
    return r;
}
__device__ __forceinline__ void named_sync(int id, int threads) {
    asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(threads) : "memory");
}

constexpr int kMaxCluster = 8;
constexpr int kMaxItems = 16;

// Shared-memory budget of a variant with `groups` consumer warpgroups.
template <int TYPE, int MT, int GROUPS, int CMAX, int SETS>
struct Budget {
    static constexpr int NT = MT / 8;
    static constexpr int WB = Lane<TYPE>::kStage;
    static constexpr int XB = NT * 8 * 32 * 16;
    static constexpr int PB = NT * 8 * TILE_ROWS * 4;
    static constexpr int RECV = (CMAX - 1) * PB;
    static constexpr int COMB = 2 * SETS * (GROUPS - 1) * PB;
    static constexpr int S0 = (227 * 1024 - 2048 - RECV - COMB) / (WB + XB);
};

// PAIR: the SwiGLU pairing (each tile twice, gate then up weights, with two
// result sets handed over; no cluster split).
template <int TYPE, int MT, bool PAIR = false>
struct Cfg {
    static constexpr int NT = MT / 8;                   // n8 token tiles
    static constexpr int WB = Lane<TYPE>::kStage;
    static constexpr int XB = NT * 8 * 32 * 16;         // pieces (n8 tile, m, lane) of 16 B
    static constexpr int PB = NT * 8 * TILE_ROWS * 4;   // one tile's fp32 partial, [row][token]
    // Up to 8 CTAs per cluster; with 32 tokens the partial sums are large, so
    // 4 where three stages still fit beside them, else 2.
    static constexpr int CMAX = PAIR ? 1 : NT >= 4 ? (Budget<TYPE, MT, 2, 4, 1>::S0 >= 3 ? 4 : 2) : kMaxCluster;
    static constexpr int SETS = PAIR ? 2 : 1;           // result sets per tile
    // Two consumer warpgroups (measured: a third one, with its tighter
    // register budget, is slower).
    static constexpr int G = 2;
    static constexpr int RECV = (CMAX - 1) * PB;        // cluster leader: the other ranks' partials
    static constexpr int COMB = 2 * SETS * (G - 1) * PB;  // groups 1.. -> group 0 hand-over, two tiles deep
    static constexpr int S0 = Budget<TYPE, MT, G, CMAX, SETS>::S0;
    static constexpr int S = S0 > 8 ? 8 : S0;
    static constexpr int kConsumers = G * kThreads;
    // Producer warps; warp w stages tokens 8w..8w+7 (one is enough up to 8
    // tokens, measured: extra warps there cost 3 % at M = 1).
    static constexpr int kXWarps = NT >= 2 ? 4 : 1;
    static constexpr int kAll = kConsumers + 32 * kXWarps;
    // A warp's 16 mma per unit chain through its accumulators; with one n8
    // tile Q4_K alternates two accumulator sets (two chains of 8, added at the
    // tile's end).  Measured: 2-3 % faster there, no gain or slower for the
    // other formats and for more tiles.
    static constexpr int kAccSets = (NT == 1 && TYPE == T_Q4_K) ? 2 : 1;
    static constexpr size_t smem = (size_t)S * (WB + XB) + COMB + RECV;
    static_assert(S >= 3, "pipeline too shallow");
};

// One weight of a launch: the single call is a launch of one item; a grouped
// call (nxq_qmatmul_grouped: MoE experts, the projections that share an
// input) puts up to kMaxItems weights of one block type in one launch.
struct MmaItem {
    const uint8_t* w;  // tiled weight
    const void* x;     // [M][K]: f16, or (M <= 2) fp32 / bf16 rounded to f16 by the producer
    void* y;           // [M][N]
    int64_t N, K;
    int chunks;        // K chunks per row
    int M;
    int cluster0;      // first cluster of this item
    // Units: tile t's tile-chunks are units t kun .. t kun + kun - 1 (kun =
    // chunks; paired: twice that, the gate's then the up weight's).  C = 1:
    // CTA q of the item takes units [s(q), s(q + 1)), s(q) = gran (q ub +
    // min(q, ur)): whole tiles (gran = kun) or any run of units (gran = 1; a
    // tile shared by several CTAs is finished by the last of them).  C > 1:
    // cluster q owns tile q.
    int ub, ur, gran;
    const uint8_t* w_up;  // SwiGLU pairing: the up weight (same shape); y = silu(x W^T) * (x W_up^T)
    const float* res;     // residual [M][N] fp32 added to the result before the store, or null
};

struct MmaParams {
    MmaItem it[kMaxItems];
    int n_items;
    int x_dtype, y_dtype;
    int C;  // CTAs per cluster: the reduction is split C ways inside a cluster
    DeviceStatus* status;
    float* part;    // C = 1, gran = 1: a partial-sum slot per CTA
    unsigned* cnt;  // ... and a counter per CTA (zero between launches)
    TpExchange tp;  // tp.on: row-split tensor parallelism, partial tiles exchanged over peer memory
};

__device__ __forceinline__ void store_y(void* y, int dt, int64_t i, float v) {
    if (dt == NXQ_F32)
        reinterpret_cast<float*>(y)[i] = v;
    else if (dt == NXQ_F16)
        reinterpret_cast<__half*>(y)[i] = __float2half_rn(v);
    else
        reinterpret_cast<__nv_bfloat16*>(y)[i] = __float2bfloat16_rn(v);
}

// x piece (16 B) by cp.async; src_bytes = 0 fills the piece with zeros.
__device__ __forceinline__ void cp_async16_zfill(void* dst, const void* src, uint32_t src_bytes) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(smem_u32(dst)), "l"(src), "r"(src_bytes)
                 : "memory");
}
// Arrives (once, counted in the barrier's expected count) on `bar` when all
// cp.async this thread issued so far have landed.
__device__ __forceinline__ void cp_async_arrive(uint64_t* bar) {
    asm volatile("cp.async.mbarrier.arrive.noinc.shared::cta.b64 [%0];" ::"r"(smem_u32(bar)) : "memory");
}

// One CTA per SM: warps 0 .. 8G-1 are G consumer groups that take the CTA's
// units in turn (group = unit index mod G), the warps after them are producers
// (one for up to 8 tokens, else four; the first also issues the tile-chunk
// copies).  A CTA's units are consecutive tile-chunks in memory.  C = 1: the
// CTA takes a run of units (MmaItem), whole tiles or not; a tile it holds
// whole is written to y directly, a tile shared with other CTAs (stream-K)
// through partial sums in global memory: the sharers that hold its later
// units store their partials and count themselves in, and the one holding its
// first units (at the end of its run) waits for the counts, adds the partials
// in CTA order and writes y.  Every CTA of the launch fits on the GPU at once
// and publishes without waiting, so the wait ends once the later CTAs have
// run their first tile.  C > 1: the cluster owns one tile, CTA rank r takes chunks
// [r K/C, (r+1) K/C), and ranks 1..C-1 push their partial sums into rank 0's
// shared memory (one bulk copy each, completing on an mbarrier there), which
// adds them in rank order.  Either way the result does not depend on timing.
// LOOKUP = true: the CTA looks its item up from its cluster index, and the
// item's fields live in registers; false: a launch of one item, read at fixed
// offsets of the kernel parameters.  Grouped launches need the lookup; single
// ones use it too up to 16 tokens (measured 1-3 % faster there), but not at
// 32 tokens, where it is 4 % slower (registers at the 96 cap).
template <int TYPE, int MT, bool LOOKUP, bool PAIR = false, bool TPX = false>
__global__ void __launch_bounds__(Cfg<TYPE, MT, PAIR>::kAll, 1) mma_gemv_kernel(const MmaParams p) {
    using Cf = Cfg<TYPE, MT, PAIR>;
    constexpr int S = Cf::S, WB = Cf::WB, XB = Cf::XB, NT = Cf::NT, PB = Cf::PB;
    constexpr int kGroups = Cf::G, kConsumers = Cf::kConsumers, kAll = Cf::kAll, kXWarps = Cf::kXWarps;
    constexpr int RS = NT * 8;  // floats per row in a partial
    constexpr int kPre = S < 3 ? S : 3;  // tile-chunks requested before griddepcontrol.wait
    extern __shared__ __align__(128) uint8_t smem[];
    uint8_t* wst = smem;                                       // S x WB
    uint8_t* xst = smem + (size_t)S * WB;                      // S x XB
    float* comb = reinterpret_cast<float*>(xst + (size_t)S * XB);           // (G-1) x 2 x PB
    float* recv = reinterpret_cast<float*>(xst + (size_t)S * XB + Cf::COMB);  // (CMAX-1) x PB
    __shared__ uint64_t full[S];   // unit landed: tile-chunk bytes + one arrival per producer thread + 1
    __shared__ uint64_t empty[S];  // the 8 warps of the consuming group are done with the stage
    __shared__ uint64_t recv_full;  // cluster leader: the C-1 partials have landed
    __shared__ int s_abort;
    __shared__ int s_last;  // stream-K: the counts of the tile this CTA finishes are in

    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int g = lane >> 2, tq = lane & 3;
    const int C = p.C, rank = (int)(blockIdx.x % (unsigned)C), qg = (int)(blockIdx.x / (unsigned)C);
    int ii = 0;
    if (LOOKUP)
        for (int j = 1; j < p.n_items; ++j)
            if (qg >= p.it[j].cluster0) ii = j;
    const MmaItem& I = p.it[LOOKUP ? ii : 0];
    const int q = qg - I.cluster0;
    const int Kc = I.chunks;
    const int kun = PAIR ? 2 * Kc : Kc;  // units per tile
    // Start of CTA b's run (C = 1).
    auto run_start = [&](int b) { return I.gran * (b * I.ub + (b < I.ur ? b : I.ur)); };
    const int g0 = C == 1 ? run_start(q) : q * kun + rank * Kc / C;
    const int g1 = C == 1 ? run_start(q + 1) : q * kun + (rank + 1) * Kc / C;
    const int n = g1 - g0;  // this CTA's units: item units g0 .. g1 - 1
    const int64_t K = I.K, N = I.N;
    const int M = I.M;

    // Unit u is item unit g0 + u: without pairing, the tile-chunk at w_base + u WB.
    const uint8_t* const w_base = I.w + (int64_t)g0 * WB;
    auto w_issue = [&](int u, int stg) {
        const uint8_t* src = w_base + (int64_t)u * WB;
        if constexpr (PAIR) {  // chunk c of tile t: the gate's for c < Kc, the up weight's after
            const int g = g0 + u, t = g / kun, c = g - t * kun;
            src = (c < Kc ? I.w : I.w_up) + ((int64_t)t * Kc + (c < Kc ? c : c - Kc)) * WB;
        }
        ptx::mbar_arrive_expect_tx(&full[stg], WB);
        ptx::bulk_g2s(wst + stg * WB, src, WB, &full[stg]);
    };

    int w_issued = 0;  // producer lane 0: tile-chunk copies issued
    if (tid == kConsumers) {
        // Barriers first, then the first kPre units' weight copies: the
        // weights are immutable once registered, so they are requested before
        // griddepcontrol.wait (programmatic dependent launch, below) and
        // before the rest of the CTA has finished its set-up.  Units kPre ..
        // S - 1 are requested after their activations, which would otherwise
        // queue behind a full ring of weight copies (measured: kPre = 1 - 4
        // are 0.5 - 0.7 us per call faster than S; 3 is kept).
        for (int st = 0; st < S; ++st) {
            ptx::mbar_init(&full[st], 1 + 32 * kXWarps);
            ptx::mbar_init(&empty[st], kWarps);
        }
        ptx::mbar_init(&recv_full, 1);
        if (C > 1 && rank == 0)
            asm volatile("mbarrier.expect_tx.relaxed.cta.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(&recv_full)),
                         "r"((uint32_t)((C - 1) * PB))
                         : "memory");
        s_abort = 0;
        ptx::fence_mbar_init();
        for (; w_issued < (n < kPre ? n : kPre); ++w_issued) w_issue(w_issued, w_issued);
    }
    // Token slots at or beyond M are never loaded; zero them once so the
    // fragment loads need no predicate.
    for (int i = tid; i < S * XB / 16; i += kAll) reinterpret_cast<uint4*>(xst)[i] = make_uint4(0u, 0u, 0u, 0u);
    if (C > 1)
        cluster_sync();  // barriers initialised before any rank pushes to the leader
    else
        __syncthreads();
    const ptx::WaitCtl ctl{&s_abort, p.status};
    // Programmatic dependent launch: the next kernel of the stream may be
    // scheduled as soon as every CTA of this grid has started; this grid reads
    // x and writes y only after griddepcontrol.wait (the previous kernel has
    // completed and its memory is visible).
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");

    if (warp >= kGroups * kWarps) {
        // ---- producers: lane 0 of the first issues the tile-chunk bulk
        // copies; producer warp pw copies the x pieces of tokens 8pw..8pw+7:
        // piece (token, t4, m) holds the 8 elements x[token][k0 + 64 t4 + 8m ..]
        // at index ((token / 8) * 8 + m) * 32 + 4 (token % 8) + t4.  Every
        // producer thread arrives once per unit on the unit's full barrier,
        // after the stage's previous unit was released.
        const int pw = kXWarps == 1 ? 0 : warp - kGroups * kWarps;
        asm volatile("griddepcontrol.wait;" ::: "memory");
        // Refills stage u % S with unit u's tile-chunk once its consumers are
        // done with unit u - S (lane 0); false if the wait gave up.  Units
        // kPre .. S - 1 take a fresh stage with no wait.
        auto refill = [&](int u) {
            int ok = 1;
            if (u < S) {
                if (u >= kPre && lane == 0 && pw == 0) {
                    w_issue(u, u);
                    ++w_issued;
                }
            } else {
                const int stg = u % S;
                if (lane == 0) {
                    ok = ptx::mbar_wait(&empty[stg], (uint32_t)(u / S - 1) & 1u, ctl, 32) ? 1 : 0;
                    if (ok && pw == 0) {
                        w_issue(u, stg);
                        ++w_issued;
                    }
                }
                ok = __shfl_sync(0xFFFFFFFFu, ok, 0);
            }
            return ok != 0;
        };
        // Unit u reads the activations of chunk (g0 + u) mod Kc (kun is a multiple of Kc).
        auto chunk_k0 = [&](int u) { return (int64_t)((g0 + u) % Kc) * CHUNK_K; };
        if (p.x_dtype == NXQ_F16) {
            // Lane (t4, m) = ((lane >> 3) & 3, lane & 7) copies piece (token, t4,
            // m) of every token: one source row and one destination step apart.
            const __half* xh = static_cast<const __half*>(I.x);
            const int t4 = (lane >> 3) & 3, m = lane & 7;
            const int tok0 = 8 * pw, tok1 = M < tok0 + 8 ? M : tok0 + 8;
            for (int u = 0, c = g0 % Kc; u < n; ++u, c = c + 1 == Kc ? 0 : c + 1) {
                if (u >= S && !refill(u)) break;
                uint4* xd = reinterpret_cast<uint4*>(xst + (u % S) * XB) + m * 32 + t4;
                const int64_t k = (int64_t)c * CHUNK_K + 64 * t4 + 8 * m;
                const uint32_t bytes = k < K ? 16u : 0u;
                const __half* src = xh + (k < K ? k : 0) + (int64_t)tok0 * K;
                for (int tok = tok0; tok < tok1; ++tok, src += K)
                    cp_async16_zfill(xd + ((tok >> 3) << 8) + ((tok & 7) << 2), src, bytes);
                cp_async_arrive(&full[u % S]);
                if (u < S) refill(u);  // a first unit's weights not yet requested: after its x
            }
        } else {
            // fp32 / bf16 activations, M <= 2 (at most 2 pieces per lane):
            // loaded here and rounded to f16 as __float2half_rn does.  The
            // loads of unit u stay in flight over the next refill; unit u is
            // converted, stored and signalled in the next iteration.
            const bool f32 = p.x_dtype == NXQ_F32;
            float4 ra[2], rb[2];
            auto issue = [&](int u) {
                const int64_t k0 = chunk_k0(u);
#pragma unroll
                for (int j = 0; j < 2; ++j) {
                    const int i = lane + 32 * j;
                    const int tok = i >> 5, t4 = (i >> 3) & 3, m = i & 7;
                    const int64_t k = k0 + 64 * t4 + 8 * m;
                    ra[j] = rb[j] = make_float4(0.f, 0.f, 0.f, 0.f);
                    if (i < M * 32 && k < K) {
                        if (f32) {
                            const float4* src = reinterpret_cast<const float4*>(static_cast<const float*>(I.x) +
                                                                                (int64_t)tok * K + k);
                            ra[j] = __ldg(src);
                            rb[j] = __ldg(src + 1);
                        } else {
                            const uint4 q = __ldg(reinterpret_cast<const uint4*>(
                                static_cast<const __nv_bfloat16*>(I.x) + (int64_t)tok * K + k));
                            ra[j] = make_float4(__uint_as_float(q.x), __uint_as_float(q.y), __uint_as_float(q.z),
                                                __uint_as_float(q.w));
                        }
                    }
                }
            };
            // A finite activation beyond the f16 range is reported in the
            // status word (kStatusRange, where = 3) and still rounded (to inf).
            bool over = false;
            auto ovf2 = [&](float a, float b) { over |= f16_overflows(a) || f16_overflows(b); };
            auto bf2h = [&](uint32_t w) {
                const float2 f = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&w));
                ovf2(f.x, f.y);
                return h2u(__float22half2_rn(f));
            };
            auto finish = [&](int u) {
                uint4* xd = reinterpret_cast<uint4*>(xst + (u % S) * XB);
#pragma unroll
                for (int j = 0; j < 2; ++j) {
                    const int i = lane + 32 * j;
                    if (i >= M * 32) continue;
                    const int tok = i >> 5, t4 = (i >> 3) & 3, m = i & 7;
                    uint4 h;
                    if (f32) {
                        ovf2(ra[j].x, ra[j].y);
                        ovf2(ra[j].z, ra[j].w);
                        ovf2(rb[j].x, rb[j].y);
                        ovf2(rb[j].z, rb[j].w);
                        h = make_uint4(h2u(__floats2half2_rn(ra[j].x, ra[j].y)), h2u(__floats2half2_rn(ra[j].z, ra[j].w)),
                                       h2u(__floats2half2_rn(rb[j].x, rb[j].y)), h2u(__floats2half2_rn(rb[j].z, rb[j].w)));
                    } else {
                        h = make_uint4(bf2h(__float_as_uint(ra[j].x)), bf2h(__float_as_uint(ra[j].y)),
                                       bf2h(__float_as_uint(ra[j].z)), bf2h(__float_as_uint(ra[j].w)));
                    }
                    xd[((tok >> 3) * 8 + m) * 32 + 4 * (tok & 7) + t4] = h;
                }
                ptx::mbar_arrive(&full[u % S]);
            };
            int u = 0;
            if (pw == 0) {
                for (; u < n; ++u) {
                    if (!refill(u)) break;
                    if (u > 0) finish(u - 1);
                    issue(u);
                }
                if (u == n && n > 0) finish(n - 1);
                if (over) raise_range(p.status, 3u);
            } else {
                for (; u < n; ++u) {
                    if (!refill(u)) break;
                    ptx::mbar_arrive(&full[u % S]);
                }
            }
        }
    } else {
        // ---- consumers: of the units [cs, ce) that this CTA holds of tile t,
        // group gi takes c = cs + gi, cs + gi + G, ... ----
        asm volatile("griddepcontrol.wait;" ::: "memory");
        const int gi = warp >> 3, wg = warp & 7;
        const int r0 = 16 * wg + g;  // the fragment rows r0, r0 + 8 of a tile
        bool dead = false;
        // Row-split tensor parallelism (single C = 1 launches): this rank's
        // partial sums of a finished tile go to its slot in every rank's
        // exchange buffer as tagged words (remote stores over NVLink); the sum
        // over ranks is taken after the tile loop.  The epoch is stable for
        // the whole launch: the last CTA to finish advances it.
        unsigned long long tp_e = 0ull;
        if constexpr (TPX) tp_e = *reinterpret_cast<volatile unsigned long long*>(p.tp.ctl);
        const unsigned long long tp_tag = (tp_e + 1ull) << 32;
        int tp_n = 0, tp_tiles[TPX ? kTpxCtaTiles : 1];
        auto tp_slot = [&](int q, int src, int t) {
            return p.tp.recv[q] + ((size_t)(tp_e & 1ull) * p.tp.world + src) * kTpxSlotWords +
                   (size_t)t * TILE_ROWS * RS;
        };
        // Words of (row, tokens tok, tok + 1): both when tok + 1 < M, the first
        // when only tok < M, none past M or past the last row (writer and
        // reader use the same rule).
        auto tp_words = [&](int64_t row, int tok) { return row >= N || tok >= M ? 0 : tok + 1 < M ? 2 : 1; };
        auto tp_put = [&](unsigned long long* w, int n, float a, float b) {
            if (n == 2)
                asm volatile("st.relaxed.sys.global.v2.u64 [%0], {%1, %2};" ::"l"(w),
                             "l"(tp_tag | __float_as_uint(a)), "l"(tp_tag | __float_as_uint(b))
                             : "memory");
            else if (n == 1)
                asm volatile("st.relaxed.sys.global.u64 [%0], %1;" ::"l"(w), "l"(tp_tag | __float_as_uint(a))
                             : "memory");
        };
        // Stores a tile's sums A (PAIR: gate; AU: up): y = A, or silu(A) * AU,
        // plus the residual.
        auto store_vals = [&](int t, const auto& A, const auto& AU) {
            if constexpr (TPX) {
                for (int q = 0; q < p.tp.world; ++q) {
                    if (p.tp.owner && q != t % p.tp.world) continue;  // owner exchange: to tile t's owner only
                    unsigned long long* sl = tp_slot(q, p.tp.rank, t);
#pragma unroll
                    for (int nt = 0; nt < NT; ++nt) {
                        const int tok = 8 * nt + 2 * tq;
                        const int64_t row = (int64_t)t * TILE_ROWS + r0;
                        tp_put(sl + r0 * RS + tok, tp_words(row, tok), A[nt][0], A[nt][1]);
                        tp_put(sl + (r0 + 8) * RS + tok, tp_words(row + 8, tok), A[nt][2], A[nt][3]);
                    }
                }
                if (tp_n < kTpxCtaTiles) tp_tiles[tp_n++] = t;
                return;
            }
#pragma unroll
            for (int nt = 0; nt < NT; ++nt)
#pragma unroll
                for (int e = 0; e < 4; ++e) {
                    const int tok = 8 * nt + 2 * tq + (e & 1);
                    const int64_t row = (int64_t)t * TILE_ROWS + r0 + 8 * (e >> 1);
                    if (tok < M && row < N) {
                        float v = A[nt][e];
                        if constexpr (PAIR) v = v / (1.0f + expf(-v)) * AU[nt][e];
                        if (I.res) v += I.res[tok * N + row];
                        store_y(I.y, p.y_dtype, tok * N + row, v);
                    }
                }
        };
        // Stream-K (C = 1, runs that start or end inside a tile): CTAs b0 ..
        // b1 of the item hold units of tile t.  b0, which holds the tile's
        // first units, reaches it at the end of its run and finishes it; b0 + 1
        // .. b1 reach it at the start of their runs (or hold runs inside it)
        // and publish their partials: each one the partial of the tile its
        // run starts in (its only one) and a count on b0's counter (no other
        // shared tile starts inside b0's run).
        auto cta_of = [&](int gu) {
            const int big = I.ur * (I.ub + 1);
            return gu < big ? gu / (I.ub + 1) : I.ur + (gu - big) / I.ub;
        };
        auto part_of = [&](int b) { return p.part + (size_t)(I.cluster0 + b) * (Cf::SETS * PB / 4); };
        for (int t = g0 / kun; t * kun < g1; ++t) {
            const int cs = g0 > t * kun ? g0 - t * kun : 0;
            const int ce = g1 < (t + 1) * kun ? g1 - t * kun : kun;
            // acc[n8 token tile][c0..c3]: c0/c1 = row 16wg+g, tokens 8nt+2t,
            // 8nt+2t+1; c2/c3 = row 16wg+8+g.
            // PAIR: accu/accu2 hold the up projection's sums.
            float acc[NT][4], acc2[Cf::kAccSets == 2 ? NT : 1][4];
            float accu[PAIR ? NT : 1][4], accu2[(PAIR && Cf::kAccSets == 2) ? NT : 1][4];
            auto zero = [](auto& A) {
#pragma unroll
                for (int i = 0; i < (int)(sizeof(A) / sizeof(A[0])); ++i)
#pragma unroll
                    for (int e = 0; e < 4; ++e) A[i][e] = 0.0f;
            };
            zero(acc);
            if constexpr (Cf::kAccSets == 2) zero(acc2);
            if constexpr (PAIR) {
                zero(accu);
                if constexpr (Cf::kAccSets == 2) zero(accu2);
            }
            // Unit c of this tile into the sums A (A2: the second chain).
            auto unit = [&](int c, auto& A, auto& A2) {
                const int u = t * kun + c - g0, stg = u % S;
                if (!dead && !ptx::mbar_wait(&full[stg], (uint32_t)(u / S) & 1u, ctl, 31)) dead = true;
                if (!dead) {
                    Lane<TYPE> LA, LB;
                    LA.load(wst + stg * WB, 16 * wg + g, tq);
                    LB.load(wst + stg * WB, 16 * wg + 8 + g, tq);
                    const uint4* xs = reinterpret_cast<const uint4*>(xst + stg * XB) + lane;
#pragma unroll
                    for (int m = 0; m < 8; ++m) {
                        uint32_t pa[4], pb[4];
                        LA.pairs(m, pa);
                        LB.pairs(m, pb);
#pragma unroll
                        for (int nt = 0; nt < NT; ++nt) {
                            const uint4 xv = xs[(nt * 8 + m) * 32];
                            mma16816(A[nt], pa[0], pb[0], pa[1], pb[1], xv.x, xv.y);
                            if constexpr (Cf::kAccSets == 2)
                                mma16816(A2[nt], pa[2], pb[2], pa[3], pb[3], xv.z, xv.w);
                            else
                                mma16816(A[nt], pa[2], pb[2], pa[3], pb[3], xv.z, xv.w);
                        }
                    }
                }
                __syncwarp();
                if (lane == 0) ptx::mbar_arrive(&empty[stg]);
            };
            int c = cs + gi;
            for (; c < (ce < Kc ? ce : Kc); c += kGroups) unit(c, acc, acc2);
            if constexpr (PAIR)
                for (; c < ce; c += kGroups) unit(c, accu, accu2);
            auto fold = [](auto& A, auto& A2) {
#pragma unroll
                for (int nt = 0; nt < NT; ++nt)
#pragma unroll
                    for (int e = 0; e < 4; ++e) A[nt][e] += A2[nt][e];
            };
            if constexpr (Cf::kAccSets == 2) {
                fold(acc, acc2);
                if constexpr (PAIR) fold(accu, accu2);
            }
            // ---- tile end: groups 1.. hand their partials to group 0 ----
            auto slot = [&](int gg, int set) { return comb + (((gg - 1) * 2 + (t & 1)) * Cf::SETS + set) * (PB / 4); };
            auto put = [&](float* cb, auto& A) {
#pragma unroll
                for (int nt = 0; nt < NT; ++nt) {
                    *reinterpret_cast<float2*>(cb + r0 * RS + 8 * nt + 2 * tq) = make_float2(A[nt][0], A[nt][1]);
                    *reinterpret_cast<float2*>(cb + (r0 + 8) * RS + 8 * nt + 2 * tq) = make_float2(A[nt][2], A[nt][3]);
                }
            };
            auto add = [&](const float* cb, auto& A) {
#pragma unroll
                for (int nt = 0; nt < NT; ++nt) {
                    const float2 a = *reinterpret_cast<const float2*>(cb + r0 * RS + 8 * nt + 2 * tq);
                    const float2 b = *reinterpret_cast<const float2*>(cb + (r0 + 8) * RS + 8 * nt + 2 * tq);
                    A[nt][0] += a.x;
                    A[nt][1] += a.y;
                    A[nt][2] += b.x;
                    A[nt][3] += b.y;
                }
            };
            if (gi > 0) {
                put(slot(gi, 0), acc);
                if constexpr (PAIR) put(slot(gi, 1), accu);
            }
            named_sync(1, kConsumers);
            if (gi > 0) continue;
            for (int gg = 1; gg < kGroups; ++gg) {
                add(slot(gg, 0), acc);
                if constexpr (PAIR) add(slot(gg, 1), accu);
            }
            if (C == 1 && cs == 0 && ce == kun) {
                store_vals(t, acc, accu);
            } else if (C == 1) {
                const int b0 = cta_of(t * kun), b1 = cta_of(t * kun + kun - 1);
                unsigned* cn = p.cnt + I.cluster0 + b0;
                if (q != b0) {
                    float* mine = part_of(q);
                    put(mine, acc);
                    if constexpr (PAIR) put(mine + PB / 4, accu);
                    named_sync(3, kThreads);
                    if (tid == 0) {
                        __threadfence();  // the group's partial (ordered by the barrier) before the count
                        const unsigned hooks = *reinterpret_cast<const volatile unsigned*>(&p.status->hooks);
                        if (!(hooks & kHookStreamKSkipCount)) atomicAdd(cn, 1u);
                    }
                } else {
                    // Wait (bounded) for the b1 - b0 counts, then add the
                    // partials in CTA order, this CTA's first: the same sum
                    // whatever the timing.
                    if (tid == 0) {
                        const unsigned need = (unsigned)(b1 - b0);
                        const long long w0 = clock64(), lim = ptx::wait_limit(p.status);
                        int ok = 1;
                        for (;;) {
                            unsigned v;
                            asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(cn) : "memory");
                            if (v >= need) break;
                            if (*ctl.abort || clock64() - w0 > lim) {
                                if (!*ctl.abort) ptx::raise_timeout(ctl, 34);
                                ok = 0;
                                break;
                            }
                            __nanosleep(64);
                        }
                        if (ok) *cn = 0u;  // every count is in: ready for the next launch
                        s_last = ok;
                    }
                    named_sync(3, kThreads);
                    if (s_last) {
                        auto add_l2 = [&](const float* cb, auto& A) {
#pragma unroll
                            for (int nt = 0; nt < NT; ++nt) {
                                const float2 a = __ldcg(reinterpret_cast<const float2*>(cb + r0 * RS + 8 * nt + 2 * tq));
                                const float2 b = __ldcg(reinterpret_cast<const float2*>(cb + (r0 + 8) * RS + 8 * nt + 2 * tq));
                                A[nt][0] += a.x;
                                A[nt][1] += a.y;
                                A[nt][2] += b.x;
                                A[nt][3] += b.y;
                            }
                        };
                        for (int b = b0 + 1; b <= b1; ++b) {
                            const float* pb = part_of(b);
                            add_l2(pb, acc);
                            if constexpr (PAIR) add_l2(pb + PB / 4, accu);
                        }
                        store_vals(t, acc, accu);
                    }
                }
            } else if (rank > 0) {
                // Push this rank's partial to the leader: stage memory is free
                // now (every unit has been consumed), so it holds the copy source.
                float* send = reinterpret_cast<float*>(smem);
#pragma unroll
                for (int nt = 0; nt < NT; ++nt) {
                    *reinterpret_cast<float2*>(send + r0 * RS + 8 * nt + 2 * tq) = make_float2(acc[nt][0], acc[nt][1]);
                    *reinterpret_cast<float2*>(send + (r0 + 8) * RS + 8 * nt + 2 * tq) = make_float2(acc[nt][2], acc[nt][3]);
                }
                asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
                named_sync(2, kThreads);
                if (tid == 0 && !s_abort) {
                    const uint32_t dst = cluster_addr(recv + (size_t)(rank - 1) * (PB / 4), 0);
                    const uint32_t bar = cluster_addr(&recv_full, 0);
                    asm volatile(
                        "cp.async.bulk.shared::cluster.shared::cta.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
                            dst),
                        "r"(smem_u32(send)), "r"((uint32_t)PB), "r"(bar)
                        : "memory");
                    asm volatile("cp.async.bulk.commit_group;" ::: "memory");
                    asm volatile("cp.async.bulk.wait_group.read 0;" ::: "memory");
                }
            } else {
                // Leader: add the other ranks' partials in rank order.
                if (tid == 0) ptx::mbar_arrive(&recv_full);
                // Waits even after an abort (bounded), so that no rank's copy
                // lands in shared memory that has gone away.
                bool ok = ptx::mbar_try_wait(&recv_full, 0);
                const long long t0 = clock64();
                while (!ok && clock64() - t0 < ptx::kWaitCycles) ok = ptx::mbar_try_wait(&recv_full, 0);
                if (!ok && lane == 0) ptx::raise_timeout(ctl, 33);
                if (ok && !s_abort) {
                    for (int rr = 1; rr < C; ++rr) {
                        const float* src = recv + (size_t)(rr - 1) * (PB / 4);
#pragma unroll
                        for (int nt = 0; nt < NT; ++nt) {
                            const float2 a = *reinterpret_cast<const float2*>(src + r0 * RS + 8 * nt + 2 * tq);
                            const float2 b = *reinterpret_cast<const float2*>(src + (r0 + 8) * RS + 8 * nt + 2 * tq);
                            acc[nt][0] += a.x;
                            acc[nt][1] += a.y;
                            acc[nt][2] += b.x;
                            acc[nt][3] += b.y;
                        }
                    }
                    store_vals(t, acc, accu);
                }
            }
        }
        if (TPX && gi == 0 && !s_abort) {
            // ---- the exchange: group 0 held every tile this CTA finished.
            // Each thread reads back its own fragment positions of every
            // rank's slot in this rank's buffer, spinning (bounded) on each
            // word until it carries this launch's tag, and adds the ranks in
            // rank order (the same bits on every rank).  No fence or flag: a
            // word and its tag travel in one 8-byte store (measured: per-tile
            // flags behind a system-scope fence cost about 12 us per call). ----
            const long long w0 = clock64(), lim = ptx::wait_limit(p.status);
            bool ok = true;
            auto tp_get = [&](const unsigned long long* w, int n, float& a, float& b) {
                if (n == 0) return;
                unsigned long long u, v = tp_tag;
                for (;;) {
                    if (n == 2)
                        asm volatile("ld.relaxed.sys.global.v2.u64 {%0, %1}, [%2];" : "=l"(u), "=l"(v) : "l"(w) : "memory");
                    else
                        asm volatile("ld.relaxed.sys.global.u64 %0, [%1];" : "=l"(u) : "l"(w) : "memory");
                    if ((u & ~0xFFFFFFFFull) == tp_tag && (v & ~0xFFFFFFFFull) == tp_tag) break;
                    if (*ctl.abort || clock64() - w0 > lim) {
                        if (!*ctl.abort) ptx::raise_timeout(ctl, 35);
                        ok = false;
                        return;
                    }
                    __nanosleep(32);
                }
                a += __uint_as_float((unsigned)u);
                if (n == 2) b += __uint_as_float((unsigned)v);
            };
            // All-to-all exchange: every rank sums every tile it finished.
            // Owner exchange (tile t owned by rank t mod world): the owner sums
            // the ranks' partials of its tiles and sends the sum to the other
            // ranks' slot (owner, t); the others store that sum.  Owned tiles
            // go first, so that the sums leave as early as they can.
            const int W = p.tp.world, me = p.tp.rank;
            for (int pass = 0; pass < (p.tp.owner ? 2 : 1) && ok; ++pass)
                for (int i = 0; i < tp_n && ok; ++i) {
                    const int t = tp_tiles[i], o = t % W;
                    if (p.tp.owner && (pass == 0) != (o == me)) continue;
                    const bool sums = !p.tp.owner || o == me;
#pragma unroll
                    for (int nt = 0; nt < NT; ++nt) {
                        float v[4] = {0.0f, 0.0f, 0.0f, 0.0f};
                        const int tok = 8 * nt + 2 * tq;
                        const int64_t row = (int64_t)t * TILE_ROWS + r0;
                        const int n0 = tp_words(row, tok), n1 = tp_words(row + 8, tok);
                        for (int src = sums ? 0 : o; src < (sums ? W : o + 1) && ok; ++src) {
                            const unsigned long long* sl = tp_slot(me, src, t);
                            tp_get(sl + r0 * RS + tok, n0, v[0], v[1]);
                            tp_get(sl + (r0 + 8) * RS + tok, n1, v[2], v[3]);
                        }
                        if (!ok) break;
                        if (p.tp.owner && sums)
                            for (int q = 0; q < W; ++q)
                                if (q != me) {
                                    unsigned long long* sl = tp_slot(q, me, t);
                                    tp_put(sl + r0 * RS + tok, n0, v[0], v[1]);
                                    tp_put(sl + (r0 + 8) * RS + tok, n1, v[2], v[3]);
                                }
#pragma unroll
                        for (int e = 0; e < 4; ++e) {
                            const int tk = tok + (e & 1);
                            const int64_t rw = row + 8 * (e >> 1);
                            if (tk < M && rw < N) store_y(I.y, p.y_dtype, tk * N + rw, v[e]);
                        }
                    }
                }
        }
    }

    __syncthreads();
    if (TPX && tid == 0) {
        // The last CTA of the launch advances the exchange epoch (every CTA
        // read it at its start).
        __threadfence();
        unsigned int* done = reinterpret_cast<unsigned int*>(p.tp.ctl + 1);
        if (atomicAdd(done, 1u) == gridDim.x - 1) {
            *reinterpret_cast<volatile unsigned int*>(done) = 0u;
            __threadfence();
            volatile unsigned long long* ep = reinterpret_cast<volatile unsigned long long*>(p.tp.ctl);
            *ep = *ep + 1ull;  // no other CTA writes it during the launch
        }
    }
    if (s_abort) {
        // Let the copies still in flight land (bounded) before the CTA's shared
        // memory goes away: only the last S tile-chunks issued can be pending.
        cp_wait<0>();
        if (tid == kConsumers) {
            for (int u = w_issued > S ? w_issued - S : 0; u < w_issued; ++u) {
                const long long t0 = clock64();
                while (!ptx::mbar_try_wait(&full[u % S], (uint32_t)(u / S) & 1u) && clock64() - t0 < ptx::kWaitCycles) {
                }
            }
        }
    }
}

bool g_mma_enabled = true;
bool g_streamk = true;  // NXQ_GEMV_SPLIT=tiles: whole tiles and clusters only
int g_sm_count = 0;

// How many clusters of 2, 4, 8 CTAs of a variant fit on the GPU at once
// (index log2 C); a split never launches more, so it runs in one wave.
template <int TYPE, int MT>
int* max_clusters() {
    static int q[4] = {0, 0, 0, 0};
    return q;
}

template <int TYPE, int MT>
int set_attr() {
    using Cf = Cfg<TYPE, MT>;
    cudaError_t e = cudaFuncSetAttribute(mma_gemv_kernel<TYPE, MT, false>,
                                         cudaFuncAttributeMaxDynamicSharedMemorySize, (int)Cf::smem);
    if (e == cudaSuccess)
        e = cudaFuncSetAttribute(mma_gemv_kernel<TYPE, MT, true>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                 (int)Cf::smem);
    if (e == cudaSuccess)
        e = cudaFuncSetAttribute(mma_gemv_kernel<TYPE, MT, false, true>,
                                 cudaFuncAttributeMaxDynamicSharedMemorySize, (int)Cfg<TYPE, MT, true>::smem);
    if (e == cudaSuccess)
        e = cudaFuncSetAttribute(mma_gemv_kernel<TYPE, MT, false, false, true>,
                                 cudaFuncAttributeMaxDynamicSharedMemorySize, (int)Cf::smem);
    if (e != cudaSuccess) return cuda_fail(e, "cudaFuncSetAttribute (mma_gemv)");
    int* mq = max_clusters<TYPE, MT>();
    mq[0] = g_sm_count;
    for (int lc = 1, c = 2; c <= Cf::CMAX; ++lc, c *= 2) {
        cudaLaunchConfig_t cfg = {};
        cfg.gridDim = dim3((unsigned)(c * 64));
        cfg.blockDim = dim3(Cf::kAll);
        cfg.dynamicSmemBytes = Cf::smem;
        cudaLaunchAttribute attr;
        attr.id = cudaLaunchAttributeClusterDimension;
        attr.val.clusterDim.x = (unsigned)c;
        attr.val.clusterDim.y = 1;
        attr.val.clusterDim.z = 1;
        cfg.attrs = &attr;
        cfg.numAttrs = 1;
        int nq = 0;
        e = cudaOccupancyMaxActiveClusters(&nq, mma_gemv_kernel<TYPE, MT, false>, &cfg);
        if (e != cudaSuccess) return cuda_fail(e, "cudaOccupancyMaxActiveClusters (mma_gemv)");
        mq[lc] = nq;
    }
    return NXQ_OK;
}

// One weight of a launch as the host sees it.
struct HostItem {
    const Weight* w;
    const void* x;
    void* y;
    int64_t M;
    const Weight* w_up = nullptr;  // SwiGLU pairing (launches of one item)
    const float* res = nullptr;    // residual added before the store
};

// Work split of a launch, one of three kinds, with at most as many clusters
// in all as fit on the GPU at once (one wave):
//   whole tiles: C = 1, item i's Q_i CTAs own floor or ceil of T_i / Q_i tiles
//     each; the SMs go one at a time to the item whose CTAs have the most
//     units (so a lone weight gets min(T, SMs) CTAs);
//   clusters: C > 1 CTAs per tile, K cut C ways (the same C for every item;
//     only when all items together have few enough tiles);
//   stream-K (when sk_margin >= 0): C = 1, item i's Q_i CTAs take equal runs
//     of its T_i kun_i units, tiles shared between CTAs finished through
//     partial sums in global memory; the SMs go to the item with the longest
//     runs.
// Picks the fewest units on the busiest CTA, ties to whole tiles, then to the
// smallest C; stream-K only when its busiest CTA has more than sk_margin units
// fewer (its shared tiles cost a wait at the end of a run, and no SM is left
// for the next launch to start on early).  Returns the number of clusters.
int pick_split(const HostItem* it, int n, const int* maxq, int cmax, int sk_margin, MmaParams* p) {
    int64_t T[kMaxItems], Kc[kMaxItems], q[kMaxItems], qs[kMaxItems], sumT = 0, minKc = INT64_MAX;
    for (int i = 0; i < n; ++i) {
        T[i] = it[i].w->shape.tiles;
        Kc[i] = it[i].w->shape.chunks * (it[i].w_up ? 2 : 1);  // a paired tile is two tiles' units
        q[i] = qs[i] = 1;
        sumT += T[i];
        if (Kc[i] < minKc) minKc = Kc[i];
    }
    auto cost1 = [&](int i) { return ((T[i] + q[i] - 1) / q[i]) * Kc[i]; };
    for (int64_t used = n; used < g_sm_count; ++used) {
        int bi = -1;
        for (int i = 0; i < n; ++i)
            if (q[i] < T[i] && (bi < 0 || cost1(i) > cost1(bi))) bi = i;
        if (bi < 0) break;
        ++q[bi];
    }
    int64_t best = 0;
    for (int i = 0; i < n; ++i) best = cost1(i) > best ? cost1(i) : best;
    int best_c = 1;
    for (int lc = 1, c = 2; c <= cmax && c <= minKc; ++lc, c *= 2) {
        const int64_t qmax = g_sm_count / c < maxq[lc] ? g_sm_count / c : maxq[lc];
        if (sumT > qmax) continue;
        int64_t cost = 0;
        for (int i = 0; i < n; ++i) cost = (Kc[i] + c - 1) / c > cost ? (Kc[i] + c - 1) / c : cost;
        if (cost < best) {
            best = cost;
            best_c = c;
        }
    }
    bool sk = false;
    if (sk_margin >= 0) {
        auto cost_sk = [&](int i) { return (T[i] * Kc[i] + qs[i] - 1) / qs[i]; };
        for (int64_t used = n; used < g_sm_count; ++used) {
            int bi = -1;
            for (int i = 0; i < n; ++i)
                if (qs[i] < T[i] * Kc[i] && (bi < 0 || cost_sk(i) > cost_sk(bi))) bi = i;
            if (bi < 0) break;
            ++qs[bi];
        }
        int64_t cost = 0;
        for (int i = 0; i < n; ++i) cost = cost_sk(i) > cost ? cost_sk(i) : cost;
        if (cost + sk_margin < best) {
            sk = true;
            best_c = 1;
        }
    }
    p->C = best_c;
    p->n_items = n;
    int cl = 0;
    for (int i = 0; i < n; ++i) {
        const int64_t qi = sk ? qs[i] : best_c == 1 ? q[i] : T[i];
        MmaItem& m = p->it[i];
        m.w = it[i].w->dev;
        m.x = it[i].x;
        m.y = it[i].y;
        m.N = it[i].w->shape.N;
        m.K = it[i].w->shape.K;
        m.chunks = (int)it[i].w->shape.chunks;
        m.M = (int)it[i].M;
        m.cluster0 = cl;
        const int64_t units = sk ? T[i] * Kc[i] : T[i];
        m.gran = sk ? 1 : (int)Kc[i];
        m.ub = best_c == 1 ? (int)(units / qi) : 0;
        m.ur = best_c == 1 ? (int)(units % qi) : 0;
        m.w_up = it[i].w_up ? it[i].w_up->dev : nullptr;
        m.res = it[i].res;
        cl += (int)qi;
    }
    for (int i = n; i < kMaxItems; ++i) p->it[i] = MmaItem{};
    return cl;
}

// tp: row-split tensor parallelism with the partial tiles exchanged over peer
// memory inside the launch (one item, no pairing, no residual); the split is
// then C = 1 only, and a CTA may finish at most kTpxCtaTiles tiles.
template <int TYPE, int MT, bool PAIR = false>
int launch(const HostItem* it, int n, int x_dtype, int y_dtype, cudaStream_t st, const TpExchange* tp = nullptr) {
    using Cf = Cfg<TYPE, MT, PAIR>;
    MmaParams p;
    p.tp = TpExchange{};
    if (tp) {
        if (PAIR || n != 1 || it[0].res || it[0].w->shape.tiles > kTpxMaxTiles) return NXQ_ERR_UNSUPPORTED;
        p.tp = *tp;
    }
    for (int i = 0; i < n; ++i)
        if (it[i].w->shape.tile_chunk_bytes != Cf::WB)
            return fail(NXQ_ERR_SHAPE, "mma_gemv: tile-chunk of %lld bytes, kernel stage %d",
                        (long long)it[i].w->shape.tile_chunk_bytes, Cf::WB);
    // Stream-K partials: a slot of up to two result sets of 32 tokens per CTA,
    // one counter per CTA; sized once for every variant.  While the stream
    // is captured into a graph and its scratch is still too small, the launch
    // splits by whole tiles or clusters instead.
    StreamScratch* sc = nullptr;
    if (g_streamk) {
        const size_t slots = (size_t)g_sm_count * 2 * kMaxMT * TILE_ROWS;
        if (int rc = scratch_try(st, slots, (size_t)g_sm_count, &sc)) return rc;
    }
    // Measured (Q4_K, Q3_K, 4096 - 16384 rows): stream-K pays when it takes
    // more than 2 units off the busiest CTA at 8 tokens, 1 at 16, any at 32.
    const int margin = sc == nullptr ? -1 : MT == 8 ? 2 : MT == 16 ? 1 : 0;
    const int clusters = pick_split(it, n, max_clusters<TYPE, MT>(), tp ? 1 : Cf::CMAX, margin, &p);
    if (tp) {
        const MmaItem& m = p.it[0];
        const int kun = m.chunks;
        const int run = m.ub + (m.ur ? 1 : 0);  // tiles (whole-tile split) or units (stream-K) per CTA
        const int held = m.gran == kun ? run : (run + kun - 1) / kun + 1;
        if (p.C != 1 || held > kTpxCtaTiles) return NXQ_ERR_UNSUPPORTED;
    }
    p.part = sc ? sc->ws : nullptr;
    p.cnt = sc ? sc->counters : nullptr;
    p.x_dtype = x_dtype;
    p.y_dtype = y_dtype;
    p.status = context_status();
    // Launched with programmatic stream serialization (see the kernel's
    // griddepcontrol.wait): it may start while the previous kernel drains.
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3((unsigned)(clusters * p.C));
    cfg.blockDim = dim3(Cf::kAll);
    cfg.dynamicSmemBytes = Cf::smem;
    cfg.stream = st;
    cudaLaunchAttribute attr[2];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    attr[1].id = cudaLaunchAttributeClusterDimension;
    attr[1].val.clusterDim.x = (unsigned)p.C;
    attr[1].val.clusterDim.y = 1;
    attr[1].val.clusterDim.z = 1;
    cfg.attrs = attr;
    cfg.numAttrs = p.C > 1 ? 2 : 1;
    cudaError_t e = PAIR ? cudaLaunchKernelEx(&cfg, mma_gemv_kernel<TYPE, MT, false, true>, p)
                    : tp ? cudaLaunchKernelEx(&cfg, mma_gemv_kernel<TYPE, MT, false, false, true>, p)
                    : (n == 1 && MT == 32) ? cudaLaunchKernelEx(&cfg, mma_gemv_kernel<TYPE, MT, false>, p)
                                           : cudaLaunchKernelEx(&cfg, mma_gemv_kernel<TYPE, MT, true>, p);
    note_launches(1);
    if (e != cudaSuccess) return cuda_fail(e, "mma_gemv launch");
    return NXQ_OK;
}

// NXF INT8 weights are tiled as Q8_0 records and run on its kernels.
bool type_ok(int type) {
    return type == T_Q4_K || type == T_Q4_0 || type == T_Q8_0 || type == T_Q3_K || type == T_Q6_K ||
           type == T_Q5_K || type == T_Q4_1 || type == T_Q2_K || is_i4g(type) || type == T_NXF_I8;
}

int launch_items(int type, int mt, const HostItem* it, int n, int x_dtype, int y_dtype, cudaStream_t st,
                 const TpExchange* tp = nullptr) {
    const bool pair = n == 1 && it[0].w_up;
#define NXQ_CASE(T)                                                                                   \
    case T:                                                                                           \
        if (pair)                                                                                     \
            return mt == 8    ? launch<T, 8, true>(it, n, x_dtype, y_dtype, st)                       \
                   : mt == 16 ? launch<T, 16, true>(it, n, x_dtype, y_dtype, st)                      \
                              : launch<T, 32, true>(it, n, x_dtype, y_dtype, st);                     \
        return mt == 8    ? launch<T, 8>(it, n, x_dtype, y_dtype, st, tp)                             \
               : mt == 16 ? launch<T, 16>(it, n, x_dtype, y_dtype, st, tp)                            \
                          : launch<T, 32>(it, n, x_dtype, y_dtype, st, tp);
    switch (type) {
        NXQ_CASE(T_Q4_K)
        NXQ_CASE(T_Q4_0)
        case T_NXF_I8:
        NXQ_CASE(T_Q8_0)
        NXQ_CASE(T_Q3_K)
        NXQ_CASE(T_I4G128)
        NXQ_CASE(T_Q6_K)
        NXQ_CASE(T_Q5_K)
        NXQ_CASE(T_Q4_1)
        NXQ_CASE(T_Q2_K)
        NXQ_CASE(T_I4G32)
        NXQ_CASE(T_I4G64)
        NXQ_CASE(T_I4G256)
        default:
            return NXQ_ERR_UNSUPPORTED;
    }
#undef NXQ_CASE
}

}  // namespace

int mma_init(int) {
    const char* env = getenv("NXQ_DECODE_KERNEL");
    g_mma_enabled = !(env && env[0] == 's');  // "simt" selects the exact CUDA-core kernel
    const char* split = getenv("NXQ_GEMV_SPLIT");
    g_streamk = !(split && strcmp(split, "tiles") == 0);
    g_sm_count = context_sm_count();
    int rc;
#define NXQ_ATTR(T)                                       \
    if ((rc = set_attr<T, 8>()) != NXQ_OK) return rc;  \
    if ((rc = set_attr<T, 16>()) != NXQ_OK) return rc; \
    if ((rc = set_attr<T, 32>()) != NXQ_OK) return rc;
    NXQ_ATTR(T_Q4_K)
    NXQ_ATTR(T_Q4_0)
    NXQ_ATTR(T_Q8_0)
    NXQ_ATTR(T_Q3_K)
    NXQ_ATTR(T_I4G128)
    NXQ_ATTR(T_Q6_K)
    NXQ_ATTR(T_Q5_K)
    NXQ_ATTR(T_Q4_1)
    NXQ_ATTR(T_Q2_K)
    NXQ_ATTR(T_I4G32)
    NXQ_ATTR(T_I4G64)
    NXQ_ATTR(T_I4G256)
#undef NXQ_ATTR
    return NXQ_OK;
}

bool mma_supported(const TiledShape& s, int64_t M) {
    return g_mma_enabled && type_ok(s.type) && M >= 1 && M <= kMaxMT;
}

void mma_kernel_name(const TiledShape& s, int64_t M, char* buf, size_t n) {
    snprintf(buf, n, "mma_gemv<%s,m%d>", type_name(s.type), M <= 8 ? 8 : M <= 16 ? 16 : 32);
}

int mma_qmatmul(const Weight* w, const void* x, int x_dtype, void* y, int y_dtype, int64_t M, cudaStream_t st,
                const float* res) {
    const TiledShape& s = w->shape;
    if (!mma_supported(s, M)) return NXQ_ERR_UNSUPPORTED;
    const int mt = M <= 8 ? 8 : M <= 16 ? 16 : 32;
    // f16 activations are read as they are; fp32 / bf16 ones are rounded to
    // f16 by the kernel's producer when M <= 2, else by a conversion kernel.
    const bool aligned = ((uintptr_t)x % 16) == 0;
    const bool direct = aligned && (x_dtype == NXQ_F16 || (M <= 2 && (x_dtype == NXQ_F32 || x_dtype == NXQ_BF16)));
    const void* xh = x;
    int xdt = x_dtype;
    if (!direct) {
        StreamScratch* sc = nullptr;
        int rc = scratch_for(st, 0, 0, (size_t)(M * s.K), &sc);
        if (rc) return rc;
        cudaError_t e = launch_to_half(x, x_dtype, sc->xh, M * s.K, st);
        if (e != cudaSuccess) return cuda_fail(e, "to_half launch");
        xh = sc->xh;
        xdt = NXQ_F16;
    }
    HostItem item{w, xh, y, M};
    item.res = res;
    return launch_items(s.type, mt, &item, 1, xdt, y_dtype, st);
}

int mma_qmatmul_tp(const Weight* w, const void* x, int x_dtype, float* y, int64_t M, cudaStream_t st,
                   const TpExchange& tp) {
    const TiledShape& s = w->shape;
    if (!mma_supported(s, M) || !tp.on) return NXQ_ERR_UNSUPPORTED;
    // Words a rank sends: all-to-all, its whole partial to every peer; owner
    // exchange, 1/world of the tiles out and back to each peer.  Beyond
    // kTpxMaxBytes a bandwidth-bound exchange loses to NCCL's allreduce.
    const int64_t words = (int64_t)(tp.world - 1) * s.N * M;
    const int64_t bytes = (tp.owner ? 2 * words / tp.world : words) * (int64_t)sizeof(unsigned long long);
    if (bytes > kTpxMaxBytes) return NXQ_ERR_UNSUPPORTED;
    const int mt = M <= 8 ? 8 : M <= 16 ? 16 : 32;
    const bool aligned = ((uintptr_t)x % 16) == 0;
    const bool direct = aligned && (x_dtype == NXQ_F16 || (M <= 2 && (x_dtype == NXQ_F32 || x_dtype == NXQ_BF16)));
    const void* xh = x;
    int xdt = x_dtype;
    if (!direct) {
        StreamScratch* sc = nullptr;
        int rc = scratch_for(st, 0, 0, (size_t)(M * s.K), &sc);
        if (rc) return rc;
        cudaError_t e = launch_to_half(x, x_dtype, sc->xh, M * s.K, st);
        if (e != cudaSuccess) return cuda_fail(e, "to_half launch");
        xh = sc->xh;
        xdt = NXQ_F16;
    }
    HostItem item{w, xh, y, M};
    return launch_items(s.type, mt, &item, 1, xdt, NXQ_F32, st, &tp);
}

int mma_qmatmul_swiglu(const Weight* wg, const Weight* wu, const void* x, int x_dtype, void* h, int h_dtype,
                       int64_t M, cudaStream_t st) {
    const TiledShape& s = wg->shape;
    const TiledShape& su = wu->shape;
    const bool aligned = ((uintptr_t)x % 16) == 0;
    const bool direct = aligned && (x_dtype == NXQ_F16 || (M <= 2 && (x_dtype == NXQ_F32 || x_dtype == NXQ_BF16)));
    // Pairing has no cluster split: without stream-K it is worth it only when
    // the weight has tiles for at least half the SMs.
    if (!mma_supported(s, M) || !direct || su.type != s.type || su.N != s.N || su.K != s.K ||
        (!g_streamk && s.tiles * 2 < g_sm_count))
        return NXQ_ERR_UNSUPPORTED;
    const int mt = M <= 8 ? 8 : M <= 16 ? 16 : 32;
    HostItem item{wg, x, h, M};
    item.w_up = wu;
    return launch_items(s.type, mt, &item, 1, x_dtype, h_dtype, st);
}

int mma_qmatmul_grouped(const Weight* const* w, int n, const void* const* x, int x_dtype, void* const* y,
                        int y_dtype, const int64_t* M, cudaStream_t st) {
    HostItem items[kMaxItems];
    int type = -1, k = 0;
    int64_t mmax = 0;
    // Every item must be one the kernel reads as it is (no conversion pass).
    for (int i = 0; i < n; ++i) {
        if (M[i] == 0) continue;
        const TiledShape& s = w[i]->shape;
        const bool aligned = ((uintptr_t)x[i] % 16) == 0;
        const bool direct =
            aligned && (x_dtype == NXQ_F16 || (M[i] <= 2 && (x_dtype == NXQ_F32 || x_dtype == NXQ_BF16)));
        if (!mma_supported(s, M[i]) || !direct || (type >= 0 && s.type != type)) return NXQ_ERR_UNSUPPORTED;
        type = s.type;
        mmax = M[i] > mmax ? M[i] : mmax;
    }
    if (type < 0) return NXQ_OK;  // nothing to do
    const int mt = mmax <= 8 ? 8 : mmax <= 16 ? 16 : 32;
    for (int i = 0; i < n; ++i) {
        if (M[i] == 0) continue;
        items[k++] = HostItem{w[i], x[i], y[i], M[i]};
        if (k == kMaxItems) {
            if (int rc = launch_items(type, mt, items, k, x_dtype, y_dtype, st)) return rc;
            k = 0;
        }
    }
    return k ? launch_items(type, mt, items, k, x_dtype, y_dtype, st) : NXQ_OK;
}

}  // namespace nxq
