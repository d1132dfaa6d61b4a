// f16 dequantization of one 32-element group of one weight row, as 16 packed
// f16 pairs (element 2c in the low half of word c, 2c+1 in the high half) -
// the layout of a K-major MMA operand row in TMEM.  Used by the tcgen05
// kernels; `stage` is a tile-chunk staged in shared memory (formats.cuh).
//
// Each weight is formed as one f16 rounding of its exact value, computed from
// f16 scale terms: Q4_K fl16(q*fl16(d*sc) + fl16(-dmin*m)); Q4_0 fl16((q-8)*d);
// Q8_0 fl16(q*d); Q3_K fl16((q-4)*fl16(d*sc)).  Codes enter through the
// magic-number trick: a nibble placed in the mantissa of 1024 (or of 64 for a
// nibble 4 bits higher) is an exact f16 integer once the magic is subtracted.
#pragma once
#include <cuda_fp16.h>

#include "formats.cuh"

namespace nxq {
namespace dq {

__device__ __forceinline__ uint32_t h2u(__half2 h) { return *reinterpret_cast<uint32_t*>(&h); }
__device__ __forceinline__ __half2 u2h(uint32_t u) { return *reinterpret_cast<__half2*>(&u); }

template <int TYPE>
struct Group;

// (a & b) | c in one LOP3 (truth table 0xEA).
__device__ __forceinline__ uint32_t and_or(uint32_t a, uint32_t b, uint32_t c) {
    uint32_t d;
    asm("lop3.b32 %0, %1, %2, %3, 0xEA;" : "=r"(d) : "r"(a), "r"(b), "r"(c));
    return d;
}

// Four f16 pairs of a code word in the tiled 4-bit order (formats.cuh,
// q4_code_pos): elements (8w, 8w+1) .. (8w+6, 8w+7) as fl16(q * s + o).
__device__ __forceinline__ void q4_word_pairs(uint32_t w, __half2 s2, __half2 o2, uint32_t* o) {
    const __half2 m_lo = u2h(0x64006400u), m_hi = u2h(0x54005400u);  // 1024, 64
    const uint32_t w8 = w >> 8;
    o[0] = h2u(__hfma2(__hsub2(u2h(and_or(w, 0x000F000Fu, 0x64006400u)), m_lo), s2, o2));
    o[1] = h2u(__hfma2(__hsub2(u2h(and_or(w, 0x00F000F0u, 0x54005400u)), m_hi), s2, o2));
    o[2] = h2u(__hfma2(__hsub2(u2h(and_or(w8, 0x000F000Fu, 0x64006400u)), m_lo), s2, o2));
    o[3] = h2u(__hfma2(__hsub2(u2h(and_or(w8, 0x00F000F0u, 0x54005400u)), m_hi), s2, o2));
}

// Q4_K (gguf_importer.cpp:838-873): record = (d, dmin, scales[12], qs[128]);
// group G = sub-block G = code bytes 16G..16G+15.
template <>
struct Group<T_Q4_K> {
    static constexpr int kStage = TILE_ROWS * 144;
    template <int G>
    __device__ __forceinline__ static void decode(const uint8_t* stage, int r, uint32_t (&o)[16]) {
        const uint8_t* rec = stage + r * 144;
        const uint4 hd = *reinterpret_cast<const uint4*>(rec);
        const float d = __half2float(__ushort_as_half((unsigned short)(hd.x & 0xFFFFu)));
        const float dmin = __half2float(__ushort_as_half((unsigned short)(hd.x >> 16)));
        const uint32_t sb = ((G < 4 ? hd.y : hd.z) >> (8 * (G & 3))) & 0xFFu;
        const uint32_t eb = (hd.w >> (8 * (G & 3))) & 0xFFu;
        const int S = (int)(sb & 63u);
        const int Mn = (int)((sb >> 6) | ((G < 4 ? (eb & 15u) : (eb >> 4)) << 2));
        const __half2 s2 = __float2half2_rn(d * (float)S);
        const __half2 o2 = __float2half2_rn(-(dmin * (float)Mn));
        const uint4 q = *reinterpret_cast<const uint4*>(rec + 16 + 16 * G);
        q4_word_pairs(q.x, s2, o2, &o[0]);
        q4_word_pairs(q.y, s2, o2, &o[4]);
        q4_word_pairs(q.z, s2, o2, &o[8]);
        q4_word_pairs(q.w, s2, o2, &o[12]);
    }
};

// NXF INT4 groups (quant/gptq.cpp:9-27): record = [(scale, zero) per group,
// padded to H bytes][codes x8 of 16 B]; 32-element group G lies in block
// 32G / gs.  The weight is fl16(q * fl16(scale) + fl16(-(zero * scale))).
template <int TYPE>
struct GroupI4G {
    static constexpr int GS = i4g_gs(TYPE), H = i4g_hdr(TYPE), REC = H + CHUNK_K / 2;
    static constexpr int kStage = TILE_ROWS * REC;
    template <int G>
    __device__ __forceinline__ static void decode(const uint8_t* stage, int r, uint32_t (&o)[16]) {
        const uint8_t* rec = stage + r * REC;
        const float2 sz = *reinterpret_cast<const float2*>(rec + 8 * (32 * G / GS));
        const __half2 s2 = __float2half2_rn(sz.x);
        const __half2 o2 = __float2half2_rn(-(sz.y * sz.x));
        const uint4 q = *reinterpret_cast<const uint4*>(rec + H + 16 * G);
        q4_word_pairs(q.x, s2, o2, &o[0]);
        q4_word_pairs(q.y, s2, o2, &o[4]);
        q4_word_pairs(q.z, s2, o2, &o[8]);
        q4_word_pairs(q.w, s2, o2, &o[12]);
    }
};
template <>
struct Group<T_I4G32> : GroupI4G<T_I4G32> {};
template <>
struct Group<T_I4G64> : GroupI4G<T_I4G64> {};
template <>
struct Group<T_I4G128> : GroupI4G<T_I4G128> {};
template <>
struct Group<T_I4G256> : GroupI4G<T_I4G256> {};

// Q4_1 (gguf_importer.cpp:699-717): record = [(d, m) x8][codes x8 of 16 B];
// group G = block G; weights fl16(q * d + m).
template <>
struct Group<T_Q4_1> {
    static constexpr int kStage = TILE_ROWS * 160;
    template <int G>
    __device__ __forceinline__ static void decode(const uint8_t* stage, int r, uint32_t (&o)[16]) {
        const uint8_t* rec = stage + r * 160;
        const uint32_t dm = *reinterpret_cast<const uint32_t*>(rec + 4 * G);
        const __half2 s2 = u2h((dm & 0xFFFFu) | (dm << 16));
        const __half2 o2 = u2h((dm >> 16) | (dm & 0xFFFF0000u));
        const uint4 q = *reinterpret_cast<const uint4*>(rec + 32 + 16 * G);
        q4_word_pairs(q.x, s2, o2, &o[0]);
        q4_word_pairs(q.y, s2, o2, &o[4]);
        q4_word_pairs(q.z, s2, o2, &o[8]);
        q4_word_pairs(q.w, s2, o2, &o[12]);
    }
};

// Q4_0 (gguf_importer.cpp:679-695): record = [d x8][codes x8 of 16 B]; group G
// = block G.
template <>
struct Group<T_Q4_0> {
    static constexpr int kStage = TILE_ROWS * 144;
    template <int G>
    __device__ __forceinline__ static void decode(const uint8_t* stage, int r, uint32_t (&o)[16]) {
        const uint8_t* rec = stage + r * 144;
        const uint32_t dbits = *reinterpret_cast<const uint16_t*>(rec + 2 * G);
        const __half2 s2 = u2h(dbits | (dbits << 16));
        const __half2 o2 = __hmul2(s2, u2h(0xC800C800u));  // -8 d, exact
        const uint4 q = *reinterpret_cast<const uint4*>(rec + 16 + 16 * G);
        q4_word_pairs(q.x, s2, o2, &o[0]);
        q4_word_pairs(q.y, s2, o2, &o[4]);
        q4_word_pairs(q.z, s2, o2, &o[8]);
        q4_word_pairs(q.w, s2, o2, &o[12]);
    }
};

// Q8_0 (gguf_importer.cpp:721-733): record = [d x8][codes x8 of 32 B].
template <>
struct Group<T_Q8_0> {
    static constexpr int kStage = TILE_ROWS * 272;
    template <int G>
    __device__ __forceinline__ static void decode(const uint8_t* stage, int r, uint32_t (&o)[16]) {
        const uint8_t* rec = stage + r * 272;
        const uint32_t dbits = *reinterpret_cast<const uint16_t*>(rec + 2 * G);
        const __half2 s2 = u2h(dbits | (dbits << 16));
        const __half2 bias = u2h(0x64806480u);  // 1152: signed byte b is 1152 + b after the xor
        const uint4* qv = reinterpret_cast<const uint4*>(rec + 16 + 32 * G);
        const uint4 q0 = qv[0], q1 = qv[1];
        const uint32_t wds[8] = {q0.x, q0.y, q0.z, q0.w, q1.x, q1.y, q1.z, q1.w};
#pragma unroll
        for (int wi = 0; wi < 8; ++wi) {
            const uint32_t t0 = __byte_perm(wds[wi], 0u, 0x4140u) ^ 0x64806480u;
            const uint32_t t1 = __byte_perm(wds[wi], 0u, 0x4342u) ^ 0x64806480u;
            o[2 * wi] = h2u(__hmul2(__hsub2(u2h(t0), bias), s2));
            o[2 * wi + 1] = h2u(__hmul2(__hsub2(u2h(t1), bias), s2));
        }
    }
};

// a | (b & c) in one LOP3 (truth table 0xF8).
__device__ __forceinline__ uint32_t or_and(uint32_t a, uint32_t b, uint32_t c) {
    uint32_t d;
    asm("lop3.b32 %0, %1, %2, %3, 0xF8;" : "=r"(d) : "r"(a), "r"(b), "r"(c));
    return d;
}

// Pair K of a Q3_K code word (formats.cuh, q3_lo_pos / q3_hi_pos): low codes
// at bits {2K, 2K+1} (+16), high bits at {2K+2} (+16) of `hs`, placed in the
// mantissa of a magic number whose unit is bit 2K (1024, 256, 64, 16), so
// subtracting magic + 4 leaves u - 4 exactly; times s = fl16(d * (sc - 32)).
template <int K>
__device__ __forceinline__ uint32_t q3_pair(uint32_t ls, uint32_t hs, __half2 s2) {
    constexpr uint32_t MG = K == 0 ? 0x64006400u : K == 1 ? 0x5C005C00u : K == 2 ? 0x54005400u : 0x4C004C00u;
    constexpr uint32_t BI = K == 0 ? 0x64046404u : K == 1 ? 0x5C105C10u : K == 2 ? 0x54405440u : 0x4D004D00u;
    const uint32_t v = or_and(and_or(ls, 0x00030003u << (2 * K), MG), hs, 0x00040004u << (2 * K));
    return h2u(__hmul2(__hsub2(u2h(v), u2h(BI)), s2));
}

// Pairs (2i, 2i+1), i = 0..7, of the 16 elements of one L word; `h` is the
// high-bit word already rotated for L1.
__device__ __forceinline__ void q3_word_pairs(uint32_t l, uint32_t h, __half2 s2, uint32_t* o) {
    o[0] = q3_pair<0>(l, h, s2);
    o[1] = q3_pair<1>(l, h, s2);
    o[2] = q3_pair<2>(l, h, s2);
    o[3] = q3_pair<3>(l, h, s2);
    const uint32_t l8 = l >> 8, h1 = h >> 1;
    o[4] = q3_pair<0>(l8, h1, s2);
    o[5] = q3_pair<1>(l8, h1, s2);
    o[6] = q3_pair<2>(l8, h1, s2);
    o[7] = q3_pair<3>(l8, h1, s2);
}

// Q3_K (gguf_importer.cpp:791-833): plane A = 8 x [L0 L1 H] (tiled code order)
// at r*96, plane B = [scales 12][d] at 128*96 + r*14; group G = elements
// 32G..32G+31, scale groups 2G (L0) and 2G+1 (L1).
template <>
struct Group<T_Q3_K> {
    static constexpr int kStage = TILE_ROWS * 110;
    template <int G>
    __device__ __forceinline__ static void decode(const uint8_t* stage, int r, uint32_t (&o)[16]) {
        const uint8_t* rec = stage + r * 96;
        const uint8_t* tl = stage + TILE_ROWS * 96 + r * 14;
        const float d = __half2float(__ushort_as_half(*reinterpret_cast<const uint16_t*>(tl + 12)));
        __half2 s2[2];
#pragma unroll
        for (int gg = 0; gg < 2; ++gg) {
            const int g = 2 * G + gg;
            const int i8 = g & 7;
            const uint32_t lo = tl[i8];
            const uint32_t hi = tl[8 + i8 / 2] >> (4 * (i8 & 1));
            const int S = g < 8 ? (int)((lo & 15u) | ((hi & 3u) << 4)) : (int)((lo >> 4) | (((hi >> 2) & 3u) << 4));
            s2[gg] = __float2half2_rn(d * (float)(S - 32));
        }
        const uint32_t* w = reinterpret_cast<const uint32_t*>(rec + 12 * G);
        const uint32_t h = w[2];
        q3_word_pairs(w[0], h, s2[0], &o[0]);
        q3_word_pairs(w[1], __funnelshift_r(h, h, 8), s2[1], &o[8]);
    }
};

// Pair K (0..3) of a Q6_K L word (formats.cuh, q6_lo_bit / q6_hi_bit): for
// K = 0, 1 the low nibbles sit at bits 4K (+16) of `l` and the high bits two
// above them in `h` (= H rotated by 2 (w % 2)); K = 2, 3 use l >> 8 and H
// rotated by 8 + 2 (w % 2).  The 6-bit code lands in the mantissa of 1024
// (K even) or 64 (K odd); subtracting magic + 32 leaves q - 32 exactly; times
// s = fl16(d * sc).
template <int K>
__device__ __forceinline__ uint32_t q6_pair(uint32_t l, uint32_t h, __half2 s2) {
    constexpr int KK = K & 1;
    constexpr uint32_t MG = KK ? 0x54005400u : 0x64006400u;  // 64, 1024
    constexpr uint32_t BI = KK ? 0x56005600u : 0x64206420u;  // 96, 1056
    const uint32_t v = or_and(and_or(l, 0x000F000Fu << (4 * KK), MG), h, 0x00300030u << (4 * KK));
    return h2u(__hmul2(__hsub2(u2h(v), u2h(BI)), s2));
}

// The four pairs of L word `l` (elements 8w .. 8w+7 of its group) whose high
// bits are in `h`, with o = 2 (w % 2).
template <int O>
__device__ __forceinline__ void q6_word_pairs(uint32_t l, uint32_t h, __half2 s2, uint32_t* o) {
    const uint32_t h0 = O ? __funnelshift_r(h, h, O) : h;
    const uint32_t h1 = __funnelshift_r(h, h, 8 + O);
    const uint32_t l8 = l >> 8;
    o[0] = q6_pair<0>(l, h0, s2);
    o[1] = q6_pair<1>(l, h0, s2);
    o[2] = q6_pair<2>(l8, h1, s2);
    o[3] = q6_pair<3>(l8, h1, s2);
}

// Pair K (0..3) of a Q2_K code word (formats.cuh, q2_tiled_byte): the 2-bit
// codes at bits {2K, 2K+1} (+16) in the mantissa of a magic number whose unit
// is bit 2K (1024, 256, 64, 16); fl16(q * s + o) as for Q4_K.
template <int K>
__device__ __forceinline__ uint32_t q2_pair(uint32_t ls, __half2 s2, __half2 o2) {
    constexpr uint32_t MG = K == 0 ? 0x64006400u : K == 1 ? 0x5C005C00u : K == 2 ? 0x54005400u : 0x4C004C00u;
    const uint32_t v = and_or(ls, 0x00030003u << (2 * K), MG);
    return h2u(__hfma2(__hsub2(u2h(v), u2h(MG)), s2, o2));
}

// Pairs (2i, 2i+1), i = 4h .. 4h+3, of the 16 elements of a Q2_K code word.
__device__ __forceinline__ void q2_half_pairs(uint32_t l, __half2 s2, __half2 o2, uint32_t* o) {
    o[0] = q2_pair<0>(l, s2, o2);
    o[1] = q2_pair<1>(l, s2, o2);
    o[2] = q2_pair<2>(l, s2, o2);
    o[3] = q2_pair<3>(l, s2, o2);
}

// Q2_K (gguf_importer.cpp:756-786): plane A = [scales[16]][8 x [L0 L1]] at
// r*80, plane B = (dmin, d) at 128*80 + r*4; group G = elements 32G..32G+31,
// scale bytes 2G (L0) and 2G+1 (L1): low nibble scale, high nibble min.
template <>
struct Group<T_Q2_K> {
    static constexpr int kStage = TILE_ROWS * 84;
    template <int G>
    __device__ __forceinline__ static void decode(const uint8_t* stage, int r, uint32_t (&o)[16]) {
        const uint8_t* rec = stage + r * 80;
        const uint32_t dd = *reinterpret_cast<const uint32_t*>(stage + TILE_ROWS * 80 + r * 4);
        const float dmin = __half2float(__ushort_as_half((unsigned short)(dd & 0xFFFFu)));
        const float d = __half2float(__ushort_as_half((unsigned short)(dd >> 16)));
        const uint2 w = *reinterpret_cast<const uint2*>(rec + 16 + 8 * G);
#pragma unroll
        for (int h = 0; h < 2; ++h) {
            const uint32_t sc = rec[2 * G + h];
            const __half2 s2 = __float2half2_rn(d * (float)(sc & 15u));
            const __half2 o2 = __float2half2_rn(-(dmin * (float)(sc >> 4)));
            const uint32_t l = h ? w.y : w.x;
            q2_half_pairs(l, s2, o2, &o[8 * h]);
            q2_half_pairs(l >> 8, s2, o2, &o[8 * h + 4]);
        }
    }
};

// Pair K (0..3) of a Q5_K L word (formats.cuh, q5_hi_bit): as q6_pair with one
// high bit (mask 0x10 << 4(K&1)); the 5-bit code q lands in the mantissa of
// 1024 or 64, and fl16(q * s + o) follows as for Q4_K.
template <int K>
__device__ __forceinline__ uint32_t q5_pair(uint32_t l, uint32_t h, __half2 s2, __half2 o2) {
    constexpr int KK = K & 1;
    constexpr uint32_t MG = KK ? 0x54005400u : 0x64006400u;  // 64, 1024
    const uint32_t v = or_and(and_or(l, 0x000F000Fu << (4 * KK), MG), h, 0x00100010u << (4 * KK));
    return h2u(__hfma2(__hsub2(u2h(v), u2h(MG)), s2, o2));
}

// The four pairs of L word w (elements 8w .. 8w+7 of its group); h is the
// group's high-bit word.
template <int W>
__device__ __forceinline__ void q5_word_pairs(uint32_t l, uint32_t h, __half2 s2, __half2 o2, uint32_t* o) {
    const uint32_t h0 = W ? __funnelshift_r(h, h, W) : h;
    const uint32_t h1 = __funnelshift_r(h, h, 8 + W);
    const uint32_t l8 = l >> 8;
    o[0] = q5_pair<0>(l, h0, s2, o2);
    o[1] = q5_pair<1>(l, h0, s2, o2);
    o[2] = q5_pair<2>(l8, h1, s2, o2);
    o[3] = q5_pair<3>(l8, h1, s2, o2);
}

// Q5_K (gguf_importer.cpp:878-915): record = [d, dmin, scales[12]][L words of 8
// groups][H word of 8 groups] (tiled code order); group G = sub-block G.
template <>
struct Group<T_Q5_K> {
    static constexpr int kStage = TILE_ROWS * 176;
    template <int G>
    __device__ __forceinline__ static void decode(const uint8_t* stage, int r, uint32_t (&o)[16]) {
        const uint8_t* rec = stage + r * 176;
        const uint4 hd = *reinterpret_cast<const uint4*>(rec);
        const float d = __half2float(__ushort_as_half((unsigned short)(hd.x & 0xFFFFu)));
        const float dmin = __half2float(__ushort_as_half((unsigned short)(hd.x >> 16)));
        const uint32_t sb = ((G < 4 ? hd.y : hd.z) >> (8 * (G & 3))) & 0xFFu;
        const uint32_t eb = (hd.w >> (8 * (G & 3))) & 0xFFu;
        const int S = (int)(sb & 63u);
        const int Mn = (int)((sb >> 6) | ((G < 4 ? (eb & 15u) : (eb >> 4)) << 2));
        const __half2 s2 = __float2half2_rn(d * (float)S);
        const __half2 o2 = __float2half2_rn(-(dmin * (float)Mn));
        const uint4 q = *reinterpret_cast<const uint4*>(rec + 16 + 16 * G);
        const uint32_t h = *reinterpret_cast<const uint32_t*>(rec + 144 + 4 * G);
        q5_word_pairs<0>(q.x, h, s2, o2, &o[0]);
        q5_word_pairs<1>(q.y, h, s2, o2, &o[4]);
        q5_word_pairs<2>(q.z, h, s2, o2, &o[8]);
        q5_word_pairs<3>(q.w, h, s2, o2, &o[12]);
    }
};

// Q6_K (gguf_importer.cpp:924-954): plane A = 8 x [L0 L1 L2 L3 H0 H1] (tiled
// code order) at r*192, plane B = 16 int8 scales at 128*192 + r*16, plane C =
// d at 128*208 + r*2; group G = elements 32G..32G+31, scales 2G and 2G+1.
template <>
struct Group<T_Q6_K> {
    static constexpr int kStage = TILE_ROWS * 210;
    template <int G>
    __device__ __forceinline__ static void decode(const uint8_t* stage, int r, uint32_t (&o)[16]) {
        const uint8_t* rec = stage + r * 192 + 24 * G;
        const int8_t* sc = reinterpret_cast<const int8_t*>(stage + TILE_ROWS * 192 + r * 16 + 2 * G);
        const float d = __half2float(__ushort_as_half(*reinterpret_cast<const uint16_t*>(stage + TILE_ROWS * 208 + r * 2)));
        const __half2 sa = __float2half2_rn(d * (float)sc[0]), sb = __float2half2_rn(d * (float)sc[1]);
        const uint2 a = *reinterpret_cast<const uint2*>(rec);
        const uint2 b = *reinterpret_cast<const uint2*>(rec + 8);
        const uint2 c = *reinterpret_cast<const uint2*>(rec + 16);
        q6_word_pairs<0>(a.x, c.x, sa, &o[0]);
        q6_word_pairs<2>(a.y, c.x, sa, &o[4]);
        q6_word_pairs<0>(b.x, c.y, sb, &o[8]);
        q6_word_pairs<2>(b.y, c.y, sb, &o[12]);
    }
};

}  // namespace dq
}  // namespace nxq
