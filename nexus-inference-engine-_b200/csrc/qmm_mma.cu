// Register-fragment dequant-fused GEMV for decode batches (M <= 32), sm_100a.
//
// Replaces the reference's Metal decode GEMV (gemv_int4_nr8.metal:31-87,
// gemv_q3k.metal:33-98; dispatched by ComputeDispatch::gemm_int4 ->
// MetalBackend::gemv_int4_nr8, metal_backend.mm:607-642) for Q4_0, Q8_0,
// Q4_K and Q3_K.
//
// Why mma.sync and not tcgen05 here: a tcgen05.mma with M=128, K=16 costs
// ~60 cycles for any N <= 128 (measured on this B200), so feeding dequantized
// weights as its 128-row operand caps a GEMV at ~34 weights/cycle/SM.  The
// warp-level mma.sync.m16n8k16 is issued by all four schedulers with operands
// straight from registers (measured 2 cycles/instruction/SM); with the
// weights as its 8-column B operand that is 64 weights/cycle/SM at M <= 16,
// leaving the packed-weight stream from HBM as the bound.  The prefill GEMM,
// where N is large, uses tcgen05.
//
// Decomposition (shared with the tcgen05 kernels): the weight is stored tiled
// (formats.cuh), a unit is one tile-chunk (128 rows x 256 k, contiguous in
// HBM), and a persistent grid of one CTA per SM takes contiguous unit ranges
// (stream-K).  A tile split between CTAs is summed by the last of them to
// finish (per-tile counter, fp32 partials in a workspace, CTA order), so the
// result is deterministic; each CTA processes its split tiles first, so those
// fixups overlap the rest of its work instead of trailing it.
//
// Per CTA, 16 warps; warp w owns weight rows 8w..8w+7 of the tile (the n8
// tile of its mma).  In lane (g, t) (g = lane/4, t = lane%4), the mma's
// k-slots {2t, 2t+1, 2t+8, 2t+9} of k-step j map to chunk elements
// 64t + 4j + {0,1,2,3}, for x and W alike, so every lane reads one row (g) and
// one private 64-element slice of it: exactly two 32-element sub-blocks, whose
// scales it alone needs.  Units are staged with cp.async into an S-deep
// shared-memory ring: the packed tile-chunk byte for byte, and x as 8-byte
// pieces in a bank-conflict-free fragment order.
//
// Numerics: each weight is formed in f16 as fl16(q * fl16(d*sc) + fl16(-dmin*m))
// (Q4_K; the other types analogously), products are exact and accumulate in
// fp32; activations enter as f16.
#include <cuda_bf16.h>
#include <cuda_fp16.h>

#include <cstdio>
#include <cstdlib>

#include "qmm_mma.h"
#include "stream_scratch.h"

namespace nxq {

namespace {

constexpr int kWarps = 8;
constexpr int kThreads = kWarps * 32;
constexpr int kMaxMT = 32;

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
    return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}
__device__ __forceinline__ void cp_async16(void* dst, const void* src) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(smem_u32(dst)), "l"(src) : "memory");
}
__device__ __forceinline__ void cp_async4(void* dst, const void* src) {
    asm volatile("cp.async.ca.shared.global [%0], [%1], 4;" ::"r"(smem_u32(dst)), "l"(src) : "memory");
}
__device__ __forceinline__ void cp_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_wait() {
    asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}

__device__ __forceinline__ void mma16816(float (&c)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                                         uint32_t b0, uint32_t b1) {
    asm("mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
        "{%0,%1,%2,%3};"
        : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
        : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

__device__ __forceinline__ uint32_t h2u(__half2 h) { return *reinterpret_cast<uint32_t*>(&h); }
__device__ __forceinline__ __half2 u2h(uint32_t u) { return *reinterpret_cast<__half2*>(&u); }
__device__ __forceinline__ uint32_t sel4(uint32_t i, const uint4& v) {
    return i == 0 ? v.x : i == 1 ? v.y : i == 2 ? v.z : v.w;
}
__device__ __forceinline__ uint32_t word_of(const uint4& v, int i) {
    return i == 0 ? v.x : i == 1 ? v.y : i == 2 ? v.z : v.w;
}
// Byte b of a 32-bit word as the f16 pair (1024 + lo nibble, 64 + hi nibble).
__device__ __forceinline__ __half2 nib_pair(uint32_t w, int b) {
    const uint32_t t = __byte_perm(w, 0u, 0x4040u | (b << 8) | b);
    return u2h((t & 0x00F0000Fu) | 0x54006400u);
}

// ---------------------------------------------------------------------------
// Per-format lane decoders.  load() reads the lane's slice of row `row` of a
// staged tile-chunk; frag(j) returns the two B registers of k-step j (weights
// at chunk elements 64t + 4j + {0,1} and {2,3}) as f16 pairs.
// ---------------------------------------------------------------------------
template <int TYPE>
struct Lane;

// Q4_K (gguf_importer.cpp:838-873): record = block (d, dmin, scales[12], qs[128]);
// the lane's elements are sub-blocks 2t, 2t+1 = code bytes 32t .. 32t+31.
template <>
struct Lane<T_Q4_K> {
    static constexpr int kStage = TILE_ROWS * 144;
    uint4 hd, q0, q1;
    __half2 s2[2], o2[2];
    __device__ __forceinline__ void load(const uint8_t* st, int row, int t) {
        const uint8_t* rec = st + row * 144;
        hd = *reinterpret_cast<const uint4*>(rec);
        q0 = *reinterpret_cast<const uint4*>(rec + 16 + 32 * t);
        q1 = *reinterpret_cast<const uint4*>(rec + 32 + 32 * t);
        const float d = __half2float(__ushort_as_half((unsigned short)(hd.x & 0xFFFFu)));
        const float dmin = __half2float(__ushort_as_half((unsigned short)(hd.x >> 16)));
#pragma unroll
        for (int sub = 0; sub < 2; ++sub) {
            const int g = 2 * t + sub;
            const uint32_t sb = ((g < 4 ? hd.y : hd.z) >> (8 * (g & 3))) & 0xFFu;
            const uint32_t eb = (hd.w >> (8 * (g & 3))) & 0xFFu;
            const int S = (int)(sb & 63u);
            const int Mn = (int)((sb >> 6) | ((g < 4 ? (eb & 15u) : (eb >> 4)) << 2));
            s2[sub] = __float2half2_rn(d * (float)S);
            o2[sub] = __float2half2_rn(-(dmin * (float)Mn));
        }
    }
    __device__ __forceinline__ void frag(int j, uint32_t& b0, uint32_t& b1) const {
        const uint32_t w = word_of(j < 8 ? q0 : q1, (j >> 1) & 3);
        const int b = 2 * (j & 1);
        const __half2 magic = u2h(0x54006400u);
        const int sub = j >> 3;
        b0 = h2u(__hfma2(__hsub2(nib_pair(w, b), magic), s2[sub], o2[sub]));
        b1 = h2u(__hfma2(__hsub2(nib_pair(w, b + 1), magic), s2[sub], o2[sub]));
    }
};

// Q4_0 (gguf_importer.cpp:679-695): record = [d x8][codes x8 of 16 B]; the
// lane's elements are blocks 2t, 2t+1.
template <>
struct Lane<T_Q4_0> {
    static constexpr int kStage = TILE_ROWS * 144;
    uint4 q0, q1;
    __half2 s2[2], o2[2];
    __device__ __forceinline__ void load(const uint8_t* st, int row, int t) {
        const uint8_t* rec = st + row * 144;
        const uint4 hd = *reinterpret_cast<const uint4*>(rec);
        q0 = *reinterpret_cast<const uint4*>(rec + 16 + 32 * t);
        q1 = *reinterpret_cast<const uint4*>(rec + 32 + 32 * t);
        const uint32_t dw = sel4((uint32_t)t, hd);
        const __half2 neg8 = u2h(0xC800C800u);
#pragma unroll
        for (int sub = 0; sub < 2; ++sub) {
            const uint32_t bits = sub ? (dw >> 16) : (dw & 0xFFFFu);
            s2[sub] = u2h(bits | (bits << 16));
            o2[sub] = __hmul2(s2[sub], neg8);  // exact
        }
    }
    __device__ __forceinline__ void frag(int j, uint32_t& b0, uint32_t& b1) const {
        const int sub = j >> 3, jj = j & 7;
        const uint32_t w = word_of(sub ? q1 : q0, jj & 3);
        const uint32_t t0 = __byte_perm(w, 0u, 0x4140u), t1 = __byte_perm(w, 0u, 0x4342u);
        __half2 v0, v1;
        if (jj < 4) {  // elements 0..15 of the block: low nibbles
            v0 = __hsub2(u2h((t0 & 0x000F000Fu) | 0x64006400u), u2h(0x64006400u));
            v1 = __hsub2(u2h((t1 & 0x000F000Fu) | 0x64006400u), u2h(0x64006400u));
        } else {  // elements 16..31: high nibbles
            v0 = __hsub2(u2h((t0 & 0x00F000F0u) | 0x54005400u), u2h(0x54005400u));
            v1 = __hsub2(u2h((t1 & 0x00F000F0u) | 0x54005400u), u2h(0x54005400u));
        }
        b0 = h2u(__hfma2(v0, s2[sub], o2[sub]));
        b1 = h2u(__hfma2(v1, s2[sub], o2[sub]));
    }
};

// Q8_0 (gguf_importer.cpp:721-733): record = [d x8][codes x8 of 32 B].
template <>
struct Lane<T_Q8_0> {
    static constexpr int kStage = TILE_ROWS * 272;
    uint4 c[4];
    __half2 s2[2];
    __device__ __forceinline__ void load(const uint8_t* st, int row, int t) {
        const uint8_t* rec = st + row * 272;
        const uint4 hd = *reinterpret_cast<const uint4*>(rec);
        const uint4* cv = reinterpret_cast<const uint4*>(rec + 16 + 64 * t);
#pragma unroll
        for (int i = 0; i < 4; ++i) c[i] = cv[i];
        const uint32_t dw = sel4((uint32_t)t, hd);
        s2[0] = u2h((dw & 0xFFFFu) | (dw << 16));
        s2[1] = u2h((dw >> 16) | (dw & 0xFFFF0000u));
    }
    __device__ __forceinline__ void frag(int j, uint32_t& b0, uint32_t& b1) const {
        const int sub = j >> 3, jj = j & 7;
        const uint32_t w = word_of(c[2 * sub + (jj >> 2)], jj & 3);
        // Signed byte b -> f16 1152 + b via (b ^ 0x80) in the mantissa of 1024.
        const __half2 bias = u2h(0x64806480u);
        const uint32_t t0 = __byte_perm(w, 0u, 0x4140u) ^ 0x64806480u;
        const uint32_t t1 = __byte_perm(w, 0u, 0x4342u) ^ 0x64806480u;
        b0 = h2u(__hmul2(__hsub2(u2h(t0), bias), s2[sub]));
        b1 = h2u(__hmul2(__hsub2(u2h(t1), bias), s2[sub]));
    }
};

// Q3_K (gguf_importer.cpp:791-833): plane A = [hmask 32][qs 64] at row*96,
// plane B = [scales 12][d] at 128*96 + row*14.  The lane's elements 64t..64t+63
// are qs bytes 16t.. and hmask bytes 8t.., in four 16-element scale groups.
template <>
struct Lane<T_Q3_K> {
    static constexpr int kStage = TILE_ROWS * 110;
    uint4 qs;
    uint2 hm;
    __half2 s2[4];
    __device__ __forceinline__ void load(const uint8_t* st, int row, int t) {
        const uint8_t* rec = st + row * 96;
        qs = *reinterpret_cast<const uint4*>(rec + 32 + 16 * t);
        hm = *reinterpret_cast<const uint2*>(rec + 8 * t);
        const uint16_t* tl = reinterpret_cast<const uint16_t*>(st + TILE_ROWS * 96 + row * 14);
        const uint32_t sc0 = tl[0] | ((uint32_t)tl[1] << 16);  // scale bytes 0..3
        const uint32_t sc1 = tl[2] | ((uint32_t)tl[3] << 16);  // 4..7
        const uint32_t sc2 = tl[4] | ((uint32_t)tl[5] << 16);  // 8..11
        const float d = __half2float(__ushort_as_half(tl[6]));
#pragma unroll
        for (int gg = 0; gg < 4; ++gg) {
            // group G = 4t + gg; i8 = G & 7 = 4(t&1) + gg; G < 8 iff t < 2
            const uint32_t lowb = (((t & 1) ? sc1 : sc0) >> (8 * gg)) & 0xFFu;
            const uint32_t hib = (sc2 >> (8 * (2 * (t & 1) + (gg >> 1)))) >> (4 * (gg & 1));
            const int S = t < 2 ? (int)((lowb & 15u) | ((hib & 3u) << 4))
                                : (int)((lowb >> 4) | (((hib >> 2) & 3u) << 4));
            s2[gg] = __float2half2_rn(d * (float)(S - 32));
        }
    }
    __device__ __forceinline__ void frag(int j, uint32_t& b0, uint32_t& b1) const {
        const uint32_t Q = (word_of(qs, j >> 2) >> (8 * (j & 3))) & 0xFFu;
        const uint32_t H = (((j >> 3) ? hm.y : hm.x) >> (8 * ((j >> 1) & 3) + 4 * (j & 1))) & 0xFu;
        const uint32_t q0 = (Q & 3u) | ((H & 1u) << 2), q1 = ((Q >> 2) & 3u) | (((H >> 1) & 1u) << 2);
        const uint32_t q2 = ((Q >> 4) & 3u) | (((H >> 2) & 1u) << 2), q3 = (Q >> 6) | (((H >> 3) & 1u) << 2);
        const __half2 bias = u2h(0x64046404u);  // 1028: removes the magic and the -4 offset
        const __half2 s = s2[j >> 2];
        b0 = h2u(__hmul2(__hsub2(u2h(q0 | (q1 << 16) | 0x64006400u), bias), s));
        b1 = h2u(__hmul2(__hsub2(u2h(q2 | (q3 << 16) | 0x64006400u), bias), s));
    }
};

template <int TYPE, int MT>
struct Cfg {
    static constexpr int WB = Lane<TYPE>::kStage;
    static constexpr int XB = (MT < 16 ? 16 : MT) * 512;  // token slots x 256 f16
    // Two CTAs per SM when a 3-deep ring fits in half the shared memory.
    static constexpr int S2 = (112 * 1024) / (WB + XB);
    static constexpr int CPS = S2 >= 3 ? 2 : 1;
    static constexpr int S0 = CPS == 2 ? S2 : (220 * 1024) / (WB + XB);
    static constexpr int S = S0 > 6 ? 6 : S0;
    static constexpr size_t smem = (size_t)S * (WB + XB);
    static_assert(S >= 3, "pipeline too shallow");
};

struct MmaParams {
    const uint8_t* w;
    TiledShape s;
    const __half* x;
    int64_t M;
    void* y;
    int y_dtype;
    float* ws;
    unsigned* counters;
    int64_t units;
    int grid;
};

__device__ __forceinline__ int range_begin(int c, int U, int G) { return (int)((int64_t)c * U / G); }
// The CTA whose range holds unit u.
__device__ __forceinline__ int owner_of(int u, int U, int G) {
    return (int)((((int64_t)u + 1) * G + U - 1) / U) - 1;
}

__device__ __forceinline__ void store_y(void* y, int dt, int64_t i, float v) {
    if (dt == NXQ_F32)
        reinterpret_cast<float*>(y)[i] = v;
    else if (dt == NXQ_F16)
        reinterpret_cast<__half*>(y)[i] = __float2half_rn(v);
    else
        reinterpret_cast<__nv_bfloat16*>(y)[i] = __float2bfloat16_rn(v);
}

// The CTA's unit range [u0, u1) as up to four segments, each inside one tile
// or made of whole tiles: split tiles first, whole tiles after.
struct Segs {
    int start[4], len[4];
    bool whole[4];
    int n;
    __device__ void add(int s, int l, bool w) {
        if (l > 0) {
            start[n] = s;
            len[n] = l;
            whole[n] = w;
            ++n;
        }
    }
};

// A walk over the segments, one unit at a time, without divisions except on
// entering a segment.
struct Cursor {
    int seg, left, t, kc;
    bool whole;
    __device__ void enter(const Segs& sg, int k, int chunks) {
        seg = k;
        if (k >= sg.n) {
            left = 0;
            return;
        }
        left = sg.len[k];
        t = sg.start[k] / chunks;
        kc = sg.start[k] - t * chunks;
        whole = sg.whole[k];
    }
    __device__ void next(const Segs& sg, int chunks) {
        if (--left > 0) {
            if (++kc == chunks) {
                kc = 0;
                ++t;
            }
        } else {
            enter(sg, seg + 1, chunks);
        }
    }
    // Last unit of a tile's segment: the tile's result is complete here.
    __device__ bool tile_end(int chunks) const { return left == 1 || kc == chunks - 1; }
};

template <int TYPE, int MT>
__global__ void __launch_bounds__(kThreads, Cfg<TYPE, MT>::CPS) mma_gemv_kernel(const MmaParams p) {
    using C = Cfg<TYPE, MT>;
    constexpr int S = C::S, WB = C::WB, XB = C::XB;
    extern __shared__ __align__(16) uint8_t smem[];
    uint8_t* wst = smem;                   // S x WB
    uint8_t* xst = smem + (size_t)S * WB;  // S x XB
    __shared__ int s_last;

    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int g = lane >> 2, tq = lane & 3;
    const int U = (int)p.units, G = p.grid, chunks = (int)p.s.chunks;
    const int64_t K = p.s.K, N = p.s.N;
    const int M = (int)p.M;
    const int u0 = range_begin(blockIdx.x, U, G), u1 = range_begin(blockIdx.x + 1, U, G);
    const int n = u1 - u0;

    Segs sg;
    sg.n = 0;
    {
        const int tf = u0 / chunks, tl = (u1 - 1) / chunks;
        if (tf == tl) {
            sg.add(u0, n, u0 == tf * chunks && u1 == (tf + 1) * chunks);
        } else {
            const bool wa = u0 == tf * chunks, wb = u1 == (tl + 1) * chunks;
            const int a_end = (tf + 1) * chunks, b_beg = tl * chunks;
            if (!wb) sg.add(b_beg, u1 - b_beg, false);
            sg.add(u0, a_end - u0, wa);
            sg.add(a_end, b_beg - a_end, true);
            if (wb) sg.add(b_beg, u1 - b_beg, true);
        }
    }

    // Loader: stages the unit under `lc` into stage `stg`.  x is stored as the
    // mma's A fragments: 16-byte slot (tile16, t4, j, g) holds, for chunk
    // elements k = 64*t4 + 4*j, the words {x[g][k,k+1], x[g+8][k,k+1],
    // x[g][k+2,k+3], x[g+8][k+2,k+3]} (g = token % 8 within a 16-token tile),
    // at slot index (tile16*64 + t4*16 + j)*8 + (g ^ 2*t4) so each 8-lane phase
    // of the 16-byte fragment loads hits distinct banks.
    Cursor lc;
    lc.enter(sg, 0, chunks);
    auto load_unit = [&](int stg) {
        const uint8_t* src = p.w + p.s.chunk_offset(lc.t, lc.kc) + 16 * tid;
        uint8_t* dst = wst + stg * WB + 16 * tid;
        constexpr int kPieces = WB / 16, kFull = kPieces / kThreads;
#pragma unroll
        for (int r = 0; r < kFull; ++r) cp_async16(dst + 16 * kThreads * r, src + 16 * kThreads * r);
        if (kPieces % kThreads && tid < kPieces % kThreads)
            cp_async16(dst + 16 * kThreads * kFull, src + 16 * kThreads * kFull);
        uint32_t* xd = reinterpret_cast<uint32_t*>(xst + stg * XB);
        const int k0 = lc.kc * CHUNK_K;
        for (int q = tid; q < M * 128; q += kThreads) {
            // q -> (token, t4, j, half): one 4-byte pair x[tok][k + 2*half .. +1]
            const int tok = q >> 7, r = q & 127, t4 = r >> 5, j = (r >> 1) & 15, half = r & 1;
            const int k = k0 + 64 * t4 + 4 * j + 2 * half;
            const int gg = tok & 7, up = (tok >> 3) & 1;
            uint32_t* d = xd + ((((tok >> 4) * 64 + t4 * 16 + j) * 8 + (gg ^ (2 * t4))) << 2) + 2 * half + up;
            if (k < K)
                cp_async4(d, p.x + (int64_t)tok * K + k);
            else
                *d = 0u;
        }
        lc.next(sg, chunks);
    };

    // Token slots at or beyond M are never loaded; zero them once so the
    // fragment loads need no predicate.
    for (int q = tid; q < S * XB / 16; q += kThreads) reinterpret_cast<uint4*>(xst)[q] = make_uint4(0u, 0u, 0u, 0u);
    __syncthreads();

    // acc[n8 tile][token tile][c0..c3]; the warp's n8 tiles are rows
    // 16*warp + g and 16*warp + 8 + g.
    constexpr int TT = MT < 16 ? 1 : MT / 16;  // 16-token tiles
    float acc[2][TT][4];
#pragma unroll
    for (int st = 0; st < S - 1; ++st) {
        if (st < n) load_unit(st);
        cp_commit();
    }
    Cursor cc;
    cc.enter(sg, 0, chunks);
    bool fresh = true;
    for (int i = 0; i < n; ++i) {
        cp_wait<S - 2>();
        __syncthreads();
        if (i + S - 1 < n) load_unit((i + S - 1) % S);
        cp_commit();

        if (fresh) {
#pragma unroll
            for (int nt = 0; nt < 2; ++nt)
#pragma unroll
                for (int tt = 0; tt < TT; ++tt)
#pragma unroll
                    for (int e = 0; e < 4; ++e) acc[nt][tt][e] = 0.0f;
            fresh = false;
        }

        // ---- compute on stage i % S ----
        const int stg = i % S;
        Lane<TYPE> LA, LB;
        LA.load(wst + stg * WB, 16 * warp + g, tq);
        LB.load(wst + stg * WB, 16 * warp + 8 + g, tq);
        const uint4* xs = reinterpret_cast<const uint4*>(xst + stg * XB) + tq * 128 + (g ^ (2 * tq));
#pragma unroll
        for (int j = 0; j < 16; ++j) {
            uint32_t a0, a1, b0, b1;
            LA.frag(j, a0, a1);
            LB.frag(j, b0, b1);
#pragma unroll
            for (int tt = 0; tt < TT; ++tt) {
                const uint4 xa = xs[tt * 512 + j * 8];
                mma16816(acc[0][tt], xa.x, xa.y, xa.z, xa.w, a0, a1);
                mma16816(acc[1][tt], xa.x, xa.y, xa.z, xa.w, b0, b1);
            }
        }

        // ---- end of this tile's segment: write or hand over the result ----
        const bool seg_end = cc.tile_end(chunks);
        const int t = cc.t;
        const bool whole = cc.whole;
        cc.next(sg, chunks);
        if (!seg_end) continue;
        fresh = true;
        if (whole) {
#pragma unroll
            for (int nt = 0; nt < 2; ++nt)
#pragma unroll
                for (int tt = 0; tt < TT; ++tt)
#pragma unroll
                    for (int e = 0; e < 4; ++e) {
                        const int tok = 16 * tt + g + (e >> 1) * 8;
                        const int64_t row = (int64_t)t * TILE_ROWS + 16 * warp + 8 * nt + 2 * tq + (e & 1);
                        if (tok < M && row < N) store_y(p.y, p.y_dtype, tok * N + row, acc[nt][tt][e]);
                    }
        } else {
            const int c = blockIdx.x;
            const int slot = u0 >= t * chunks ? 0 : 1;  // 0: tile t is where this CTA's range starts
            float* mine = p.ws + ((size_t)c * 2 + slot) * (kMaxMT * TILE_ROWS);
#pragma unroll
            for (int nt = 0; nt < 2; ++nt)
#pragma unroll
                for (int tt = 0; tt < TT; ++tt)
#pragma unroll
                    for (int e = 0; e < 4; ++e) {
                        const int tok = 16 * tt + g + (e >> 1) * 8;
                        if (tok < M) mine[tok * TILE_ROWS + 16 * warp + 8 * nt + 2 * tq + (e & 1)] = acc[nt][tt][e];
                    }
            __threadfence();
            __syncthreads();
            const int cf = owner_of(t * chunks, U, G);
            const int cl = owner_of((t + 1) * chunks - 1, U, G);
            if (tid == 0) {
                const unsigned old = atomicAdd(&p.counters[t], 1u);
                s_last = (old == (unsigned)(cl - cf)) ? 1 : 0;
            }
            __syncthreads();
            if (s_last) {
                __threadfence();
                // Contributors after the first start inside tile t (slot 0); the
                // first uses slot 0 only if its range starts exactly at the tile.
                const int first_slot = range_begin(cf, U, G) >= t * chunks ? 0 : 1;
                for (int q = tid; q < M * TILE_ROWS; q += kThreads) {
                    const int tok = q >> 7, rr = q & (TILE_ROWS - 1);
                    float a = 0.0f;
                    for (int c2 = cf; c2 <= cl; ++c2) {
                        const int s2 = c2 == cf ? first_slot : 0;
                        a += __ldcg(p.ws + ((size_t)c2 * 2 + s2) * (kMaxMT * TILE_ROWS) + tok * TILE_ROWS + rr);
                    }
                    const int64_t row = (int64_t)t * TILE_ROWS + rr;
                    if (row < N) store_y(p.y, p.y_dtype, tok * N + row, a);
                }
                if (tid == 0) p.counters[t] = 0u;
            }
        }
    }
    cp_wait<0>();
}

bool g_mma_enabled = true;

template <int TYPE, int MT>
int set_attr() {
    using C = Cfg<TYPE, MT>;
    cudaError_t e = cudaFuncSetAttribute(mma_gemv_kernel<TYPE, MT>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         (int)C::smem);
    if (e != cudaSuccess) return cuda_fail(e, "cudaFuncSetAttribute (mma_gemv)");
    return NXQ_OK;
}

template <int TYPE, int MT>
int launch(const Weight* w, const __half* x, void* y, int y_dtype, int64_t M, StreamScratch* sc, int grid,
           cudaStream_t st) {
    MmaParams p;
    p.w = w->dev;
    p.s = w->shape;
    p.x = x;
    p.M = M;
    p.y = y;
    p.y_dtype = y_dtype;
    p.ws = sc->ws;
    p.counters = sc->counters;
    p.units = w->shape.tiles * w->shape.chunks;
    p.grid = grid;
    mma_gemv_kernel<TYPE, MT><<<grid, kThreads, Cfg<TYPE, MT>::smem, st>>>(p);
    cudaError_t e = cudaGetLastError();
    note_launches(1);
    if (e != cudaSuccess) return cuda_fail(e, "mma_gemv launch");
    return NXQ_OK;
}

bool type_ok(int type) { return type == T_Q4_K || type == T_Q4_0 || type == T_Q8_0 || type == T_Q3_K; }

int cps_of(int type, int mt) {
#define NXQ_CPS(T) \
    if (type == T) return mt == 8 ? Cfg<T, 8>::CPS : mt == 16 ? Cfg<T, 16>::CPS : Cfg<T, 32>::CPS;
    NXQ_CPS(T_Q4_K)
    NXQ_CPS(T_Q4_0)
    NXQ_CPS(T_Q8_0)
    NXQ_CPS(T_Q3_K)
#undef NXQ_CPS
    return 1;
}

}  // namespace

int mma_init(int) {
    const char* env = getenv("NXQ_DECODE_KERNEL");
    g_mma_enabled = !(env && env[0] && env[0] != 'm');  // "tc" / "simt" select another decode kernel
    int rc;
#define NXQ_ATTR(T)                                       \
    if ((rc = set_attr<T, 8>()) != NXQ_OK) return rc;  \
    if ((rc = set_attr<T, 16>()) != NXQ_OK) return rc; \
    if ((rc = set_attr<T, 32>()) != NXQ_OK) return rc;
    NXQ_ATTR(T_Q4_K)
    NXQ_ATTR(T_Q4_0)
    NXQ_ATTR(T_Q8_0)
    NXQ_ATTR(T_Q3_K)
#undef NXQ_ATTR
    return NXQ_OK;
}

// Batches of up to 8 tokens: at 9..32 tokens the tcgen05 kernel, whose
// per-instruction cost does not grow with N, is faster (measured).
bool mma_supported(const TiledShape& s, int64_t M) {
    return g_mma_enabled && type_ok(s.type) && M >= 1 && M <= 8;
}

void mma_kernel_name(const TiledShape& s, int64_t M, char* buf, size_t n) {
    snprintf(buf, n, "mma_gemv<%s,m%d>", type_name(s.type), M <= 8 ? 8 : M <= 16 ? 16 : 32);
}

int mma_qmatmul(const Weight* w, const void* x, int x_dtype, void* y, int y_dtype, int64_t M, cudaStream_t st) {
    const TiledShape& s = w->shape;
    if (!mma_supported(s, M)) return NXQ_ERR_UNSUPPORTED;
    const int64_t units = s.tiles * s.chunks;
    const int mt = M <= 8 ? 8 : M <= 16 ? 16 : 32;
    const int cps = cps_of(s.type, mt);
    int grid = cps * context_sm_count();
    if (grid > units) grid = (int)units;
    const bool direct = x_dtype == NXQ_F16 && ((uintptr_t)x % 16) == 0;
    StreamScratch* sc = nullptr;
    int rc = scratch_for(st, (size_t)grid * 2 * kMaxMT * TILE_ROWS, (size_t)s.tiles,
                         direct ? 0 : (size_t)(M * s.K), &sc);
    if (rc) return rc;
    const __half* xh = static_cast<const __half*>(x);
    if (!direct) {
        cudaError_t e = launch_to_half(x, x_dtype, sc->xh, M * s.K, st);
        if (e != cudaSuccess) return cuda_fail(e, "to_half launch");
        xh = sc->xh;
    }
#define NXQ_CASE(T)                                                        \
    case T:                                                                \
        return mt == 8    ? launch<T, 8>(w, xh, y, y_dtype, M, sc, grid, st)  \
               : mt == 16 ? launch<T, 16>(w, xh, y, y_dtype, M, sc, grid, st) \
                          : launch<T, 32>(w, xh, y, y_dtype, M, sc, grid, st);
    switch (s.type) {
        NXQ_CASE(T_Q4_K)
        NXQ_CASE(T_Q4_0)
        NXQ_CASE(T_Q8_0)
        NXQ_CASE(T_Q3_K)
        default:
            return NXQ_ERR_UNSUPPORTED;
    }
#undef NXQ_CASE
}

}  // namespace nxq
