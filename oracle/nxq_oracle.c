/* Test infrastructure: CPU oracle for the quantized-matmul hot path.
 * See nxq_oracle.h for what it restates and how it is pinned.  Built with
 * -ffp-contract=off so every multiply and subtract rounds separately, in the
 * order the reference writes them. */
#include "nxq_oracle.h"

#include <math.h>
#include <pthread.h>
#include <stdlib.h>
#include <string.h>

static uint16_t rd16(const uint8_t* p) { return (uint16_t)(p[0] | (p[1] << 8)); }

static float bits_to_float(uint32_t u) {
    float f;
    memcpy(&f, &u, sizeof f);
    return f;
}

/* gguf_importer.cpp:202-237.  A half with exponent field e and fraction f is
 *   e == 0  : (-1)^s * f * 2^-24           (zero or subnormal; exact in fp32)
 *   e == 31 : sign | all-ones exponent | f << 13   (Inf, NaN with payload)
 *   else    : sign | (e + 112) << 23 | f << 13. */
float nxqo_half_to_float(uint16_t h) {
    uint32_t sign = (uint32_t)(h >> 15) << 31;
    uint32_t e = (h >> 10) & 31u;
    uint32_t f = h & 1023u;
    if (e == 0) {
        float mag = ldexpf((float)f, -24);
        return sign ? -mag : mag;
    }
    if (e == 31) return bits_to_float(sign | 0x7F800000u | (f << 13));
    return bits_to_float(sign | ((e + 112u) << 23) | (f << 13));
}

/* bf16 -> fp32 (gguf_importer.cpp:240-245). */
static float bf16_to_float(uint16_t h) { return bits_to_float((uint32_t)h << 16); }

int nxqo_block_shape(int type, int* elems, int* bytes) {
    int e = 0, b = 0;
    switch (type) {
        case NXQO_F32: e = 1; b = 4; break;
        case NXQO_F16: case NXQO_BF16: e = 1; b = 2; break;
        case NXQO_Q4_0: e = 32; b = 18; break;
        case NXQO_Q4_1: e = 32; b = 20; break;
        case NXQO_Q8_0: e = 32; b = 34; break;
        case NXQO_Q2_K: e = 256; b = 84; break;
        case NXQO_Q3_K: e = 256; b = 110; break;
        case NXQO_Q4_K: e = 256; b = 144; break;
        case NXQO_I4G32: case NXQO_I4G64: case NXQO_I4G128: case NXQO_I4G256:
            e = 32 * (type - 100);
            b = 8 + e / 2;
            break;
        case NXQO_Q5_K: e = 256; b = 176; break;
        case NXQO_Q6_K: e = 256; b = 210; break;
        case NXQO_NXF_I8: e = 32; b = 32; break;
        case NXQO_NXF_F16: e = 32; b = 64; break;
        case NXQO_NXF_F32: e = 32; b = 128; break;
        default: return 0;
    }
    if (elems) *elems = e;
    if (bytes) *bytes = b;
    return 1;
}

/* ---- one block each; `y` receives the block's elements in order ---------- */

/* Q4_0, 18 B / 32 (gguf_importer.cpp:679-695): byte j of the 16 code bytes
 * gives element j (low nibble) and element j+16 (high nibble), minus 8, times d. */
static void blk_q4_0(const uint8_t* b, float* y) {
    float d = nxqo_half_to_float(rd16(b));
    for (int j = 0; j < 16; ++j) {
        int c = b[2 + j];
        y[j] = (float)((c & 15) - 8) * d;
        y[j + 16] = (float)((c >> 4) - 8) * d;
    }
}

/* Q4_1, 20 B / 32 (gguf_importer.cpp:699-717): q * d + m. */
static void blk_q4_1(const uint8_t* b, float* y) {
    float d = nxqo_half_to_float(rd16(b));
    float m = nxqo_half_to_float(rd16(b + 2));
    for (int j = 0; j < 16; ++j) {
        int c = b[4 + j];
        y[j] = (float)(c & 15) * d + m;
        y[j + 16] = (float)(c >> 4) * d + m;
    }
}

/* Q8_0, 34 B / 32 (gguf_importer.cpp:721-733): signed byte times d. */
static void blk_q8_0(const uint8_t* b, float* y) {
    float d = nxqo_half_to_float(rd16(b));
    for (int j = 0; j < 32; ++j) y[j] = (float)(int8_t)b[2 + j] * d;
}

/* Q2_K, 84 B / 256 (gguf_importer.cpp:756-786): 16 groups of 16; byte g of the
 * first 16 holds the group's scale (low nibble) and min (high nibble); 2-bit
 * codes packed four per byte, element e at bits 2*(e%4) of byte 16 + e/4;
 * dmin at 80, d at 82.  y = (d*sc)*q - (dmin*mn). */
static void blk_q2_k(const uint8_t* b, float* y) {
    float dmin = nxqo_half_to_float(rd16(b + 80));
    float d = nxqo_half_to_float(rd16(b + 82));
    for (int g = 0; g < 16; ++g) {
        float s = d * (float)(b[g] & 15);
        float m = dmin * (float)(b[g] >> 4);
        for (int i = 0; i < 16; ++i) {
            int e = 16 * g + i;
            int q = (b[16 + e / 4] >> (2 * (e % 4))) & 3;
            y[e] = s * (float)q - m;
        }
    }
}

/* Q3_K, 110 B / 256 (gguf_importer.cpp:791-833): hmask[32] @0, qs[64] @32,
 * scales[12] @96, d @108.  Sixteen 6-bit group scales (groups of 16): scale i
 * (i<8) takes the low nibble of scales[i], scale i+8 the high nibble, and both
 * take two more bits from scales[8 + i/2]; all are offset by -32.  Element e has
 * 2 low bits at qs[e/4] >> 2*(e%4) and its high bit at hmask[e/8] >> (e%8).
 * y = (d * sc) * (q - 4). */
static void blk_q3_k(const uint8_t* b, float* y) {
    const uint8_t* hm = b;
    const uint8_t* qs = b + 32;
    const uint8_t* sc = b + 96;
    float d = nxqo_half_to_float(rd16(b + 108));
    int s[16];
    for (int i = 0; i < 8; ++i) {
        int hi = sc[8 + i / 2] >> (4 * (i % 2));
        s[i] = ((sc[i] & 15) | ((hi & 3) << 4)) - 32;
        s[i + 8] = ((sc[i] >> 4) | (((hi >> 2) & 3) << 4)) - 32;
    }
    for (int e = 0; e < 256; ++e) {
        int q = ((qs[e / 4] >> (2 * (e % 4))) & 3) | (((hm[e / 8] >> (e % 8)) & 1) << 2);
        y[e] = d * (float)s[e / 16] * ((float)q - 4.0f);
    }
}

/* The 6-bit scale/min unpack shared by Q4_K and Q5_K
 * (gguf_importer.cpp:856-861, :897-902). */
static void unpack_k_scales(const uint8_t* sc, int* s, int* m) {
    for (int i = 0; i < 4; ++i) {
        s[i] = sc[i] & 63;
        s[i + 4] = sc[i + 4] & 63;
        m[i] = (sc[i] >> 6) | ((sc[i + 8] & 15) << 2);
        m[i + 4] = (sc[i + 4] >> 6) | ((sc[i + 8] >> 4) << 2);
    }
}

/* Q4_K, 144 B / 256 (gguf_importer.cpp:838-873): d @0, dmin @2, scales @4,
 * codes @16.  Code byte j gives elements 2j (low nibble) and 2j+1 (high);
 * element e is in sub-block e/32.  y = (d*sc)*q - (dmin*mn). */
static void blk_q4_k(const uint8_t* b, float* y) {
    float d = nxqo_half_to_float(rd16(b));
    float dmin = nxqo_half_to_float(rd16(b + 2));
    int s[8], m[8];
    unpack_k_scales(b + 4, s, m);
    for (int j = 0; j < 128; ++j) {
        int c = b[16 + j];
        int g = (2 * j) / 32;
        y[2 * j] = d * (float)s[g] * (float)(c & 15) - dmin * (float)m[g];
        y[2 * j + 1] = d * (float)s[g] * (float)(c >> 4) - dmin * (float)m[g];
    }
}

/* Q5_K, 176 B / 256 (gguf_importer.cpp:878-915): d @0, dmin @2, scales @4,
 * qh[32] @16, qs[128] @48; the fifth bit of element e is qh[e/8] >> (e%8). */
static void blk_q5_k(const uint8_t* b, float* y) {
    float d = nxqo_half_to_float(rd16(b));
    float dmin = nxqo_half_to_float(rd16(b + 2));
    const uint8_t* qh = b + 16;
    const uint8_t* qs = b + 48;
    int s[8], m[8];
    unpack_k_scales(b + 4, s, m);
    for (int j = 0; j < 128; ++j) {
        for (int h = 0; h < 2; ++h) {
            int e = 2 * j + h;
            int q = (h ? (qs[j] >> 4) : (qs[j] & 15)) | (((qh[e / 8] >> (e % 8)) & 1) << 4);
            int g = e / 32;
            y[e] = d * (float)s[g] * (float)q - dmin * (float)m[g];
        }
    }
}

/* Q6_K, 210 B / 256 (gguf_importer.cpp:924-954): ql[128] @0, qh[64] @128,
 * int8 scales[16] @192, d @208.  y = (d*sc) * (q - 32). */
static void blk_q6_k(const uint8_t* b, float* y) {
    const uint8_t* ql = b;
    const uint8_t* qh = b + 128;
    const int8_t* sc = (const int8_t*)(b + 192);
    float d = nxqo_half_to_float(rd16(b + 208));
    for (int e = 0; e < 256; ++e) {
        int lo = (e & 1) ? (ql[e / 2] >> 4) : (ql[e / 2] & 15);
        int hi = (qh[e / 4] >> (2 * (e % 4))) & 3;
        y[e] = d * (float)sc[e / 16] * ((float)(lo | (hi << 4)) - 32.0f);
    }
}

/* quant/gptq.cpp:9-27: out[i] = ((float)q_i - zero) * scale, q_i nibble i of
 * data (low nibble first), scale/zero of group i / group_size. */
void nxqo_dequant_int4(float* out, const uint8_t* data, const float* scales, const float* zeros,
                       int64_t n, int group_size) {
    for (int64_t i = 0; i < n; ++i) {
        const int64_t g = i / group_size;
        const int q = (i & 1) ? (data[i >> 1] >> 4) & 15 : data[i >> 1] & 15;
        const float zero = zeros ? zeros[g] : 0.0f;
        out[i] = ((float)q - zero) * scales[g];
    }
}

/* One NXF INT4 group block: [scale f32][zero f32][gs/2 code bytes]. */
static void blk_i4g(const uint8_t* b, float* y, int gs) {
    float scale, zero;
    memcpy(&scale, b, 4);
    memcpy(&zero, b + 4, 4);
    nxqo_dequant_int4(y, b + 8, &scale, &zero, gs, gs);
}
static void blk_i4g32(const uint8_t* b, float* y) { blk_i4g(b, y, 32); }
static void blk_i4g64(const uint8_t* b, float* y) { blk_i4g(b, y, 64); }
static void blk_i4g128(const uint8_t* b, float* y) { blk_i4g(b, y, 128); }
static void blk_i4g256(const uint8_t* b, float* y) { blk_i4g(b, y, 256); }

/* NXF INT8 chunk (hybrid_model.cpp:248-255): out = (float)(int8)q / 127.0f. */
static void blk_nxf_i8(const uint8_t* b, float* y) {
    for (int j = 0; j < 32; ++j) y[j] = (float)(int8_t)b[j] / 127.0f;
}

/* NXF FP16 chunk (hybrid_model.cpp:192-210): exponent 0 (zero or subnormal)
 * gives a signed zero; exponent 31 keeps the mantissa (Inf, NaN); otherwise
 * the exponent is rebiased by 112 and the mantissa shifted by 13. */
static void blk_nxf_f16(const uint8_t* b, float* y) {
    for (int j = 0; j < 32; ++j) {
        const uint32_t h = rd16(b + 2 * j), sign = (h & 0x8000u) << 16, e = (h >> 10) & 31u, m = h & 1023u;
        const uint32_t f = e == 0 ? sign : e == 31 ? (sign | 0x7F800000u | (m << 13)) : (sign | ((e + 112u) << 23) | (m << 13));
        y[j] = bits_to_float(f);
    }
}

/* NXF FP32 chunk (hybrid_model.cpp:165-176): the floats as stored. */
static void blk_nxf_f32(const uint8_t* b, float* y) { memcpy(y, b, 128); }

typedef void (*blk_fn)(const uint8_t*, float*);

static blk_fn block_decoder(int type) {
    switch (type) {
        case NXQO_Q4_0: return blk_q4_0;
        case NXQO_Q4_1: return blk_q4_1;
        case NXQO_Q8_0: return blk_q8_0;
        case NXQO_Q2_K: return blk_q2_k;
        case NXQO_Q3_K: return blk_q3_k;
        case NXQO_Q4_K: return blk_q4_k;
        case NXQO_Q5_K: return blk_q5_k;
        case NXQO_Q6_K: return blk_q6_k;
        case NXQO_I4G32: return blk_i4g32;
        case NXQO_I4G64: return blk_i4g64;
        case NXQO_I4G128: return blk_i4g128;
        case NXQO_I4G256: return blk_i4g256;
        case NXQO_NXF_I8: return blk_nxf_i8;
        case NXQO_NXF_F16: return blk_nxf_f16;
        case NXQO_NXF_F32: return blk_nxf_f32;
        default: return NULL;
    }
}

/* gguf_importer.cpp:958-1000: plain types are converted element-wise, block
 * types block by block; n is rounded down to whole blocks as the reference's
 * num_blocks = n / QK does.  Unknown types are zero-filled (:993-998). */
int nxqo_dequant(int type, const uint8_t* src, int64_t n, float* out) {
    if (type == NXQO_F32) { memcpy(out, src, (size_t)n * 4); return 0; }
    if (type == NXQO_F16 || type == NXQO_BF16) {
        for (int64_t i = 0; i < n; ++i) {
            uint16_t h = rd16(src + 2 * i);
            out[i] = type == NXQO_F16 ? nxqo_half_to_float(h) : bf16_to_float(h);
        }
        return 0;
    }
    blk_fn fn = block_decoder(type);
    int qk = 0, bb = 0;
    if (!fn || !nxqo_block_shape(type, &qk, &bb)) {
        memset(out, 0, (size_t)n * 4);
        return -1;
    }
    int64_t nb = n / qk;
    for (int64_t i = 0; i < nb; ++i) fn(src + i * bb, out + i * qk);
    return 0;
}

static int own_decoder(uint32_t type, const uint8_t* src, uint64_t n, float* out) {
    return nxqo_dequant((int)type, src, (int64_t)n, out);
}

/* fp32 dot product with eight interleaved partial sums, the summation shape of
 * a blocked BLAS kernel; every product and sum is an fp32 operation. */
static float dot_f32(const float* a, const float* b, int64_t K) {
    float acc[8] = {0, 0, 0, 0, 0, 0, 0, 0};
    int64_t k = 0;
    for (; k + 8 <= K; k += 8)
        for (int l = 0; l < 8; ++l) acc[l] += a[k + l] * b[k + l];
    float s = 0.0f;
    for (int l = 0; l < 8; ++l) s += acc[l];
    for (; k < K; ++k) s += a[k] * b[k];
    return s;
}

/* Splits [0, count) into nthreads contiguous ranges and runs fn on each in its
 * own pthread (the calling thread takes range 0). */
typedef struct {
    void (*fn)(void* ctx, int64_t lo, int64_t hi);
    void* ctx;
    int64_t lo, hi;
} work_range;

static void* run_range(void* p) {
    work_range* r = (work_range*)p;
    r->fn(r->ctx, r->lo, r->hi);
    return NULL;
}

static void parallel_ranges(int nthreads, int64_t count,
                            void (*fn)(void*, int64_t, int64_t), void* ctx) {
    if (nthreads < 1) nthreads = 1;
    if (nthreads > 256) nthreads = 256;
    if (count < nthreads) nthreads = count > 0 ? (int)count : 1;
    work_range r[256];
    pthread_t th[256];
    int started[256] = {0};
    for (int t = 0; t < nthreads; ++t) {
        r[t].fn = fn;
        r[t].ctx = ctx;
        r[t].lo = count * t / nthreads;
        r[t].hi = count * (t + 1) / nthreads;
    }
    for (int t = 1; t < nthreads; ++t)
        started[t] = pthread_create(&th[t], NULL, run_range, &r[t]) == 0;
    run_range(&r[0]);
    for (int t = 1; t < nthreads; ++t) {
        if (started[t]) pthread_join(th[t], NULL);
        else run_range(&r[t]);
    }
}

typedef struct {
    const float *x, *w;
    float* y;
    int64_t M, N, K;
} gemm_ctx;

static void gemm_rows(void* p, int64_t lo, int64_t hi) {
    gemm_ctx* c = (gemm_ctx*)p;
    for (int64_t n = lo; n < hi; ++n)
        for (int64_t m = 0; m < c->M; ++m)
            c->y[m * c->N + n] = dot_f32(c->x + m * c->K, c->w + n * c->K, c->K);
}

void nxqo_gemm_transb(const float* x, const float* w, float* y,
                      int64_t M, int64_t N, int64_t K, int nthreads) {
    gemm_ctx c = {x, w, y, M, N, K};
    parallel_ranges(nthreads, N, gemm_rows, &c);
}

/* Rows are decoded in batches so each decoder call covers many blocks, as the
 * reference's whole-tensor decode does. */
#define ROWS_PER_BATCH 16

typedef struct {
    nxqo_decoder_fn decoder;
    int type;
    const uint8_t* blocks;
    int64_t N, K, M, row_bytes;
    const float* x;
    float* y;
    int bad;
    pthread_mutex_t mu;
} qmm_ctx;

static void qmm_batches(void* p, int64_t lo, int64_t hi) {
    qmm_ctx* c = (qmm_ctx*)p;
    float* w = (float*)malloc((size_t)(ROWS_PER_BATCH * c->K) * sizeof(float));
    int bad = w == NULL;
    for (int64_t t = lo; t < hi && w; ++t) {
        int64_t n0 = t * ROWS_PER_BATCH;
        int64_t nr = c->N - n0 < ROWS_PER_BATCH ? c->N - n0 : ROWS_PER_BATCH;
        if (c->decoder((uint32_t)c->type, c->blocks + n0 * c->row_bytes,
                       (uint64_t)(nr * c->K), w) != 0)
            bad = 1;
        for (int64_t r = 0; r < nr; ++r)
            for (int64_t m = 0; m < c->M; ++m)
                c->y[m * c->N + n0 + r] = dot_f32(c->x + m * c->K, w + r * c->K, c->K);
    }
    free(w);
    if (bad) {
        pthread_mutex_lock(&c->mu);
        c->bad = 1;
        pthread_mutex_unlock(&c->mu);
    }
}

int nxqo_qmatmul(nxqo_decoder_fn decoder, int type, const uint8_t* blocks,
                 int64_t N, int64_t K, const float* x, int64_t M, float* y,
                 int nthreads) {
    int qk = 0, bb = 0;
    if (!nxqo_block_shape(type, &qk, &bb) || qk == 1 || K <= 0 || N < 0 || M < 0 || K % qk)
        return -1;
    qmm_ctx c;
    c.decoder = decoder ? decoder : own_decoder;
    c.type = type;
    c.blocks = blocks;
    c.N = N; c.K = K; c.M = M;
    c.row_bytes = (K / qk) * bb;
    c.x = x; c.y = y;
    c.bad = 0;
    pthread_mutex_init(&c.mu, NULL);
    parallel_ranges(nthreads, (N + ROWS_PER_BATCH - 1) / ROWS_PER_BATCH, qmm_batches, &c);
    pthread_mutex_destroy(&c.mu);
    return c.bad ? -1 : 0;
}
