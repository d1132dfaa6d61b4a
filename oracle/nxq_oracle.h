/* Test infrastructure: CPU oracle for the quantized-matmul hot path.
 *
 * A plain-C restatement of the reference's GGUF block decoders
 * (nexus/src/import/gguf_importer.cpp) and of its fp32 matmul semantics
 * (nexus/src/compute/accelerate/gemm.cpp:16-41, used with transB=true as in
 * nexus/src/model/transformer.cpp:249-253).  It exists to check the CUDA path;
 * it is never the thing measured or shipped.  Only tests/,
 * __graft_entry__.smoke() and bench.py's CPU-baseline leg may load it.
 *
 * Parity pins:
 *   - decoders: pinned bit-for-bit against the reference's own decoders,
 *     compiled from the reference sources into oracle/_ref/ (oracle/Makefile),
 *     and against the committed fixtures in tests/golden/.
 *   - matmul: the reference's matmul is Apple Accelerate cblas_sgemm, which is
 *     closed and absent here; no reference test pins its outputs.  The fp32
 *     GEMM below restates its documented semantics (row-major, alpha=1,
 *     beta=0) and is "parity unpinned" beyond that.
 */
#ifndef NXQ_ORACLE_H
#define NXQ_ORACLE_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* GGUF type ids (nexus/src/import/gguf_importer.h:28-57). */
enum {
    NXQO_F32 = 0, NXQO_F16 = 1, NXQO_Q4_0 = 2, NXQO_Q4_1 = 3, NXQO_Q8_0 = 8,
    NXQO_Q2_K = 10, NXQO_Q3_K = 11, NXQO_Q4_K = 12, NXQO_Q5_K = 13,
    NXQO_Q6_K = 14, NXQO_BF16 = 30,
    /* NXF INT4 groups of 32/64/128/256 as blocks [scale f32][zero f32][codes]
     * (the library's NXQ_TYPE_I4G*; quant/gptq.cpp:9-27 per group) */
    NXQO_I4G32 = 101, NXQO_I4G64 = 102, NXQO_I4G128 = 104, NXQO_I4G256 = 108,
    /* NXF chunks decoded at load time by HybridModel::Impl::load_tensor
     * (hybrid_model.cpp:145-265), as blocks of 32 elements (the library's
     * NXQ_TYPE_NXF_*): INT8 (float)q / 127.0f; FP16 with subnormals read as
     * zero; FP32 as stored */
    NXQO_NXF_I8 = 120, NXQO_NXF_F16 = 121, NXQO_NXF_F32 = 122
};

/* quant/gptq.cpp:9-27, dequant_int4, over flat arrays: element i is nibble i of
 * data (low nibble first), out[i] = ((float)q - zero[g]) * scale[g] with
 * g = i / group_size (zeros NULL: 0). */
void nxqo_dequant_int4(float* out, const uint8_t* data, const float* scales, const float* zeros,
                       int64_t n, int group_size);

/* Elements per block and bytes per block for `type`; returns 0 if unknown. */
int nxqo_block_shape(int type, int* elems, int* bytes);

/* IEEE half -> float, subnormals kept, Inf/NaN payload kept
 * (gguf_importer.cpp:202-237). */
float nxqo_half_to_float(uint16_t h);

/* Decode `n` elements of `type` blocks to fp32 (gguf_importer.cpp:958-1000).
 * Returns 0, or -1 for a type the reference zero-fills. */
int nxqo_dequant(int type, const uint8_t* src, int64_t n, float* out);

/* y[m][n] = sum_k x[m][k] * w[n][k], fp32 accumulate (gemm.cpp:16-41, transB). */
void nxqo_gemm_transb(const float* x, const float* w, float* y,
                      int64_t M, int64_t N, int64_t K, int nthreads);

/* Signature of a block decoder: the oracle's own (nxqo_dequant, wrapped) or the
 * reference's compiled one (oracle/_ref: ref_dequant). */
typedef int (*nxqo_decoder_fn)(uint32_t type, const uint8_t* src, uint64_t n, float* out);

/* The reference CPU path, row-streamed to bound memory: decode each weight row
 * (load_tensor, hybrid_model.cpp:145-265) with `decoder` (NULL = this oracle),
 * then fp32 dot products against x (gemm_f32, gemm.cpp:16-41).  W is [N][K]
 * rows of blocks.  Returns 0, or -1 on a bad type/shape. */
int nxqo_qmatmul(nxqo_decoder_fn decoder, int type, const uint8_t* blocks,
                 int64_t N, int64_t K, const float* x, int64_t M, float* y,
                 int nthreads);

#ifdef __cplusplus
}
#endif
#endif
