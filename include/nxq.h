/* nxq.h — C ABI of the B200 quantized-matmul library (libnxq.so).
 *
 * Drop-in replacement for the NEXUS engine's quantized-matmul operator path:
 *   ComputeDispatch::gemm_int4 / gemv_int4   nexus/src/compute/compute_dispatch.h:47-61
 *   MetalBackend::gemv_int4_nr8 / gemm_int4_gpu / wrap_pointer
 *                                            nexus/src/compute/metal/metal_backend.h:60-87
 * applied to GGUF block-quantized weights (Q4_0, Q8_0, Q4_K, Q3_K, ...) whose
 * values are defined by nexus/src/import/gguf_importer.cpp:677-1000, and to
 * the NXF INT4 group format (nexus/src/quant/gptq.cpp:9-70).  Weights reach
 * HBM from host arrays (nxq_weight_register*), GGUF files (nxq_gguf_*) or NXF
 * files (nxq_nxf_*).
 *
 * Conventions
 *   - Plain C types only; every call returns an nxq_status (0 = ok, < 0 error)
 *     and records a message readable with nxq_last_error().
 *   - A weight W is logically [N][K] (N output rows, K reduction), row-major,
 *     blocks contiguous along K: the GGUF tensor order, used by the reference
 *     as gemm_f32(..., transB=true) (nexus/src/model/transformer.cpp:249-253).
 *   - y[M][N] = x[M][K] * W^T, fp32 accumulation.
 *   - "device" pointers are CUDA device pointers on the current nxq device;
 *     `stream` is a cudaStream_t (NULL = the legacy default stream).
 *   - One context per process per device (nxq_init); calls on distinct streams
 *     may run concurrently; weight registration and release are serialized
 *     internally.
 */
#ifndef NXQ_H
#define NXQ_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#if defined(__GNUC__)
#define NXQ_API __attribute__((visibility("default")))
#else
#define NXQ_API
#endif

#define NXQ_ABI_VERSION 1

/* Status codes.  The reference returns void from ComputeDispatch and silently
 * zero-fills on failure (compute_dispatch.cpp:174-176); here every failure is a
 * negative code, and zero-filling is only an opt-in of the C++ shim. */
typedef enum {
    NXQ_OK = 0,
    NXQ_ERR_ARG = -1,         /* null pointer, negative size, bad enum value   */
    NXQ_ERR_CODEC = -2,       /* block type not supported by this entry point  */
    NXQ_ERR_SHAPE = -3,       /* K not a multiple of the block, bytes mismatch */
    NXQ_ERR_CUDA = -4,        /* a CUDA runtime/driver call failed             */
    NXQ_ERR_TIMEOUT = -5,     /* a bounded device-side wait ran out            */
    NXQ_ERR_NOMEM = -6,       /* device or host allocation failed              */
    NXQ_ERR_STATE = -7,       /* not initialised / wrong device / TP not set up */
    NXQ_ERR_NCCL = -8,        /* NCCL unavailable or a collective failed       */
    NXQ_ERR_UNSUPPORTED = -9, /* no GPU of the required architecture           */
    NXQ_ERR_FORMAT = -10,     /* a GGUF / NXF file that is malformed or truncated */
    NXQ_ERR_RANGE = -11       /* an activation outside the f16 range (see below) */
} nxq_status;

/* Numeric range of the tensor-core kernels.  The decode GEMV and the prefill
 * GEMM multiply in f16 with fp32 accumulation: f16 activations are used as
 * they are, fp32 and bf16 activations are rounded to f16 first (the reference
 * keeps them in fp32).  A finite activation of magnitude >= 65520 has no f16
 * value; the kernel that rounds it records NXQ_ERR_RANGE in the context's
 * status word, which the next nxq_stream_sync (or the synchronous
 * nxq_qmatmul_host) returns, and that call's outputs are not finite.  The
 * CUDA-core kernel (NXQ_DECODE_KERNEL=simt / NXQ_PREFILL_KERNEL=simt, and
 * nxq_qmatmul_noalloc) computes in fp32 and has no such limit. */

/* Block types: the GGUF type ids of nexus/src/import/gguf_importer.h:28-57,
 * and the NXF INT4 group format (quant/gptq.cpp:9-70: w = (q - zero) * scale,
 * one fp32 scale and zero per group of gs elements along K) as blocks of one
 * group, [scale f32][zero f32][gs/2 code bytes: element 2i in the low, 2i+1
 * in the high nibble of byte i], ids 100 + gs/32 (outside the GGUF range). */
typedef enum {
    NXQ_TYPE_Q4_0 = 2,
    NXQ_TYPE_Q4_1 = 3,
    NXQ_TYPE_Q8_0 = 8,
    NXQ_TYPE_Q2_K = 10,
    NXQ_TYPE_Q3_K = 11,
    NXQ_TYPE_Q4_K = 12,
    NXQ_TYPE_Q5_K = 13,
    NXQ_TYPE_Q6_K = 14,
    NXQ_TYPE_I4G32 = 101,
    NXQ_TYPE_I4G64 = 102,
    NXQ_TYPE_I4G128 = 104,
    NXQ_TYPE_I4G256 = 108,
    /* NXF chunks the reference's engine decodes at load time
     * (HybridModel::Impl::load_tensor, hybrid_model.cpp:145-265), as blocks of
     * 32 consecutive elements along K of the chunk's flat [N][K] array:
     *   NXQ_TYPE_NXF_I8   Codec::INT8: 32 int8 codes, w = (float)q / 127
     *                     (hybrid_model.cpp:248-255); decode GEMV and prefill
     *                     GEMM as Q8_0 with the scale fl16(1/127)
     *   NXQ_TYPE_NXF_F16  Codec::FP16: 32 halves, subnormals read as zero
     *                     (hybrid_model.cpp:192-210); CUDA-core kernel
     *   NXQ_TYPE_NXF_F32  Codec::FP32, or any chunk of 4 bytes per element
     *                     (hybrid_model.cpp:165-176): 32 floats; CUDA-core kernel */
    NXQ_TYPE_NXF_I8 = 120,
    NXQ_TYPE_NXF_F16 = 121,
    NXQ_TYPE_NXF_F32 = 122
} nxq_type;

/* Activation / output element types: nexus::DType F32=0, F16=1, BF16=2
 * (nexus/src/core/config.h:39-46). */
typedef enum { NXQ_F32 = 0, NXQ_F16 = 1, NXQ_BF16 = 2 } nxq_dtype;

/* Tensor-parallel split of one projection (north-star TP; the reference has no
 * multi-device path).  COL: rank r owns output rows [r*N/T, (r+1)*N/T).  ROW:
 * rank r owns reduction columns [r*K/T, (r+1)*K/T) of every row and the
 * partial outputs are summed with an allreduce. */
typedef enum { NXQ_SPLIT_COL = 0, NXQ_SPLIT_ROW = 1 } nxq_split;

/* Opaque handle to HBM-resident packed weights.  Replaces the reference's
 * MetalBackend::buffer_id from wrap_pointer over mmap'd chunks
 * (metal_backend.h:40, metal_backend.mm:814-834; compute_dispatch.cpp:147-154). */
typedef struct nxq_weight_s* nxq_weight_t;

/* ---- context -------------------------------------------------------------- */

/* Select `device`, check it is sm_100, create the context.  Replaces
 * ComputeDispatch::init_gpu (compute_dispatch.cpp:47).  Idempotent per device. */
NXQ_API int nxq_init(int device);

/* Release every registered weight, scratch buffer and TP communicator. */
NXQ_API int nxq_shutdown(void);

/* Copy the calling thread's last error message (NUL-terminated, truncated to n). */
NXQ_API int nxq_last_error(char* buf, size_t n);

/* NXQ_ABI_VERSION of the loaded library. */
NXQ_API int nxq_abi_version(void);

/* Block geometry of `type`: elements per block and bytes per block
 * (gguf_importer.cpp:291-345, with Q3_K's decoder size of 110 bytes, :797). */
NXQ_API int nxq_block_geometry(int type, int* block_elems, int* block_bytes);

/* ---- weight residency ----------------------------------------------------- */

/* Upload `bytes` of GGUF blocks (N rows of K/QK blocks) from host memory and
 * keep them resident in HBM in the library's tiled layout.  Replaces
 * wrap_pointer + wrapped_buffer_cache_ (compute_dispatch.cpp:147-154): the
 * device owns the copy and the host buffer may be freed after return.
 * bytes must equal N * (K/QK) * block_bytes. */
NXQ_API int nxq_weight_register(const void* host_blocks, size_t bytes, int type,
                                int64_t N, int64_t K, nxq_weight_t* out);

/* As nxq_weight_register, from GGUF blocks already in device memory (for
 * loaders that stage on the GPU).  Stream-ordered on `stream`; returns after
 * the tiled copy is complete. */
NXQ_API int nxq_weight_register_device(const void* dev_blocks, size_t bytes, int type,
                                       int64_t N, int64_t K, void* stream,
                                       nxq_weight_t* out);

/* Register only this rank's shard of a full host weight for tensor parallelism:
 * COL keeps rows [r*N/T, (r+1)*N/T); ROW keeps, for every row, the blocks of
 * columns [r*K/T, (r+1)*K/T).  N/T (COL) or K/T (ROW) must divide evenly and
 * K/T must be a multiple of the block size. */
NXQ_API int nxq_weight_register_shard(const void* host_blocks, size_t bytes, int type,
                                      int64_t N, int64_t K, int split, int rank,
                                      int world, nxq_weight_t* out);

/* Host-only (no GPU needed): copy rank `rank`'s shard of a full GGUF weight
 * into `out` (out_bytes must be bytes / world), still in GGUF row-major block
 * order, under the same COL/ROW rules as nxq_weight_register_shard.  For
 * loaders that slice before upload or ship shards to other hosts. */
NXQ_API int nxq_shard_extract(const void* host_blocks, size_t bytes, int type, int64_t N,
                              int64_t K, int split, int rank, int world, void* out,
                              size_t out_bytes);

/* NXF INT4 group weights from their separate arrays (the operands of
 * ComputeDispatch::gemv_int4, compute_dispatch.h:47-49): packed 4-bit codes,
 * fp32 scales and zeros (zeros may be NULL: zero 0) for groups of group_size
 * (32, 64, 128 or 256; a divisor of K) elements along K.  `layout` says how the
 * arrays are ordered:
 *   NXQ_INT4_ROWS   quant/gptq.cpp's flat order over W[N][K]: element (n, k) is
 *                   nibble (n*K + k) of codes (low nibble first), group
 *                   (n*K + k) / group_size of scales and zeros;
 *   NXQ_INT4_KMAJOR gemv_dequant_int4's order (gemm_dequant.metal:29-70): codes
 *                   [K/2][N], byte (k/2)*N + n holding k (low) and k+1 (high);
 *                   scales, zeros [K/group_size][N].
 * nxq_int4_pack (host only, no GPU) writes the NXQ_TYPE_I4G<gs> blocks [N][K/gs]
 * into out (out_bytes = N * (K/gs) * (8 + gs/2)); nxq_weight_register_int4 packs
 * and registers them. */
typedef enum { NXQ_INT4_ROWS = 0, NXQ_INT4_KMAJOR = 1 } nxq_int4_layout;
NXQ_API int nxq_int4_pack(const uint8_t* codes, const float* scales, const float* zeros, int64_t N,
                          int64_t K, int group_size, int layout, void* out, size_t out_bytes);
NXQ_API int nxq_weight_register_int4(const uint8_t* codes, const float* scales, const float* zeros,
                                     int64_t N, int64_t K, int group_size, int layout,
                                     nxq_weight_t* out);

/* Free the HBM copy (ComputeDispatch::clear_buffer_cache, compute_dispatch.cpp:853-860). */
NXQ_API int nxq_weight_release(nxq_weight_t w);

/* Shape and footprint of a registered weight (any pointer may be NULL). */
NXQ_API int nxq_weight_info(nxq_weight_t w, int* type, int64_t* N, int64_t* K,
                            size_t* packed_bytes, size_t* device_bytes);

/* ---- compute ---------------------------------------------------------------- */

/* Decode the whole weight to fp32 y_dev[N][K], bit-identical to
 * dequant_gguf_to_fp32 (gguf_importer.cpp:958-1000).  Stream-ordered. */
NXQ_API int nxq_dequant(nxq_weight_t w, float* y_dev, void* stream);

/* y_dev[M][N] = x_dev[M][K] * W^T on `stream`, fp32 accumulation.
 * x_dtype, y_dtype in nxq_dtype.  Device-resident form of
 * MetalBackend::gemm_int4_gpu (metal_backend.h:86-87) with M honoured and the
 * block codec taken from the weight.  M >= 1; any M is accepted (decode and
 * prefill shapes share this entry point).  The first call on a stream
 * allocates that stream's scratch (partial sums of row tiles shared between
 * CTAs, an f16 copy of non-f16 activations); a call captured into a CUDA
 * graph cannot allocate, so make one call of the largest shape on the stream
 * before capturing (the decode GEMV then splits without scratch, slower). */
NXQ_API int nxq_qmatmul(nxq_weight_t w, const void* x_dev, int x_dtype, void* y_dev,
                        int y_dtype, int64_t M, void* stream);

/* Allocation-free form of nxq_qmatmul, for callers that must not allocate GPU
 * memory during the call: allocator or memory-pool callbacks, latency-critical
 * loops that cannot afford cudaMalloc's implicit synchronization, and hosts
 * that reserve all GPU memory up front.  It has no counterpart in the
 * reference.  It always runs the exact-decode CUDA-core kernel and keeps that
 * kernel's split-K partial sums in one fixed 8 MiB device array that every
 * GPU loading the library holds until exit; M * N may not exceed 2^21
 * (NXQ_ERR_SHAPE otherwise).  The first call on a device looks up the array's
 * device address, so make that first call before any stream capture.  All
 * calls share the array: calls that may overlap on the GPU (on different
 * streams) race, and the caller must order them.  Same arguments, dtypes and
 * results (within the matmul tolerance) as nxq_qmatmul. */
NXQ_API int nxq_qmatmul_noalloc(nxq_weight_t w, const void* x_dev, int x_dtype, void* y_dev,
                                int y_dtype, int64_t M, void* stream);

/* Several projections in as few launches as possible: y_dev[i][M[i]][N_i] =
 * x_dev[i][M[i]][K_i] * W_i^T for i < count, on `stream`.  The grouped/MoE
 * GEMV: all active experts of a layer (batched_moe_ffn's single dispatch,
 * compute_dispatch.cpp:211-275, batched_expert_gemv.metal:47-160), or the
 * projections that share an input (q/k/v, gate/up) - the caller passes the same
 * x_dev for those.  Weights of one block type with 1 <= M[i] <= 32 and f16
 * activations (fp32/bf16 with M[i] <= 2) run as one decode launch per 16
 * weights; anything else runs as nxq_qmatmul calls in order.  M[i] = 0 skips
 * item i.  Results within the matmul tolerance of separate nxq_qmatmul calls. */
NXQ_API int nxq_qmatmul_grouped(const nxq_weight_t* w, int count, const void* const* x_dev,
                                int x_dtype, void* const* y_dev, int y_dtype, const int64_t* M,
                                void* stream);

/* Fused epilogues (the reference's fused_ffn_int4.metal:120-123 and
 * activations.metal:51, after its gate/up and projection GEMVs):
 *   nxq_qmatmul_swiglu:   h_dev[M][N] = silu(x Wg^T) * (x Wu^T), silu(g) = g / (1 + exp(-g)),
 *                         for gate and up weights of the same shape and type;
 *                         one decode launch for M <= 32 (a row tile's gate and
 *                         up tile-chunks are one run of units, a tile shared
 *                         by several CTAs finished by one of them), else gate
 *                         and up, then one small kernel.
 *   nxq_qmatmul_residual: y_dev[M][N] = x W^T + res_dev[M][N] (fp32 residual;
 *                         y_dev may be res_dev), added before the decode
 *                         kernel's store, else by a small kernel after it.
 * Results within the matmul tolerance of the unfused computation. */
NXQ_API int nxq_qmatmul_swiglu(nxq_weight_t w_gate, nxq_weight_t w_up, const void* x_dev, int x_dtype,
                               void* h_dev, int h_dtype, int64_t M, void* stream);
NXQ_API int nxq_qmatmul_residual(nxq_weight_t w, const void* x_dev, int x_dtype, const float* res_dev,
                                 void* y_dev, int y_dtype, int64_t M, void* stream);

/* Fused RMSNorm prologue (fused_qkv_int4.metal:50-71): every token row of x_dev
 * [M][K] is normalized once, xn = x * r * norm_dev with r = 1/sqrt(sum(x^2)/K +
 * eps) (fp32, rounded to f16), and y_dev[i] = xn W_i^T for the `count` weights
 * that take it (q/k/v: count 3; all of equal K), as one normalization kernel
 * and one grouped decode launch (M <= 32; nxq_qmatmul calls beyond). */
NXQ_API int nxq_rmsnorm_qmatmul(const nxq_weight_t* w, int count, const void* x_dev, int x_dtype,
                                const float* norm_dev, float eps, void* const* y_dev, int y_dtype,
                                int64_t M, void* stream);

/* Host-buffer form, synchronous: the drop-in for ComputeDispatch::gemm_int4
 * (compute_dispatch.h:59-61, .cpp:142-176) - fp32 activations [M][K] in, fp32
 * output [M][N] out, weights resident.  The reference ignores M
 * (compute_dispatch.cpp:156-164); here every row of x is used. */
NXQ_API int nxq_qmatmul_host(nxq_weight_t w, const float* x_host, float* y_host, int64_t M);

/* Block until all work nxq queued on `stream` is done; reports the first
 * device-side error recorded since the last report: a bounded wait that ran
 * out (NXQ_ERR_TIMEOUT) or an activation outside the f16 range
 * (NXQ_ERR_RANGE). */
NXQ_API int nxq_stream_sync(void* stream);

/* Limit of every bounded device-side wait on another thread's progress (a
 * copy landing, a stream-K partial sum arriving), in microseconds; 0 restores
 * the default of about 2 s.  A wait that runs out ends its kernel with
 * NXQ_ERR_TIMEOUT at the next nxq_stream_sync instead of hanging the GPU; a
 * short limit detects a lost arrival sooner.  Synchronizes the device.  No
 * counterpart in the reference (its Metal command buffers have no
 * device-side waits). */
NXQ_API int nxq_set_wait_limit(uint64_t microseconds);

/* Test hooks for failure-detection tests: they make a bounded wait run out on
 * purpose (nothing faults, traps or waits beyond the limit).  Off by default;
 * each call synchronizes the device.
 *   NXQ_HOOK_STREAMK_SKIP_COUNT: in the decode GEMV's stream-K split, the CTAs
 *     that publish a partial sum of a row tile another CTA finishes do not
 *     count themselves in, so that CTA's wait for the counts runs out
 *     (NXQ_ERR_TIMEOUT; that call's output is incomplete).  No counterpart in
 *     the reference. */
typedef enum { NXQ_HOOK_STREAMK_SKIP_COUNT = 1, NXQ_HOOK_TP_STREAM_PENDING = 2 } nxq_test_hook_id;
NXQ_API int nxq_test_hook(int hook, int on);

/* Name of the kernel nxq_qmatmul would launch for (w, M, dtypes), e.g.
 * "mma_gemv<Q4_K,m8>", "tc_gemm<Q4_K,n256>" or "simt<Q3_K,mb8>".  Profiling aid; the reference's
 * counterpart is the pipeline-name log of metal_context_impl.h:77-78. */
NXQ_API int nxq_qmatmul_kernel_name(nxq_weight_t w, int64_t M, int x_dtype, int y_dtype,
                                    char* buf, size_t n);

/* Number of kernels libnxq has launched in this process so far. */
NXQ_API int nxq_launch_count(uint64_t* out);

/* ---- tensor parallelism (NCCL over NVLink) -------------------------------- */

/* Size in bytes of the opaque id nxq_tp_unique_id writes (ncclUniqueId). */
NXQ_API int nxq_tp_unique_id_size(void);

/* Rank 0 creates the id and shares it out of band (e.g. torch.distributed). */
NXQ_API int nxq_tp_unique_id(void* out, size_t n);

/* Join the TP group (ncclCommInitRank) on the current nxq device. */
NXQ_API int nxq_tp_init(int rank, int world, const void* unique_id, size_t n);

/* Tear down the TP communicator. */
NXQ_API int nxq_tp_shutdown(void);

/* One sharded projection on `stream`.
 *   COL: x_dev is the full [M][K]; y_dev receives this rank's [M][N/T] slice.
 *   ROW: x_dev is this rank's [M][K/T] slice; y_dev receives the full [M][N]
 *        sum over ranks (in-place NCCL allreduce of the fp32 partials).
 * y_dtype NXQ_F32 only for ROW (the allreduce runs in fp32).
 * By default (NXQ_TP_ALLREDUCE unset or "fused" when nxq_tp_init runs, 2 to
 * 8 ranks), a ROW call of 1 <= M <= 32 tokens and at most 65536 output rows
 * runs as ONE kernel per rank instead of a matmul and an allreduce: the
 * decode GEMV writes each finished 128-row tile's fp32 partials into every
 * rank's exchange buffer (plain NVLink stores into buffers mapped through
 * CUDA IPC at nxq_tp_init; each value with the launch's tag in one 8-byte
 * word), then reads the ranks' partials of its tiles from its own buffer,
 * waiting (bounded by nxq_set_wait_limit; NXQ_ERR_TIMEOUT) until each word
 * carries the launch's tag, and stores their sum in rank order (the same bits
 * on every rank).  With NXQ_TP_EXCHANGE=owner the exchange has tile owners
 * instead: rank r sends its partials of tile t only to rank t mod world,
 * which sums the ranks' partials in rank order and sends the sum back
 * (2 (world-1)/world of the output per rank instead of world-1 times it,
 * over two hops).  Calls whose exchange would
 * exceed 8 MB per rank use NCCL.  Every rank must issue the same sequence of
 * ROW calls, on one stream per rank.  NXQ_TP_ALLREDUCE=nccl keeps every ROW
 * call on NCCL. */
NXQ_API int nxq_tp_qmatmul(nxq_weight_t shard, const void* x_dev, int x_dtype, void* y_dev,
                           int y_dtype, int64_t M, int split, void* stream);

/* Sum `count` fp32 values across the TP group in place on `stream`, by
 * ncclAllReduce.  With NXQ_TP_ALLREDUCE=p2p set when nxq_tp_init runs, sums
 * of up to 2^21 values (8 MB) run instead as one kernel over NVLink peer
 * memory: every rank's symmetric buffer is mapped by the others through CUDA
 * IPC at nxq_tp_init (the handles travel over the NCCL communicator), each
 * rank copies its partial into its own buffer, raises per-slice ready flags
 * in the peers' buffers, waits (bounded) for theirs and adds the ranks'
 * slices in rank order, so every rank gets the same bits (measured slower
 * than NCCL on two B200, hence not the default).  Like NCCL collectives, every
 * rank issues the same sequence of allreduces; the peer-memory path also
 * wants one rank's allreduces on one stream (they share the buffers).  A
 * collective that fails to enqueue aborts the communicator (NXQ_ERR_NCCL). */
NXQ_API int nxq_tp_allreduce_f32(float* buf_dev, int64_t count, void* stream);

/* Which peer-memory path this rank uses: 2 = decode ROW calls fused with
 * their reduction (the default), 1 = allreduces up to 8 MB over peer memory
 * (NXQ_TP_ALLREDUCE=p2p), 0 = NCCL only (NXQ_TP_ALLREDUCE=nccl, one rank, or
 * buffers that could not be mapped). */
NXQ_API int nxq_tp_p2p_enabled(int* on);

/* Failure detection for the TP group (the reference has one device and
 * zero-fills silently, compute_dispatch.cpp:174-176): waits until the work
 * queued on `stream` (matmuls and allreduces) has finished, polling the stream
 * and ncclCommGetAsyncError.  If NCCL reports an error, the stream fails, or
 * timeout_ms passes first (a peer that left never joins its collective), the
 * communicator is aborted (ncclCommAbort, which ends the NCCL kernels still
 * waiting) and NXQ_ERR_NCCL / NXQ_ERR_CUDA / NXQ_ERR_TIMEOUT is returned; from
 * then on every TP call returns NXQ_ERR_STATE until nxq_tp_shutdown and a new
 * nxq_tp_init.  Every TP call also checks for a pending asynchronous NCCL
 * error first.  Host-only logic apart from the stream query. */
NXQ_API int nxq_tp_wait(void* stream, int64_t timeout_ms);

/* Host-side test hook of the TP layer (needs no GPU):
 *   NXQ_HOOK_TP_STREAM_PENDING: nxq_tp_wait sees the stream as still running,
 *     as it would while a collective waits for a peer that left, so its
 *     deadline path runs. */
NXQ_API int nxq_tp_test_hook(int hook, int on);

/* ---- residency loader: GGUF v2/v3 files straight into HBM ---------------------
 * Replaces the reference's import path (GGUFImporter::parse_gguf,
 * gguf_importer.cpp:359-455: header, metadata key/values, tensor index, data
 * section aligned to general.alignment, default 32) followed by mmap +
 * wrap_pointer streaming (compute_dispatch.cpp:142-154): the file is mapped
 * read-only, every field is bounds-checked against the file size, and a
 * tensor's blocks go from the mapping to the tiled HBM copy in one
 * registration.  Parsing needs no GPU; registration needs nxq_init.  Metadata
 * arrays are skipped (their element type and count are kept), as the
 * reference does.  A malformed or truncated file is NXQ_ERR_FORMAT. */
typedef struct nxq_gguf_s* nxq_gguf_t;

/* GGUF metadata value types (GGUFValueType, gguf_importer.h:60-74). */
typedef enum {
    NXQ_GGUF_U8 = 0, NXQ_GGUF_I8 = 1, NXQ_GGUF_U16 = 2, NXQ_GGUF_I16 = 3,
    NXQ_GGUF_U32 = 4, NXQ_GGUF_I32 = 5, NXQ_GGUF_F32 = 6, NXQ_GGUF_BOOL = 7,
    NXQ_GGUF_STRING = 8, NXQ_GGUF_ARRAY = 9, NXQ_GGUF_U64 = 10, NXQ_GGUF_I64 = 11,
    NXQ_GGUF_F64 = 12
} nxq_gguf_value_type;

NXQ_API int nxq_gguf_open(const char* path, nxq_gguf_t* out);
NXQ_API int nxq_gguf_close(nxq_gguf_t g);

/* Format version (2 or 3), data-section alignment and offset. */
NXQ_API int nxq_gguf_header(nxq_gguf_t g, uint32_t* version, uint64_t* alignment,
                            uint64_t* data_start);

NXQ_API int nxq_gguf_tensor_count(nxq_gguf_t g, int64_t* n);

/* Tensor i of the index: name (NUL-terminated, truncated to name_len), GGUF type
 * id, dims (dims[0] is the fastest-varying; up to 4, unused ones 1), offset from
 * the data section and size in bytes (0 for a type nxq does not know). */
NXQ_API int nxq_gguf_tensor_info(nxq_gguf_t g, int64_t i, char* name, size_t name_len, int* type,
                                 int* n_dims, int64_t dims[4], uint64_t* offset, uint64_t* bytes);

/* Index of the tensor called `name`; NXQ_ERR_ARG if there is none. */
NXQ_API int nxq_gguf_find(nxq_gguf_t g, const char* name, int64_t* index);

/* Host pointer to tensor i's bytes inside the mapping (valid until close). */
NXQ_API int nxq_gguf_tensor_data(nxq_gguf_t g, int64_t i, const void** data, uint64_t* bytes);

/* Metadata: key i and its value type; scalar values by key (integers and bool
 * as uint64 / int64, floats as double), strings (NUL-terminated, truncated to
 * n), and an array's element type and length. */
NXQ_API int nxq_gguf_meta_count(nxq_gguf_t g, int64_t* n);
NXQ_API int nxq_gguf_meta_key(nxq_gguf_t g, int64_t i, char* key, size_t n, int* value_type);
NXQ_API int nxq_gguf_meta_uint(nxq_gguf_t g, const char* key, uint64_t* v);
NXQ_API int nxq_gguf_meta_int(nxq_gguf_t g, const char* key, int64_t* v);
NXQ_API int nxq_gguf_meta_float(nxq_gguf_t g, const char* key, double* v);
NXQ_API int nxq_gguf_meta_string(nxq_gguf_t g, const char* key, char* buf, size_t n);
NXQ_API int nxq_gguf_meta_array(nxq_gguf_t g, const char* key, int* elem_type, uint64_t* count);

/* Register tensor i as a weight [N][K]: K = dims[0], N = dims[1] (2-D, or higher
 * dimensions of size 1).  For a 3-D tensor [E][N][K] (stacked experts) `slice`
 * picks expert `slice`; pass 0 otherwise. */
NXQ_API int nxq_gguf_register(nxq_gguf_t g, int64_t i, int64_t slice, nxq_weight_t* out);

/* As nxq_gguf_register, this rank's tensor-parallel shard only
 * (nxq_weight_register_shard rules). */
NXQ_API int nxq_gguf_register_shard(nxq_gguf_t g, int64_t i, int64_t slice, int split, int rank,
                                    int world, nxq_weight_t* out);

/* ---- residency loader: NXF files ------------------------------------------
 * Replaces the reference's NXF read path (NXFReader::open / get_tensor /
 * map_chunk, format/nxf_reader.cpp:166-258 and 295-409; layouts in
 * format/nxf.h:27-51), which maps chunks for the engine to stream at every
 * call: a 64-byte header (magic "NXF1", version 1, manifest and tensor-index
 * offsets and sizes, total file size), a flat JSON manifest, and a tensor
 * index of name, shape (shape[0] fastest, as GGUF dims), dtype and 24-byte
 * chunk descriptors (file offset, stored and decoded size, xxHash32 of the
 * stored bytes, codec, group size).  The file is mapped read-only and every
 * field is bounds-checked; registration checks each chunk's xxHash32 (the
 * reference stores it but never checks it) and builds the tiled HBM copy.
 * Registered codecs (Codec, core/config.h:21-36): INT4 = 4 - a chunk is
 * [4-bit codes in NXQ_INT4_ROWS order][fp32 scales][fp32 zeros] per group of
 * the descriptor's group size (32, 64, 128), as GGUFImporter writes it
 * (import/gguf_importer.cpp:1144-1170) -, the GGUF-block passthroughs
 * Q3K = 11, Q4K = 12, Q2K = 13, and the flat arrays the engine decodes at
 * load time (hybrid_model.cpp:165-255): INT8 = 3 (w = q / 127), FP16 = 1
 * (subnormals read as zero) and FP32 = 0, also any chunk of 4 bytes per
 * element (the writer's small-tensor passthrough), as NXQ_TYPE_NXF_I8 / F16 /
 * F32 (K a multiple of 32).  Parsing needs no GPU; registration needs
 * nxq_init.  A malformed or truncated file, or a checksum mismatch, is
 * NXQ_ERR_FORMAT; another codec is NXQ_ERR_CODEC. */
typedef struct nxq_nxf_s* nxq_nxf_t;

NXQ_API int nxq_nxf_open(const char* path, nxq_nxf_t* out);
NXQ_API int nxq_nxf_close(nxq_nxf_t f);
NXQ_API int nxq_nxf_tensor_count(nxq_nxf_t f, int64_t* n);

/* Tensor i, in file order: name (NUL-terminated, truncated to name_len),
 * dtype, dims (up to 4, unused ones 1), chunk count, the first chunk's codec
 * and group size, and the stored bytes of all chunks. */
NXQ_API int nxq_nxf_tensor_info(nxq_nxf_t f, int64_t i, char* name, size_t name_len, int* dtype,
                                int* n_dims, int64_t dims[4], int64_t* n_chunks, int* codec,
                                int* group_size, uint64_t* bytes);
NXQ_API int nxq_nxf_chunk_info(nxq_nxf_t f, int64_t i, int64_t c, uint64_t* offset,
                               uint32_t* stored, uint32_t* decoded, uint32_t* checksum,
                               int* codec, int* group_size);

/* Index of the tensor called `name`; NXQ_ERR_ARG if there is none. */
NXQ_API int nxq_nxf_find(nxq_nxf_t f, const char* name, int64_t* index);

/* Checks tensor i's chunks (one codec and group size, no entropy coding,
 * xxHash32 as stored) without registering it. */
NXQ_API int nxq_nxf_verify(nxq_nxf_t f, int64_t i);

/* xxHash32 (seed 0) of n bytes, the checksum NXF chunk descriptors carry. */
NXQ_API int nxq_nxf_xxh32(const void* data, size_t n, uint32_t* out);

/* The manifest's JSON text (NUL-terminated, truncated to n; *size = its
 * length), and the value of a key as a number or a string. */
NXQ_API int nxq_nxf_manifest(nxq_nxf_t f, char* buf, size_t n, uint64_t* size);
NXQ_API int nxq_nxf_manifest_number(nxq_nxf_t f, const char* key, double* v);
NXQ_API int nxq_nxf_manifest_string(nxq_nxf_t f, const char* key, char* buf, size_t n);

/* Register tensor i as a weight [N][K]: K = dims[0], N = dims[1]; for a
 * 3-D tensor [E][N][K] (stacked experts) `slice` picks one, else pass 0.  The
 * _shard form registers this rank's tensor-parallel shard
 * (nxq_weight_register_shard rules; INT4 tensors as their group blocks). */
NXQ_API int nxq_nxf_register(nxq_nxf_t f, int64_t i, int64_t slice, nxq_weight_t* out);
NXQ_API int nxq_nxf_register_shard(nxq_nxf_t f, int64_t i, int64_t slice, int split, int rank,
                                   int world, nxq_weight_t* out);

#ifdef __cplusplus
}
#endif
#endif /* NXQ_H */
