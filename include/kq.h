/*
 * kq.h -- C ABI of the B200 GGUF K-quant matmul path (libkq.so).
 *
 * Drop-in replacement for the K-quant matrix products of the reference engine
 * src/v182_r22_breakthrough_engine.c ("ENG"): the GGUF Q4_K / Q5_K / Q6_K / Q8_0 weight
 * super-blocks multiplied by Q8_K / Q8_0 activations behind sdot_gemm_multi_dispatch, the
 * per-type row kernels, the LM-head row scans and the NPU INT4 FFN entry point.  In the
 * reference all of these are `static` functions of one translation unit; each declaration
 * below names the reference function it replaces (file:line).
 *
 * Conventions
 *  - Every function returns an int status: KQ_OK (0) or a negative kq_status code.  No call
 *    aborts; kq_last_error() describes the last failure of a context.
 *  - Weight bytes are the GGUF blocks exactly as stored in the file (row-major, row size
 *    kq_row_bytes(type, cols)).  kq_weight_upload copies them to HBM once (the reference
 *    reads them from its mmap, ENG:4174).
 *  - Activations are IEEE binary16 bit patterns (uint16_t), the reference's __fp16.
 *  - Functions without a suffix take HOST pointers and block until the results are in host
 *    memory, like the reference's synchronous calls.  Functions ending in _async take DEVICE
 *    pointers and only enqueue work on the context's CUDA stream.
 *  - A context is used by one host thread at a time (the reference's coordinator thread,
 *    ENG:3845); different contexts are independent.
 */
#ifndef KQ_H
#define KQ_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* GGML tensor type ids, ENG:115-120 */
#define KQ_TYPE_F32  0
#define KQ_TYPE_F16  1
#define KQ_TYPE_Q8_0 8
#define KQ_TYPE_Q4_K 12
#define KQ_TYPE_Q5_K 13
#define KQ_TYPE_Q6_K 14

/* Limits of this implementation (the reference's are SDOT_MAX_BATCH 32 / SDOT_MAX_K 9216,
 * ENG:862-865; here K and M are limited only by these constants and device memory). */
#define KQ_MAX_TASKS 4          /* tasks per dispatch, like PoolJob.sdot_tasks_inline[4] (ENG:3453) */
#define KQ_MAX_K 65536          /* reduction length */
#define KQ_MAX_M 4096           /* activation rows per call */

typedef enum kq_status {
    KQ_OK = 0,
    KQ_ERR_INVALID_ARGUMENT = -1,   /* NULL pointer, negative size, bad stride */
    KQ_ERR_UNSUPPORTED_TYPE = -2,   /* type is not Q4_K / Q5_K / Q6_K / Q8_0 */
    KQ_ERR_SHAPE = -3,              /* K not a multiple of 256, M/K out of range, row range outside the weight */
    KQ_ERR_CUDA = -4,               /* a CUDA runtime call failed */
    KQ_ERR_OUT_OF_MEMORY = -5,
    KQ_ERR_NO_DEVICE = -6,
    KQ_ERR_TIMEOUT = -7,            /* a bounded device-side wait gave up (the kernel returned early) */
    KQ_ERR_NOT_READY = -8,          /* no pre-quantized activation is pending in the context */
    KQ_ERR_FORMAT = -9,             /* not a GGUF v2/v3 image, or a record / tensor past its end */
    KQ_ERR_NOT_FOUND = -10          /* no such file, tensor name or tensor index */
} kq_status;

typedef struct kq_ctx kq_ctx;
typedef struct kq_weight kq_weight;

/* ---------------------------------------------------------------- library / context */

const char *kq_version(void);
const char *kq_status_string(int status);

/* Create a context on CUDA device `device` with its own non-blocking stream.  Replaces the
 * engine's pool start-up init_thread_pool (ENG:3843-3855). */
int kq_init(int device, kq_ctx **out);
int kq_destroy(kq_ctx *ctx);
/* Use an existing cudaStream_t (passed as void*) for all later work of this context. */
int kq_set_stream(kq_ctx *ctx, void *cuda_stream);
void *kq_get_stream(const kq_ctx *ctx);
/* Wait for the context's stream and report any device-side error (e.g. KQ_ERR_TIMEOUT). */
int kq_synchronize(kq_ctx *ctx);
const char *kq_last_error(const kq_ctx *ctx);
/* Options: "pdl" -- programmatic dependent launch between consecutive kernels (default 1);
 * "timeout_ms" / "timeout_us" -- limit of every device-side wait (default 1000 ms);
 * "inject_timeout" -- failure-path test: matrix-product kernels first wait on a barrier that
 * nothing completes, so the wait runs out, the kernel returns early and the call reports
 * KQ_ERR_TIMEOUT (default 0);
 * "gemm_path" -- products of more than 8 activation rows: 0 chooses by a cost model, 1 always
 * the weight-row-major tensor-core kernel (tcgen05; weight rows as the MMA's A operand), 2 always
 * the GEMV kernel in tiles of 8 rows, 3 always the token-major tensor-core kernel (activation
 * tokens as A in tensor memory, row groups spread over all SMs) (default 0);
 * "gemv_split" -- GEMV launches (up to 8 activation rows) whose row groups would spread unevenly
 * over the SMs give every CTA an equal range of 16-row x 256-value tiles instead; a row group
 * shared by neighbouring CTAs is summed in block order by the last of them (1, default); 0 keeps
 * whole row groups per CTA;
 * "gemv_half" -- Q4_K / Q5_K GEMV launches of 1-2 activation rows whose row groups divide
 * unevenly over the SMs, or whose largest share does not fit one CTA's shared memory whole, give
 * every CTA a contiguous range of 8-row halves of row groups instead (1, default); 0 keeps whole
 * row groups.  Results are identical either way;
 * "ffn_fused" -- kq_run_ffn / kq_run_ffn_async for 1-2 rows with Q4_K / Q5_K gate and up and a
 * Q4_K / Q5_K / Q6_K down projection run the whole block as one persistent kernel, one CTA per SM,
 * all resident at once, with one grid-wide barrier between gate/up and down (1, default); the
 * results are bit for bit those of the four launches that 0 selects (and that other shapes use);
 * "swiglu_exp" -- where SwiGLU takes expf(-g) from: 0 (default) a table of the host C library's
 * expf at the 65,536 fp16 values of g, made once by kq_init -- the function the reference's
 * scalar SwiGLU calls (ENG:4354), so the results match it bit for bit on the same host; 1 an fp64
 * exp on the GPU rounded once to fp32 (the correctly rounded value except in rare double-rounding
 * cases; glibc 2.39's expf is not correctly rounded at 16 fp16 inputs);
 * "graph_released" -- a context whose calls were captured into a CUDA graph keeps its scratch
 * buffers where the graph recorded them: a later call that would have to grow one returns
 * KQ_ERR_INVALID_ARGUMENT instead of freeing it.  Setting 1 declares those graphs destroyed and
 * lets scratch grow again.  (Calls made during a capture never allocate: make one eager call of
 * the largest shape before capturing.) */
int kq_set_option(kq_ctx *ctx, const char *name, long long value);

/* compute_ggml_bytes / ggml_row_bytes (ENG:364-374, ENG:3940): bytes of one GGUF row of k
 * elements; 0 for unknown types. */
uint64_t kq_row_bytes(uint32_t type, uint64_t k);

/* ---------------------------------------------------------------- weights */

/* Copy a rows x cols GGUF tensor (host bytes) to HBM in this library's device layout.
 * Replaces the mmap'ed weight pointer of init_sdot_task (ENG:4163-4181). */
int kq_weight_upload(kq_ctx *ctx, const void *gguf_bytes, uint32_t type, int rows, int cols, kq_weight **out);
/* Same, from GGUF bytes already in device memory (not retained after the call). */
int kq_weight_upload_device(kq_ctx *ctx, const void *gguf_bytes_dev, uint32_t type, int rows, int cols,
                            kq_weight **out);
int kq_weight_free(kq_ctx *ctx, kq_weight *w);
/* Shape queries; device_bytes is the HBM footprint of the device layout. */
int kq_weight_info(const kq_weight *w, uint32_t *type, int *rows, int *cols, uint64_t *device_bytes);

/* ---------------------------------------------------------------- activations */

/* quantize_row_fp16_to_q8_k (ENG:925-990) for M rows of K values: out receives
 * BlockQ8K[M][K/256] (292 B each: float d, int8 qs[256], int32 bsum32[8]).  Bit-exact. */
int kq_quantize_q8k(kq_ctx *ctx, const uint16_t *x, int M, int K, void *out);
/* quantize_row_fp16_to_q8_0 (ENG:1016-1064): out receives BlockQ8_0_Fast[M][K/32] (36 B each). */
int kq_quantize_q8_0(kq_ctx *ctx, const uint16_t *x, int M, int K, void *out);
int kq_quantize_q8k_async(kq_ctx *ctx, const uint16_t *x_dev, int M, int K, void *out_dev);
int kq_quantize_q8_0_async(kq_ctx *ctx, const uint16_t *x_dev, int M, int K, void *out_dev);

/* ---------------------------------------------------------------- matrix products */

/* One output matrix of a dispatch; mirrors SdotMatrixTask (ENG:888-899).
 * Output rows [row_begin, row_begin + rows) of weight w (the reference offsets w_base by
 * row_start * row_bytes for LM-head chunks, ENG:9689).
 *   dst      : fp16 [M][dst_stride], dst[m*dst_stride + r] = fp16(sum + residual)   (may be NULL)
 *   residual : fp16 [M][res_stride] added before rounding (may be NULL), ENG:3602-3607
 *   dst_f32  : fp32 [M][dst_f32_stride] un-rounded sums (may be NULL; for parity and fp32 users) */
typedef struct kq_task {
    const kq_weight *w;
    int row_begin;
    int rows;
    uint16_t *dst;
    size_t dst_stride;
    const uint16_t *residual;
    size_t res_stride;
    float *dst_f32;
    size_t dst_f32_stride;
} kq_task;

/* sdot_gemm_multi_dispatch (ENG:4188-4262): up to KQ_MAX_TASKS matrices sharing one fp16 input
 * x [M][K].  The input is quantized to Q8_K (and/or Q8_0 for Q8_0 weights) inside the kernel,
 * unless a producer (kq_rmsnorm_fp16_rows / kq_swiglu_fp16_rows) left a pre-quantized Q8_K
 * activation of the same M x K in the context, exactly like g_sdot_input_q8k_prequantized
 * (ENG:4184, ENG:4205-4218).  HOST pointers; blocking.  Outputs in pinned (page-locked, mapped)
 * host memory are written in place by the kernel; other outputs go through device staging and a
 * copy back. */
int kq_sdot_gemm_multi_dispatch(kq_ctx *ctx, const uint16_t *x, int M, int K, const kq_task *tasks, int n_tasks);
/* Same with DEVICE pointers (x and every task pointer); asynchronous.  x_stride = elements
 * between rows of x (>= K). */
int kq_gemm_multi_async(kq_ctx *ctx, const uint16_t *x_dev, size_t x_stride, int M, int K,
                        const kq_task *tasks, int n_tasks);
/* Same from pre-quantized DEVICE activations: act_q8k = BlockQ8K[M][K/256] (for Q4_K/Q5_K/Q6_K
 * tasks) and/or act_q80 = BlockQ8_0_Fast[M][K/32] (for Q8_0 tasks). */
int kq_gemm_multi_q8_async(kq_ctx *ctx, const void *act_q8k_dev, const void *act_q80_dev, int M, int K,
                           const kq_task *tasks, int n_tasks);

/* sdot_row_<type>_batch (ENG:1951, 3109, 3234, 3368): one weight row against the M rows of
 * the context's current quantized input (left by the last dispatch or producer); out_sums[M]. */
int kq_sdot_row_batch(kq_ctx *ctx, const kq_weight *w, uint32_t row, int M, float *out_sums);
/* eval_single_lm_row_dot (ENG:10986-11105): row row_idx against input row m. */
int kq_eval_single_lm_row_dot(kq_ctx *ctx, const kq_weight *w, uint32_t row_idx, int m, float *out);

/* Per-super-block integer intermediates of rows [row_begin, row_begin+rows) of w against a
 * pre-quantized DEVICE activation (BlockQ8K[M][K/256], or BlockQ8_0_Fast[M][K/32] for Q8_0):
 * sumi[m][r][b] = sum_j sc_j * dot_j (Q6_K: sum_s sc_s * dot_s, Q8_0: the 32-element dot per
 * 32-block) and summ[m][r][b] = sum_j m_j * bsum32_j (Q4_K/Q5_K; 0 otherwise), the locals of
 * eval_single_lm_row_dot (ENG:11009-11024, 11042-11061, 11076-11099) and sdot_row_q8_0_batch
 * (ENG:3402-3404).  out_f32 [M][rows] (may be NULL).  DEVICE pointers; asynchronous. */
int kq_debug_block_sums_async(kq_ctx *ctx, const kq_weight *w, int row_begin, int rows, const void *act_dev,
                              int M, int32_t *sumi_dev, int32_t *summ_dev, float *out_f32_dev);

/* ---------------------------------------------------------------- producers (fused prologue/epilogue) */

/* rmsnorm_fp16_rows_fast (ENG:4264-4314): x_out = fp16(x * inv_rms * gamma), eps 1e-6, and the
 * normalised rows quantized to Q8_K and kept in the context as the pending pre-quantized input
 * of the next dispatch.  HOST pointers; blocking. */
int kq_rmsnorm_fp16_rows(kq_ctx *ctx, const uint16_t *x_in, const uint16_t *gamma, uint16_t *x_out, int M, int K);
/* swiglu_fp16_rows_fast (ENG:4326-4383): gate = fp16(silu(gate) * up) in place, quantized to
 * Q8_K and kept as the pending input.  HOST pointers; blocking. */
int kq_swiglu_fp16_rows(kq_ctx *ctx, uint16_t *gate_inout, const uint16_t *up_in, int M, int N);
/* DEVICE-pointer forms; q8k_out_dev (BlockQ8K[M][K/256]) may be NULL to use the context's
 * pending-input buffer. */
int kq_rmsnorm_q8k_async(kq_ctx *ctx, const uint16_t *x_dev, const uint16_t *gamma_dev, uint16_t *out_dev,
                         int M, int K, void *q8k_out_dev);
int kq_swiglu_q8k_async(kq_ctx *ctx, uint16_t *gate_dev, const uint16_t *up_dev, int M, int N, void *q8k_out_dev);

/* ---------------------------------------------------------------- FFN block */

/* Replaces run_real_npu_universal_ffn (npu_tree_verifier_v22.c:682-761, declared
 * npu_tree_verifier_v22.h:132-143) with the numerics of the engine's CPU SDOT FFN it falls back
 * to (ENG:8283-8298): x_out = x_in + W_down . swiglu(W_gate . xn, W_up . xn), xn = rmsnorm(x_in,
 * gamma).  x_in/x_out [batch_len][hidden] fp16, hidden = gate->cols, ffn = gate->rows.
 * Any batch_len >= 1 (the NPU graph took 1..4).  HOST pointers; blocking; KQ_OK on success
 * (the reference returns 1 on success, 0 to fall back). */
int kq_run_ffn(kq_ctx *ctx, const kq_weight *gate, const kq_weight *up, const kq_weight *down, int batch_len,
               const uint16_t *x_in, const uint16_t *gamma, uint16_t *x_out);
int kq_run_ffn_async(kq_ctx *ctx, const kq_weight *gate, const kq_weight *up, const kq_weight *down,
                     int batch_len, const uint16_t *x_in_dev, const uint16_t *gamma_dev, uint16_t *x_out_dev);

/* ---------------------------------------------------------------- LM head */

/* Full-vocabulary LM head over M normalised fp16 rows x [M][K]: logits (fp16 [M][rows], may be
 * NULL) and the per-row argmax of the fp16 logits (strict '>', first maximal row wins), the
 * scan of run_final_norm_and_lm_head_pipelined / _batch_sdot (ENG:9686-9707, ENG:11165-11193)
 * without the early-exit thresholds (ENG:9735-9745, ENG:11237-11249).  HOST pointers; blocking. */
int kq_lm_head_argmax(kq_ctx *ctx, const kq_weight *w, const uint16_t *x, int M, uint16_t *logits,
                      uint32_t *top_toks, float *top_vals);
int kq_lm_head_argmax_async(kq_ctx *ctx, const kq_weight *w, const uint16_t *x_dev, int M, uint16_t *logits_dev,
                            float *logits_f32_dev, uint32_t *top_toks_dev, float *top_vals_dev);

/* LM-head argmax that allocates nothing.  No counterpart in the reference: an addition for
 * callers that cannot allocate device memory when they call -- a decode loop whose memory is fixed
 * after start-up, or code running inside another runtime's allocator, where a cudaMalloc would
 * break that runtime's accounting or stall.  It computes the fused GEMV over all rows of w, fp16
 * logits to logits_dev when not NULL, and the argmax of the fp16 logits (strict '>', first maximal
 * row wins) to toks_dev / vals_dev, with no context: DEVICE pointers, enqueued on `stream` (a
 * cudaStream_t; NULL = the default stream) of the current device, where w must live (another
 * device's weight: KQ_ERR_INVALID_ARGUMENT).
 *  - Results: for Q4_K / Q5_K / Q6_K weights the same bits as kq_lm_head_argmax_async (both are
 *    bit-exact to the reference); for Q8_0 weights the logits agree within the Q8_0 long-row
 *    tolerance (1e-5 of the output scale plus one fp16 ulp; the two calls may sum Q8_0 block terms
 *    in different orders), so between nearly equal logits the argmax may differ.
 *  - Cost: tiles of up to 8 activation rows, one pass over the weights per tile: M rows read the
 *    weights ceil(M / 8) times (kq_lm_head_argmax_async reads them once for M > 8).
 *  - Scratch: a static device array of KQ_NOALLOC_MAX_M argmax slots and a status word, which
 *    every GPU that loads the library keeps until exit; M > KQ_NOALLOC_MAX_M returns KQ_ERR_SHAPE.
 *    The first call on a device (and the first after that device's context was reset) looks up
 *    the array's device address (cudaGetSymbolAddress), so make the first call on each device
 *    before any stream capture.  All calls share the array and clear it on their stream at the
 *    start: calls that overlap on the GPU (different streams) race and must be serialised by the
 *    caller.
 *  - A device-side wait that timed out (a kernel that stopped early) cannot be returned as a
 *    status by an asynchronous call: every row then gets the sentinel token 0xFFFFFFFF and value
 *    NaN instead. */
#define KQ_NOALLOC_MAX_M 64
int kq_lm_head_argmax_noalloc(const kq_weight *w, const uint16_t *x_dev, int M, uint16_t *logits_dev,
                              uint32_t *top_toks_dev, float *top_vals_dev, void *stream);

/* eval_indexed_ext_lm_rows_parallel (ENG:9581-9614, work item ENG:9473-9579): the rows listed
 * in row_ids against the context's current quantized input (M rows), fp32 comparison;
 * top_toks/top_vals [M] are updated in place when a row beats them (strict '>').
 * logits_m1 (fp16, indexed by row id, M == 1 only) may be NULL.  HOST pointers; blocking. */
int kq_eval_indexed_rows_argmax(kq_ctx *ctx, const kq_weight *w, const uint32_t *row_ids, int n_rows, int M,
                                uint16_t *logits_m1, uint32_t *top_toks, float *top_vals);

/* ---------------------------------------------------------------- dequantization */

/* dequant_contiguous_fast (ENG:3856-3896) of rows [row_begin, row_begin+rows) to fp16,
 * bit-exact to dequant_block_<type> (ENG:598-853).  dst fp16 [rows][cols]. */
int kq_dequant_rows(kq_ctx *ctx, const kq_weight *w, int row_begin, int rows, uint16_t *dst);
int kq_dequant_rows_async(kq_ctx *ctx, const kq_weight *w, int row_begin, int rows, uint16_t *dst_dev);
/* Embedding lookup: the decode step's dequant_contiguous_fast of row token_id of
 * token_embd.weight (ENG:8667-8670; the same tensor is the tied LM head), for n tokens at once:
 * dst fp16 [n][cols], row i = row ids[i], bit-exact to dequant_block_<type>.  HOST ids / dst,
 * blocking; an id >= rows is KQ_ERR_SHAPE before anything runs. */
int kq_embed_rows(kq_ctx *ctx, const kq_weight *w, const uint32_t *ids, int n, uint16_t *dst);
/* Same with DEVICE ids / dst, asynchronous: an id >= rows gives a row of zeros (nothing is read
 * out of bounds) and the next kq_synchronize reports KQ_ERR_SHAPE. */
int kq_embed_rows_async(kq_ctx *ctx, const kq_weight *w, const uint32_t *ids_dev, int n, uint16_t *dst_dev);

/* ---------------------------------------------------------------- GGUF files */

/* The tensor directory of a GGUF v2/v3 file, as parse_gguf_file (ENG:376-413) builds it over the
 * engine's mmap: magic "GGUF", the key/value pairs (only general.alignment is kept; default 32),
 * the tensor records, and the data section at the next multiple of the alignment.  Every record
 * and every tensor's byte range is checked against the file size (KQ_ERR_FORMAT otherwise). */
typedef struct kq_gguf kq_gguf;
typedef struct kq_gguf_tensor {
    const char *name;      /* NUL-terminated, owned by the kq_gguf (GgufTensorInfo.name, ENG:168) */
    uint32_t type;         /* GGML type id */
    uint32_t n_dims;       /* 1..4 */
    uint64_t dims[4];      /* dims[0] = values per row, dims[1] = rows; unused dimensions are 1 */
    uint64_t n_elems;
    uint64_t offset;       /* absolute byte offset of the data in the file (abs_offset, ENG:410-412) */
    uint64_t bytes;        /* compute_ggml_bytes(type, n_elems) (ENG:364-374); 0 for other types */
    const void *data;      /* the tensor's bytes in the mapped file / caller's image */
} kq_gguf_tensor;

/* Map a GGUF file read-only and parse its directory (the engine's model open, ENG:376). */
int kq_gguf_open(const char *path, kq_gguf **out);
/* Same over a GGUF image already in host memory (borrowed until kq_gguf_close). */
int kq_gguf_open_memory(const void *bytes, size_t size, kq_gguf **out);
int kq_gguf_close(kq_gguf *g);
int kq_gguf_info(const kq_gguf *g, uint32_t *version, uint64_t *alignment, uint64_t *data_offset);
/* Number of tensor records (GgufContext.n_tensors, ENG:185), or a negative status. */
int kq_gguf_tensor_count(const kq_gguf *g);
int kq_gguf_get_tensor(const kq_gguf *g, int index, kq_gguf_tensor *out);
/* find_tensor (ENG:415-420): the index of the record named `name`, or KQ_ERR_NOT_FOUND. */
int kq_gguf_find_tensor(const kq_gguf *g, const char *name);
/* Upload tensor `index` -- a Q4_K / Q5_K / Q6_K / Q8_0 matrix of dims[1] rows x dims[0] values --
 * with kq_weight_upload (the weight pointer init_sdot_task takes from the mmap, ENG:4163-4181). */
int kq_gguf_upload(kq_ctx *ctx, const kq_gguf *g, int index, kq_weight **out);
/* Device weight cache of a whole model: out[i] receives every quantized matrix of the file
 * (dims[0] a multiple of 256), NULL for the other records (norms, embeddings in f32/f16 ...);
 * out has kq_gguf_tensor_count entries.  On failure nothing stays uploaded. */
int kq_gguf_upload_all(kq_ctx *ctx, const kq_gguf *g, kq_weight **out, int *n_uploaded);

/* ---------------------------------------------------------------- several GPUs: the LM head
 * with its all-gather in the GEMV (no counterpart in the single-process reference; its LM head is
 * ENG:9686-9707, the all-gather is what north_star adds for vocabulary rows split over GPUs).
 *
 * One process per GPU.  Each rank allocates a gather region with kq_peer_alloc, the ranks exchange
 * the IPC handles (any channel: torch.distributed, MPI, a file) and open each other's regions with
 * kq_peer_open.  A region holds control words and two buffers of [M][row_stride] 64-bit entries
 * (kq_peer_region_bytes).  kq_gemm_peer_gather_async streams this rank's vocabulary slice and its
 * epilogue stores every logit into the current buffer of EVERY rank's region over NVLink, as one
 * aligned 64-bit store of (step number, fp32 value) -- plain stores, no TMA, no multicast, no
 * fence or flag.  kq_peer_gather_wait_async reads the current buffer until every entry carries the
 * step number (bounded: KQ_ERR_TIMEOUT after the context's timeout) and copies the fp32 values to
 * `out`.  row_stride is the total number of rows, and the ranks' slices must cover every row each
 * step.  Steps alternate between the two buffers, so a rank may start step s + 1 while a peer still
 * reads step s.  Every rank must issue the same sequence of gather and wait calls, each wait after
 * its gather on the same stream, and nothing of a step may be skipped. */
#define KQ_MAX_PEERS 8
#define KQ_IPC_HANDLE_BYTES 64
typedef struct kq_peer_gather {
    int world, rank;
    int M;                         /* activation rows of every step (1..8) */
    long long row_stride;          /* entries per row: the total number of vocabulary rows */
    int row_begin;                 /* global row of this rank's first weight row */
    void *regions[KQ_MAX_PEERS];   /* every rank's region: this rank's own, the others as opened */
} kq_peer_gather;
size_t kq_peer_region_bytes(int M, long long row_stride);
/* cudaMalloc'd, zeroed region of `bytes` on the context's device and its IPC handle
 * (KQ_IPC_HANDLE_BYTES bytes written to ipc_handle). */
int kq_peer_alloc(kq_ctx *ctx, size_t bytes, void **region_dev, void *ipc_handle);
int kq_peer_free(kq_ctx *ctx, void *region_dev);
/* Map another process's region (its handle) into this context's device. */
int kq_peer_open(kq_ctx *ctx, const void *ipc_handle, void **region_dev);
int kq_peer_close(kq_ctx *ctx, void *region_dev);
/* This rank's slice: all rows of w against the fp16 activation x_dev [M][K] (K = w's cols).  With
 * out_dev (fp32 [M][row_stride]) the step completes inside this call's kernel: this rank's logits go
 * to out_dev from the epilogue, and the kernel's last CTAs wait (bounded) for the other ranks'
 * entries and write them to out_dev -- no wait call follows.  With out_dev NULL the step is
 * completed by kq_peer_gather_wait_async. */
int kq_gemm_peer_gather_async(kq_ctx *ctx, const kq_weight *w, const uint16_t *x_dev, const kq_peer_gather *pg,
                              float *out_dev);
/* Wait for every rank's slice of the current step (after a kq_gemm_peer_gather_async without
 * out_dev); out_dev (fp32 [M][row_stride]) receives the gathered logits (NULL: wait only). */
int kq_peer_gather_wait_async(kq_ctx *ctx, const kq_peer_gather *pg, float *out_dev);

#ifdef __cplusplus
}
#endif
#endif /* KQ_H */
