/*
 * ref_harness.c -- builds the UNMODIFIED reference engine (src/v182_r22_breakthrough_engine.c
 * of the reference, "ENG") for x86-64 and exports thin entry points around its static K-quant
 * functions.  TEST INFRASTRUCTURE ONLY: it generates the golden fixtures in tests/golden/ and
 * is the CPU arm of bench.py (--impl reference / cpu_baseline).  Nothing in the product
 * package links or loads it.
 *
 * Build (oracle/Makefile): gcc -std=gnu11 -O2 -ffp-contract=off -DHOST_SYNTAX_CHECK
 * -D__fp16=_Float16 -Dmain=ref_main -I<reference>/src.  HOST_SYNTAX_CHECK is the reference's
 * own escape hatch (ENG:63); _Float16 has the same binary16 format as ARM __fp16.  Without
 * __ARM_NEON every NEON block drops out and the scalar #else paths remain.
 *
 * The reference declares sdot_row_q4_k_batch (ENG:918) but defines it only under NEON
 * (ENG:1951).  The definition below supplies it by calling the reference's own scalar Q4_K
 * row dot, eval_single_lm_row_dot (ENG:10986-11027), once per token.
 */
#define _GNU_SOURCE
#include "v182_r22_breakthrough_engine.c"

#include <sched.h>

static void sdot_row_q4_k_batch(const uint8_t *restrict w_row, const QuantizedBatchInput *restrict Q,
                                int M, int K, float *restrict out_sums) {
    for (int m = 0; m < M; ++m) out_sums[m] = eval_single_lm_row_dot(w_row, GGML_TYPE_Q4_K, 0, 0, Q, m, K);
}

#define KQREF_API __attribute__((visibility("default")))

KQREF_API int kqref_max_batch(void) { return SDOT_MAX_BATCH; }
KQREF_API int kqref_max_k(void) { return SDOT_MAX_K; }
KQREF_API int kqref_pool_threads(void) { return POOL_THREADS; }

KQREF_API uint64_t kqref_row_bytes(uint32_t type, uint64_t k) { return compute_ggml_bytes(type, k); }

KQREF_API void kqref_quantize_row_q8k(const uint16_t *x, void *y, int k) {
    quantize_row_fp16_to_q8_k((const __fp16 *)x, (BlockQ8K *)y, k);
}

KQREF_API void kqref_quantize_row_q8_0(const uint16_t *x, void *y, int k) {
    quantize_row_fp16_to_q8_0((const __fp16 *)x, (BlockQ8_0_Fast *)y, k);
}

KQREF_API void kqref_dequant_row(uint32_t type, const uint8_t *w, int n, uint16_t *dst) {
    __fp16 *o = (__fp16 *)dst;
    if (type == GGML_TYPE_Q8_0) for (int b = 0; b < n / 32; ++b) dequant_block_q8_0(w + (size_t)b * 34, o + 32 * b);
    if (type == GGML_TYPE_Q4_K) for (int b = 0; b < n / 256; ++b) dequant_block_q4_k(w + (size_t)b * 144, o + 256 * b);
    if (type == GGML_TYPE_Q5_K) for (int b = 0; b < n / 256; ++b) dequant_block_q5_k(w + (size_t)b * 176, o + 256 * b);
    if (type == GGML_TYPE_Q6_K) for (int b = 0; b < n / 256; ++b) dequant_block_q6_k(w + (size_t)b * 210, o + 256 * b);
}

/* Load M activation rows into the engine's global quantized input (g_sdot_input, ENG:901),
 * the buffer every reference row kernel reads.  q8k: BlockQ8K[M][K/256] or NULL;
 * q80: BlockQ8_0_Fast[M][K/32] or NULL.  Returns 0 when M/K exceed the engine's limits. */
KQREF_API int kqref_load_input(const void *q8k, const void *q80, int M, int K) {
    if (M < 1 || M > SDOT_MAX_BATCH || K < 32 || K > SDOT_MAX_K) return 0;
    g_sdot_input.M = M;
    g_sdot_input.K = K;
    for (int m = 0; m < M; ++m) {
        if (q8k) memcpy(g_sdot_input.q8k[m], (const BlockQ8K *)q8k + (size_t)m * (K / 256), sizeof(BlockQ8K) * (K / 256));
        if (q80) memcpy(g_sdot_input.q80[m], (const BlockQ8_0_Fast *)q80 + (size_t)m * (K / 32), sizeof(BlockQ8_0_Fast) * (K / 32));
    }
    return 1;
}

/* The reference's per-row batch kernels over the loaded input: out_sums[m] for one row. */
KQREF_API void kqref_row_batch(uint32_t type, const uint8_t *w_row, int M, int K, float *out_sums) {
    if (type == GGML_TYPE_Q4_K) sdot_row_q4_k_batch(w_row, &g_sdot_input, M, K, out_sums);
    else if (type == GGML_TYPE_Q5_K) sdot_row_q5_k_batch(w_row, &g_sdot_input, M, K, out_sums);
    else if (type == GGML_TYPE_Q6_K) sdot_row_q6_k_batch(w_row, &g_sdot_input, M, K, out_sums);
    else if (type == GGML_TYPE_Q8_0) sdot_row_q8_0_batch(w_row, &g_sdot_input, M, K, out_sums);
}

KQREF_API float kqref_lm_row_dot(const uint8_t *w_base, uint32_t type, size_t row_bytes, uint32_t row, int m, int K) {
    return eval_single_lm_row_dot(w_base, type, row_bytes, row, &g_sdot_input, m, K);
}

KQREF_API void kqref_rmsnorm(const uint16_t *x, const uint16_t *gamma, uint16_t *out, int M, int K) {
    rmsnorm_fp16_rows_fast((const __fp16 *)x, (const __fp16 *)gamma, (__fp16 *)out, M, K);
}

/* Copy back the Q8_K activation the producers left in g_sdot_input (ENG:4304, ENG:4357). */
KQREF_API void kqref_get_q8k(int M, int K, void *out) {
    for (int m = 0; m < M; ++m)
        memcpy((BlockQ8K *)out + (size_t)m * (K / 256), g_sdot_input.q8k[m], sizeof(BlockQ8K) * (K / 256));
}

/* Start the reference's pinned pool (ENG:3843).  init_thread_pool pins the calling thread to
 * cpu 7; the caller's own affinity is put back afterwards so the host process is unaffected. */
KQREF_API void kqref_init_pool(void) {
    cpu_set_t saved;
    int have = sched_getaffinity(0, sizeof(saved), &saved) == 0;
    init_thread_pool();
    if (have) sched_setaffinity(0, sizeof(saved), &saved);
}

KQREF_API void kqref_swiglu(uint16_t *gate, const uint16_t *up, int M, int N) {
    swiglu_fp16_rows_fast((__fp16 *)gate, (const __fp16 *)up, M, N);
}

KQREF_API void kqref_turbo(int on) {
    if (on) pool_enter_turbo_mode();
    else pool_exit_turbo_mode();
}

/* One task of sdot_gemm_multi_dispatch (SdotMatrixTask, ENG:888-899). */
typedef struct {
    const uint8_t *w_base;
    uint32_t type;
    int rows;
    uint16_t *dst;
    size_t dst_stride;
    const uint16_t *residual;
    size_t res_stride;
} kqref_task;

/* sdot_gemm_multi_dispatch (ENG:4188-4262) on the reference pool.  prequantized != 0 keeps the
 * Q8_K activation already in g_sdot_input (the g_sdot_input_q8k_prequantized flag, ENG:4184). */
KQREF_API void kqref_dispatch(const uint16_t *x, int M, int K, const kqref_task *t, int n_tasks, int prequantized) {
    SdotMatrixTask tasks[4];
    if (n_tasks > 4) n_tasks = 4;
    for (int i = 0; i < n_tasks; ++i) {
        tasks[i].w_base = t[i].w_base;
        tasks[i].type = t[i].type;
        tasks[i].row_bytes = ggml_row_bytes(t[i].type, (size_t)K);
        tasks[i].dst = (__fp16 *)t[i].dst;
        tasks[i].dst_stride = t[i].dst_stride;
        tasks[i].residual = (const __fp16 *)t[i].residual;
        tasks[i].res_stride = t[i].res_stride;
        tasks[i].rows = t[i].rows;
        tasks[i].cols = K;
        tasks[i].start_row = 0;
    }
    g_sdot_input_q8k_prequantized = prequantized ? 1 : 0;
    sdot_gemm_multi_dispatch((const __fp16 *)x, M, K, tasks, n_tasks);
}

/* The single-thread figure: sdot_gemm_multi_dispatch's work (ENG:4188-4262) -- the input quantized
 * once, then the reference's own job function exec_sdot_job_work_stealing (ENG:3491-3619) over all
 * rows -- run by the calling thread alone instead of the pool. */
KQREF_API void kqref_dispatch_1thread(const uint16_t *x, int M, int K, const kqref_task *t, int n_tasks) {
    static PoolJob job;
    int need_q8k = 0, need_q80 = 0, total = 0;
    if (n_tasks > 4) n_tasks = 4;
    memset(&job, 0, sizeof(job));
    for (int i = 0; i < n_tasks; ++i) {
        SdotMatrixTask *T = &job.sdot_tasks_inline[i];
        T->w_base = t[i].w_base;
        T->type = t[i].type;
        T->row_bytes = ggml_row_bytes(t[i].type, (size_t)K);
        T->dst = (__fp16 *)t[i].dst;
        T->dst_stride = t[i].dst_stride;
        T->residual = (const __fp16 *)t[i].residual;
        T->res_stride = t[i].res_stride;
        T->rows = t[i].rows;
        T->cols = K;
        T->start_row = total;
        total += t[i].rows;
        if (t[i].type == GGML_TYPE_Q8_0) need_q80 = 1;
        else need_q8k = 1;
    }
    g_sdot_input.M = M;
    g_sdot_input.K = K;
    g_sdot_input.x_fp16 = (const __fp16 *)x;
    for (int m = 0; m < M; ++m) {
        if (need_q8k) quantize_row_fp16_to_q8_k((const __fp16 *)x + (size_t)m * K, g_sdot_input.q8k[m], K);
        if (need_q80) quantize_row_fp16_to_q8_0((const __fp16 *)x + (size_t)m * K, g_sdot_input.q80[m], K);
    }
    job.type = 100;
    job.n_sdot_tasks = n_tasks;
    job.sdot_total_rows = total;
    job.total_chunks = (total + SDOT_ROW_GRAIN - 1) / SDOT_ROW_GRAIN;
    exec_sdot_job_work_stealing(&job);
}

/* One tensor record of the reference's GGUF parser (GgufTensorInfo, ENG:167-176). */
typedef struct {
    char name[128];
    uint32_t n_dims;
    uint64_t dims[4];
    uint32_t type;
    uint64_t rel_offset, abs_offset, n_elems, byte_size;
} kqref_gguf_tensor;

/* parse_gguf_file (ENG:376-413) over a GGUF image in memory, as the engine runs it on its mmap.
 * Returns the parser's result (1 ok, 0 rejected); on success fills up to cap tensor records and
 * the header fields.  The context is large (MAX_TENSORS records), so it lives on the heap. */
KQREF_API int kqref_gguf_parse(const void *bytes, size_t size, uint32_t *n_tensors, uint64_t *alignment,
                               uint64_t *data_offset, kqref_gguf_tensor *out, int cap) {
    GgufContext *ctx = (GgufContext *)calloc(1, sizeof(GgufContext));
    if (!ctx) return -1;
    ctx->base = (const uint8_t *)bytes;
    ctx->file_size = size;
    ctx->pos = 0;
    const int ok = parse_gguf_file(ctx);
    if (ok) {
        *n_tensors = ctx->n_tensors;
        *alignment = ctx->alignment;
        *data_offset = ctx->data_offset;
        for (uint32_t i = 0; i < ctx->n_tensors && (int)i < cap; ++i) {
            const GgufTensorInfo *t = &ctx->tensors[i];
            memcpy(out[i].name, t->name, sizeof(out[i].name));
            out[i].n_dims = t->n_dims;
            for (int d = 0; d < 4; ++d) out[i].dims[d] = t->dims[d];
            out[i].type = t->type;
            out[i].rel_offset = t->rel_offset;
            out[i].abs_offset = t->abs_offset;
            out[i].n_elems = t->n_elems;
            out[i].byte_size = t->byte_size;
        }
    }
    free(ctx->vocab_ptrs);
    free(ctx->vocab_lens);
    free(ctx);
    return ok;
}

/* find_tensor (ENG:415-420): index of the named tensor, or -1. */
KQREF_API int kqref_gguf_find(const void *bytes, size_t size, const char *name) {
    GgufContext *ctx = (GgufContext *)calloc(1, sizeof(GgufContext));
    if (!ctx) return -2;
    ctx->base = (const uint8_t *)bytes;
    ctx->file_size = size;
    int idx = -2;
    if (parse_gguf_file(ctx)) {
        const GgufTensorInfo *t = find_tensor(ctx, name);
        idx = t ? (int)(t - ctx->tensors) : -1;
    }
    free(ctx->vocab_ptrs);
    free(ctx->vocab_lens);
    free(ctx);
    return idx;
}
