/*
 * kq_oracle.h -- CPU restatement of the reference engine's GGUF K-quant matmul path.
 *
 * TEST INFRASTRUCTURE ONLY.  This library is the parity checker for the CUDA kernels in
 * npu880_mtk_npu_llm_runtime_b200/csrc.  Only tests/, __graft_entry__.smoke() and the
 * cpu_baseline leg of bench.py may load it.  The product path never calls into it.
 *
 * Every function restates the SCALAR (non-NEON) path of the reference engine
 * src/v182_r22_breakthrough_engine.c ("ENG" below); each cites the lines it follows.
 * The restatement is pinned bit-exactly against the reference itself (compiled unmodified
 * from its own sources by oracle/Makefile into oracle/_ref/) through the golden fixtures in
 * tests/golden/.
 *
 * fp32 evaluation order matches the reference scalar code operation by operation; the
 * library is compiled WITHOUT fp-contraction into FMA (x86-64 baseline has no FMA and the
 * Makefile passes -ffp-contract=off), exactly like the reference harness build.
 */
#ifndef KQ_ORACLE_H
#define KQ_ORACLE_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* GGML type ids, ENG:115-120 */
#define KQO_TYPE_F32  0
#define KQO_TYPE_F16  1
#define KQO_TYPE_Q8_0 8
#define KQO_TYPE_Q4_K 12
#define KQO_TYPE_Q5_K 13
#define KQO_TYPE_Q6_K 14

/* Activation block quantized to 8 bits per 256 values: ENG:868-872 (BlockQ8K, 292 bytes).
 * Not ggml's Q8_K: float d and eight 32-element sums. */
typedef struct {
    float   d;
    int8_t  qs[256];
    int32_t bsum32[8];
} kqo_block_q8k;

/* Activation block quantized to 8 bits per 32 values: ENG:874-877 (BlockQ8_0_Fast, 36 bytes). */
typedef struct {
    float  d;
    int8_t qs[32];
} kqo_block_q8_0;

/* compute_ggml_bytes, ENG:364-374 (row size of K elements; 0 for unknown types) */
uint64_t kqo_row_bytes(uint32_t type, uint64_t k);

/* half <-> float, RNE (ENG:592-596 uses the compiler's __fp16 conversion) */
float    kqo_f16_to_f32(uint16_t h);
uint16_t kqo_f32_to_f16(float f);
void     kqo_f32_to_f16_array(const float *x, uint16_t *y, size_t n);

/* get_scale_min_k4, ENG:743-749 */
void kqo_get_scale_min_k4(int j, const uint8_t *q, uint8_t *d, uint8_t *m);

/* quantize_row_fp16_to_q8_k (scalar path), ENG:925-990; k % 256 == 0 */
void kqo_quantize_row_q8k(const uint16_t *x, kqo_block_q8k *y, int k);
/* quantize_row_fp16_to_q8_0 (scalar path), ENG:1016-1064; k % 32 == 0 */
void kqo_quantize_row_q8_0(const uint16_t *x, kqo_block_q8_0 *y, int k);

/* One weight row dotted with one quantized activation row: the per-row vec_dot of
 * eval_single_lm_row_dot (ENG:10986-11105) / sdot_row_q5_k_batch, _q6_k_batch, _q8_0_batch
 * (scalar paths ENG:3192-3231, 3323-3365, 3393-3407).
 *   type Q4_K/Q5_K/Q6_K: act is kqo_block_q8k[k/256]; Q8_0: act is kqo_block_q8_0[k/32].
 * If sumi != NULL, the per-super-block integer intermediate is written there
 * (Q4_K/Q5_K: sum_j sc_j*dot_j; Q6_K: sum_s sc_s*dot_s; Q8_0: the 32-element dot), one per
 * block.  If summ != NULL (Q4_K/Q5_K only), sum_j m_j*bsum32_j per super-block.
 * Returns the fp32 row result; unknown types return -1e30f like ENG:11104. */
float kqo_vec_dot(uint32_t type, const uint8_t *w_row, const void *act, int k,
                  int32_t *sumi, int32_t *summ);

/* rows x M product: out[m*ld_out + r] = vec_dot(row r, act row m).
 * act rows are contiguous: Q8_K act is kqo_block_q8k[M][k/256], Q8_0 is kqo_block_q8_0[M][k/32]. */
void kqo_gemm(uint32_t type, const uint8_t *w, size_t row_bytes, int rows, int k,
              const void *act, int M, float *out, size_t ld_out);

/* Per-row fp16 epilogue of exec_sdot_job_work_stealing, ENG:3586-3612:
 * dst[m*dst_stride + r] = (fp16)(sum [+ (float)residual[m*res_stride + r]]) */
void kqo_epilogue_f16(const float *sums, size_t ld_sums, int rows, int M,
                      uint16_t *dst, size_t dst_stride,
                      const uint16_t *residual, size_t res_stride);

/* Dequantizers (scalar paths) to fp16: dequant_block_q8_0 ENG:598-615,
 * dequant_block_q6_k ENG:673-741, dequant_block_q4_k ENG:758-801, dequant_block_q5_k
 * ENG:803-853.  n_elems must be a multiple of the block size. */
void kqo_dequant_row(uint32_t type, const uint8_t *w_row, int n_elems, uint16_t *dst);

/* rmsnorm_fp16_rows_fast, scalar path ENG:4291-4299 (eps 1e-6).  When q8k != NULL and
 * K % 256 == 0 the normalised fp16 rows are also quantized to Q8_K (ENG:4304-4306). */
void kqo_rmsnorm_rows(const uint16_t *x_in, const uint16_t *gamma, uint16_t *x_out,
                      int M, int K, kqo_block_q8k *q8k);

/* swiglu_chunk_worker scalar path ENG:4350-4357: gate = fp16(silu(gate) * up) in place,
 * then Q8_K of each 256 chunk when q8k != NULL.  N % 256 == 0. */
void kqo_swiglu_rows(uint16_t *gate_inout, const uint16_t *up_in, int M, int N,
                     kqo_block_q8k *q8k);

/* The CPU SDOT FFN sequence ENG:8283-8298 (the fallback of run_real_npu_universal_ffn):
 *   xn = rmsnorm(x_in, gamma) -> Q8_K; g = fp16(W_gate . xn); u = fp16(W_up . xn);
 *   h = fp16(silu(g) * u) -> Q8_K; x_out = fp16(W_down . h + x_in)
 * Shapes: x_in/x_out [M][hidden], W_gate/W_up [ffn][hidden], W_down [hidden][ffn]. */
void kqo_ffn(uint32_t gate_type, const uint8_t *w_gate, uint32_t up_type, const uint8_t *w_up,
             uint32_t down_type, const uint8_t *w_down, int hidden, int ffn,
             const uint16_t *x_in, const uint16_t *gamma, uint16_t *x_out, int M);

/* Argmax over a row-id list, strict '>' so the first maximal row in list order wins.
 *   f16_compare == 0: compare fp32 row results, the scan of exec_cyrillic_lm_work_item
 *                     (scalar branch ENG:9557-9571);
 *   f16_compare != 0: compare the fp16-rounded logits the dispatch stored, the scan of
 *                     run_final_norm_and_lm_head_batch_sdot (ENG:11182-11193) and of
 *                     run_final_norm_and_lm_head_pipelined (ENG:9699-9707).
 * best_val receives the compared value (fp32, or the fp16 value widened to fp32).
 * If logits != NULL, logits[m*n_rows + i] receives the fp32 result of row_ids[i]. */
void kqo_rows_argmax(uint32_t type, const uint8_t *w, size_t row_bytes, int k,
                     const uint32_t *row_ids, int n_rows, const void *act, int M,
                     int f16_compare, float *logits, uint32_t *best_id, float *best_val);

#ifdef __cplusplus
}
#endif
#endif
