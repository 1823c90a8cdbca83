// kq_internal.h -- host-side declarations shared by the CUDA translation units of libkq.
#pragma once

#include <cstddef>
#include <cstdint>
#include <cuda_runtime.h>

#include "kq_common.cuh"  // PeerOut

// A GGUF tensor resident in HBM in this library's row-group tile layout (opaque kq_weight of
// kq.h; layout in kq_common.cuh).
struct kq_weight {
    int device;        // CUDA device holding d
    uint32_t type;
    int rows, cols;
    size_t row_bytes;  // GGUF bytes per row (compute_ggml_bytes)
    uint8_t *d;        // tiled tensor, ceil(rows / 16) * 16 rows
    size_t bytes;
};

namespace kq {

// One matrix of a dispatch: weight rows [row_begin, row_begin + rows) of a tiled tensor.
struct GemvTaskHost {
    const uint8_t *w;      // tiled tensor (row group 0), device
    int row_begin;
    int rows;
    void *dst;             // __half*, output column r = local row r (or out_ids[r])
    long long dst_stride;
    const void *res;       // const __half*
    long long res_stride;
    float *dst_f32;
    long long f32_stride;
    int *dbg_sumi;         // [M][rows][blocks per row] or nullptr
    int *dbg_summ;
    const uint32_t *out_ids = nullptr;  // device; output column of local row r
    int index_base = 0;                 // argmax index of local row r
};

struct GemvLaunch {
    int type;
    int K;
    int M;                     // 1..8
    GemvTaskHost tasks[4];
    int n_tasks;
    // input: exactly one of x (fp16 [M][x_stride]), act (BlockQ8K[M][K/256] or BlockQ8_0_Fast[M][K/32])
    const void *x;
    long long x_stride;
    const void *act;
    int *status;
    unsigned long long timeout_ns;
    bool pdl;
    int num_sms;
    unsigned long long *argmax = nullptr;  // [M] packed keys (device), or nullptr
    int argmax_f16 = 0;
    int inject_wait = 0;  // failure-path test hook (see kq_set_option "inject_timeout")
    // Balanced split (optional): CTAs own equal tile ranges, row groups may be shared.  Needs
    // split_terms (gemv_split_bytes) and split_count (gemv_split_slots ints, all zero; every
    // launch leaves them zero unless it stopped early on a timeout).  nullptr: whole row groups.
    float *split_terms = nullptr;
    size_t split_terms_bytes = 0;
    int *split_count = nullptr;
    // Half row-group ownership allowed (Q4_K / Q5_K, 1-2 rows, where the plan finds it better)
    bool half_ok = true;
    PeerOut peer;  // n > 0: task 0's fp32 outputs also into every rank's gather buffer
};

// Wait (bounded) until every entry of the gather buffer of the step after this rank's completed
// steps carries that step's tag, write the values to `out` (may be nullptr) and count the step as
// completed.
struct PeerWait {
    unsigned long long *step;        // this rank's completed steps
    unsigned *arrivals;              // the wait kernel's CTA arrivals
    const unsigned long long *buf;   // this rank's entries
    long long buf_stride;            // entries per buffer
    long long n_entries;             // entries to read (M x row_stride)
    float *out;
    int *status;
    unsigned long long timeout_ns;
    bool pdl;  // may launch while the preceding kernel runs (it waits for it with griddepcontrol.wait)
};
cudaError_t launch_peer_wait(const PeerWait &W, cudaStream_t stream);

// Many-token product on the tensor cores (kq_gemm_tc.cu): tasks of one type, the input as fp16
// x or pre-quantized act (as in GemvLaunch), packed into `scratch` (tc_scratch_bytes) first.
struct TcLaunch {
    int type;
    int K;
    int M;
    GemvTaskHost tasks[4];
    int n_tasks;
    const void *x;
    long long x_stride;
    const void *act;
    void *scratch;
    size_t scratch_bytes;
    int *status;
    unsigned long long timeout_ns;
    int num_sms = 0;
    void *terms = nullptr;       // split-K block terms (tc_split_terms_bytes)
    size_t terms_bytes = 0;
};

// kq_gemv.cu
cudaError_t launch_gemv(const GemvLaunch &L, cudaStream_t stream);

// The FFN block for 1-2 tokens as one persistent kernel (kq_ffn_fused.cu): RMSNorm + Q8_K ->
// gate / up -> SwiGLU + Q8_K -> down + residual, bit for bit the four-launch form.
struct FfnFusedLaunch {
    int gate_type, down_type;  // gate and up share a type
    int hidden, ffn, M;        // M in 1..2
    const uint8_t *gate, *up, *down;  // tiled weights
    const void *x, *gamma;     // fp16 [M][hidden], [hidden]
    void *g, *u;               // fp16 [M][ffn] scratch, 16-byte aligned
    void *y;                   // fp16 [M][hidden]
    const float *exp_tab;      // SwiGLU expf table, or nullptr
    float *split_terms;        // gemv_split_bytes(down_type, ffn, M, num_sms)
    int *split_count;          // gemv_split_slots(num_sms) ints, zero
    unsigned *gbar;            // 2 words, zero before the first launch
    int *pair;                 // ffn / 16 ints, zero before the first launch
    int *status;
    unsigned long long timeout_ns;
    bool pdl;
    int num_sms;               // the grid: one CTA per SM, all resident
};
bool ffn_fused_supported(int gate_type, int down_type, int hidden, int ffn, int M, int num_sms);
// cudaErrorNotSupported when the shapes or types have no plan
cudaError_t launch_ffn_fused(const FfnFusedLaunch &L, cudaStream_t stream);
// scratch of a split GEMV launch of M (<= 8) tokens: term bytes and counter slots
size_t gemv_split_bytes(int type, int K, int M, int num_sms);
int gemv_split_slots(int num_sms);
// rows ids[0..n) of a tiled tensor -> a new tiled tensor of n rows (weight_bytes(type, n, K))
// kq_gemm_tc.cu
size_t tc_scratch_bytes(int type, int M, int K);
// bytes of the split-K term buffer the row-major kernel needs for these tasks (0: no split)
size_t tc_split_terms_bytes(int type, int M, int K, const int *task_rows, const int *task_rgs, int n_tasks, int sms);
// rough time of the row-major kernel for tasks of task_rgs[i] row groups (cost model, microseconds)
double tc_estimate_us(int type, int M, int K, const int *task_rgs, int n_tasks, int sms);
cudaError_t launch_gemm_tc(const TcLaunch &L, cudaStream_t stream);
// token-major variant (activation in tensor memory, row groups spread over all SMs)
size_t tc2_scratch_bytes(int type, int M, int K);
cudaError_t launch_gemm_tc2(const TcLaunch &L, cudaStream_t stream);

cudaError_t launch_gather_rows(int type, int K, const uint8_t *src, const uint32_t *ids, int n, uint8_t *dst,
                               cudaStream_t stream);

// kq_act.cu
cudaError_t launch_quantize(int target_type /*12 = Q8_K, 8 = Q8_0*/, const void *x, long long x_stride, int M, int K,
                            void *out, cudaStream_t stream);
cudaError_t launch_repack(int type, const uint8_t *gguf, uint8_t *dev, int rows, int K, cudaStream_t stream);
cudaError_t launch_rmsnorm_q8k(const void *x, const void *gamma, void *out, void *q8k, int M, int K, cudaStream_t stream,
                               bool pdl);
// exp_tab: expf(-g) per fp16 pattern of g (fill_swiglu_exp_table), or nullptr for an fp64 exp on the GPU
cudaError_t launch_swiglu_q8k(void *gate, const void *up, void *q8k, int M, int N, cudaStream_t stream, bool pdl,
                              const float *exp_tab);
// host: tab[65536] = expf(-g) with this host's C library, g = every fp16 bit pattern
void fill_swiglu_exp_table(float *tab);
// keys[m] = argmax key over the fp16 logits [M][stride] rows 0..rows-1 (keys zeroed before)
cudaError_t launch_logits_argmax(const void *logits, long long stride, int rows, int M, unsigned long long *keys,
                                 cudaStream_t stream);
// status (optional): when it holds an error, every row gets token 0xFFFFFFFF and value NaN
cudaError_t launch_argmax_finalize(const unsigned long long *keys, int M, const uint32_t *ids, uint32_t *toks,
                                   float *vals, cudaStream_t stream, const int *status = nullptr);
// rows [row_begin, row_begin + rows) to fp16, or (ids != nullptr) rows ids[0..rows) of a weight of
// w_rows rows, out-of-range ids giving zeros and DEV_ERR_INDEX in *status
cudaError_t launch_dequant(int type, const uint8_t *tiled, int row_begin, int rows, int K, void *out, cudaStream_t stream,
                           const uint32_t *ids = nullptr, int w_rows = 0, int *status = nullptr);

}  // namespace kq
