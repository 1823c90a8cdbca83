// kq_gemv.cu -- K-quant x Q8 matrix-vector / small-batch product for sm_100a.
//
// Replaces the engine's NEON row kernels (sdot_4rows_<type>_m1 / _batch, sdot_row_<type>_batch,
// src/v182_r22_breakthrough_engine.c:1226-3440) and its pinned work-stealing pool
// (exec_sdot_job_work_stealing, ENG:3491-3619) for M <= 8 activation rows.
//
// Design (HBM-bound: every weight byte is read once, activations are tiny):
//  * Persistent-style grid, at most a few CTAs per SM.  CTA c owns a contiguous range of the
//    dispatch's concatenated output rows (the reference's 64-row grains, ENG:3502, become
//    one balanced range per CTA).
//  * Warp 8 is the producer: one lane streams the CTA's rows through an NS-deep ring of
//    shared-memory stages with cp.async.bulk (the TMA engine), one bulk copy per stage of
//    whole consecutive rows, completion counted on an mbarrier, L2 evict-first.
//  * Warps 0-7 are consumers.  Before the first stage they quantize the fp16 activation to
//    Q8_K / Q8_0 in shared memory (bit-exact to quantize_row_fp16_to_q8_k, ENG:925-990) or copy
//    a pre-quantized one.  Per stage, each thread takes whole 256-value units (one super-block,
//    or eight Q8_0 blocks) and computes the exact integer sub-block sums with dp4a, then the
//    fp32 block term with the reference's operation order.  After a consumer barrier the stage
//    is released and one thread per (row, token) adds the block terms in block order -- the
//    same fp32 sequence as the reference's `acc += term` loop, so results are bit-identical to
//    the scalar reference -- and applies the epilogue (fp32 out, fp16 out, fp16 residual).
//  * Every wait is bounded (globaltimer); on timeout the kernel records DEV_ERR_TIMEOUT,
//    drains its own copies in flight (bounded) and returns.
#include "kq_common.cuh"
#include "kq_internal.h"

#include <algorithm>
#include <mutex>
#include <unordered_map>

namespace kq {

constexpr int kConsumerWarps = 8;
constexpr int kConsumers = kConsumerWarps * 32;
constexpr int kThreads = kConsumers + 32;
constexpr int kMaxStages = 8;

struct GemvTaskDev {
    const uint8_t *w;
    int rows;
    int row_start;  // first row of this task in the concatenated row space
    __half *dst;
    long long dst_stride;
    const __half *res;
    long long res_stride;
    float *dst_f32;
    long long f32_stride;
    int *dbg_sumi;
    int *dbg_summ;
    const uint32_t *row_ids;  // gathered rows: stage row i is weight row row_ids[r0 + i]
    int scatter;              // write dst/dst_f32 at column row_ids[r] instead of r
    int index_base;           // argmax index of local row r is index_base + r
};

struct GemvParams {
    GemvTaskDev task[4];
    int n_tasks;
    int total_rows;
    int K;
    int nbu;              // 256-value units per row
    int M;
    unsigned int row_bytes;
    int rows_per_stage;
    int n_stages;
    unsigned int stage_bytes;
    int terms_per_row;    // nbu (K-quants) or 8 * nbu (Q8_0)
    const __half *x;
    long long x_stride;
    const void *act;
    int *status;
    unsigned long long timeout_ns;
    unsigned long long *argmax;  // [M] packed (ordered value, ~index) keys, or nullptr
    int argmax_f16;              // compare the fp16-rounded results (the dispatch's stored logits)
    int inject_wait;             // failure test: consumers first wait on a barrier nothing arrives at
    unsigned int off_act, off_terms, off_stages, off_bars;
};

// Total order on floats as unsigned keys: larger float -> larger key.
__device__ __forceinline__ unsigned long long argmax_key(float v, uint32_t index) {
    const uint32_t b = __float_as_uint(v);
    const uint32_t o = (b & 0x80000000u) ? ~b : (b | 0x80000000u);
    return ((unsigned long long)o << 32) | (unsigned long long)(0xFFFFFFFFu - index);
}

// ------------------------------------------------------------------ activation staging

// Quantize 256 fp16 values of one token into an ActUnit (one warp).  K-quant weights get the
// Q8_K block (ENG:925-990); Q8_0 weights get eight Q8_0 blocks (ENG:1016-1064).
template <int TYPE>
__device__ __forceinline__ void stage_act_from_fp16(const __half *xu, bool vec_ok, ActUnit *a, int lane) {
    float v[8];
    if (vec_ok) {
        const uint4 raw = *reinterpret_cast<const uint4 *>(xu + 8 * lane);
        const __half2 *h2 = reinterpret_cast<const __half2 *>(&raw);
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            const float2 f = __half22float2(h2[i]);
            v[2 * i] = f.x;
            v[2 * i + 1] = f.y;
        }
    } else {
#pragma unroll
        for (int i = 0; i < 8; ++i) v[i] = __half2float(xu[8 * lane + i]);
    }
    float amax = 0.0f;
#pragma unroll
    for (int i = 0; i < 8; ++i) amax = fmaxf(amax, fabsf(v[i]));
    // K-quants: max over the whole 256 (32 lanes); Q8_0: over each 32-value block (4 lanes)
    const int span = (TYPE == TYPE_Q8_0) ? 4 : 32;
#pragma unroll
    for (int o = 1; o < span; o <<= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));

    int q[8];
    if (amax == 0.0f) {
#pragma unroll
        for (int i = 0; i < 8; ++i) q[i] = 0;
    } else {
        const float inv = __fdiv_rn(127.0f, amax);
#pragma unroll
        for (int i = 0; i < 8; ++i) {
            int t = __float2int_rn(__fmul_rn(v[i], inv));
            q[i] = max(-127, min(127, t));
        }
    }
    const uint32_t lo = (uint32_t)(q[0] & 0xFF) | ((uint32_t)(q[1] & 0xFF) << 8) | ((uint32_t)(q[2] & 0xFF) << 16) |
                        ((uint32_t)(q[3] & 0xFF) << 24);
    const uint32_t hi = (uint32_t)(q[4] & 0xFF) | ((uint32_t)(q[5] & 0xFF) << 8) | ((uint32_t)(q[6] & 0xFF) << 16) |
                        ((uint32_t)(q[7] & 0xFF) << 24);
    *reinterpret_cast<uint2 *>(a->qs + 8 * lane) = make_uint2(lo, hi);
    int s8 = q[0] + q[1] + q[2] + q[3] + q[4] + q[5] + q[6] + q[7];
    const int s16 = s8 + __shfl_xor_sync(0xffffffffu, s8, 1);
    const int s32 = s16 + __shfl_xor_sync(0xffffffffu, s16, 2);
    if ((lane & 1) == 0) a->xsum16[lane >> 1] = s16;
    if (TYPE == TYPE_Q8_0) {
        if ((lane & 3) == 0) a->aux[lane >> 2] = __float_as_int(amax == 0.0f ? 0.0f : __fdiv_rn(amax, 127.0f));
    } else {
        if ((lane & 3) == 0) a->aux[lane >> 2] = s32;
        if (lane == 0) a->d = (amax == 0.0f) ? 0.0f : __fdiv_rn(amax, 127.0f);
    }
}

// Copy one pre-quantized BlockQ8K (292 B, 4-byte aligned) into an ActUnit (one warp).
__device__ __forceinline__ void stage_act_from_q8k(const BlockQ8K *src, ActUnit *a, int lane) {
    const uint32_t *w = reinterpret_cast<const uint32_t *>(src);
    const uint32_t lo = w[1 + 2 * lane], hi = w[2 + 2 * lane];
    *reinterpret_cast<uint2 *>(a->qs + 8 * lane) = make_uint2(lo, hi);
    int s8 = 0;
#pragma unroll
    for (int i = 0; i < 4; ++i) s8 += (int)(int8_t)byte_of(lo, i) + (int)(int8_t)byte_of(hi, i);
    const int s16 = s8 + __shfl_xor_sync(0xffffffffu, s8, 1);
    if ((lane & 1) == 0) a->xsum16[lane >> 1] = s16;
    if (lane < 8) a->aux[lane] = (int)w[65 + lane];
    if (lane == 0) a->d = __int_as_float((int)w[0]);
}

// Copy eight pre-quantized BlockQ8_0_Fast (36 B each) into an ActUnit (one warp).
__device__ __forceinline__ void stage_act_from_q80(const BlockQ80 *src, ActUnit *a, int lane) {
    const int j = lane >> 2, part = lane & 3;
    const uint32_t *w = reinterpret_cast<const uint32_t *>(src + j);
    const uint32_t lo = w[1 + 2 * part], hi = w[2 + 2 * part];
    *reinterpret_cast<uint2 *>(a->qs + 8 * lane) = make_uint2(lo, hi);
    if (part == 0) a->aux[j] = (int)w[0];
}

// ------------------------------------------------------------------ per-unit dot products

// Q4_K super-block (ENG:758-801 layout) x Q8_K, all tokens.  Integer sums are exact; the
// fp32 term is dx * (d * sumi - dmin * summ) with each operation rounded separately
// (eval_single_lm_row_dot, ENG:11025).
template <int MT>
__device__ __forceinline__ void unit_q4k(const uint8_t *blk, const ActUnit *au, int nbu, int M, float *term,
                                         int *dsumi, int *dsumm, long long dstride) {
    const uint4 h = *reinterpret_cast<const uint4 *>(blk);
    uint4 q[8];
#pragma unroll
    for (int i = 0; i < 8; ++i) q[i] = reinterpret_cast<const uint4 *>(blk + 16)[i];
    const float d = half_bits_to_float(h.x), dmin = half_bits_to_float(h.x >> 16);
    // get_scale_min_k4 (ENG:743-749) for all eight sub-blocks at once
    const uint32_t sc03 = h.y & 0x3F3F3F3Fu, mn03 = h.z & 0x3F3F3F3Fu;
    const uint32_t sc47 = (h.w & 0x0F0F0F0Fu) | ((h.y >> 2) & 0x30303030u);
    const uint32_t mn47 = ((h.w >> 4) & 0x0F0F0F0Fu) | ((h.z >> 2) & 0x30303030u);
#pragma unroll
    for (int m = 0; m < MT; ++m) {
        if (m < M) {
            const ActUnit *a = au + (size_t)m * nbu;
            const uint4 *xv = reinterpret_cast<const uint4 *>(a->qs);
            int sumi = 0;
#pragma unroll
            for (int c = 0; c < 4; ++c) {
                const uint4 x0 = xv[4 * c + 0], x1 = xv[4 * c + 1], x2 = xv[4 * c + 2], x3 = xv[4 * c + 3];
                const uint4 qa = q[2 * c], qb = q[2 * c + 1];
                int dl = 0, dh = 0;
                dl = dp4a_us(qa.x & 0x0F0F0F0Fu, (int)x0.x, dl);
                dl = dp4a_us(qa.y & 0x0F0F0F0Fu, (int)x0.y, dl);
                dl = dp4a_us(qa.z & 0x0F0F0F0Fu, (int)x0.z, dl);
                dl = dp4a_us(qa.w & 0x0F0F0F0Fu, (int)x0.w, dl);
                dl = dp4a_us(qb.x & 0x0F0F0F0Fu, (int)x1.x, dl);
                dl = dp4a_us(qb.y & 0x0F0F0F0Fu, (int)x1.y, dl);
                dl = dp4a_us(qb.z & 0x0F0F0F0Fu, (int)x1.z, dl);
                dl = dp4a_us(qb.w & 0x0F0F0F0Fu, (int)x1.w, dl);
                dh = dp4a_us((qa.x >> 4) & 0x0F0F0F0Fu, (int)x2.x, dh);
                dh = dp4a_us((qa.y >> 4) & 0x0F0F0F0Fu, (int)x2.y, dh);
                dh = dp4a_us((qa.z >> 4) & 0x0F0F0F0Fu, (int)x2.z, dh);
                dh = dp4a_us((qa.w >> 4) & 0x0F0F0F0Fu, (int)x2.w, dh);
                dh = dp4a_us((qb.x >> 4) & 0x0F0F0F0Fu, (int)x3.x, dh);
                dh = dp4a_us((qb.y >> 4) & 0x0F0F0F0Fu, (int)x3.y, dh);
                dh = dp4a_us((qb.z >> 4) & 0x0F0F0F0Fu, (int)x3.z, dh);
                dh = dp4a_us((qb.w >> 4) & 0x0F0F0F0Fu, (int)x3.w, dh);
                const uint32_t scw = (c < 2) ? sc03 : sc47;
                sumi += (int)byte_of(scw, 2 * (c & 1)) * dl + (int)byte_of(scw, 2 * (c & 1) + 1) * dh;
            }
            const int4 b0 = *reinterpret_cast<const int4 *>(a->aux);
            const int4 b1 = *reinterpret_cast<const int4 *>(a->aux + 4);
            const int summ = (int)byte_of(mn03, 0) * b0.x + (int)byte_of(mn03, 1) * b0.y +
                             (int)byte_of(mn03, 2) * b0.z + (int)byte_of(mn03, 3) * b0.w +
                             (int)byte_of(mn47, 0) * b1.x + (int)byte_of(mn47, 1) * b1.y +
                             (int)byte_of(mn47, 2) * b1.z + (int)byte_of(mn47, 3) * b1.w;
            const float t = __fsub_rn(__fmul_rn(d, __int2float_rn(sumi)), __fmul_rn(dmin, __int2float_rn(summ)));
            term[m] = __fmul_rn(a->d, t);
            if (dsumi) {
                dsumi[m * dstride] = sumi;
                dsumm[m * dstride] = summ;
            }
        }
    }
}

// Q5_K super-block (ENG:803-853 layout): the fifth bit of value l of chunk c is bit 2c (low
// half) / 2c+1 (high half) of qh[l].
template <int MT>
__device__ __forceinline__ void unit_q5k(const uint8_t *blk, const ActUnit *au, int nbu, int M, float *term,
                                         int *dsumi, int *dsumm, long long dstride) {
    const uint4 h = *reinterpret_cast<const uint4 *>(blk);
    const uint4 qh0 = reinterpret_cast<const uint4 *>(blk + 16)[0];
    const uint4 qh1 = reinterpret_cast<const uint4 *>(blk + 16)[1];
    uint4 q[8];
#pragma unroll
    for (int i = 0; i < 8; ++i) q[i] = reinterpret_cast<const uint4 *>(blk + 48)[i];
    const uint32_t qhw[8] = {qh0.x, qh0.y, qh0.z, qh0.w, qh1.x, qh1.y, qh1.z, qh1.w};
    const float d = half_bits_to_float(h.x), dmin = half_bits_to_float(h.x >> 16);
    const uint32_t sc03 = h.y & 0x3F3F3F3Fu, mn03 = h.z & 0x3F3F3F3Fu;
    const uint32_t sc47 = (h.w & 0x0F0F0F0Fu) | ((h.y >> 2) & 0x30303030u);
    const uint32_t mn47 = ((h.w >> 4) & 0x0F0F0F0Fu) | ((h.z >> 2) & 0x30303030u);
#pragma unroll
    for (int m = 0; m < MT; ++m) {
        if (m < M) {
            const ActUnit *a = au + (size_t)m * nbu;
            const uint4 *xv = reinterpret_cast<const uint4 *>(a->qs);
            int sumi = 0;
#pragma unroll
            for (int c = 0; c < 4; ++c) {
                const uint4 x0 = xv[4 * c + 0], x1 = xv[4 * c + 1], x2 = xv[4 * c + 2], x3 = xv[4 * c + 3];
                const uint32_t qw[8] = {q[2 * c].x, q[2 * c].y, q[2 * c].z, q[2 * c].w,
                                        q[2 * c + 1].x, q[2 * c + 1].y, q[2 * c + 1].z, q[2 * c + 1].w};
                const uint32_t xl[8] = {x0.x, x0.y, x0.z, x0.w, x1.x, x1.y, x1.z, x1.w};
                const uint32_t xh[8] = {x2.x, x2.y, x2.z, x2.w, x3.x, x3.y, x3.z, x3.w};
                int dl = 0, dh = 0;
#pragma unroll
                for (int i = 0; i < 8; ++i) {
                    const uint32_t wl = (qw[i] & 0x0F0F0F0Fu) | (((qhw[i] >> (2 * c)) & 0x01010101u) << 4);
                    const uint32_t wh = ((qw[i] >> 4) & 0x0F0F0F0Fu) | (((qhw[i] >> (2 * c + 1)) & 0x01010101u) << 4);
                    dl = dp4a_us(wl, (int)xl[i], dl);
                    dh = dp4a_us(wh, (int)xh[i], dh);
                }
                const uint32_t scw = (c < 2) ? sc03 : sc47;
                sumi += (int)byte_of(scw, 2 * (c & 1)) * dl + (int)byte_of(scw, 2 * (c & 1) + 1) * dh;
            }
            const int4 b0 = *reinterpret_cast<const int4 *>(a->aux);
            const int4 b1 = *reinterpret_cast<const int4 *>(a->aux + 4);
            const int summ = (int)byte_of(mn03, 0) * b0.x + (int)byte_of(mn03, 1) * b0.y +
                             (int)byte_of(mn03, 2) * b0.z + (int)byte_of(mn03, 3) * b0.w +
                             (int)byte_of(mn47, 0) * b1.x + (int)byte_of(mn47, 1) * b1.y +
                             (int)byte_of(mn47, 2) * b1.z + (int)byte_of(mn47, 3) * b1.w;
            const float t = __fsub_rn(__fmul_rn(d, __int2float_rn(sumi)), __fmul_rn(dmin, __int2float_rn(summ)));
            term[m] = __fmul_rn(a->d, t);
            if (dsumi) {
                dsumi[m * dstride] = sumi;
                dsumm[m * dstride] = summ;
            }
        }
    }
}

// Q6_K super-block, device layout [ql 128][qh 64][scales 16] (d passed separately).
// Value e = 128h + 32g + l: low 4 bits from ql[64h + l + 32(g&1)] (high nibble when g >= 2),
// bits 4-5 from qh[32h + l] >> 2g, minus 32; sub-block s = 8h + 2g + (l >= 16) (ENG:11065-11101).
// sum (q - 32) x = sum q x - 32 * (sum of the 16 activation quants), all exact integers.
template <int MT>
__device__ __forceinline__ void unit_q6k(const uint8_t *blk, float d, const ActUnit *au, int nbu, int M,
                                         float *term, int *dsumi, int *dsumm, long long dstride) {
    uint32_t ql[32], qh[16];
#pragma unroll
    for (int i = 0; i < 8; ++i) {
        const uint4 v = reinterpret_cast<const uint4 *>(blk)[i];
        ql[4 * i] = v.x; ql[4 * i + 1] = v.y; ql[4 * i + 2] = v.z; ql[4 * i + 3] = v.w;
    }
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        const uint4 v = reinterpret_cast<const uint4 *>(blk + 128)[i];
        qh[4 * i] = v.x; qh[4 * i + 1] = v.y; qh[4 * i + 2] = v.z; qh[4 * i + 3] = v.w;
    }
    const uint4 scv = reinterpret_cast<const uint4 *>(blk + 192)[0];
    const uint32_t scw[4] = {scv.x, scv.y, scv.z, scv.w};
#pragma unroll
    for (int m = 0; m < MT; ++m) {
        if (m < M) {
            const ActUnit *a = au + (size_t)m * nbu;
            const uint4 *xv = reinterpret_cast<const uint4 *>(a->qs);
            int sumi = 0;
#pragma unroll
            for (int hh = 0; hh < 2; ++hh) {
#pragma unroll
                for (int half16 = 0; half16 < 2; ++half16) {
                    int dg[4] = {0, 0, 0, 0};
                    const uint4 xg0 = xv[8 * hh + 0 + half16];
                    const uint4 xg1 = xv[8 * hh + 2 + half16];
                    const uint4 xg2 = xv[8 * hh + 4 + half16];
                    const uint4 xg3 = xv[8 * hh + 6 + half16];
                    const uint32_t x0[4] = {xg0.x, xg0.y, xg0.z, xg0.w};
                    const uint32_t x1[4] = {xg1.x, xg1.y, xg1.z, xg1.w};
                    const uint32_t x2[4] = {xg2.x, xg2.y, xg2.z, xg2.w};
                    const uint32_t x3[4] = {xg3.x, xg3.y, xg3.z, xg3.w};
#pragma unroll
                    for (int ww = 0; ww < 4; ++ww) {
                        const int w = 4 * half16 + ww;
                        const uint32_t B0 = ql[16 * hh + w], B1 = ql[16 * hh + 8 + w], HB = qh[8 * hh + w];
                        const uint32_t q0 = (B0 & 0x0F0F0F0Fu) | ((HB << 4) & 0x30303030u);
                        const uint32_t q1 = (B1 & 0x0F0F0F0Fu) | ((HB << 2) & 0x30303030u);
                        const uint32_t q2 = ((B0 >> 4) & 0x0F0F0F0Fu) | (HB & 0x30303030u);
                        const uint32_t q3 = ((B1 >> 4) & 0x0F0F0F0Fu) | ((HB >> 2) & 0x30303030u);
                        dg[0] = dp4a_us(q0, (int)x0[ww], dg[0]);
                        dg[1] = dp4a_us(q1, (int)x1[ww], dg[1]);
                        dg[2] = dp4a_us(q2, (int)x2[ww], dg[2]);
                        dg[3] = dp4a_us(q3, (int)x3[ww], dg[3]);
                    }
#pragma unroll
                    for (int g = 0; g < 4; ++g) {
                        const int s = 8 * hh + 2 * g + half16;
                        const int sc = (int)(int8_t)byte_of(scw[s >> 2], s & 3);
                        sumi += sc * (dg[g] - 32 * a->xsum16[s]);
                    }
                }
            }
            term[m] = __fmul_rn(__fmul_rn(d, a->d), __int2float_rn(sumi));
            if (dsumi) {
                dsumi[m * dstride] = sumi;
                dsumm[m * dstride] = 0;
            }
        }
    }
}

// Eight Q8_0 blocks (device layout: 256 int8 quants here, 8 fp16 scales in the row's d plane).
// term j = (d_j * dx_j) * dot_j (sdot_row_q8_0_batch, ENG:3393-3407).  T = 8 terms per unit.
template <int MT>
__device__ __forceinline__ void unit_q80(const uint8_t *qs, const uint8_t *dptr, const ActUnit *au, int nbu, int M,
                                         float *term /* [8][MT] */, int *dsumi, int *dsumm, long long dstride) {
    uint4 q[16];
#pragma unroll
    for (int i = 0; i < 16; ++i) q[i] = reinterpret_cast<const uint4 *>(qs)[i];
    const uint4 dv = *reinterpret_cast<const uint4 *>(dptr);
    const uint32_t dw[4] = {dv.x, dv.y, dv.z, dv.w};
#pragma unroll
    for (int m = 0; m < MT; ++m) {
        if (m < M) {
            const ActUnit *a = au + (size_t)m * nbu;
            const uint4 *xv = reinterpret_cast<const uint4 *>(a->qs);
#pragma unroll
            for (int j = 0; j < 8; ++j) {
                const uint4 xa = xv[2 * j], xb = xv[2 * j + 1];
                const uint4 wa = q[2 * j], wb = q[2 * j + 1];
                int dot = 0;
                dot = dp4a_ss((int)wa.x, (int)xa.x, dot);
                dot = dp4a_ss((int)wa.y, (int)xa.y, dot);
                dot = dp4a_ss((int)wa.z, (int)xa.z, dot);
                dot = dp4a_ss((int)wa.w, (int)xa.w, dot);
                dot = dp4a_ss((int)wb.x, (int)xb.x, dot);
                dot = dp4a_ss((int)wb.y, (int)xb.y, dot);
                dot = dp4a_ss((int)wb.z, (int)xb.z, dot);
                dot = dp4a_ss((int)wb.w, (int)xb.w, dot);
                const float dwj = half_bits_to_float(dw[j >> 1] >> (16 * (j & 1)));
                const float dxj = __int_as_float(a->aux[j]);
                term[j * MT + m] = __fmul_rn(__fmul_rn(dwj, dxj), __int2float_rn(dot));
                if (dsumi) {
                    dsumi[m * dstride + j] = dot;
                    dsumm[m * dstride + j] = 0;
                }
            }
        }
    }
}

// ------------------------------------------------------------------ stage iteration

// The CTA's rows are walked in stages of at most rows_per_stage consecutive rows of one task.
struct StageCursor {
    int g, g_end, t;
};

__device__ __forceinline__ bool next_stage(const GemvParams &p, StageCursor &c, int &t, int &r0, int &R) {
    if (c.g >= c.g_end) return false;
    while (c.t + 1 < p.n_tasks && c.g >= p.task[c.t + 1].row_start) ++c.t;
    t = c.t;
    r0 = c.g - p.task[t].row_start;
    R = min(p.rows_per_stage, min(c.g_end - c.g, p.task[t].rows - r0));
    c.g += R;
    return true;
}

// ------------------------------------------------------------------ the kernel

template <int TYPE, int MT>
__global__ void __launch_bounds__(kThreads) gemv_kernel(const __grid_constant__ GemvParams p) {
    extern __shared__ __align__(128) uint8_t smem[];
    ActUnit *act = reinterpret_cast<ActUnit *>(smem + p.off_act);
    float *terms = reinterpret_cast<float *>(smem + p.off_terms);
    uint8_t *stages = smem + p.off_stages;
    uint64_t *bars = reinterpret_cast<uint64_t *>(smem + p.off_bars);  // full[NS], empty[NS], dead
    volatile int *flags = reinterpret_cast<volatile int *>(bars + 2 * kMaxStages + 1);  // [0] error, [1] issued

    __shared__ unsigned long long s_best[8];
    const int tid = threadIdx.x;
    const int warp = tid >> 5, lane = tid & 31;
    const int NS = p.n_stages;
    if (tid < 8) s_best[tid] = 0ull;

    // balanced contiguous row range of this CTA
    const long long tot = p.total_rows;
    const int g_begin = (int)(tot * blockIdx.x / gridDim.x);
    const int g_end = (int)(tot * (blockIdx.x + 1) / gridDim.x);

    if (tid == 0) {
        for (int s = 0; s < NS; ++s) {
            mbar_init(smem_u32(&bars[s]), 1);
            mbar_init(smem_u32(&bars[kMaxStages + s]), 1);
        }
        mbar_init(smem_u32(&bars[2 * kMaxStages]), 1);  // never arrived at (failure-path test)
        flags[0] = 0;
        flags[1] = 0;
        mbar_init_fence();
    }
    __syncthreads();
    pdl_launch_dependents();

    int consumed = 0;
    if (warp == kConsumerWarps) {
        // ---------------- producer: weights do not depend on earlier kernels, start at once
        if (lane == 0) {
            const uint64_t policy = l2_evict_first_policy();
            StageCursor cur{g_begin, g_end, 0};
            int t, r0, R, s = 0;
            while (next_stage(p, cur, t, r0, R)) {
                const int slot = s % NS;
                if (s >= NS) {
                    if (!mbar_wait_bounded(smem_u32(&bars[kMaxStages + slot]), ((s / NS) - 1) & 1, p.timeout_ns,
                                           p.status))
                        break;
                }
                const uint32_t bytes = (uint32_t)R * p.row_bytes;
                const uint32_t full = smem_u32(&bars[slot]);
                const uint32_t sdst = smem_u32(stages + (size_t)slot * p.stage_bytes);
                mbar_arrive_expect_tx(full, bytes);
                if (p.task[t].row_ids) {
                    for (int i = 0; i < R; ++i)
                        bulk_g2s(sdst + i * p.row_bytes, p.task[t].w + (size_t)p.task[t].row_ids[r0 + i] * p.row_bytes,
                                 p.row_bytes, full, policy);
                } else {
                    bulk_g2s(sdst, p.task[t].w + (size_t)r0 * p.row_bytes, bytes, full, policy);
                }
                ++s;
            }
            flags[1] = s;
        }
    } else {
        // ---------------- consumers
        pdl_wait();  // activations / residuals may come from the previous kernel
        const int ctid = tid;
        // stage the activation: one warp per (token, unit)
        const int n_units = p.M * p.nbu;
        for (int u = warp; u < n_units; u += kConsumerWarps) {
            const int m = u / p.nbu, b = u % p.nbu;
            ActUnit *a = act + u;
            if (p.x) {
                const __half *xu = p.x + (size_t)m * p.x_stride + (size_t)b * 256;
                const bool vec_ok = ((reinterpret_cast<uintptr_t>(xu) & 15) == 0);
                stage_act_from_fp16<TYPE>(xu, vec_ok, a, lane);
            } else if (TYPE == TYPE_Q8_0) {
                stage_act_from_q80(reinterpret_cast<const BlockQ80 *>(p.act) + (size_t)m * (p.K / 32) + 8 * b, a, lane);
            } else {
                stage_act_from_q8k(reinterpret_cast<const BlockQ8K *>(p.act) + (size_t)m * p.nbu + b, a, lane);
            }
        }
        if (p.inject_wait && ctid == 0) {
            // failure-path test: a wait whose barrier nothing completes must end by its time limit
            flags[0] = mbar_wait_bounded(smem_u32(&bars[2 * kMaxStages]), 0, p.timeout_ns, p.status) ? 0 : 1;
        }
        named_bar_sync(1, kConsumers);
        const bool injected_failure = p.inject_wait && flags[0];

        constexpr int T = (TYPE == TYPE_Q8_0) ? 8 : 1;
        const int tpr = p.terms_per_row;  // nbu * T
        StageCursor cur{g_begin, g_end, 0};
        int t, r0, R;
        while (!injected_failure && next_stage(p, cur, t, r0, R)) {
            const int slot = consumed % NS;
            if (ctid == 0) {
                const bool ok = mbar_wait_bounded(smem_u32(&bars[slot]), (consumed / NS) & 1, p.timeout_ns, p.status);
                flags[0] = ok ? 0 : 1;
            }
            named_bar_sync(1, kConsumers);
            if (flags[0]) break;

            const GemvTaskDev &tk = p.task[t];
            const uint8_t *sbase = stages + (size_t)slot * p.stage_bytes;
            float *tb = terms + (size_t)(consumed & 1) * p.rows_per_stage * tpr * MT;
            const int units = R * p.nbu;
            for (int u = ctid; u < units; u += kConsumers) {
                const int row = u / p.nbu, b = u % p.nbu;
                const uint8_t *wrow = sbase + (size_t)row * p.row_bytes;
                float *term = tb + ((size_t)row * tpr + (size_t)b * T) * MT;
                int *dsi = nullptr, *dsm = nullptr;
                long long dstride = 0;
                if (tk.dbg_sumi) {
                    const long long bpr = (long long)p.nbu * T;
                    dstride = (long long)tk.rows * bpr;
                    dsi = tk.dbg_sumi + (long long)(r0 + row) * bpr + (long long)b * T;
                    dsm = tk.dbg_summ + (long long)(r0 + row) * bpr + (long long)b * T;
                }
                const ActUnit *au = act + b;
                if (TYPE == TYPE_Q4_K) {
                    unit_q4k<MT>(wrow + (size_t)b * 144, au, p.nbu, p.M, term, dsi, dsm, dstride);
                } else if (TYPE == TYPE_Q5_K) {
                    unit_q5k<MT>(wrow + (size_t)b * 176, au, p.nbu, p.M, term, dsi, dsm, dstride);
                } else if (TYPE == TYPE_Q6_K) {
                    const uint16_t dbits = *reinterpret_cast<const uint16_t *>(wrow + (size_t)p.nbu * 208 + 2 * b);
                    unit_q6k<MT>(wrow + (size_t)b * 208, half_bits_to_float(dbits), au, p.nbu, p.M, term, dsi, dsm,
                                 dstride);
                } else {
                    unit_q80<MT>(wrow + (size_t)b * 256, wrow + (size_t)p.K + (size_t)b * 16, au, p.nbu, p.M, term,
                                 dsi, dsm, dstride);
                }
            }
            named_bar_sync(1, kConsumers);
            if (ctid == 0) mbar_arrive(smem_u32(&bars[kMaxStages + slot]));  // stage buffer free again

            // in-order block sums (the reference's `acc += term` sequence) + epilogue
            for (int idx = ctid; idx < R * p.M; idx += kConsumers) {
                const int row = idx % R, m = idx / R;
                const float *tr = tb + (size_t)row * tpr * MT + m;
                float acc = 0.0f;
                for (int j = 0; j < tpr; ++j) acc = __fadd_rn(acc, tr[(size_t)j * MT]);
                const int r = r0 + row;
                const size_t col = tk.scatter ? (size_t)tk.row_ids[r] : (size_t)r;
                if (tk.dst_f32) tk.dst_f32[(size_t)m * tk.f32_stride + col] = acc;
                if (tk.dst) {
                    float v = acc;
                    if (tk.res) v = __fadd_rn(v, __half2float(tk.res[(size_t)m * tk.res_stride + col]));
                    tk.dst[(size_t)m * tk.dst_stride + col] = __float2half_rn(v);
                }
                if (p.argmax) {
                    const float cmp = p.argmax_f16 ? __half2float(__float2half_rn(acc)) : acc;
                    atomicMax(&s_best[m], argmax_key(cmp, (uint32_t)(tk.index_base + r)));
                }
            }
            ++consumed;
        }
        if (p.argmax) {
            named_bar_sync(1, kConsumers);
            if (ctid < p.M) atomicMax(&p.argmax[ctid], s_best[ctid]);
        }
    }
    __syncthreads();
    // drain: copies issued but not consumed (only after an error) must land before exit;
    // consumer thread 0 (tid 0) holds the consumed count
    if (tid == 0) {
        const int issued = flags[1];
        for (int s = consumed; s < issued; ++s) mbar_wait_bounded(smem_u32(&bars[s % NS]), (s / NS) & 1, p.timeout_ns, p.status);
    }
}

// ------------------------------------------------------------------ host launcher

namespace {

struct Plan {
    int rows_per_stage, n_stages, ctas_per_sm;
    unsigned stage_bytes, off_act, off_terms, off_stages, off_bars, smem;
};

unsigned align_up(unsigned v, unsigned a) { return (v + a - 1) / a * a; }

Plan make_plan(int type, int K, int M, int MT, size_t row_bytes) {
    const int nbu = K / 256;
    const int T = (type == TYPE_Q8_0) ? 8 : 1;
    const unsigned act_bytes = align_up((unsigned)(M * nbu * (int)sizeof(ActUnit)), 128);
    Plan best{};
    // Prefer two CTAs per SM (next kernel's CTAs can start while this one drains); fall back to
    // one CTA per SM with a deeper ring when the activation is large.
    for (int ctas = 2; ctas >= 1; --ctas) {
        const unsigned budget = (ctas == 2) ? 112 * 1024 : 220 * 1024;
        unsigned stage = (unsigned)std::max<size_t>(row_bytes, (ctas == 2) ? 24576 : 32768);
        int rps = (int)(stage / row_bytes);
        stage = (unsigned)(rps * row_bytes);
        for (int ns = (ctas == 2 ? 4 : 6); ns >= 2; --ns) {
            const unsigned terms = align_up((unsigned)(2 * rps * nbu * T * MT * 4), 128);
            const unsigned bars = (2 * kMaxStages + 1) * 8 + 16;
            const unsigned total = act_bytes + terms + ns * align_up(stage, 128) + bars;
            if (total <= budget) {
                best.rows_per_stage = rps;
                best.n_stages = ns;
                best.ctas_per_sm = ctas;
                best.stage_bytes = align_up(stage, 128);
                best.off_act = 0;
                best.off_terms = act_bytes;
                best.off_stages = act_bytes + terms;
                best.off_bars = best.off_stages + ns * best.stage_bytes;
                best.smem = best.off_bars + bars;
                return best;
            }
        }
    }
    best.smem = 0;  // does not fit
    return best;
}

template <int TYPE, int MT>
cudaError_t launch_t(const GemvLaunch &L, cudaStream_t stream) {
    const Plan pl = make_plan(TYPE, L.K, L.M, MT, L.row_bytes);
    if (pl.smem == 0) return cudaErrorInvalidConfiguration;
    GemvParams p{};
    int total = 0;
    for (int i = 0; i < L.n_tasks; ++i) {
        const GemvTaskHost &h = L.tasks[i];
        GemvTaskDev &d = p.task[i];
        d.w = h.w;
        d.rows = h.rows;
        d.row_start = total;
        d.dst = reinterpret_cast<__half *>(h.dst);
        d.dst_stride = h.dst_stride;
        d.res = reinterpret_cast<const __half *>(h.res);
        d.res_stride = h.res_stride;
        d.dst_f32 = h.dst_f32;
        d.f32_stride = h.f32_stride;
        d.dbg_sumi = h.dbg_sumi;
        d.dbg_summ = h.dbg_summ;
        d.row_ids = h.row_ids;
        d.scatter = h.scatter;
        d.index_base = h.index_base;
        total += h.rows;
    }
    if (total == 0) return cudaSuccess;
    p.n_tasks = L.n_tasks;
    p.total_rows = total;
    p.K = L.K;
    p.nbu = L.K / 256;
    p.M = L.M;
    p.row_bytes = (unsigned)L.row_bytes;
    p.rows_per_stage = pl.rows_per_stage;
    p.n_stages = pl.n_stages;
    p.stage_bytes = pl.stage_bytes;
    p.terms_per_row = p.nbu * ((TYPE == TYPE_Q8_0) ? 8 : 1);
    p.x = reinterpret_cast<const __half *>(L.x);
    p.x_stride = L.x_stride;
    p.act = L.act;
    p.status = L.status;
    p.timeout_ns = L.timeout_ns;
    p.argmax = L.argmax;
    p.argmax_f16 = L.argmax_f16;
    p.inject_wait = L.inject_wait;
    p.off_act = pl.off_act;
    p.off_terms = pl.off_terms;
    p.off_stages = pl.off_stages;
    p.off_bars = pl.off_bars;

    auto kern = gemv_kernel<TYPE, MT>;
    static std::mutex mu;
    static std::unordered_map<int, unsigned> configured;  // device -> smem size set
    int dev = 0;
    cudaGetDevice(&dev);
    {
        std::lock_guard<std::mutex> lk(mu);
        unsigned &have = configured[dev];
        if (have < pl.smem) {
            // plans stay below 221 KB of dynamic shared memory; 225 KB leaves room for the
            // kernel's static shared words within the 227 KB per-block limit
            cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, 225 * 1024);
            if (e != cudaSuccess) return e;
            have = 225 * 1024;
        }
    }
    const int grid = std::max(1, std::min(total, pl.ctas_per_sm * L.num_sms));
    cudaLaunchConfig_t cfg{};
    cfg.gridDim = dim3(grid);
    cfg.blockDim = dim3(kThreads);
    cfg.dynamicSmemBytes = pl.smem;
    cfg.stream = stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = L.pdl ? 1 : 0;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, kern, p);
}

template <int TYPE>
cudaError_t launch_type(const GemvLaunch &L, cudaStream_t stream) {
    if (L.M <= 1) return launch_t<TYPE, 1>(L, stream);
    if (L.M <= 2) return launch_t<TYPE, 2>(L, stream);
    if (L.M <= 4) return launch_t<TYPE, 4>(L, stream);
    return launch_t<TYPE, 8>(L, stream);
}

}  // namespace

cudaError_t launch_gemv(const GemvLaunch &L, cudaStream_t stream) {
    if (L.M < 1 || L.M > 8) return cudaErrorInvalidValue;
    switch (L.type) {
        case TYPE_Q4_K: return launch_type<TYPE_Q4_K>(L, stream);
        case TYPE_Q5_K: return launch_type<TYPE_Q5_K>(L, stream);
        case TYPE_Q6_K: return launch_type<TYPE_Q6_K>(L, stream);
        case TYPE_Q8_0: return launch_type<TYPE_Q8_0>(L, stream);
        default: return cudaErrorInvalidValue;
    }
}

}  // namespace kq
