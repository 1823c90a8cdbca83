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

constexpr int kMaxWarps = 12;                  // consumer warps per CTA (W <= 12)
constexpr int kMaxThreads = (kMaxWarps + 1) * 32;

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
    int rows_per_stage;   // P * rows_per_sub
    int rows_per_sub;
    int subs_per_stage;   // P
    int units_per_row;    // 256-value units (Q8_0: 32-value blocks)
    int n_warps;          // consumer warps W
    int n_stages;         // S
    unsigned int stage_bytes;
    const __half *x;
    long long x_stride;
    const void *act;
    int *status;
    unsigned long long timeout_ns;
    unsigned long long *argmax;  // [M] packed (ordered value, ~index) keys, or nullptr
    int argmax_f16;              // compare the fp16-rounded results (the dispatch's stored logits)
    int inject_wait;             // failure test: consumers first wait on a barrier nothing arrives at
    unsigned int off_act, off_stages, off_bars;
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
//
// A "unit" is 256 weight values of one row: one Q4_K/Q5_K/Q6_K super-block, or eight Q8_0
// blocks; one lane computes a whole unit for all tokens, chunk by chunk (weights read from the
// shared-memory stage once per chunk, tokens in the inner loop), keeping registers low.
// Integer sums are exact; every fp32 term is formed with the reference's operation order and
// written to term[j * MT + m] (j = 0 for K-quants, j = Q8_0 block for Q8_0).

// Q4_K (ENG:758-801): term = dx * (d * sumi - dmin * summ)  (ENG:11025).  High nibbles are
// used in place (x16) and the factor is divided out exactly at the end.
template <int MT>
__device__ __forceinline__ void unit_q4k(const uint8_t *blk, const ActUnit *a0, int nbu, int M, float *term,
                                         int *dsi, int *dsm, long long dstride) {
    const uint4 h = *reinterpret_cast<const uint4 *>(blk);
    const uint32_t sc03 = h.y & 0x3F3F3F3Fu;
    const uint32_t sc47 = (h.w & 0x0F0F0F0Fu) | ((h.y >> 2) & 0x30303030u);
    int s16[MT];
#pragma unroll
    for (int m = 0; m < MT; ++m) s16[m] = 0;
#pragma unroll
    for (int c = 0; c < 4; ++c) {
        const uint4 qa = reinterpret_cast<const uint4 *>(blk + 16)[2 * c];
        const uint4 qb = reinterpret_cast<const uint4 *>(blk + 16)[2 * c + 1];
        const uint32_t w[8] = {qa.x, qa.y, qa.z, qa.w, qb.x, qb.y, qb.z, qb.w};
        const uint32_t scw = (c < 2) ? sc03 : sc47;
        const int s_lo = (int)byte_of(scw, 2 * (c & 1)), s_hi = (int)byte_of(scw, 2 * (c & 1) + 1);
#pragma unroll
        for (int m = 0; m < MT; ++m) {
            if (m < M) {
                const uint4 *xv = reinterpret_cast<const uint4 *>(a0[(size_t)m * nbu].qs + 64 * c);
                const uint4 x0 = xv[0], x1 = xv[1], x2 = xv[2], x3 = xv[3];
                const uint32_t xl[8] = {x0.x, x0.y, x0.z, x0.w, x1.x, x1.y, x1.z, x1.w};
                const uint32_t xh[8] = {x2.x, x2.y, x2.z, x2.w, x3.x, x3.y, x3.z, x3.w};
                // four independent dp4a chains per chunk
                int dl0 = 0, dl1 = 0, dh0 = 0, dh1 = 0;
#pragma unroll
                for (int i = 0; i < 8; i += 2) {
                    dl0 = dp4a_us(w[i] & 0x0F0F0F0Fu, (int)xl[i], dl0);
                    dl1 = dp4a_us(w[i + 1] & 0x0F0F0F0Fu, (int)xl[i + 1], dl1);
                    dh0 = dp4a_us(w[i] & 0xF0F0F0F0u, (int)xh[i], dh0);  // 16 x the high-nibble dot
                    dh1 = dp4a_us(w[i + 1] & 0xF0F0F0F0u, (int)xh[i + 1], dh1);
                }
                s16[m] += s_lo * ((dl0 + dl1) << 4) + s_hi * (dh0 + dh1);
            }
        }
    }
    const float d = half_bits_to_float(h.x), dmin = half_bits_to_float(h.x >> 16);
    const uint32_t mn03 = h.z & 0x3F3F3F3Fu;
    const uint32_t mn47 = ((h.w >> 4) & 0x0F0F0F0Fu) | ((h.z >> 2) & 0x30303030u);
#pragma unroll
    for (int m = 0; m < MT; ++m) {
        if (m < M) {
            const ActUnit *a = a0 + (size_t)m * nbu;
            const int sumi = s16[m] >> 4;
            const int4 b0 = *reinterpret_cast<const int4 *>(a->aux);
            const int4 b1 = *reinterpret_cast<const int4 *>(a->aux + 4);
            const int summ = (int)byte_of(mn03, 0) * b0.x + (int)byte_of(mn03, 1) * b0.y +
                             (int)byte_of(mn03, 2) * b0.z + (int)byte_of(mn03, 3) * b0.w +
                             (int)byte_of(mn47, 0) * b1.x + (int)byte_of(mn47, 1) * b1.y +
                             (int)byte_of(mn47, 2) * b1.z + (int)byte_of(mn47, 3) * b1.w;
            const float t = __fsub_rn(__fmul_rn(d, __int2float_rn(sumi)), __fmul_rn(dmin, __int2float_rn(summ)));
            term[m] = __fmul_rn(a->d, t);
            if (dsi) {
                dsi[m * dstride] = sumi;
                dsm[m * dstride] = summ;
            }
        }
    }
}

// Q5_K (ENG:803-853): as Q4_K with the fifth bit of value l of chunk c in bit 2c (low half) /
// 2c+1 (high half) of qh[l]  (ENG:11028-11062).
template <int MT>
__device__ __forceinline__ void unit_q5k(const uint8_t *blk, const ActUnit *a0, int nbu, int M, float *term,
                                         int *dsi, int *dsm, long long dstride) {
    const uint4 h = *reinterpret_cast<const uint4 *>(blk);
    const uint4 qh0 = reinterpret_cast<const uint4 *>(blk + 16)[0];
    const uint4 qh1 = reinterpret_cast<const uint4 *>(blk + 16)[1];
    const uint32_t hb[8] = {qh0.x, qh0.y, qh0.z, qh0.w, qh1.x, qh1.y, qh1.z, qh1.w};
    const uint32_t sc03 = h.y & 0x3F3F3F3Fu;
    const uint32_t sc47 = (h.w & 0x0F0F0F0Fu) | ((h.y >> 2) & 0x30303030u);
    int s16[MT];
#pragma unroll
    for (int m = 0; m < MT; ++m) s16[m] = 0;
#pragma unroll
    for (int c = 0; c < 4; ++c) {
        const uint4 qa = reinterpret_cast<const uint4 *>(blk + 48)[2 * c];
        const uint4 qb = reinterpret_cast<const uint4 *>(blk + 48)[2 * c + 1];
        const uint32_t w[8] = {qa.x, qa.y, qa.z, qa.w, qb.x, qb.y, qb.z, qb.w};
        uint32_t wl[8], wh[8];
#pragma unroll
        for (int i = 0; i < 8; ++i) {
            wl[i] = (w[i] & 0x0F0F0F0Fu) | (((hb[i] >> (2 * c)) & 0x01010101u) << 4);
            wh[i] = ((w[i] >> 4) & 0x0F0F0F0Fu) | (((hb[i] >> (2 * c + 1)) & 0x01010101u) << 4);
        }
        const uint32_t scw = (c < 2) ? sc03 : sc47;
        const int s_lo = (int)byte_of(scw, 2 * (c & 1)), s_hi = (int)byte_of(scw, 2 * (c & 1) + 1);
#pragma unroll
        for (int m = 0; m < MT; ++m) {
            if (m < M) {
                const uint4 *xv = reinterpret_cast<const uint4 *>(a0[(size_t)m * nbu].qs + 64 * c);
                const uint4 x0 = xv[0], x1 = xv[1], x2 = xv[2], x3 = xv[3];
                const uint32_t xl[8] = {x0.x, x0.y, x0.z, x0.w, x1.x, x1.y, x1.z, x1.w};
                const uint32_t xh[8] = {x2.x, x2.y, x2.z, x2.w, x3.x, x3.y, x3.z, x3.w};
                int dl = 0, dh = 0;
#pragma unroll
                for (int i = 0; i < 8; ++i) {
                    dl = dp4a_us(wl[i], (int)xl[i], dl);
                    dh = dp4a_us(wh[i], (int)xh[i], dh);
                }
                s16[m] += (s_lo * dl + s_hi * dh) << 4;
            }
        }
    }
    const float d = half_bits_to_float(h.x), dmin = half_bits_to_float(h.x >> 16);
    const uint32_t mn03 = h.z & 0x3F3F3F3Fu;
    const uint32_t mn47 = ((h.w >> 4) & 0x0F0F0F0Fu) | ((h.z >> 2) & 0x30303030u);
#pragma unroll
    for (int m = 0; m < MT; ++m) {
        if (m < M) {
            const ActUnit *a = a0 + (size_t)m * nbu;
            const int sumi = s16[m] >> 4;
            const int4 b0 = *reinterpret_cast<const int4 *>(a->aux);
            const int4 b1 = *reinterpret_cast<const int4 *>(a->aux + 4);
            const int summ = (int)byte_of(mn03, 0) * b0.x + (int)byte_of(mn03, 1) * b0.y +
                             (int)byte_of(mn03, 2) * b0.z + (int)byte_of(mn03, 3) * b0.w +
                             (int)byte_of(mn47, 0) * b1.x + (int)byte_of(mn47, 1) * b1.y +
                             (int)byte_of(mn47, 2) * b1.z + (int)byte_of(mn47, 3) * b1.w;
            const float t = __fsub_rn(__fmul_rn(d, __int2float_rn(sumi)), __fmul_rn(dmin, __int2float_rn(summ)));
            term[m] = __fmul_rn(a->d, t);
            if (dsi) {
                dsi[m * dstride] = sumi;
                dsm[m * dstride] = summ;
            }
        }
    }
}

// Q6_K, device block [ql 128][qh 64][scales 16] + d from the row's d plane (ENG:673-741).
// Value e = 128h + 32g + l: low 4 bits in ql[64h + l + 32(g&1)] (>> 4 when g >= 2), bits 4-5 in
// qh[32h + l] >> 2g, minus 32; sub-block s = 8h + 2g + (l >= 16) (ENG:11065-11101).
// sum (q - 32) x = sum q x - 32 * (sum of the 16 activation quants, ActUnit.xsum16).
// term = (d * dx) * sumi  (ENG:11100).  Processed per (h, 16-value half): 16 sub-block dots.
template <int MT>
__device__ __forceinline__ void unit_q6k(const uint8_t *blk, float d, const ActUnit *a0, int nbu, int M, float *term,
                                         int *dsi, int *dsm, long long dstride) {
    const uint4 scv = reinterpret_cast<const uint4 *>(blk + 192)[0];
    const uint32_t scw[4] = {scv.x, scv.y, scv.z, scv.w};
    int sumi[MT];
#pragma unroll
    for (int m = 0; m < MT; ++m) sumi[m] = 0;
#pragma unroll
    for (int hh = 0; hh < 2; ++hh) {
#pragma unroll
        for (int half16 = 0; half16 < 2; ++half16) {
            // 16 values l in [16 half16, 16 half16 + 16) of the four groups g of half hh
            const uint4 b0 = *reinterpret_cast<const uint4 *>(blk + 64 * hh + 16 * half16);
            const uint4 b1 = *reinterpret_cast<const uint4 *>(blk + 64 * hh + 32 + 16 * half16);
            const uint4 hv = *reinterpret_cast<const uint4 *>(blk + 128 + 32 * hh + 16 * half16);
            const uint32_t B0[4] = {b0.x, b0.y, b0.z, b0.w}, B1[4] = {b1.x, b1.y, b1.z, b1.w};
            const uint32_t HB[4] = {hv.x, hv.y, hv.z, hv.w};
            uint32_t q[4][4];
#pragma unroll
            for (int k = 0; k < 4; ++k) {
                q[0][k] = (B0[k] & 0x0F0F0F0Fu) | ((HB[k] << 4) & 0x30303030u);
                q[1][k] = (B1[k] & 0x0F0F0F0Fu) | ((HB[k] << 2) & 0x30303030u);
                q[2][k] = ((B0[k] >> 4) & 0x0F0F0F0Fu) | (HB[k] & 0x30303030u);
                q[3][k] = ((B1[k] >> 4) & 0x0F0F0F0Fu) | ((HB[k] >> 2) & 0x30303030u);
            }
            int sc[4];
#pragma unroll
            for (int g = 0; g < 4; ++g) {
                const int sidx = 8 * hh + 2 * g + half16;
                sc[g] = (int)(int8_t)byte_of(scw[sidx >> 2], sidx & 3);
            }
#pragma unroll
            for (int m = 0; m < MT; ++m) {
                if (m < M) {
                    const ActUnit *a = a0 + (size_t)m * nbu;
                    const uint4 *xv = reinterpret_cast<const uint4 *>(a->qs);
                    int acc = 0;
#pragma unroll
                    for (int g = 0; g < 4; ++g) {
                        const uint4 x = xv[8 * hh + 2 * g + half16];
                        int dot = dp4a_us(q[g][0], (int)x.x, 0);
                        dot = dp4a_us(q[g][1], (int)x.y, dot);
                        dot = dp4a_us(q[g][2], (int)x.z, dot);
                        dot = dp4a_us(q[g][3], (int)x.w, dot);
                        acc += sc[g] * (dot - 32 * a->xsum16[8 * hh + 2 * g + half16]);
                    }
                    sumi[m] += acc;
                }
            }
        }
    }
#pragma unroll
    for (int m = 0; m < MT; ++m) {
        if (m < M) {
            const ActUnit *a = a0 + (size_t)m * nbu;
            term[m] = __fmul_rn(__fmul_rn(d, a->d), __int2float_rn(sumi[m]));
            if (dsi) {
                dsi[m * dstride] = sumi[m];
                dsm[m * dstride] = 0;
            }
        }
    }
}

// One Q8_0 block of 32 values (device: int8 quants at 32 * j, fp16 scale in the row's d plane).
// term = (d * dx) * dot  (sdot_row_q8_0_batch, ENG:3393-3407).  The activation block is
// sub-block j & 7 of ActUnit j >> 3.
template <int MT>
__device__ __forceinline__ void unit_q80(const uint8_t *qs, const uint8_t *dptr, int j, const ActUnit *act, int nbu,
                                         int M, float *term, int *dsi, int *dsm, long long dstride) {
    const uint4 wa = reinterpret_cast<const uint4 *>(qs)[0];
    const uint4 wb = reinterpret_cast<const uint4 *>(qs)[1];
    const float dw = half_bits_to_float(*reinterpret_cast<const uint16_t *>(dptr));
    const int au = j >> 3, sub = j & 7;
#pragma unroll
    for (int m = 0; m < MT; ++m) {
        if (m < M) {
            const ActUnit *a = act + (size_t)m * nbu + au;
            const uint4 xa = reinterpret_cast<const uint4 *>(a->qs)[2 * sub];
            const uint4 xb = reinterpret_cast<const uint4 *>(a->qs)[2 * sub + 1];
            int dot = dp4a_ss((int)wa.x, (int)xa.x, 0);
            dot = dp4a_ss((int)wa.y, (int)xa.y, dot);
            dot = dp4a_ss((int)wa.z, (int)xa.z, dot);
            dot = dp4a_ss((int)wa.w, (int)xa.w, dot);
            dot = dp4a_ss((int)wb.x, (int)xb.x, dot);
            dot = dp4a_ss((int)wb.y, (int)xb.y, dot);
            dot = dp4a_ss((int)wb.z, (int)xb.z, dot);
            dot = dp4a_ss((int)wb.w, (int)xb.w, dot);
            term[m] = __fmul_rn(__fmul_rn(dw, __int_as_float(a->aux[sub])), __int2float_rn(dot));
            if (dsi) {
                dsi[m * dstride] = dot;
                dsm[m * dstride] = 0;
            }
        }
    }
}

// ------------------------------------------------------------------ row -> task

// Index of the task owning concatenated row g (tasks are in ascending row_start order).
__device__ __forceinline__ int task_of(const GemvParams &p, int g) {
    int t = 0;
#pragma unroll
    for (int i = 1; i < 4; ++i) t += (i < p.n_tasks && g >= p.task[i].row_start) ? 1 : 0;
    return t;
}

// ------------------------------------------------------------------ the kernel
//
// Each CTA owns a contiguous range [g_begin, g_end) of the dispatch's concatenated output rows
// and walks it in stages of rows_per_stage rows; stage s starts at g_begin + s * rows_per_stage.
// The producer warp (index W) streams stages into an S-slot ring: one cp.async.bulk per task
// segment of the stage (>= 16 KB per stage in total; one copy per row for gathered rows).  A
// stage holds P sub-stages of rows_per_sub rows (rows_per_sub * units-per-row <= 32, or one
// row) and sub-stage q = s * P + part belongs to consumer warp q % W.  The warp waits on the
// stage's full barrier, computes one unit per lane (a row longer than 32 units in passes), adds
// each row's unit terms in unit order through shuffles into the row's leader lane (the
// reference's `acc += term` sequence), arrives on the stage's empty barrier (P arrivals free the
// slot) and writes the epilogue.  There is no CTA-wide barrier in the main loop.
// (P * S) % W == 0: the previous use of the slot of a warp's next sub-stage was one of the
// warp's own sub-stages, which it already waited for, so a waiter never runs two phases ahead
// of a full barrier (where the parity test of mbarrier.try_wait.parity would pass on the wrong
// phase).

template <int TYPE, int MT>
__global__ void __launch_bounds__(kMaxThreads, 2) gemv_kernel(const __grid_constant__ GemvParams p) {
    extern __shared__ __align__(128) uint8_t smem[];
    __shared__ unsigned long long s_best[8];
    __shared__ int s_abort, s_issued;

    ActUnit *act = reinterpret_cast<ActUnit *>(smem + p.off_act);
    uint8_t *ring = smem + p.off_stages;
    uint64_t *bars = reinterpret_cast<uint64_t *>(smem + p.off_bars);  // full[S], empty[S], dead
    const int S = p.n_stages, W = p.n_warps, P = p.subs_per_stage, RS = p.rows_per_sub;
    const int RPS = p.rows_per_stage;
    const int tid = threadIdx.x;
    const int warp = tid >> 5, lane = tid & 31;

    const long long tot = p.total_rows;
    const int g_begin = (int)(tot * blockIdx.x / gridDim.x);
    const int g_end = (int)(tot * (blockIdx.x + 1) / gridDim.x);
    const int n_stages_cta = (g_end - g_begin + RPS - 1) / RPS;

    if (tid < 8) s_best[tid] = 0ull;
    if (tid == 0) {
        for (int s = 0; s < S; ++s) {
            mbar_init(smem_u32(&bars[s]), 1);
            mbar_init(smem_u32(&bars[S + s]), P);
        }
        mbar_init(smem_u32(&bars[2 * S]), 1);  // never arrived at (failure-path test)
        s_abort = 0;
        s_issued = 0;
        mbar_init_fence();
    }
    __syncthreads();
    pdl_launch_dependents();

    if (warp == W) {
        // ---------------- producer: the weight stream does not depend on earlier kernels
        if (lane == 0) {
            const uint64_t policy = l2_evict_first_policy();
            int s = 0;
            for (; s < n_stages_cta; ++s) {
                const int slot = s % S;
                if (s >= S) {
                    if (!mbar_wait_bounded(smem_u32(&bars[S + slot]), ((s / S) - 1) & 1, p.timeout_ns, p.status)) {
                        s_abort = 1;
                        break;
                    }
                }
                const int a = g_begin + s * RPS, b = min(g_end, a + RPS);
                const uint32_t full = smem_u32(&bars[slot]);
                const uint32_t sdst = smem_u32(ring + (size_t)slot * p.stage_bytes);
                mbar_arrive_expect_tx(full, (uint32_t)(b - a) * p.row_bytes);
                int g = a;
                while (g < b) {
                    const int t = task_of(p, g);
                    const int tend = min(b, p.task[t].row_start + p.task[t].rows);
                    const int r0 = g - p.task[t].row_start;
                    const uint32_t off = (uint32_t)(g - a) * p.row_bytes;
                    if (p.task[t].row_ids) {
                        for (int i = 0; i < tend - g; ++i)
                            bulk_g2s(sdst + off + i * p.row_bytes,
                                     p.task[t].w + (size_t)p.task[t].row_ids[r0 + i] * p.row_bytes, p.row_bytes, full,
                                     policy);
                    } else {
                        bulk_g2s(sdst + off, p.task[t].w + (size_t)r0 * p.row_bytes, (uint32_t)(tend - g) * p.row_bytes,
                                 full, policy);
                    }
                    g = tend;
                }
                s_issued = s + 1;
            }
        }
    } else {
        // ---------------- consumers
        pdl_wait();  // activations / residuals may come from the previous kernel
        const int nbu = p.nbu;
        const int n_units = p.M * nbu;
        for (int u = warp; u < n_units; u += W) {
            const int m = u / nbu, b = u % nbu;
            ActUnit *a = act + u;
            if (p.x) {
                const __half *xu = p.x + (size_t)m * p.x_stride + (size_t)b * 256;
                stage_act_from_fp16<TYPE>(xu, (reinterpret_cast<uintptr_t>(xu) & 15) == 0, a, lane);
            } else if (TYPE == TYPE_Q8_0) {
                stage_act_from_q80(reinterpret_cast<const BlockQ80 *>(p.act) + (size_t)m * (p.K / 32) + 8 * b, a, lane);
            } else {
                stage_act_from_q8k(reinterpret_cast<const BlockQ8K *>(p.act) + (size_t)m * nbu + b, a, lane);
            }
        }
        if (p.inject_wait && tid == 0) {
            // failure-path test: a wait whose barrier nothing completes must end by its time limit
            if (!mbar_wait_bounded(smem_u32(&bars[2 * S]), 0, p.timeout_ns, p.status)) s_abort = 1;
        }
        named_bar_sync(1, W * 32);

        const int upr = p.units_per_row;  // 256-value units (32-value blocks for Q8_0)
        const int multi = (RS > 1);       // several whole rows per sub-stage
        const int npass = multi ? 1 : (upr + 31) / 32;
        const int lrow = multi ? lane / upr : 0;
        const int lead = multi ? lrow * upr : 0;  // leader lane of this lane's row
        const int n_sub = n_stages_cta * P;
        // sub-stage q = sidx * P + part lives in ring slot sidx % S, phase (sidx / S) & 1; the
        // counters advance by W sub-stages per iteration without integer division
        int sidx = warp / P, part = warp - (warp / P) * P;
        int slot = sidx % S, phase = (sidx / S) & 1;
        int a = g_begin + sidx * RPS;  // first row of the stage
        for (int q = warp; q < n_sub; q += W) {
            if (*reinterpret_cast<volatile int *>(&s_abort)) break;
            int ok = 1;
            if (lane == 0) ok = mbar_wait_bounded(smem_u32(&bars[slot]), phase, p.timeout_ns, p.status) ? 1 : 0;
            ok = __shfl_sync(0xffffffffu, ok, 0);
            if (!ok) {
                if (lane == 0) s_abort = 1;
                break;
            }
            const int sR = max(0, min(RS, min(g_end, a + RPS) - (a + part * RS)));  // rows of this sub-stage
            const int g = a + part * RS + min(lrow, max(sR - 1, 0));  // this lane's row (concatenated)
            const int t = task_of(p, g);
            const GemvTaskDev &tk = p.task[t];
            const int r = g - tk.row_start;                      // row within the task
            const uint8_t *wrow = ring + (size_t)slot * p.stage_bytes + (size_t)(g - a) * p.row_bytes;
            const int units = sR * upr;
            const bool is_lead = multi ? (lane == lead && lane < units) : (lane == 0 && sR > 0);
            float acc[MT];
#pragma unroll
            for (int m = 0; m < MT; ++m) acc[m] = 0.0f;
            for (int pass = 0; pass < npass; ++pass) {
                const int b = multi ? lane - lead : 32 * pass + lane;
                const bool valid = multi ? (lane < units) : (sR > 0 && b < upr);
                const int cnt = multi ? upr : min(32, upr - 32 * pass);  // the row's units in this pass
                float term[MT];
#pragma unroll
                for (int m = 0; m < MT; ++m) term[m] = 0.0f;
                if (valid) {
                    int *dsi = nullptr, *dsm = nullptr;
                    long long dstride = 0;
                    if (tk.dbg_sumi) {
                        dstride = (long long)tk.rows * upr;
                        const long long off = (long long)r * upr + b;
                        dsi = tk.dbg_sumi + off;
                        dsm = tk.dbg_summ + off;
                    }
                    if (TYPE == TYPE_Q4_K) {
                        unit_q4k<MT>(wrow + 144 * b, act + b, nbu, p.M, term, dsi, dsm, dstride);
                    } else if (TYPE == TYPE_Q5_K) {
                        unit_q5k<MT>(wrow + 176 * b, act + b, nbu, p.M, term, dsi, dsm, dstride);
                    } else if (TYPE == TYPE_Q6_K) {
                        const float dq = half_bits_to_float(*reinterpret_cast<const uint16_t *>(wrow + 208 * nbu + 2 * b));
                        unit_q6k<MT>(wrow + 208 * b, dq, act + b, nbu, p.M, term, dsi, dsm, dstride);
                    } else {
                        unit_q80<MT>(wrow + 32 * b, wrow + p.K + 2 * b, b, act, nbu, p.M, term, dsi, dsm, dstride);
                    }
                }
                // in-order sum of the row's unit terms into the leader (the reference's `acc += term`)
#pragma unroll 4
                for (int i = 0; i < cnt; ++i) {
                    const int src = min(lead + i, 31);
#pragma unroll
                    for (int m = 0; m < MT; ++m) acc[m] = __fadd_rn(acc[m], __shfl_sync(0xffffffffu, term[m], src));
                }
            }
            __syncwarp();
            if (lane == 0) mbar_arrive(smem_u32(&bars[S + slot]));  // P arrivals free the slot
            if (is_lead) {
                const size_t col = tk.scatter ? (size_t)tk.row_ids[r] : (size_t)r;
#pragma unroll
                for (int m = 0; m < MT; ++m) {
                    if (m < p.M) {
                        if (tk.dst_f32) tk.dst_f32[(size_t)m * tk.f32_stride + col] = acc[m];
                        if (tk.dst) {
                            float v = acc[m];
                            if (tk.res) v = __fadd_rn(v, __half2float(tk.res[(size_t)m * tk.res_stride + col]));
                            tk.dst[(size_t)m * tk.dst_stride + col] = __float2half_rn(v);
                        }
                        if (p.argmax) {
                            const float cmp = p.argmax_f16 ? __half2float(__float2half_rn(acc[m])) : acc[m];
                            atomicMax(&s_best[m], argmax_key(cmp, (uint32_t)(tk.index_base + r)));
                        }
                    }
                }
            }
            part += W;
            while (part >= P) {
                part -= P;
                ++sidx;
                a += RPS;
                if (++slot == S) {
                    slot = 0;
                    phase ^= 1;
                }
            }
        }
    }
    __syncthreads();
    if (p.argmax && tid < p.M && !s_abort) atomicMax(&p.argmax[tid], s_best[tid]);
    // drain: a slot's most recent copy must land before the CTA exits (matters only after an
    // early stop); consumers never arrive on full barriers, so the last S issued stages are
    // exactly the outstanding candidates
    if (tid == 0) {
        const int issued = s_issued;
        for (int s = max(0, issued - S); s < issued; ++s)
            mbar_wait_bounded(smem_u32(&bars[s % S]), (s / S) & 1, p.timeout_ns, p.status);
    }
}

// ------------------------------------------------------------------ host launcher

namespace {

struct Plan {
    int rows_per_sub, subs, n_stages, n_warps, grid;
    unsigned stage_bytes, off_act, off_stages, off_bars, smem;
};

unsigned align_up(unsigned v, unsigned a) { return (v + a - 1) / a * a; }

// Geometry of one launch.
//  * Sub-stage = the rows one consumer warp handles at once: floor(32 / units-per-row) whole
//    rows (one unit per lane), or one row.  Stage = P sub-stages, P * sub_bytes >= 16 KB
//    (smaller bulk copies do not reach full HBM bandwidth).
//  * Prefetch mode: when a CTA's whole share of rows fits in ~110 KB, one CTA per SM with a
//    ring that holds all of it.  Its smem, registers and threads stay under half an SM, so the
//    next kernel's CTA (programmatic dependent launch) is resident meanwhile and streams its
//    own weights while this one computes; back-to-back small GEMVs then overlap their HBM
//    traffic.
//  * Throughput mode (larger matrices): two CTAs per SM, ring within ~100 KB each.
//  * W consumer warps with (P * S) % W == 0, which keeps every full-barrier wait within one
//    phase (see the kernel).
Plan make_plan(int type, int K, int M, size_t row_bytes, int total_rows, int num_sms) {
    Plan pl{};
    const int nbu = K / 256;
    const int upr = (type == TYPE_Q8_0) ? K / 32 : nbu;
    const int rsub = upr <= 16 ? 32 / upr : 1;
    const size_t sub_bytes = (size_t)rsub * row_bytes;
    const unsigned act = align_up((unsigned)(M * nbu * (int)sizeof(ActUnit)), 128);
    int pmin = 1;
    while ((size_t)pmin * sub_bytes < 16 * 1024 && pmin < 16) ++pmin;
    auto smem_of = [&](int P, int S) {
        return act + S * align_up((unsigned)(P * sub_bytes), 128) + (2 * S + 1) * 8 + 256;
    };
    auto fill = [&](int P, int S, int W, int ctas_per_sm) {
        const unsigned stage = align_up((unsigned)(P * sub_bytes), 128);
        const int rps = P * rsub;
        pl.rows_per_sub = rsub;
        pl.subs = P;
        pl.n_stages = S;
        pl.n_warps = W;
        pl.stage_bytes = stage;
        pl.off_act = 0;
        pl.off_stages = act;
        pl.off_bars = act + S * stage;
        pl.smem = pl.off_bars + (2 * S + 1) * 8;
        pl.grid = std::max(1, std::min(ctas_per_sm * num_sms, (total_rows + rps - 1) / rps));
    };
    // candidates: P in [pmin, pmin + 4], W in [6, 12]; prefer more warps, then more bytes in flight
    int bP = 0, bS = 0, bW = 0, bctas = 0;
    size_t bflight = 0;
    auto consider = [&](int P, int S, int W, int ctas) {
        const size_t flight = (size_t)S * align_up((unsigned)(P * sub_bytes), 128);
        if (W > bW || (W == bW && flight > bflight)) {
            bP = P, bS = S, bW = W, bctas = ctas, bflight = flight;
        }
    };
    // prefetch mode: the ring holds the CTA's whole share
    for (int P = pmin; P <= pmin + 4; ++P) {
        const int rps = P * rsub;
        const int share_stages = ((total_rows + num_sms - 1) / num_sms + rps - 1) / rps;
        for (int W = 12; W >= 6; --W)
            for (int S = std::max(2, share_stages); S <= share_stages + W; ++S) {
                if ((P * S) % W) continue;
                if (smem_of(P, S) <= 110 * 1024) consider(P, S, W, 1);
                break;
            }
    }
    if (bW) {
        fill(bP, bS, bW, bctas);
        return pl;
    }
    // throughput mode: two CTAs per SM within ~100 KB each, else one CTA with up to 220 KB
    for (unsigned budget : {100u * 1024u, 220u * 1024u}) {
        for (int P = pmin; P <= pmin + 4; ++P)
            for (int W = 12; W >= 6; --W) {
                int best = 0;
                for (int S = 2; S <= 32; ++S) {
                    if ((P * S) % W) continue;
                    if (smem_of(P, S) > budget) break;
                    best = S;
                }
                if (best) consider(P, best, W, budget <= 100 * 1024 ? 2 : 1);
            }
        if (bW) {
            fill(bP, bS, bW, bctas);
            return pl;
        }
    }
    return pl;  // smem 0: does not fit
}

template <int TYPE, int MT>
cudaError_t launch_t(const GemvLaunch &L, cudaStream_t stream) {
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
    const Plan pl = make_plan(TYPE, L.K, L.M, L.row_bytes, total, L.num_sms);
    if (pl.smem == 0) return cudaErrorInvalidConfiguration;
    p.n_tasks = L.n_tasks;
    p.total_rows = total;
    p.K = L.K;
    p.nbu = L.K / 256;
    p.M = L.M;
    p.row_bytes = (unsigned)L.row_bytes;
    p.rows_per_stage = pl.subs * pl.rows_per_sub;
    p.rows_per_sub = pl.rows_per_sub;
    p.subs_per_stage = pl.subs;
    p.units_per_row = (TYPE == TYPE_Q8_0) ? L.K / 32 : L.K / 256;
    p.n_warps = pl.n_warps;
    p.n_stages = pl.n_stages;
    p.stage_bytes = pl.stage_bytes;
    p.x = reinterpret_cast<const __half *>(L.x);
    p.x_stride = L.x_stride;
    p.act = L.act;
    p.status = L.status;
    p.timeout_ns = L.timeout_ns;
    p.argmax = L.argmax;
    p.argmax_f16 = L.argmax_f16;
    p.inject_wait = L.inject_wait;
    p.off_act = pl.off_act;
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
    const int grid = pl.grid;
    cudaLaunchConfig_t cfg{};
    cfg.gridDim = dim3(grid);
    cfg.blockDim = dim3((pl.n_warps + 1) * 32);
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
