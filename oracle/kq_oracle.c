/*
 * kq_oracle.c -- CPU restatement (test infrastructure) of the reference engine's K-quant
 * matmul path.  See kq_oracle.h for the contract; "ENG" = src/v182_r22_breakthrough_engine.c
 * of the reference.  Each function restates the reference's SCALAR path operation by
 * operation, so fp32 results are bit-identical to the reference built for x86-64
 * (no FMA contraction on either side).
 *
 * Only tests/, __graft_entry__.smoke() and bench.py's cpu_baseline leg use this file.
 */
#include "kq_oracle.h"

#include <math.h>
#include <stdlib.h>
#include <string.h>

uint64_t kqo_row_bytes(uint32_t type, uint64_t k) {
    /* ENG:364-374 */
    switch (type) {
        case KQO_TYPE_F32:  return k * 4u;
        case KQO_TYPE_F16:  return k * 2u;
        case KQO_TYPE_Q8_0: return (k / 32u) * 34u;
        case KQO_TYPE_Q4_K: return (k / 256u) * 144u;
        case KQO_TYPE_Q5_K: return (k / 256u) * 176u;
        case KQO_TYPE_Q6_K: return (k / 256u) * 210u;
        default:            return 0;
    }
}

/* binary16 <-> binary32 through the compiler's _Float16 (IEEE RNE), the x86 stand-in for
 * the reference's ARM __fp16 (same binary16 format). */
float kqo_f16_to_f32(uint16_t h) {
    _Float16 v;
    memcpy(&v, &h, 2);
    return (float)v;
}

uint16_t kqo_f32_to_f16(float f) {
    _Float16 v = (_Float16)f;
    uint16_t h;
    memcpy(&h, &v, 2);
    return h;
}

void kqo_f32_to_f16_array(const float *x, uint16_t *y, size_t n) {
    for (size_t i = 0; i < n; ++i) y[i] = kqo_f32_to_f16(x[i]);
}

static inline uint16_t ld_u16(const uint8_t *p) {
    uint16_t v;
    memcpy(&v, p, 2);
    return v;
}

void kqo_get_scale_min_k4(int j, const uint8_t *q, uint8_t *d, uint8_t *m) {
    /* ENG:743-749: sub-blocks 0..3 keep their 6 bits in bytes 0..7; sub-blocks 4..7 keep the
     * low 4 bits in bytes 8..11 and the top 2 bits in the spare high bits of bytes 0..7. */
    if (j < 4) {
        *d = (uint8_t)(q[j] & 63);
        *m = (uint8_t)(q[j + 4] & 63);
    } else {
        *d = (uint8_t)((q[j + 4] & 0x0F) | ((q[j - 4] >> 6) << 4));
        *m = (uint8_t)((q[j + 4] >> 4) | ((q[j] >> 6) << 4));
    }
}

void kqo_quantize_row_q8k(const uint16_t *x, kqo_block_q8k *y, int k) {
    /* ENG:925-990, scalar branches ENG:941-945 and ENG:976-988 */
    const int nb = k / 256;
    for (int b = 0; b < nb; ++b) {
        const uint16_t *xb = x + (size_t)b * 256;
        float amax = 0.0f;
        for (int i = 0; i < 256; ++i) {
            const float a = fabsf(kqo_f16_to_f32(xb[i]));
            if (a > amax) amax = a;
        }
        if (amax == 0.0f) {
            y[b].d = 0.0f;
            memset(y[b].qs, 0, sizeof y[b].qs);
            memset(y[b].bsum32, 0, sizeof y[b].bsum32);
            continue;
        }
        y[b].d = amax / 127.0f;
        const float inv = 127.0f / amax;
        for (int s = 0; s < 8; ++s) {
            int32_t acc = 0;
            for (int l = 0; l < 32; ++l) {
                long v = lrintf(kqo_f16_to_f32(xb[s * 32 + l]) * inv);
                if (v > 127) v = 127;
                if (v < -127) v = -127;
                y[b].qs[s * 32 + l] = (int8_t)v;
                acc += (int32_t)v;
            }
            y[b].bsum32[s] = acc;
        }
    }
}

void kqo_quantize_row_q8_0(const uint16_t *x, kqo_block_q8_0 *y, int k) {
    /* ENG:1016-1064, scalar branches ENG:1029-1034 and ENG:1055-1062 */
    const int nb = k / 32;
    for (int b = 0; b < nb; ++b) {
        const uint16_t *xb = x + (size_t)b * 32;
        float amax = 0.0f;
        for (int i = 0; i < 32; ++i) {
            const float a = fabsf(kqo_f16_to_f32(xb[i]));
            if (a > amax) amax = a;
        }
        if (amax == 0.0f) {
            y[b].d = 0.0f;
            memset(y[b].qs, 0, sizeof y[b].qs);
            continue;
        }
        y[b].d = amax / 127.0f;
        const float inv = 127.0f / amax;
        for (int l = 0; l < 32; ++l) {
            long v = lrintf(kqo_f16_to_f32(xb[l]) * inv);
            if (v > 127) v = 127;
            if (v < -127) v = -127;
            y[b].qs[l] = (int8_t)v;
        }
    }
}

/* Q4_K super-block (144 B: d, dmin, scales[12], qs[128]) x Q8_K block.
 * ENG:10996-11027 (eval_single_lm_row_dot, Q4_K branch). */
static void dot_q4k_block(const uint8_t *blk, const kqo_block_q8k *a, int32_t *o_sumi, int32_t *o_summ) {
    const uint8_t *scales = blk + 4;
    const uint8_t *q = blk + 16;
    int32_t sumi = 0, summ = 0;
    for (int c = 0; c < 4; ++c) {              /* four 64-element chunks */
        uint8_t sc_lo, m_lo, sc_hi, m_hi;
        kqo_get_scale_min_k4(2 * c + 0, scales, &sc_lo, &m_lo);
        kqo_get_scale_min_k4(2 * c + 1, scales, &sc_hi, &m_hi);
        int32_t dlo = 0, dhi = 0;
        for (int l = 0; l < 32; ++l) {
            const uint8_t byte = q[32 * c + l];
            dlo += (int32_t)(byte & 0x0F) * (int32_t)a->qs[64 * c + l];
            dhi += (int32_t)(byte >> 4) * (int32_t)a->qs[64 * c + 32 + l];
        }
        sumi += (int32_t)sc_lo * dlo + (int32_t)sc_hi * dhi;
        summ += (int32_t)m_lo * a->bsum32[2 * c] + (int32_t)m_hi * a->bsum32[2 * c + 1];
    }
    *o_sumi = sumi;
    *o_summ = summ;
}

/* Q5_K super-block (176 B: d, dmin, scales[12], qh[32], qs[128]) x Q8_K block.
 * ENG:11028-11064; the 5th bit of element l of chunk c is bit 2c (low half) / 2c+1 (high half)
 * of qh[l]. */
static void dot_q5k_block(const uint8_t *blk, const kqo_block_q8k *a, int32_t *o_sumi, int32_t *o_summ) {
    const uint8_t *scales = blk + 4;
    const uint8_t *qh = blk + 16;
    const uint8_t *ql = blk + 48;
    int32_t sumi = 0, summ = 0;
    for (int c = 0; c < 4; ++c) {
        uint8_t sc_lo, m_lo, sc_hi, m_hi;
        kqo_get_scale_min_k4(2 * c + 0, scales, &sc_lo, &m_lo);
        kqo_get_scale_min_k4(2 * c + 1, scales, &sc_hi, &m_hi);
        const uint8_t bit_lo = (uint8_t)(1u << (2 * c));
        const uint8_t bit_hi = (uint8_t)(2u << (2 * c));
        int32_t dlo = 0, dhi = 0;
        for (int l = 0; l < 32; ++l) {
            const uint8_t byte = ql[32 * c + l];
            const int w_lo = (int)(byte & 0x0F) + ((qh[l] & bit_lo) ? 16 : 0);
            const int w_hi = (int)(byte >> 4) + ((qh[l] & bit_hi) ? 16 : 0);
            dlo += w_lo * (int32_t)a->qs[64 * c + l];
            dhi += w_hi * (int32_t)a->qs[64 * c + 32 + l];
        }
        sumi += (int32_t)sc_lo * dlo + (int32_t)sc_hi * dhi;
        summ += (int32_t)m_lo * a->bsum32[2 * c] + (int32_t)m_hi * a->bsum32[2 * c + 1];
    }
    *o_sumi = sumi;
    *o_summ = summ;
}

/* Q6_K super-block (210 B: ql[128], qh[64], scales[16] int8, d @208) x Q8_K block.
 * ENG:11065-11101.  Element e = 128*h + 32*g + l (h half, g group 0..3, l 0..31):
 *   low nibble from ql[64h + l + 32*(g&1)] (>> 4 when g >= 2),
 *   two high bits from qh[32h + l] >> 2g, value minus 32, scale sc[8h + 2g + (l >= 16)]. */
static int32_t dot_q6k_block(const uint8_t *blk, const kqo_block_q8k *a) {
    const uint8_t *ql = blk;
    const uint8_t *qh = blk + 128;
    const int8_t *sc = (const int8_t *)(blk + 192);
    int32_t sumi = 0;
    for (int h = 0; h < 2; ++h) {
        for (int half16 = 0; half16 < 2; ++half16) {       /* l in [16*half16, 16*half16 + 16) */
            int32_t dg[4] = {0, 0, 0, 0};
            for (int l = 16 * half16; l < 16 * half16 + 16; ++l) {
                const uint8_t b0 = ql[64 * h + l];
                const uint8_t b1 = ql[64 * h + l + 32];
                const uint8_t hb = qh[32 * h + l];
                const int w0 = (int)((b0 & 0x0F) | (((hb >> 0) & 3) << 4)) - 32;
                const int w1 = (int)((b1 & 0x0F) | (((hb >> 2) & 3) << 4)) - 32;
                const int w2 = (int)((b0 >> 4) | (((hb >> 4) & 3) << 4)) - 32;
                const int w3 = (int)((b1 >> 4) | (((hb >> 6) & 3) << 4)) - 32;
                const int8_t *xa = a->qs + 128 * h;
                dg[0] += w0 * (int32_t)xa[l + 0];
                dg[1] += w1 * (int32_t)xa[l + 32];
                dg[2] += w2 * (int32_t)xa[l + 64];
                dg[3] += w3 * (int32_t)xa[l + 96];
            }
            const int8_t *sh = sc + 8 * h;
            sumi += (int32_t)sh[half16 + 0] * dg[0] + (int32_t)sh[half16 + 2] * dg[1]
                  + (int32_t)sh[half16 + 4] * dg[2] + (int32_t)sh[half16 + 6] * dg[3];
        }
    }
    return sumi;
}

float kqo_vec_dot(uint32_t type, const uint8_t *w_row, const void *act, int k,
                  int32_t *sumi_out, int32_t *summ_out) {
    float acc = 0.0f;
    if (type == KQO_TYPE_Q4_K || type == KQO_TYPE_Q5_K) {
        /* acc += dx * (d * sumi - dmin * summ), ENG:11025 / ENG:11062 */
        const kqo_block_q8k *a = (const kqo_block_q8k *)act;
        const int nb = k / 256;
        const size_t bb = (type == KQO_TYPE_Q4_K) ? 144 : 176;
        for (int b = 0; b < nb; ++b) {
            const uint8_t *blk = w_row + (size_t)b * bb;
            const float d = kqo_f16_to_f32(ld_u16(blk));
            const float dmin = kqo_f16_to_f32(ld_u16(blk + 2));
            int32_t si, sm;
            if (type == KQO_TYPE_Q4_K) dot_q4k_block(blk, &a[b], &si, &sm);
            else dot_q5k_block(blk, &a[b], &si, &sm);
            if (sumi_out) sumi_out[b] = si;
            if (summ_out) summ_out[b] = sm;
            const float t_d = d * (float)si;
            const float t_m = dmin * (float)sm;
            const float t = t_d - t_m;
            acc += a[b].d * t;
        }
        return acc;
    }
    if (type == KQO_TYPE_Q6_K) {
        /* acc += (d * dx) * sumi, ENG:11100 */
        const kqo_block_q8k *a = (const kqo_block_q8k *)act;
        const int nb = k / 256;
        for (int b = 0; b < nb; ++b) {
            const uint8_t *blk = w_row + (size_t)b * 210;
            const float d = kqo_f16_to_f32(ld_u16(blk + 208));
            const int32_t si = dot_q6k_block(blk, &a[b]);
            if (sumi_out) sumi_out[b] = si;
            if (summ_out) summ_out[b] = 0;
            const float s = d * a[b].d;
            acc += s * (float)si;
        }
        return acc;
    }
    if (type == KQO_TYPE_Q8_0) {
        /* out += (d * dx) * dot per 32 elements, ENG:3393-3407 */
        const kqo_block_q8_0 *a = (const kqo_block_q8_0 *)act;
        const int nb = k / 32;
        for (int b = 0; b < nb; ++b) {
            const uint8_t *blk = w_row + (size_t)b * 34;
            const float d = kqo_f16_to_f32(ld_u16(blk));
            const int8_t *qw = (const int8_t *)(blk + 2);
            int32_t dot = 0;
            for (int i = 0; i < 32; ++i) dot += (int32_t)qw[i] * (int32_t)a[b].qs[i];
            if (sumi_out) sumi_out[b] = dot;
            if (summ_out) summ_out[b] = 0;
            const float s = d * a[b].d;
            acc += s * (float)dot;
        }
        return acc;
    }
    return -1e30f;
}

void kqo_gemm(uint32_t type, const uint8_t *w, size_t row_bytes, int rows, int k,
              const void *act, int M, float *out, size_t ld_out) {
    const size_t act_row = (type == KQO_TYPE_Q8_0) ? (size_t)(k / 32) * sizeof(kqo_block_q8_0)
                                                   : (size_t)(k / 256) * sizeof(kqo_block_q8k);
    for (int m = 0; m < M; ++m) {
        const void *a = (const uint8_t *)act + (size_t)m * act_row;
        for (int r = 0; r < rows; ++r) {
            out[(size_t)m * ld_out + r] = kqo_vec_dot(type, w + (size_t)r * row_bytes, a, k, NULL, NULL);
        }
    }
}

void kqo_epilogue_f16(const float *sums, size_t ld_sums, int rows, int M,
                      uint16_t *dst, size_t dst_stride,
                      const uint16_t *residual, size_t res_stride) {
    /* ENG:3602-3611 */
    for (int m = 0; m < M; ++m) {
        for (int r = 0; r < rows; ++r) {
            float v = sums[(size_t)m * ld_sums + r];
            if (residual) v = v + kqo_f16_to_f32(residual[(size_t)m * res_stride + r]);
            dst[(size_t)m * dst_stride + r] = kqo_f32_to_f16(v);
        }
    }
}

void kqo_dequant_row(uint32_t type, const uint8_t *w, int n, uint16_t *dst) {
    if (type == KQO_TYPE_Q8_0) {
        /* ENG:598-615: fp16(d * q) */
        for (int b = 0; b < n / 32; ++b) {
            const uint8_t *blk = w + (size_t)b * 34;
            const float d = kqo_f16_to_f32(ld_u16(blk));
            const int8_t *q = (const int8_t *)(blk + 2);
            for (int i = 0; i < 32; ++i) dst[32 * b + i] = kqo_f32_to_f16(d * (float)q[i]);
        }
    } else if (type == KQO_TYPE_Q4_K || type == KQO_TYPE_Q5_K) {
        /* ENG:786-800 / ENG:837-852: fp16(d*sc*q - dmin*m) with (d*sc) and (dmin*m) rounded first */
        const size_t bb = (type == KQO_TYPE_Q4_K) ? 144 : 176;
        for (int b = 0; b < n / 256; ++b) {
            const uint8_t *blk = w + (size_t)b * bb;
            const float d = kqo_f16_to_f32(ld_u16(blk));
            const float dmin = kqo_f16_to_f32(ld_u16(blk + 2));
            const uint8_t *scales = blk + 4;
            const uint8_t *qh = blk + 16;
            const uint8_t *q = (type == KQO_TYPE_Q4_K) ? blk + 16 : blk + 48;
            uint16_t *o = dst + (size_t)256 * b;
            for (int c = 0; c < 4; ++c) {
                uint8_t sc0, m0, sc1, m1;
                kqo_get_scale_min_k4(2 * c, scales, &sc0, &m0);
                kqo_get_scale_min_k4(2 * c + 1, scales, &sc1, &m1);
                const float d0 = d * (float)sc0, mm0 = dmin * (float)m0;
                const float d1 = d * (float)sc1, mm1 = dmin * (float)m1;
                for (int l = 0; l < 32; ++l) {
                    const uint8_t byte = q[32 * c + l];
                    int v0 = byte & 0x0F, v1 = byte >> 4;
                    if (type == KQO_TYPE_Q5_K) {
                        v0 += (qh[l] & (1u << (2 * c))) ? 16 : 0;
                        v1 += (qh[l] & (2u << (2 * c))) ? 16 : 0;
                    }
                    o[64 * c + l] = kqo_f32_to_f16(d0 * (float)v0 - mm0);
                    o[64 * c + 32 + l] = kqo_f32_to_f16(d1 * (float)v1 - mm1);
                }
            }
        }
    } else if (type == KQO_TYPE_Q6_K) {
        /* ENG:712-740: fp16((d*sc) * (q - 32)) */
        for (int b = 0; b < n / 256; ++b) {
            const uint8_t *blk = w + (size_t)b * 210;
            const uint8_t *ql = blk;
            const uint8_t *qh = blk + 128;
            const int8_t *sc = (const int8_t *)(blk + 192);
            const float d = kqo_f16_to_f32(ld_u16(blk + 208));
            uint16_t *o = dst + (size_t)256 * b;
            for (int h = 0; h < 2; ++h) {
                for (int l = 0; l < 32; ++l) {
                    const int half16 = l >> 4;
                    const uint8_t b0 = ql[64 * h + l], b1 = ql[64 * h + l + 32], hb = qh[32 * h + l];
                    const int w0 = (int)((b0 & 0x0F) | (((hb >> 0) & 3) << 4)) - 32;
                    const int w1 = (int)((b1 & 0x0F) | (((hb >> 2) & 3) << 4)) - 32;
                    const int w2 = (int)((b0 >> 4) | (((hb >> 4) & 3) << 4)) - 32;
                    const int w3 = (int)((b1 >> 4) | (((hb >> 6) & 3) << 4)) - 32;
                    const int8_t *sh = sc + 8 * h;
                    o[128 * h + l + 0]  = kqo_f32_to_f16((d * (float)sh[half16 + 0]) * (float)w0);
                    o[128 * h + l + 32] = kqo_f32_to_f16((d * (float)sh[half16 + 2]) * (float)w1);
                    o[128 * h + l + 64] = kqo_f32_to_f16((d * (float)sh[half16 + 4]) * (float)w2);
                    o[128 * h + l + 96] = kqo_f32_to_f16((d * (float)sh[half16 + 6]) * (float)w3);
                }
            }
        }
    }
}

void kqo_rmsnorm_rows(const uint16_t *x_in, const uint16_t *gamma, uint16_t *x_out,
                      int M, int K, kqo_block_q8k *q8k) {
    /* ENG:4264-4314, scalar branch ENG:4291-4299 */
    const float inv_k = 1.0f / (float)K;
    for (int m = 0; m < M; ++m) {
        const uint16_t *xr = x_in + (size_t)m * K;
        uint16_t *yr = x_out + (size_t)m * K;
        float ss = 0.0f;
        for (int i = 0; i < K; ++i) {
            const float v = kqo_f16_to_f32(xr[i]);
            ss += v * v;
        }
        const float inv_rms = 1.0f / sqrtf(ss * inv_k + 1.0e-6f);
        for (int i = 0; i < K; ++i) {
            yr[i] = kqo_f32_to_f16(kqo_f16_to_f32(xr[i]) * inv_rms * kqo_f16_to_f32(gamma[i]));
        }
        if (q8k && (K % 256) == 0) kqo_quantize_row_q8k(yr, q8k + (size_t)m * (K / 256), K);
    }
}

void kqo_swiglu_rows(uint16_t *gate, const uint16_t *up, int M, int N, kqo_block_q8k *q8k) {
    /* ENG:4326-4358, scalar branch ENG:4350-4356 (libm expf) */
    for (int m = 0; m < M; ++m) {
        for (int i = 0; i < N; ++i) {
            const size_t o = (size_t)m * N + i;
            const float g = kqo_f16_to_f32(gate[o]);
            const float u = kqo_f16_to_f32(up[o]);
            gate[o] = kqo_f32_to_f16((g / (1.0f + expf(-g))) * u);
        }
        if (q8k) kqo_quantize_row_q8k(gate + (size_t)m * N, q8k + (size_t)m * (N / 256), N);
    }
}

void kqo_ffn(uint32_t gate_type, const uint8_t *w_gate, uint32_t up_type, const uint8_t *w_up,
             uint32_t down_type, const uint8_t *w_down, int hidden, int ffn,
             const uint16_t *x_in, const uint16_t *gamma, uint16_t *x_out, int M) {
    /* ENG:8283-8298 */
    uint16_t *xn = malloc(sizeof(uint16_t) * (size_t)M * hidden);
    uint16_t *g = malloc(sizeof(uint16_t) * (size_t)M * ffn);
    uint16_t *u = malloc(sizeof(uint16_t) * (size_t)M * ffn);
    float *s = malloc(sizeof(float) * (size_t)M * (ffn > hidden ? ffn : hidden));
    kqo_block_q8k *qa = malloc(sizeof(kqo_block_q8k) * (size_t)M * (hidden / 256));
    kqo_block_q8k *qh = malloc(sizeof(kqo_block_q8k) * (size_t)M * (ffn / 256));
    kqo_block_q8_0 *qa0 = malloc(sizeof(kqo_block_q8_0) * (size_t)M * (hidden / 32));
    kqo_block_q8_0 *qh0 = malloc(sizeof(kqo_block_q8_0) * (size_t)M * (ffn / 32));

    kqo_rmsnorm_rows(x_in, gamma, xn, M, hidden, qa);
    /* a Q8_0 weight needs the Q8_0 activation (ENG:4212-4216); Q8_K stays pre-quantized */
    for (int m = 0; m < M; ++m) kqo_quantize_row_q8_0(xn + (size_t)m * hidden, qa0 + (size_t)m * (hidden / 32), hidden);

    kqo_gemm(gate_type, w_gate, kqo_row_bytes(gate_type, hidden), ffn, hidden,
             gate_type == KQO_TYPE_Q8_0 ? (const void *)qa0 : (const void *)qa, M, s, ffn);
    kqo_epilogue_f16(s, ffn, ffn, M, g, ffn, NULL, 0);
    kqo_gemm(up_type, w_up, kqo_row_bytes(up_type, hidden), ffn, hidden,
             up_type == KQO_TYPE_Q8_0 ? (const void *)qa0 : (const void *)qa, M, s, ffn);
    kqo_epilogue_f16(s, ffn, ffn, M, u, ffn, NULL, 0);

    kqo_swiglu_rows(g, u, M, ffn, qh);
    for (int m = 0; m < M; ++m) kqo_quantize_row_q8_0(g + (size_t)m * ffn, qh0 + (size_t)m * (ffn / 32), ffn);

    kqo_gemm(down_type, w_down, kqo_row_bytes(down_type, ffn), hidden, ffn,
             down_type == KQO_TYPE_Q8_0 ? (const void *)qh0 : (const void *)qh, M, s, hidden);
    kqo_epilogue_f16(s, hidden, hidden, M, x_out, hidden, x_in, hidden);

    free(xn); free(g); free(u); free(s); free(qa); free(qh); free(qa0); free(qh0);
}

void kqo_rows_argmax(uint32_t type, const uint8_t *w, size_t row_bytes, int k,
                     const uint32_t *row_ids, int n_rows, const void *act, int M,
                     int f16_compare, float *logits, uint32_t *best_id, float *best_val) {
    const size_t act_row = (type == KQO_TYPE_Q8_0) ? (size_t)(k / 32) * sizeof(kqo_block_q8_0)
                                                   : (size_t)(k / 256) * sizeof(kqo_block_q8k);
    for (int m = 0; m < M; ++m) {
        const void *a = (const uint8_t *)act + (size_t)m * act_row;
        float bv = -1e30f;          /* ENG:9490-9493 */
        uint32_t bi = 0;
        for (int i = 0; i < n_rows; ++i) {
            const uint32_t rid = row_ids ? row_ids[i] : (uint32_t)i;
            float v = kqo_vec_dot(type, w + (size_t)rid * row_bytes, a, k, NULL, NULL);
            if (logits) logits[(size_t)m * n_rows + i] = v;
            if (f16_compare) v = kqo_f16_to_f32(kqo_f32_to_f16(v));
            if (v > bv) { bv = v; bi = rid; }
        }
        best_id[m] = bi;
        best_val[m] = bv;
    }
}
