// kq_gemv_dev.cuh -- device parts of the small-batch K-quant products shared by the GEMV kernel
// (kq_gemv.cu) and the fused FFN kernel (kq_ffn_fused.cu): launch parameters, activation
// staging, the per-tile products and the in-order folds.  The layout and arithmetic are
// described at the top of kq_gemv.cu.
#pragma once

#include "kq_common.cuh"

namespace kq {

constexpr int kMaxTermSlots = 32;

// consumer warps: 15 for the dp4a kernels (M <= 2, 64 registers: two CTAs of 512 threads per
// SM), 12 for the MMA kernels (72 registers)
template <int MT>
__host__ __device__ constexpr int warps_of() { return MT <= 2 ? 15 : 12; }
template <int MT>
__host__ __device__ constexpr int threads_of() { return (warps_of<MT>() + 1) * 32; }

struct GemvTaskDev {
    const uint8_t *w;  // tiled weight, row group 0 of the tensor
    int rg_first;      // first row group of the task (row_begin / 16)
    int n_rg;          // row groups of the task
    int rg_start;      // first row group of the task in the launch's concatenated space
    int row_begin, rows;
    __half *dst;
    long long dst_stride;
    const __half *res;
    long long res_stride;
    float *dst_f32;
    long long f32_stride;
    int *dbg_sumi;
    int *dbg_summ;
    const uint32_t *out_ids;  // output column of local row r is out_ids[r] (else r)
    int index_base;           // argmax index of local row r is index_base + r
};

struct GemvParams {
    GemvTaskDev task[4];
    int n_tasks;
    int total_rg;
    int K;
    int nbu;               // 256-value units per row = tiles per row group
    int M;
    unsigned tile_bytes;
    int tiles_per_stage;   // T
    int n_stages;          // S
    int term_slots;        // TS (large launches)
    int terms_per_rg;      // J: terms per (row, token) of a row group
    int q80_exact;         // Q8_0: one term per 32-block (exact order); else one per tile
    unsigned stage_bytes;
    const __half *x;
    long long x_stride;
    const void *act;
    int *status;
    unsigned long long timeout_ns;
    unsigned long long *argmax;  // [M] packed (ordered value, ~index) keys, or nullptr
    int argmax_f16;              // compare the fp16-rounded results (the dispatch's stored logits)
    int inject_wait;             // failure test: consumers first wait on a barrier nothing arrives at
    unsigned off_x, off_dx, off_xs, off_terms, off_stages, off_bars;
    // Tile-range ownership (the kernels' SPLIT variant): CTA c owns tiles [T c / G, T (c + 1) / G)
    // of the launch's T = total_rg * nbu tiles, so a row group can be shared by consecutive CTAs.
    // Each CTA stores its block terms of a shared row group in slot s = (CTA holding the row
    // group's first tile) of gterms ([G][J][16 MT] floats) and counts its arrival in gcount[s];
    // the last CTA to arrive adds all J terms in block order and resets gcount[s] to 0.
    long long total_tiles;
    float *gterms;
    int *gcount;
    PeerOut peer;  // task 0's fp32 outputs also into every rank's gather buffer (peer.n > 0)
    // Half row-group ownership (Q4_K / Q5_K, <= 2 tokens, the whole share in one stage): CTA c
    // owns the 8-row halves [2 R c / G, 2 R (c + 1) / G) of the launch's R row groups, so no CTA
    // holds more than one half above the mean and no row is shared between CTAs.
    int half;
};


// token-slot pitch of the dx / -32*xsum tables (mma reads of tokens 2t, 2t+1 stay inside)
template <int MT>
__device__ __forceinline__ constexpr int xpitch() { return MT < 2 ? 2 : MT; }
template <int MT>
__device__ __forceinline__ int tok_pair(int t) { return min(2 * t, xpitch<MT>() - 2); }
template <int MT>
__device__ __forceinline__ constexpr bool use_dp() { return MT <= 2; }

// ------------------------------------------------------------------ activation staging
//
// Shared-memory activation of MT token slots (tokens >= M are never read for an output):
//  * x, int8 quants.  dp4a items (M <= 2): per token nbu units of 320 bytes, value k of a unit
//    at 80 (k / 64) + k % 64 (Q6_K: 160 (k / 128) + k % 128), so the four quarter-lanes of a
//    row read four different bank groups.  MMA items: [tok][K + 16] (the pad puts the tokens of
//    one ldmatrix in different bank groups).
//  * dx: the Q8_K scale of (unit, token) at [u][tok] (Q8_0: the block scale at [u*8+j][tok]).
//  * Q4_K/Q5_K: the block's bsum32[8] at [tok][u][8].
//  * Q6_K: -32 * (sum of the 16 quants of sub-block s = 8h + 2g + l), dp4a: [u][2h+l][tok][g],
//    MMA: [u][s][tok].

__device__ __forceinline__ int sum_s8x4(uint32_t w) {
    return (int)(int8_t)(w & 0xFF) + (int)(int8_t)((w >> 8) & 0xFF) + (int)(int8_t)((w >> 16) & 0xFF) +
           (int)(int8_t)(w >> 24);
}

// Quantize 8 fp16 values per lane of one 256-value unit: Q8_K (per 256, ENG:925-990) or Q8_0
// (per 32-value block = 4 lanes, ENG:1016-1064).  Returns the packed quants and the scale.
template <int TYPE>
__device__ __forceinline__ void quantize_lane(const uint4 raw, uint32_t &lo, uint32_t &hi, float &d) {
    float v[8];
    const __half2 *h2 = reinterpret_cast<const __half2 *>(&raw);
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        const float2 f = __half22float2(h2[i]);
        v[2 * i] = f.x;
        v[2 * i + 1] = f.y;
    }
    float amax = 0.0f;
#pragma unroll
    for (int i = 0; i < 8; ++i) amax = fmaxf(amax, fabsf(v[i]));
    constexpr int span = (TYPE == TYPE_Q8_0) ? 4 : 32;
#pragma unroll
    for (int o = 1; o < span; o <<= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
    int q[8];
    if (amax == 0.0f) {
#pragma unroll
        for (int i = 0; i < 8; ++i) q[i] = 0;
    } else {
        const float inv = __fdiv_rn(127.0f, amax);
#pragma unroll
        for (int i = 0; i < 8; ++i) q[i] = max(-127, min(127, __float2int_rn(__fmul_rn(v[i], inv))));
    }
    lo = (uint32_t)(q[0] & 0xFF) | ((uint32_t)(q[1] & 0xFF) << 8) | ((uint32_t)(q[2] & 0xFF) << 16) |
         ((uint32_t)(q[3] & 0xFF) << 24);
    hi = (uint32_t)(q[4] & 0xFF) | ((uint32_t)(q[5] & 0xFF) << 8) | ((uint32_t)(q[6] & 0xFF) << 16) |
         ((uint32_t)(q[7] & 0xFF) << 24);
    d = (amax == 0.0f) ? 0.0f : __fdiv_rn(amax, 127.0f);
}

// Pre-quantized input (BlockQ8K / BlockQ8_0_Fast): every 4-byte word goes straight to its place
// in shared memory with cp.async -- all copies of the CTA in flight at once, no register round
// trip -- so the staging costs one global-memory latency whatever M and K.  Q6_K's
// -32 * (sub-block sums) are then formed from the staged quants.
template <int TYPE, int MT>
__device__ __noinline__ void stage_activation_q(const GemvParams &p, uint8_t *smem, int warp, int lane, int W) {
    constexpr int XP = xpitch<MT>();
    uint8_t *xq = smem + p.off_x;
    int *aux = reinterpret_cast<int *>(smem + p.off_xs);
    const uint32_t xq_s = smem_u32(xq), dx_s = smem_u32(smem + p.off_dx), aux_s = smem_u32(aux);
    const int nbu = p.nbu, n_units = p.M * nbu;
    for (int i = warp; i < n_units; i += W) {
        const int m = i / nbu, u = i - m * nbu;
        const size_t xbase = use_dp<MT>() ? (size_t)(m * nbu + u) * 320 : (size_t)m * (p.K + 16) + 256 * u;
        if (TYPE == TYPE_Q8_0) {
            // lane: quants 8(L%4)..+7 of block L/4 and that block's scale
            const uint8_t *blk = reinterpret_cast<const uint8_t *>(reinterpret_cast<const BlockQ80 *>(p.act) +
                                                                   ((size_t)m * nbu + u) * 8 + (lane >> 2));
#pragma unroll
            for (int h = 0; h < 2; ++h) {
                const int v = 8 * lane + 4 * h;
                const size_t xo = use_dp<MT>() ? xbase + 80 * (v >> 6) + (v & 63) : xbase + v;
                cp_async4(xq_s + (uint32_t)xo, blk + 4 + 8 * (lane & 3) + 4 * h);
            }
            if ((lane & 3) == 0) cp_async4(dx_s + 4u * (uint32_t)((u * 8 + (lane >> 2)) * XP + m), blk);
        } else {
            // BlockQ8K (ENG:868-872): float d at 0, qs[256] at 4, bsum32[8] at 260
            const uint8_t *blk =
                reinterpret_cast<const uint8_t *>(reinterpret_cast<const BlockQ8K *>(p.act) + (size_t)m * nbu + u);
#pragma unroll
            for (int h = 0; h < 2; ++h) {
                const int v = 4 * lane + 128 * h;
                size_t xo;
                if (!use_dp<MT>()) xo = xbase + v;
                else if (TYPE == TYPE_Q6_K) xo = xbase + 160 * (v >> 7) + (v & 127);
                else xo = xbase + 80 * (v >> 6) + (v & 63);
                cp_async4(xq_s + (uint32_t)xo, blk + 4 + v);
            }
            if (lane == 0) cp_async4(dx_s + 4u * (uint32_t)(u * XP + m), blk);
            if ((TYPE == TYPE_Q4_K || TYPE == TYPE_Q5_K) && lane < 8)
                cp_async4(aux_s + 4u * (uint32_t)((m * nbu + u) * 8 + lane), blk + 260 + 4 * lane);
        }
    }
    cp_async_wait_all();
    if (TYPE == TYPE_Q6_K) {
        named_bar_sync(1, W * 32);  // every consumer's copies have landed
        for (int i = warp * 32 + lane; i < n_units * 16; i += W * 32) {
            const int s = i & 15, mu = i >> 4, m = mu / nbu, u = mu - m * nbu, v = 16 * s;
            const size_t xo = use_dp<MT>() ? (size_t)(m * nbu + u) * 320 + 160 * (v >> 7) + (v & 127)
                                           : (size_t)m * (p.K + 16) + 256 * u + v;
            const uint4 q = *reinterpret_cast<const uint4 *>(xq + xo);
            const int s16 = sum_s8x4(q.x) + sum_s8x4(q.y) + sum_s8x4(q.z) + sum_s8x4(q.w);
            const int h = s >> 3, g = (s >> 1) & 3, l = s & 1;
            if (use_dp<MT>()) aux[((u * 4 + 2 * h + l) * MT + m) * 4 + g] = -32 * s16;
            else aux[(u * 16 + s) * XP + m] = -32 * s16;
        }
    }
}

// Stage the M tokens' activation (consumer warps): fp16 input quantized in-kernel, or (up to 2
// tokens) a pre-quantized input copied through registers.  Loads of up to 4 units per warp are
// issued before any is used, so the staging costs about one global-memory latency.  Pre-quantized
// inputs of more tokens (hundreds of units per CTA) go through stage_activation_q.
// Store one 256-value unit (m, u) of the activation in the layout above.  Lane L holds values
// 8L .. 8L+7 as quants (lo, hi) with the unit's scale d (Q8_0: the scale of block L / 4) and,
// for a pre-quantized Q8_K input, bsum = that block's bsum32[L] (lanes < 8).  `fresh`: the quants
// were made here (the sub-block sums are formed from them), else they came with their bsum32.
template <int TYPE, int MT>
__device__ __forceinline__ void store_act_unit(const GemvParams &p, uint8_t *smem, int m, int u, int lane,
                                               uint32_t lo, uint32_t hi, float d, int bsum, bool fresh) {
    constexpr int XP = xpitch<MT>();
    uint8_t *xq = smem + p.off_x;
    float *dx = reinterpret_cast<float *>(smem + p.off_dx);
    int *aux = reinterpret_cast<int *>(smem + p.off_xs);
    const int nbu = p.nbu;
    size_t xo;
    if (!use_dp<MT>()) xo = (size_t)m * (p.K + 16) + 256 * u + 8 * lane;
    else if (TYPE == TYPE_Q6_K) xo = (size_t)(m * nbu + u) * 320 + 160 * (lane >> 4) + 8 * (lane & 15);
    else xo = (size_t)(m * nbu + u) * 320 + 80 * (lane >> 3) + 8 * (lane & 7);
    *reinterpret_cast<uint2 *>(xq + xo) = make_uint2(lo, hi);
    if (TYPE == TYPE_Q8_0) {
        if ((lane & 3) == 0) dx[(u * 8 + (lane >> 2)) * XP + m] = d;
    } else {
        if (lane == 0) dx[u * XP + m] = d;
    }
    if (TYPE == TYPE_Q6_K) {
        const int s8 = sum_s8x4(lo) + sum_s8x4(hi);
        const int s16 = s8 + __shfl_xor_sync(0xffffffffu, s8, 1);
        if ((lane & 1) == 0) {
            const int s = lane >> 1, h = s >> 3, g = (s >> 1) & 3, l = s & 1;
            if (use_dp<MT>()) aux[((u * 4 + 2 * h + l) * MT + m) * 4 + g] = -32 * s16;
            else aux[(u * 16 + s) * XP + m] = -32 * s16;
        }
    } else if (TYPE == TYPE_Q4_K || TYPE == TYPE_Q5_K) {
        if (fresh) {
            int s = sum_s8x4(lo) + sum_s8x4(hi);
            s += __shfl_xor_sync(0xffffffffu, s, 1);
            s += __shfl_xor_sync(0xffffffffu, s, 2);
            if ((lane & 3) == 0) aux[(m * nbu + u) * 8 + (lane >> 2)] = s;
        } else if (lane < 8) {
            aux[(m * nbu + u) * 8 + lane] = bsum;
        }
    }
}

template <int TYPE, int MT>
__device__ __forceinline__ void stage_activation(const GemvParams &p, uint8_t *smem, int warp, int lane, int W) {
    if (MT > 2 && !p.x) {
        stage_activation_q<TYPE, MT>(p, smem, warp, lane, W);
        return;
    }
    const int nbu = p.nbu, n_units = p.M * nbu;
    for (int i0 = warp; i0 < n_units; i0 += 4 * W) {
        uint4 raw[4];
        int bs[4];
#pragma unroll
        for (int b = 0; b < 4; ++b) {
            const int i = i0 + b * W;
            raw[b] = make_uint4(0, 0, 0, 0);
            bs[b] = 0;
            if (i < n_units) {
                const int m = i / nbu, u = i - (i / nbu) * nbu;
                if (MT > 2 || p.x) {
                    const __half *xu = p.x + (size_t)m * p.x_stride + (size_t)u * 256 + 8 * lane;
                    if ((reinterpret_cast<uintptr_t>(xu) & 15) == 0) {
                        raw[b] = *reinterpret_cast<const uint4 *>(xu);
                    } else {
                        uint32_t hv[8];
#pragma unroll
                        for (int k = 0; k < 8; ++k) hv[k] = reinterpret_cast<const uint16_t *>(xu)[k];
                        raw[b] = make_uint4(hv[0] | (hv[1] << 16), hv[2] | (hv[3] << 16), hv[4] | (hv[5] << 16),
                                            hv[6] | (hv[7] << 16));
                    }
                } else if (TYPE == TYPE_Q8_0) {
                    // eight BlockQ8_0_Fast: lane takes quants 8(L%4)..+7 of block L/4 and its scale
                    const uint32_t *w = reinterpret_cast<const uint32_t *>(
                        reinterpret_cast<const BlockQ80 *>(p.act) + ((size_t)m * nbu + u) * 8 + (lane >> 2));
                    raw[b] = make_uint4(w[1 + 2 * (lane & 3)], w[2 + 2 * (lane & 3)], w[0], 0);
                } else {
                    const uint32_t *w =
                        reinterpret_cast<const uint32_t *>(reinterpret_cast<const BlockQ8K *>(p.act) + (size_t)m * nbu + u);
                    raw[b] = make_uint4(w[1 + 2 * lane], w[2 + 2 * lane], w[0], 0);
                    if (lane < 8) bs[b] = (int)w[65 + lane];  // bsum32 as stored (ENG:868-872)
                }
            }
        }
#pragma unroll
        for (int b = 0; b < 4; ++b) {
            const int i = i0 + b * W;
            if (i >= n_units) break;  // uniform across the warp
            const int m = i / nbu, u = i - (i / nbu) * nbu;
            uint32_t lo, hi;
            float d;
            const bool fresh = MT > 2 || p.x;
            if (fresh) {
                quantize_lane<TYPE>(raw[b], lo, hi, d);
            } else {
                lo = raw[b].x;
                hi = raw[b].y;
                d = __uint_as_float(raw[b].z);
            }
            store_act_unit<TYPE, MT>(p, smem, m, u, lane, lo, hi, d, bs[b], fresh);
        }
    }
}

// ------------------------------------------------------------------ per-item products
//
// A tile is 16 weight rows x 256 values of unit u (row-major, kq_common.cuh).  Each (row,
// token) gets the fp32 block term with the reference's operation order, stored at
// terms[j * 16 * MT + row * MT + token] (j = 0, or the Q8_0 block in exact mode).

struct DbgOut {
    int *si, *sm;       // [M][rows][blocks per row] (rows of the task), or si == nullptr
    int r0;             // task-local row of tile row 0 (may be negative)
    int rows;           // task rows
    int bpr;            // blocks per row
    int blk0;           // first block of the tile
    int M;
};

__device__ __forceinline__ void dbg_put(const DbgOut &db, int rr, int tok, int blk, int si, int sm) {
    const int r = db.r0 + rr;
    if (tok < db.M && r >= 0 && r < db.rows) {
        const size_t o = ((size_t)tok * db.rows + r) * db.bpr + db.blk0 + blk;
        db.si[o] = si;
        db.sm[o] = sm;
    }
}

template <int MT>
__device__ __forceinline__ void store_terms4(float *terms, int lane, const float tm[4]) {
    const int g = lane >> 2, t = lane & 3;
    if (2 * t < MT) {
        terms[g * MT + 2 * t] = tm[0];
        terms[(g + 8) * MT + 2 * t] = tm[2];
    }
    if (2 * t + 1 < MT) {
        terms[g * MT + 2 * t + 1] = tm[1];
        terms[(g + 8) * MT + 2 * t + 1] = tm[3];
    }
}

// ---- dp4a tiles (M <= 2): lane 2r + h takes half h of row r (two 64-value chunks).

template <int TYPE, int MT>
__device__ __forceinline__ void tile_q45k_dp(const uint8_t *tile, const uint8_t *xu, int XSD, const float *dxu,
                                             const int *bsu, int nbu8, int lane, float *terms, const DbgOut &db) {
    constexpr int RB = (TYPE == TYPE_Q4_K) ? 144 : 176, QS = (TYPE == TYPE_Q4_K) ? 16 : 48;
    const int rr = lane >> 1, hf = lane & 1;
    const uint8_t *row = tile + RB * rr;
    const uint4 h = lds128(row);
    const uint32_t sc = hf ? ((h.w & 0x0F0F0F0Fu) | ((h.y >> 2) & 0x30303030u)) : (h.y & 0x3F3F3F3Fu);
    const uint32_t mn = hf ? (((h.w >> 4) & 0x0F0F0F0Fu) | ((h.z >> 2) & 0x30303030u)) : (h.z & 0x3F3F3F3Fu);
    uint32_t qh[8];
    if (TYPE == TYPE_Q5_K) {
        const uint4 a = lds128(row + 16), b = lds128(row + 32);
        qh[0] = a.x, qh[1] = a.y, qh[2] = a.z, qh[3] = a.w, qh[4] = b.x, qh[5] = b.y, qh[6] = b.z, qh[7] = b.w;
    }
    int si[MT];
#pragma unroll
    for (int m = 0; m < MT; ++m) si[m] = 0;
#pragma unroll
    for (int cc = 0; cc < 2; ++cc) {
        const int c = 2 * hf + cc;
        const uint4 qa = lds128(row + QS + 32 * c), qb = lds128(row + QS + 32 * c + 16);
        const uint32_t w[8] = {qa.x, qa.y, qa.z, qa.w, qb.x, qb.y, qb.z, qb.w};
        uint32_t wl[8], wh[8];
#pragma unroll
        for (int i = 0; i < 8; ++i) {
            if (TYPE == TYPE_Q4_K) {
                wl[i] = w[i] & 0x0F0F0F0Fu;
                wh[i] = w[i] & 0xF0F0F0F0u;  // 16 x the high nibble
            } else {
                wl[i] = (w[i] & 0x0F0F0F0Fu) | (((qh[i] >> (2 * c)) & 0x01010101u) << 4);
                wh[i] = ((w[i] >> 4) & 0x0F0F0F0Fu) | (((qh[i] >> (2 * c + 1)) & 0x01010101u) << 4);
            }
        }
        const int s_lo = ubyte(sc, 2 * cc), s_hi = ubyte(sc, 2 * cc + 1);
#pragma unroll
        for (int m = 0; m < MT; ++m) {
            const uint8_t *xm = xu + m * XSD + 80 * c;
            const uint4 x0 = lds128(xm), x1 = lds128(xm + 16), x2 = lds128(xm + 32), x3 = lds128(xm + 48);
            const uint32_t xl[8] = {x0.x, x0.y, x0.z, x0.w, x1.x, x1.y, x1.z, x1.w};
            const uint32_t xh[8] = {x2.x, x2.y, x2.z, x2.w, x3.x, x3.y, x3.z, x3.w};
            int dl0 = 0, dl1 = 0, dh0 = 0, dh1 = 0;
#pragma unroll
            for (int i = 0; i < 8; i += 2) {
                dl0 = dp4a_us(wl[i], xl[i], dl0);
                dl1 = dp4a_us(wl[i + 1], xl[i + 1], dl1);
                dh0 = dp4a_us(wh[i], xh[i], dh0);
                dh1 = dp4a_us(wh[i + 1], xh[i + 1], dh1);
            }
            if (TYPE == TYPE_Q4_K) si[m] += s_lo * ((dl0 + dl1) << 4) + s_hi * (dh0 + dh1);
            else si[m] += s_lo * (dl0 + dl1) + s_hi * (dh0 + dh1);
        }
    }
    const float d = half_bits_to_float(h.x), dmin = half_bits_to_float(h.x >> 16);
#pragma unroll
    for (int m = 0; m < MT; ++m) {
        const int4 b = *reinterpret_cast<const int4 *>(bsu + m * nbu8 + 4 * hf);
        int sm = ubyte(mn, 0) * b.x + ubyte(mn, 1) * b.y + ubyte(mn, 2) * b.z + ubyte(mn, 3) * b.w;
        const int sit = si[m] + __shfl_xor_sync(0xffffffffu, si[m], 1);
        sm += __shfl_xor_sync(0xffffffffu, sm, 1);
        if (hf == 0) {
            const int sumi = (TYPE == TYPE_Q4_K) ? (sit >> 4) : sit;
            terms[rr * MT + m] =
                __fmul_rn(dxu[m], __fsub_rn(__fmul_rn(d, __int2float_rn(sumi)), __fmul_rn(dmin, __int2float_rn(sm))));
            if (db.si) dbg_put(db, rr, m, 0, sumi, sm);
        }
    }
}

template <int MT>
__device__ __forceinline__ void tile_q6k_dp(const uint8_t *tile, const uint8_t *xu, int XSD, const float *dxu,
                                            const int *xsu, int lane, float *terms, const DbgOut &db) {
    const int rr = lane >> 1, h = lane & 1;
    const uint8_t *row = tile + 208 * rr;
    const uint4 a0 = lds128(row + 64 * h), a1 = lds128(row + 64 * h + 16);
    const uint4 b0 = lds128(row + 64 * h + 32), b1 = lds128(row + 64 * h + 48);
    const uint4 q0 = lds128(row + 128 + 32 * h), q1 = lds128(row + 144 + 32 * h);
    const uint2 scv = lds64(row + 192 + 8 * h);
    const uint32_t A[8] = {a0.x, a0.y, a0.z, a0.w, a1.x, a1.y, a1.z, a1.w};
    const uint32_t B[8] = {b0.x, b0.y, b0.z, b0.w, b1.x, b1.y, b1.z, b1.w};
    const uint32_t H[8] = {q0.x, q0.y, q0.z, q0.w, q1.x, q1.y, q1.z, q1.w};
    int acc[MT];
#pragma unroll
    for (int m = 0; m < MT; ++m) acc[m] = 0;
#pragma unroll
    for (int g = 0; g < 4; ++g) {
        uint32_t q[8];
#pragma unroll
        for (int i = 0; i < 8; ++i) {
            if (g == 0) q[i] = (A[i] & 0x0F0F0F0Fu) | ((H[i] << 4) & 0x30303030u);
            else if (g == 1) q[i] = (B[i] & 0x0F0F0F0Fu) | ((H[i] << 2) & 0x30303030u);
            else if (g == 2) q[i] = ((A[i] >> 4) & 0x0F0F0F0Fu) | (H[i] & 0x30303030u);
            else q[i] = ((B[i] >> 4) & 0x0F0F0F0Fu) | ((H[i] >> 2) & 0x30303030u);
        }
        const uint32_t sw = (g < 2) ? scv.x : scv.y;
        const int sc0 = sbyte(sw, 2 * (g & 1)), sc1 = sbyte(sw, 2 * (g & 1) + 1);
#pragma unroll
        for (int m = 0; m < MT; ++m) {
            const uint8_t *xm = xu + m * XSD + 160 * h + 32 * g;
            const uint4 x0 = lds128(xm), x1 = lds128(xm + 16);
            // -32 * sums of sub-blocks 8h + 2g (quarter 2h) and 8h + 2g + 1 (quarter 2h + 1)
            int d0 = xsu[((2 * h) * MT + m) * 4 + g], d1 = xsu[((2 * h + 1) * MT + m) * 4 + g];
            d0 = dp4a_us(q[0], x0.x, d0);
            d1 = dp4a_us(q[4], x1.x, d1);
            d0 = dp4a_us(q[1], x0.y, d0);
            d1 = dp4a_us(q[5], x1.y, d1);
            d0 = dp4a_us(q[2], x0.z, d0);
            d1 = dp4a_us(q[6], x1.z, d1);
            d0 = dp4a_us(q[3], x0.w, d0);
            d1 = dp4a_us(q[7], x1.w, d1);
            acc[m] += sc0 * d0 + sc1 * d1;
        }
    }
    const float d = half_bits_to_float(*reinterpret_cast<const uint16_t *>(tile + 3328 + 2 * rr));
#pragma unroll
    for (int m = 0; m < MT; ++m) {
        const int a = acc[m] + __shfl_xor_sync(0xffffffffu, acc[m], 1);
        if (h == 0) {
            terms[rr * MT + m] = __fmul_rn(__fmul_rn(d, dxu[m]), __int2float_rn(a));
            if (db.si) dbg_put(db, rr, m, 0, a, 0);
        }
    }
}

template <int MT>
__device__ __forceinline__ void tile_q80_dp(const uint8_t *tile, const uint8_t *xu, int XSD, const float *dxu,
                                            int lane, float *terms, int exact, const DbgOut &db) {
    constexpr int XP = xpitch<MT>();
    const int rr = lane >> 1, h = lane & 1;
    const uint8_t *row = tile + 272 * rr;
    const uint2 dv = lds64(row + 8 * h);
    float tv[4][MT];
#pragma unroll
    for (int b = 0; b < 4; ++b) {
        const int jj = 4 * h + b;
        const uint4 w0 = lds128(row + 16 + 32 * jj), w1 = lds128(row + 32 + 32 * jj);
        const float dw = half_bits_to_float(((b < 2) ? dv.x : dv.y) >> (16 * (b & 1)));
#pragma unroll
        for (int m = 0; m < MT; ++m) {
            const uint8_t *xm = xu + m * XSD + 80 * (jj >> 1) + 32 * (jj & 1);
            const uint4 x0 = lds128(xm), x1 = lds128(xm + 16);
            int d0 = dp4a_ss(w0.x, x0.x, 0), d1 = dp4a_ss(w0.y, x0.y, 0);
            d0 = dp4a_ss(w0.z, x0.z, d0);
            d1 = dp4a_ss(w0.w, x0.w, d1);
            d0 = dp4a_ss(w1.x, x1.x, d0);
            d1 = dp4a_ss(w1.y, x1.y, d1);
            d0 = dp4a_ss(w1.z, x1.z, d0);
            d1 = dp4a_ss(w1.w, x1.w, d1);
            const int dot = d0 + d1;
            tv[b][m] = __fmul_rn(__fmul_rn(dw, dxu[jj * XP + m]), __int2float_rn(dot));
            if (exact) terms[jj * 16 * MT + rr * MT + m] = tv[b][m];
            if (db.si) dbg_put(db, rr, m, jj, dot, 0);
        }
    }
    if (!exact) {
#pragma unroll
        for (int m = 0; m < MT; ++m) {
            float acc = 0.0f;
#pragma unroll
            for (int b = 0; b < 4; ++b) acc = __fadd_rn(acc, tv[b][m]);
#pragma unroll
            for (int b = 0; b < 4; ++b) acc = __fadd_rn(acc, __shfl_xor_sync(0xffffffffu, tv[b][m], 1));
            if (h == 0) terms[rr * MT + m] = acc;
        }
    }
}

// ---- MMA tiles (M > 2)

// Q4_K / Q5_K with m16n8k32: per 64-value chunk c, one ldmatrix gives rows g, g+8 x bytes
// 4t..4t+3 and 16+4t..16+4t+3 of qs[32c..32c+31] (low nibbles = sub-block 2c, high = 2c+1);
// a second gives the activation of tokens 0..7 for both sub-blocks.  Mins are one more MMA
// against each row's min replicated over the sub-block (sum_l m_j x_l = m_j * bsum_j).
template <int TYPE, int MT>
__device__ __forceinline__ void tile_q45k_mma(const uint8_t *tile, const int8_t *xu, int XS, const float *dxu,
                                              int lane, float *terms, const DbgOut &db) {
    constexpr int RB = (TYPE == TYPE_Q4_K) ? 144 : 176, QS = (TYPE == TYPE_Q4_K) ? 16 : 48;
    const int g = lane >> 2, t = lane & 3, tp = tok_pair<MT>(t);
    const uint4 h0 = lds128(tile + RB * g), h1 = lds128(tile + RB * (g + 8));
    const uint32_t sc0[2] = {h0.y & 0x3F3F3F3Fu, (h0.w & 0x0F0F0F0Fu) | ((h0.y >> 2) & 0x30303030u)};
    const uint32_t sc1[2] = {h1.y & 0x3F3F3F3Fu, (h1.w & 0x0F0F0F0Fu) | ((h1.y >> 2) & 0x30303030u)};
    const uint32_t mn0[2] = {h0.z & 0x3F3F3F3Fu, ((h0.w >> 4) & 0x0F0F0F0Fu) | ((h0.z >> 2) & 0x30303030u)};
    const uint32_t mn1[2] = {h1.z & 0x3F3F3F3Fu, ((h1.w >> 4) & 0x0F0F0F0Fu) | ((h1.z >> 2) & 0x30303030u)};
    // ldmatrix row addresses: weight row (lane % 16), column half (lane / 16); token (lane % 8) % MT
    const uint32_t wrow = smem_u32(tile + RB * (lane & 15) + 16 * (lane >> 4));
    const uint32_t xrow = smem_u32(xu + (lane & 7 & (MT - 1)) * XS + 16 * (lane >> 3));
    uint4 qh = make_uint4(0, 0, 0, 0);  // Q5_K: qh bytes 4t.. / 16+4t.. of rows g, g+8
    if (TYPE == TYPE_Q5_K) qh = ldsm_x4(wrow + 16);
    int slo[4] = {0, 0, 0, 0}, shi[4] = {0, 0, 0, 0}, mm[4] = {0, 0, 0, 0};
#pragma unroll
    for (int c = 0; c < 4; ++c) {
        const uint4 a = ldsm_x4(wrow + QS + 32 * c);  // row g lo4, row g+8 lo4, row g hi4, row g+8 hi4
        const uint4 xb = ldsm_x4(xrow + 64 * c);      // sub-block 2c (b0, b1), sub-block 2c+1 (b0, b1)
        const uint32_t av[4] = {a.x, a.y, a.z, a.w};
        const uint32_t hv[4] = {qh.x, qh.y, qh.z, qh.w};
        uint32_t al[4], ah[4];
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            if (TYPE == TYPE_Q4_K) {
                al[i] = av[i] & 0x0F0F0F0Fu;
                ah[i] = av[i] & 0xF0F0F0F0u;  // 16 x the high nibble
            } else {
                al[i] = (av[i] & 0x0F0F0F0Fu) | (((hv[i] >> (2 * c)) & 0x01010101u) << 4);
                ah[i] = ((av[i] >> 4) & 0x0F0F0F0Fu) | (((hv[i] >> (2 * c + 1)) & 0x01010101u) << 4);
            }
        }
        int dl[4], dh[4];
        mma_k32_u8s8(dl, al[0], al[1], al[2], al[3], xb.x, xb.y, 0, 0, 0, 0);
        mma_k32_u8s8(dh, ah[0], ah[1], ah[2], ah[3], xb.z, xb.w, 0, 0, 0, 0);
        const int k0 = 2 * (c & 1);
        const uint32_t s0 = sc0[c >> 1], s1 = sc1[c >> 1];
        const int a0l = ubyte(s0, k0), a0h = ubyte(s0, k0 + 1), a1l = ubyte(s1, k0), a1h = ubyte(s1, k0 + 1);
        slo[0] += a0l * dl[0];
        slo[1] += a0l * dl[1];
        slo[2] += a1l * dl[2];
        slo[3] += a1l * dl[3];
        shi[0] += a0h * dh[0];
        shi[1] += a0h * dh[1];
        shi[2] += a1h * dh[2];
        shi[3] += a1h * dh[3];
        const uint32_t n0 = mn0[c >> 1], n1 = mn1[c >> 1];
        const uint32_t r0l = rep_byte(n0, k0), r1l = rep_byte(n1, k0), r0h = rep_byte(n0, k0 + 1),
                       r1h = rep_byte(n1, k0 + 1);
        mma_k32_u8s8(mm, r0l, r1l, r0l, r1l, xb.x, xb.y, mm[0], mm[1], mm[2], mm[3]);
        mma_k32_u8s8(mm, r0h, r1h, r0h, r1h, xb.z, xb.w, mm[0], mm[1], mm[2], mm[3]);
    }
    const float d0 = half_bits_to_float(h0.x), dm0 = half_bits_to_float(h0.x >> 16);
    const float d1 = half_bits_to_float(h1.x), dm1 = half_bits_to_float(h1.x >> 16);
    const float2 dxv = *reinterpret_cast<const float2 *>(dxu + tp);
    float tm[4];
#pragma unroll
    for (int e = 0; e < 4; ++e) {
        const int sumi = (TYPE == TYPE_Q4_K) ? slo[e] + (shi[e] >> 4) : slo[e] + shi[e];
        const float d = (e < 2) ? d0 : d1, dm = (e < 2) ? dm0 : dm1;
        const float dxe = (e & 1) ? dxv.y : dxv.x;
        tm[e] = __fmul_rn(dxe, __fsub_rn(__fmul_rn(d, __int2float_rn(sumi)), __fmul_rn(dm, __int2float_rn(mm[e]))));
        if (db.si) dbg_put(db, g + 8 * (e >> 1), 2 * t + (e & 1), 0, sumi, mm[e]);
    }
    store_terms4<MT>(terms, lane, tm);
}

// Q6_K with m16n8k16 per 16-value sub-block s = 8h + 2g' + hf: ldmatrix gives rows g, g+8 x
// ql[64h + 16hf + 4t..+3] and ql[64h + 32 + 16hf + 4t..+3], another qh[32h + 16hf + 4t..+3];
// the accumulator starts at -32 * (sum of the sub-block's activation quants).
template <int MT>
__device__ __forceinline__ void tile_q6k_mma(const uint8_t *tile, const int8_t *xu, int XS, const float *dxu,
                                             const int *xsu, int lane, float *terms, const DbgOut &db) {
    constexpr int XP = xpitch<MT>();
    const int g = lane >> 2, t = lane & 3, tp = tok_pair<MT>(t);
    const uint4 scA = lds128(tile + 208 * g + 192), scB = lds128(tile + 208 * (g + 8) + 192);
    const uint32_t sa[4] = {scA.x, scA.y, scA.z, scA.w}, sb[4] = {scB.x, scB.y, scB.z, scB.w};
    const uint32_t wrow = smem_u32(tile + 208 * (lane & 15));
    const int col = 32 * (lane >> 4);  // matrices 2, 3: the qlB half
    const uint32_t xrow = smem_u32(xu + (lane & 7 & (MT - 1)) * XS + 32 * (lane >> 3));
    int acc[4] = {0, 0, 0, 0};
#pragma unroll
    for (int hq = 0; hq < 4; ++hq) {
        const int h = hq >> 1, hf = hq & 1;
        const uint4 qv = ldsm_x4(wrow + 64 * h + 16 * hf + col);  // qlA g, qlA g+8, qlB g, qlB g+8
        const uint2 hv = ldsm_x2(wrow + 128 + 32 * h + 16 * hf);   // qh g, qh g+8 (lanes 0-15 give rows)
        const uint4 xv = ldsm_x4(xrow + 128 * h + 16 * hf);        // g' = 0..3 (values 32g' apart)
        const uint32_t xw[4] = {xv.x, xv.y, xv.z, xv.w};
#pragma unroll
        for (int gp = 0; gp < 4; ++gp) {
            const uint32_t la = (gp & 1) ? qv.z : qv.x, lb = (gp & 1) ? qv.w : qv.y;
            uint32_t qa, qb;
            if (gp == 0) {
                qa = (la & 0x0F0F0F0Fu) | ((hv.x << 4) & 0x30303030u);
                qb = (lb & 0x0F0F0F0Fu) | ((hv.y << 4) & 0x30303030u);
            } else if (gp == 1) {
                qa = (la & 0x0F0F0F0Fu) | ((hv.x << 2) & 0x30303030u);
                qb = (lb & 0x0F0F0F0Fu) | ((hv.y << 2) & 0x30303030u);
            } else if (gp == 2) {
                qa = ((la >> 4) & 0x0F0F0F0Fu) | (hv.x & 0x30303030u);
                qb = ((lb >> 4) & 0x0F0F0F0Fu) | (hv.y & 0x30303030u);
            } else {
                qa = ((la >> 4) & 0x0F0F0F0Fu) | ((hv.x >> 2) & 0x30303030u);
                qb = ((lb >> 4) & 0x0F0F0F0Fu) | ((hv.y >> 2) & 0x30303030u);
            }
            const int s = 8 * h + 2 * gp + hf;
            const int2 ci = *reinterpret_cast<const int2 *>(xsu + s * XP + tp);
            int D[4];
            mma_k16_u8s8(D, qa, qb, xw[gp], ci.x, ci.y, ci.x, ci.y);
            const int sA = sbyte(sa[s >> 2], s & 3), sB = sbyte(sb[s >> 2], s & 3);
            acc[0] += sA * D[0];
            acc[1] += sA * D[1];
            acc[2] += sB * D[2];
            acc[3] += sB * D[3];
        }
    }
    const float d0 = half_bits_to_float(*reinterpret_cast<const uint16_t *>(tile + 3328 + 2 * g));
    const float d1 = half_bits_to_float(*reinterpret_cast<const uint16_t *>(tile + 3328 + 2 * (g + 8)));
    const float2 dxv = *reinterpret_cast<const float2 *>(dxu + tp);
    float tm[4];
#pragma unroll
    for (int e = 0; e < 4; ++e) {
        const float d = (e < 2) ? d0 : d1, dxe = (e & 1) ? dxv.y : dxv.x;
        tm[e] = __fmul_rn(__fmul_rn(d, dxe), __int2float_rn(acc[e]));
        if (db.si) dbg_put(db, g + 8 * (e >> 1), 2 * t + (e & 1), 0, acc[e], 0);
    }
    store_terms4<MT>(terms, lane, tm);
}

// Q8_0 with m16n8k32 per 32-block (s8 x s8).
template <int MT>
__device__ __forceinline__ void tile_q80_mma(const uint8_t *tile, const int8_t *xu, int XS, const float *dxu,
                                             int lane, float *terms, int exact, const DbgOut &db) {
    constexpr int XP = xpitch<MT>();
    const int g = lane >> 2, t = lane & 3, tp = tok_pair<MT>(t);
    const uint4 dA = lds128(tile + 272 * g), dB = lds128(tile + 272 * (g + 8));
    const uint32_t da[4] = {dA.x, dA.y, dA.z, dA.w}, dbv[4] = {dB.x, dB.y, dB.z, dB.w};
    const uint32_t wrow = smem_u32(tile + 272 * (lane & 15) + 16 + 16 * (lane >> 4));
    const uint32_t xrow = smem_u32(xu + (lane & 7 & (MT - 1)) * XS + 16 * (lane >> 3));
    float part[4] = {0.0f, 0.0f, 0.0f, 0.0f};
#pragma unroll
    for (int jp = 0; jp < 4; ++jp) {
        const uint4 xb = ldsm_x4(xrow + 64 * jp);  // block 2jp (b0, b1), block 2jp+1 (b0, b1)
#pragma unroll
        for (int hh = 0; hh < 2; ++hh) {
            const int jj = 2 * jp + hh;
            const uint4 a = ldsm_x4(wrow + 32 * jj);
            int D[4];
            mma_k32_s8s8(D, a.x, a.y, a.z, a.w, hh ? xb.z : xb.x, hh ? xb.w : xb.y);
            const float wa = half_bits_to_float(da[jj >> 1] >> (16 * (jj & 1)));
            const float wb = half_bits_to_float(dbv[jj >> 1] >> (16 * (jj & 1)));
            const float2 dxv = *reinterpret_cast<const float2 *>(dxu + jj * XP + tp);
            float tm[4];
            tm[0] = __fmul_rn(__fmul_rn(wa, dxv.x), __int2float_rn(D[0]));
            tm[1] = __fmul_rn(__fmul_rn(wa, dxv.y), __int2float_rn(D[1]));
            tm[2] = __fmul_rn(__fmul_rn(wb, dxv.x), __int2float_rn(D[2]));
            tm[3] = __fmul_rn(__fmul_rn(wb, dxv.y), __int2float_rn(D[3]));
            if (exact) {
                store_terms4<MT>(terms + jj * 16 * MT, lane, tm);
            } else {
#pragma unroll
                for (int e = 0; e < 4; ++e) part[e] = __fadd_rn(part[e], tm[e]);
            }
            if (db.si) {
#pragma unroll
                for (int e = 0; e < 4; ++e) dbg_put(db, g + 8 * (e >> 1), 2 * t + (e & 1), jj, D[e], 0);
            }
        }
    }
    if (!exact) store_terms4<MT>(terms, lane, part);
}

// ------------------------------------------------------------------ row group -> task

__device__ __forceinline__ int task_of_rg(const GemvParams &p, int rg) {
    int t = 0;
#pragma unroll
    for (int i = 1; i < 4; ++i) t += (i < p.n_tasks && rg >= p.task[i].rg_start) ? 1 : 0;
    return t;
}

// Write the finished result of one (row, token).
__device__ __forceinline__ void epilogue(const GemvParams &p, const GemvTaskDev &tk, int r, int tok, float acc,
                                         unsigned long long *s_best) {
    const size_t col = tk.out_ids ? (size_t)tk.out_ids[r] : (size_t)r;
    if (tk.dst_f32) tk.dst_f32[(size_t)tok * tk.f32_stride + col] = acc;
    if (p.peer.n) {
        const unsigned long long st = peer_step(p.peer);
        const size_t o = (size_t)(st & 1ull) * p.peer.buf_stride + (size_t)tok * p.peer.row_stride +
                         (size_t)(p.peer.row0 + r);
#pragma unroll
        for (int q = 0; q < PEER_MAX; ++q)
            if (q < p.peer.n) peer_store(p.peer.buf[q] + o, acc, (uint32_t)st);
    }
    if (tk.dst) {
        float v = acc;
        if (tk.res) v = __fadd_rn(v, __half2float(tk.res[(size_t)tok * tk.res_stride + col]));
        tk.dst[(size_t)tok * tk.dst_stride + col] = __float2half_rn(v);
    }
    if (p.argmax) {
        const float cmp = p.argmax_f16 ? __half2float(__float2half_rn(acc)) : acc;
        atomicMax(&s_best[tok], argmax_key(cmp, (uint32_t)(tk.index_base + r)));
    }
}

// One tile, terms into `tdst` (the unit's term row).
template <int TYPE, int MT>
__device__ __forceinline__ void compute_item(const GemvParams &p, const uint8_t *tile, int u,
                                             const uint8_t *smem, int lane, float *tdst, const DbgOut &db) {
    constexpr int XP = xpitch<MT>();
    const uint8_t *xq = smem + p.off_x;
    const float *dxt = reinterpret_cast<const float *>(smem + p.off_dx);
    const int *aux = reinterpret_cast<const int *>(smem + p.off_xs);
    const int nbu = p.nbu;
    if (use_dp<MT>()) {
        const int XSD = 320 * nbu;
        const uint8_t *xu = xq + 320 * u;
        if (TYPE == TYPE_Q4_K || TYPE == TYPE_Q5_K)
            tile_q45k_dp<TYPE, MT>(tile, xu, XSD, dxt + u * XP, aux + u * 8, nbu * 8, lane, tdst, db);
        else if (TYPE == TYPE_Q6_K)
            tile_q6k_dp<MT>(tile, xu, XSD, dxt + u * XP, aux + u * 16 * MT, lane, tdst, db);
        else
            tile_q80_dp<MT>(tile, xu, XSD, dxt + u * 8 * XP, lane, tdst, p.q80_exact, db);
    } else {
        const int XS = p.K + 16;
        const int8_t *xu = reinterpret_cast<const int8_t *>(xq) + 256 * u;
        if (TYPE == TYPE_Q4_K || TYPE == TYPE_Q5_K)
            tile_q45k_mma<TYPE, MT>(tile, xu, XS, dxt + u * XP, lane, tdst, db);
        else if (TYPE == TYPE_Q6_K)
            tile_q6k_mma<MT>(tile, xu, XS, dxt + u * XP, aux + u * 16 * XP, lane, tdst, db);
        else
            tile_q80_mma<MT>(tile, xu, XS, dxt + u * 8 * XP, lane, tdst, p.q80_exact, db);
    }
}

__device__ __forceinline__ DbgOut make_dbg(const GemvParams &p, const GemvTaskDev &tk, int rg, int u, int is_q80) {
    DbgOut db;
    db.si = tk.dbg_sumi;
    db.sm = tk.dbg_summ;
    db.r0 = (tk.rg_first + rg - tk.rg_start) * 16 - tk.row_begin;
    db.rows = tk.rows;
    db.bpr = is_q80 ? p.nbu * 8 : p.nbu;
    db.blk0 = is_q80 ? u * 8 : u;
    db.M = p.M;
    return db;
}

// Sum the block terms of one (row, token) of local row group lr in order and write it.
template <int MT>
__device__ __forceinline__ void fold_one(const GemvParams &p, const GemvTaskDev *tasks, const float *tb, int J, int e,
                                         int rg, unsigned long long *s_best) {
    const int rr = e / MT, tok = e - rr * MT;
    const GemvTaskDev &tk = tasks[task_of_rg(p, rg)];
    const int r = (tk.rg_first + rg - tk.rg_start) * 16 + rr - tk.row_begin;
    if (tok >= p.M || r < 0 || r >= tk.rows) return;
    constexpr int ST = 16 * MT;
    float acc = 0.0f;
    int j = 0;
    for (; j + 4 <= J; j += 4) {
        const float a0 = tb[(j + 0) * ST + e], a1 = tb[(j + 1) * ST + e];
        const float a2 = tb[(j + 2) * ST + e], a3 = tb[(j + 3) * ST + e];
        acc = __fadd_rn(__fadd_rn(__fadd_rn(__fadd_rn(acc, a0), a1), a2), a3);
    }
    for (; j < J; ++j) acc = __fadd_rn(acc, tb[j * ST + e]);
    epilogue(p, tk, r, tok, acc, s_best);
}

// Row group rg is shared with other CTAs (split launch): store this CTA's block terms (units
// [ua, ub), smem term block tb of J x 16 MT floats) in the row group's global slot -- indexed by
// the CTA that holds its first tile, which holds no other shared row group's first tile -- and
// count the arrival.  The CTA that arrives last copies the other CTAs' terms into tb (16-byte
// copies through L2, all in flight), calls fold_e(e) for every (row, token) e of the row group
// (which adds the J terms in block order and writes the result), clears the count for the next
// launch and returns true.  No CTA waits for another.  One warp.
// The split space is T tiles owned in equal ranges by the grid's CTAs; the row group's first tile
// is tile `first` of it.
template <int MT, class FoldE>
__device__ __forceinline__ bool fold_shared_f(const GemvParams &p, float *tb, int J, int JU, int ua, int ub,
                                              long long first, long long T, int lane, FoldE fold_e) {
    constexpr int E = 16 * MT;  // floats per term (16 rows x MT tokens): a multiple of 4
    const long long G = gridDim.x;
    const int c_first = (int)(((first + 1) * G - 1) / T);     // CTA owning tile `first`
    const int c_last = (int)(((first + p.nbu) * G - 1) / T);  // CTA owning the row group's last tile
    float4 *g4 = reinterpret_cast<float4 *>(p.gterms + (size_t)c_first * J * E);
    const float4 *t4 = reinterpret_cast<const float4 *>(tb);
    const int k0 = ua * JU * E / 4, k1 = ub * JU * E / 4, kn = J * E / 4;
    for (int k = k0 + lane; k < k1; k += 32) __stcg(g4 + k, t4[k]);
    __threadfence();
    __syncwarp();
    int last = 0;
    if (lane == 0) last = atomicAdd(&p.gcount[c_first], 1) == c_last - c_first;
    last = __shfl_sync(0xffffffffu, last, 0);
    if (!last) return false;
    __threadfence();
    const uint32_t tbs = smem_u32(tb);
    for (int k = lane; k < kn; k += 32)
        if (k < k0 || k >= k1) cp_async16_cg(tbs + 16u * (uint32_t)k, g4 + k);
    cp_async_wait_all();
    __syncwarp();
    for (int e = lane; e < E; e += 32) fold_e(e);
    __syncwarp();
    if (lane == 0) p.gcount[c_first] = 0;
    return true;
}

template <int MT>
__device__ __forceinline__ void fold_shared(const GemvParams &p, const GemvTaskDev *tasks, float *tb, int J, int JU,
                                            int ua, int ub, int rg, int lane, unsigned long long *s_best) {
    fold_shared_f<MT>(p, tb, J, JU, ua, ub, (long long)rg * p.nbu, p.total_tiles, lane,
                      [&](int e) { fold_one<MT>(p, tasks, tb, J, e, rg, s_best); });
}

}  // namespace kq
