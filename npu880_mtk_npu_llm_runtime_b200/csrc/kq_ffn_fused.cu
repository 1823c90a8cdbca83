// kq_ffn_fused.cu -- the FFN block for 1-2 tokens as one persistent kernel.
//
// Replaces, for decode and small tree-verify batches, the engine's FFN sequence
// (ENG:8283-8298: RMSNorm -> Q8_K -> gate / up -> SwiGLU -> Q8_K -> down + residual) that the
// NPU adapter ran as one graph (run_real_npu_universal_ffn, TV:682-761).  Results are bit for bit
// those of the four-launch form (kq_run_ffn_async with the option "ffn_fused" = 0), which are
// the reference's.
//
// One CTA per SM, all resident at once (the shared memory plan leaves room for one CTA per SM
// and the grid is the SM count).  Warp W streams the CTA's weight tiles -- first its gate/up
// share, then its down share -- through one ring of stages with cp.async.bulk from the moment
// the CTA starts, so the down weights arrive while gate/up is computed.  Consumer warps 0..W-1:
//  1. stage the input rows, the sequential fp32 sum of squares of each row (rms_seq_sum, teams
//     of 5 warps), normalize, quantize to Q8_K into the gate/up activation (every CTA for
//     itself: no exchange);
//  2. gate/up: the row groups of gate and up alternate (gate rows 16 w.., up rows 16 w.., gate
//     rows 16 (w+1).., ...) and each CTA owns whole pairs (gate w, up w) (ffn_share); the warp
//     completing a row group folds it in unit order; outputs go to global memory in fp16, then the
//     CTA computes SwiGLU of its pairs (ENG:4350-4356, the same exp table as kq_swiglu_q8k) in place
//     of g -- each value once;
//  3. one grid-wide barrier (bounded wait; an arrival count and a generation word);
//  4. Q8_K of all of h into the down activation (every CTA for itself);
//  5. down + residual, shared out and folded like 2.
// Every wait is bounded; on a timeout the kernel records DEV_ERR_TIMEOUT, stops issuing and
// computing, drains its own copies in flight (bounded) and returns.
#include "kq_gemv_dev.cuh"
#include "kq_internal.h"
#include "kq_rms_seq.cuh"

#include <algorithm>
#include <mutex>
#include <unordered_map>

namespace kq {

constexpr int FFN_TEAM_WARPS = RMS_MIN_THREADS / 32;  // warps per RMSNorm row team

struct FfnFusedParams {
    GemvParams pa;  // gate/up (row groups alternating); activation = Q8_K of the normalized rows
    GemvParams pb;  // down (task 0) with the residual; activation = Q8_K of SwiGLU(g, u)
    const uint8_t *wg, *wu;  // tiled gate / up weights
    const __half *x;         // [M][hidden] block input (the residual too)
    const __half *gamma;     // [hidden]
    __half *g, *u;           // [M][ffn] gate / up outputs; SwiGLU overwrites g with h
    const float *exp_tab;    // expf(-g) per fp16 pattern, or nullptr (fp64 exp)
    unsigned *gbar;          // [2] grid barrier: arrivals, generation
    int *pair;               // [ffn / 16] folds done of (gate w, up w), back to 0 after use
    int hidden, ffn, M;
    unsigned off_rows, off_hsum, off_desc;  // phase 1 scratch (inside the down activation)
    unsigned off_stages, off_bars;
    unsigned stage_bytes;
    int S, TA, TB;  // ring stages, tiles per stage of each phase
    int *status;
    unsigned long long timeout_ns;
};

// This CTA's share of a phase's tiles, as two runs done in this order:
//  run 0: an equal range of a split space of row groups (tiles xs .. xs + xt of the phase), whose
//         row groups neighbouring CTAs share and fold with fold_shared_f (the last to finish adds
//         all block terms in unit order; nobody waits);
//  run 1: whole groups of `gran` row groups.
// Gate/up (gran 2: a pair (gate w, up w), so every SwiGLU pair is local) is whole pairs only,
// spread as evenly as whole pairs allow (608 pairs: 4 or 5 per CTA).  Down (gran 1) gives every
// CTA the same number of whole row groups and splits the remaining row groups (160 = 148 + 12 at
// hidden 2,560) over all CTAs, computed first so that their folds across CTAs happen while the
// CTA's own row groups are computed.  Splitting the 16 remaining gate/up pairs the same way was
// slower (32.6 against 30.2 us per block at 1 token): their 10-unit row groups spread over 4-5
// CTAs each, and the folds and pair counts across CTAs cost more than the uneven pairs.  Measured: whole row groups beat equal tile
// ranges, whose folds through L2 sat at the end of every CTA; the 12 CTAs holding two down row
// groups then set the end of the launch, hence the split remainder.
struct FfnShare {
    long long xs, xt;   // split space: first phase tile, tiles
    int x0, nx;         // this CTA's split tiles [x0, x0 + nx) of the space
    int rgx_lo, nlx;    // row groups run 0 touches
    int rg1, n1;        // whole row groups of run 1
    int n, n_lr;        // tiles, row groups (term slots: run 0's first)
};

__device__ __forceinline__ FfnShare ffn_share(const GemvParams &p, int gran, bool split_rest) {
    FfnShare s;
    const long long groups = p.total_rg / gran, G = gridDim.x, c = blockIdx.x;
    long long whole, g_lo;
    if (split_rest) {
        whole = groups / G;  // whole groups per CTA, the same for all
        g_lo = whole * c;
        s.xs = whole * G * gran * p.nbu;
        s.xt = (groups - whole * G) * gran * p.nbu;
    } else {
        g_lo = groups * c / G;
        whole = groups * (c + 1) / G - g_lo;
        s.xs = 0;
        s.xt = 0;
    }
    s.rg1 = (int)(g_lo * gran);
    s.n1 = (int)(whole * gran);
    const long long xa = s.xt * c / G, xb = s.xt * (c + 1) / G;
    s.x0 = (int)xa;
    s.nx = (int)(xb - xa);
    s.rgx_lo = (int)((s.xs + xa) / p.nbu);
    s.nlx = s.nx > 0 ? (int)((s.xs + xb + p.nbu - 1) / p.nbu) - s.rgx_lo : 0;
    s.n = s.nx + s.n1 * p.nbu;
    s.n_lr = s.nlx + s.n1;
    return s;
}

// local tile i of the share -> phase tile index
__device__ __forceinline__ long long ffn_tile(const FfnShare &s, int i, int nbu) {
    return i < s.nx ? s.xs + s.x0 + i : (long long)s.rg1 * nbu + (i - s.nx);
}

// term slot of row group rg, and its units [ua, ub) owned by this CTA
__device__ __forceinline__ void ffn_slot(const FfnShare &s, int nbu, int rg, bool split, int &lr, int &ua, int &ub) {
    if (split) {
        lr = rg - s.rgx_lo;
        const long long b0 = (long long)rg * nbu;
        ua = (int)max(0ll, s.xs + s.x0 - b0);
        ub = (int)min((long long)nbu, s.xs + s.x0 + s.nx - b0);
    } else {
        lr = s.nlx + (rg - s.rg1);
        ua = 0;
        ub = nbu;
    }
}

// Grid-wide barrier of the grid's CTAs (all resident), one thread per CTA.  Arrival is a release
// (this CTA's earlier writes are published), the last arrival acquires all of them, clears the
// count for the next launch and publishes a new generation, which the others wait for with
// acquire loads.  Bounded: false on timeout.
__device__ __forceinline__ bool ffn_grid_barrier(unsigned *gbar, unsigned long long timeout_ns, int *status) {
    unsigned gen, old;
    asm volatile("ld.relaxed.gpu.global.u32 %0, [%1];" : "=r"(gen) : "l"(gbar + 1) : "memory");
    asm volatile("atom.acq_rel.gpu.global.add.u32 %0, [%1], 1;" : "=r"(old) : "l"(gbar) : "memory");
    if (old == gridDim.x - 1) {
        asm volatile("st.relaxed.gpu.global.u32 [%0], %1;" ::"l"(gbar), "r"(0u) : "memory");
        asm volatile("st.release.gpu.global.u32 [%0], %1;" ::"l"(gbar + 1), "r"(gen + 1u) : "memory");
        return true;
    }
    const unsigned long long t0 = global_timer_ns();
    while (true) {
        for (int i = 0; i < 32; ++i) {
            unsigned v;
            asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(gbar + 1) : "memory");
            if (v != gen) return true;
        }
        if (global_timer_ns() - t0 > timeout_ns) {
            report_error(status, DEV_ERR_TIMEOUT);
            return false;
        }
    }
}

__device__ __forceinline__ uint4 ffn_load8(const __half *p) {
    if ((reinterpret_cast<uintptr_t>(p) & 15) == 0) return *reinterpret_cast<const uint4 *>(p);
    uint32_t hv[8];
#pragma unroll
    for (int k = 0; k < 8; ++k) hv[k] = __half_as_ushort(p[k]);
    return make_uint4(hv[0] | (hv[1] << 16), hv[2] | (hv[3] << 16), hv[4] | (hv[5] << 16), hv[6] | (hv[7] << 16));
}

// SwiGLU of one fp16 pair, the reference's scalar operation order (ENG:4350-4356) with the exp
// table of kq_swiglu_q8k.
__device__ __forceinline__ uint16_t ffn_swiglu1(uint16_t gb, uint16_t ub, const float *exp_tab) {
    const float gf = __half2float(__ushort_as_half(gb)), uf = __half2float(__ushort_as_half(ub));
    const float e = exp_tab ? __ldg(exp_tab + gb) : (float)exp(-(double)gf);
    return __half_as_ushort(__float2half_rn(__fmul_rn(__fdiv_rn(gf, __fadd_rn(1.0f, e)), uf)));
}

// h = SwiGLU(g, u) of the 16 rows of pair w in place of g (all M tokens), by one warp.
__device__ __forceinline__ void ffn_swiglu_rows(const FfnFusedParams &P, int w, int lane) {
    for (int e = lane; e < 16 * P.M; e += 32) {
        const size_t o = (size_t)(e >> 4) * P.ffn + w * 16 + (e & 15);
        const uint16_t gb = __ldcg(reinterpret_cast<const unsigned short *>(P.g) + o);
        const uint16_t ub = __ldcg(reinterpret_cast<const unsigned short *>(P.u) + o);
        reinterpret_cast<unsigned short *>(P.g)[o] = ffn_swiglu1(gb, ub, P.exp_tab);
    }
}

// Fold element e = (row rr, token) of gate/up row group q: the J block terms in block order.
template <int MT>
__device__ __forceinline__ void ffn_fold_a(const FfnFusedParams &P, const float *tb, int J, int e, int q) {
    const int rr = e / MT, tok = e - rr * MT;
    if (tok >= P.M) return;
    constexpr int ST = 16 * MT;
    float acc = 0.0f;
    for (int j = 0; j < J; ++j) acc = __fadd_rn(acc, tb[j * ST + e]);
    __half *dst = (q & 1) ? P.u : P.g;
    dst[(size_t)tok * P.ffn + (q >> 1) * 16 + rr] = __float2half_rn(acc);
}

// The tiles of one phase (a GEMV over the CTA's share): warp w takes tiles w, w + W, ...; a tile's
// stage is st0 + i / T.  Each tile is released to the ring with `other` arrivals (the other
// phase's tiles per stage: every stage then counts TA x TB), a partial stage's missing tiles by its
// first tile.  The warp that completes a row group folds it (fold_shared_f when another CTA holds
// some of its units); in phase A, s_fin[lr] marks the row groups whose final fold this CTA made.
template <int TYPE, int MT, bool PHASE_A>
__device__ __forceinline__ void ffn_phase(const FfnFusedParams &P, const GemvParams &p, const FfnShare &sh,
                                          const GemvTaskDev *tasks, int *s_done, int *s_fin, int st0, int T, int other,
                                          uint8_t *smem, uint8_t *ring, uint64_t *bars, float *terms, int *s_issued,
                                          int *s_abort, unsigned long long *s_best, int warp, int lane) {
    constexpr int W = warps_of<MT>();
    constexpr int E = 16 * MT;
    const int S = P.S, nbu = p.nbu, J = p.terms_per_rg;
    for (int i = warp; i < sh.n; i += W) {
        if (*reinterpret_cast<volatile int *>(s_abort)) break;
        const int k = i / T, st = st0 + k, tt = i - k * T, slot = st % S;
        int ok = 1;
        if (lane == 0)
            ok = wait_ge_bounded(s_issued, st + 1, P.timeout_ns, P.status) &&
                 mbar_wait_bounded(smem_u32(&bars[slot]), (uint32_t)((st / S) & 1), P.timeout_ns, P.status);
        ok = __shfl_sync(0xffffffffu, ok, 0);
        if (!ok) {
            if (lane == 0) *reinterpret_cast<volatile int *>(s_abort) = 1;
            break;
        }
        const long long tau = ffn_tile(sh, i, nbu);
        const int rg = (int)(tau / nbu), u = (int)(tau - (long long)rg * nbu);
        const bool split = i < sh.nx;
        int lr, ua, ub;
        ffn_slot(sh, nbu, rg, split, lr, ua, ub);
        const uint8_t *tile = ring + (size_t)slot * P.stage_bytes + (size_t)tt * p.tile_bytes;
        DbgOut db;
        db.si = nullptr;
        float *tb = terms + (size_t)lr * J * E;
        compute_item<TYPE, MT>(p, tile, u, smem, lane, tb + (size_t)u * E, db);
        __syncwarp();
        int last = 0;
        if (lane == 0) {
            const int n_in = min(sh.n - k * T, T);  // tiles of this stage
            mbar_arrive_cnt(smem_u32(&bars[S + slot]), (uint32_t)(other + (tt == 0 ? (T - n_in) * other : 0)));
            __threadfence_block();
            last = atomicAdd(&s_done[lr], 1) == ub - ua - 1;
        }
        last = __shfl_sync(0xffffffffu, last, 0);
        if (last) {
            __threadfence_block();
            const bool shared = ua > 0 || ub < nbu;
            const long long first = (long long)rg * nbu - sh.xs;  // the row group's first tile in the split space
            if (PHASE_A) {
                bool done = true;
                if (shared)
                    done = fold_shared_f<MT>(p, tb, J, 1, ua, ub, first, sh.xt, lane,
                                             [&](int e) { ffn_fold_a<MT>(P, tb, J, e, rg); });
                else
                    for (int e = lane; e < E; e += 32) ffn_fold_a<MT>(P, tb, J, e, rg);
                if (done && lane == 0) s_fin[lr] = 1;  // this CTA made the row group's final fold
            } else {
                if (shared)
                    fold_shared_f<MT>(p, tb, J, 1, ua, ub, first, sh.xt, lane,
                                      [&](int e) { fold_one<MT>(p, tasks, tb, J, e, rg, s_best); });
                else
                    for (int e = lane; e < E; e += 32) fold_one<MT>(p, tasks, tb, J, e, rg, s_best);
            }
        }
    }
}

template <int GT, int DT, int MT>
__global__ void __launch_bounds__(threads_of<MT>(), 1) kq_ffn_fused(const __grid_constant__ FfnFusedParams P) {
    extern __shared__ __align__(128) uint8_t smem[];
    __shared__ unsigned long long s_best[8];  // fold_one's argmax keys (no argmax here)
    __shared__ int s_abort, s_issued;
    __shared__ int s_done_a[kMaxTermSlots], s_done_b[kMaxTermSlots], s_fin[kMaxTermSlots];
    __shared__ float s_inv[8];
    __shared__ GemvTaskDev s_tb[1];

    const GemvParams &pa = P.pa, &pb = P.pb;
    constexpr int W = warps_of<MT>();
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int S = P.S;
    uint8_t *ring = smem + P.off_stages;
    uint64_t *bars = reinterpret_cast<uint64_t *>(smem + P.off_bars);  // full[S], empty[S]
    float *terms = reinterpret_cast<float *>(smem + pa.off_terms);
    const FfnShare sa = ffn_share(pa, 2, false), sb = ffn_share(pb, 1, true);
    const int na_st = (sa.n + P.TA - 1) / P.TA, nb_st = (sb.n + P.TB - 1) / P.TB, n_st = na_st + nb_st;

    if (tid == 0) s_tb[0] = pb.task[0];
    if (tid < 8) s_best[tid] = 0ull;
    if (tid < kMaxTermSlots) {
        s_done_a[tid] = 0;
        s_done_b[tid] = 0;
        s_fin[tid] = 0;
    }
    if (tid == 0) {
        for (int s = 0; s < S; ++s) {
            mbar_init(smem_u32(&bars[s]), 1);
            mbar_init(smem_u32(&bars[S + s]), (uint32_t)(P.TA * P.TB));
        }
        s_abort = 0;
        s_issued = 0;
        mbar_init_fence();
    }
    __syncthreads();

    if (warp == W) {
        // ---------------- producer: gate/up tiles, then down tiles, through one ring
        if (lane == 0) {
            const uint64_t policy = l2_evict_first_policy();
            for (int s = 0; s < n_st; ++s) {
                const int slot = s % S;
                if (s >= S &&
                    !mbar_wait_bounded_sleep(smem_u32(&bars[S + slot]), (uint32_t)(((s / S) - 1) & 1), P.timeout_ns,
                                             P.status)) {
                    s_abort = 1;
                    break;
                }
                if (*reinterpret_cast<volatile int *>(&s_abort)) break;
                const bool ph_a = s < na_st;
                const GemvParams &p = ph_a ? pa : pb;
                const FfnShare &sh = ph_a ? sa : sb;
                const int T = ph_a ? P.TA : P.TB;
                const int a = (ph_a ? s : s - na_st) * T, b = min(sh.n, a + T);
                const uint32_t full = smem_u32(&bars[slot]);
                const uint32_t sdst = smem_u32(ring + (size_t)slot * P.stage_bytes);
                mbar_arrive_expect_tx(full, (uint32_t)(b - a) * p.tile_bytes);
                int i = a;
                while (i < b) {
                    // a copy stays inside one run (split / whole) and, for gate/up, one row group
                    const long long tau = ffn_tile(sh, i, p.nbu);
                    const int rg = (int)(tau / p.nbu);
                    int iend = (i < sh.nx) ? min(b, sh.nx) : b;
                    const uint8_t *src;
                    if (ph_a) {
                        // gate/up row group rg: weight row group rg / 2 of gate (even) or up (odd)
                        src = ((rg & 1) ? P.wu : P.wg) + ((size_t)(rg >> 1) * p.nbu + (size_t)(tau - (long long)rg * p.nbu)) * p.tile_bytes;
                        iend = min(iend, i + (int)((long long)(rg + 1) * p.nbu - tau));
                    } else {
                        src = p.task[0].w + (size_t)tau * p.tile_bytes;
                    }
                    bulk_g2s(sdst + (uint32_t)(i - a) * p.tile_bytes, src, (uint32_t)(iend - i) * p.tile_bytes, full,
                             policy);
                    i = iend;
                }
                *reinterpret_cast<volatile int *>(&s_issued) = s + 1;
            }
        }
    } else {
        pdl_wait();  // the block input may come from the previous kernel
        const int M = P.M, K = P.hidden, nbh = K / 256, nh = K / 128;
        // ---------------- 1. RMSNorm + Q8_K into the gate/up activation
        __half *rows = reinterpret_cast<__half *>(smem + P.off_rows);  // [M][K]
        float *hsum = reinterpret_cast<float *>(smem + P.off_hsum);    // [M][K / 128]
        uint4 *desc = reinterpret_cast<uint4 *>(smem + P.off_desc);    // [teams][RMS_MAX_SEG * 4]
        for (int i = warp; i < M * nbh; i += W) {
            const int m = i / nbh, u = i - m * nbh;
            const uint4 raw = ffn_load8(P.x + (size_t)m * K + u * 256 + 8 * lane);
            *reinterpret_cast<uint4 *>(rows + (size_t)m * K + u * 256 + 8 * lane) = raw;
            const __half2 *h2 = reinterpret_cast<const __half2 *>(&raw);
            float h = 0.0f;
#pragma unroll
            for (int k = 0; k < 4; ++k) {
                const float2 v = __half22float2(h2[k]);
                h += v.x * v.x + v.y * v.y;  // an estimate: any order
            }
#pragma unroll
            for (int o = 8; o > 0; o >>= 1) h += __shfl_xor_sync(0xffffffffu, h, o);
            if ((lane & 15) == 0) hsum[m * nh + 2 * u + (lane >> 4)] = h;
        }
        named_bar_sync(1, W * 32);
        {
            const int team = warp / FFN_TEAM_WARPS, n_teams = W / FFN_TEAM_WARPS;
            if (team < n_teams) {
                const int ttid = tid - team * FFN_TEAM_WARPS * 32;
                auto tbar = [team] { named_bar_sync(2 + team, FFN_TEAM_WARPS * 32); };
                for (int m = team; m < M; m += n_teams) {
                    const float ss = rms_seq_sum(RmsSqF16{rows + (size_t)m * K}, hsum + m * nh,
                                                 desc + team * RMS_MAX_SEG * 4, K, ttid, tbar);
                    if (ttid == 0) {
                        const float inv_k = __fdiv_rn(1.0f, (float)K);
                        s_inv[m] = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fmul_rn(ss, inv_k), 1.0e-6f)));
                    }
                    tbar();  // the team's descriptors are rewritten for its next row
                }
            }
        }
        named_bar_sync(1, W * 32);
        for (int i = warp; i < M * nbh; i += W) {
            const int m = i / nbh, u = i - m * nbh;
            const int base = u * 256 + 8 * lane;
            const uint4 graw = ffn_load8(P.gamma + base);
            const uint4 xraw = *reinterpret_cast<const uint4 *>(rows + (size_t)m * K + base);
            const __half2 *g2 = reinterpret_cast<const __half2 *>(&graw);
            const __half2 *x2 = reinterpret_cast<const __half2 *>(&xraw);
            const float inv = s_inv[m];
            uint32_t packed[4];
#pragma unroll
            for (int k = 0; k < 4; ++k) {
                const float2 xv = __half22float2(x2[k]), gv = __half22float2(g2[k]);
                const __half h0 = __float2half_rn(__fmul_rn(__fmul_rn(xv.x, inv), gv.x));
                const __half h1 = __float2half_rn(__fmul_rn(__fmul_rn(xv.y, inv), gv.y));
                packed[k] = (uint32_t)__half_as_ushort(h0) | ((uint32_t)__half_as_ushort(h1) << 16);
            }
            uint32_t lo, hi;
            float d;
            quantize_lane<GT>(make_uint4(packed[0], packed[1], packed[2], packed[3]), lo, hi, d);
            store_act_unit<GT, MT>(pa, smem, m, u, lane, lo, hi, d, 0, true);
        }
        named_bar_sync(1, W * 32);

        // ---------------- 2. gate / up (and SwiGLU of each completed pair)
        ffn_phase<GT, MT, true>(P, pa, sa, nullptr, s_done_a, s_fin, 0, P.TA, P.TB, smem, ring, bars, terms,
                                &s_issued, &s_abort, s_best, warp, lane);
        named_bar_sync(1, W * 32);  // this CTA's g, u rows are written
        // SwiGLU of every pair (gate w, up w) whose two final folds this CTA made; a pair whose
        // folds were made by two CTAs is counted in P.pair[w] and computed by the second
        for (int lr = warp; lr < sa.n_lr; lr += W) {
            if (!s_fin[lr]) continue;
            const int q = lr < sa.nlx ? sa.rgx_lo + lr : sa.rg1 + (lr - sa.nlx), pq = q ^ 1;
            const int plr = (pq >= sa.rg1 && pq < sa.rg1 + sa.n1) ? sa.nlx + (pq - sa.rg1)
                            : (pq >= sa.rgx_lo && pq < sa.rgx_lo + sa.nlx) ? pq - sa.rgx_lo : -1;
            const bool local = plr >= 0 && s_fin[plr];
            int mine;
            if (local) {
                mine = (q & 1) == 0;
            } else {
                mine = 0;
                if (lane == 0) {
                    __threadfence();  // this CTA's g, u rows before the count (cumulative over the barrier)
                    mine = atomicAdd(&P.pair[q >> 1], 1) == 1;
                    if (mine) __threadfence();
                }
                mine = __shfl_sync(0xffffffffu, mine, 0);
            }
            if (mine) {
                ffn_swiglu_rows(P, q >> 1, lane);
                if (!local && lane == 0) P.pair[q >> 1] = 0;  // ready for the next launch
            }
        }
        named_bar_sync(1, W * 32);

        // ---------------- 3. grid-wide barrier (every CTA arrives, even after an early stop, so
        // that the others are not held up)
        if (tid == 0 && !ffn_grid_barrier(P.gbar, P.timeout_ns, P.status)) s_abort = 1;
        named_bar_sync(1, W * 32);
        pdl_launch_dependents();  // every CTA of this grid is resident: the next grid may come in

        // ---------------- 4. Q8_K of h (ENG:4357) into the down activation
        const int F = P.ffn, nbf = F / 256;
        if (!*reinterpret_cast<volatile int *>(&s_abort)) {
            for (int i = warp; i < M * nbf; i += W) {
                const int m = i / nbf, u = i - m * nbf;
                const uint4 hraw = __ldcg(reinterpret_cast<const uint4 *>(P.g + (size_t)m * F + (size_t)u * 256 + 8 * lane));
                uint32_t lo, hi;
                float d;
                quantize_lane<DT>(hraw, lo, hi, d);
                store_act_unit<DT, MT>(pb, smem, m, u, lane, lo, hi, d, 0, true);
            }
        }
        named_bar_sync(1, W * 32);

        // ---------------- 5. down + residual
        ffn_phase<DT, MT, false>(P, pb, sb, s_tb, s_done_b, nullptr, na_st, P.TB, P.TA, smem, ring, bars, terms,
                                 &s_issued, &s_abort, s_best, warp, lane);
    }
    __syncthreads();
    // drain after an early stop: copies of the last S issued stages may still be in flight
    if (tid == 0 && s_abort) {
        const int issued = s_issued;
        for (int s = max(0, issued - S); s < issued; ++s)
            mbar_wait_bounded(smem_u32(&bars[s % S]), (uint32_t)((s / S) & 1), P.timeout_ns, P.status);
    }
}

// ------------------------------------------------------------------ host launcher

namespace {

unsigned ffn_al(size_t v) { return (unsigned)((v + 127) / 128 * 128); }

struct FfnPlan {
    bool ok = false;
    int TA = 0, TB = 0, S = 0;
    unsigned stage = 0, a_x = 0, a_dx = 0, a_xs = 0, b_x = 0, b_dx = 0, b_xs = 0;
    unsigned rows = 0, hsum = 0, desc = 0, terms = 0, stages = 0, bars = 0, smem = 0;
};

// Shared memory of one CTA: gate/up activation | down activation (phase 1's rows, estimates and
// descriptors live there until SwiGLU overwrites them) | block terms of the larger share | ring of
// S stages of >= 16 KB (TA gate/up tiles or TB down tiles) | 2 S mbarriers.
FfnPlan ffn_plan(int gt, int dt, int hidden, int ffn, int MT, int grid) {
    FfnPlan pl;
    const int nbh = hidden / 256, nbf = ffn / 256, XP = MT < 2 ? 2 : MT;
    const unsigned xa = ffn_al((size_t)MT * 320 * nbh), dxa = ffn_al((size_t)nbh * XP * 4),
                   xsa = ffn_al((size_t)MT * nbh * 8 * 4);
    const unsigned xb = ffn_al((size_t)MT * 320 * nbf), dxb = ffn_al((size_t)nbf * XP * 4),
                   xsb = dt == TYPE_Q6_K ? ffn_al((size_t)nbf * 16 * MT * 4) : ffn_al((size_t)MT * nbf * 8 * 4);
    const int n_teams = warps_of<1>() / (RMS_MIN_THREADS / 32);
    const unsigned rows = ffn_al((size_t)MT * hidden * 2), hs = ffn_al((size_t)MT * (hidden / 128) * 4),
                   desc = ffn_al((size_t)n_teams * RMS_MAX_SEG * 4 * 16);
    const unsigned act_a = xa + dxa + xsa, region_b = std::max(xb + dxb + xsb, rows + hs + desc);
    const long long rg_f = ffn / 16, rg_h = hidden / 16;
    // whole pairs of gate/up row groups and whole down row groups per CTA
    const long long rga = 2 * ((rg_f + grid - 1) / grid);  // whole gate/up pairs
    // down: the same whole row groups everywhere, plus a range of the split remainder
    const long long whole_b = rg_h / grid, per_x = ((rg_h - whole_b * grid) * nbf + grid - 1) / grid;
    const long long rgb = whole_b + (per_x > 0 ? (per_x + nbf - 2) / nbf + 1 : 0);
    if (rga > kMaxTermSlots || rgb > kMaxTermSlots) return pl;
    const unsigned terms = ffn_al((size_t)std::max(rga * nbh, rgb * nbf) * 16 * MT * 4);
    const unsigned tba = (unsigned)tile_bytes(gt), tbb = (unsigned)tile_bytes(dt);
    pl.TA = (int)((16384 + tba - 1) / tba);
    pl.TB = (int)((16384 + tbb - 1) / tbb);
    pl.stage = ffn_al(std::max(pl.TA * tba, pl.TB * tbb));
    const unsigned fixed = act_a + region_b + terms;
    const unsigned budget = 220u * 1024u;
    if (fixed + 2 * (pl.stage + 16) > budget) return pl;
    pl.S = (int)std::min<unsigned>(64u, (budget - fixed) / (pl.stage + 16));
    pl.a_x = 0;
    pl.a_dx = xa;
    pl.a_xs = xa + dxa;
    pl.b_x = act_a;
    pl.b_dx = act_a + xb;
    pl.b_xs = act_a + xb + dxb;
    pl.rows = act_a;
    pl.hsum = act_a + rows;
    pl.desc = act_a + rows + hs;
    pl.terms = act_a + region_b;
    pl.stages = pl.terms + terms;
    pl.bars = pl.stages + pl.S * pl.stage;
    pl.smem = pl.bars + 2 * pl.S * 8;
    pl.ok = true;
    return pl;
}

GemvTaskDev ffn_task(const uint8_t *w, int rows, void *dst, long long dst_stride, const void *res,
                     long long res_stride, int rg_start) {
    GemvTaskDev d{};
    d.w = w;
    d.rg_first = 0;
    d.n_rg = (rows + 15) / 16;
    d.rg_start = rg_start;
    d.row_begin = 0;
    d.rows = rows;
    d.dst = reinterpret_cast<__half *>(dst);
    d.dst_stride = dst_stride;
    d.res = reinterpret_cast<const __half *>(res);
    d.res_stride = res_stride;
    return d;
}

template <int GT, int DT, int MT>
cudaError_t launch_ffn_t(const FfnFusedLaunch &L, const FfnPlan &pl, cudaStream_t stream) {
    FfnFusedParams P{};
    const int nbh = L.hidden / 256, nbf = L.ffn / 256;
    GemvParams &a = P.pa;  // gate/up row groups alternate: row group q is rows 16 (q / 2).. of gate or up
    a.n_tasks = 0;
    a.total_rg = 2 * (L.ffn / 16);
    a.K = L.hidden;
    a.nbu = nbh;
    a.terms_per_rg = nbh;
    a.off_x = pl.a_x;
    a.off_dx = pl.a_dx;
    a.off_xs = pl.a_xs;
    a.tile_bytes = (unsigned)tile_bytes(GT);
    GemvParams &b = P.pb;
    b.task[0] = ffn_task(L.down, L.hidden, L.y, L.hidden, L.x, L.hidden, 0);
    b.n_tasks = 1;
    b.total_rg = L.hidden / 16;
    b.K = L.ffn;
    b.nbu = nbf;
    b.terms_per_rg = nbf;
    b.off_x = pl.b_x;
    b.off_dx = pl.b_dx;
    b.off_xs = pl.b_xs;
    b.tile_bytes = (unsigned)tile_bytes(DT);
    for (GemvParams *p : {&a, &b}) {
        p->M = L.M;
        p->total_tiles = (long long)p->total_rg * p->nbu;
        p->off_terms = pl.terms;
        p->status = L.status;
        p->timeout_ns = L.timeout_ns;
        p->gterms = L.split_terms;
        p->gcount = L.split_count;
    }
    P.wg = L.gate;
    P.wu = L.up;
    P.x = reinterpret_cast<const __half *>(L.x);
    P.gamma = reinterpret_cast<const __half *>(L.gamma);
    P.g = reinterpret_cast<__half *>(L.g);
    P.u = reinterpret_cast<__half *>(L.u);
    P.pair = L.pair;
    P.exp_tab = L.exp_tab;
    P.gbar = L.gbar;
    P.hidden = L.hidden;
    P.ffn = L.ffn;
    P.M = L.M;
    P.off_rows = pl.rows;
    P.off_hsum = pl.hsum;
    P.off_desc = pl.desc;
    P.off_stages = pl.stages;
    P.off_bars = pl.bars;
    P.stage_bytes = pl.stage;
    P.S = pl.S;
    P.TA = pl.TA;
    P.TB = pl.TB;
    P.status = L.status;
    P.timeout_ns = L.timeout_ns;

    auto kern = kq_ffn_fused<GT, DT, MT>;
    {
        static std::mutex mu;
        static std::unordered_map<int, bool> configured;
        int dev = 0;
        cudaGetDevice(&dev);
        std::lock_guard<std::mutex> lk(mu);
        if (!configured[dev]) {
            cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, 225 * 1024);
            if (e != cudaSuccess) return e;
            configured[dev] = true;
        }
    }
    cudaLaunchConfig_t cfg{};
    cfg.gridDim = dim3(L.num_sms);
    cfg.blockDim = dim3(threads_of<MT>());
    // more than half of an SM's shared memory: one CTA per SM
    cfg.dynamicSmemBytes = std::max<unsigned>(pl.smem, 120u * 1024u);
    cfg.stream = stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = L.pdl ? 1 : 0;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, kern, P);
}

template <int GT, int DT>
cudaError_t launch_ffn_gd(const FfnFusedLaunch &L, const FfnPlan &pl, cudaStream_t stream) {
    return L.M <= 1 ? launch_ffn_t<GT, DT, 1>(L, pl, stream) : launch_ffn_t<GT, DT, 2>(L, pl, stream);
}

template <int GT>
cudaError_t launch_ffn_g(const FfnFusedLaunch &L, const FfnPlan &pl, cudaStream_t stream) {
    switch (L.down_type) {
        case TYPE_Q4_K: return launch_ffn_gd<GT, TYPE_Q4_K>(L, pl, stream);
        case TYPE_Q5_K: return launch_ffn_gd<GT, TYPE_Q5_K>(L, pl, stream);
        case TYPE_Q6_K: return launch_ffn_gd<GT, TYPE_Q6_K>(L, pl, stream);
        default: return cudaErrorNotSupported;
    }
}

}  // namespace

bool ffn_fused_supported(int gate_type, int down_type, int hidden, int ffn, int M, int num_sms) {
    if (M < 1 || M > 2 || num_sms < 1 || num_sms > 1024) return false;
    if (gate_type != TYPE_Q4_K && gate_type != TYPE_Q5_K) return false;
    if (down_type != TYPE_Q4_K && down_type != TYPE_Q5_K && down_type != TYPE_Q6_K) return false;
    if (hidden % 256 || ffn % 256 || hidden > RMS_MAX_SEG * 128 * 8) return false;
    return ffn_plan(gate_type, down_type, hidden, ffn, M, num_sms).ok;
}

cudaError_t launch_ffn_fused(const FfnFusedLaunch &L, cudaStream_t stream) {
    if (!ffn_fused_supported(L.gate_type, L.down_type, L.hidden, L.ffn, L.M, L.num_sms)) return cudaErrorNotSupported;
    const FfnPlan pl = ffn_plan(L.gate_type, L.down_type, L.hidden, L.ffn, L.M <= 1 ? 1 : 2, L.num_sms);
    switch (L.gate_type) {
        case TYPE_Q4_K: return launch_ffn_g<TYPE_Q4_K>(L, pl, stream);
        case TYPE_Q5_K: return launch_ffn_g<TYPE_Q5_K>(L, pl, stream);
        default: return cudaErrorNotSupported;
    }
}

}  // namespace kq
