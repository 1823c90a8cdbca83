// kq_gemv.cu -- K-quant x Q8 matrix-vector / small-batch product (M <= 8 tokens) for sm_100a.
//
// Replaces the engine's NEON row kernels (sdot_4rows_<type>_m1 / _batch, sdot_row_<type>_batch,
// src/v182_r22_breakthrough_engine.c:1226-3440) and its pinned work-stealing pool
// (exec_sdot_job_work_stealing, ENG:3491-3619).
//
// Design (HBM-bound: every weight byte is read once, activations are tiny):
//  * Weights are in the row-group tile layout of kq_common.cuh; the launch's tiles form one
//    sequence (row group major), each CTA owning a contiguous range of it.
//  * Warp W is the producer: one lane streams the CTA's tiles into shared-memory stages
//    (>= 16 KB) with cp.async.bulk, completion counted on mbarriers, L2 evict-first.
//  * Consumer warps 0..W-1 first stage the activation in shared memory (quantized to Q8_K /
//    Q8_0 bit-exactly as quantize_row_fp16_to_q8_k / _q8_0, ENG:925-1064, or copied from a
//    pre-quantized input).  Then they take work items round-robin and compute, for every
//    (row, token), the exact integer sub-block sums and the fp32 block term with the
//    reference's operation order into a term buffer:
//      - M <= 2: dp4a, an item is a tile with two lanes per row; the two lanes of a row read
//        different bank groups of the activation, shared by all rows (a broadcast);
//      - M > 2: an item is a tile; integer MMAs (m16n8k32, Q6_K m16n8k16) with ldmatrix
//        fragments give the sub-block dot products of all tokens at once.
//  * Each (row, token) result is the sum of its block terms in block order -- the reference's
//    `acc += term` sequence, so fp32 results equal the reference's bit for bit -- followed by
//    the epilogue: fp32 out, fp16 out with optional fp16 residual, argmax keys.
//  * Q4_K / Q5_K launches of 1-2 tokens whose shares would not fit shared memory whole or would
//    spread unevenly (config 0: 608 row groups over 148 SMs) give each CTA 8-row halves of row
//    groups instead: the whole share lands in one stage, the warps compute terms only, and the rows
//    are folded after a consumer barrier, spread over the threads (HalfShare, half_walk).
//  * Otherwise each CTA owns whole row groups and streams them through a ring of stages.  When the terms
//    of its whole share fit in shared memory (small launches) the warps compute all items and
//    fold everything after one barrier (when the ring holds the whole share, every stage is
//    probed once and, where one has not landed yet, each tile waits for its own stage only);
//    otherwise the warp that completes a row group folds it (shared-memory counters).
//    Under half an SM per CTA, the next kernel's CTA (programmatic dependent launch, enabled at
//    CTA start) prefetches its weights during this one's wait and arithmetic.
//  * Every wait is bounded (globaltimer); on timeout the kernel records DEV_ERR_TIMEOUT,
//    drains its own copies in flight (bounded) and returns.
#include "kq_gemv_dev.cuh"
#include "kq_internal.h"

#include <algorithm>
#include <mutex>
#include <unordered_map>

namespace kq {

// ------------------------------------------------------------------ the ranks' gather, in the GEMV
//
// After the CTA's outputs: count the CTA's arrival; the last PEER_TAIL_CTAS to arrive (every other
// CTA of the grid has finished) each wait for, and write to p.peer.out, an equal share of the
// other ranks' entries of this step -- stores of other GPUs' kernels only, never of a CTA of this
// grid, so nothing waits for a CTA that may not be resident.  The last of them to finish clears
// the counts and counts the step as completed.
constexpr unsigned PEER_TAIL_CTAS = 64;

__device__ __noinline__ void peer_tail(const GemvParams &p, int tid, bool aborted) {
    __shared__ int s_tail, s_fail;
    const PeerOut &po = p.peer;
    const unsigned G = gridDim.x, Kt = G < PEER_TAIL_CTAS ? G : PEER_TAIL_CTAS;
    if (tid == 0) {
        const unsigned a = atomicAdd(po.arrivals, 1u);
        s_tail = (a >= G - Kt) ? (int)(a - (G - Kt)) : -1;
        s_fail = 0;
    }
    __syncthreads();
    const int t = s_tail;
    if (t < 0) return;
    const unsigned long long st = peer_step(po);
    const long long other = po.row_stride - po.rows, total = (long long)po.M * other;
    if (!aborted && total > 0) {
        const unsigned long long *src = po.buf[po.rank] + (size_t)(st & 1ull) * po.buf_stride;
        const long long r0 = po.row0, rows = po.rows, rs = po.row_stride;
        auto map = [=](long long j) {
            const long long tok = j / other, c = j - tok * other;
            return tok * rs + (c < r0 ? c : c + rows);
        };
        peer_collect(src, (uint32_t)st, total * t / Kt, total * (t + 1) / Kt, tid, (int)blockDim.x, map, po.out,
                     global_timer_ns(), p.timeout_ns, p.status, &s_fail);
    }
    __syncthreads();
    if (tid == 0) {
        __threadfence();
        if (atomicAdd(po.tail_done, 1u) == Kt - 1) {
            *reinterpret_cast<volatile unsigned *>(po.arrivals) = 0u;
            *reinterpret_cast<volatile unsigned *>(po.tail_done) = 0u;
            __threadfence();
            *reinterpret_cast<volatile unsigned long long *>(po.step_rw) = st;
        }
    }
}

// ------------------------------------------------------------------ half row-group ownership
//
// A CTA owns the 8-row halves [h_lo, h_hi) (half h = rows 8 (h % 2).. of row group h / 2).  Its
// ring holds exactly those rows, in one stage:
//   [ha: the first row group's second half, units 0..nbu-1]
//   [the full row groups' tiles, as in global memory]
//   [hb: the last row group's first half, units 0..nbu-1]
// (ha = h_lo odd, hb = h_hi odd); a half tile (8 rows of one unit) is half a tile's bytes.
struct HalfShare {
    int h_lo, h_hi, rg_lo, ha, hb, nfull, hbytes;

    __device__ __forceinline__ HalfShare(int lo, int hi, int tile_bytes)
        : h_lo(lo), h_hi(hi), rg_lo(lo >> 1), ha(lo & 1), hb(hi & 1), nfull((hi - (hi & 1) - lo - (lo & 1)) >> 1),
          hbytes(tile_bytes / 2) {}

    // owned halves of local row group lr, and the first of them (0 or 1)
    __device__ __forceinline__ int halves(int lr) const {
        const int n_lr = ((h_hi + 1) >> 1) - rg_lo;
        return ((lr == 0 && ha) || (lr == n_lr - 1 && hb)) ? 1 : 2;
    }
    __device__ __forceinline__ int first_half(int lr) const { return (lr == 0 && ha) ? 1 : 0; }
};

// Producer lane: every copy of the share onto full barrier `bar` (one phase).
__device__ __forceinline__ void half_issue(const GemvParams &p, const HalfShare &hs, uint8_t *ring, uint32_t bar) {
    const int nbu = p.nbu, HB = hs.hbytes;
    const uint64_t policy = l2_evict_first_policy();
    const uint32_t base = smem_u32(ring);
    auto src = [&](int rg, int u) {
        const GemvTaskDev &tk = p.task[task_of_rg(p, rg)];
        return tk.w + ((size_t)(tk.rg_first - tk.rg_start) * nbu + (size_t)rg * nbu + u) * p.tile_bytes;
    };
    mbar_arrive_expect_tx(bar, (uint32_t)((hs.h_hi - hs.h_lo) * nbu * HB));
    if (hs.ha)
        for (int u = 0; u < nbu; ++u) bulk_g2s(base + u * HB, src(hs.rg_lo, u) + HB, HB, bar, policy);
    const int r0 = hs.rg_lo + hs.ha, re = r0 + hs.nfull;
    for (int rg = r0; rg < re;) {  // whole tiles, one copy per task's run of row groups
        const GemvTaskDev &tk = p.task[task_of_rg(p, rg)];
        const int rend = min(re, tk.rg_start + tk.n_rg);
        bulk_g2s(base + (hs.ha + 2 * (rg - r0)) * nbu * HB, src(rg, 0), (uint32_t)((rend - rg) * nbu) * p.tile_bytes,
                 bar, policy);
        rg = rend;
    }
    if (hs.hb)
        for (int u = 0; u < nbu; ++u)
            bulk_g2s(base + (hs.ha + 2 * hs.nfull) * nbu * HB + u * HB, src(re, u), HB, bar, policy);
}

// Consumers.  Warp w takes passes w, w + W, ... of the share: first the boundary passes -- with
// both a first and a last half row group, pass u is unit u of both (lanes 0-15 the first, 16-31
// the last); with one of them, pass j is its units 2j and 2j + 1 -- then the whole tiles of the
// full row groups, one per pass, as in a whole-row-group launch (warp-uniform unit, two lanes per
// row).  Terms only: the rows are folded after all passes (a fold inside the walk holds up the
// warp that makes it, and the walk's length is the slowest warp's).
template <int TYPE, int MT>
__device__ __forceinline__ void half_walk(const GemvParams &p, const GemvTaskDev *s_task, const HalfShare &hs,
                                          const uint8_t *ring, const uint8_t *smem, float *terms, int warp, int lane,
                                          int W, bool any_dbg) {
    const int nbu = p.nbu, J = p.terms_per_rg, tstride = 16 * MT, HB = hs.hbytes;
    const int n_lr = ((hs.h_hi + 1) >> 1) - hs.rg_lo;
    const int n_b = (hs.ha && hs.hb) ? nbu : (hs.ha || hs.hb) ? (nbu + 1) >> 1 : 0;
    const int g = lane >> 4, l16 = lane & 15;
    const int base_f = hs.ha * nbu * HB;                   // the full row groups' tiles
    const int base_b = (hs.ha + 2 * hs.nfull) * nbu * HB;  // the last half row group
    int j = warp;
    for (; j < n_b; j += W) {
        // per lane group: which half (first or last row group) and unit
        int u, lr, hh, off;
        if (hs.ha && hs.hb) {
            u = j;
            lr = g ? n_lr - 1 : 0;
            hh = g ? 0 : 1;
            off = (g ? base_b : 0) + u * HB;
        } else {
            u = min(2 * j + g, nbu - 1);  // an odd last pass: lanes 16-31 repeat lanes 0-15's unit
            lr = hs.ha ? 0 : n_lr - 1;
            hh = hs.ha ? 1 : 0;
            off = (hs.ha ? 0 : base_b) + u * HB;
        }
        DbgOut db;
        db.si = nullptr;
        if (any_dbg) {
            const GemvTaskDev &tk = s_task[task_of_rg(p, hs.rg_lo + lr)];
            if (tk.dbg_sumi) {
                db = make_dbg(p, tk, hs.rg_lo + lr, u, 0);
                db.r0 += 8 * hh;
            }
        }
        compute_item<TYPE, MT>(p, ring + off, u, smem, l16, terms + (lr * J + u) * tstride + 8 * hh * MT, db);
    }
    // whole tiles: pass n_b + t is tile t = k nbu + u of the full row groups (local row group ha + k)
    int t = j - n_b, k = 0, u = t;
    while (u >= nbu) {
        u -= nbu;
        ++k;
    }
    for (; t < hs.nfull * nbu; t += W) {
        const int lr = hs.ha + k;
        DbgOut db;
        db.si = nullptr;
        if (any_dbg) {
            const GemvTaskDev &tk = s_task[task_of_rg(p, hs.rg_lo + lr)];
            if (tk.dbg_sumi) db = make_dbg(p, tk, hs.rg_lo + lr, u, 0);
        }
        compute_item<TYPE, MT>(p, ring + base_f + t * 2 * HB, u, smem, lane, terms + (lr * J + u) * tstride, db);
        u += W;
        while (u >= nbu) {
            u -= nbu;
            ++k;
        }
    }
}

// ------------------------------------------------------------------ the kernel
//
// CTA c owns row groups [rg_lo, rg_hi) = tiles [t0, t1) of the launch's tile sequence
// (tile = rg * nbu + u).  Stage s holds local tiles [s*T, s*T + T) in ring slot s % S;
// consumers wait for a stage to be issued before testing its full barrier (so the barrier's
// phase parity refers to that stage) and arrive on its empty barrier when done with an item.
// Warp w takes tiles w, w + W, ...
//  SMALL: the terms of the whole share stay in shared memory (local row group lr at
//         terms[lr * J ...]); all row groups are folded after a consumer barrier.
//  !SMALL: terms of row group lr go to term slot lr % TS, use lr / TS; a writer waits until the
//         slot's previous use is folded and the warp completing the row group folds it
//         (monotonic shared-memory counters).

template <int TYPE, int MT, bool SMALL, bool SPLIT>
__global__ void __launch_bounds__(threads_of<MT>(), 2) kq_gemv(const __grid_constant__ GemvParams p) {
    extern __shared__ __align__(128) uint8_t smem[];
    __shared__ unsigned long long s_best[8];
    __shared__ int s_abort, s_issued;
    __shared__ int s_done[kMaxTermSlots], s_folded[kMaxTermSlots];
    // the tasks' fields, read per tile and per output row: from shared memory rather than by a
    // run-time index into the kernel parameters
    __shared__ GemvTaskDev s_task[4];

    uint8_t *ring = smem + p.off_stages;
    uint64_t *bars = reinterpret_cast<uint64_t *>(smem + p.off_bars);  // full[S], empty[S], dead
    float *terms = reinterpret_cast<float *>(smem + p.off_terms);
    const int S = p.n_stages, T = p.tiles_per_stage, TS = p.term_slots, J = p.terms_per_rg;
    constexpr int W = warps_of<MT>();
    const int nbu = p.nbu;
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int tstride = 16 * MT;  // floats per term row

    // this CTA's tiles [t0, t0 + n_tiles) of the launch's row-group-major tile sequence: whole
    // row groups, or (SPLIT) an equal share of tiles whose first / last row group may be shared
    int rg_lo, rg_hi, t0, n_tiles, u_first = 0, u_end = nbu;
    // half row-group ownership (GemvParams::half): halves [h_lo, h_hi)
    constexpr bool HALF_OK = SMALL && !SPLIT && MT <= 2 && (TYPE == TYPE_Q4_K || TYPE == TYPE_Q5_K);
    const bool half = HALF_OK && p.half;
    int h_lo = 0, h_hi = 0;
    if (SPLIT) {
        const long long tl = p.total_tiles * blockIdx.x / gridDim.x;
        const long long th = p.total_tiles * (blockIdx.x + 1) / gridDim.x;
        t0 = (int)tl;
        n_tiles = (int)(th - tl);
        rg_lo = (int)(tl / nbu);
        rg_hi = (int)((th + nbu - 1) / nbu);
        u_first = t0 - rg_lo * nbu;                         // owned units of row group rg_lo: [u_first, nbu)
        u_end = (int)(th - (long long)(rg_hi - 1) * nbu);  // owned units of row group rg_hi - 1: [0, u_end)
    } else if (half) {
        const long long nh = 2ll * p.total_rg;
        h_lo = (int)(nh * blockIdx.x / gridDim.x);
        h_hi = (int)(nh * (blockIdx.x + 1) / gridDim.x);
        rg_lo = h_lo >> 1;
        rg_hi = (h_hi + 1) >> 1;
        t0 = rg_lo * nbu;
        n_tiles = (rg_hi - rg_lo) * nbu;  // tiles touched (a half tile counted whole)
    } else {
        rg_lo = (int)((long long)p.total_rg * blockIdx.x / gridDim.x);
        rg_hi = (int)((long long)p.total_rg * (blockIdx.x + 1) / gridDim.x);
        t0 = rg_lo * nbu;
        n_tiles = (rg_hi - rg_lo) * nbu;
    }
    const int n_lr = rg_hi - rg_lo;
    const int n_stages_cta = (n_tiles + T - 1) / T;

    if (tid < 4 && tid < p.n_tasks) s_task[tid] = p.task[tid];
    if (tid < 8) s_best[tid] = 0ull;
    if (tid < kMaxTermSlots) {
        s_done[tid] = 0;
        s_folded[tid] = 0;
    }
    if (tid == 0) {
        for (int s = 0; s < S; ++s) {
            mbar_init(smem_u32(&bars[s]), 1);
            mbar_init(smem_u32(&bars[S + s]), T);
        }
        mbar_init(smem_u32(&bars[2 * S]), 1);  // never arrived at (failure-path test)
        s_abort = 0;
        s_issued = 0;
        mbar_init_fence();
    }
    __syncthreads();

    // The next kernel in the stream may launch (programmatic dependent launch) as soon as every
    // CTA of this one is resident: it only streams its weights before its own griddepcontrol.wait,
    // so its weight stream overlaps this kernel's wait, activation staging and arithmetic (a chain
    // of such launches is then bound by the weight stream, not by the dependent-launch release).
    pdl_launch_dependents();
    const HalfShare hs(h_lo, h_hi, (int)p.tile_bytes);
    if (half && warp == W) {
        // ---------------- producer, halves: the whole share in one stage (the consumers wait for it)
        if (lane == 0) {
            half_issue(p, hs, ring, smem_u32(&bars[0]));
            s_issued = 1;
        }
        __syncwarp();
        __syncthreads();  // activation staged
    } else if (warp == W) {
        // ---------------- producer: the weight stream does not depend on earlier kernels
        const uint64_t policy = l2_evict_first_policy();
        auto issue = [&](int s) {
            const int slot = s % S;
            const int a = s * T, b = min(n_tiles, a + T);
            const uint32_t full = smem_u32(&bars[slot]);
            const uint32_t sdst = smem_u32(ring + (size_t)slot * p.stage_bytes);
            mbar_arrive_expect_tx(full, (uint32_t)(b - a) * p.tile_bytes);
            int i = a;
            while (i < b) {
                const int tau = t0 + i, rg = tau / nbu;
                const GemvTaskDev &tk = p.task[task_of_rg(p, rg)];
                const int iend = min(b, (tk.rg_start + tk.n_rg) * nbu - t0);
                const size_t src_tile = (size_t)(tk.rg_first - tk.rg_start) * nbu + tau;
                bulk_g2s(sdst + (uint32_t)(i - a) * p.tile_bytes, tk.w + src_tile * p.tile_bytes,
                         (uint32_t)(iend - i) * p.tile_bytes, full, policy);
                i = iend;
            }
            *reinterpret_cast<volatile int *>(&s_issued) = s + 1;
        };
        const int first = min(S, n_stages_cta);  // stages that need no free slot
        if (lane == 0)
            for (int s = 0; s < first; ++s) issue(s);
        __syncwarp();
        __syncthreads();  // activation staged
        if (lane == 0) {
            for (int s = first; s < n_stages_cta; ++s) {
                if (!mbar_wait_bounded(smem_u32(&bars[S + s % S]), ((s / S) - 1) & 1, p.timeout_ns, p.status)) {
                    s_abort = 1;
                    break;
                }
                issue(s);
            }
        }
    } else {
        // ---------------- consumers
        pdl_wait();  // activations / residuals may come from the previous kernel
        stage_activation<TYPE, MT>(p, smem, warp, lane, W);
        if (p.inject_wait && tid == 0) {
            // failure-path test: a wait whose barrier nothing completes must end by its time limit
            if (!mbar_wait_bounded(smem_u32(&bars[2 * S]), 0, p.timeout_ns, p.status)) s_abort = 1;
        }
        __syncthreads();  // activation staged

        // tile walk: tile i advances by W; stage/slot/phase, unit and row group incremental.
        constexpr int TSTEP = W;
        const bool all_in = !half && SMALL && n_stages_cta <= S;
        const int JU = (TYPE == TYPE_Q8_0 && p.q80_exact) ? 8 : 1;  // terms per unit
        bool any_dbg = false;
        for (int k = 0; k < p.n_tasks; ++k) any_dbg |= s_task[k].dbg_sumi != nullptr;
        // all in (the ring holds the whole share, every stage issued at CTA start): no slot is
        // reused, so no consumer frees one; without a split each row group is folded by the warp
        // that completes it (the row-group counters s_done), overlapping the folds with the other
        // warps' tiles
        const bool early_fold = all_in && !SPLIT && n_lr <= kMaxTermSlots;
        if (HALF_OK && half) {
            // the share's one stage (landed during the previous kernel in a chain of launches)
            int ok = 1;
            if (lane == 0) ok = mbar_wait_bounded(smem_u32(&bars[0]), 0, p.timeout_ns, p.status);
            ok = __shfl_sync(0xffffffffu, ok, 0);
            __syncwarp();
            if (!ok && lane == 0) s_abort = 1;
            if (ok && !*reinterpret_cast<volatile int *>(&s_abort))
                half_walk<TYPE, MT>(p, s_task, hs, ring, smem, terms, warp, lane, W, any_dbg);
            // fold the owned rows of every row group after all passes, spread over the consumers
            named_bar_sync(1, W * 32);
            if (!*reinterpret_cast<volatile int *>(&s_abort)) {
                const int E = 16 * MT;
                for (int idx = tid; idx < n_lr * E; idx += W * 32) {
                    const int l = idx / E, e = idx - l * E, e0 = 8 * hs.first_half(l) * MT;
                    if (e >= e0 && e < e0 + 8 * hs.halves(l) * MT)
                        fold_one<MT>(p, s_task, terms + (size_t)l * J * tstride, J, e, rg_lo + l, s_best);
                }
            }
        }
        if (all_in) {
            int tt = warp, sg = 0;
            while (tt >= T) {
                tt -= T;
                ++sg;
            }
            int u = u_first + warp, lr = 0;
            while (u >= nbu) {
                u -= nbu;
                ++lr;
            }
            // every stage was issued at CTA start.  In a chain of launches they landed during the
            // previous kernel (one probe each, then no waits); after a cold start (e.g. one call
            // after a host copy) each tile waits only for its own stage, so the arithmetic starts
            // while the later stages still stream in
            int seen = 1;
            if (lane == 0)
                for (int s = 0; s < n_stages_cta; ++s) seen &= mbar_test_wait(smem_u32(&bars[s]), 0) ? 1 : 0;
            seen = __shfl_sync(0xffffffffu, seen, 0) ? n_stages_cta : 0;
            __syncwarp();  // lane 0 saw the stages complete: order the warp's reads after it
            const bool go = !*reinterpret_cast<volatile int *>(&s_abort);
            for (int i = warp; go && i < n_tiles; i += TSTEP) {
                if (sg >= seen) {
                    int ok = 1;
                    if (lane == 0) ok = mbar_wait_bounded(smem_u32(&bars[sg]), 0, p.timeout_ns, p.status);
                    ok = __shfl_sync(0xffffffffu, ok, 0);
                    if (!ok) {
                        if (lane == 0) s_abort = 1;
                        break;
                    }
                    __syncwarp();
                    seen = sg + 1;
                }
                const uint8_t *tile = ring + sg * p.stage_bytes + tt * p.tile_bytes;
                DbgOut db;
                db.si = nullptr;
                if (any_dbg) {
                    const GemvTaskDev &tk = s_task[task_of_rg(p, rg_lo + lr)];
                    if (tk.dbg_sumi) db = make_dbg(p, tk, rg_lo + lr, u, TYPE == TYPE_Q8_0);
                }
                float *tdst = terms + (lr * J + u * JU) * tstride;
                compute_item<TYPE, MT>(p, tile, u, smem, lane, tdst, db);
                __syncwarp();
                if (early_fold) {
                    int last = 0;
                    if (lane == 0) {
                        __threadfence_block();
                        last = atomicAdd(&s_done[lr], 1) == nbu - 1;
                    }
                    last = __shfl_sync(0xffffffffu, last, 0);
                    if (last) {
                        __threadfence_block();
                        for (int e = lane; e < 16 * MT; e += 32)
                            fold_one<MT>(p, s_task, terms + (size_t)lr * J * tstride, J, e, rg_lo + lr, s_best);
                    }
                }
                tt += TSTEP;
                while (tt >= T) {
                    tt -= T;
                    ++sg;
                }
                u += TSTEP;
                while (u >= nbu) {
                    u -= nbu;
                    ++lr;
                }
            }
        }
        int i = (all_in || half) ? n_tiles : warp;
        int tt = i, sg = 0, slot = 0, ph = 0;
        while (tt >= T) {
            tt -= T;
            ++sg;
            if (++slot == S) {
                slot = 0;
                ph ^= 1;
            }
        }
        int u = u_first + i, lr = 0;
        while (u >= nbu) {
            u -= nbu;
            ++lr;
        }
        int ts = lr % TS, use = lr / TS;
        for (; i < n_tiles; i += TSTEP) {
            if (*reinterpret_cast<volatile int *>(&s_abort)) break;
            if (!all_in) {
                int ok = 1;
                if (lane == 0) {
                    ok = wait_ge_bounded(&s_issued, sg + 1, p.timeout_ns, p.status) &&
                         mbar_wait_bounded(smem_u32(&bars[slot]), ph, p.timeout_ns, p.status) &&
                         (SMALL || wait_ge_bounded(&s_folded[ts], use, p.timeout_ns, p.status));
                }
                ok = __shfl_sync(0xffffffffu, ok, 0);
                if (!ok) {
                    if (lane == 0) s_abort = 1;
                    break;
                }
            }
            const uint8_t *tile = ring + slot * p.stage_bytes + tt * p.tile_bytes;
            const int rg = rg_lo + lr;
            const GemvTaskDev &tk = s_task[task_of_rg(p, rg)];
            DbgOut db;
            db.si = nullptr;
            if (tk.dbg_sumi) db = make_dbg(p, tk, rg, u, TYPE == TYPE_Q8_0);
            float *tdst = terms + ((SMALL ? lr : ts) * J + u * JU) * tstride;
            compute_item<TYPE, MT>(p, tile, u, smem, lane, tdst, db);
            __syncwarp();
            if (SMALL) {
                if (!all_in && lane == 0) mbar_arrive(smem_u32(&bars[S + slot]));  // T arrivals free the slot
            } else {
                int last = 0;
                // the row group is complete when its owned tiles are: slot 0's count misses the
                // first row group's unowned units, the last row group misses its own
                const int ua = (SPLIT && lr == 0) ? u_first : 0, ub = (SPLIT && lr == n_lr - 1) ? u_end : nbu;
                const int missing = SPLIT ? ((ts == 0) ? u_first : 0) + nbu - ub : 0;
                if (lane == 0) {
                    mbar_arrive(smem_u32(&bars[S + slot]));
                    __threadfence_block();
                    last = (atomicAdd(&s_done[ts], 1) == (use + 1) * nbu - missing - 1);
                }
                last = __shfl_sync(0xffffffffu, last, 0);
                if (last) {
                    // fold the row group: block terms in order, then the epilogue
                    __threadfence_block();
                    float *tb = terms + ts * J * tstride;
                    if (SPLIT && (ua > 0 || ub < nbu)) fold_shared<MT>(p, s_task, tb, J, JU, ua, ub, rg, lane, s_best);
                    else
                        for (int e = lane; e < 16 * MT; e += 32) fold_one<MT>(p, s_task, tb, J, e, rg, s_best);
                    __syncwarp();
                    if (lane == 0) {
                        __threadfence_block();
                        *reinterpret_cast<volatile int *>(&s_folded[ts]) = use + 1;
                    }
                }
            }
            tt += TSTEP;
            while (tt >= T) {
                tt -= T;
                ++sg;
                if (++slot == S) {
                    slot = 0;
                    ph ^= 1;
                }
            }
            u += TSTEP;
            while (u >= nbu) {
                u -= nbu;
                ++lr;
                if (++ts == TS) {
                    ts = 0;
                    ++use;
                }
            }
        }
        if (SMALL && !early_fold && !half) {
            // ---------------- fold all row groups of the share
            named_bar_sync(1, W * 32);
            const int E = 16 * MT;
            const bool part0 = SPLIT && u_first > 0, part1 = SPLIT && u_end < nbu;  // first / last row group shared
            for (int idx = tid; idx < n_lr * E; idx += W * 32) {
                const int l = idx / E, e = idx - l * E;
                if ((l == 0 && part0) || (l == n_lr - 1 && part1)) continue;
                fold_one<MT>(p, s_task, terms + (size_t)l * J * tstride, J, e, rg_lo + l, s_best);
            }
            if (part0 && warp == 0)
                fold_shared<MT>(p, s_task, terms, J, JU, u_first, n_lr == 1 ? u_end : nbu, rg_lo, lane, s_best);
            if (part1 && (n_lr > 1 || !part0) && warp == (W > 1 ? 1 : 0))
                fold_shared<MT>(p, s_task, terms + (size_t)(n_lr - 1) * J * tstride, J, JU, 0, u_end, rg_hi - 1,
                                lane, s_best);
        }
    }
    __syncthreads();
    if (p.argmax && tid < p.M && !s_abort) atomicMax(&p.argmax[tid], s_best[tid]);
    if (p.peer.out) peer_tail(p, tid, s_abort != 0);
    // drain: a slot's most recent copy must land before the CTA exits (matters only after an
    // early stop); consumers never arrive on full barriers, so the last S issued stages are
    // exactly the outstanding candidates
    // (without an early stop the consumers waited for every issued stage already)
    if (tid == 0 && s_abort) {
        const int issued = s_issued;
        for (int s = max(0, issued - S); s < issued; ++s)
            mbar_wait_bounded(smem_u32(&bars[s % S]), (s / S) & 1, p.timeout_ns, p.status);
    }
}

// ------------------------------------------------------------------ host launcher

// A split launch has at most 2 CTAs per SM, each the first-tile owner of at most one shared row
// group: one slot of J block terms x 16 MT (row, token) pairs per possible CTA.
int gemv_split_slots(int num_sms) { return 2 * num_sms; }

size_t gemv_split_bytes(int type, int K, int M, int num_sms) {
    const int MT = M <= 1 ? 1 : M <= 2 ? 2 : M <= 4 ? 4 : 8;
    const size_t J = (size_t)(K / 256) * (type == TYPE_Q8_0 ? 8 : 1);
    return (size_t)gemv_split_slots(num_sms) * J * 16 * MT * sizeof(float);
}

namespace {

struct Plan {
    int small, T, S, TS, J, q80_exact, grid;
    unsigned stage_bytes, off_x, off_dx, off_xs, off_terms, off_stages, off_bars, smem;
};

unsigned align_up(unsigned v, unsigned a) { return (v + a - 1) / a * a; }

// Geometry of one launch (MT token slots).
//  * Stage = T tiles, >= 16 KB (smaller bulk copies do not reach full HBM bandwidth).
//  * Whole row groups per CTA.  One CTA per SM (two when each has plenty of work) within
//    ~110 KB of shared memory, so a second CTA -- this kernel's or the next one's -- fits beside
//    it, else one with up to 220 KB.  The ring takes what is left after the activation and the
//    term buffers, up to the CTA's whole share.
//  * SMALL (dp4a only) when the terms of the whole share fit: fold after one barrier.  Else term
//    slots cover the row groups that can be in flight (ring tiles / nbu + 2).
//  * Q8_0 keeps one term per 32-block (the reference's exact order) when that fits, else one
//    per tile.
Plan make_plan(int type, int K, int MT, int total_rg, int num_sms, int n_warps, bool split) {
    Plan pl{};
    const int nbu = K / 256;
    const long long total_tiles = (long long)total_rg * nbu;
    const unsigned TB = (unsigned)tile_bytes(type);
    const int XP = MT < 2 ? 2 : MT;
    const bool dp = MT <= 2;
    const unsigned x_bytes = align_up((unsigned)(dp ? MT * 320 * nbu : MT * (K + 16)), 128);
    const unsigned dx_bytes = align_up((unsigned)(nbu * (type == TYPE_Q8_0 ? 8 : 1) * XP * 4), 128);
    const unsigned xs_bytes = (type == TYPE_Q6_K)   ? align_up((unsigned)(nbu * 16 * (dp ? MT : XP) * 4), 128)
                              : (type == TYPE_Q8_0) ? 0
                                                    : align_up((unsigned)(MT * nbu * 8 * 4), 128);
    const unsigned fixed = x_bytes + dx_bytes + xs_bytes;
    const int T = std::max(1, (int)((16384 + TB - 1) / TB));
    const unsigned stage = align_up(T * TB, 128);
    // Q8_0: the reference's per-block term order (exact) takes precedence over the smaller budget
    for (int exact = (type == TYPE_Q8_0) ? 1 : 0; exact >= 0; --exact) {
    const int J = (type == TYPE_Q8_0 && exact) ? 8 * nbu : nbu;
    for (unsigned budget : {110u * 1024u, 220u * 1024u}) {
        for (int ctas : {2, 1}) {
            if (ctas == 2 && budget > 110u * 1024u) continue;
            // split: tile ranges (a CTA spans at most ceil((tiles - 1) / nbu) + 1 row groups);
            // else whole row groups
            const int grid = std::max(1, (int)std::min<long long>(split ? total_tiles : total_rg, ctas * num_sms));
            const int tiles_cta = split ? (int)((total_tiles + grid - 1) / grid) : (total_rg + grid - 1) / grid * nbu;
            const int rg_cta = split ? std::min(total_rg, (tiles_cta + nbu - 2) / nbu + 1) : tiles_cta / nbu;
            // one CTA per SM with room for the next kernel's when a share is small (M <= 2: the
            // next kernel's weight prefetch hides behind this one's arithmetic); many-token
            // launches are long enough that two of their own CTAs per SM pay more
            if (ctas == 2 && MT <= 2 && tiles_cta < 8 * n_warps) continue;
            const int stages_cta = (tiles_cta + T - 1) / T;
            for (int small = dp ? 1 : 0; small >= 0; --small) {
                {
                    for (int S = std::min(stages_cta, 32); S >= 1; --S) {
                        const int TS = small ? rg_cta
                                             : std::min(std::min(rg_cta, kMaxTermSlots), (S * T + nbu - 1) / nbu + 2);
                        const unsigned term_bytes = align_up((unsigned)(TS * J * 16 * MT * 4), 128);
                        const unsigned total = fixed + term_bytes + S * stage + (2 * S + 1) * 8;
                        if (total > budget) continue;
                        if (S < std::min(stages_cta, 2)) break;  // a ring needs two slots unless one stage is all
                        pl.small = small;
                        pl.T = T;
                        pl.S = S;
                        pl.TS = small ? 1 : TS;
                        pl.J = J;
                        pl.q80_exact = (type == TYPE_Q8_0) ? exact : 0;
                        pl.grid = grid;
                        pl.stage_bytes = stage;
                        pl.off_x = 0;
                        pl.off_dx = x_bytes;
                        pl.off_xs = x_bytes + dx_bytes;
                        pl.off_terms = fixed;
                        pl.off_stages = fixed + term_bytes;
                        pl.off_bars = pl.off_stages + S * stage;
                        pl.smem = pl.off_bars + (2 * S + 1) * 8;
                        return pl;
                    }
                }
            }
        }
    }
    }
    return pl;  // smem 0: does not fit
}

// Half row-group ownership (Q4_K / Q5_K, <= 2 tokens): at most one CTA per SM, each CTA's whole
// share of 8-row halves in one stage and the terms of every row group it touches in shared
// memory, all within ~110 KB so that the next kernel's CTA fits beside it.  smem 0: no such plan.
Plan make_half_plan(int type, int K, int MT, int total_rg, int num_sms) {
    Plan pl{};
    if (MT > 2 || (type != TYPE_Q4_K && type != TYPE_Q5_K)) return pl;
    const int nbu = K / 256;
    const unsigned x_bytes = align_up((unsigned)(MT * 320 * nbu), 128);
    const unsigned dx_bytes = align_up((unsigned)(nbu * 2 * 4), 128);
    const unsigned xs_bytes = align_up((unsigned)(MT * nbu * 8 * 4), 128);
    const unsigned fixed = x_bytes + dx_bytes + xs_bytes;
    const int grid = std::max(1, std::min(2 * total_rg, num_sms));
    const int hc = (2 * total_rg + grid - 1) / grid;   // halves of the largest share
    const int rg_cta = std::min(total_rg, hc / 2 + 1);  // row groups it can touch
    const unsigned stage = align_up((unsigned)(hc * nbu) * (unsigned)tile_bytes(type) / 2, 128);
    const unsigned term_bytes = align_up((unsigned)(rg_cta * nbu * 16 * MT * 4), 128);
    const unsigned total = fixed + term_bytes + stage + 3 * 8;
    if (total > 110u * 1024u || rg_cta > kMaxTermSlots) return pl;
    pl.small = 1;
    pl.T = hc * nbu;
    pl.S = 1;
    pl.TS = 1;
    pl.J = nbu;
    pl.q80_exact = 0;
    pl.grid = grid;
    pl.stage_bytes = stage;
    pl.off_x = 0;
    pl.off_dx = x_bytes;
    pl.off_xs = x_bytes + dx_bytes;
    pl.off_terms = fixed;
    pl.off_stages = fixed + term_bytes;
    pl.off_bars = pl.off_stages + stage;
    pl.smem = pl.off_bars + 3 * 8;
    return pl;
}

template <typename Kern>
cudaError_t configure_smem(Kern kern) {
    static std::mutex mu;
    static std::unordered_map<int, std::unordered_map<const void *, bool>> configured;
    int dev = 0;
    cudaGetDevice(&dev);
    std::lock_guard<std::mutex> lk(mu);
    bool &done = configured[dev][reinterpret_cast<const void *>(kern)];
    if (!done) {
        // plans stay below 221 KB of dynamic shared memory; 225 KB leaves room for the kernel's
        // static shared words within the 227 KB per-block limit
        cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, 225 * 1024);
        if (e != cudaSuccess) return e;
        done = true;
    }
    return cudaSuccess;
}

template <int TYPE, int MT>
cudaError_t launch_t(const GemvLaunch &L, cudaStream_t stream) {
    GemvParams p{};
    int total_rg = 0;
    for (int i = 0; i < L.n_tasks; ++i) {
        const GemvTaskHost &h = L.tasks[i];
        GemvTaskDev &d = p.task[i];
        d.w = h.w;
        d.row_begin = h.row_begin;
        d.rows = h.rows;
        d.rg_first = h.row_begin / 16;
        d.n_rg = h.rows > 0 ? (h.row_begin + h.rows - 1) / 16 - d.rg_first + 1 : 0;
        d.rg_start = total_rg;
        d.dst = reinterpret_cast<__half *>(h.dst);
        d.dst_stride = h.dst_stride;
        d.res = reinterpret_cast<const __half *>(h.res);
        d.res_stride = h.res_stride;
        d.dst_f32 = h.dst_f32;
        d.f32_stride = h.f32_stride;
        d.dbg_sumi = h.dbg_sumi;
        d.dbg_summ = h.dbg_summ;
        d.out_ids = h.out_ids;
        d.index_base = h.index_base;
        total_rg += d.n_rg;
    }
    if (total_rg == 0) return cudaSuccess;
    Plan pl = make_plan(TYPE, L.K, MT, total_rg, L.num_sms, warps_of<MT>(), false);
    // Balanced tile ranges only where whole row groups at one CTA per SM leave the SMs badly
    // unequal (e.g. 160 row groups over 148 SMs, or fewer row groups than SMs): each shared row
    // group costs its last CTA a few L2 round trips before it can finish, and where a second CTA
    // fits beside the first the SMs that hold two row groups run them side by side anyway.
    bool split = L.split_terms != nullptr && L.split_count != nullptr && pl.grid <= L.num_sms;
    if (split) {
        const Plan ps = make_plan(TYPE, L.K, MT, total_rg, L.num_sms, warps_of<MT>(), true);
        const long long nbu = L.K / 256, tt = (long long)total_rg * nbu;
        auto sm_load = [&](const Plan &q, bool sp) {  // tiles of the busiest SM
            const long long per = sp ? (tt + q.grid - 1) / q.grid : (long long)((total_rg + q.grid - 1) / q.grid) * nbu;
            return per * ((q.grid + L.num_sms - 1) / L.num_sms);
        };
        split = ps.smem != 0 && (pl.smem == 0 || sm_load(pl, false) * 10 >= sm_load(ps, true) * 14);
        if (split) pl = ps;
    }
    // Halves where whole row groups leave the largest share partly outside shared memory (its last
    // stages refill while the launch computes) or give its warps more tile passes: config 0's 608
    // row groups over 148 SMs are 4 or 5 row groups per CTA (50 tiles, 40 fit), as halves 8 or 9
    // (at most 45 tiles' rows, all resident, 3 passes per warp).
    bool half = false;
    if (L.half_ok && !split && pl.smem != 0 && pl.small && pl.grid <= L.num_sms) {
        const Plan ph = make_half_plan(TYPE, L.K, MT, total_rg, L.num_sms);
        if (ph.smem != 0) {
            const int nbu = L.K / 256, Wn = warps_of<MT>();
            const int tiles_whole = (total_rg + pl.grid - 1) / pl.grid * nbu;
            const bool whole_in = (tiles_whole + pl.T - 1) / pl.T <= pl.S;
            const int hc = (2 * total_rg + ph.grid - 1) / ph.grid;
            const int passes_half = ((hc * nbu + 1) / 2 + Wn - 1) / Wn, passes_whole = (tiles_whole + Wn - 1) / Wn;
            half = !whole_in || passes_half < passes_whole;
            if (half) pl = ph;
        }
    }
    if (pl.smem == 0) return cudaErrorInvalidConfiguration;
    if (split && gemv_split_bytes(TYPE, L.K, L.M, L.num_sms) > L.split_terms_bytes) return cudaErrorInvalidValue;
    p.half = half ? 1 : 0;
    p.total_tiles = (long long)total_rg * (L.K / 256);
    p.gterms = split ? L.split_terms : nullptr;
    p.gcount = split ? L.split_count : nullptr;
    p.n_tasks = L.n_tasks;
    p.total_rg = total_rg;
    p.K = L.K;
    p.nbu = L.K / 256;
    p.M = L.M;
    p.tile_bytes = (unsigned)tile_bytes(TYPE);
    p.tiles_per_stage = pl.T;
    p.n_stages = pl.S;
    p.term_slots = pl.TS;
    p.terms_per_rg = pl.J;
    p.q80_exact = pl.q80_exact;
    p.stage_bytes = pl.stage_bytes;
    p.x = reinterpret_cast<const __half *>(L.x);
    p.x_stride = L.x_stride;
    p.act = L.act;
    p.status = L.status;
    p.timeout_ns = L.timeout_ns;
    p.argmax = L.argmax;
    p.argmax_f16 = L.argmax_f16;
    p.inject_wait = L.inject_wait;
    p.peer = L.peer;
    p.off_x = pl.off_x;
    p.off_dx = pl.off_dx;
    p.off_xs = pl.off_xs;
    p.off_terms = pl.off_terms;
    p.off_stages = pl.off_stages;
    p.off_bars = pl.off_bars;

    auto kern = pl.small ? (split ? kq_gemv<TYPE, MT, true, true> : kq_gemv<TYPE, MT, true, false>)
                         : (split ? kq_gemv<TYPE, MT, false, true> : kq_gemv<TYPE, MT, false, false>);
    if (cudaError_t e = configure_smem(kern)) return e;
    cudaLaunchConfig_t cfg{};
    cfg.gridDim = dim3(pl.grid);
    cfg.blockDim = dim3(threads_of<MT>());
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

// ------------------------------------------------------------------ gathered rows

// Copy weight rows ids[0..n) into a fresh tiled tensor (row i of dst = row ids[i] of src), so a
// row-id list runs through the same GEMV kernel.  One thread per GGUF byte of a row.
__global__ void kq_gather_rows(int type, int nbu, const uint8_t *src, const uint32_t *ids, int n, uint8_t *dst,
                                   size_t gguf_row_bytes) {
    const size_t total = (size_t)n * gguf_row_bytes;
    for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < total; i += (size_t)gridDim.x * blockDim.x) {
        const int r = (int)(i / gguf_row_bytes);
        const size_t ob = i - (size_t)r * gguf_row_bytes;
        dst[tile_byte_offset(type, nbu, r, ob)] = src[tile_byte_offset(type, nbu, (int)ids[r], ob)];
    }
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

cudaError_t launch_gather_rows(int type, int K, const uint8_t *src, const uint32_t *ids, int n, uint8_t *dst,
                               cudaStream_t stream) {
    if (n <= 0) return cudaSuccess;
    const size_t rb = (size_t)(K / 256) * unit_bytes(type);
    cudaError_t e = cudaMemsetAsync(dst, 0, weight_bytes(type, n, K), stream);
    if (e != cudaSuccess) return e;
    const size_t total = (size_t)n * rb;
    const int blocks = (int)std::min<size_t>((total + 255) / 256, 148 * 16);
    kq_gather_rows<<<blocks, 256, 0, stream>>>(type, K / 256, src, ids, n, dst, rb);
    return cudaGetLastError();
}

// ------------------------------------------------------------------ the ranks' gather

// Every thread reads its share of the M x row_stride entries of buffer s % 2 (s = completed steps
// + 1) until each carries tag s -- bounded: the first thread to give up records DEV_ERR_TIMEOUT and
// every thread stops waiting -- and writes the values to `out`.  The last CTA to finish counts the
// step as completed.  It may be launched while this rank's GEMV still runs (programmatic dependent
// launch), but reads nothing before the GEMV grid has completed (griddepcontrol.wait), so it never
// spins on a kernel of its own GPU; it lets the next kernel launch at once.
__global__ void __launch_bounds__(256) kq_peer_gather_wait(const __grid_constant__ PeerWait W) {
    __shared__ unsigned long long s_step;
    __shared__ int s_fail;
    const int tid = threadIdx.x;
    // the next GEMV (launched with programmatic dependent launch) may stream its weights while
    // this kernel waits; it reads the step counter and the buffers only after this grid completes
    asm volatile("griddepcontrol.launch_dependents;");
    // this rank's GEMV must be complete before anything is read: a dependent-launch wait (the
    // hardware orders it), not a spin on a kernel of this GPU
    asm volatile("griddepcontrol.wait;" ::: "memory");
    if (tid == 0) {
        s_step = *reinterpret_cast<const volatile unsigned long long *>(W.step) + 1ull;
        s_fail = 0;
    }
    __syncthreads();
    const unsigned long long s = s_step;
    const uint32_t tag = (uint32_t)s;
    const unsigned long long *src = W.buf + (size_t)(s & 1ull) * W.buf_stride;
    // every thread of the grid: entries 4 t .. 4 t + 3, then the next 4 x (threads of the grid)
    peer_collect(src, tag, 0, W.n_entries, (int)(blockIdx.x * blockDim.x + tid), (int)(gridDim.x * blockDim.x),
                 [](long long j) { return j; }, W.out, global_timer_ns(), W.timeout_ns, W.status, &s_fail);
    __syncthreads();
    if (tid == 0) {
        __threadfence();
        if (atomicAdd(W.arrivals, 1u) == gridDim.x - 1) {
            *reinterpret_cast<volatile unsigned *>(W.arrivals) = 0u;
            __threadfence();
            *reinterpret_cast<volatile unsigned long long *>(W.step) = s;
        }
    }
}

cudaError_t launch_peer_wait(const PeerWait &W, cudaStream_t stream) {
    cudaLaunchConfig_t cfg{};
    cfg.gridDim = dim3((unsigned)std::min<long long>(1024, std::max<long long>(1, (W.n_entries + 1023) / 1024)));
    cfg.blockDim = dim3(256);
    cfg.stream = stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = W.pdl ? 1 : 0;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, kq_peer_gather_wait, W);
}

}  // namespace kq
