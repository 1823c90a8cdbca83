// kq_gemm_tc.cu -- K-quant x Q8_K matrix product for many tokens (prefill, tree verify, batched
// decode) on the 5th-generation tensor cores (tcgen05.mma kind::i8, accumulators in TMEM).
//
// Replaces the engine's batch row kernels (sdot_4rows_<type>_batch, ENG:1336-3106, the SMMLA
// paths) for M > 8 activation rows.  Results equal the reference's bit for bit: every integer
// sub-block sum is exact, and each (row, token) adds the fp32 block terms in block order.
//
// The reference's block arithmetic, sumi = sum_j sc_j * dot_j with 6-bit per-(row, sub-block)
// scales, does not map onto one int8 MMA (sc * q needs 10-12 bits).  It is split into pieces
// that fit a byte, each one MMA over the whole 256-value super-block, recombined exactly in the
// epilogue:
//   Q4_K / Q5_K   sc = 8 sh + sl:  A0 = q * sh, A1 = q * sl (u8);  sumi = 8 D0 + D1.  The mins
//                 term summ = sum_j m_j * bsum_j comes from two K = 32 MMAs: the row's m_0..m_7
//                 against the token's bsum32 split as bsum = 64 bh + bl (bl 0..63, bh -64..63):
//                 D2 = sum_j m_j bl_j, D3 = sum_j m_j bh_j, summ = D2 + 64 D3
//   Q6_K          P = sc * (q - 32) in -3968..4096 for any int8 scale: P = 64 Ph + Pl with
//                 Pl = P & 63 (0..63) and Ph = P >> 6 (-62..64): A0 = Ph, A1 = Pl (s8);
//                 sumi = 64 D0 + D1  (= sum_s sc_s * sum_l (q_l - 32) x_l)
//   Q8_0          A = the quants (s8); one MMA per 32-value block into its own accumulator
// D_i are int32 per (row, token) in TMEM.
//
// CTA: 128 weight rows (8 row groups) x BN tokens, all of K.  Warps 0-7 (two per TMEM lane
// quadrant: each thread half of one row's values, then half of its tokens) build the A operands
// of a super-block from the quantized tiles, thread 0 issues the MMAs, and the same warps run
// the epilogue of the previous super-block while the tensor core works (two TMEM accumulator
// buffers).  Warp 8 streams weight tiles, the activation tile
// (pre-packed in the MMA's K-major layout) and its scales through an S-stage ring with
// cp.async.bulk.  Every wait is bounded.
#include "kq_common.cuh"
#include "kq_internal.h"

#include <algorithm>
#include <mutex>
#include <unordered_map>

namespace kq {

namespace {

constexpr int kTcCompute = 256;  // 8 warps: two per TMEM lane quadrant, each half a row / half the tokens
constexpr int kTcSplitBN = 32;   // largest token tile that may split K
constexpr int kTcQ80SplitUnits = 16;  // Q8_0 rows of at least this many 256-value units may split K
constexpr int kTcThreads = kTcCompute + 32;

// ROWS weight rows (128, or 64 when 128-row CTAs would leave SMs idle) x BN tokens per CTA
template <int TYPE, int BN_, int ROWS_>
struct TcCfg {
    static constexpr int BN = BN_, ROWS = ROWS_;
    static constexpr int RG = ROWS / 16;                                             // row groups per CTA
    static constexpr int NA = (TYPE == TYPE_Q8_0) ? 1 : 2;                      // A operands over K = 256
    static constexpr bool MINS = (TYPE == TYPE_Q4_K || TYPE == TYPE_Q5_K);      // + two K = 32 mins MMAs
    static constexpr int NACC = MINS ? 4 : NA;                                  // accumulators per unit
    static constexpr int DX = (TYPE == TYPE_Q8_0) ? 8 : 1;                      // scales per token and unit
    static constexpr unsigned OPS = (unsigned)ROWS * 256u;                      // bytes of one A operand
    static constexpr unsigned B_BYTES = BN * 256;
    static constexpr unsigned W_BYTES = (unsigned)RG * (unsigned)tile_bytes(TYPE);
    static constexpr unsigned DX_BYTES = BN * DX * 4;
    static constexpr unsigned B2_BYTES = MINS ? BN * 32u : 0u;                   // bsum bytes (bl | bh | 0)
    static constexpr unsigned STAGE = B_BYTES + W_BYTES + DX_BYTES + B2_BYTES;  // multiple of 16
    static constexpr unsigned A2_BYTES = MINS ? 2u * ROWS * 32u : 0u;           // m_j operands (A2a, A2b)
    static constexpr unsigned A_BYTES = NA * OPS + A2_BYTES;
    static constexpr int S_FIT = (int)((200u * 1024u - A_BYTES) / STAGE);
    static constexpr int S = S_FIT < 2 ? 2 : (S_FIT > 6 ? 6 : S_FIT);          // ring stages
    static constexpr unsigned SMEM = A_BYTES + S * STAGE + 1024;
    static_assert((TYPE == TYPE_Q8_0 ? 8 : NACC) * BN <= 256, "accumulator buffer exceeds 256 TMEM columns");
};

struct TcParams {
    const uint8_t *w;          // tiled weight tensor (row group 0)
    int rg_first;              // first row group of the task
    int row_begin, rows;       // output rows = weight rows [row_begin, row_begin + rows)
    int K, nbu, M;
    int n_tok_tiles;           // tiles of BN tokens in the packed activation
    const uint8_t *act;        // packed activation: [token tile][unit][BN * 256] K-major
    const float *dx;           // [token tile][unit][BN * DX] scales
    const uint8_t *bs2;        // Q4_K / Q5_K: [token tile][unit][BN * 32] bsum bytes, K-major (8-row groups 256 B apart)
    __half *dst;
    long long dst_stride;
    const __half *res;
    long long res_stride;
    float *dst_f32;
    long long f32_stride;
    int *status;
    unsigned long long timeout_ns;
    // split K over gridDim.z chunks: each CTA writes the fp32 block terms of its units to
    // terms[u][token][task row] and kq_tc_fold adds them in unit order (nullptr: one chunk)
    float *terms;
};

__device__ __forceinline__ uint64_t umma_desc(uint32_t saddr, uint32_t lbo, uint32_t sbo) {
    // K-major, no swizzle: ((8 rows, n), 2 x 16 B) : ((16 B, SBO), LBO); sm100 descriptor version 1
    return (uint64_t)((saddr >> 4) & 0x3FFFu) | ((uint64_t)((lbo >> 4) & 0x3FFFu) << 16) |
           ((uint64_t)((sbo >> 4) & 0x3FFFu) << 32) | (1ull << 46);
}

// byte offset of (row, k) in a K-major operand of 256 bytes per row: [row/8][k/16][row%8][k%16]
__device__ __forceinline__ uint32_t canon256(int row, int kc16) { return (row >> 3) * 2048 + kc16 * 128 + (row & 7) * 16; }

__device__ __forceinline__ void tc_mma(uint32_t tmem_d, uint64_t da, uint64_t db, uint32_t idesc, uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::i8 [%0], %1, %2, %3, {%5, %6, %7, %8}, p;\n\t}\n" ::"r"(tmem_d),
        "l"(da), "l"(db), "r"(idesc), "r"(accumulate), "r"(0), "r"(0), "r"(0), "r"(0));
}

__device__ __forceinline__ void tc_commit(uint32_t bar) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(bar) : "memory");
}

__device__ __forceinline__ void tmem_ld16(uint32_t taddr, uint32_t (&r)[16]) {
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
          "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
        : "r"(taddr));
}

__device__ __forceinline__ void tmem_ld32(uint32_t taddr, uint32_t (&r)[32]) {
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
        "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
          "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]),
          "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]),
          "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
        : "r"(taddr));
}

// one lane of a converged warp (the MMA is issued by a single thread; converged issue keeps its
// operands in uniform registers)
__device__ __forceinline__ bool elect_one() {
    uint32_t pred;
    asm volatile("{ .reg .pred P; elect.sync _|P, 0xffffffff; selp.u32 %0, 1, 0, P; }" : "=r"(pred));
    return pred != 0;
}

__device__ __forceinline__ void tmem_wait_ld() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void fence_async_smem() { asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); }

// per-byte a - b as int8, for bytes a in [0, 127] and b in [0, 128] (no borrow crosses a byte)
// Q6_K operand bytes of one word of four 6-bit quants q (0..63) for any int8 scale sc:
// P = sc * (q - 32) = 64 Ph + Pl, Pl = P & 63, Ph = P >> 6, as int8 bytes in ph / pl.  Two quants
// at a time in 16-bit lanes: one multiply-add gives V = sc * q + 4096 - 32 sc = P + 4096, whose
// exact value per lane is in 128..8192 (so the 32-bit result, taken modulo 2^32, holds both lanes
// unchanged); then Ph = (V >> 6) - 64 and Pl = V & 63.  Checked on the CPU for every (q, sc).
__device__ __forceinline__ void q6_pieces2(uint32_t q, int sc, uint32_t &ph, uint32_t &pl) {
    const uint32_t k2 = (uint32_t)(4096 - 32 * sc) * 0x00010001u;
    const uint32_t w02 = __byte_perm(q, 0u, 0x4240), w13 = __byte_perm(q, 0u, 0x4341);  // q0|q2<<16, q1|q3<<16
    const uint32_t v02 = w02 * (uint32_t)sc + k2, v13 = w13 * (uint32_t)sc + k2;
    const uint32_t h02 = ((v02 >> 6) + 0x00C000C0u) & 0x00FF00FFu, h13 = ((v13 >> 6) + 0x00C000C0u) & 0x00FF00FFu;
    ph = __byte_perm(h02, h13, 0x6240);
    pl = __byte_perm(v02 & 0x003F003Fu, v13 & 0x003F003Fu, 0x6240);
}

// ---- A operands of one super-block: half hs (values 128 hs .. 128 hs + 127) of row r, from the
// row's tile bytes.  Also returns what the epilogue needs of the row: d (and dmin).

// MINS_K32 (row-major kernel): instead of a third operand of each row's min replicated over its
// sub-block, half hs writes row r of A2a (hs 0: m_0..m_7 at K 0..7) or A2b (hs 1: at K 8..15), the
// rest zero, K-major with 8-row groups 256 bytes apart, after the two K = 256 operands.
template <int TYPE, unsigned OPS = 32768u, bool MINS_K32 = false>
__device__ __forceinline__ void prep_row(const uint8_t *tile, int rr, int hs, uint8_t *A, int r, float &d0, float &d1) {
    if (TYPE == TYPE_Q4_K || TYPE == TYPE_Q5_K) {
        constexpr int RB = (TYPE == TYPE_Q4_K) ? 144 : 176, QS = (TYPE == TYPE_Q4_K) ? 16 : 48;
        const uint8_t *row = tile + RB * rr;
        const uint4 h = lds128(row);
        d0 = half_bits_to_float(h.x);
        d1 = half_bits_to_float(h.x >> 16);
        const uint32_t sc[2] = {h.y & 0x3F3F3F3Fu, (h.w & 0x0F0F0F0Fu) | ((h.y >> 2) & 0x30303030u)};
        const uint32_t mn[2] = {h.z & 0x3F3F3F3Fu, ((h.w >> 4) & 0x0F0F0F0Fu) | ((h.z >> 2) & 0x30303030u)};
        uint32_t qh[8];
        if (TYPE == TYPE_Q5_K) {
            const uint4 a = lds128(row + 16), b = lds128(row + 32);
            qh[0] = a.x, qh[1] = a.y, qh[2] = a.z, qh[3] = a.w, qh[4] = b.x, qh[5] = b.y, qh[6] = b.z, qh[7] = b.w;
        }
        const uint32_t scw = hs ? sc[1] : sc[0], mnw = hs ? mn[1] : mn[0];
        if (MINS_K32) {
            uint8_t *a2 = A + 2 * OPS + (size_t)hs * (OPS / 8) + (r >> 3) * 256 + (r & 7) * 16;
            *reinterpret_cast<uint4 *>(a2) = hs ? make_uint4(0u, 0u, mn[0], mn[1]) : make_uint4(mn[0], mn[1], 0u, 0u);
            *reinterpret_cast<uint4 *>(a2 + 128) = make_uint4(0u, 0u, 0u, 0u);
        }
#pragma unroll
        for (int cc = 0; cc < 2; ++cc) {
            const int c = 2 * hs + cc;
            const uint4 qa = lds128(row + QS + 32 * c), qb = lds128(row + QS + 32 * c + 16);
            const uint32_t w[8] = {qa.x, qa.y, qa.z, qa.w, qb.x, qb.y, qb.z, qb.w};
#pragma unroll
            for (int hi = 0; hi < 2; ++hi) {
                const int j = 2 * c + hi;  // sub-block
                const int s = ubyte(scw, 2 * cc + hi), m = ubyte(mnw, 2 * cc + hi);
                const uint32_t sh = (uint32_t)(s >> 3), sl = (uint32_t)(s & 7), mrep = 0x01010101u * (uint32_t)m;
                uint32_t q[8];
#pragma unroll
                for (int i = 0; i < 8; ++i) {
                    q[i] = hi ? ((w[i] >> 4) & 0x0F0F0F0Fu) : (w[i] & 0x0F0F0F0Fu);
                    if (TYPE == TYPE_Q5_K) q[i] |= ((qh[i] >> j) & 0x01010101u) << 4;
                }
#pragma unroll
                for (int h16 = 0; h16 < 2; ++h16) {  // two 16-byte chunks of the 32-value sub-block
                    const uint32_t o = canon256(r, 2 * j + h16);
                    const uint32_t *qq = q + 4 * h16;
                    *reinterpret_cast<uint4 *>(A + o) = make_uint4(qq[0] * sh, qq[1] * sh, qq[2] * sh, qq[3] * sh);
                    *reinterpret_cast<uint4 *>(A + OPS + o) = make_uint4(qq[0] * sl, qq[1] * sl, qq[2] * sl, qq[3] * sl);
                    if (!MINS_K32) *reinterpret_cast<uint4 *>(A + 2 * OPS + o) = make_uint4(mrep, mrep, mrep, mrep);
                }
            }
        }
    } else if (TYPE == TYPE_Q6_K) {
        const uint8_t *row = tile + 208 * rr;
        d0 = half_bits_to_float(*reinterpret_cast<const uint16_t *>(tile + 3328 + 2 * rr));
        d1 = 0.0f;
        const uint4 s0 = lds128(row + 192);
        const uint32_t scw[4] = {s0.x, s0.y, s0.z, s0.w};
        {
            const int hh = hs;
#pragma unroll
            for (int hf = 0; hf < 2; ++hf) {
                // values 128hh + 32g + 16hf + i, i < 16, for g = 0..3 (sub-block s = 8hh + 2g + hf)
                const uint4 A4 = lds128(row + 64 * hh + 16 * hf), B4 = lds128(row + 64 * hh + 32 + 16 * hf);
                const uint4 H4 = lds128(row + 128 + 32 * hh + 16 * hf);
                const uint32_t av[4] = {A4.x, A4.y, A4.z, A4.w}, bv[4] = {B4.x, B4.y, B4.z, B4.w};
                const uint32_t hv[4] = {H4.x, H4.y, H4.z, H4.w};
#pragma unroll
                for (int g = 0; g < 4; ++g) {
                    const int s = 8 * hh + 2 * g + hf;
                    const int sc = sbyte(hh ? scw[2 + (g >> 1)] : scw[g >> 1], 2 * (g & 1) + hf);
                    uint32_t q[4];
#pragma unroll
                    for (int i = 0; i < 4; ++i) {
                        if (g == 0) q[i] = (av[i] & 0x0F0F0F0Fu) | ((hv[i] << 4) & 0x30303030u);
                        else if (g == 1) q[i] = (bv[i] & 0x0F0F0F0Fu) | ((hv[i] << 2) & 0x30303030u);
                        else if (g == 2) q[i] = ((av[i] >> 4) & 0x0F0F0F0Fu) | (hv[i] & 0x30303030u);
                        else q[i] = ((bv[i] >> 4) & 0x0F0F0F0Fu) | ((hv[i] >> 2) & 0x30303030u);
                    }
                    const uint32_t o = canon256(r, s);  // sub-block s = 16-byte chunk s
                    uint32_t p0[4], p1[4];
#pragma unroll
                    for (int i = 0; i < 4; ++i) q6_pieces2(q[i], sc, p0[i], p1[i]);
                    *reinterpret_cast<uint4 *>(A + o) = make_uint4(p0[0], p0[1], p0[2], p0[3]);
                    *reinterpret_cast<uint4 *>(A + OPS + o) = make_uint4(p1[0], p1[1], p1[2], p1[3]);
                }
            }
        }
    } else {  // Q8_0: row = eight fp16 d, then 256 quants; the scales are read by the caller
        const uint8_t *row = tile + 272 * rr;
        d0 = d1 = 0.0f;
#pragma unroll
        for (int k = 0; k < 8; ++k) {
            const int kc = 8 * hs + k;
            *reinterpret_cast<uint4 *>(A + canon256(r, kc)) = lds128(row + 16 + 16 * kc);
        }
    }
}

// ------------------------------------------------------------------ the kernel

// TMEM load of N consecutive 32-bit columns of this thread's lane (N = 8, 16 or 32)
template <int N>
__device__ __forceinline__ void tmem_ldn(uint32_t taddr, uint32_t (&r)[N]) {
    if constexpr (N == 32) {
        tmem_ld32(taddr, r);
    } else if constexpr (N == 16) {
        tmem_ld16(taddr, r);
    } else {
        static_assert(N == 8, "tmem_ldn: N must be 8, 16 or 32");
        asm volatile("tcgen05.ld.sync.aligned.32x32b.x8.b32 {%0,%1,%2,%3,%4,%5,%6,%7}, [%8];"
                     : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7])
                     : "r"(taddr));
    }
}

template <int TYPE, int BN_, int ROWS_>
__global__ void __launch_bounds__(kTcThreads, 1) kq_gemm_tc(const __grid_constant__ TcParams p) {
    using C = TcCfg<TYPE, BN_, ROWS_>;
    constexpr int BN = C::BN, NA = C::NA, S = C::S, RG = C::RG, ROWS = C::ROWS;
    extern __shared__ __align__(1024) uint8_t smem_raw[];
    uint8_t *smem = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~(uintptr_t)1023);
    __shared__ uint64_t bar_full[S], bar_empty[S], bar_mma[2];
    __shared__ uint32_t s_tmem;
    __shared__ int s_abort;

    uint8_t *A = smem;                      // NA operands of ROWS x 256 bytes
    uint8_t *ring = smem + C::A_BYTES;      // S stages: B | weights | dx
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int tok_tile = blockIdx.x, row_tile = blockIdx.y;
    const int nbu = p.nbu;
    const int rg0 = p.rg_first + RG * row_tile;                        // first row group of the CTA
    const int rg_end = (p.row_begin + p.rows - 1) / 16 + 1;            // past the task's last row group
    const int n_rg = min(RG, rg_end - rg0);
    // units [u0, u0 + nb) of this K chunk (all of K without split)
    const int u0 = (int)((long long)p.nbu * blockIdx.z / gridDim.z);
    const int nb = (int)((long long)p.nbu * (blockIdx.z + 1) / gridDim.z) - u0;

    if (tid == 0) {
        for (int s = 0; s < S; ++s) {
            mbar_init(smem_u32(&bar_full[s]), 1);
            mbar_init(smem_u32(&bar_empty[s]), kTcCompute / 32);  // one arrival per compute warp
        }
        mbar_init(smem_u32(&bar_mma[0]), 1);
        mbar_init(smem_u32(&bar_mma[1]), 1);
        s_abort = 0;
        mbar_init_fence();
    }
    if (warp == 0) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], 512;" ::"r"(smem_u32(&s_tmem)));
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = s_tmem;

    if (warp == kTcCompute / 32) {
        // ---------------- producer
        if (lane == 0) {
            const uint64_t policy = l2_evict_first_policy();
            for (int b = 0; b < nb; ++b) {
                const int st = b % S;
                if (b >= S && !mbar_wait_bounded(smem_u32(&bar_empty[st]), ((b / S) - 1) & 1, p.timeout_ns, p.status)) {
                    s_abort = 1;
                    break;
                }
                const uint32_t full = smem_u32(&bar_full[st]);
                uint8_t *sb = ring + (size_t)st * C::STAGE;
                mbar_arrive_expect_tx(full, C::B_BYTES + (uint32_t)n_rg * (uint32_t)tile_bytes(TYPE) + C::DX_BYTES + C::B2_BYTES);
                const size_t tix = (size_t)tok_tile * nbu + u0 + b;
                bulk_g2s(smem_u32(sb), p.act + tix * C::B_BYTES, C::B_BYTES, full, policy);
                for (int g = 0; g < n_rg; ++g)
                    bulk_g2s(smem_u32(sb + C::B_BYTES + g * tile_bytes(TYPE)),
                             p.w + ((size_t)(rg0 + g) * nbu + u0 + b) * tile_bytes(TYPE), tile_bytes(TYPE), full, policy);
                bulk_g2s(smem_u32(sb + C::B_BYTES + C::W_BYTES), p.dx + tix * (BN * C::DX), C::DX_BYTES, full, policy);
                if (C::MINS)
                    bulk_g2s(smem_u32(sb + C::B_BYTES + C::W_BYTES + C::DX_BYTES), p.bs2 + tix * C::B2_BYTES, C::B2_BYTES,
                             full, policy);
            }
        }
        __syncwarp();
    } else {
        // ---------------- rows: A operands, MMA issue (warp 0), epilogue.  Warp w covers TMEM lane
        // quadrant w % 4 and half w / 4 of each row's values (A operands) and of the tokens
        // (epilogue).  128-row CTAs: row 32 (w % 4) + lane; 64-row CTAs (M = 64 MMA, rows 16 q ..
        // 16 q + 15 in lanes 0-15 of quadrant q): row 16 (w % 4) + lane for lanes 0-15.
        constexpr int BH = BN / 2;
        const int quad = warp & 3, hs = warp >> 2;
        const int r = (ROWS == 128) ? 32 * quad + lane : 16 * quad + (lane & 15);  // weight row within the CTA
        const bool row_lane = (ROWS == 128) || lane < 16;
        const int g = r >> 4, rr = r & 15;
        float acc[BH];
#pragma unroll
        for (int m = 0; m < BH; ++m) acc[m] = 0.0f;
        float dpp[2][2] = {{0.f, 0.f}, {0.f, 0.f}};  // per buffer: d, dmin (Q8_0: block scales, packed)
        uint32_t dqq[2][2] = {{0u, 0u}, {0u, 0u}};
        const uint32_t idesc = (2u << 4) | ((TYPE == TYPE_Q6_K || TYPE == TYPE_Q8_0) ? (1u << 7) : 0u) | (1u << 10) |
                               ((uint32_t)(BN >> 3) << 17) | ((uint32_t)(ROWS >> 4) << 24);
        const uint32_t lane_base = ((uint32_t)(32 * quad) << 16) + (uint32_t)(hs * BH);

        const int lr_out = rg0 * 16 + r - p.row_begin;  // task-local row of this thread
        const bool row_out = row_lane && r < n_rg * 16 && lr_out >= 0 && lr_out < p.rows;
        // block term number q (of the whole row) of token slot i: added in order (one chunk) or
        // stored for the fold
        auto put = [&](int q, int i, float t) {
            if constexpr (kTcSplitBN >= BN) {  // split K is planned only for small token tiles
                if (p.terms) {
                    const int tok = tok_tile * BN + hs * BH + i;
                    if (row_out && tok < p.M) p.terms[((size_t)q * p.M + tok) * p.rows + lr_out] = t;
                    return;
                }
            }
            acc[i] = __fadd_rn(acc[i], t);
        };
        // epilogue of super-block e (its accumulators in buffer e & 1, scales in stage e % S)
        auto epilogue = [&](int e) {
            const int buf = e & 1;
            const float *dxs = reinterpret_cast<const float *>(ring + (size_t)(e % S) * C::STAGE + C::B_BYTES + C::W_BYTES) +
                               hs * BH * C::DX;
            const uint32_t tb = tmem + lane_base + (uint32_t)(buf * 256);
            if (TYPE == TYPE_Q8_0) {
                const uint32_t dw4[4] = {__float_as_uint(dpp[buf][0]), __float_as_uint(dpp[buf][1]), dqq[buf][0], dqq[buf][1]};
                // split K (long rows only): the unit's eight 32-block terms are summed in block
                // order into one term per unit, so the stored terms stay one per unit as for the
                // K-quants -- the same products, fp32 grouped per unit (within 1e-5 of the
                // reference's sequential order); unsplit: each block term in order, exact
                bool unit_terms = false;
                if constexpr (kTcSplitBN >= BN) unit_terms = p.terms != nullptr;
                float ut[BH];
#pragma unroll
                for (int i = 0; i < BH; ++i) ut[i] = 0.0f;
#pragma unroll
                for (int jj = 0; jj < 8; ++jj) {
                    uint32_t D[BH];
                    tmem_ldn<BH>(tb + (uint32_t)(jj * BN), D);
                    tmem_wait_ld();
                    const float dw = half_bits_to_float(dw4[jj >> 1] >> (16 * (jj & 1)));
#pragma unroll
                    for (int i = 0; i < BH; ++i) {
                        const float t = __fmul_rn(__fmul_rn(dw, dxs[i * 8 + jj]), __int2float_rn((int)D[i]));
                        if (unit_terms) ut[i] = __fadd_rn(ut[i], t);
                        else put((u0 + e) * 8 + jj, i, t);
                    }
                }
                if (unit_terms) {
#pragma unroll
                    for (int i = 0; i < BH; ++i) put(u0 + e, i, ut[i]);
                }
            } else {
                // split-capable tiles read the accumulators in chunks of at most 16 token columns
                // (keeps them in registers next to the split bookkeeping)
                constexpr int CW = (BN > kTcSplitBN || BH < 16) ? BH : 16;
                const float d = dpp[buf][0], dmin = dpp[buf][1];
#pragma unroll
                for (int c0 = 0; c0 < BH; c0 += CW) {
                    constexpr int NACC = C::NACC;
                    uint32_t D[NACC][CW];
#pragma unroll
                    for (int a = 0; a < NACC; ++a) tmem_ldn<CW>(tb + (uint32_t)(a * BN + c0), D[a]);
                    tmem_wait_ld();
#pragma unroll
                    for (int i = 0; i < CW; ++i) {
                        const float dx = dxs[c0 + i];
                        float t;
                        if (TYPE == TYPE_Q6_K) {
                            const int sumi = 64 * (int)D[0][i] + (int)D[1][i];
                            t = __fmul_rn(__fmul_rn(d, dx), __int2float_rn(sumi));
                        } else {
                            const int sumi = 8 * (int)D[0][i] + (int)D[1][i];
                            const int summ = (int)D[2][i] + 64 * (int)D[NACC - 1][i];
                            t = __fmul_rn(dx, __fsub_rn(__fmul_rn(d, __int2float_rn(sumi)), __fmul_rn(dmin, __int2float_rn(summ))));
                        }
                        put(u0 + e, c0 + i, t);
                    }
                }
            }
            tc_fence_before();
        };

        // Waits record a failure in s_abort; every warp reads it after the next barrier, so all
        // eight leave the loop together.
        for (int b = 0; b <= nb; ++b) {
            if (b < nb) {
                const int st = b % S;
                int ok = 1;
                if (lane == 0) {
                    ok = mbar_wait_bounded(smem_u32(&bar_full[st]), (b / S) & 1, p.timeout_ns, p.status) &&
                         (b < 1 || mbar_wait_bounded(smem_u32(&bar_mma[(b - 1) & 1]), ((b - 1) >> 1) & 1, p.timeout_ns,
                                                     p.status));
                    if (!ok) s_abort = 1;
                }
                ok = __shfl_sync(0xffffffffu, ok, 0);
                if (ok && row_lane) {
                    // A operands of super-block b (the MMAs of b - 1 have finished reading A)
                    const uint8_t *tile = ring + (size_t)st * C::STAGE + C::B_BYTES + (size_t)min(g, n_rg - 1) * tile_bytes(TYPE);
                    float d0, d1;
                    prep_row<TYPE, C::OPS, C::MINS>(tile, rr, hs, A, r, d0, d1);
                    if (TYPE == TYPE_Q8_0) {
                        const uint4 dv = lds128(tile + 272 * rr);
                        dpp[b & 1][0] = __uint_as_float(dv.x);
                        dpp[b & 1][1] = __uint_as_float(dv.y);
                        dqq[b & 1][0] = dv.z;
                        dqq[b & 1][1] = dv.w;
                    } else {
                        dpp[b & 1][0] = d0;
                        dpp[b & 1][1] = d1;
                    }
                }
                fence_async_smem();
                tc_fence_before();
                named_bar_sync(1, kTcCompute);
                tc_fence_after();
                if (*reinterpret_cast<volatile int *>(&s_abort)) break;
                if (warp == 0) {
                    // converged warp, one elected lane: the MMA operands stay in uniform registers;
                    // the NA accumulator chains are interleaved so the tensor core overlaps them
                    const uint32_t sa = smem_u32(A), sbm = smem_u32(ring + (size_t)st * C::STAGE);
                    const uint32_t td = tmem + (uint32_t)((b & 1) * 256);
                    if (elect_one()) {
                        if (TYPE == TYPE_Q8_0) {
#pragma unroll
                            for (int jj = 0; jj < 8; ++jj)
                                tc_mma(td + (uint32_t)(jj * BN), umma_desc(sa + 256 * jj, 128, 2048),
                                       umma_desc(sbm + 256 * jj, 128, 2048), idesc, 0);
                        } else {
#pragma unroll
                            for (int ks = 0; ks < 8; ++ks)
#pragma unroll
                                for (int a = 0; a < NA; ++a)
                                    tc_mma(td + (uint32_t)(a * BN), umma_desc(sa + a * C::OPS + 256 * ks, 128, 2048),
                                           umma_desc(sbm + 256 * ks, 128, 2048), idesc, ks > 0);
                            if (C::MINS) {
                                // mins: m_j (A2a / A2b) against bl | bh of the token's bsum32 (K = 32)
                                const uint32_t sb2 = sbm + C::B_BYTES + C::W_BYTES + C::DX_BYTES;
                                const uint32_t sa2 = sa + NA * C::OPS;
                                tc_mma(td + (uint32_t)(2 * BN), umma_desc(sa2, 128, 256), umma_desc(sb2, 128, 256), idesc, 0);
                                tc_mma(td + (uint32_t)(3 * BN), umma_desc(sa2 + C::A2_BYTES / 2, 128, 256),
                                       umma_desc(sb2, 128, 256), idesc, 0);
                            }
                        }
                        tc_commit(smem_u32(&bar_mma[b & 1]));
                    }
                    __syncwarp();
                }
            }
            if (b >= 1) {
                // epilogue of b - 1 overlaps the MMAs of b
                const int e = b - 1;
                int ok = 1;
                if (lane == 0) {
                    ok = mbar_wait_bounded(smem_u32(&bar_mma[e & 1]), (e >> 1) & 1, p.timeout_ns, p.status);
                    if (!ok) s_abort = 1;
                }
                ok = __shfl_sync(0xffffffffu, ok, 0);
                tc_fence_after();
                if (ok) epilogue(e);
                // this warp no longer reads the stage of e (its dx, weights, B): the producer refills
                // it after all eight arrivals.  No block barrier here -- a warp that is done starts
                // the A operands of b + 1 while others still read accumulators of e; the barrier
                // after the A operands orders every read of buffer e & 1 before the MMAs that
                // overwrite it, and checks s_abort.
                __syncwarp();
                if (lane == 0) mbar_arrive(smem_u32(&bar_empty[e % S]));
            }
        }
        // results: row r, tokens tok_tile * BN + hs * BH + m
        const int lr = lr_out;
        if (!*reinterpret_cast<volatile int *>(&s_abort) && !(kTcSplitBN >= BN && p.terms) && row_out) {
#pragma unroll
            for (int m = 0; m < BH; ++m) {
                const int tok = tok_tile * BN + hs * BH + m;
                if (tok >= p.M) break;
                if (p.dst_f32) p.dst_f32[(size_t)tok * p.f32_stride + lr] = acc[m];
                if (p.dst) {
                    float v = acc[m];
                    if (p.res) v = __fadd_rn(v, __half2float(p.res[(size_t)tok * p.res_stride + lr]));
                    p.dst[(size_t)tok * p.dst_stride + lr] = __float2half_rn(v);
                }
            }
        }
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    if (warp == 0) asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, 512;" ::"r"(tmem));
    // drain: copies in flight must land before the CTA exits (only after an early stop)
    if (tid == kTcCompute) {
        for (int b = max(0, nb - S); b < nb; ++b)
            mbar_wait_bounded(smem_u32(&bar_full[b % S]), (b / S) & 1, p.timeout_ns, p.status);
    }
}

// Sum of the block terms of one split-K product in unit order (the reference's acc += term
// sequence), then the outputs as the single-chunk epilogue writes them.  One thread per (token,
// task row); terms[u][token][row] with nterm terms per row (one per 256-value unit).
__global__ void kq_tc_fold(const float *terms, int nterm, int M, int rows, __half *dst, long long dst_stride,
                               const __half *res, long long res_stride, float *dst_f32, long long f32_stride) {
    const long long idx = (long long)blockIdx.x * blockDim.x + threadIdx.x;
    if (idx >= (long long)M * rows) return;
    const int tok = (int)(idx / rows), lr = (int)(idx % rows);
    const float *t0 = terms + (size_t)tok * rows + lr;
    const size_t ts = (size_t)M * rows;  // stride between units
    // loads 16 at a time (independent), adds one by one in unit order
    float acc = 0.0f;
    int u = 0;
    for (; u + 16 <= nterm; u += 16) {
        float t[16];
#pragma unroll
        for (int k = 0; k < 16; ++k) t[k] = t0[(size_t)(u + k) * ts];
#pragma unroll
        for (int k = 0; k < 16; ++k) acc = __fadd_rn(acc, t[k]);
    }
    float t[16];
#pragma unroll
    for (int k = 0; k < 16; ++k) t[k] = (u + k < nterm) ? t0[(size_t)(u + k) * ts] : 0.0f;
#pragma unroll
    for (int k = 0; k < 16; ++k)
        if (u + k < nterm) acc = __fadd_rn(acc, t[k]);
    if (dst_f32) dst_f32[(size_t)tok * f32_stride + lr] = acc;
    if (dst) {
        float v = acc;
        if (res) v = __fadd_rn(v, __half2float(res[(size_t)tok * res_stride + lr]));
        dst[(size_t)tok * dst_stride + lr] = __float2half_rn(v);
    }
}

// ------------------------------------------------------------------ activation packing
//
// x fp16 [M][K] -> Q8_K (quantize_row_fp16_to_q8_k, ENG:925-990) or Q8_0 per 32 (ENG:1016-1064),
// written as the MMA's B operand: [token tile][unit][BN tokens x 256 bytes, K-major canonical]
// plus the scales [token tile][unit][token][DX].  Tokens past M are zero.  One warp per (token,
// unit); lane L holds values 8L .. 8L+7.

template <int TYPE, int BN>
__global__ void kq_pack_act(const __half *x, long long x_stride, const void *act, int M, int K, int n_tok_tiles,
                                uint8_t *out, float *dx, uint8_t *bs2) {
    constexpr int DX = (TYPE == TYPE_Q8_0) ? 8 : 1;
    const int nbu = K / 256;
    const int lane = threadIdx.x & 31;
    const long long warps = (long long)gridDim.x * (blockDim.x >> 5);
    for (long long wi = (long long)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
         wi < (long long)n_tok_tiles * BN * nbu; wi += warps) {
        const int m = (int)(wi / nbu), u = (int)(wi % nbu);
        uint32_t lo = 0, hi = 0;
        float d = 0.0f;
        if (m < M) {
            if (x) {
                const __half *xu = x + (size_t)m * x_stride + (size_t)u * 256 + 8 * lane;
                float v[8];
#pragma unroll
                for (int i = 0; i < 8; ++i) v[i] = __half2float(xu[i]);
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
            } else if (TYPE == TYPE_Q8_0) {
                const uint32_t *w = reinterpret_cast<const uint32_t *>(reinterpret_cast<const BlockQ80 *>(act) +
                                                                       ((size_t)m * nbu + u) * 8 + (lane >> 2));
                lo = w[1 + 2 * (lane & 3)];
                hi = w[2 + 2 * (lane & 3)];
                d = __uint_as_float(w[0]);
            } else {
                const uint32_t *w =
                    reinterpret_cast<const uint32_t *>(reinterpret_cast<const BlockQ8K *>(act) + (size_t)m * nbu + u);
                lo = w[1 + 2 * lane];
                hi = w[2 + 2 * lane];
                d = __uint_as_float(w[0]);
            }
        }
        const int tt = m / BN, mm = m % BN;
        const size_t tix = (size_t)tt * nbu + u;
        uint8_t *o = out + tix * (BN * 256) + (mm >> 3) * 2048 + (lane >> 1) * 128 + (mm & 7) * 16 + 8 * (lane & 1);
        *reinterpret_cast<uint2 *>(o) = make_uint2(lo, hi);
        if (TYPE == TYPE_Q8_0) {
            if ((lane & 3) == 0) dx[tix * (BN * DX) + mm * DX + (lane >> 2)] = d;
        } else {
            if (lane == 0) dx[tix * BN + mm] = d;
        }
        if (TYPE == TYPE_Q4_K || TYPE == TYPE_Q5_K) {
            // bsum32 of sub-block j = lane / 4 as bl = bsum & 63 (K = j) and bh = bsum >> 6 (K = 8 + j),
            // K 16..31 zero: one token row of the K = 32 mins operand (8-row groups 256 B apart)
            auto sum4 = [](uint32_t w) {
                return (int)(int8_t)(w & 0xFF) + (int)(int8_t)((w >> 8) & 0xFF) + (int)(int8_t)((w >> 16) & 0xFF) +
                       (int)(int8_t)(w >> 24);
            };
            int bsum = sum4(lo) + sum4(hi);
            bsum += __shfl_xor_sync(0xffffffffu, bsum, 1);
            bsum += __shfl_xor_sync(0xffffffffu, bsum, 2);
            uint8_t *b2 = bs2 + tix * (BN * 32) + (mm >> 3) * 256 + (mm & 7) * 16;
            if ((lane & 3) == 0) {
                const int j = lane >> 2;
                b2[j] = (uint8_t)(bsum & 63);
                b2[8 + j] = (uint8_t)(int8_t)(bsum >> 6);
            }
            if (lane == 0) *reinterpret_cast<uint4 *>(b2 + 128) = make_uint4(0u, 0u, 0u, 0u);
        }
    }
}

template <int TYPE, int BN, int ROWS>
cudaError_t configure_tc() {
    static std::mutex mu;
    static std::unordered_map<int, bool> configured;
    int dev = 0;
    cudaGetDevice(&dev);
    std::lock_guard<std::mutex> lk(mu);
    if (!configured[dev]) {
        cudaError_t e = cudaFuncSetAttribute(kq_gemm_tc<TYPE, BN, ROWS>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                             TcCfg<TYPE, BN, ROWS>::SMEM);
        if (e != cudaSuccess) return e;
        configured[dev] = true;
    }
    return cudaSuccess;
}

// Geometry of one task of the row-major kernel: 64- or 128-row CTAs, and K chunks (split K: block
// terms stored, folded by kq_tc_fold) when the grid would use at most half of the SMs and
// every chunk keeps at least 4 units.  Each candidate is costed per 256-value unit per wave of
// CTAs (B200 timings; Q8_0's eight 32-block accumulators per unit make it the slowest) and the
// cheapest is taken.
struct TcTaskPlan {
    bool r64;
    int ks;
    double us;
};

TcTaskPlan tc_task_plan(int type, int bn, long long n_tok_tiles, long long n_rg, int nbu, int sms) {
    TcTaskPlan best{false, 1, 1e300};
    for (int r64 = 0; r64 < 2; ++r64) {
        const long long ctas = n_tok_tiles * ((n_rg + (r64 ? 3 : 7)) / (r64 ? 4 : 8));
        int ks = 1;
        // Q8_0 splits only long rows (its split terms are per-unit sums, see the epilogue)
        if ((type != TYPE_Q8_0 || nbu >= kTcQ80SplitUnits) && bn <= kTcSplitBN && nbu >= 8 && 2 * ctas <= sms)
            ks = (int)std::max<long long>(1, std::min<long long>(nbu / 4, sms / ctas));
        const bool small = r64 || bn < 64;
        const double unit = (type == TYPE_Q8_0) ? 6.0 : (type == TYPE_Q6_K) ? (small ? 2.5 : 4.2) : (small ? 2.1 : 2.8);
        const double us = (double)((ctas * ks + sms - 1) / sms) * ((nbu + ks - 1) / ks) * unit + (ks > 1 ? 3.0 : 0.0);
        if (us < best.us) best = TcTaskPlan{r64 != 0, ks, us};
    }
    return best;
}

// tokens per CTA of the row-major kernel: the smallest tile that holds M (at most 64; Q8_0 32)
int tc_bn(int type, int M) {
    const int cap = (type == TYPE_Q8_0) ? 32 : 64;
    return M <= 16 ? 16 : (M <= 32 || cap == 32) ? 32 : 64;
}

// Token tile of a launch: the natural one, or 32 where two 32-token tiles with K split beat one
// 64-token tile without (few long rows, e.g. the 2,560 x 9,728 down projection).  The packed
// activation of 32-token tiles never exceeds that of 64-token ones.
int tc_pick_bn(int type, int M, int nbu, const int *task_rgs, int n_tasks, int sms) {
    const int natural = tc_bn(type, M);
    int best = natural;
    double best_us = 1e300;
    for (int bn : {natural, 32}) {
        if (bn > natural) continue;
        const long long tiles = (M + bn - 1) / bn;
        double us = 0.0;
        for (int i = 0; i < n_tasks; ++i) us += tc_task_plan(type, bn, tiles, task_rgs[i], nbu, sms).us;
        if (us < best_us) {
            best_us = us;
            best = bn;
        }
    }
    return best;
}

// fp32 block terms of one split-K task: (terms per row) x M x rows
size_t tc_terms_bytes(int type, int M, int K, int rows) {
    (void)type;  // one term per 256-value unit for every type (Q8_0: the unit's eight block terms summed)
    const size_t nterm = (size_t)(K / 256);
    return nterm * (size_t)M * (size_t)rows * 4;
}

template <int TYPE, int BN>
cudaError_t launch_tc_bn(const TcLaunch &L, cudaStream_t stream) {
    constexpr int DX = (TYPE == TYPE_Q8_0) ? 8 : 1;
    const int nbu = L.K / 256;
    const int n_tok_tiles = (L.M + BN - 1) / BN;
    constexpr size_t B2 = (TYPE == TYPE_Q4_K || TYPE == TYPE_Q5_K) ? 32 : 0;  // bsum bytes per token
    const size_t need = (size_t)n_tok_tiles * nbu * ((size_t)BN * 256 + (size_t)BN * DX * 4 + (size_t)BN * B2);
    if (L.scratch_bytes < need) return cudaErrorInvalidValue;
    uint8_t *act = reinterpret_cast<uint8_t *>(L.scratch);
    float *dx = reinterpret_cast<float *>(act + (size_t)n_tok_tiles * nbu * BN * 256);
    uint8_t *bs2 = reinterpret_cast<uint8_t *>(dx + (size_t)n_tok_tiles * nbu * BN * DX);
    {
        const long long items = (long long)n_tok_tiles * BN * nbu;
        const int blocks = (int)std::min<long long>((items + 7) / 8, 148 * 16);
        kq_pack_act<TYPE, BN><<<blocks, 256, 0, stream>>>(reinterpret_cast<const __half *>(L.x), L.x_stride, L.act,
                                                               L.M, L.K, n_tok_tiles, act, dx, bs2);
        cudaError_t e = cudaGetLastError();
        if (e != cudaSuccess) return e;
    }
    const int sms = L.num_sms > 0 ? L.num_sms : 148;
    size_t terms_used = 0;
    for (int i = 0; i < L.n_tasks; ++i) {
        const GemvTaskHost &h = L.tasks[i];
        if (h.rows <= 0) continue;
        TcParams p{};
        p.w = h.w;
        p.rg_first = h.row_begin / 16;
        p.row_begin = h.row_begin;
        p.rows = h.rows;
        p.K = L.K;
        p.nbu = nbu;
        p.M = L.M;
        p.n_tok_tiles = n_tok_tiles;
        p.act = act;
        p.dx = dx;
        p.bs2 = bs2;
        p.dst = reinterpret_cast<__half *>(h.dst);
        p.dst_stride = h.dst_stride;
        p.res = reinterpret_cast<const __half *>(h.res);
        p.res_stride = h.res_stride;
        p.dst_f32 = h.dst_f32;
        p.f32_stride = h.f32_stride;
        p.status = L.status;
        p.timeout_ns = L.timeout_ns;
        const int n_rg = (h.row_begin + h.rows - 1) / 16 - p.rg_first + 1;
        const TcTaskPlan tp = tc_task_plan(TYPE, BN, n_tok_tiles, n_rg, nbu, sms);
        const bool rows64 = tp.r64;
        const int ks = tp.ks;
        if (ks > 1) {
            if (!L.terms || L.terms_bytes < terms_used + tc_terms_bytes(TYPE, L.M, L.K, h.rows)) return cudaErrorInvalidValue;
            p.terms = reinterpret_cast<float *>(reinterpret_cast<uint8_t *>(L.terms) + terms_used);
            terms_used += tc_terms_bytes(TYPE, L.M, L.K, h.rows);
        }
        cudaError_t e;
        if (rows64) {
            if ((e = configure_tc<TYPE, BN, 64>())) return e;
            kq_gemm_tc<TYPE, BN, 64><<<dim3(n_tok_tiles, (n_rg + 3) / 4, ks), kTcThreads, TcCfg<TYPE, BN, 64>::SMEM, stream>>>(p);
        } else {
            if ((e = configure_tc<TYPE, BN, 128>())) return e;
            kq_gemm_tc<TYPE, BN, 128><<<dim3(n_tok_tiles, (n_rg + 7) / 8, ks), kTcThreads, TcCfg<TYPE, BN, 128>::SMEM, stream>>>(p);
        }
        e = cudaGetLastError();
        if (e != cudaSuccess) return e;
        if (ks > 1) {
            const long long n = (long long)L.M * h.rows;
            kq_tc_fold<<<(unsigned)((n + 255) / 256), 256, 0, stream>>>(p.terms, nbu, L.M, h.rows,
                                                                       p.dst, p.dst_stride, p.res, p.res_stride, p.dst_f32,
                                                                       p.f32_stride);
            e = cudaGetLastError();
            if (e != cudaSuccess) return e;
        }
    }
    return cudaSuccess;
}

template <int TYPE>
cudaError_t launch_tc_t(const TcLaunch &L, cudaStream_t stream) {
    int task_rgs[4];
    for (int i = 0; i < L.n_tasks; ++i)
        task_rgs[i] = L.tasks[i].rows > 0 ? (L.tasks[i].row_begin + L.tasks[i].rows - 1) / 16 - L.tasks[i].row_begin / 16 + 1 : 0;
    switch (tc_pick_bn(TYPE, L.M, L.K / 256, task_rgs, L.n_tasks, L.num_sms > 0 ? L.num_sms : 148)) {
        case 16: return launch_tc_bn<TYPE, 16>(L, stream);
        case 32: return launch_tc_bn<TYPE, 32>(L, stream);
        default:
            if constexpr (TYPE != TYPE_Q8_0) return launch_tc_bn<TYPE, 64>(L, stream);
            return cudaErrorInvalidValue;
    }
}


// ================================================================== token-major kernel
//
// For up to 128 tokens per CTA the roles are swapped: the activation quants of one 256-value
// unit are the MMA's A operand (M = 128 token lanes, written to tensor memory with tcgen05.st,
// 64 columns), and the byte-split weight operands of a group of G row groups are the B operand
// in shared memory (N = G x NOP x 16 rows, K-major).  A CTA owns a contiguous range of row groups
// (like the GEMV) and walks the units in order, so every (row, token) adds its block terms in
// block order in the registers of the thread that owns the token's lane.
//
// Items i = (unit u, group of G row groups) in unit-major order flow through four roles:
//   warp 12    producer: activation unit u (quants + scales) and the group's weight tiles (cp.async.bulk)
//   warps 8-11 write activation unit u into TMEM (lane quadrant w % 4 each) and build the B
//              operand of item i (one row group each; Q8_0 items round-robin)
//   warp 13    issues the item's MMAs (converged warp, one elected lane) and commits
//   warps 0-7  epilogue: warp w reads lane quadrant w % 4 for the row groups c of the chunk with
//              c % 2 == w / 4.
// Token t sits in TMEM lane 32 (t % 4) + t / 4, so a small token count still spreads over all
// four lane quadrants and all eight epilogue warps.
// One MMA accumulator chain per item: N = 192 (Q4_K/Q5_K 4 x 48; Q6_K 3 x 32 = 96) keeps the tensor
// core near its peak rate; Q8_0 items are one row group with eight independent 32-block chains.
// TMEM: columns [0, 128) two activation buffers, [128, 512) SD item accumulators.

template <int TYPE>
struct Tc2Cfg {
    static constexpr int NOP = (TYPE == TYPE_Q6_K) ? 2 : (TYPE == TYPE_Q8_0) ? 1 : 3;
    static constexpr int G = (TYPE == TYPE_Q6_K) ? 3 : (TYPE == TYPE_Q8_0) ? 1 : 4;  // row groups per item
    static constexpr int NMMA = (TYPE == TYPE_Q8_0) ? 16 : G * NOP * 16;              // N of one MMA
    static constexpr int NCOL = (TYPE == TYPE_Q8_0) ? 128 : NMMA;                     // D columns per item
    static constexpr int SD = 384 / NCOL;                                             // accumulator slots (2, Q8_0 3)
    static constexpr int SB = SD;                                                     // B operand slots
    static constexpr int SH = 4;                                                      // header slots
    static constexpr int SX = 4;                                                      // activation-scale slots
    static constexpr int RGMAX_C = (TYPE == TYPE_Q6_K) ? 6 : 8;                      // row groups per chunk
    static constexpr unsigned BSLOT = (unsigned)(G * NOP) * 4096u;                    // 16 rows x 256 B per operand
    static constexpr unsigned HDR = (unsigned)G * 256u;                               // per-row scales of an item
    static constexpr int DX = (TYPE == TYPE_Q8_0) ? 8 : 1;
    static constexpr int SW = 4, SAMAX = 8;  // activation slots: as many as fit the region, up to 8
    static constexpr unsigned TB = (unsigned)tile_bytes(TYPE);
    static constexpr unsigned WSLOT = (unsigned)G * TB;
    static constexpr unsigned AROW = 272u;  // padded token row: conflict-free 16-byte reads
    static constexpr unsigned AQ = 128u * AROW;
    static constexpr unsigned AREGION = 2u * (AQ + 128u * DX * 4u);  // two slots of 128 tokens
    static constexpr unsigned OFF_H = SB * BSLOT;
    static constexpr unsigned OFF_A = OFF_H + SH * HDR;
    static constexpr unsigned OFF_X = OFF_A + AREGION;
    static constexpr unsigned XSLOT = 128u * DX * 4u;
    static constexpr unsigned OFF_W = OFF_X + SX * XSLOT;
    static constexpr unsigned SMEM = OFF_W + SW * WSLOT + 1024;
    // b_fmt: Q5_K operands reach 217 (u8), all others fit s8; a_fmt s8 (activation quants)
    static constexpr uint32_t IDESC = (2u << 4) | (1u << 7) | ((TYPE == TYPE_Q5_K) ? 0u : (1u << 10)) |
                                      ((uint32_t)(NMMA >> 3) << 17) | ((128u >> 4) << 24);
};
constexpr int kTc2Threads = 14 * 32;

struct Tc2Task {
    const uint8_t *w;
    int rg_first, rg_start, n_rg;  // tiled row group of the task's first row, its first launch row group, count
    int row_begin, rows;
    __half *dst;
    long long dst_stride;
    const __half *res;
    long long res_stride;
    float *dst_f32;
    long long f32_stride;
};

struct Tc2Params {
    Tc2Task task[4];
    int n_tasks, total_rg, nbu, M;
    const uint8_t *act;  // [token block][unit][128][AROW]
    const float *dx;     // [token block][unit][128][DX]
    int *status;
    unsigned long long timeout_ns;
};

__device__ __forceinline__ int tc2_task_of(const Tc2Params &p, int rg) {
    int t = 0;
#pragma unroll
    for (int i = 1; i < 4; ++i) t += (i < p.n_tasks && rg >= p.task[i].rg_start) ? 1 : 0;
    return t;
}

__device__ __forceinline__ void tmem_st32(uint32_t taddr, const uint32_t (&v)[32]) {
    asm volatile(
        "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,"
        "%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31,%32};" ::"r"(taddr),
        "r"(v[0]), "r"(v[1]), "r"(v[2]), "r"(v[3]), "r"(v[4]), "r"(v[5]), "r"(v[6]), "r"(v[7]), "r"(v[8]), "r"(v[9]),
        "r"(v[10]), "r"(v[11]), "r"(v[12]), "r"(v[13]), "r"(v[14]), "r"(v[15]), "r"(v[16]), "r"(v[17]), "r"(v[18]),
        "r"(v[19]), "r"(v[20]), "r"(v[21]), "r"(v[22]), "r"(v[23]), "r"(v[24]), "r"(v[25]), "r"(v[26]), "r"(v[27]),
        "r"(v[28]), "r"(v[29]), "r"(v[30]), "r"(v[31])
        : "memory");
}
__device__ __forceinline__ void tmem_wait_st() { asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory"); }

__device__ __forceinline__ void tc_mma_ts(uint32_t tmem_d, uint32_t tmem_a, uint64_t db, uint32_t idesc, uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::i8 [%0], [%1], %2, %3, {%5, %6, %7, %8}, p;\n\t}\n" ::"r"(tmem_d),
        "r"(tmem_a), "l"(db), "r"(idesc), "r"(accumulate), "r"(0), "r"(0), "r"(0), "r"(0));
}


template <int TYPE>
__global__ void __launch_bounds__(kTc2Threads, 1) kq_gemm_tc2(const __grid_constant__ Tc2Params p) {
    using C = Tc2Cfg<TYPE>;
    constexpr int SB = C::SB, SD = C::SD, SH = C::SH, SX = C::SX, SW = C::SW, SAM = C::SAMAX, G = C::G, NOP = C::NOP,
                  RGM = C::RGMAX_C;
    constexpr bool COOP = G > 1;  // prep warps share an item (one row group each)
    extern __shared__ __align__(1024) uint8_t smem_raw[];
    uint8_t *smem = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~(uintptr_t)1023);
    __shared__ uint64_t w_full[SW], w_empty[SW], a_full_s[SAM], a_empty_s[SAM], t_full[2], t_empty[2];
    __shared__ uint64_t b_full[SB], b_empty[SB], d_full[SD], d_free[SD], h_free[SH], x_free[SX];
    __shared__ uint32_t s_tmem;
    __shared__ int s_abort;

    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int tb = blockIdx.y, nbu = p.nbu;
    const int Mb = min(128, p.M - 128 * tb);  // tokens of this block
    // activation slot: Mb16 token rows of quants, then their scales; as many slots as fit
    const int Mb16 = (Mb + 15) & ~15;
    const unsigned a_dx_off = (unsigned)Mb16 * C::AROW;
    const unsigned a_slot = (a_dx_off + (unsigned)Mb16 * C::DX * 4u + 127u) & ~127u;
    const int SA = min(SAM, (int)(C::AREGION / a_slot));
    const int rg_lo = (int)((long long)p.total_rg * blockIdx.x / gridDim.x);
    const int rg_hi = (int)((long long)p.total_rg * (blockIdx.x + 1) / gridDim.x);
    const int n_chunks = (rg_hi - rg_lo + RGM - 1) / RGM;

    if (tid == 0) {
        for (int s = 0; s < SW; ++s) {
            mbar_init(smem_u32(&w_full[s]), 1);
            mbar_init(smem_u32(&w_empty[s]), COOP ? 4 : 1);
        }
        for (int s = 0; s < SAM; ++s) {
            mbar_init(smem_u32(&a_full_s[s]), 1);
            mbar_init(smem_u32(&a_empty_s[s]), 4);
        }
        for (int s = 0; s < 2; ++s) {
            mbar_init(smem_u32(&t_full[s]), 4);
            mbar_init(smem_u32(&t_empty[s]), 1);
        }
        for (int s = 0; s < SB; ++s) {
            mbar_init(smem_u32(&b_full[s]), COOP ? 4 : 1);
            mbar_init(smem_u32(&b_empty[s]), 1);
        }
        for (int s = 0; s < SD; ++s) {
            mbar_init(smem_u32(&d_full[s]), 1);
            mbar_init(smem_u32(&d_free[s]), 8);
        }
        for (int s = 0; s < SH; ++s) mbar_init(smem_u32(&h_free[s]), 8);
        for (int s = 0; s < SX; ++s) mbar_init(smem_u32(&x_free[s]), 8);
        s_abort = 0;
        mbar_init_fence();
    }
    if (warp == 0) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], 512;" ::"r"(smem_u32(&s_tmem)));
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = s_tmem;
    volatile int *abort_flag = &s_abort;
    // bounded wait; a timeout stops every role (each checks the flag before its next wait)
    auto wait = [&](uint64_t *bar, uint32_t parity) -> bool {
        if (*abort_flag) return false;
        if (!mbar_wait_bounded_sleep(smem_u32(bar), parity, p.timeout_ns, p.status)) {
            *abort_flag = 1;
            return false;
        }
        return true;
    };
    // chunk ch: row groups [g0, g0 + ng), items of ceil(ng / G) groups per unit
    auto chunk_of = [&](int ch, int &g0, int &ng) {
        g0 = rg_lo + ch * RGM;
        ng = min(RGM, rg_hi - g0);
    };

    if (warp == 12) {
        // ---------------- producer.  Activation units run one unit ahead of the weight tiles, so
        // the epilogue warps, which load unit u + 1 into TMEM before the items of unit u, never wait
        // on tiles that wait on them.
        if (lane == 0) {
            const uint64_t policy = l2_evict_first_policy();
            auto issue_act = [&](int gunit, int u) -> bool {
                const int as = gunit % SA;
                if (!wait(&a_empty_s[as], ((gunit / SA) & 1) ^ 1)) return false;
                const uint32_t qb = (uint32_t)Mb * C::AROW, db = ((uint32_t)Mb * C::DX * 4u + 15u) & ~15u;
                uint8_t *slot = smem + C::OFF_A + (size_t)as * a_slot;
                mbar_arrive_expect_tx(smem_u32(&a_full_s[as]), qb + db);
                const size_t blk = (size_t)tb * nbu + u;
                bulk_g2s(smem_u32(slot), p.act + blk * C::AQ, qb, smem_u32(&a_full_s[as]), policy);
                bulk_g2s(smem_u32(slot + a_dx_off), p.dx + blk * 128 * C::DX, db, smem_u32(&a_full_s[as]), policy);
                return true;
            };
            int i = 0, gu = 0;
            for (int ch = 0; ch < n_chunks && !*abort_flag; ++ch) {
                int g0, ng;
                chunk_of(ch, g0, ng);
                const int ni = (ng + G - 1) / G;
                if (!issue_act(gu, 0)) break;
                for (int u = 0; u < nbu && !*abort_flag; ++u, ++gu) {
                    if (u + 1 < nbu && !issue_act(gu + 1, u + 1)) break;
                    for (int j = 0; j < ni; ++j, ++i) {
                        const int ws = i % SW;
                        if (!wait(&w_empty[ws], ((i / SW) & 1) ^ 1)) break;
                        const int gn = min(G, ng - j * G);
                        mbar_arrive_expect_tx(smem_u32(&w_full[ws]), (uint32_t)gn * C::TB);
                        for (int gi = 0; gi < gn; ++gi) {
                            const int rg = g0 + j * G + gi;
                            const Tc2Task &tk = p.task[tc2_task_of(p, rg)];
                            const size_t tile = (size_t)(tk.rg_first + rg - tk.rg_start) * nbu + u;
                            bulk_g2s(smem_u32(smem + C::OFF_W + (size_t)ws * C::WSLOT + (size_t)gi * C::TB),
                                     tk.w + tile * C::TB, C::TB, smem_u32(&w_full[ws]), policy);
                        }
                    }
                }
            }
        }
    } else if (warp >= 8 && warp < 12) {
        // ---------------- B operands
        // lanes 0-15 take the first half of rows 0-15, lanes 16-31 the second half: the 16-byte
        // stores of 8 consecutive lanes then land in 8 different bank groups
        const int pw = warp - 8, rr = lane & 15, hs = lane >> 4;
        const int tq = 4 * lane + pw;  // token of this thread's TMEM lane (quadrant pw = warp % 4)
        int i = 0, gu = 0;
        for (int ch = 0; ch < n_chunks && !*abort_flag; ++ch) {
            int g0, ng;
            chunk_of(ch, g0, ng);
            const int ni = (ng + G - 1) / G;
            for (int u = 0; u < nbu && !*abort_flag; ++u, ++gu) {
                {
                    // activation unit gu -> TMEM buffer gu & 1
                    const int as = gu % SA, ab = gu & 1;
                    int ok = 1;
                    if (lane == 0)
                        ok = wait(&a_full_s[as], (gu / SA) & 1) && wait(&t_empty[ab], ((gu >> 1) & 1) ^ 1) &&
                             wait(&x_free[gu % SX], ((gu / SX) & 1) ^ 1);
                    ok = __shfl_sync(0xffffffffu, ok, 0);
                    if (!ok) break;
                    tc_fence_after();
                    const uint8_t *row = smem + C::OFF_A + (size_t)as * a_slot + (size_t)tq * C::AROW;
                    {
                        // the token's scales, kept for the epilogue after the activation slot is reused
                        const float *dxs = reinterpret_cast<const float *>(smem + C::OFF_A + (size_t)as * a_slot + a_dx_off);
                        float *dxd = reinterpret_cast<float *>(smem + C::OFF_X + (size_t)(gu % SX) * C::XSLOT);
#pragma unroll
                        for (int b = 0; b < C::DX; ++b) dxd[tq * C::DX + b] = (tq < Mb) ? dxs[tq * C::DX + b] : 0.0f;
                    }
#pragma unroll
                    for (int half = 0; half < 2; ++half) {
                        uint32_t v[32];
#pragma unroll
                        for (int k = 0; k < 8; ++k) {
                            const uint4 w4 = (tq < Mb) ? lds128(row + 128 * half + 16 * k) : make_uint4(0u, 0u, 0u, 0u);
                            v[4 * k] = w4.x, v[4 * k + 1] = w4.y, v[4 * k + 2] = w4.z, v[4 * k + 3] = w4.w;
                        }
                        tmem_st32(tmem + ((uint32_t)(32 * pw) << 16) + (uint32_t)(64 * ab + 32 * half), v);
                    }
                    tmem_wait_st();
                    tc_fence_before();
                    __syncwarp();
                    if (lane == 0) {
                        mbar_arrive(smem_u32(&t_full[ab]));
                        mbar_arrive(smem_u32(&a_empty_s[as]));
                    }
                }
                for (int j = 0; j < ni; ++j, ++i) {
                    if (!COOP && (i & 3) != pw) continue;
                    const int ws = i % SW, sb = i % SB, sh = i % SH;
                    int ok = 1;
                    if (lane == 0)
                        ok = wait(&w_full[ws], (i / SW) & 1) && wait(&b_empty[sb], ((i / SB) & 1) ^ 1) &&
                             wait(&h_free[sh], ((i / SH) & 1) ^ 1);
                    ok = __shfl_sync(0xffffffffu, ok, 0);
                    if (!ok) break;
                    const int gi = COOP ? pw : 0;
                    if (gi < min(G, ng - j * G)) {
                        const uint8_t *tile = smem + C::OFF_W + (size_t)ws * C::WSLOT + (size_t)gi * C::TB;
                        uint8_t *B = smem + (size_t)sb * C::BSLOT + (size_t)gi * NOP * 4096;
                        float d0, d1;
                        prep_row<TYPE, 4096u>(tile, rr, hs, B, rr, d0, d1);
                        if (hs == 0) {
                            uint8_t *h = smem + C::OFF_H + (size_t)sh * C::HDR + (size_t)gi * 256;
                            if (TYPE == TYPE_Q8_0) *reinterpret_cast<uint4 *>(h + 16 * rr) = lds128(tile + 272 * rr);
                            else *reinterpret_cast<float2 *>(h + 8 * rr) = make_float2(d0, d1);
                        }
                        fence_async_smem();
                    }
                    __syncwarp();
                    if (lane == 0) {
                        mbar_arrive(smem_u32(&b_full[sb]));
                        mbar_arrive(smem_u32(&w_empty[ws]));
                    }
                }
            }
        }
    } else if (warp == 13) {
        // ---------------- MMA issue (converged warp, elected lane)
        int i = 0, gu = 0;
        for (int ch = 0; ch < n_chunks && !*abort_flag; ++ch) {
            int g0, ng;
            chunk_of(ch, g0, ng);
            const int ni = (ng + G - 1) / G;
            for (int u = 0; u < nbu && !*abort_flag; ++u, ++gu) {
                const int ab = gu & 1;
                if (!wait(&t_full[ab], (gu >> 1) & 1)) break;
                for (int j = 0; j < ni; ++j, ++i) {
                    const int sb = i % SB, sd = i % SD;
                    if (!wait(&b_full[sb], (i / SB) & 1) || !wait(&d_free[sd], ((i / SD) & 1) ^ 1)) break;
                    tc_fence_after();
                    const uint32_t ta = tmem + (uint32_t)(64 * ab), td = tmem + 128u + (uint32_t)(sd * C::NCOL);
                    const uint32_t sbase = smem_u32(smem + (size_t)sb * C::BSLOT);
                    if (elect_one()) {
#pragma unroll
                        for (int ks = 0; ks < 8; ++ks) {
                            if (TYPE == TYPE_Q8_0)
                                tc_mma_ts(td + (uint32_t)(16 * ks), ta + (uint32_t)(8 * ks),
                                          umma_desc(sbase + 256 * ks, 128, 2048), C::IDESC, 0);
                            else
                                tc_mma_ts(td, ta + (uint32_t)(8 * ks), umma_desc(sbase + 256 * ks, 128, 2048), C::IDESC, ks > 0);
                        }
                        tc_commit(smem_u32(&d_full[sd]));
                        tc_commit(smem_u32(&b_empty[sb]));
                        if (j == ni - 1) tc_commit(smem_u32(&t_empty[ab]));
                    }
                    __syncwarp();
                }
            }
        }
    } else {
        // ---------------- epilogue (warps 0-7)
        const int q = warp & 3, h = warp >> 2;
        const int t = 4 * lane + q;      // token of this thread's TMEM lane
        const bool live = q < Mb;        // this quadrant holds tokens of the block
        const uint32_t lane_base = (uint32_t)(32 * q) << 16;
        float acc[4][16];  // chunk row groups c with c % 2 == h, at acc[c / 2]
        float dxr[C::DX];  // the token's scales of the current unit
        int i = 0, gu = 0;
        for (int ch = 0; ch < n_chunks && !*abort_flag; ++ch) {
            int g0, ng;
            chunk_of(ch, g0, ng);
            const int ni = (ng + G - 1) / G;
#pragma unroll
            for (int k = 0; k < 4; ++k)
#pragma unroll
                for (int r = 0; r < 16; ++r) acc[k][r] = 0.0f;
            for (int u = 0; u < nbu; ++u, ++gu) {
                // items of the unit, unrolled so that every accumulator index is a constant
#pragma unroll
                for (int j = 0; j < RGM / G; ++j) {
                    if (j >= ni) break;
                    const int it = i + j, sd = it % SD;
                    int ok = 1;
                    if (lane == 0) ok = wait(&d_full[sd], (it / SD) & 1);
                    ok = __shfl_sync(0xffffffffu, ok, 0);
                    if (!ok) break;
                    tc_fence_after();
                    if (j == 0) {
                        // written by the prep warps before this unit's MMAs were issued
                        const float *dxs = reinterpret_cast<const float *>(smem + C::OFF_X + (size_t)(gu % SX) * C::XSLOT);
#pragma unroll
                        for (int b = 0; b < C::DX; ++b) dxr[b] = dxs[t * C::DX + b];
                    }
                    if (live) {
#pragma unroll
                        for (int gi = 0; gi < G; ++gi) {
                            const int c = j * G + gi;  // row group within the chunk
                            if (c >= ng || (c & 1) != h) continue;
                            const uint8_t *hdr = smem + C::OFF_H + (size_t)(it % SH) * C::HDR + (size_t)gi * 256;
                            const uint32_t td = tmem + lane_base + 128u + (uint32_t)(sd * C::NCOL + gi * NOP * 16);
                            if (TYPE == TYPE_Q8_0) {
                                // the eight 32-block terms of each (row, token), added in block order
#pragma unroll
                                for (int b = 0; b < 8; ++b) {
                                    uint32_t D[16];
                                    tmem_ld16(td + (uint32_t)(16 * b), D);
                                    tmem_wait_ld();
                                    const float dxb = dxr[b];
#pragma unroll
                                    for (int r = 0; r < 16; ++r) {
                                        const uint32_t dw = *reinterpret_cast<const uint32_t *>(hdr + 16 * r + 4 * (b >> 1));
                                        const float wd = half_bits_to_float(dw >> (16 * (b & 1)));
                                        acc[c >> 1][r] = __fadd_rn(acc[c >> 1][r],
                                                                   __fmul_rn(__fmul_rn(wd, dxb), __int2float_rn((int)D[r])));
                                    }
                                }
                            } else {
                                float tm[16];
                                uint32_t D[NOP][16];
#pragma unroll
                                for (int o = 0; o < NOP; ++o) tmem_ld16(td + (uint32_t)(16 * o), D[o]);
                                tmem_wait_ld();
                                const float dx = dxr[0];
#pragma unroll
                                for (int r = 0; r < 16; ++r) {
                                    if (TYPE == TYPE_Q6_K) {
                                        const float d = *reinterpret_cast<const float *>(hdr + 8 * r);
                                        const int sumi = 64 * (int)D[0][r] + (int)D[1][r];
                                        tm[r] = __fmul_rn(__fmul_rn(d, dx), __int2float_rn(sumi));
                                    } else {
                                        const float2 dd = *reinterpret_cast<const float2 *>(hdr + 8 * r);
                                        const int sumi = 8 * (int)D[0][r] + (int)D[1][r];
                                        const int summ = (int)D[2][r];
                                        tm[r] = __fmul_rn(dx, __fsub_rn(__fmul_rn(dd.x, __int2float_rn(sumi)),
                                                                        __fmul_rn(dd.y, __int2float_rn(summ))));
                                    }
                                }
#pragma unroll
                                for (int r = 0; r < 16; ++r) acc[c >> 1][r] = __fadd_rn(acc[c >> 1][r], tm[r]);
                            }
                        }
                    }
                    tc_fence_before();
                    __syncwarp();
                    if (lane == 0) {
                        mbar_arrive(smem_u32(&d_free[sd]));
                        mbar_arrive(smem_u32(&h_free[it % SH]));
                    }
                }
                i += ni;
                __syncwarp();
                if (lane == 0) mbar_arrive(smem_u32(&x_free[gu % SX]));
                if (*abort_flag) break;
            }
            if (*abort_flag) break;
            // results of the chunk: token t, rows of row groups g0 + c (c % 2 == h)
            if (t < Mb) {
                const int tok = 128 * tb + t;
#pragma unroll
                for (int k = 0; k < 4; ++k) {
                    const int c = 2 * k + h;
                    if (c >= ng) break;
                    const int rg = g0 + c;
                    const Tc2Task &tk = p.task[tc2_task_of(p, rg)];
#pragma unroll
                    for (int r = 0; r < 16; ++r) {
                        const int lr = (tk.rg_first + rg - tk.rg_start) * 16 + r - tk.row_begin;
                        if (lr < 0 || lr >= tk.rows) continue;
                        const float v = acc[k][r];
                        if (tk.dst_f32) tk.dst_f32[(size_t)tok * tk.f32_stride + lr] = v;
                        if (tk.dst) {
                            float o = v;
                            if (tk.res) o = __fadd_rn(o, __half2float(tk.res[(size_t)tok * tk.res_stride + lr]));
                            tk.dst[(size_t)tok * tk.dst_stride + lr] = __float2half_rn(o);
                        }
                    }
                }
            }
        }
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    if (warp == 0) asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, 512;" ::"r"(tmem));
    // drain: after an early stop, copies in flight must land before the CTA exits
    if (warp == 12 && lane == 0 && *abort_flag) {
        int items = 0;
        for (int ch = 0; ch < n_chunks; ++ch) {
            int g0, ng;
            chunk_of(ch, g0, ng);
            items += ((ng + G - 1) / G) * nbu;
        }
        const int units = n_chunks * nbu;
        for (int k = max(0, items - SW); k < items; ++k)
            mbar_wait_bounded(smem_u32(&w_full[k % SW]), (k / SW) & 1, p.timeout_ns, nullptr);
        for (int k = max(0, units - SA); k < units; ++k)
            mbar_wait_bounded(smem_u32(&a_full_s[k % SA]), (k / SA) & 1, p.timeout_ns, nullptr);
    }
}

// x fp16 [M][K] (quantized as quantize_row_fp16_to_q8_k / _q8_0) or pre-quantized blocks ->
// [token block][unit][128 tokens][272 B] quants + [token block][unit][128][DX] scales.  One
// warp per (token, unit); lane L holds values 8L .. 8L+7.
template <int TYPE>
__global__ void kq_pack_act2(const __half *x, long long x_stride, const void *act, int M, int K, uint8_t *out,
                                 float *dx) {
    constexpr int DX = Tc2Cfg<TYPE>::DX;
    constexpr unsigned AROW = Tc2Cfg<TYPE>::AROW;
    const int nbu = K / 256;
    const int lane = threadIdx.x & 31;
    const long long warps = (long long)gridDim.x * (blockDim.x >> 5);
    for (long long wi = (long long)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5); wi < (long long)M * nbu;
         wi += warps) {
        const int m = (int)(wi / nbu), u = (int)(wi % nbu);
        uint32_t lo, hi;
        float d;
        if (x) {
            const __half *xu = x + (size_t)m * x_stride + (size_t)u * 256 + 8 * lane;
            float v[8];
#pragma unroll
            for (int k = 0; k < 8; ++k) v[k] = __half2float(xu[k]);
            float amax = 0.0f;
#pragma unroll
            for (int k = 0; k < 8; ++k) amax = fmaxf(amax, fabsf(v[k]));
            constexpr int span = (TYPE == TYPE_Q8_0) ? 4 : 32;
#pragma unroll
            for (int o = 1; o < span; o <<= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
            int qv[8];
            if (amax == 0.0f) {
#pragma unroll
                for (int k = 0; k < 8; ++k) qv[k] = 0;
            } else {
                const float inv = __fdiv_rn(127.0f, amax);
#pragma unroll
                for (int k = 0; k < 8; ++k) qv[k] = max(-127, min(127, __float2int_rn(__fmul_rn(v[k], inv))));
            }
            lo = (uint32_t)(qv[0] & 0xFF) | ((uint32_t)(qv[1] & 0xFF) << 8) | ((uint32_t)(qv[2] & 0xFF) << 16) |
                 ((uint32_t)(qv[3] & 0xFF) << 24);
            hi = (uint32_t)(qv[4] & 0xFF) | ((uint32_t)(qv[5] & 0xFF) << 8) | ((uint32_t)(qv[6] & 0xFF) << 16) |
                 ((uint32_t)(qv[7] & 0xFF) << 24);
            d = (amax == 0.0f) ? 0.0f : __fdiv_rn(amax, 127.0f);
        } else if (TYPE == TYPE_Q8_0) {
            const uint32_t *w = reinterpret_cast<const uint32_t *>(reinterpret_cast<const BlockQ80 *>(act) +
                                                                   ((size_t)m * nbu + u) * 8 + (lane >> 2));
            lo = w[1 + 2 * (lane & 3)];
            hi = w[2 + 2 * (lane & 3)];
            d = __uint_as_float(w[0]);
        } else {
            const uint32_t *w =
                reinterpret_cast<const uint32_t *>(reinterpret_cast<const BlockQ8K *>(act) + (size_t)m * nbu + u);
            lo = w[1 + 2 * lane];
            hi = w[2 + 2 * lane];
            d = __uint_as_float(w[0]);
        }
        const int tb = m >> 7, t = m & 127;
        const size_t blk = (size_t)tb * nbu + u;
        *reinterpret_cast<uint2 *>(out + blk * (128 * AROW) + (size_t)t * AROW + 8 * lane) = make_uint2(lo, hi);
        if (TYPE == TYPE_Q8_0) {
            if ((lane & 3) == 0) dx[(blk * 128 + t) * DX + (lane >> 2)] = d;
        } else {
            if (lane == 0) dx[blk * 128 + t] = d;
        }
    }
}

template <int TYPE>
cudaError_t launch_tc2_t(const TcLaunch &L, cudaStream_t stream) {
    using C = Tc2Cfg<TYPE>;
    const int nbu = L.K / 256;
    const int n_tb = (L.M + 127) / 128;
    const size_t qbytes = (size_t)n_tb * nbu * C::AQ;
    const size_t need = qbytes + (size_t)n_tb * nbu * 128 * C::DX * 4;
    if (L.scratch_bytes < need) return cudaErrorInvalidValue;
    uint8_t *act = reinterpret_cast<uint8_t *>(L.scratch);
    float *dx = reinterpret_cast<float *>(act + qbytes);
    {
        const long long items = (long long)L.M * nbu;
        const int blocks = (int)std::min<long long>((items + 7) / 8, 148 * 16);
        kq_pack_act2<TYPE><<<blocks, 256, 0, stream>>>(reinterpret_cast<const __half *>(L.x), L.x_stride, L.act,
                                                            L.M, L.K, act, dx);
        cudaError_t e = cudaGetLastError();
        if (e != cudaSuccess) return e;
    }
    static std::mutex mu;
    static std::unordered_map<int, bool> configured;
    int dev = 0;
    cudaGetDevice(&dev);
    {
        std::lock_guard<std::mutex> lk(mu);
        if (!configured[dev]) {
            cudaError_t e = cudaFuncSetAttribute(kq_gemm_tc2<TYPE>, cudaFuncAttributeMaxDynamicSharedMemorySize, C::SMEM);
            if (e != cudaSuccess) return e;
            configured[dev] = true;
        }
    }
    Tc2Params p{};
    int total_rg = 0;
    for (int i = 0; i < L.n_tasks; ++i) {
        const GemvTaskHost &h = L.tasks[i];
        if (h.rows <= 0) continue;
        Tc2Task &t = p.task[p.n_tasks++];
        t.w = h.w;
        t.rg_first = h.row_begin / 16;
        t.rg_start = total_rg;
        t.n_rg = (h.row_begin + h.rows - 1) / 16 - t.rg_first + 1;
        t.row_begin = h.row_begin;
        t.rows = h.rows;
        t.dst = reinterpret_cast<__half *>(h.dst);
        t.dst_stride = h.dst_stride;
        t.res = reinterpret_cast<const __half *>(h.res);
        t.res_stride = h.res_stride;
        t.dst_f32 = h.dst_f32;
        t.f32_stride = h.f32_stride;
        total_rg += t.n_rg;
    }
    if (total_rg == 0) return cudaSuccess;
    p.total_rg = total_rg;
    p.nbu = nbu;
    p.M = L.M;
    p.act = act;
    p.dx = dx;
    p.status = L.status;
    p.timeout_ns = L.timeout_ns;
    const int sms = L.num_sms > 0 ? L.num_sms : 148;
    const int gx = std::min(total_rg, std::max((sms + n_tb - 1) / n_tb, (total_rg + C::RGMAX_C - 1) / C::RGMAX_C));
    kq_gemm_tc2<TYPE><<<dim3(gx, n_tb), kTc2Threads, C::SMEM, stream>>>(p);
    return cudaGetLastError();
}

}  // namespace

size_t tc_scratch_bytes(int type, int M, int K) {
    const int nbu = K / 256, bn = tc_bn(type, M), dxn = (type == TYPE_Q8_0) ? 8 : 1;
    const size_t b2 = (type == TYPE_Q4_K || type == TYPE_Q5_K) ? 32 : 0;
    return (size_t)((M + bn - 1) / bn) * nbu * ((size_t)bn * 256 + (size_t)bn * dxn * 4 + (size_t)bn * b2);
}

size_t tc_split_terms_bytes(int type, int M, int K, const int *task_rows, const int *task_rgs, int n_tasks, int sms) {
    const int nbu = K / 256, bn = tc_pick_bn(type, M, nbu, task_rgs, n_tasks, sms);
    const long long tiles = (M + bn - 1) / bn;
    size_t total = 0;
    for (int i = 0; i < n_tasks; ++i)
        if (tc_task_plan(type, bn, tiles, task_rgs[i], nbu, sms).ks > 1) total += tc_terms_bytes(type, M, K, task_rows[i]);
    return total;
}

double tc_estimate_us(int type, int M, int K, const int *task_rgs, int n_tasks, int sms) {
    const int nbu = K / 256, bn = tc_pick_bn(type, M, nbu, task_rgs, n_tasks, sms);
    const long long tiles = (M + bn - 1) / bn;
    double t = 0.0;
    for (int i = 0; i < n_tasks; ++i) t += tc_task_plan(type, bn, tiles, task_rgs[i], nbu, sms).us;
    return t;
}

size_t tc2_scratch_bytes(int type, int M, int K) {
    const size_t blocks = (size_t)((M + 127) / 128) * (K / 256);
    return blocks * (128 * 272 + 128 * (type == TYPE_Q8_0 ? 8 : 1) * 4);
}

cudaError_t launch_gemm_tc2(const TcLaunch &L, cudaStream_t stream) {
    if (L.M < 1 || L.K % 256) return cudaErrorInvalidValue;
    switch (L.type) {
        case TYPE_Q4_K: return launch_tc2_t<TYPE_Q4_K>(L, stream);
        case TYPE_Q5_K: return launch_tc2_t<TYPE_Q5_K>(L, stream);
        case TYPE_Q6_K: return launch_tc2_t<TYPE_Q6_K>(L, stream);
        case TYPE_Q8_0: return launch_tc2_t<TYPE_Q8_0>(L, stream);
        default: return cudaErrorInvalidValue;
    }
}

cudaError_t launch_gemm_tc(const TcLaunch &L, cudaStream_t stream) {
    if (L.M < 1 || L.K % 256) return cudaErrorInvalidValue;
    switch (L.type) {
        case TYPE_Q4_K: return launch_tc_t<TYPE_Q4_K>(L, stream);
        case TYPE_Q5_K: return launch_tc_t<TYPE_Q5_K>(L, stream);
        case TYPE_Q6_K: return launch_tc_t<TYPE_Q6_K>(L, stream);
        case TYPE_Q8_0: return launch_tc_t<TYPE_Q8_0>(L, stream);
        default: return cudaErrorInvalidValue;
    }
}

}  // namespace kq
