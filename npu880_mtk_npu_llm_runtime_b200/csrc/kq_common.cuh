// kq_common.cuh -- shared device definitions of the B200 K-quant matmul path.
//
// Device weight layout: row-group tiles.  Rows are taken 16 at a time (the last group is
// zero-padded); row group rg holds one tile per 256-value unit u = 0 .. K/256-1, stored
// [rg][u][tile], so any run of consecutive tiles is one contiguous cp.async.bulk copy.  A tile
// holds the unit's bytes of its 16 rows one row after another, each row 16-byte aligned at a
// stride that is an odd multiple of 16 bytes (so 8 rows read at the same column fall in 8
// different bank groups -- conflict-free per-row loads and ldmatrix):
//   Q4_K  16 x 144 B GGUF blocks                                    (2304 B)
//   Q5_K  16 x 176 B GGUF blocks                                    (2816 B)
//   Q6_K  16 x 208 B (ql[128] qh[64] scales[16]), then 16 fp16 d     (3360 B)
//   Q8_0  16 x 272 B: the eight fp16 d of the row's 8 blocks, then their 256 quants (4352 B)
// tile_byte_offset() is the exact map from a GGUF byte to its place in a tile.
#pragma once

#include <cstddef>
#include <cstdint>
#include <cuda_fp16.h>

namespace kq {

constexpr int TYPE_Q8_0 = 8;
constexpr int TYPE_Q4_K = 12;
constexpr int TYPE_Q5_K = 13;
constexpr int TYPE_Q6_K = 14;

// device-side error codes written to the context's status word
constexpr int DEV_OK = 0;
constexpr int DEV_ERR_TIMEOUT = 1;
constexpr int DEV_ERR_INDEX = 2;  // a row id past the end of a weight (the access was skipped)

// BlockQ8K of the reference (ENG:868-872): 292 bytes
struct BlockQ8K {
    float d;
    int8_t qs[256];
    int32_t bsum32[8];
};
static_assert(sizeof(BlockQ8K) == 292, "BlockQ8K layout");

// BlockQ8_0_Fast of the reference (ENG:874-877): 36 bytes
struct BlockQ80 {
    float d;
    int8_t qs[32];
};
static_assert(sizeof(BlockQ80) == 36, "BlockQ8_0_Fast layout");

__host__ __device__ constexpr int block_bytes(int type) {
    return type == TYPE_Q4_K ? 144 : type == TYPE_Q5_K ? 176 : type == TYPE_Q6_K ? 210 : type == TYPE_Q8_0 ? 34 : 0;
}
__host__ __device__ constexpr int block_elems(int type) { return type == TYPE_Q8_0 ? 32 : 256; }

// GGUF bytes of 256 values (one tile row)
__host__ __device__ constexpr int unit_bytes(int type) {
    return type == TYPE_Q4_K ? 144 : type == TYPE_Q5_K ? 176 : type == TYPE_Q6_K ? 210 : type == TYPE_Q8_0 ? 272 : 0;
}
__host__ __device__ constexpr int tile_bytes(int type) { return 16 * unit_bytes(type); }

// device bytes of a rows x K weight (K % 256 == 0)
__host__ __device__ inline size_t weight_bytes(int type, int rows, int K) {
    return (size_t)((rows + 15) / 16) * (size_t)(K / 256) * (size_t)tile_bytes(type);
}

// Offset in the tiled tensor of byte ob of GGUF row `row` (ob counts from the start of the
// row's GGUF bytes).
__host__ __device__ inline size_t tile_byte_offset(int type, int nbu, int row, size_t ob) {
    const int rr = row & 15;
    size_t u, off;
    if (type == TYPE_Q8_0) {
        const size_t blk = ob / 34, o = ob % 34;
        u = blk / 8;
        const size_t jj = blk % 8;
        off = 272 * rr + (o < 2 ? 2 * jj + o : 16 + 32 * jj + (o - 2));
    } else {
        const int bb = unit_bytes(type);
        u = ob / bb;
        const size_t o = ob % bb;
        if (type == TYPE_Q6_K) off = (o < 208) ? 208 * rr + o : 3328 + 2 * rr + (o - 208);
        else off = (size_t)bb * rr + o;
    }
    return ((size_t)(row >> 4) * nbu + u) * (size_t)tile_bytes(type) + off;
}

// ------------------------------------------------------------------ PTX helpers

__device__ __forceinline__ uint32_t smem_u32(const void *p) {
    return (uint32_t)__cvta_generic_to_shared(p);
}

__device__ __forceinline__ uint64_t global_timer_ns() {
    uint64_t t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}

__device__ __forceinline__ void mbar_init(uint32_t bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(bar), "r"(count));
}

__device__ __forceinline__ void mbar_init_fence() {
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint32_t bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(bar), "r"(bytes) : "memory");
}

__device__ __forceinline__ void mbar_arrive(uint32_t bar) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(bar) : "memory");
}

// `count` arrivals at once
__device__ __forceinline__ void mbar_arrive_cnt(uint32_t bar, uint32_t count) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0], %1;" ::"r"(bar), "r"(count) : "memory");
}

// Non-blocking probe: has the phase with this parity completed?
__device__ __forceinline__ bool mbar_test_wait(uint32_t bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{ .reg .pred p; mbarrier.test_wait.parity.shared::cta.b64 p, [%1], %2; selp.u32 %0, 1, 0, p; }"
        : "=r"(ok)
        : "r"(bar), "r"(parity)
        : "memory");
    return ok != 0;
}

__device__ __forceinline__ bool mbar_try_wait(uint32_t bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{ .reg .pred p; mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2; selp.u32 %0, 1, 0, p; }"
        : "=r"(ok)
        : "r"(bar), "r"(parity)
        : "memory");
    return ok != 0;
}

// try_wait with a suspend-time hint: the thread sleeps until the phase completes or about
// hint_ns passes, instead of spinning and taking issue slots from the warps doing the work.
__device__ __forceinline__ bool mbar_try_wait_sleep(uint32_t bar, uint32_t parity, uint32_t hint_ns) {
    uint32_t ok;
    asm volatile(
        "{ .reg .pred p; mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3; selp.u32 %0, 1, 0, p; }"
        : "=r"(ok)
        : "r"(bar), "r"(parity), "r"(hint_ns)
        : "memory");
    return ok != 0;
}

// Record a device-side error in the context's status word (pinned host memory mapped into the
// device: the host reads it after the stream synchronizes, without a copy).  Every writer stores
// the same kind of code, so a plain store suffices.
__device__ __forceinline__ void report_error(int *status, int code) {
    *reinterpret_cast<volatile int *>(status) = code;
    __threadfence_system();
}

// Bounded wait on an mbarrier phase.  Gives up after timeout_ns of wall time, records
// DEV_ERR_TIMEOUT in *status and returns false; never traps.  Polls without a suspend hint
// (a suspended thread wakes up later than a polling one, which costs latency on the critical
// path of a short kernel) and reads the clock every 64 polls.
__device__ __forceinline__ bool mbar_wait_bounded(uint32_t bar, uint32_t parity, uint64_t timeout_ns, int *status) {
    if (mbar_try_wait(bar, parity)) return true;
    const uint64_t t0 = global_timer_ns();
    while (true) {
        for (int i = 0; i < 64; ++i)
            if (mbar_try_wait(bar, parity)) return true;
        if (global_timer_ns() - t0 > timeout_ns) {
            if (status) report_error(status, DEV_ERR_TIMEOUT);
            return false;
        }
    }
}

// Bounded wait that sleeps between polls (suspend-time hint): for kernels whose roles wait on one
// another most of the time, so that waiting warps leave the issue slots to the working ones.
__device__ __forceinline__ bool mbar_wait_bounded_sleep(uint32_t bar, uint32_t parity, uint64_t timeout_ns,
                                                        int *status) {
    if (mbar_try_wait(bar, parity)) return true;
    const uint64_t t0 = global_timer_ns();
    while (true) {
        for (int i = 0; i < 8; ++i)
            if (mbar_try_wait_sleep(bar, parity, 200u)) return true;
        if (global_timer_ns() - t0 > timeout_ns) {
            if (status) report_error(status, DEV_ERR_TIMEOUT);
            return false;
        }
    }
}

// 1-D bulk copy global -> shared (TMA engine), completion counted on an mbarrier.
// dst, src and bytes must be multiples of 16.
__device__ __forceinline__ void bulk_g2s(uint32_t dst, const void *src, uint32_t bytes, uint32_t bar,
                                         uint64_t policy) {
    asm volatile(
        "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint [%0], [%1], %2, [%3], %4;" ::"r"(dst),
        "l"(src), "r"(bytes), "r"(bar), "l"(policy)
        : "memory");
}

// L2 policy for weight streams: read once, evict first (keeps activations/outputs resident).
__device__ __forceinline__ uint64_t l2_evict_first_policy() {
    uint64_t p;
    asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(p));
    return p;
}

// Programmatic dependent launch: let the next kernel in the stream start its prologue, and
// wait for the previous kernel's memory before touching its outputs.
__device__ __forceinline__ void pdl_launch_dependents() { asm volatile("griddepcontrol.launch_dependents;"); }
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }

// Named barrier over the consumer warps (id 1); `threads` must be a multiple of 32.
__device__ __forceinline__ void named_bar_sync(int id, int threads) {
    asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(threads) : "memory");
}

// 4-byte asynchronous copy global -> shared (no register round trip, any number in flight);
// both addresses 4-byte aligned.  The issuing thread waits with cp_async_wait_all.
__device__ __forceinline__ void cp_async4(uint32_t sdst, const void *src) {
    asm volatile("cp.async.ca.shared.global [%0], [%1], 4;" ::"r"(sdst), "l"(src) : "memory");
}
// 16-byte asynchronous copy global -> shared through L2 only (data other CTAs wrote); both
// addresses 16-byte aligned.
__device__ __forceinline__ void cp_async16_cg(uint32_t sdst, const void *src) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(sdst), "l"(src) : "memory");
}
__device__ __forceinline__ void cp_async_wait_all() {
    asm volatile("cp.async.commit_group;\n\tcp.async.wait_group 0;" ::: "memory");
}

// Total order on floats as unsigned keys: larger float -> larger key.
__device__ __forceinline__ unsigned long long argmax_key(float v, uint32_t index) {
    const uint32_t b = __float_as_uint(v);
    const uint32_t o = (b & 0x80000000u) ? ~b : (b | 0x80000000u);
    return ((unsigned long long)o << 32) | (unsigned long long)(0xFFFFFFFFu - index);
}

__device__ __forceinline__ float half_bits_to_float(uint32_t bits16) {
    return __half2float(__ushort_as_half((unsigned short)(bits16 & 0xFFFFu)));
}

__device__ __forceinline__ uint32_t byte_of(uint32_t w, int i) { return (w >> (8 * i)) & 0xFFu; }

// ------------------------------------------------------------------ integer MMA (mma.sync)
// m16n8k32 and m16n8k16, 8-bit operands, int32 accumulate.  Fragments (lane = 4g + t):
// A a0/a1 = rows g / g+8 at k-slots 4t..4t+3, a2/a3 the same rows at 16+4t..16+4t+3 (k32);
// B b0 = k-slots 4t..4t+3 of column g, b1 = 16+4t..; D d0,d1 = row g, columns 2t, 2t+1,
// d2,d3 = row g+8.  Which k a slot stands for is free as long as A and B agree.
__device__ __forceinline__ void mma_k32_u8s8(int (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                                             uint32_t b0, uint32_t b1, int c0, int c1, int c2, int c3) {
    asm("mma.sync.aligned.m16n8k32.row.col.s32.u8.s8.s32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%10,%11,%12,%13};"
        : "=r"(d[0]), "=r"(d[1]), "=r"(d[2]), "=r"(d[3])
        : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1), "r"(c0), "r"(c1), "r"(c2), "r"(c3));
}
__device__ __forceinline__ void mma_k32_s8s8(int (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                                             uint32_t b0, uint32_t b1) {
    asm("mma.sync.aligned.m16n8k32.row.col.s32.s8.s8.s32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%10,%11,%12,%13};"
        : "=r"(d[0]), "=r"(d[1]), "=r"(d[2]), "=r"(d[3])
        : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1), "r"(0), "r"(0), "r"(0), "r"(0));
}
__device__ __forceinline__ void mma_k16_u8s8(int (&d)[4], uint32_t a0, uint32_t a1, uint32_t b0, int c0, int c1,
                                             int c2, int c3) {
    asm("mma.sync.aligned.m16n8k16.row.col.s32.u8.s8.s32 {%0,%1,%2,%3}, {%4,%5}, {%6}, {%7,%8,%9,%10};"
        : "=r"(d[0]), "=r"(d[1]), "=r"(d[2]), "=r"(d[3])
        : "r"(a0), "r"(a1), "r"(b0), "r"(c0), "r"(c1), "r"(c2), "r"(c3));
}

__device__ __forceinline__ uint4 lds128(const void *p) { return *reinterpret_cast<const uint4 *>(p); }
// ldmatrix: four (x4) / two (x2) 8x8 b16 matrices; lane i supplies the address of row i % 8 of
// matrix i / 8; thread 4g+t receives bytes 4t..4t+3 of row g of each matrix.
__device__ __forceinline__ uint4 ldsm_x4(uint32_t saddr) {
    uint4 r;
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
                 : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w)
                 : "r"(saddr));
    return r;
}
__device__ __forceinline__ uint2 ldsm_x2(uint32_t saddr) {
    uint2 r;
    asm volatile("ldmatrix.sync.aligned.m8n8.x2.shared.b16 {%0,%1}, [%2];" : "=r"(r.x), "=r"(r.y) : "r"(saddr));
    return r;
}
// 4-way int8 dot products with 32-bit accumulate (u8 x s8, s8 x s8)
__device__ __forceinline__ int dp4a_us(uint32_t a_u8x4, uint32_t b_s8x4, int c) {
    int d;
    asm("dp4a.u32.s32 %0, %1, %2, %3;" : "=r"(d) : "r"(a_u8x4), "r"(b_s8x4), "r"(c));
    return d;
}
__device__ __forceinline__ int dp4a_ss(uint32_t a, uint32_t b, int c) {
    int d;
    asm("dp4a.s32.s32 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(c));
    return d;
}
__device__ __forceinline__ uint2 lds64(const void *p) { return *reinterpret_cast<const uint2 *>(p); }

// byte k of w, zero-extended / replicated into all four bytes
__device__ __forceinline__ int ubyte(uint32_t w, int k) { return (int)__byte_perm(w, 0u, 0x4440u | (unsigned)k); }
__device__ __forceinline__ uint32_t rep_byte(uint32_t w, int k) { return __byte_perm(w, 0u, 0x1111u * (unsigned)k); }
// byte k of w sign-extended (prmt with the sign-replicate selector bit)
__device__ __forceinline__ int sbyte(uint32_t w, int k) {
    int r;
    const unsigned sel = (unsigned)k | ((8u | (unsigned)k) * 0x1110u);
    asm("prmt.b32 %0, %1, 0, %2;" : "=r"(r) : "r"(w), "r"(sel));
    return r;
}

// fp32 outputs of a GEMV also stored into every rank's gather buffer (several GPUs, one process
// each, buffers mapped over NVLink).  A kq_peer_gather region is 256 bytes of control words --
// this rank's completed steps (u64 at 64), the wait kernel's CTA arrivals (u32 at 76) -- then two
// buffers of [M][row_stride] 64-bit entries, used by alternate steps.  Each entry is one aligned
// 64-bit store of (step tag << 32 | fp32 bits): a reader that sees the tag of the step it waits
// for has the value, with no fence or flag between writer and reader.
constexpr int PEER_MAX = 8;
constexpr size_t PEER_CTRL_BYTES = 256;
struct PeerOut {
    int n = 0, rank = 0;
    unsigned long long *buf[PEER_MAX];         // every rank's entries (region + 256)
    const unsigned long long *step = nullptr;  // this rank's completed steps
    long long row_stride = 0, buf_stride = 0;  // entries per row (all rows) / per buffer
    int row0 = 0;                              // global row of local row 0
    // completion inside the GEMV (out != nullptr): the launch's last CTAs wait for the other ranks'
    // entries of this step and write them to out (this rank's rows go there from the epilogue),
    // then the step is counted as completed
    float *out = nullptr;                      // fp32 [M][row_stride]
    int rows = 0, M = 0;                       // this rank's rows, tokens
    unsigned *arrivals = nullptr, *tail_done = nullptr;  // CTA arrivals, tail CTAs finished
    unsigned long long *step_rw = nullptr;     // the completed-steps word, written by the last tail CTA
};

// Bounded read of the tagged entries src[map(j)] for j in [jb, je), four per thread at a time,
// into out[map(j)] (when out is set): an entry without `tag` yet is read again.  On timeout the
// thread records DEV_ERR_TIMEOUT and sets *fail, which the other threads see and stop waiting.
template <class Map>
__device__ __forceinline__ void peer_collect(const unsigned long long *src, uint32_t tag, long long jb, long long je,
                                             int tid, int nthreads, Map map, float *out, uint64_t t0,
                                             unsigned long long timeout_ns, int *status, volatile int *fail) {
    for (long long j0 = jb + 4ll * tid; j0 < je; j0 += 4ll * nthreads) {
        unsigned long long e[4];
        long long o[4];
#pragma unroll
        for (int k = 0; k < 4; ++k) {
            o[k] = (j0 + k < je) ? map(j0 + k) : 0;
            if (j0 + k < je) asm volatile("ld.relaxed.sys.global.u64 %0, [%1];" : "=l"(e[k]) : "l"(src + o[k]) : "memory");
        }
#pragma unroll
        for (int k = 0; k < 4; ++k) {
            if (j0 + k >= je) break;
            int polls = 0;
            while ((uint32_t)(e[k] >> 32) != tag) {
                if ((++polls & 63) == 0) {
                    if (*fail) break;
                    if (global_timer_ns() - t0 > timeout_ns) {
                        report_error(status, DEV_ERR_TIMEOUT);
                        *fail = 1;
                        break;
                    }
                }
                asm volatile("ld.relaxed.sys.global.u64 %0, [%1];" : "=l"(e[k]) : "l"(src + o[k]) : "memory");
            }
            if (out) out[o[k]] = __uint_as_float((uint32_t)e[k]);
        }
    }
}

// The step the current launch produces: one more than the steps this rank completed (written by
// an earlier kernel, constant during this one: read through the read-only cache).
__device__ __forceinline__ unsigned long long peer_step(const PeerOut &po) { return __ldg(po.step) + 1ull; }

__device__ __forceinline__ void peer_store(unsigned long long *p, float v, uint32_t tag) {
    const unsigned long long e = ((unsigned long long)tag << 32) | (unsigned long long)__float_as_uint(v);
    asm volatile("st.relaxed.sys.global.u64 [%0], %1;" ::"l"(p), "l"(e) : "memory");
}

// Bounded wait until *p >= v (a shared-memory counter other warps advance).
__device__ __forceinline__ bool wait_ge_bounded(const int *p, int v, uint64_t timeout_ns, int *status) {
    const volatile int *vp = p;
    if (*vp >= v) return true;
    const uint64_t t0 = global_timer_ns();
    while (true) {
        for (int i = 0; i < 64; ++i)
            if (*vp >= v) return true;
        if (global_timer_ns() - t0 > timeout_ns) {
            if (status) report_error(status, DEV_ERR_TIMEOUT);
            return false;
        }
    }
}

}  // namespace kq
