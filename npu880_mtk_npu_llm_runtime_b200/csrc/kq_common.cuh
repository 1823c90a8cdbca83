// kq_common.cuh -- shared device definitions of the B200 K-quant matmul path.
//
// Device weight layout (one contiguous row after another, every row 16-byte aligned so a
// stage of consecutive rows is one cp.async.bulk copy):
//   Q4_K : the GGUF bytes unchanged, 144 B per 256 values (16 B header + 128 B nibbles)
//   Q5_K : the GGUF bytes unchanged, 176 B per 256 values
//   Q6_K : per row [nb x 208 B: ql[128] qh[64] scales[16]] [nb x fp16 d] [pad to 16 B]
//          (the GGUF block is ql, qh, scales, d = 210 B; d moves to a per-row plane so the
//          208-byte remainder stays 16-byte aligned)
//   Q8_0 : per row [K int8 quants] [K/32 x fp16 d] [pad to 16 B]
// Activations are staged per (token, 256-value unit) in shared memory as kq::ActUnit.
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

// One token's 256 activation values in shared memory.  368 B = 23 x 16 B: consecutive units
// start in different 16-byte bank groups, so lanes reading different units do not conflict.
struct __align__(16) ActUnit {
    int8_t qs[256];
    int32_t aux[8];     // K-quants: bsum32[8] (sum of each 32 quants); Q8_0: fp32 d of each 32-block
    int32_t xsum16[16]; // sum of each 16 quants (Q6_K's 16-value sub-blocks)
    float d;            // K-quants: the Q8_K block scale
    int32_t pad[3];
};
static_assert(sizeof(ActUnit) == 368, "ActUnit layout");

__host__ __device__ constexpr int block_bytes(int type) {
    return type == TYPE_Q4_K ? 144 : type == TYPE_Q5_K ? 176 : type == TYPE_Q6_K ? 210 : type == TYPE_Q8_0 ? 34 : 0;
}
__host__ __device__ constexpr int block_elems(int type) { return type == TYPE_Q8_0 ? 32 : 256; }

// bytes of one row in the device layout (K % 256 == 0)
__host__ __device__ inline size_t dev_row_bytes(int type, int K) {
    const size_t nbu = (size_t)K / 256;
    switch (type) {
        case TYPE_Q4_K: return nbu * 144;
        case TYPE_Q5_K: return nbu * 176;
        case TYPE_Q6_K: return (nbu * 210 + 15) & ~(size_t)15;
        case TYPE_Q8_0: return ((size_t)K + (size_t)K / 32 * 2 + 15) & ~(size_t)15;
        default: return 0;
    }
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
            if (status) atomicExch(status, DEV_ERR_TIMEOUT);
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

// 4-way int8 dot products with 32-bit accumulate
__device__ __forceinline__ int dp4a_us(uint32_t a_u8x4, int b_s8x4, int c) {
    int d;
    asm("dp4a.u32.s32 %0, %1, %2, %3;" : "=r"(d) : "r"(a_u8x4), "r"(b_s8x4), "r"(c));
    return d;
}
__device__ __forceinline__ int dp4a_ss(int a, int b, int c) { return __dp4a(a, b, c); }

__device__ __forceinline__ float half_bits_to_float(uint32_t bits16) {
    return __half2float(__ushort_as_half((unsigned short)(bits16 & 0xFFFFu)));
}

__device__ __forceinline__ uint32_t byte_of(uint32_t w, int i) { return (w >> (8 * i)) & 0xFFu; }

}  // namespace kq
