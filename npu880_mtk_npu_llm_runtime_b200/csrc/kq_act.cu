// kq_act.cu -- activation quantizers, fused producers, weight repack and dequant for sm_100a.
//
// All of these are bandwidth-trivial next to the weight stream; they are written so that the
// integer/byte outputs are bit-exact to the reference engine (src/v182_r22_breakthrough_engine.c):
//   quantize_row_fp16_to_q8_k  ENG:925-990    -> kq_quantize<Q8_K>
//   quantize_row_fp16_to_q8_0  ENG:1016-1064  -> kq_quantize<Q8_0>
//   rmsnorm_fp16_rows_fast     ENG:4264-4314  -> kq_rmsnorm_q8k (the sequential fp32 sum)
//   swiglu_fp16_rows_fast      ENG:4326-4383  -> kq_swiglu_q8k (the C library's expf)
//   dequant_block_<type>       ENG:598-853    -> kq_dequant
#include "kq_common.cuh"
#include "kq_internal.h"
#include "kq_rms_seq.cuh"

#include <algorithm>
#include <cmath>
#include <cstring>
#include <mutex>

namespace kq {

// Quantize the 256 values v[8*lane .. 8*lane+7] held by a warp to Q8_K and store a BlockQ8K.
// v are fp32 copies of fp16 values (exact).
__device__ __forceinline__ void warp_store_q8k(const float v[8], BlockQ8K *out, int lane) {
    float amax = 0.0f;
#pragma unroll
    for (int i = 0; i < 8; ++i) amax = fmaxf(amax, fabsf(v[i]));
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
    int q[8];
    if (amax == 0.0f) {
#pragma unroll
        for (int i = 0; i < 8; ++i) q[i] = 0;
    } else {
        const float inv = __fdiv_rn(127.0f, amax);
#pragma unroll
        for (int i = 0; i < 8; ++i) q[i] = max(-127, min(127, __float2int_rn(__fmul_rn(v[i], inv))));
    }
    uint32_t *w = reinterpret_cast<uint32_t *>(out);
    w[1 + 2 * lane] = (uint32_t)(q[0] & 0xFF) | ((uint32_t)(q[1] & 0xFF) << 8) | ((uint32_t)(q[2] & 0xFF) << 16) |
                      ((uint32_t)(q[3] & 0xFF) << 24);
    w[2 + 2 * lane] = (uint32_t)(q[4] & 0xFF) | ((uint32_t)(q[5] & 0xFF) << 8) | ((uint32_t)(q[6] & 0xFF) << 16) |
                      ((uint32_t)(q[7] & 0xFF) << 24);
    int s = q[0] + q[1] + q[2] + q[3] + q[4] + q[5] + q[6] + q[7];
    s += __shfl_xor_sync(0xffffffffu, s, 1);
    s += __shfl_xor_sync(0xffffffffu, s, 2);
    if ((lane & 3) == 0) w[65 + (lane >> 2)] = (uint32_t)s;
    if (lane == 0) out->d = (amax == 0.0f) ? 0.0f : __fdiv_rn(amax, 127.0f);
}

// Same for four Q8_0 blocks per 8 lanes: lanes 4j..4j+3 hold block j of the 256 values.
__device__ __forceinline__ void warp_store_q80(const float v[8], BlockQ80 *out8, int lane) {
    float amax = 0.0f;
#pragma unroll
    for (int i = 0; i < 8; ++i) amax = fmaxf(amax, fabsf(v[i]));
    amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, 1));
    amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, 2));
    int q[8];
    if (amax == 0.0f) {
#pragma unroll
        for (int i = 0; i < 8; ++i) q[i] = 0;
    } else {
        const float inv = __fdiv_rn(127.0f, amax);
#pragma unroll
        for (int i = 0; i < 8; ++i) q[i] = max(-127, min(127, __float2int_rn(__fmul_rn(v[i], inv))));
    }
    const int j = lane >> 2, part = lane & 3;
    uint32_t *w = reinterpret_cast<uint32_t *>(out8 + j);
    w[1 + 2 * part] = (uint32_t)(q[0] & 0xFF) | ((uint32_t)(q[1] & 0xFF) << 8) | ((uint32_t)(q[2] & 0xFF) << 16) |
                      ((uint32_t)(q[3] & 0xFF) << 24);
    w[2 + 2 * part] = (uint32_t)(q[4] & 0xFF) | ((uint32_t)(q[5] & 0xFF) << 8) | ((uint32_t)(q[6] & 0xFF) << 16) |
                      ((uint32_t)(q[7] & 0xFF) << 24);
    if (part == 0) out8[j].d = (amax == 0.0f) ? 0.0f : __fdiv_rn(amax, 127.0f);
}

__device__ __forceinline__ void load8_f16(const __half *p, float v[8]) {
    if ((reinterpret_cast<uintptr_t>(p) & 15) == 0) {
        const uint4 raw = *reinterpret_cast<const uint4 *>(p);
        const __half2 *h2 = reinterpret_cast<const __half2 *>(&raw);
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            const float2 f = __half22float2(h2[i]);
            v[2 * i] = f.x;
            v[2 * i + 1] = f.y;
        }
    } else {
#pragma unroll
        for (int i = 0; i < 8; ++i) v[i] = __half2float(p[i]);
    }
}

// One warp per 256-value unit of one row.
template <int TARGET>
__global__ void __launch_bounds__(256) kq_quantize(const __half *x, long long x_stride, int M, int K, void *out) {
    const int nbu = K / 256;
    const int unit = blockIdx.x * 8 + (threadIdx.x >> 5);
    const int lane = threadIdx.x & 31;
    if (unit >= M * nbu) return;
    const int m = unit / nbu, b = unit % nbu;
    float v[8];
    load8_f16(x + (size_t)m * x_stride + (size_t)b * 256 + 8 * lane, v);
    if (TARGET == TYPE_Q8_0) {
        warp_store_q80(v, reinterpret_cast<BlockQ80 *>(out) + (size_t)m * (K / 32) + 8 * b, lane);
    } else {
        warp_store_q8k(v, reinterpret_cast<BlockQ8K *>(out) + (size_t)m * nbu + b, lane);
    }
}

cudaError_t launch_quantize(int target_type, const void *x, long long x_stride, int M, int K, void *out,
                            cudaStream_t stream) {
    const int units = M * (K / 256);
    if (units == 0) return cudaSuccess;
    const dim3 grid((units + 7) / 8), block(256);
    if (target_type == TYPE_Q8_0)
        kq_quantize<TYPE_Q8_0><<<grid, block, 0, stream>>>(reinterpret_cast<const __half *>(x), x_stride, M, K, out);
    else
        kq_quantize<TYPE_Q4_K><<<grid, block, 0, stream>>>(reinterpret_cast<const __half *>(x), x_stride, M, K, out);
    return cudaGetLastError();
}

// ------------------------------------------------------------------ RMSNorm (+ Q8_K)
//
// x_out = fp16((x * inv_rms) * gamma), inv_rms = 1 / sqrt(sum_sq * (1/K) + 1e-6), every operation
// rounded as in the reference's scalar branch (ENG:4291-4299), where sum_sq is the fp32 sum of
// the squares added one after another in index order: rms_seq_sum (kq_rms_seq.cuh) computes
// exactly that sum with a few dozen short chains instead of one chain of K adds.
constexpr int RMS_THREADS = 1024;
static_assert(RMS_THREADS >= RMS_MIN_THREADS, "threads for the chains");

// Rows up to this length also stage their squares (2 + 4 bytes per value in shared memory).
constexpr int RMS_SQ_MAX_K = 32768;

// One CTA per row; the row is staged in dynamic shared memory (K fp16, then K fp32 squares when
// K <= RMS_SQ_MAX_K).
__global__ void __launch_bounds__(RMS_THREADS) kq_rmsnorm_q8k(const __half *x, const __half *gamma, __half *out,
                                                                  BlockQ8K *q8k, int K) {
    extern __shared__ __align__(16) uint8_t rms_smem[];
    __half *xs = reinterpret_cast<__half *>(rms_smem);
    float *sq = reinterpret_cast<float *>(rms_smem + (size_t)K * 2);  // 16-byte aligned: K % 256 == 0
    const bool have_sq = K <= RMS_SQ_MAX_K;
    __shared__ float s_hsum[RMS_SQ_MAX_K / 128 * 2];  // K / 128 estimates (K <= 65536)
    __shared__ uint4 s_desc[RMS_MAX_SEG * 4];
    __shared__ float s_inv;
    const int m = blockIdx.x, tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const __half *xr = x + (size_t)m * K;
    __half *yr = out + (size_t)m * K;
    const int nbu = K / 256;
    asm volatile("griddepcontrol.wait;" ::: "memory");
    // the next kernel may start now: its weight stream does not depend on this one
    asm volatile("griddepcontrol.launch_dependents;");
    // this warp's first unit of gamma, consumed after the sum: its load latency hides behind it
    float gv[8];
    if (warp < nbu) load8_f16(gamma + warp * 256 + 8 * lane, gv);
    const bool x_al = (reinterpret_cast<uintptr_t>(xr) & 15) == 0;
    for (int i = 8 * tid; i < K; i += 8 * RMS_THREADS) {  // a warp covers whole 256-value units
        uint4 raw;
        if (x_al) {
            raw = *reinterpret_cast<const uint4 *>(xr + i);
        } else {
            uint32_t hv[8];
#pragma unroll
            for (int k = 0; k < 8; ++k) hv[k] = __half_as_ushort(xr[i + k]);
            raw = make_uint4(hv[0] | (hv[1] << 16), hv[2] | (hv[3] << 16), hv[4] | (hv[5] << 16), hv[6] | (hv[7] << 16));
        }
        *reinterpret_cast<uint4 *>(xs + i) = raw;
        const __half2 *h2 = reinterpret_cast<const __half2 *>(&raw);
        float f[8];
#pragma unroll
        for (int k = 0; k < 4; ++k) {
            const float2 v = __half22float2(h2[k]);
            f[2 * k] = __fmul_rn(v.x, v.x);
            f[2 * k + 1] = __fmul_rn(v.y, v.y);
        }
        if (have_sq) {
            *reinterpret_cast<float4 *>(sq + i) = make_float4(f[0], f[1], f[2], f[3]);
            *reinterpret_cast<float4 *>(sq + i + 4) = make_float4(f[4], f[5], f[6], f[7]);
        }
        // estimate of the sum of each 128 values (16 lanes), any order
        float h = ((f[0] + f[1]) + (f[2] + f[3])) + ((f[4] + f[5]) + (f[6] + f[7]));
#pragma unroll
        for (int o = 8; o > 0; o >>= 1) h += __shfl_xor_sync(0xffffffffu, h, o);
        if ((lane & 15) == 0) s_hsum[i / 128] = h;
    }
    __syncthreads();
    auto bar = [] { __syncthreads(); };
    const float ssum = have_sq ? rms_seq_sum(RmsSqF32{sq}, s_hsum, s_desc, K, tid, bar)
                               : rms_seq_sum(RmsSqF16{xs}, s_hsum, s_desc, K, tid, bar);
    if (tid == 0) {
        const float inv_k = __fdiv_rn(1.0f, (float)K);
        s_inv = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fmul_rn(ssum, inv_k), 1.0e-6f)));
    }
    __syncthreads();
    const float inv_rms = s_inv;
    for (int b = warp; b < nbu; b += RMS_THREADS / 32) {
        const int base = b * 256 + 8 * lane;
        if (b != warp) load8_f16(gamma + base, gv);
        float v[8];
        uint32_t packed[4];
#pragma unroll
        for (int i = 0; i < 8; i += 2) {
            const float y0 = __fmul_rn(__fmul_rn(__half2float(xs[base + i]), inv_rms), gv[i]);
            const float y1 = __fmul_rn(__fmul_rn(__half2float(xs[base + i + 1]), inv_rms), gv[i + 1]);
            const __half h0 = __float2half_rn(y0), h1 = __float2half_rn(y1);
            v[i] = __half2float(h0);
            v[i + 1] = __half2float(h1);
            packed[i / 2] = (uint32_t)__half_as_ushort(h0) | ((uint32_t)__half_as_ushort(h1) << 16);
        }
        if ((reinterpret_cast<uintptr_t>(yr + base) & 15) == 0) {
            *reinterpret_cast<uint4 *>(yr + base) = make_uint4(packed[0], packed[1], packed[2], packed[3]);
        } else {
#pragma unroll
            for (int i = 0; i < 4; ++i) *reinterpret_cast<uint32_t *>(yr + base + 2 * i) = packed[i];
        }
        if (q8k) warp_store_q8k(v, q8k + (size_t)m * nbu + b, lane);
    }
}

cudaError_t launch_rmsnorm_q8k(const void *x, const void *gamma, void *out, void *q8k, int M, int K,
                               cudaStream_t stream, bool pdl) {
    if (M == 0) return cudaSuccess;
    // the staged row takes up to 192 KB (K <= 32768: fp16 values and fp32 squares; longer rows
    // only the values, up to 128 KB): raise the kernel's dynamic shared memory limit once per device
    static std::mutex mu;
    static bool configured[64] = {};
    int dev = 0;
    cudaGetDevice(&dev);
    if (dev >= 0 && dev < 64) {
        std::lock_guard<std::mutex> lk(mu);
        if (!configured[dev]) {
            cudaError_t e =
                cudaFuncSetAttribute(kq_rmsnorm_q8k, cudaFuncAttributeMaxDynamicSharedMemorySize, 192 * 1024);
            if (e != cudaSuccess) return e;
            configured[dev] = true;
        }
    }
    cudaLaunchConfig_t cfg{};
    cfg.gridDim = dim3(M);
    cfg.blockDim = dim3(RMS_THREADS);
    cfg.dynamicSmemBytes = (size_t)K * (K <= RMS_SQ_MAX_K ? 6 : 2);
    cfg.stream = stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = pdl ? 1 : 0;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, kq_rmsnorm_q8k, reinterpret_cast<const __half *>(x),
                              reinterpret_cast<const __half *>(gamma), reinterpret_cast<__half *>(out),
                              reinterpret_cast<BlockQ8K *>(q8k), K);
}

// ------------------------------------------------------------------ SwiGLU (+ Q8_K)

// One warp per 256-value unit: gate = fp16((g / (1 + expf(-g))) * u), ENG:4350-4356, then Q8_K
// of the rounded values (ENG:4357).  expf is the C library's, which is not correctly rounded (its
// last bit depends on the library), so its values come from exp_tab: expf(-g) for each of the
// 65,536 fp16 patterns of g, tabulated with the host's expf when the context was created.  With
// exp_tab == nullptr the kernel computes exp in fp64 and rounds once to fp32 (the correctly
// rounded value except in rare double-rounding cases), for callers that want no host table.
__global__ void __launch_bounds__(256) kq_swiglu_q8k(__half *gate, const __half *up, BlockQ8K *q8k, int M, int N,
                                                         const float *exp_tab) {
    asm volatile("griddepcontrol.wait;" ::: "memory");
    asm volatile("griddepcontrol.launch_dependents;");
    const int nbu = N / 256;
    const int unit = blockIdx.x * 8 + (threadIdx.x >> 5);
    const int lane = threadIdx.x & 31;
    if (unit >= M * nbu) return;
    const int m = unit / nbu, b = unit % nbu;
    const size_t off = (size_t)m * N + (size_t)b * 256 + 8 * lane;
    uint16_t gb[8];
    float u[8], v[8];
    if ((reinterpret_cast<uintptr_t>(gate + off) & 15) == 0) {
        const uint4 raw = *reinterpret_cast<const uint4 *>(gate + off);
        const uint32_t w[4] = {raw.x, raw.y, raw.z, raw.w};
#pragma unroll
        for (int i = 0; i < 8; ++i) gb[i] = (uint16_t)(w[i >> 1] >> (16 * (i & 1)));
    } else {
#pragma unroll
        for (int i = 0; i < 8; ++i) gb[i] = __half_as_ushort(gate[off + i]);
    }
    load8_f16(up + off, u);
    uint32_t packed[4];
#pragma unroll
    for (int i = 0; i < 8; i += 2) {
        __half hv[2];
#pragma unroll
        for (int k = 0; k < 2; ++k) {
            const float g = __half2float(__ushort_as_half(gb[i + k]));
            const float e = exp_tab ? __ldg(exp_tab + gb[i + k]) : (float)exp(-(double)g);
            hv[k] = __float2half_rn(__fmul_rn(__fdiv_rn(g, __fadd_rn(1.0f, e)), u[i + k]));
            v[i + k] = __half2float(hv[k]);
        }
        packed[i / 2] = (uint32_t)__half_as_ushort(hv[0]) | ((uint32_t)__half_as_ushort(hv[1]) << 16);
    }
    if ((reinterpret_cast<uintptr_t>(gate + off) & 15) == 0) {
        *reinterpret_cast<uint4 *>(gate + off) = make_uint4(packed[0], packed[1], packed[2], packed[3]);
    } else {
#pragma unroll
        for (int i = 0; i < 4; ++i) *reinterpret_cast<uint32_t *>(gate + off + 2 * i) = packed[i];
    }
    if (q8k) warp_store_q8k(v, q8k + (size_t)m * nbu + b, lane);
}

cudaError_t launch_swiglu_q8k(void *gate, const void *up, void *q8k, int M, int N, cudaStream_t stream, bool pdl,
                              const float *exp_tab) {
    const int units = M * (N / 256);
    if (units == 0) return cudaSuccess;
    cudaLaunchConfig_t cfg{};
    cfg.gridDim = dim3((units + 7) / 8);
    cfg.blockDim = dim3(256);
    cfg.stream = stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = pdl ? 1 : 0;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, kq_swiglu_q8k, reinterpret_cast<__half *>(gate),
                              reinterpret_cast<const __half *>(up), reinterpret_cast<BlockQ8K *>(q8k), M, N, exp_tab);
}

// expf(-g) for every fp16 bit pattern g (the table kq_swiglu_q8k reads), with this host's C
// library -- the expf the reference's scalar SwiGLU calls (ENG:4354).
void fill_swiglu_exp_table(float *tab) {
    for (uint32_t h = 0; h < 65536u; ++h) {
        // binary16 -> binary32, exact
        const uint32_t sign = (h & 0x8000u) << 16, e = (h >> 10) & 0x1Fu, f = h & 0x3FFu;
        uint32_t bits;
        if (e == 0x1F) {
            bits = sign | 0x7F800000u | (f << 13);
        } else if (e != 0) {
            bits = sign | ((e + 112u) << 23) | (f << 13);
        } else if (f == 0) {
            bits = sign;
        } else {  // subnormal: normalise
            int sh = 0;
            uint32_t mnt = f;
            while (!(mnt & 0x400u)) {
                mnt <<= 1;
                ++sh;
            }
            bits = sign | ((uint32_t)(113 - sh) << 23) | ((mnt & 0x3FFu) << 13);
        }
        float g;
        std::memcpy(&g, &bits, 4);
        volatile float ng = -g;  // computed at run time by the library, never folded
        tab[h] = expf(ng);
    }
}

// ------------------------------------------------------------------ weight repack

// GGUF rows -> row-group tiles (kq_common.cuh).  One thread per GGUF byte (the padding rows of
// the last group were zeroed before); runs once per tensor at upload.
__global__ void kq_repack(int type, int nbu, const uint8_t *gguf, uint8_t *dev, int rows, size_t gguf_rb) {
    const size_t total = (size_t)rows * gguf_rb;
    for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < total; i += (size_t)gridDim.x * blockDim.x) {
        const int r = (int)(i / gguf_rb);
        dev[tile_byte_offset(type, nbu, r, i - (size_t)r * gguf_rb)] = gguf[i];
    }
}

cudaError_t launch_repack(int type, const uint8_t *gguf, uint8_t *dev, int rows, int K, cudaStream_t stream) {
    cudaError_t e = cudaMemsetAsync(dev, 0, weight_bytes(type, rows, K), stream);
    if (e != cudaSuccess) return e;
    const size_t rb = (size_t)(K / 256) * unit_bytes(type);
    const size_t total = (size_t)rows * rb;
    const int threads = 256;
    const int blocks = (int)std::min<size_t>((total + threads - 1) / threads, 148 * 64);
    kq_repack<<<blocks, threads, 0, stream>>>(type, K / 256, gguf, dev, rows, rb);
    return cudaGetLastError();
}

// ------------------------------------------------------------------ dequant to fp16

// GGUF byte ob of row r, read from the tiled tensor.
__device__ __forceinline__ uint8_t gguf_byte(int type, int nbu, const uint8_t *t, int r, size_t ob) {
    return t[tile_byte_offset(type, nbu, r, ob)];
}

// One thread per output value of rows [row_begin, row_begin + rows); same rounding sequence as
// the reference's scalar dequant loops.
// ids != nullptr: output row j is weight row ids[j] (an embedding lookup); an id past the
// weight's w_rows rows gives zeros and records DEV_ERR_INDEX (never read out of bounds).
__global__ void kq_dequant(int type, const uint8_t *tiled, int row_begin, int rows, int K, __half *out,
                               const uint32_t *ids, int w_rows, int *status) {
    const int nbu = K / 256;
    const size_t total = (size_t)rows * K;
    for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < total; i += (size_t)gridDim.x * blockDim.x) {
        int r = row_begin + (int)(i / K);
        const int e = (int)(i % K);
        if (ids) {
            const uint32_t id = ids[i / K];
            if (id >= (uint32_t)w_rows) {
                out[i] = __float2half_rn(0.0f);
                if (e == 0 && status) report_error(status, DEV_ERR_INDEX);
                continue;
            }
            r = (int)id;
        }
        float y;
        if (type == TYPE_Q8_0) {
            const size_t b = (size_t)(e / 32) * 34;
            const uint32_t db = gguf_byte(type, nbu, tiled, r, b) | ((uint32_t)gguf_byte(type, nbu, tiled, r, b + 1) << 8);
            y = __fmul_rn(half_bits_to_float(db), (float)(int8_t)gguf_byte(type, nbu, tiled, r, b + 2 + e % 32));
        } else if (type == TYPE_Q6_K) {
            const size_t b = (size_t)(e / 256) * 210;
            const int w = e % 256;
            const int hh = w / 128, g = (w % 128) / 32, l = w % 32;
            const uint8_t ql = gguf_byte(type, nbu, tiled, r, b + 64 * hh + l + 32 * (g & 1));
            const uint8_t qh = gguf_byte(type, nbu, tiled, r, b + 128 + 32 * hh + l);
            const int lo = (g >= 2) ? (ql >> 4) : (ql & 0x0F);
            const int q = (lo | (((qh >> (2 * g)) & 3) << 4)) - 32;
            const int sc = (int)(int8_t)gguf_byte(type, nbu, tiled, r, b + 192 + 8 * hh + 2 * g + (l >= 16));
            const uint32_t db = gguf_byte(type, nbu, tiled, r, b + 208) | ((uint32_t)gguf_byte(type, nbu, tiled, r, b + 209) << 8);
            y = __fmul_rn(__fmul_rn(half_bits_to_float(db), (float)sc), (float)q);
        } else {
            const int bbytes = (type == TYPE_Q4_K) ? 144 : 176;
            const size_t b = (size_t)(e / 256) * bbytes;
            const int w = e % 256;
            const int c = w / 64, hi = (w % 64) / 32, l = w % 32;
            const int j = 2 * c + hi;
            auto sb = [&](int k) { return (int)gguf_byte(type, nbu, tiled, r, b + 4 + k); };
            int sc, mn;
            if (j < 4) {
                sc = sb(j) & 63;
                mn = sb(j + 4) & 63;
            } else {
                sc = (sb(j + 4) & 0x0F) | ((sb(j - 4) >> 6) << 4);
                mn = (sb(j + 4) >> 4) | ((sb(j) >> 6) << 4);
            }
            const size_t qs = (type == TYPE_Q4_K) ? b + 16 : b + 48;
            const uint8_t qb = gguf_byte(type, nbu, tiled, r, qs + 32 * c + l);
            int q = hi ? (qb >> 4) : (qb & 0x0F);
            if (type == TYPE_Q5_K) q += ((gguf_byte(type, nbu, tiled, r, b + 16 + l) >> j) & 1) ? 16 : 0;
            uint32_t dd = 0;
            for (int k = 0; k < 4; ++k) dd |= (uint32_t)gguf_byte(type, nbu, tiled, r, b + k) << (8 * k);
            const float d = half_bits_to_float(dd), dmin = half_bits_to_float(dd >> 16);
            y = __fsub_rn(__fmul_rn(__fmul_rn(d, (float)sc), (float)q), __fmul_rn(dmin, (float)mn));
        }
        out[i] = __float2half_rn(y);
    }
}

cudaError_t launch_dequant(int type, const uint8_t *tiled, int row_begin, int rows, int K, void *out,
                           cudaStream_t stream, const uint32_t *ids, int w_rows, int *status) {
    const size_t total = (size_t)rows * K;
    if (total == 0) return cudaSuccess;
    const int blocks = (int)std::min<size_t>((total + 255) / 256, 148 * 32);
    kq_dequant<<<blocks, 256, 0, stream>>>(type, tiled, row_begin, rows, K, reinterpret_cast<__half *>(out), ids,
                                               w_rows, status);
    return cudaGetLastError();
}

// ------------------------------------------------------------------ argmax keys -> (row, value)

// Argmax keys of stored fp16 logits (the LM head's scan of the fp16 logits, ENG:9699-9707, for
// products that wrote their logits first): keys[m] = max over rows r of argmax_key(logit, r), so
// the largest logit wins and, among equal ones, the first row -- the strict '>' scan.  keys must
// start at 0.  Grid: x over rows, y = token.
__global__ void __launch_bounds__(256) kq_logits_argmax(const __half *logits, long long stride, int rows,
                                                             unsigned long long *keys) {
    const int m = blockIdx.y;
    const __half *lg = logits + (size_t)m * stride;
    unsigned long long best = 0ull;
    const int t = blockIdx.x * blockDim.x + threadIdx.x, nt = gridDim.x * blockDim.x;
    auto scan8 = [&](const uint4 v, int r8) {
        const uint32_t w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
        for (int i = 0; i < 8; ++i) {
            const float f = __half2float(__ushort_as_half((unsigned short)(w[i >> 1] >> (16 * (i & 1)))));
            const unsigned long long k = argmax_key(f, (uint32_t)(8 * r8 + i));
            best = k > best ? k : best;
        }
    };
    if ((rows & 7) == 0 && (stride & 7) == 0 && (reinterpret_cast<uintptr_t>(logits) & 15) == 0) {
        // 8 logits per 16-byte load, two loads in flight per thread
        const int n8 = rows / 8;
        for (int r8 = t; r8 < n8; r8 += 2 * nt) {
            const uint4 v0 = __ldcs(reinterpret_cast<const uint4 *>(lg + 8 * (size_t)r8));
            const bool two = r8 + nt < n8;
            uint4 v1 = make_uint4(0u, 0u, 0u, 0u);
            if (two) v1 = __ldcs(reinterpret_cast<const uint4 *>(lg + 8 * (size_t)(r8 + nt)));
            scan8(v0, r8);
            if (two) scan8(v1, r8 + nt);
        }
    } else {
        for (int r = t; r < rows; r += nt) {
            const unsigned long long k = argmax_key(__half2float(lg[r]), (uint32_t)r);
            best = k > best ? k : best;
        }
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
        const unsigned long long k = __shfl_xor_sync(0xffffffffu, best, o);
        best = k > best ? k : best;
    }
    // one atomic per block: the blocks of a token all update the same key
    __shared__ unsigned long long s_best[8];
    if ((threadIdx.x & 31) == 0) s_best[threadIdx.x >> 5] = best;
    __syncthreads();
    if (threadIdx.x == 0) {
#pragma unroll
        for (int w = 1; w < 8; ++w) best = s_best[w] > best ? s_best[w] : best;
        if (best) atomicMax(&keys[m], best);
    }
}

cudaError_t launch_logits_argmax(const void *logits, long long stride, int rows, int M, unsigned long long *keys,
                                 cudaStream_t stream) {
    if (M <= 0 || rows <= 0) return cudaSuccess;
    const int bx = std::min((rows / 8 + 511) / 512 + 1, 64);
    kq_logits_argmax<<<dim3(bx, M), 256, 0, stream>>>(reinterpret_cast<const __half *>(logits), stride, rows, keys);
    return cudaGetLastError();
}

// keys[m] = (ordered value << 32) | (0xFFFFFFFF - index); index maps through ids when given.  When
// `status` is given and holds an error (a product kernel stopped early on a wait timeout), every
// row gets the "no result" sentinel instead: token 0xFFFFFFFF, value NaN.
__global__ void kq_argmax_finalize(const unsigned long long *keys, int M, const uint32_t *ids, uint32_t *toks,
                                   float *vals, const int *status) {
    const int m = blockIdx.x * blockDim.x + threadIdx.x;
    if (m >= M) return;
    if (status && *reinterpret_cast<const volatile int *>(status) != DEV_OK) {
        if (toks) toks[m] = 0xFFFFFFFFu;
        if (vals) vals[m] = __int_as_float(0x7FC00000);
        return;
    }
    const unsigned long long k = keys[m];
    if (k == 0ull) {  // no row reported (empty list or a kernel that stopped early)
        if (toks) toks[m] = 0xFFFFFFFFu;
        if (vals) vals[m] = -INFINITY;
        return;
    }
    const uint32_t o = (uint32_t)(k >> 32);
    const uint32_t b = (o & 0x80000000u) ? (o & 0x7FFFFFFFu) : ~o;
    const uint32_t idx = 0xFFFFFFFFu - (uint32_t)(k & 0xFFFFFFFFull);
    if (toks) toks[m] = ids ? ids[idx] : idx;
    if (vals) vals[m] = __uint_as_float(b);
}

cudaError_t launch_argmax_finalize(const unsigned long long *keys, int M, const uint32_t *ids, uint32_t *toks,
                                   float *vals, cudaStream_t stream, const int *status) {
    kq_argmax_finalize<<<(M + 127) / 128, 128, 0, stream>>>(keys, M, ids, toks, vals, status);
    return cudaGetLastError();
}

}  // namespace kq
