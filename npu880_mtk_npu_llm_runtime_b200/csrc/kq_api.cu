// kq_api.cu -- the C ABI of libkq (include/kq.h): contexts, device weights, dispatch.
//
// Host-side replacement of the engine's dispatch layer (sdot_gemm_multi_dispatch and its
// pool, src/v182_r22_breakthrough_engine.c:3442-4262): argument validation, the
// pre-quantized-input state, host<->device staging for the host-pointer entry points, and
// the grouping of tasks into kernel launches.
#include "kq_common.cuh"
#include "kq_internal.h"
#include "../../include/kq.h"

#include <algorithm>
#include <cstdarg>
#include <cstdio>
#include <cstring>
#include <string>
#include <vector>

namespace {

struct DevBuf {
    void *p = nullptr;
    size_t cap = 0;
};

}  // namespace

struct kq_ctx {
    int device = 0;
    cudaStream_t stream = nullptr;
    bool own_stream = false;
    int num_sms = 0;
    int gemm_path = 0;           // M > 8: 0 auto, 1 tensor cores, 2 GEMV in tiles of 8 tokens
    int *h_status = nullptr;     // error word: pinned host memory mapped into the device
    int *d_status = nullptr;     // its device address (kernels write errors there)
    bool pdl = true;
    float *exp_tab = nullptr;    // SwiGLU: expf(-g) for every fp16 g, from this host's C library
    bool swiglu_gpu_exp = false; // option "swiglu_exp" = 1: exp in fp64 on the GPU instead
    bool inject_timeout = false;  // test hook: GEMV consumers wait on a barrier nothing completes
    unsigned long long timeout_ns = 1000000000ull;
    std::string err;

    // scratch (grown on demand, freed at destroy)
    DevBuf x, res, out16, out32, q8k_pending, q8k_cur, q80_cur, tmp, misc, keys, tcpack, tcterms;
    DevBuf lmlogits;  // fp16 logits of a many-token LM head when the caller keeps none
    // balanced GEMV launches: shared-row-group term slots and arrival counts (zero between
    // launches; re-cleared after a launch that stopped early)
    DevBuf gsplit, gcount;  // gcount: the split launches' arrival counts, then the fused FFN's grid barrier
    bool gemv_split = true;
    bool gemv_half = true;  // Q4_K / Q5_K GEMV launches of 1-2 rows: 8-row halves per CTA where better
    bool ffn_fused = true;  // FFN blocks of 1-2 tokens as one persistent kernel where a plan exists
    bool split_dirty = false;
    bool graph_holds_scratch = false;  // a call of this context was captured into a CUDA graph

    // the engine's g_sdot_input state: pending pre-quantized Q8_K input (ENG:4184) and the
    // current input rows for row-level calls (kept as fp16 on the device, quantized lazily)
    bool pending = false;
    int pending_M = 0, pending_K = 0;
    int cur_M = 0, cur_K = 0;
    bool cur_q8k_valid = false, cur_q80_valid = false, cur_x_valid = false;
};

namespace {

int fail(kq_ctx *c, int code, const char *fmt, ...) {
    if (c) {
        char buf[512];
        va_list ap;
        va_start(ap, fmt);
        vsnprintf(buf, sizeof buf, fmt, ap);
        va_end(ap);
        c->err = buf;
    }
    return code;
}

int cuda_fail(kq_ctx *c, cudaError_t e, const char *what) {
    return fail(c, e == cudaErrorMemoryAllocation ? KQ_ERR_OUT_OF_MEMORY : KQ_ERR_CUDA, "%s: %s", what,
                cudaGetErrorString(e));
}

#define KQ_CUDA(ctx, call)                                   \
    do {                                                     \
        cudaError_t e_ = (call);                             \
        if (e_ != cudaSuccess) return cuda_fail(ctx, e_, #call); \
    } while (0)

bool is_kquant(uint32_t t) { return t == KQ_TYPE_Q4_K || t == KQ_TYPE_Q5_K || t == KQ_TYPE_Q6_K; }
bool supported(uint32_t t) { return is_kquant(t) || t == KQ_TYPE_Q8_0; }

// Scratch of at least `bytes`.  A buffer that must grow is freed and allocated again, which a
// CUDA graph captured from this context's calls would not see: work captured into a graph keeps
// the scratch addresses it was recorded with.  So once a call of this context was captured
// (graph_holds_scratch), growing an existing buffer is refused with an error instead, until the
// caller declares the graphs gone (option "graph_released"); a buffer not yet allocated may
// still be allocated outside a capture.  During a capture nothing may be allocated.
int ensure(kq_ctx *c, DevBuf &b, size_t bytes) {
    cudaStreamCaptureStatus cap = cudaStreamCaptureStatusNone;
    if (cudaStreamIsCapturing(c->stream, &cap) != cudaSuccess) cap = cudaStreamCaptureStatusNone;
    if (cap != cudaStreamCaptureStatusNone) c->graph_holds_scratch = true;
    if (b.cap >= bytes) return KQ_OK;
    if (cap != cudaStreamCaptureStatusNone)
        return fail(c, KQ_ERR_INVALID_ARGUMENT,
                    "scratch of %zu bytes needed during stream capture: make one eager call of the largest shape "
                    "before capturing",
                    bytes);
    if (b.p && c->graph_holds_scratch)
        return fail(c, KQ_ERR_INVALID_ARGUMENT,
                    "scratch must grow to %zu bytes but a captured CUDA graph may still use it: destroy those graphs "
                    "and set option \"graph_released\" first",
                    bytes);
    if (b.p) {
        cudaStreamSynchronize(c->stream);
        cudaFree(b.p);
        b.p = nullptr;
        b.cap = 0;
    }
    size_t want = std::max<size_t>(bytes, 4096);
    want = (want + 255) & ~(size_t)255;
    cudaError_t e = cudaMalloc(&b.p, want);
    if (e != cudaSuccess) return cuda_fail(c, e, "cudaMalloc(scratch)");
    b.cap = want;
    return KQ_OK;
}

// Read and clear the device status word after the stream drained.  The word lives in mapped
// pinned host memory, so one synchronize covers the work and the status: no copy.
int check_device_status(kq_ctx *c) {
    cudaError_t e = cudaStreamSynchronize(c->stream);
    if (e != cudaSuccess) return cuda_fail(c, e, "cudaStreamSynchronize");
    volatile int *hs = c->h_status;
    const int st = *hs;
    if (st == kq::DEV_OK) return KQ_OK;
    *hs = kq::DEV_OK;
    c->split_dirty = true;  // a kernel that stopped early may have left arrival counts behind
    if (st == kq::DEV_ERR_TIMEOUT) return fail(c, KQ_ERR_TIMEOUT, "a device-side wait timed out");
    if (st == kq::DEV_ERR_INDEX) return fail(c, KQ_ERR_SHAPE, "a row id is past the end of the weight");
    return fail(c, KQ_ERR_CUDA, "device error code %d", st);
}

int sync_and_check(kq_ctx *c) { return check_device_status(c); }

const float *swiglu_table(const kq_ctx *c) { return c->swiglu_gpu_exp ? nullptr : c->exp_tab; }

int validate_task(kq_ctx *c, const kq_task &t, int K) {
    if (!t.w) return fail(c, KQ_ERR_INVALID_ARGUMENT, "task weight is NULL");
    if (t.w->device != c->device)
        return fail(c, KQ_ERR_INVALID_ARGUMENT, "task weight lives on device %d, the context on device %d", t.w->device,
                    c->device);
    if (t.w->cols != K) return fail(c, KQ_ERR_SHAPE, "task weight has %d columns, input K = %d", t.w->cols, K);
    if (t.rows < 0 || t.row_begin < 0 || (long long)t.row_begin + t.rows > t.w->rows)
        return fail(c, KQ_ERR_SHAPE, "task rows [%d, %d) outside weight rows %d", t.row_begin, t.row_begin + t.rows,
                    t.w->rows);
    if (t.dst && t.dst_stride < (size_t)t.rows) return fail(c, KQ_ERR_INVALID_ARGUMENT, "dst_stride < rows");
    if (t.residual && t.res_stride < (size_t)t.rows) return fail(c, KQ_ERR_INVALID_ARGUMENT, "res_stride < rows");
    if (t.dst_f32 && t.dst_f32_stride < (size_t)t.rows)
        return fail(c, KQ_ERR_INVALID_ARGUMENT, "dst_f32_stride < rows");
    return KQ_OK;
}

// A weight is used only by contexts on the device that holds it.
int check_weight_device(kq_ctx *c, const kq_weight *w) {
    if (w->device != c->device)
        return fail(c, KQ_ERR_INVALID_ARGUMENT, "weight lives on device %d, the context on device %d", w->device,
                    c->device);
    return KQ_OK;
}

int validate_mk(kq_ctx *c, int M, int K) {
    if (M < 1 || M > KQ_MAX_M) return fail(c, KQ_ERR_SHAPE, "M = %d outside [1, %d]", M, KQ_MAX_M);
    if (K < 256 || K > KQ_MAX_K || (K % 256) != 0)
        return fail(c, KQ_ERR_SHAPE, "K = %d must be a positive multiple of 256 up to %d", K, KQ_MAX_K);
    return KQ_OK;
}

// Scratch of a balanced GEMV launch (CTAs own equal tile ranges; see GemvParams::split).  The
// launch keeps whole row groups per CTA when the option is off or the term slots would exceed
// 64 MB (very long Q8_0 rows).
// The arrival counts of balanced launches (gemv_split_slots ints), then the two words of the fused
// FFN kernel's grid barrier and its `extra` pair counts, all zero; cleared again after a launch
// that stopped early.
int split_counts(kq_ctx *c, size_t extra = 0) {
    const size_t cb = sizeof(int) * ((size_t)kq::gemv_split_slots(c->num_sms) + 2 + extra);
    if (!c->gcount.p || c->split_dirty || c->gcount.cap < cb) {
        if (int r = ensure(c, c->gcount, cb)) return r;
        KQ_CUDA(c, cudaMemsetAsync(c->gcount.p, 0, cb, c->stream));
        c->split_dirty = false;
    }
    return KQ_OK;
}

int gemv_split_scratch(kq_ctx *c, int type, int K, int mt, kq::GemvLaunch &L) {
    if (!c->gemv_split) return KQ_OK;
    const size_t bytes = kq::gemv_split_bytes(type, K, mt, c->num_sms);
    if (bytes > ((size_t)64 << 20)) return KQ_OK;
    if (int r = ensure(c, c->gsplit, bytes)) return r;
    if (int r = split_counts(c)) return r;
    L.split_terms = static_cast<float *>(c->gsplit.p);
    L.split_terms_bytes = c->gsplit.cap;
    L.split_count = static_cast<int *>(c->gcount.p);
    return KQ_OK;
}

// Run the tasks (device pointers) over input rows [0, M): fp16 x, or pre-quantized act_q8k /
// act_q80.  Tasks of the same type share a launch; M is processed in tiles of up to 8 rows.
struct GemvExtra {
    int *dbg_sumi = nullptr, *dbg_summ = nullptr;
    unsigned long long *argmax = nullptr;  // [M] keys
    int argmax_f16 = 0;
    const uint32_t *out_ids = nullptr;     // tasks[0]: output column of local row r (device)
    bool no_pdl = false;                   // the weights were written by the previous kernel
    const kq::PeerOut *peer = nullptr;     // task 0's fp32 outputs also into every rank's gather buffer
};

int run_gemv(kq_ctx *c, const kq_task *tasks, int n, int M, int K, const __half *x, long long x_stride,
             const void *act_q8k, const void *act_q80, const GemvExtra &ex = GemvExtra()) {
    const int types[4] = {KQ_TYPE_Q4_K, KQ_TYPE_Q5_K, KQ_TYPE_Q6_K, KQ_TYPE_Q8_0};
    for (int ti = 0; ti < 4; ++ti) {
        const int type = types[ti];
        std::vector<int> idx;
        for (int i = 0; i < n; ++i)
            if ((int)tasks[i].w->type == type && tasks[i].rows > 0) idx.push_back(i);
        if (idx.empty()) continue;
        const void *act = (type == KQ_TYPE_Q8_0) ? act_q80 : act_q8k;
        if (!x && !act) return fail(c, KQ_ERR_NOT_READY, "no activation for type %d", type);
        // M > 8: one of two tensor-core kernels or GEMV tiles of 8 tokens, by a cost model fitted
        // to B200 timings of the FFN and attention shapes (M = 9..512):
        //  * weight-row-major tensor-core kernel (kq_gemm_tc.cu, 128 or 64 rows x 16..64 tokens per
        //    CTA, all of K serially): ~2-4 us per 256-value unit per wave of CTAs (tc_estimate_us);
        //  * token-major kernel (row groups spread over all SMs): ~3.5 us per item (a unit of
        //    up to 4 row groups, Q6_K 3) per wave;
        //  * GEMV tiles: the weights streamed once per 8 tokens at ~1 TB/s plus ~5 us a launch.
        int tc_kernel = 0;  // 0 GEMV tiles, 1 row-major, 3 token-major
        if (M > 8 && !ex.dbg_sumi && !ex.argmax && !ex.out_ids) {
            long long rgs = 0;
            double wbytes = 0.0;
            for (int j : idx) {
                rgs += (tasks[j].row_begin + tasks[j].rows - 1) / 16 - tasks[j].row_begin / 16 + 1;
                wbytes += (double)tasks[j].rows * (double)tasks[j].w->row_bytes;
            }
            const int nbu = K / 256, sms = c->num_sms;
            int task_rgs[KQ_MAX_TASKS];
            for (size_t j = 0; j < idx.size(); ++j)
                task_rgs[j] = (tasks[idx[j]].row_begin + tasks[idx[j]].rows - 1) / 16 - tasks[idx[j]].row_begin / 16 + 1;
            const double t1 = kq::tc_estimate_us(type, M, K, task_rgs, (int)idx.size(), sms) * 1e-6;
            const int n_tb = (M + 127) / 128, g = (type == KQ_TYPE_Q6_K) ? 3 : (type == KQ_TYPE_Q8_0) ? 1 : 4;
            const int rgmax = (type == KQ_TYPE_Q6_K) ? 6 : 8;
            const long long gx = std::min<long long>(rgs, std::max<long long>((sms + n_tb - 1) / n_tb, (rgs + rgmax - 1) / rgmax));
            const double items = std::max(1.0, (double)rgs / (double)gx / g);  // items per unit of an average CTA
            const double t3 = (double)((gx * n_tb + sms - 1) / sms) * nbu * items * 3.5e-6;
            const double tg = (double)((M + 7) / 8) * (wbytes / 1.0e12 + 5.0e-6);
            if (c->gemm_path == 1 || c->gemm_path == 3) tc_kernel = c->gemm_path;
            else if (c->gemm_path == 0) tc_kernel = (tg <= std::min(t1, t3)) ? 0 : (t1 <= t3 ? 1 : 3);
        }
        const bool use_tc = tc_kernel != 0;
        if (use_tc) {
            // many tokens: the tensor-core kernel (activation packed into the context's buffer)
            kq::TcLaunch T{};
            T.type = type;
            T.K = K;
            T.M = M;
            T.n_tasks = (int)idx.size();
            for (int j = 0; j < T.n_tasks; ++j) {
                const kq_task &t = tasks[idx[j]];
                kq::GemvTaskHost &h = T.tasks[j];
                h.w = t.w->d;
                h.row_begin = t.row_begin;
                h.rows = t.rows;
                h.dst = t.dst;
                h.dst_stride = (long long)t.dst_stride;
                h.res = t.residual;
                h.res_stride = (long long)t.res_stride;
                h.dst_f32 = t.dst_f32;
                h.f32_stride = (long long)t.dst_f32_stride;
            }
            T.x = x;
            T.x_stride = x_stride;
            T.act = x ? nullptr : act;
            const bool tc2 = tc_kernel == 3;
            T.scratch_bytes = tc2 ? kq::tc2_scratch_bytes(type, M, K) : kq::tc_scratch_bytes(type, M, K);
            if (int r = ensure(c, c->tcpack, T.scratch_bytes)) return r;
            T.scratch = c->tcpack.p;
            T.status = c->d_status;
            T.timeout_ns = c->timeout_ns;
            T.num_sms = c->num_sms;
            if (!tc2) {
                int trows[KQ_MAX_TASKS], trgs[KQ_MAX_TASKS];
                for (int j = 0; j < T.n_tasks; ++j) {
                    trows[j] = T.tasks[j].rows;
                    trgs[j] = (T.tasks[j].row_begin + T.tasks[j].rows - 1) / 16 - T.tasks[j].row_begin / 16 + 1;
                }
                T.terms_bytes = kq::tc_split_terms_bytes(type, M, K, trows, trgs, T.n_tasks, c->num_sms);
                if (T.terms_bytes) {
                    if (int r = ensure(c, c->tcterms, T.terms_bytes)) return r;
                    T.terms = c->tcterms.p;
                }
            }
            if (cudaError_t e = tc2 ? kq::launch_gemm_tc2(T, c->stream) : kq::launch_gemm_tc(T, c->stream))
                return cuda_fail(c, e, "tensor-core gemm launch");
            continue;
        }
        int m0 = 0;
        while (m0 < M) {
            int mt = std::min(8, M - m0);
            kq::GemvLaunch L{};
            L.type = type;
            L.K = K;
            L.n_tasks = (int)idx.size();
            for (int j = 0; j < L.n_tasks; ++j) {
                const kq_task &t = tasks[idx[j]];
                kq::GemvTaskHost &h = L.tasks[j];
                h.w = t.w->d;
                h.row_begin = t.row_begin;
                h.rows = t.rows;
                h.dst = t.dst ? (void *)(t.dst + (size_t)m0 * t.dst_stride) : nullptr;
                h.dst_stride = (long long)t.dst_stride;
                h.res = t.residual ? (const void *)(t.residual + (size_t)m0 * t.res_stride) : nullptr;
                h.res_stride = (long long)t.res_stride;
                h.dst_f32 = t.dst_f32 ? t.dst_f32 + (size_t)m0 * t.dst_f32_stride : nullptr;
                h.f32_stride = (long long)t.dst_f32_stride;
                if (ex.dbg_sumi && idx[j] == 0) {
                    const size_t bpr = (type == KQ_TYPE_Q8_0) ? (size_t)K / 32 : (size_t)K / 256;
                    h.dbg_sumi = ex.dbg_sumi + (size_t)m0 * t.rows * bpr;
                    h.dbg_summ = ex.dbg_summ + (size_t)m0 * t.rows * bpr;
                }
                if (ex.out_ids && idx[j] == 0) h.out_ids = ex.out_ids;
                h.index_base = t.row_begin;
            }
            if (x) {
                L.x = x + (size_t)m0 * x_stride;
                L.x_stride = x_stride;
            } else if (type == KQ_TYPE_Q8_0) {
                L.act = reinterpret_cast<const kq::BlockQ80 *>(act) + (size_t)m0 * (K / 32);
            } else {
                L.act = reinterpret_cast<const kq::BlockQ8K *>(act) + (size_t)m0 * (K / 256);
            }
            L.M = mt;
            L.status = c->d_status;
            L.timeout_ns = c->timeout_ns;
            L.pdl = c->pdl && !ex.no_pdl;
            L.num_sms = c->num_sms;
            L.argmax = ex.argmax ? ex.argmax + m0 : nullptr;
            L.argmax_f16 = ex.argmax_f16;
            L.inject_wait = c->inject_timeout ? 1 : 0;
            if (ex.peer) L.peer = *ex.peer;
            if (int r = gemv_split_scratch(c, type, K, mt, L)) return r;
            L.half_ok = c->gemv_half;
            cudaError_t e = kq::launch_gemv(L, c->stream);
            if (e == cudaErrorInvalidConfiguration && mt > 1) {
                // activation too large for shared memory at this tile: halve the tile
                cudaGetLastError();
                L.M = mt = std::max(1, mt / 2);
                e = kq::launch_gemv(L, c->stream);
            }
            if (e != cudaSuccess) return cuda_fail(c, e, "gemv launch");
            m0 += mt;
        }
    }
    return KQ_OK;
}

void set_current_x(kq_ctx *c, int M, int K) {
    c->cur_M = M;
    c->cur_K = K;
    c->cur_x_valid = true;
    c->cur_q8k_valid = false;
    c->cur_q80_valid = false;
}

// Make sure the current input is available quantized as `type` (Q8_K for K-quants, Q8_0).
int current_act(kq_ctx *c, uint32_t type, const void **act) {
    if (c->cur_M == 0) return fail(c, KQ_ERR_NOT_READY, "no current quantized input in the context");
    const int M = c->cur_M, K = c->cur_K;
    if (type == KQ_TYPE_Q8_0) {
        if (!c->cur_q80_valid) {
            if (!c->cur_x_valid) return fail(c, KQ_ERR_NOT_READY, "current input has no Q8_0 form");
            int r = ensure(c, c->q80_cur, (size_t)M * (K / 32) * sizeof(kq::BlockQ80));
            if (r) return r;
            KQ_CUDA(c, kq::launch_quantize(KQ_TYPE_Q8_0, c->x.p, K, M, K, c->q80_cur.p, c->stream));
            c->cur_q80_valid = true;
        }
        *act = c->q80_cur.p;
    } else {
        if (!c->cur_q8k_valid) {
            if (!c->cur_x_valid) return fail(c, KQ_ERR_NOT_READY, "current input has no Q8_K form");
            int r = ensure(c, c->q8k_cur, (size_t)M * (K / 256) * sizeof(kq::BlockQ8K));
            if (r) return r;
            KQ_CUDA(c, kq::launch_quantize(KQ_TYPE_Q4_K, c->x.p, K, M, K, c->q8k_cur.p, c->stream));
            c->cur_q8k_valid = true;
        }
        *act = c->q8k_cur.p;
    }
    return KQ_OK;
}

// Device address of a host buffer that is pinned and mapped (cudaHostAlloc / cudaMallocHost /
// cudaHostRegister memory under unified addressing), else nullptr.  Results written there by a
// kernel are visible to the host after the stream synchronizes, so no copy is needed.
void *mapped_device_ptr(const void *host) {
    cudaPointerAttributes a{};
    if (cudaPointerGetAttributes(&a, host) != cudaSuccess) {
        cudaGetLastError();  // pageable memory can report an error on some drivers: not sticky
        return nullptr;
    }
    return (a.type == cudaMemoryTypeHost && a.devicePointer) ? a.devicePointer : nullptr;
}

// Strided row copy; one linear copy when the rows are contiguous on both sides (cheaper to issue).
cudaError_t copy_rows(void *dst, size_t dpitch, const void *src, size_t spitch, size_t width, size_t height,
                      cudaMemcpyKind kind, cudaStream_t s) {
    if (height == 1 || (dpitch == width && spitch == width))
        return cudaMemcpyAsync(dst, src, width * height, kind, s);
    return cudaMemcpy2DAsync(dst, dpitch, src, spitch, width, height, kind, s);
}

int h2d(kq_ctx *c, DevBuf &b, const void *src, size_t bytes) {
    int r = ensure(c, b, bytes);
    if (r) return r;
    KQ_CUDA(c, cudaMemcpyAsync(b.p, src, bytes, cudaMemcpyHostToDevice, c->stream));
    return KQ_OK;
}

}  // namespace

// =================================================================== library / context

extern "C" const char *kq_version(void) { return "kq-b200 0.1 (sm_100a)"; }

extern "C" const char *kq_status_string(int s) {
    switch (s) {
        case KQ_OK: return "ok";
        case KQ_ERR_INVALID_ARGUMENT: return "invalid argument";
        case KQ_ERR_UNSUPPORTED_TYPE: return "unsupported type";
        case KQ_ERR_SHAPE: return "shape error";
        case KQ_ERR_CUDA: return "CUDA error";
        case KQ_ERR_OUT_OF_MEMORY: return "out of device memory";
        case KQ_ERR_NO_DEVICE: return "no CUDA device";
        case KQ_ERR_TIMEOUT: return "device-side wait timed out";
        case KQ_ERR_NOT_READY: return "no pending quantized input";
        case KQ_ERR_FORMAT: return "not a GGUF v2/v3 image or truncated";
        case KQ_ERR_NOT_FOUND: return "not found";
        default: return "unknown status";
    }
}

extern "C" int kq_init(int device, kq_ctx **out) {
    if (!out) return KQ_ERR_INVALID_ARGUMENT;
    *out = nullptr;
    int n = 0;
    if (cudaGetDeviceCount(&n) != cudaSuccess || n == 0) {
        cudaGetLastError();
        return KQ_ERR_NO_DEVICE;
    }
    if (device < 0 || device >= n) return KQ_ERR_INVALID_ARGUMENT;
    kq_ctx *c = new kq_ctx();
    c->device = device;
    if (cudaSetDevice(device) != cudaSuccess) {
        delete c;
        return KQ_ERR_CUDA;
    }
    cudaDeviceProp prop{};
    cudaGetDeviceProperties(&prop, device);
    c->num_sms = prop.multiProcessorCount;
    if (prop.major < 10) {
        delete c;
        return KQ_ERR_NO_DEVICE;  // built for sm_100a only
    }
    if (cudaStreamCreateWithFlags(&c->stream, cudaStreamNonBlocking) != cudaSuccess ||
        cudaHostAlloc(&c->h_status, sizeof(int), cudaHostAllocMapped) != cudaSuccess ||
        cudaHostGetDevicePointer(&c->d_status, c->h_status, 0) != cudaSuccess) {
        if (c->stream) cudaStreamDestroy(c->stream);
        if (c->h_status) cudaFreeHost(c->h_status);
        delete c;
        return KQ_ERR_CUDA;
    }
    *c->h_status = kq::DEV_OK;
    c->own_stream = true;
    {
        std::vector<float> tab(65536);
        kq::fill_swiglu_exp_table(tab.data());
        if (cudaMalloc(&c->exp_tab, tab.size() * sizeof(float)) != cudaSuccess ||
            cudaMemcpy(c->exp_tab, tab.data(), tab.size() * sizeof(float), cudaMemcpyHostToDevice) != cudaSuccess) {
            if (c->exp_tab) cudaFree(c->exp_tab);
            cudaStreamDestroy(c->stream);
            cudaFreeHost(c->h_status);
            delete c;
            return KQ_ERR_CUDA;
        }
    }
    *out = c;
    return KQ_OK;
}

extern "C" int kq_destroy(kq_ctx *c) {
    if (!c) return KQ_ERR_INVALID_ARGUMENT;
    cudaSetDevice(c->device);
    cudaStreamSynchronize(c->stream);
    for (DevBuf *b : {&c->x, &c->res, &c->out16, &c->out32, &c->q8k_pending, &c->q8k_cur, &c->q80_cur, &c->tmp,
                      &c->misc, &c->keys, &c->tcpack, &c->tcterms, &c->gsplit, &c->gcount, &c->lmlogits})
        if (b->p) cudaFree(b->p);
    cudaFree(c->exp_tab);
    cudaFreeHost(c->h_status);
    if (c->own_stream) cudaStreamDestroy(c->stream);
    delete c;
    return KQ_OK;
}

extern "C" int kq_set_stream(kq_ctx *c, void *s) {
    if (!c) return KQ_ERR_INVALID_ARGUMENT;
    if (reinterpret_cast<cudaStream_t>(s) == c->stream) return KQ_OK;
    // drain the previous stream unless it is being captured into a graph (a sync would end
    // the capture); work captured there belongs to the graph, not to this context
    cudaStreamCaptureStatus cap = cudaStreamCaptureStatusNone;
    cudaStreamIsCapturing(c->stream, &cap);
    if (cap == cudaStreamCaptureStatusNone) cudaStreamSynchronize(c->stream);
    if (c->own_stream) cudaStreamDestroy(c->stream);
    c->stream = reinterpret_cast<cudaStream_t>(s);
    c->own_stream = false;
    return KQ_OK;
}

extern "C" void *kq_get_stream(const kq_ctx *c) { return c ? (void *)c->stream : nullptr; }

extern "C" int kq_synchronize(kq_ctx *c) {
    if (!c) return KQ_ERR_INVALID_ARGUMENT;
    cudaSetDevice(c->device);
    return sync_and_check(c);
}

extern "C" const char *kq_last_error(const kq_ctx *c) { return c ? c->err.c_str() : "no context"; }

extern "C" int kq_set_option(kq_ctx *c, const char *name, long long value) {
    if (!c || !name) return KQ_ERR_INVALID_ARGUMENT;
    if (!strcmp(name, "pdl")) {
        c->pdl = value != 0;
        return KQ_OK;
    }
    if (!strcmp(name, "inject_timeout")) {
        c->inject_timeout = value != 0;
        return KQ_OK;
    }
    if (!strcmp(name, "timeout_ms")) {
        if (value <= 0) return fail(c, KQ_ERR_INVALID_ARGUMENT, "timeout_ms must be positive");
        c->timeout_ns = (unsigned long long)value * 1000000ull;
        return KQ_OK;
    }
    if (!strcmp(name, "gemm_path")) {
        if (value < 0 || value > 3) return fail(c, KQ_ERR_INVALID_ARGUMENT, "gemm_path must be 0..3");
        c->gemm_path = (int)value;
        return KQ_OK;
    }
    if (!strcmp(name, "graph_released")) {
        c->graph_holds_scratch = value == 0;
        return KQ_OK;
    }
    if (!strcmp(name, "swiglu_exp")) {
        if (value < 0 || value > 1) return fail(c, KQ_ERR_INVALID_ARGUMENT, "swiglu_exp must be 0 or 1");
        c->swiglu_gpu_exp = value == 1;
        return KQ_OK;
    }
    if (!strcmp(name, "ffn_fused")) {
        c->ffn_fused = value != 0;
        return KQ_OK;
    }
    if (!strcmp(name, "gemv_split")) {
        c->gemv_split = value != 0;
        return KQ_OK;
    }
    if (!strcmp(name, "gemv_half")) {
        c->gemv_half = value != 0;
        return KQ_OK;
    }
    if (!strcmp(name, "timeout_us")) {
        if (value <= 0) return fail(c, KQ_ERR_INVALID_ARGUMENT, "timeout_us must be positive");
        c->timeout_ns = (unsigned long long)value * 1000ull;
        return KQ_OK;
    }
    return fail(c, KQ_ERR_INVALID_ARGUMENT, "unknown option '%s'", name);
}

extern "C" uint64_t kq_row_bytes(uint32_t type, uint64_t k) {
    // compute_ggml_bytes, ENG:364-374
    switch (type) {
        case KQ_TYPE_F32: return k * 4;
        case KQ_TYPE_F16: return k * 2;
        case KQ_TYPE_Q8_0: return (k / 32) * 34;
        case KQ_TYPE_Q4_K: return (k / 256) * 144;
        case KQ_TYPE_Q5_K: return (k / 256) * 176;
        case KQ_TYPE_Q6_K: return (k / 256) * 210;
        default: return 0;
    }
}

// =================================================================== weights

static int weight_create(kq_ctx *c, const void *src, bool src_on_device, uint32_t type, int rows, int cols,
                         kq_weight **out) {
    if (!c || !src || !out) return fail(c, KQ_ERR_INVALID_ARGUMENT, "NULL argument");
    *out = nullptr;
    if (!supported(type)) return fail(c, KQ_ERR_UNSUPPORTED_TYPE, "type %u is not Q4_K/Q5_K/Q6_K/Q8_0", type);
    if (rows < 1) return fail(c, KQ_ERR_SHAPE, "rows = %d", rows);
    if (cols < 256 || cols > KQ_MAX_K || cols % 256)
        return fail(c, KQ_ERR_SHAPE, "cols = %d must be a positive multiple of 256 up to %d", cols, KQ_MAX_K);
    cudaSetDevice(c->device);
    const size_t gguf_bytes = (size_t)rows * kq_row_bytes(type, cols);
    kq_weight *w = new kq_weight();
    w->device = c->device;
    w->type = type;
    w->rows = rows;
    w->cols = cols;
    w->row_bytes = kq_row_bytes(type, cols);
    w->bytes = kq::weight_bytes((int)type, rows, cols);
    cudaError_t e = cudaMalloc(&w->d, w->bytes);
    if (e != cudaSuccess) {
        delete w;
        return cuda_fail(c, e, "cudaMalloc(weight)");
    }
    void *staging = nullptr;
    const uint8_t *gsrc = reinterpret_cast<const uint8_t *>(src);
    if (!src_on_device) {
        e = cudaMalloc(&staging, gguf_bytes);
        if (e == cudaSuccess) e = cudaMemcpyAsync(staging, src, gguf_bytes, cudaMemcpyHostToDevice, c->stream);
        if (e == cudaSuccess) e = kq::launch_repack((int)type, (const uint8_t *)staging, w->d, rows, cols, c->stream);
    } else {
        e = kq::launch_repack((int)type, gsrc, w->d, rows, cols, c->stream);
    }
    if (e == cudaSuccess) e = cudaStreamSynchronize(c->stream);
    if (staging) cudaFree(staging);
    if (e != cudaSuccess) {
        cudaFree(w->d);
        delete w;
        return cuda_fail(c, e, "weight upload");
    }
    *out = w;
    return KQ_OK;
}

extern "C" int kq_weight_upload(kq_ctx *c, const void *b, uint32_t type, int rows, int cols, kq_weight **out) {
    return weight_create(c, b, false, type, rows, cols, out);
}

extern "C" int kq_weight_upload_device(kq_ctx *c, const void *b, uint32_t type, int rows, int cols, kq_weight **out) {
    return weight_create(c, b, true, type, rows, cols, out);
}

extern "C" int kq_weight_free(kq_ctx *c, kq_weight *w) {
    if (!w) return KQ_ERR_INVALID_ARGUMENT;
    if (c) {
        cudaSetDevice(c->device);
        cudaStreamSynchronize(c->stream);
    }
    int prev = 0;
    cudaGetDevice(&prev);
    if (prev != w->device) cudaSetDevice(w->device);
    cudaFree(w->d);
    if (prev != w->device) cudaSetDevice(prev);
    delete w;
    return KQ_OK;
}

extern "C" int kq_weight_info(const kq_weight *w, uint32_t *type, int *rows, int *cols, uint64_t *device_bytes) {
    if (!w) return KQ_ERR_INVALID_ARGUMENT;
    if (type) *type = w->type;
    if (rows) *rows = w->rows;
    if (cols) *cols = w->cols;
    if (device_bytes) *device_bytes = w->bytes;
    return KQ_OK;
}

// =================================================================== activations

extern "C" int kq_quantize_q8k_async(kq_ctx *c, const uint16_t *x, int M, int K, void *out) {
    if (!c || !x || !out) return fail(c, KQ_ERR_INVALID_ARGUMENT, "NULL argument");
    if (int r = validate_mk(c, M, K)) return r;
    KQ_CUDA(c, kq::launch_quantize(KQ_TYPE_Q4_K, x, K, M, K, out, c->stream));
    return KQ_OK;
}

extern "C" int kq_quantize_q8_0_async(kq_ctx *c, const uint16_t *x, int M, int K, void *out) {
    if (!c || !x || !out) return fail(c, KQ_ERR_INVALID_ARGUMENT, "NULL argument");
    if (int r = validate_mk(c, M, K)) return r;
    KQ_CUDA(c, kq::launch_quantize(KQ_TYPE_Q8_0, x, K, M, K, out, c->stream));
    return KQ_OK;
}

static int quantize_host(kq_ctx *c, int target, const uint16_t *x, int M, int K, void *out) {
    if (!c || !x || !out) return fail(c, KQ_ERR_INVALID_ARGUMENT, "NULL argument");
    if (int r = validate_mk(c, M, K)) return r;
    cudaSetDevice(c->device);
    const size_t ob = target == KQ_TYPE_Q8_0 ? (size_t)M * (K / 32) * sizeof(kq::BlockQ80)
                                             : (size_t)M * (K / 256) * sizeof(kq::BlockQ8K);
    if (int r = h2d(c, c->x, x, (size_t)M * K * 2)) return r;
    if (int r = ensure(c, c->tmp, ob)) return r;
    KQ_CUDA(c, kq::launch_quantize(target, c->x.p, K, M, K, c->tmp.p, c->stream));
    KQ_CUDA(c, cudaMemcpyAsync(out, c->tmp.p, ob, cudaMemcpyDeviceToHost, c->stream));
    set_current_x(c, M, K);
    return sync_and_check(c);
}

extern "C" int kq_quantize_q8k(kq_ctx *c, const uint16_t *x, int M, int K, void *out) {
    return quantize_host(c, KQ_TYPE_Q4_K, x, M, K, out);
}

extern "C" int kq_quantize_q8_0(kq_ctx *c, const uint16_t *x, int M, int K, void *out) {
    return quantize_host(c, KQ_TYPE_Q8_0, x, M, K, out);
}

// =================================================================== matrix products

static int validate_tasks(kq_ctx *c, const kq_task *tasks, int n, int K) {
    if (!tasks || n < 1 || n > KQ_MAX_TASKS)
        return fail(c, KQ_ERR_INVALID_ARGUMENT, "n_tasks = %d outside [1, %d]", n, KQ_MAX_TASKS);
    for (int i = 0; i < n; ++i)
        if (int r = validate_task(c, tasks[i], K)) return r;
    return KQ_OK;
}

extern "C" int kq_gemm_multi_async(kq_ctx *c, const uint16_t *x, size_t x_stride, int M, int K, const kq_task *tasks,
                                   int n) {
    if (!c || !x) return fail(c, KQ_ERR_INVALID_ARGUMENT, "NULL argument");
    if (int r = validate_mk(c, M, K)) return r;
    if (int r = validate_tasks(c, tasks, n, K)) return r;
    if (x_stride < (size_t)K) return fail(c, KQ_ERR_INVALID_ARGUMENT, "x_stride < K");
    return run_gemv(c, tasks, n, M, K, reinterpret_cast<const __half *>(x), (long long)x_stride, nullptr, nullptr);
}

extern "C" int kq_gemm_multi_q8_async(kq_ctx *c, const void *q8k, const void *q80, int M, int K, const kq_task *tasks,
                                      int n) {
    if (!c) return KQ_ERR_INVALID_ARGUMENT;
    if (int r = validate_mk(c, M, K)) return r;
    if (int r = validate_tasks(c, tasks, n, K)) return r;
    for (int i = 0; i < n; ++i) {
        if (tasks[i].w->type == KQ_TYPE_Q8_0 && !q80) return fail(c, KQ_ERR_INVALID_ARGUMENT, "Q8_0 task needs act_q80");
        if (tasks[i].w->type != KQ_TYPE_Q8_0 && !q8k) return fail(c, KQ_ERR_INVALID_ARGUMENT, "K-quant task needs act_q8k");
    }
    return run_gemv(c, tasks, n, M, K, nullptr, 0, q8k, q80);
}

extern "C" int kq_sdot_gemm_multi_dispatch(kq_ctx *c, const uint16_t *x, int M, int K, const kq_task *tasks, int n) {
    if (!c || !x) return fail(c, KQ_ERR_INVALID_ARGUMENT, "NULL argument");
    if (int r = validate_mk(c, M, K)) return r;
    if (int r = validate_tasks(c, tasks, n, K)) return r;
    cudaSetDevice(c->device);
    // the pre-quantized flag is consumed by this call whatever happens (ENG:4205-4206)
    const bool use_pending = c->pending && c->pending_M == M && c->pending_K == K;
    c->pending = false;

    if (int r = h2d(c, c->x, x, (size_t)M * K * 2)) return r;
    // device staging of outputs and residuals, one contiguous [M][rows] slab per task
    size_t o16 = 0, o32 = 0, ores = 0;
    std::vector<size_t> off16(n), off32(n), offr(n);
    for (int i = 0; i < n; ++i) {
        off16[i] = o16;
        o16 += tasks[i].dst ? (size_t)M * tasks[i].rows * 2 : 0;
        off32[i] = o32;
        o32 += tasks[i].dst_f32 ? (size_t)M * tasks[i].rows * 4 : 0;
        offr[i] = ores;
        ores += tasks[i].residual ? (size_t)M * tasks[i].rows * 2 : 0;
    }
    if (int r = ensure(c, c->out16, o16 + 16)) return r;
    if (int r = ensure(c, c->out32, o32 + 16)) return r;
    if (int r = ensure(c, c->res, ores + 16)) return r;
    kq_task dt[KQ_MAX_TASKS];
    bool direct16[KQ_MAX_TASKS] = {}, direct32[KQ_MAX_TASKS] = {};
    for (int i = 0; i < n; ++i) {
        dt[i] = tasks[i];
        const size_t rows = (size_t)tasks[i].rows;
        // outputs in pinned host memory are written by the kernel in place; others are staged
        if (tasks[i].dst) {
            if (void *dp = mapped_device_ptr(tasks[i].dst)) {
                dt[i].dst = static_cast<uint16_t *>(dp);
                direct16[i] = true;
            } else {
                dt[i].dst = reinterpret_cast<uint16_t *>((uint8_t *)c->out16.p + off16[i]);
                dt[i].dst_stride = rows;
            }
        }
        if (tasks[i].dst_f32) {
            if (void *dp = mapped_device_ptr(tasks[i].dst_f32)) {
                dt[i].dst_f32 = static_cast<float *>(dp);
                direct32[i] = true;
            } else {
                dt[i].dst_f32 = reinterpret_cast<float *>((uint8_t *)c->out32.p + off32[i]);
                dt[i].dst_f32_stride = rows;
            }
        }
        if (tasks[i].residual) {
            uint16_t *rd = reinterpret_cast<uint16_t *>((uint8_t *)c->res.p + offr[i]);
            KQ_CUDA(c, copy_rows(rd, rows * 2, tasks[i].residual, tasks[i].res_stride * 2, rows * 2, M,
                                         cudaMemcpyHostToDevice, c->stream));
            dt[i].residual = rd;
            dt[i].res_stride = rows;
        }
    }
    int r;
    if (use_pending) {
        // Q8_K already produced on the device; Q8_0 tasks still quantize x (ENG:4212-4216)
        bool any_q80 = false;
        for (int i = 0; i < n; ++i) any_q80 |= tasks[i].w->type == KQ_TYPE_Q8_0;
        const void *q80 = nullptr;
        if (any_q80) {
            if ((r = ensure(c, c->q80_cur, (size_t)M * (K / 32) * sizeof(kq::BlockQ80)))) return r;
            KQ_CUDA(c, kq::launch_quantize(KQ_TYPE_Q8_0, c->x.p, K, M, K, c->q80_cur.p, c->stream));
            q80 = c->q80_cur.p;
        }
        r = run_gemv(c, dt, n, M, K, nullptr, 0, c->q8k_pending.p, q80);
        // the pending Q8_K becomes the current input for row-level calls
        std::swap(c->q8k_pending, c->q8k_cur);
        c->cur_M = M;
        c->cur_K = K;
        c->cur_x_valid = true;
        c->cur_q8k_valid = true;
        c->cur_q80_valid = any_q80;
    } else {
        r = run_gemv(c, dt, n, M, K, reinterpret_cast<const __half *>(c->x.p), K, nullptr, nullptr);
        set_current_x(c, M, K);
    }
    if (r) return r;
    for (int i = 0; i < n; ++i) {
        const size_t rows = (size_t)tasks[i].rows;
        if (tasks[i].dst && !direct16[i])
            KQ_CUDA(c, copy_rows(tasks[i].dst, tasks[i].dst_stride * 2, dt[i].dst, rows * 2, rows * 2, M,
                                         cudaMemcpyDeviceToHost, c->stream));
        if (tasks[i].dst_f32 && !direct32[i])
            KQ_CUDA(c, copy_rows(tasks[i].dst_f32, tasks[i].dst_f32_stride * 4, dt[i].dst_f32, rows * 4,
                                         rows * 4, M, cudaMemcpyDeviceToHost, c->stream));
    }
    return sync_and_check(c);
}

// Row-level entry points over the current input.
static int row_level(kq_ctx *c, const kq_weight *w, uint32_t row, int m0, int M, float *out) {
    if (!c || !w || !out) return fail(c, KQ_ERR_INVALID_ARGUMENT, "NULL argument");
    if (int r = check_weight_device(c, w)) return r;
    if ((int)row >= w->rows) return fail(c, KQ_ERR_SHAPE, "row %u >= rows %d", row, w->rows);
    if (c->cur_M == 0) return fail(c, KQ_ERR_NOT_READY, "no current input");
    if (w->cols != c->cur_K) return fail(c, KQ_ERR_SHAPE, "weight cols %d != current K %d", w->cols, c->cur_K);
    if (m0 < 0 || M < 1 || m0 + M > c->cur_M) return fail(c, KQ_ERR_SHAPE, "token range outside current input");
    cudaSetDevice(c->device);
    const void *act = nullptr;
    if (int r = current_act(c, w->type, &act)) return r;
    if (int r = ensure(c, c->misc, (size_t)M * 4)) return r;
    kq_task t{};
    t.w = w;
    t.row_begin = (int)row;
    t.rows = 1;
    t.dst_f32 = reinterpret_cast<float *>(c->misc.p);
    t.dst_f32_stride = 1;
    const int K = c->cur_K;
    const void *a = (w->type == KQ_TYPE_Q8_0)
                        ? (const void *)(reinterpret_cast<const kq::BlockQ80 *>(act) + (size_t)m0 * (K / 32))
                        : (const void *)(reinterpret_cast<const kq::BlockQ8K *>(act) + (size_t)m0 * (K / 256));
    int r = run_gemv(c, &t, 1, M, K, nullptr, 0, w->type == KQ_TYPE_Q8_0 ? nullptr : a,
                     w->type == KQ_TYPE_Q8_0 ? a : nullptr);
    if (r) return r;
    KQ_CUDA(c, cudaMemcpyAsync(out, c->misc.p, (size_t)M * 4, cudaMemcpyDeviceToHost, c->stream));
    return sync_and_check(c);
}

extern "C" int kq_sdot_row_batch(kq_ctx *c, const kq_weight *w, uint32_t row, int M, float *out_sums) {
    return row_level(c, w, row, 0, M, out_sums);
}

extern "C" int kq_eval_single_lm_row_dot(kq_ctx *c, const kq_weight *w, uint32_t row_idx, int m, float *out) {
    return row_level(c, w, row_idx, m, 1, out);
}

extern "C" int kq_debug_block_sums_async(kq_ctx *c, const kq_weight *w, int row_begin, int rows, const void *act,
                                         int M, int32_t *sumi, int32_t *summ, float *out_f32) {
    if (!c || !w || !act || !sumi || !summ) return fail(c, KQ_ERR_INVALID_ARGUMENT, "NULL argument");
    if (int r = validate_mk(c, M, w->cols)) return r;
    kq_task t{};
    t.w = w;
    t.row_begin = row_begin;
    t.rows = rows;
    t.dst_f32 = out_f32;
    t.dst_f32_stride = (size_t)rows;
    if (int r = validate_task(c, t, w->cols)) return r;
    const bool q80 = w->type == KQ_TYPE_Q8_0;
    GemvExtra ex;
    ex.dbg_sumi = sumi;
    ex.dbg_summ = summ;
    return run_gemv(c, &t, 1, M, w->cols, nullptr, 0, q80 ? nullptr : act, q80 ? act : nullptr, ex);
}

// =================================================================== producers

extern "C" int kq_rmsnorm_q8k_async(kq_ctx *c, const uint16_t *x, const uint16_t *gamma, uint16_t *out, int M, int K,
                                    void *q8k) {
    if (!c || !x || !gamma || !out) return fail(c, KQ_ERR_INVALID_ARGUMENT, "NULL argument");
    if (int r = validate_mk(c, M, K)) return r;
    if (!q8k) {
        if (int r = ensure(c, c->q8k_pending, (size_t)M * (K / 256) * sizeof(kq::BlockQ8K))) return r;
        q8k = c->q8k_pending.p;
        c->pending = true;
        c->pending_M = M;
        c->pending_K = K;
    }
    KQ_CUDA(c, kq::launch_rmsnorm_q8k(x, gamma, out, q8k, M, K, c->stream, c->pdl));
    return KQ_OK;
}

extern "C" int kq_swiglu_q8k_async(kq_ctx *c, uint16_t *gate, const uint16_t *up, int M, int N, void *q8k) {
    if (!c || !gate || !up) return fail(c, KQ_ERR_INVALID_ARGUMENT, "NULL argument");
    if (int r = validate_mk(c, M, N)) return r;
    if (!q8k) {
        if (int r = ensure(c, c->q8k_pending, (size_t)M * (N / 256) * sizeof(kq::BlockQ8K))) return r;
        q8k = c->q8k_pending.p;
        c->pending = true;
        c->pending_M = M;
        c->pending_K = N;
    }
    KQ_CUDA(c, kq::launch_swiglu_q8k(gate, up, q8k, M, N, c->stream, c->pdl, swiglu_table(c)));
    return KQ_OK;
}

extern "C" int kq_rmsnorm_fp16_rows(kq_ctx *c, const uint16_t *x_in, const uint16_t *gamma, uint16_t *x_out, int M,
                                    int K) {
    if (!c || !x_in || !gamma || !x_out) return fail(c, KQ_ERR_INVALID_ARGUMENT, "NULL argument");
    if (int r = validate_mk(c, M, K)) return r;
    cudaSetDevice(c->device);
    const size_t xb = (size_t)M * K * 2;
    if (int r = ensure(c, c->tmp, xb + (size_t)K * 2 + 16)) return r;
    uint16_t *dx = reinterpret_cast<uint16_t *>(c->tmp.p);
    uint16_t *dg = dx + (size_t)M * K;
    KQ_CUDA(c, cudaMemcpyAsync(dx, x_in, xb, cudaMemcpyHostToDevice, c->stream));
    KQ_CUDA(c, cudaMemcpyAsync(dg, gamma, (size_t)K * 2, cudaMemcpyHostToDevice, c->stream));
    if (int r = ensure(c, c->x, xb)) return r;
    if (int r = kq_rmsnorm_q8k_async(c, dx, dg, reinterpret_cast<uint16_t *>(c->x.p), M, K, nullptr)) return r;
    KQ_CUDA(c, cudaMemcpyAsync(x_out, c->x.p, xb, cudaMemcpyDeviceToHost, c->stream));
    return sync_and_check(c);
}

extern "C" int kq_swiglu_fp16_rows(kq_ctx *c, uint16_t *gate, const uint16_t *up, int M, int N) {
    if (!c || !gate || !up) return fail(c, KQ_ERR_INVALID_ARGUMENT, "NULL argument");
    if (int r = validate_mk(c, M, N)) return r;
    cudaSetDevice(c->device);
    const size_t xb = (size_t)M * N * 2;
    if (int r = ensure(c, c->tmp, xb)) return r;
    if (int r = ensure(c, c->x, xb)) return r;
    KQ_CUDA(c, cudaMemcpyAsync(c->x.p, gate, xb, cudaMemcpyHostToDevice, c->stream));
    KQ_CUDA(c, cudaMemcpyAsync(c->tmp.p, up, xb, cudaMemcpyHostToDevice, c->stream));
    if (int r = kq_swiglu_q8k_async(c, reinterpret_cast<uint16_t *>(c->x.p), reinterpret_cast<uint16_t *>(c->tmp.p), M,
                                    N, nullptr))
        return r;
    KQ_CUDA(c, cudaMemcpyAsync(gate, c->x.p, xb, cudaMemcpyDeviceToHost, c->stream));
    return sync_and_check(c);
}

// =================================================================== FFN block

extern "C" int kq_run_ffn_async(kq_ctx *c, const kq_weight *gate, const kq_weight *up, const kq_weight *down, int M,
                                const uint16_t *x_in, const uint16_t *gamma, uint16_t *x_out) {
    if (!c || !gate || !up || !down || !x_in || !gamma || !x_out)
        return fail(c, KQ_ERR_INVALID_ARGUMENT, "NULL argument");
    for (const kq_weight *w : {gate, up, down})
        if (int r = check_weight_device(c, w)) return r;
    const int hidden = gate->cols, ffn = gate->rows;
    if (up->cols != hidden || up->rows != ffn || down->cols != ffn || down->rows != hidden)
        return fail(c, KQ_ERR_SHAPE, "FFN weights do not chain: gate %dx%d up %dx%d down %dx%d", gate->rows,
                    gate->cols, up->rows, up->cols, down->rows, down->cols);
    if (int r = validate_mk(c, M, hidden)) return r;
    if (ffn % 256) return fail(c, KQ_ERR_SHAPE, "ffn dim %d not a multiple of 256", ffn);
    // scratch: xn [M][hidden] fp16 | g [M][ffn] | u [M][ffn] | q8k(xn) | q8k(h) | q80 forms
    const size_t xnb = (size_t)M * hidden * 2, gb = (size_t)M * ffn * 2;
    const size_t qa = (size_t)M * (hidden / 256) * sizeof(kq::BlockQ8K);
    const size_t qh = (size_t)M * (ffn / 256) * sizeof(kq::BlockQ8K);
    const size_t qa0 = (size_t)M * (hidden / 32) * sizeof(kq::BlockQ80);
    const size_t qh0 = (size_t)M * (ffn / 32) * sizeof(kq::BlockQ80);
    auto al = [](size_t v) { return (v + 255) & ~(size_t)255; };
    const size_t total = al(xnb) + 2 * al(gb) + al(qa) + al(qh) + al(qa0) + al(qh0);
    if (int r = ensure(c, c->misc, total)) return r;
    uint8_t *base = reinterpret_cast<uint8_t *>(c->misc.p);
    uint16_t *xn = reinterpret_cast<uint16_t *>(base);
    uint16_t *g = reinterpret_cast<uint16_t *>(base + al(xnb));
    uint16_t *u = reinterpret_cast<uint16_t *>(base + al(xnb) + al(gb));
    void *q_a = base + al(xnb) + 2 * al(gb);
    void *q_h = (uint8_t *)q_a + al(qa);
    void *q_a0 = (uint8_t *)q_h + al(qh);
    void *q_h0 = (uint8_t *)q_a0 + al(qa0);

    if (c->ffn_fused && gate->type == up->type &&
        kq::ffn_fused_supported((int)gate->type, (int)down->type, hidden, ffn, M, c->num_sms)) {
        // the whole block as one persistent kernel (bit for bit the launches below)
        const size_t sb = kq::gemv_split_bytes((int)down->type, ffn, M, c->num_sms);
        if (int r = ensure(c, c->gsplit, sb)) return r;
        if (int r = split_counts(c, (size_t)ffn / 16)) return r;
        kq::FfnFusedLaunch F{};
        F.gate_type = (int)gate->type;
        F.down_type = (int)down->type;
        F.hidden = hidden;
        F.ffn = ffn;
        F.M = M;
        F.gate = gate->d;
        F.up = up->d;
        F.down = down->d;
        F.x = x_in;
        F.gamma = gamma;
        F.g = g;
        F.u = u;
        F.y = x_out;
        F.exp_tab = swiglu_table(c);
        F.split_terms = static_cast<float *>(c->gsplit.p);
        F.split_count = static_cast<int *>(c->gcount.p);
        F.gbar = reinterpret_cast<unsigned *>(static_cast<int *>(c->gcount.p) + kq::gemv_split_slots(c->num_sms));
        F.pair = static_cast<int *>(c->gcount.p) + kq::gemv_split_slots(c->num_sms) + 2;
        F.status = c->d_status;
        F.timeout_ns = c->timeout_ns;
        F.pdl = c->pdl;
        F.num_sms = c->num_sms;
        KQ_CUDA(c, kq::launch_ffn_fused(F, c->stream));
        return KQ_OK;
    }
    // RMSNorm (+ Q8_K), ENG:8285
    KQ_CUDA(c, kq::launch_rmsnorm_q8k(x_in, gamma, xn, q_a, M, hidden, c->stream, c->pdl));
    const bool gu_q80 = gate->type == KQ_TYPE_Q8_0 || up->type == KQ_TYPE_Q8_0;
    if (gu_q80) KQ_CUDA(c, kq::launch_quantize(KQ_TYPE_Q8_0, xn, hidden, M, hidden, q_a0, c->stream));
    // gate / up, ENG:8287-8290
    kq_task gu[2] = {};
    gu[0].w = gate;
    gu[0].rows = ffn;
    gu[0].dst = g;
    gu[0].dst_stride = ffn;
    gu[1].w = up;
    gu[1].rows = ffn;
    gu[1].dst = u;
    gu[1].dst_stride = ffn;
    if (int r = run_gemv(c, gu, 2, M, hidden, nullptr, 0, q_a, gu_q80 ? q_a0 : nullptr)) return r;
    // SwiGLU (+ Q8_K), ENG:8292
    KQ_CUDA(c, kq::launch_swiglu_q8k(g, u, q_h, M, ffn, c->stream, c->pdl, swiglu_table(c)));
    if (down->type == KQ_TYPE_Q8_0) KQ_CUDA(c, kq::launch_quantize(KQ_TYPE_Q8_0, g, ffn, M, ffn, q_h0, c->stream));
    // down + residual, ENG:8294-8296
    kq_task dn{};
    dn.w = down;
    dn.rows = hidden;
    dn.dst = x_out;
    dn.dst_stride = hidden;
    dn.residual = x_in;
    dn.res_stride = hidden;
    return run_gemv(c, &dn, 1, M, ffn, nullptr, 0, q_h, down->type == KQ_TYPE_Q8_0 ? q_h0 : nullptr);
}

extern "C" int kq_run_ffn(kq_ctx *c, const kq_weight *gate, const kq_weight *up, const kq_weight *down, int M,
                          const uint16_t *x_in, const uint16_t *gamma, uint16_t *x_out) {
    if (!c || !gate || !x_in || !gamma || !x_out) return fail(c, KQ_ERR_INVALID_ARGUMENT, "NULL argument");
    if (M < 1 || M > KQ_MAX_M) return fail(c, KQ_ERR_SHAPE, "batch_len = %d", M);
    cudaSetDevice(c->device);
    const int hidden = gate->cols;
    const size_t xb = (size_t)M * hidden * 2;
    if (int r = ensure(c, c->x, 2 * xb + (size_t)hidden * 2 + 32)) return r;
    uint16_t *dx = reinterpret_cast<uint16_t *>(c->x.p);
    uint16_t *dy = dx + (size_t)M * hidden;
    uint16_t *dg = dy + (size_t)M * hidden;
    KQ_CUDA(c, cudaMemcpyAsync(dx, x_in, xb, cudaMemcpyHostToDevice, c->stream));
    KQ_CUDA(c, cudaMemcpyAsync(dg, gamma, (size_t)hidden * 2, cudaMemcpyHostToDevice, c->stream));
    if (int r = kq_run_ffn_async(c, gate, up, down, M, dx, dg, dy)) return r;
    KQ_CUDA(c, cudaMemcpyAsync(x_out, dy, xb, cudaMemcpyDeviceToHost, c->stream));
    c->cur_M = 0;  // the FFN leaves no current input behind
    return sync_and_check(c);
}

// =================================================================== dequant

extern "C" int kq_dequant_rows_async(kq_ctx *c, const kq_weight *w, int row_begin, int rows, uint16_t *dst) {
    if (!c || !w || !dst) return fail(c, KQ_ERR_INVALID_ARGUMENT, "NULL argument");
    if (int r = check_weight_device(c, w)) return r;
    if (row_begin < 0 || rows < 0 || (long long)row_begin + rows > w->rows) return fail(c, KQ_ERR_SHAPE, "row range");
    KQ_CUDA(c, kq::launch_dequant((int)w->type, w->d, row_begin, rows, w->cols, dst, c->stream));
    return KQ_OK;
}

extern "C" int kq_dequant_rows(kq_ctx *c, const kq_weight *w, int row_begin, int rows, uint16_t *dst) {
    if (!c || !w || !dst) return fail(c, KQ_ERR_INVALID_ARGUMENT, "NULL argument");
    cudaSetDevice(c->device);
    const size_t b = (size_t)rows * w->cols * 2;
    if (int r = ensure(c, c->tmp, b + 16)) return r;
    if (int r = kq_dequant_rows_async(c, w, row_begin, rows, reinterpret_cast<uint16_t *>(c->tmp.p))) return r;
    KQ_CUDA(c, cudaMemcpyAsync(dst, c->tmp.p, b, cudaMemcpyDeviceToHost, c->stream));
    return sync_and_check(c);
}

extern "C" int kq_embed_rows_async(kq_ctx *c, const kq_weight *w, const uint32_t *ids, int n, uint16_t *dst) {
    if (!c || !w || !ids || !dst) return fail(c, KQ_ERR_INVALID_ARGUMENT, "NULL argument");
    if (int r = check_weight_device(c, w)) return r;
    if (n < 0) return fail(c, KQ_ERR_SHAPE, "n = %d", n);
    KQ_CUDA(c, kq::launch_dequant((int)w->type, w->d, 0, n, w->cols, dst, c->stream, ids, w->rows, c->d_status));
    return KQ_OK;
}

extern "C" int kq_embed_rows(kq_ctx *c, const kq_weight *w, const uint32_t *ids, int n, uint16_t *dst) {
    if (!c || !w || !ids || !dst) return fail(c, KQ_ERR_INVALID_ARGUMENT, "NULL argument");
    if (n < 0) return fail(c, KQ_ERR_SHAPE, "n = %d", n);
    for (int i = 0; i < n; ++i)
        if (ids[i] >= (uint32_t)w->rows) return fail(c, KQ_ERR_SHAPE, "id %u past the weight's %d rows", ids[i], w->rows);
    if (n == 0) return KQ_OK;
    cudaSetDevice(c->device);
    const size_t ob = (size_t)n * w->cols * 2, ib = ((size_t)n * 4 + 255) & ~(size_t)255;
    if (int r = ensure(c, c->tmp, ib + ob + 16)) return r;
    uint32_t *dids = reinterpret_cast<uint32_t *>(c->tmp.p);
    uint16_t *dout = reinterpret_cast<uint16_t *>(reinterpret_cast<uint8_t *>(c->tmp.p) + ib);
    KQ_CUDA(c, cudaMemcpyAsync(dids, ids, (size_t)n * 4, cudaMemcpyHostToDevice, c->stream));
    if (int r = kq_embed_rows_async(c, w, dids, n, dout)) return r;
    KQ_CUDA(c, cudaMemcpyAsync(dst, dout, ob, cudaMemcpyDeviceToHost, c->stream));
    return sync_and_check(c);
}

// =================================================================== LM head

extern "C" int kq_lm_head_argmax_async(kq_ctx *c, const kq_weight *w, const uint16_t *x, int M, uint16_t *logits,
                                       float *logits_f32, uint32_t *toks, float *vals) {
    if (!c || !w || !x) return fail(c, KQ_ERR_INVALID_ARGUMENT, "NULL argument");
    if (int r = check_weight_device(c, w)) return r;
    if (int r = validate_mk(c, M, w->cols)) return r;
    if (int r = ensure(c, c->keys, (size_t)M * 8)) return r;
    auto *keys = reinterpret_cast<unsigned long long *>(c->keys.p);
    KQ_CUDA(c, cudaMemsetAsync(keys, 0, (size_t)M * 8, c->stream));
    kq_task t{};
    t.w = w;
    t.rows = w->rows;
    t.dst = logits;
    t.dst_stride = (size_t)w->rows;
    t.dst_f32 = logits_f32;
    t.dst_f32_stride = (size_t)w->rows;
    if (M > 8) {
        // many tokens: the logits come from the tensor-core path (or GEMV tiles, by the cost
        // model) into the caller's fp16 buffer or a scratch one, then one scan of the fp16 logits
        if (!t.dst) {
            if (int r = ensure(c, c->lmlogits, (size_t)M * w->rows * 2)) return r;
            t.dst = reinterpret_cast<uint16_t *>(c->lmlogits.p);
        }
        if (int r = run_gemv(c, &t, 1, M, w->cols, reinterpret_cast<const __half *>(x), w->cols, nullptr, nullptr))
            return r;
        KQ_CUDA(c, kq::launch_logits_argmax(t.dst, (long long)w->rows, w->rows, M, keys, c->stream));
        KQ_CUDA(c, kq::launch_argmax_finalize(keys, M, nullptr, toks, vals, c->stream));
        return KQ_OK;
    }
    GemvExtra ex;
    ex.argmax = keys;
    ex.argmax_f16 = 1;  // the reference scans the fp16 logits the dispatch stored (ENG:9699-9707)
    if (int r = run_gemv(c, &t, 1, M, w->cols, reinterpret_cast<const __half *>(x), w->cols, nullptr, nullptr, ex))
        return r;
    KQ_CUDA(c, kq::launch_argmax_finalize(keys, M, nullptr, toks, vals, c->stream));
    return KQ_OK;
}

extern "C" int kq_lm_head_argmax(kq_ctx *c, const kq_weight *w, const uint16_t *x, int M, uint16_t *logits,
                                 uint32_t *toks, float *vals) {
    if (!c || !w || !x || !toks || !vals) return fail(c, KQ_ERR_INVALID_ARGUMENT, "NULL argument");
    if (int r = validate_mk(c, M, w->cols)) return r;
    cudaSetDevice(c->device);
    const int K = w->cols, V = w->rows;
    if (int r = h2d(c, c->x, x, (size_t)M * K * 2)) return r;
    if (logits)
        if (int r = ensure(c, c->out16, (size_t)M * V * 2)) return r;
    if (int r = ensure(c, c->misc, (size_t)M * 8)) return r;
    uint32_t *dt = reinterpret_cast<uint32_t *>(c->misc.p);
    float *dv = reinterpret_cast<float *>(dt + M);
    if (int r = kq_lm_head_argmax_async(c, w, reinterpret_cast<uint16_t *>(c->x.p), M,
                                        logits ? reinterpret_cast<uint16_t *>(c->out16.p) : nullptr, nullptr, dt, dv))
        return r;
    set_current_x(c, M, K);
    if (logits) KQ_CUDA(c, cudaMemcpyAsync(logits, c->out16.p, (size_t)M * V * 2, cudaMemcpyDeviceToHost, c->stream));
    KQ_CUDA(c, cudaMemcpyAsync(toks, dt, (size_t)M * 4, cudaMemcpyDeviceToHost, c->stream));
    KQ_CUDA(c, cudaMemcpyAsync(vals, dv, (size_t)M * 4, cudaMemcpyDeviceToHost, c->stream));
    return sync_and_check(c);
}

extern "C" int kq_eval_indexed_rows_argmax(kq_ctx *c, const kq_weight *w, const uint32_t *row_ids, int n_rows, int M,
                                           uint16_t *logits_m1, uint32_t *top_toks, float *top_vals) {
    if (!c || !w || !row_ids || !top_toks || !top_vals) return fail(c, KQ_ERR_INVALID_ARGUMENT, "NULL argument");
    if (int r = check_weight_device(c, w)) return r;
    if (n_rows <= 0 || M <= 0) return KQ_OK;  // ENG:9591
    if (logits_m1 && M != 1) return fail(c, KQ_ERR_INVALID_ARGUMENT, "logits_m1 needs M == 1 (ENG:9569)");
    if (c->cur_M == 0) return fail(c, KQ_ERR_NOT_READY, "no current input");
    if (w->cols != c->cur_K || M > c->cur_M) return fail(c, KQ_ERR_SHAPE, "input shape mismatch");
    for (int i = 0; i < n_rows; ++i)
        if ((int)row_ids[i] >= w->rows) return fail(c, KQ_ERR_SHAPE, "row id %u >= rows %d", row_ids[i], w->rows);
    cudaSetDevice(c->device);
    const void *act = nullptr;
    if (int r = current_act(c, w->type, &act)) return r;
    const size_t idb = (size_t)n_rows * 4, kb = (size_t)M * 8;
    const size_t gb = kq::weight_bytes((int)w->type, n_rows, w->cols);
    const size_t o_keys = (idb + 255) & ~(size_t)255, o_w = (o_keys + kb + (size_t)M * 8 + 255) & ~(size_t)255;
    if (int r = ensure(c, c->misc, o_w + gb)) return r;
    uint32_t *dids = reinterpret_cast<uint32_t *>(c->misc.p);
    auto *keys = reinterpret_cast<unsigned long long *>((uint8_t *)c->misc.p + o_keys);
    uint32_t *dt = reinterpret_cast<uint32_t *>(keys + M);
    float *dv = reinterpret_cast<float *>(dt + M);
    KQ_CUDA(c, cudaMemcpyAsync(dids, row_ids, idb, cudaMemcpyHostToDevice, c->stream));
    KQ_CUDA(c, cudaMemsetAsync(keys, 0, kb, c->stream));
    // the listed rows, gathered into a tiled tensor of n_rows rows
    kq_weight gw = *w;
    gw.rows = n_rows;
    gw.d = (uint8_t *)c->misc.p + o_w;
    gw.bytes = gb;
    KQ_CUDA(c, kq::launch_gather_rows((int)w->type, w->cols, w->d, dids, n_rows, gw.d, c->stream));
    kq_task t{};
    t.w = &gw;
    t.rows = n_rows;
    if (logits_m1) {
        if (int r = h2d(c, c->out16, logits_m1, (size_t)w->rows * 2)) return r;
        t.dst = reinterpret_cast<uint16_t *>(c->out16.p);
        t.dst_stride = (size_t)w->rows;
    }
    GemvExtra ex;
    ex.argmax = keys;
    ex.argmax_f16 = 0;  // the work item compares fp32 row results (ENG:9557-9571)
    ex.out_ids = dids;
    ex.no_pdl = true;
    const bool q80 = w->type == KQ_TYPE_Q8_0;
    if (int r = run_gemv(c, &t, 1, M, w->cols, nullptr, 0, q80 ? nullptr : act, q80 ? act : nullptr, ex)) return r;
    KQ_CUDA(c, kq::launch_argmax_finalize(keys, M, dids, dt, dv, c->stream));
    std::vector<uint32_t> bt(M);
    std::vector<float> bv(M);
    KQ_CUDA(c, cudaMemcpyAsync(bt.data(), dt, (size_t)M * 4, cudaMemcpyDeviceToHost, c->stream));
    KQ_CUDA(c, cudaMemcpyAsync(bv.data(), dv, (size_t)M * 4, cudaMemcpyDeviceToHost, c->stream));
    if (logits_m1)
        KQ_CUDA(c, cudaMemcpyAsync(logits_m1, c->out16.p, (size_t)w->rows * 2, cudaMemcpyDeviceToHost, c->stream));
    if (int r = sync_and_check(c)) return r;
    for (int m = 0; m < M; ++m) {  // merge into the running best, strict '>' (ENG:9606-9612)
        if (bv[m] > top_vals[m]) {
            top_vals[m] = bv[m];
            top_toks[m] = bt[m];
        }
    }
    return KQ_OK;
}

// =================================================================== several GPUs: the gather

namespace {

int check_peer_gather(kq_ctx *c, const kq_peer_gather *pg) {
    if (!pg) return fail(c, KQ_ERR_INVALID_ARGUMENT, "NULL kq_peer_gather");
    if (pg->world < 1 || pg->world > KQ_MAX_PEERS || pg->rank < 0 || pg->rank >= pg->world)
        return fail(c, KQ_ERR_INVALID_ARGUMENT, "rank %d of world %d (1..%d ranks)", pg->rank, pg->world, KQ_MAX_PEERS);
    if (pg->M < 1 || pg->M > 8) return fail(c, KQ_ERR_SHAPE, "gather M = %d outside [1, 8]", pg->M);
    if (pg->row_stride < 1 || pg->row_begin < 0)
        return fail(c, KQ_ERR_SHAPE, "row_stride %lld, row_begin %d", pg->row_stride, pg->row_begin);
    for (int q = 0; q < pg->world; ++q)
        if (!pg->regions[q]) return fail(c, KQ_ERR_INVALID_ARGUMENT, "region of rank %d is NULL", q);
    return KQ_OK;
}

}  // namespace

extern "C" size_t kq_peer_region_bytes(int M, long long row_stride) {
    if (M < 1 || row_stride < 1) return 0;
    return kq::PEER_CTRL_BYTES + 2 * (size_t)M * (size_t)row_stride * sizeof(unsigned long long);
}

extern "C" int kq_peer_alloc(kq_ctx *c, size_t bytes, void **region_dev, void *ipc_handle) {
    if (!c || !region_dev || !ipc_handle) return fail(c, KQ_ERR_INVALID_ARGUMENT, "NULL argument");
    if (bytes < kq::PEER_CTRL_BYTES) return fail(c, KQ_ERR_INVALID_ARGUMENT, "region of %zu bytes", bytes);
    static_assert(sizeof(cudaIpcMemHandle_t) == KQ_IPC_HANDLE_BYTES, "IPC handle size");
    cudaSetDevice(c->device);
    void *p = nullptr;
    KQ_CUDA(c, cudaMalloc(&p, bytes));
    cudaError_t e = cudaMemset(p, 0, bytes);
    cudaIpcMemHandle_t h;
    if (e == cudaSuccess) e = cudaIpcGetMemHandle(&h, p);
    if (e != cudaSuccess) {
        cudaFree(p);
        return cuda_fail(c, e, "peer region");
    }
    memcpy(ipc_handle, &h, sizeof h);
    *region_dev = p;
    return KQ_OK;
}

extern "C" int kq_peer_free(kq_ctx *c, void *region_dev) {
    if (!c || !region_dev) return fail(c, KQ_ERR_INVALID_ARGUMENT, "NULL argument");
    cudaSetDevice(c->device);
    KQ_CUDA(c, cudaFree(region_dev));
    return KQ_OK;
}

extern "C" int kq_peer_open(kq_ctx *c, const void *ipc_handle, void **region_dev) {
    if (!c || !ipc_handle || !region_dev) return fail(c, KQ_ERR_INVALID_ARGUMENT, "NULL argument");
    cudaSetDevice(c->device);
    cudaIpcMemHandle_t h;
    memcpy(&h, ipc_handle, sizeof h);
    KQ_CUDA(c, cudaIpcOpenMemHandle(region_dev, h, cudaIpcMemLazyEnablePeerAccess));
    return KQ_OK;
}

extern "C" int kq_peer_close(kq_ctx *c, void *region_dev) {
    if (!c || !region_dev) return fail(c, KQ_ERR_INVALID_ARGUMENT, "NULL argument");
    cudaSetDevice(c->device);
    KQ_CUDA(c, cudaIpcCloseMemHandle(region_dev));
    return KQ_OK;
}

extern "C" int kq_gemm_peer_gather_async(kq_ctx *c, const kq_weight *w, const uint16_t *x_dev,
                                         const kq_peer_gather *pg, float *out_dev) {
    if (!c || !w || !x_dev) return fail(c, KQ_ERR_INVALID_ARGUMENT, "NULL argument");
    if (int r = check_peer_gather(c, pg)) return r;
    if (int r = check_weight_device(c, w)) return r;
    if ((long long)pg->row_begin + w->rows > pg->row_stride)
        return fail(c, KQ_ERR_SHAPE, "rows [%d, %d) past row_stride %lld", pg->row_begin, pg->row_begin + w->rows,
                    pg->row_stride);
    cudaSetDevice(c->device);
    kq::PeerOut po;
    po.n = pg->world;
    po.rank = pg->rank;
    for (int q = 0; q < pg->world; ++q)
        po.buf[q] = reinterpret_cast<unsigned long long *>(static_cast<uint8_t *>(pg->regions[q]) + kq::PEER_CTRL_BYTES);
    uint8_t *own = static_cast<uint8_t *>(pg->regions[pg->rank]);
    po.step = reinterpret_cast<const unsigned long long *>(own + 64);
    po.row_stride = pg->row_stride;
    po.buf_stride = (long long)pg->M * pg->row_stride;
    po.row0 = pg->row_begin;
    kq_task t{};
    t.w = w;
    t.row_begin = 0;
    t.rows = w->rows;
    if (out_dev) {
        // the step completes inside the GEMV: this rank's rows straight to out, the others' rows
        // collected by the launch's last CTAs
        po.out = out_dev;
        po.rows = w->rows;
        po.M = pg->M;
        po.arrivals = reinterpret_cast<unsigned *>(own + 72);
        po.tail_done = reinterpret_cast<unsigned *>(own + 80);
        po.step_rw = reinterpret_cast<unsigned long long *>(own + 64);
        t.dst_f32 = out_dev + pg->row_begin;
        t.dst_f32_stride = (size_t)pg->row_stride;
    }
    GemvExtra ex;
    ex.peer = &po;
    return run_gemv(c, &t, 1, pg->M, w->cols, reinterpret_cast<const __half *>(x_dev), w->cols, nullptr, nullptr, ex);
}

extern "C" int kq_peer_gather_wait_async(kq_ctx *c, const kq_peer_gather *pg, float *out_dev) {
    if (!c) return fail(c, KQ_ERR_INVALID_ARGUMENT, "NULL argument");
    if (int r = check_peer_gather(c, pg)) return r;
    cudaSetDevice(c->device);
    uint8_t *own = static_cast<uint8_t *>(pg->regions[pg->rank]);
    kq::PeerWait W{};
    W.step = reinterpret_cast<unsigned long long *>(own + 64);
    W.arrivals = reinterpret_cast<unsigned *>(own + 76);
    W.buf = reinterpret_cast<const unsigned long long *>(own + kq::PEER_CTRL_BYTES);
    W.buf_stride = (long long)pg->M * pg->row_stride;
    W.n_entries = (long long)pg->M * pg->row_stride;
    W.out = out_dev;
    W.status = c->d_status;
    W.timeout_ns = c->timeout_ns;
    W.pdl = c->pdl;
    KQ_CUDA(c, kq::launch_peer_wait(W, c->stream));
    return KQ_OK;
}
