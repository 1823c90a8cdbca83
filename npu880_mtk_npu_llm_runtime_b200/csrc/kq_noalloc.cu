// kq_noalloc.cu -- kq_lm_head_argmax_noalloc: the LM-head argmax without any allocation.
//
// For callers that cannot allocate device memory at call time.  The only scratch the LM-head
// argmax needs beyond its inputs and outputs -- one 64-bit (value, row) key per activation row,
// reduced with atomicMax -- lives in a file-scope static device array of KQ_NOALLOC_MAX_M slots,
// together with the device-side status word the kernels write on a wait timeout.  No cudaMalloc,
// cudaFree or allocating library routine is called.
#include "kq_common.cuh"
#include "kq_internal.h"
#include "../../include/kq.h"

#include <cuda.h>
#include <mutex>

namespace {

// Shared by every call on a device and kept between calls (cleared by each call).
static __device__ __align__(256) unsigned long long g_noalloc_keys[KQ_NOALLOC_MAX_M];
static __device__ __align__(256) int g_noalloc_status;

struct DeviceScratch {
    unsigned long long ctx_id = 0;       // CUDA context the addresses belong to (0: none yet)
    unsigned long long *keys = nullptr;  // device address of g_noalloc_keys
    int *status = nullptr;               // device address of g_noalloc_status
    int num_sms = 0;
};

constexpr int kMaxDevices = 64;
DeviceScratch g_scratch[kMaxDevices];
std::mutex g_scratch_mu;

// Unique id of the current CUDA context (cuCtxGetId, reached through the runtime so the library
// needs no link to the driver library); 0 when it cannot be had.
unsigned long long current_context_id() {
    using GetCurrent = CUresult (*)(CUcontext *);
    using GetId = CUresult (*)(CUcontext, unsigned long long *);
    static GetCurrent get_current = nullptr;
    static GetId get_id = nullptr;
    static std::once_flag once;
    std::call_once(once, [] {
        void *f = nullptr;
        cudaDriverEntryPointQueryResult q{};
        if (cudaGetDriverEntryPoint("cuCtxGetCurrent", &f, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            get_current = reinterpret_cast<GetCurrent>(f);
        f = nullptr;
        if (cudaGetDriverEntryPoint("cuCtxGetId", &f, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            get_id = reinterpret_cast<GetId>(f);
    });
    CUcontext ctx = nullptr;
    unsigned long long id = 0;
    if (!get_current || !get_id || get_current(&ctx) != CUDA_SUCCESS || !ctx || get_id(ctx, &id) != CUDA_SUCCESS)
        return 0;
    return id;
}

// With the device current: the device addresses of the static arrays, looked up once per
// device, and again when the device's context was replaced (cudaDeviceReset and a new context
// give the arrays new addresses; a first call made before the device had a context looks them up
// once more on its next call).  In host code the symbols themselves are host-side stand-ins,
// not device addresses.
int scratch_for_current_device(int *device, DeviceScratch **out) {
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess) return KQ_ERR_CUDA;
    if (dev < 0 || dev >= kMaxDevices) return KQ_ERR_INVALID_ARGUMENT;
    const unsigned long long id = current_context_id();
    std::lock_guard<std::mutex> lk(g_scratch_mu);
    DeviceScratch &s = g_scratch[dev];
    if (s.ctx_id == 0 || (id != 0 && id != s.ctx_id)) {
        void *keys = nullptr, *status = nullptr;
        if (cudaGetSymbolAddress(&keys, g_noalloc_keys) != cudaSuccess) return KQ_ERR_CUDA;
        if (cudaGetSymbolAddress(&status, g_noalloc_status) != cudaSuccess) return KQ_ERR_CUDA;
        int sms = 0;
        if (cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess) return KQ_ERR_CUDA;
        s.keys = static_cast<unsigned long long *>(keys);
        s.status = static_cast<int *>(status);
        s.num_sms = sms;
        s.ctx_id = id ? id : ~0ull;
    }
    *device = dev;
    *out = &s;
    return KQ_OK;
}

}  // namespace

extern "C" int kq_lm_head_argmax_noalloc(const kq_weight *w, const uint16_t *x_dev, int M, uint16_t *logits_dev,
                                         uint32_t *top_toks_dev, float *top_vals_dev, void *stream) {
    if (!w || !x_dev || !top_toks_dev || !top_vals_dev) return KQ_ERR_INVALID_ARGUMENT;
    if (w->type != KQ_TYPE_Q4_K && w->type != KQ_TYPE_Q5_K && w->type != KQ_TYPE_Q6_K && w->type != KQ_TYPE_Q8_0)
        return KQ_ERR_UNSUPPORTED_TYPE;
    if (M < 1 || M > KQ_NOALLOC_MAX_M) return KQ_ERR_SHAPE;
    const int K = w->cols;
    if (K < 256 || K > KQ_MAX_K || K % 256 || w->rows < 1) return KQ_ERR_SHAPE;
    int dev = 0;
    DeviceScratch *sc = nullptr;
    if (int r = scratch_for_current_device(&dev, &sc)) return r;
    if (w->device != dev) return KQ_ERR_INVALID_ARGUMENT;  // the weight lives on another GPU
    cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);

    // the array keeps the previous call's keys and status: clear what this call uses
    if (cudaMemsetAsync(sc->keys, 0, sizeof(unsigned long long) * M, st) != cudaSuccess) return KQ_ERR_CUDA;
    if (cudaMemsetAsync(sc->status, 0, sizeof(int), st) != cudaSuccess) return KQ_ERR_CUDA;

    // the fused GEMV + argmax of kq_lm_head_argmax_async, in tiles of up to 8 activation rows
    // (one pass over the weights per tile)
    for (int m0 = 0; m0 < M; m0 += 8) {
        const int mt = (M - m0 < 8) ? M - m0 : 8;
        kq::GemvLaunch L{};
        L.type = (int)w->type;
        L.K = K;
        L.M = mt;
        L.n_tasks = 1;
        kq::GemvTaskHost &h = L.tasks[0];
        h.w = w->d;
        h.row_begin = 0;
        h.rows = w->rows;
        h.dst = logits_dev ? (void *)(logits_dev + (size_t)m0 * w->rows) : nullptr;
        h.dst_stride = w->rows;
        h.index_base = 0;
        L.x = x_dev + (size_t)m0 * K;
        L.x_stride = K;
        L.status = sc->status;
        L.timeout_ns = 1000000000ull;
        L.pdl = true;
        L.num_sms = sc->num_sms;
        L.argmax = sc->keys + m0;
        L.argmax_f16 = 1;  // the reference scans the fp16 logits (ENG:9699-9707)
        if (kq::launch_gemv(L, st) != cudaSuccess) return KQ_ERR_CUDA;
    }
    // a timeout in any tile gives every row the (0xFFFFFFFF, NaN) sentinel
    if (kq::launch_argmax_finalize(sc->keys, M, nullptr, top_toks_dev, top_vals_dev, st, sc->status) != cudaSuccess)
        return KQ_ERR_CUDA;
    return KQ_OK;
}
