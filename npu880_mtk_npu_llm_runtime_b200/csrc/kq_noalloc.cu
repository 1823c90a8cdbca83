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

#include <mutex>

namespace {

// Shared by every call on a device and kept between calls (cleared by each call).
static __device__ __align__(256) unsigned long long g_noalloc_keys[KQ_NOALLOC_MAX_M];
static __device__ __align__(256) int g_noalloc_status;

struct DeviceScratch {
    bool ready = false;
    unsigned long long *keys = nullptr;  // device address of g_noalloc_keys
    int *status = nullptr;               // device address of g_noalloc_status
    int num_sms = 0;
};

constexpr int kMaxDevices = 64;
DeviceScratch g_scratch[kMaxDevices];
std::mutex g_scratch_mu;

// Once per device, with that device current: the device addresses of the static arrays.  In
// host code the symbols themselves are host-side stand-ins, not device addresses.
int scratch_for_current_device(DeviceScratch **out) {
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess) return KQ_ERR_CUDA;
    if (dev < 0 || dev >= kMaxDevices) return KQ_ERR_INVALID_ARGUMENT;
    std::lock_guard<std::mutex> lk(g_scratch_mu);
    DeviceScratch &s = g_scratch[dev];
    if (!s.ready) {
        void *keys = nullptr, *status = nullptr;
        if (cudaGetSymbolAddress(&keys, g_noalloc_keys) != cudaSuccess) return KQ_ERR_CUDA;
        if (cudaGetSymbolAddress(&status, g_noalloc_status) != cudaSuccess) return KQ_ERR_CUDA;
        int sms = 0;
        if (cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess) return KQ_ERR_CUDA;
        s.keys = static_cast<unsigned long long *>(keys);
        s.status = static_cast<int *>(status);
        s.num_sms = sms;
        s.ready = true;
    }
    *out = &s;
    return KQ_OK;
}

}  // namespace

extern "C" int kq_lm_head_argmax_noalloc(const kq_weight *w, const uint16_t *x_dev, int M, uint16_t *logits_dev,
                                         uint32_t *top_toks_dev, float *top_vals_dev, void *stream) {
    if (!w || !x_dev || !top_toks_dev || !top_vals_dev) return KQ_ERR_INVALID_ARGUMENT;
    if (M < 1 || M > KQ_NOALLOC_MAX_M) return KQ_ERR_SHAPE;
    const int K = w->cols;
    if (K < 256 || K % 256 || w->rows < 1) return KQ_ERR_SHAPE;
    DeviceScratch *sc = nullptr;
    if (int r = scratch_for_current_device(&sc)) return r;
    cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);

    // the array keeps the previous call's keys: clear the slots this call reduces into
    if (cudaMemsetAsync(sc->keys, 0, sizeof(unsigned long long) * M, st) != cudaSuccess) return KQ_ERR_CUDA;
    if (cudaMemsetAsync(sc->status, 0, sizeof(int), st) != cudaSuccess) return KQ_ERR_CUDA;

    // the fused GEMV + argmax of kq_lm_head_argmax_async, in tiles of up to 8 activation rows
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
    if (kq::launch_argmax_finalize(sc->keys, M, nullptr, top_toks_dev, top_vals_dev, st) != cudaSuccess)
        return KQ_ERR_CUDA;
    return KQ_OK;
}
