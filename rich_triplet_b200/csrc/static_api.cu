// static_api.cu -- rt_gemv_bf16_argmax_static: the greedy LM-head GEMV
// (y = W x over a BF16 matrix, then the argmax of y) whose only scratch is a
// file-scope device array, so the call path allocates no device memory.
//
// The kernel is the library's GEMV with the greedy epilogue: every CTA leaves
// its greedy state (largest value, its row, the sum of exp(y - max)) in a
// slot, bumps an arrival counter, and the last CTA to arrive combines the
// slots, writes the token and puts the counter back to zero.  Here the slots
// and the counter live in g_argmax_scratch instead of a context- or
// engine-owned allocation.  A launch in which a bounded wait gave up still
// runs the arrival protocol: its last CTA writes token -1 and returns every
// counter it used to zero, so the next call starts clean.
#include <cstddef>
#include <cstdlib>
#include <mutex>

#include "common.cuh"
#include "gemv.cuh"
#include "rt_internal.h"

namespace {

constexpr int kSlots = RT_ARGMAX_STATIC_SLOTS;
constexpr int kWarpsPerCta = 16;                             // the GEMV's largest CTA
constexpr int64_t kMaxTiles = RT_ARGMAX_STATIC_MAX_ROWS / 16;  // 16-row tiles
constexpr int kMaxDevices = 64;

struct ArgmaxScratch {
    rt::GreedySlot slot[kSlots];             // per-CTA greedy state
    uint32_t counter;                        // CTAs arrived; zero when a launch starts
    uint32_t tile_cnt[kMaxTiles];            // split-tile unit counters; zero when a launch starts
    float part[kSlots * kWarpsPerCta * 32];  // split-tile partial row sums
};

// Zero-initialised at module load; every launch that completes leaves
// `counter` and `tile_cnt` at zero again.
static __device__ __align__(256) ArgmaxScratch g_argmax_scratch;

struct DeviceSetup {
    bool ready = false;
    int num_sms = 0;
    ArgmaxScratch* scratch = nullptr;
};
DeviceSetup g_setup[kMaxDevices];
std::mutex g_setup_mu;

int report(char* errbuf, size_t errlen, int code, const char* fmt, ...) {
    if (errbuf && errlen) {
        va_list ap;
        va_start(ap, fmt);
        vsnprintf(errbuf, errlen, fmt, ap);
        va_end(ap);
    }
    return code;
}

// First call on a device: resolve the scratch address and raise the GEMV
// kernels' shared-memory limit (host-side calls only; nothing is allocated).
int setup_device(int dev, DeviceSetup* out, char* errbuf, size_t errlen) {
    std::lock_guard<std::mutex> lock(g_setup_mu);
    DeviceSetup& s = g_setup[dev];
    if (!s.ready) {
        void* p = nullptr;
        cudaError_t e = cudaGetSymbolAddress(&p, g_argmax_scratch);
        if (e != cudaSuccess)
            return report(errbuf, errlen, RT_E_CUDA, "rt_gemv_bf16_argmax_static: cudaGetSymbolAddress: %s",
                          cudaGetErrorString(e));
        int sms = 0;
        e = cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
        if (e != cudaSuccess || sms <= 0)
            return report(errbuf, errlen, RT_E_CUDA, "rt_gemv_bf16_argmax_static: SM count: %s",
                          cudaGetErrorString(e));
        rt::gemv_prepare();
        s.scratch = static_cast<ArgmaxScratch*>(p);
        s.num_sms = sms;
        s.ready = true;
    }
    *out = s;
    return RT_OK;
}

}  // namespace

extern "C" int rt_gemv_bf16_argmax_static(const void* w_dev, int64_t rows, int cols, const float* x_dev, float* y_dev,
                                          int32_t* token_dev, void* stream, char* errbuf, size_t errlen) {
    if (errbuf && errlen) errbuf[0] = '\0';
    if (!w_dev || !x_dev || !y_dev || !token_dev)
        return report(errbuf, errlen, RT_E_INVAL, "rt_gemv_bf16_argmax_static: null argument");
    if ((reinterpret_cast<uintptr_t>(w_dev) & 15) || (reinterpret_cast<uintptr_t>(x_dev) & 15))
        return report(errbuf, errlen, RT_E_INVAL, "rt_gemv_bf16_argmax_static: w and x must be 16-byte aligned");
    if (rows <= 0 || rows > RT_ARGMAX_STATIC_MAX_ROWS)
        return report(errbuf, errlen, RT_E_SHAPE, "rt_gemv_bf16_argmax_static: rows %lld outside [1, %d]",
                      static_cast<long long>(rows), RT_ARGMAX_STATIC_MAX_ROWS);
    if (cols <= 0 || cols % 8 || cols > (1 << 20))
        return report(errbuf, errlen, RT_E_SHAPE,
                      "rt_gemv_bf16_argmax_static: cols %d must be a positive multiple of 8, at most 2^20", cols);
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess)
        return report(errbuf, errlen, RT_E_CUDA, "rt_gemv_bf16_argmax_static: cudaGetDevice: %s", cudaGetErrorString(e));
    if (dev < 0 || dev >= kMaxDevices)
        return report(errbuf, errlen, RT_E_INVAL, "rt_gemv_bf16_argmax_static: device %d beyond the %d supported", dev,
                      kMaxDevices);
    DeviceSetup s;
    int rc = setup_device(dev, &s, errbuf, errlen);
    if (rc != RT_OK) return rc;

    const rt::GemvPlan p = rt::gemv_plan(rt::kBF16, rows, cols, 1, rt::kProPlain, rt::kEpiArgmax, s.num_sms, 1);
    if (p.warps == 0)
        return report(errbuf, errlen, RT_E_SHAPE, "rt_gemv_bf16_argmax_static: no launch geometry for cols %d", cols);
    if (p.grid > kSlots || p.warps > kWarpsPerCta || p.cnt_words > kMaxTiles ||
        p.part_floats > int64_t{kSlots} * kWarpsPerCta * 32)
        return report(errbuf, errlen, RT_E_SHAPE,
                      "rt_gemv_bf16_argmax_static: launch needs %d argmax slots, the static scratch holds %d", p.grid,
                      kSlots);
    CUtensorMap tmap;
    if (!rt::gemv_make_tmap(rt::kBF16, w_dev, rows, cols, p, &tmap))
        return report(errbuf, errlen, RT_E_CUDA, "rt_gemv_bf16_argmax_static: TMA descriptor rejected for [%lld, %d]",
                      static_cast<long long>(rows), cols);
    rt::GemvArgs a = {};
    a.w = static_cast<const uint8_t*>(w_dev);
    a.rows = rows;
    a.K = cols;
    a.x = x_dev;
    a.y = y_dev;
    uint8_t* base = reinterpret_cast<uint8_t*>(s.scratch);  // device address: offsets only, never dereferenced here
    a.am_slot = reinterpret_cast<rt::GreedySlot*>(base + offsetof(ArgmaxScratch, slot));
    a.am_counter = reinterpret_cast<uint32_t*>(base + offsetof(ArgmaxScratch, counter));
    a.tile_cnt = reinterpret_cast<uint32_t*>(base + offsetof(ArgmaxScratch, tile_cnt));
    a.part = reinterpret_cast<float*>(base + offsetof(ArgmaxScratch, part));
    a.token_out = token_dev;
    a.fail_token = 1;  // a launch whose bounded wait gave up reports itself as token -1
    // Test override: RT_TEST_MBAR_WAIT_ITERS=n bounds each weight-stream wait
    // to n polls, so that a test can make the bounded wait give up.
    if (const char* w = getenv("RT_TEST_MBAR_WAIT_ITERS")) a.wait_iters = static_cast<uint32_t>(strtoul(w, nullptr, 10));
    e = rt::gemv_launch(rt::kBF16, rt::kProPlain, rt::kEpiArgmax, a, tmap, p, static_cast<cudaStream_t>(stream), false);
    if (e != cudaSuccess)
        return report(errbuf, errlen, RT_E_CUDA, "rt_gemv_bf16_argmax_static: launch: %s", cudaGetErrorString(e));
    return RT_OK;
}
