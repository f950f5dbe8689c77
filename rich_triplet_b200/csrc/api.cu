// api.cu -- C ABI (include/rt_cuda.h): context, weights, GEMV, conversions.
#include <stdarg.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>

#include <algorithm>
#include <vector>
#include <atomic>
#include <mutex>

#include "convert.cuh"
#include "gemm.cuh"
#include "gemv.cuh"

#include "rt_internal.h"

namespace rt {

int fail(rt_ctx* ctx, int code, const char* fmt, ...) {
    if (ctx) {
        char buf[512];
        va_list ap;
        va_start(ap, fmt);
        vsnprintf(buf, sizeof(buf), fmt, ap);
        va_end(ap);
        ctx->err = buf;
    }
    return code;
}

static std::atomic<long> g_alloc_count{0};

int dev_alloc(rt_ctx* ctx, void** p, size_t bytes, const char* what) {
    *p = nullptr;
    const long n = ++g_alloc_count;
    const char* inj = getenv("RT_FAULT_INJECT_ALLOC");
    if (inj && atol(inj) == n) return fail(ctx, RT_E_NOMEM, "injected allocation failure (%s, %zu bytes)", what, bytes);
    cudaError_t e = cudaMalloc(p, bytes ? bytes : 16);
    if (e != cudaSuccess) {
        cudaGetLastError();
        *p = nullptr;
        return fail(ctx, e == cudaErrorMemoryAllocation ? RT_E_NOMEM : RT_E_CUDA, "cudaMalloc(%s, %zu bytes): %s", what,
                    bytes, cudaGetErrorString(e));
    }
    return RT_OK;
}

uint64_t weight_bytes(int fmt, int64_t rows, int64_t cols) {
    if (rows <= 0 || cols <= 0) return 0;
    switch (fmt) {
        case RT_FMT_Q4K: return cols % 256 ? 0 : static_cast<uint64_t>(rows) * (cols / 256) * 144;
        case RT_FMT_BF16: return static_cast<uint64_t>(rows) * cols * 2;
        case RT_FMT_F32: return static_cast<uint64_t>(rows) * cols * 4;
        case RT_FMT_Q4_0: return cols % 32 ? 0 : static_cast<uint64_t>(rows) * (cols / 32) * 18;
        case RT_FMT_Q6K: return cols % 256 ? 0 : static_cast<uint64_t>(rows) * (cols / 256) * 210;
        default: return 0;
    }
}

}  // namespace rt

using rt::fail;

extern "C" {

const char* rt_version(void) { return "rich-triplet-b200 0.1 (sm_100a)"; }

int rt_init(int device, rt_ctx** out) {
    if (!out) return RT_E_INVAL;
    *out = nullptr;
    int n = 0;
    cudaError_t e = cudaGetDeviceCount(&n);
    if (e != cudaSuccess || n == 0) {
        cudaGetLastError();
        return RT_E_CUDA;
    }
    if (device < 0 || device >= n) return RT_E_INVAL;
    rt_ctx* ctx = new rt_ctx();
    ctx->device = device;
    if (cudaSetDevice(device) != cudaSuccess ||
        cudaDeviceGetAttribute(&ctx->num_sms, cudaDevAttrMultiProcessorCount, device) != cudaSuccess ||
        cudaStreamCreateWithFlags(&ctx->stream, cudaStreamNonBlocking) != cudaSuccess) {
        cudaGetLastError();
        delete ctx;
        return RT_E_CUDA;
    }
    if (rt::dev_alloc(ctx, reinterpret_cast<void**>(&ctx->d_err), sizeof(int) * 4, "error word") != RT_OK) {
        cudaStreamDestroy(ctx->stream);
        delete ctx;
        return RT_E_NOMEM;
    }
    cudaMemset(ctx->d_err, 0, sizeof(int) * 4);
    rt::gemv_prepare();
    (void)rt::gemv_cluster_prepare();
    cudaGetLastError();
    if (rt::gemm_q4k_prepare() != cudaSuccess) cudaGetLastError();  // a launch then reports the failure
    *out = ctx;
    return RT_OK;
}

void rt_destroy(rt_ctx* ctx) {
    if (!ctx) return;
    cudaSetDevice(ctx->device);
    if (ctx->stream) cudaStreamSynchronize(ctx->stream);
    cudaFree(ctx->scratch);
    cudaFree(ctx->io);
    cudaFree(ctx->gemv_part);
    cudaFree(ctx->gemv_cnt);
    cudaFree(ctx->d_err);
    if (ctx->stream) cudaStreamDestroy(ctx->stream);
    delete ctx;
}

const char* rt_last_error(const rt_ctx* ctx) { return ctx ? ctx->err.c_str() : "null context"; }

void* rt_stream(rt_ctx* ctx) { return ctx ? static_cast<void*>(ctx->stream) : nullptr; }

int rt_sync(rt_ctx* ctx) {
    if (!ctx) return RT_E_INVAL;
    RT_CHECK_CUDA(ctx, cudaStreamSynchronize(ctx->stream));
    int herr = 0;
    RT_CHECK_CUDA(ctx, cudaMemcpy(&herr, ctx->d_err, sizeof(int), cudaMemcpyDeviceToHost));
    if (herr) {
        cudaMemset(ctx->d_err, 0, sizeof(int));
        return fail(ctx, RT_E_TIMEOUT, "a kernel reported error word %d (bounded wait gave up)", herr);
    }
    return RT_OK;
}

int rt_weight_upload(rt_ctx* ctx, int fmt, const void* host, uint64_t bytes, int64_t rows, int64_t cols, rt_w** out) {
    if (!ctx || !host || !out) return fail(ctx, RT_E_INVAL, "rt_weight_upload: null argument");
    *out = nullptr;
    if (fmt != RT_FMT_Q4K && fmt != RT_FMT_BF16 && fmt != RT_FMT_F32)
        return fail(ctx, RT_E_FORMAT, "rt_weight_upload: format %d is not a resident weight format", fmt);
    const uint64_t need = rt::weight_bytes(fmt, rows, cols);
    if (need == 0) return fail(ctx, RT_E_SHAPE, "rt_weight_upload: invalid shape [%lld, %lld] for format %d",
                               static_cast<long long>(rows), static_cast<long long>(cols), fmt);
    if (fmt == RT_FMT_BF16 && cols % 8) return fail(ctx, RT_E_SHAPE, "rt_weight_upload: BF16 needs cols %% 8 == 0");
    if (bytes != need)
        return fail(ctx, RT_E_SHAPE, "rt_weight_upload: %llu bytes given, [%lld, %lld] needs %llu",
                    static_cast<unsigned long long>(bytes), static_cast<long long>(rows), static_cast<long long>(cols),
                    static_cast<unsigned long long>(need));
    RT_CHECK_CUDA(ctx, cudaSetDevice(ctx->device));
    rt_w* w = new rt_w();
    w->fmt = fmt;
    w->rows = rows;
    w->cols = cols;
    w->bytes = bytes;
    int rc = rt::dev_alloc(ctx, &w->d, bytes, "weight");
    if (rc != RT_OK) {
        delete w;
        return rc;
    }
    cudaError_t e = cudaMemcpyAsync(w->d, host, bytes, cudaMemcpyHostToDevice, ctx->stream);
    if (e == cudaSuccess) e = cudaStreamSynchronize(ctx->stream);
    if (e != cudaSuccess) {
        cudaFree(w->d);
        delete w;
        return fail(ctx, RT_E_CUDA, "rt_weight_upload: %s", cudaGetErrorString(e));
    }
    *out = w;
    return RT_OK;
}

int rt_weight_download(rt_ctx* ctx, const rt_w* w, void* host, uint64_t bytes) {
    if (!ctx || !w || !host) return fail(ctx, RT_E_INVAL, "rt_weight_download: null argument");
    if (bytes != w->bytes) return fail(ctx, RT_E_SHAPE, "rt_weight_download: weight holds %llu bytes",
                                       static_cast<unsigned long long>(w->bytes));
    RT_CHECK_CUDA(ctx, cudaMemcpyAsync(host, w->d, bytes, cudaMemcpyDeviceToHost, ctx->stream));
    RT_CHECK_CUDA(ctx, cudaStreamSynchronize(ctx->stream));
    return RT_OK;
}

int rt_weight_info(const rt_w* w, int* fmt, int64_t* rows, int64_t* cols, uint64_t* bytes) {
    if (!w) return RT_E_INVAL;
    if (fmt) *fmt = w->fmt;
    if (rows) *rows = w->rows;
    if (cols) *cols = w->cols;
    if (bytes) *bytes = w->bytes;
    return RT_OK;
}

const void* rt_weight_device_ptr(const rt_w* w) { return w ? w->d : nullptr; }

void rt_weight_free(rt_ctx* ctx, rt_w* w) {
    if (!w) return;
    if (ctx) {
        cudaSetDevice(ctx->device);
        cudaStreamSynchronize(ctx->stream);
    }
    cudaFree(w->d);
    delete w;
}

}  // extern "C"

namespace {

int ensure_scratch(rt_ctx* ctx, size_t floats) {
    if (ctx->scratch_floats >= floats) return RT_OK;
    RT_CHECK_CUDA(ctx, cudaStreamSynchronize(ctx->stream));
    cudaFree(ctx->scratch);
    ctx->scratch = nullptr;
    ctx->scratch_floats = 0;
    int rc = rt::dev_alloc(ctx, reinterpret_cast<void**>(&ctx->scratch), floats * sizeof(float), "gemv scratch");
    if (rc != RT_OK) return rc;
    ctx->scratch_floats = floats;
    return RT_OK;
}

int ensure_io(rt_ctx* ctx, size_t floats) {
    if (ctx->io_floats >= floats) return RT_OK;
    RT_CHECK_CUDA(ctx, cudaStreamSynchronize(ctx->stream));
    cudaFree(ctx->io);
    ctx->io = nullptr;
    ctx->io_floats = 0;
    int rc = rt::dev_alloc(ctx, reinterpret_cast<void**>(&ctx->io), floats * sizeof(float), "qlinear io");
    if (rc != RT_OK) return rc;
    ctx->io_floats = floats;
    return RT_OK;
}

int ensure_gemv_scratch(rt_ctx* ctx, const rt::GemvPlan& p) {
    if (ctx->gemv_part_floats >= p.part_floats && ctx->gemv_cnt_words >= p.cnt_words) return RT_OK;
    RT_CHECK_CUDA(ctx, cudaStreamSynchronize(ctx->stream));
    const int64_t pf = std::max(ctx->gemv_part_floats, p.part_floats);
    const int64_t cw = std::max(ctx->gemv_cnt_words, p.cnt_words);
    cudaFree(ctx->gemv_part);
    cudaFree(ctx->gemv_cnt);
    ctx->gemv_part = nullptr;
    ctx->gemv_cnt = nullptr;
    ctx->gemv_part_floats = ctx->gemv_cnt_words = 0;
    int rc = rt::dev_alloc(ctx, reinterpret_cast<void**>(&ctx->gemv_part), sizeof(float) * pf, "gemv partials");
    if (rc != RT_OK) return rc;
    rc = rt::dev_alloc(ctx, reinterpret_cast<void**>(&ctx->gemv_cnt), sizeof(uint32_t) * cw, "gemv counters");
    if (rc != RT_OK) return rc;
    RT_CHECK_CUDA(ctx, cudaMemsetAsync(ctx->gemv_cnt, 0, sizeof(uint32_t) * cw, ctx->stream));
    ctx->gemv_part_floats = pf;
    ctx->gemv_cnt_words = cw;
    return RT_OK;
}

int gemv_common(rt_ctx* ctx, const rt_w* wc, const float* x, float* y, int flags, int kind) {
    rt_w* w = const_cast<rt_w*>(wc);  // caches its launch plan and TMA descriptor
    if (!ctx || !w || !x || !y) return fail(ctx, RT_E_INVAL, "gemv: null argument");
    if (flags != RT_HOST && flags != RT_DEVICE) return fail(ctx, RT_E_INVAL, "gemv: flags must be RT_HOST or RT_DEVICE");
    const int want = kind == rt::kQ4K ? RT_FMT_Q4K : RT_FMT_BF16;
    if (w->fmt != want) return fail(ctx, RT_E_FORMAT, "gemv: weight format %d, this entry point takes %d", w->fmt, want);
    if (w->cols > (1 << 20)) return fail(ctx, RT_E_SHAPE, "gemv: cols %lld too large", static_cast<long long>(w->cols));
    RT_CHECK_CUDA(ctx, cudaSetDevice(ctx->device));
    const int K = static_cast<int>(w->cols);
    if (!w->gemv_ready) {
        // Q4_K: the cluster kernel (gemv_cluster.cu); BF16: the generic one
        w->plan = kind == rt::kQ4K ? rt::gemv_cluster_plan(w->rows, K, ctx->num_sms)
                                   : rt::gemv_plan(kind, w->rows, K, 1, rt::kProPlain, rt::kEpiPlain, ctx->num_sms, 1);
        if (w->plan.warps == 0) return fail(ctx, RT_E_SHAPE, "gemv: no launch geometry for cols %d", K);
        if (!rt::gemv_make_tmap(kind, w->d, w->rows, K, w->plan, &w->tmap))
            return fail(ctx, RT_E_CUDA, "gemv: TMA descriptor rejected for [%lld, %d]", static_cast<long long>(w->rows), K);
        w->gemv_ready = true;
    }
    const rt::GemvPlan& p = w->plan;
    if (int rc = ensure_gemv_scratch(ctx, p); rc != RT_OK) return rc;
    const float* dx = x;
    float* dy = y;
    if (flags == RT_DEVICE && (reinterpret_cast<uintptr_t>(x) & 15))
        return fail(ctx, RT_E_INVAL, "gemv: device x must be 16-byte aligned");
    if (flags == RT_HOST) {
        int rc = ensure_scratch(ctx, static_cast<size_t>(K) + static_cast<size_t>(w->rows));
        if (rc != RT_OK) return rc;
        dx = ctx->scratch;
        dy = ctx->scratch + K;
        RT_CHECK_CUDA(ctx, cudaMemcpyAsync(const_cast<float*>(dx), x, sizeof(float) * K, cudaMemcpyHostToDevice, ctx->stream));
    }
    rt::GemvArgs a = {};
    a.w = static_cast<const uint8_t*>(w->d);
    a.rows = w->rows;
    a.K = K;
    a.x = dx;
    a.y = dy;
    a.part = ctx->gemv_part;
    a.tile_cnt = ctx->gemv_cnt;
    a.err = ctx->d_err;
    if (kind == rt::kQ4K)
        RT_CHECK_CUDA(ctx, rt::gemv_cluster_launch(a, w->tmap, p, ctx->stream, false));
    else
        RT_CHECK_CUDA(ctx, rt::gemv_launch(kind, rt::kProPlain, rt::kEpiPlain, a, w->tmap, p, ctx->stream, false));
    if (flags == RT_HOST) {
        RT_CHECK_CUDA(ctx, cudaMemcpyAsync(y, dy, sizeof(float) * w->rows, cudaMemcpyDeviceToHost, ctx->stream));
        return rt_sync(ctx);
    }
    return RT_OK;
}

int gemm_common(rt_ctx* ctx, const rt_w* w, const void* a, int64_t m, float* c, int flags, int fmt,
                bool a_f32 = false) {
    if (!ctx || !w || !a || !c) return fail(ctx, RT_E_INVAL, "rt_gemm: null argument");
    if (flags != RT_HOST && flags != RT_DEVICE) return fail(ctx, RT_E_INVAL, "rt_gemm: flags must be RT_HOST or RT_DEVICE");
    if (w->fmt != fmt) return fail(ctx, RT_E_FORMAT, "rt_gemm: weight format %d, this entry point takes %d", w->fmt, fmt);
    const int64_t n = w->rows;
    const int k = static_cast<int>(w->cols);
    const rt::GemmPlan p = rt::gemm_q4k_plan(m, n, k, ctx->num_sms, fmt == RT_FMT_BF16, true);
    if (p.bm == 0) return fail(ctx, RT_E_SHAPE, "rt_gemm: no launch geometry for M %lld, N %lld, K %d",
                               static_cast<long long>(m), static_cast<long long>(n), k);
    RT_CHECK_CUDA(ctx, cudaSetDevice(ctx->device));
    const size_t a_bytes = static_cast<size_t>(m) * k * (a_f32 ? 4 : 2);
    const size_t a16_bytes = static_cast<size_t>(m) * k * 2;
    if (flags == RT_DEVICE && ((reinterpret_cast<uintptr_t>(a) & 15) || (reinterpret_cast<uintptr_t>(c) & 15)))
        return fail(ctx, RT_E_INVAL, "rt_gemm: device A and C must be 16-byte aligned");
    // scratch: [A (host calls)] [A as fp16 rows] [row scales] [C (host calls)]
    // [split partials], each 256-byte aligned
    auto al = [](size_t floats) { return (floats + 63) / 64 * 64; };
    const size_t a_floats = flags == RT_HOST ? al((a_bytes + 3) / 4) : 0;
    const size_t a16_floats = al((a16_bytes + 3) / 4), s_floats = al(static_cast<size_t>(m));
    const size_t c_floats = flags == RT_HOST ? al(static_cast<size_t>(m) * n) : 0;
    const size_t part_floats = p.splits > 1 ? static_cast<size_t>(p.splits) * m * n : 0;
    int rc = ensure_scratch(ctx, a_floats + a16_floats + s_floats + c_floats + part_floats);
    if (rc != RT_OK) return rc;
    const void* da = flags == RT_HOST ? static_cast<const void*>(ctx->scratch) : a;
    uint16_t* a16 = reinterpret_cast<uint16_t*>(ctx->scratch + a_floats);
    float* ascale = ctx->scratch + a_floats + a16_floats;
    float* dc = flags == RT_HOST ? ascale + s_floats : c;
    float* parts = ascale + s_floats + c_floats;
    if (flags == RT_HOST)
        RT_CHECK_CUDA(ctx, cudaMemcpyAsync(const_cast<void*>(da), a, a_bytes, cudaMemcpyHostToDevice, ctx->stream));
    if (a_f32)
        RT_CHECK_CUDA(ctx, rt::a_f32_to_f16_launch(static_cast<const float*>(da), m, k, a16, ascale, ctx->stream));
    else
        RT_CHECK_CUDA(ctx, rt::a_to_f16_launch(static_cast<const uint16_t*>(da), m, k, a16, ascale, ctx->stream));
    CUtensorMap tm_a, tm_w;
    if (!rt::gemm_q4k_tmaps(a16, m, w->d, n, k, p, &tm_a, &tm_w))
        return fail(ctx, RT_E_CUDA, "rt_gemm: TMA descriptor rejected");
    RT_CHECK_CUDA(ctx, rt::gemm_q4k_launch(tm_a, tm_w, ascale, p.splits > 1 ? parts : dc, m, n, k, p, ctx->d_err,
                                           ctx->stream, a16));
    if (p.splits > 1)
        RT_CHECK_CUDA(ctx, rt::sum_parts_launch(parts, p.splits, static_cast<int64_t>(m) * n, dc, ctx->num_sms, ctx->stream));
    if (flags == RT_HOST) {
        RT_CHECK_CUDA(ctx, cudaMemcpyAsync(c, dc, sizeof(float) * static_cast<size_t>(m) * n, cudaMemcpyDeviceToHost,
                                           ctx->stream));
        return rt_sync(ctx);
    }
    return RT_OK;
}

}  // namespace

extern "C" {

int rt_gemv_q4k(rt_ctx* ctx, const rt_w* w, const float* x, float* y, int flags) {
    return gemv_common(ctx, w, x, y, flags, rt::kQ4K);
}

int rt_gemv_bf16(rt_ctx* ctx, const rt_w* w, const float* x, float* y, int flags) {
    return gemv_common(ctx, w, x, y, flags, rt::kBF16);
}

int rt_gemm_q4k(rt_ctx* ctx, const rt_w* w, const void* a, int64_t m, float* c, int flags) {
    return gemm_common(ctx, w, a, m, c, flags, RT_FMT_Q4K);
}

int rt_gemm_bf16(rt_ctx* ctx, const rt_w* w, const void* a, int64_t m, float* c, int flags) {
    return gemm_common(ctx, w, a, m, c, flags, RT_FMT_BF16);
}

int rt_qlinear_forward(rt_ctx* ctx, const rt_w* w, const float* x, int64_t t, const float* bias, float* y, int flags) {
    if (!ctx || !w || !x || !y) return fail(ctx, RT_E_INVAL, "rt_qlinear_forward: null argument");
    if (flags != RT_HOST && flags != RT_DEVICE)
        return fail(ctx, RT_E_INVAL, "rt_qlinear_forward: flags must be RT_HOST or RT_DEVICE");
    if (w->fmt != RT_FMT_Q4K && w->fmt != RT_FMT_BF16)
        return fail(ctx, RT_E_FORMAT, "rt_qlinear_forward: weight format %d (Q4_K or BF16 only)", w->fmt);
    if (t < 1 || t > (int64_t{1} << 24)) return fail(ctx, RT_E_SHAPE, "rt_qlinear_forward: t = %lld rows", static_cast<long long>(t));
    RT_CHECK_CUDA(ctx, cudaSetDevice(ctx->device));
    const int64_t in = w->cols, out = w->rows;
    const float* dx = x;
    const float* db = bias;
    float* dy = y;
    if (flags == RT_HOST) {
        // device copies: [x][bias][y], each 256-byte aligned
        auto al = [](int64_t f) { return static_cast<size_t>((f + 63) / 64 * 64); };
        const size_t xf = al(t * in), bf = bias ? al(out) : 0, yf = al(t * out);
        if (int rc = ensure_io(ctx, xf + bf + yf); rc != RT_OK) return rc;
        float* dxw = ctx->io;
        float* dbw = ctx->io + xf;
        dy = ctx->io + xf + bf;
        RT_CHECK_CUDA(ctx, cudaMemcpyAsync(dxw, x, sizeof(float) * t * in, cudaMemcpyHostToDevice, ctx->stream));
        if (bias) RT_CHECK_CUDA(ctx, cudaMemcpyAsync(dbw, bias, sizeof(float) * out, cudaMemcpyHostToDevice, ctx->stream));
        dx = dxw;
        db = bias ? dbw : nullptr;
    } else if ((reinterpret_cast<uintptr_t>(x) & 15) || (reinterpret_cast<uintptr_t>(y) & 15)) {
        return fail(ctx, RT_E_INVAL, "rt_qlinear_forward: device x and y must be 16-byte aligned");
    }
    // One row: the GEMV (x split into three int8 planes, f32-level accuracy);
    // more: the tensor-core GEMM over fp16 operands.
    int rc = t == 1 ? gemv_common(ctx, w, dx, dy, RT_DEVICE, w->fmt == RT_FMT_Q4K ? rt::kQ4K : rt::kBF16)
                    : gemm_common(ctx, w, dx, t, dy, RT_DEVICE, w->fmt, true);
    if (rc != RT_OK) return rc;
    if (db) RT_CHECK_CUDA(ctx, rt::bias_rows_launch(dy, t, out, db, ctx->num_sms, ctx->stream));
    if (flags == RT_HOST) {
        RT_CHECK_CUDA(ctx, cudaMemcpyAsync(y, dy, sizeof(float) * t * out, cudaMemcpyDeviceToHost, ctx->stream));
        return rt_sync(ctx);
    }
    return RT_OK;
}

int rt_gemm_plan(int64_t m, int64_t n, int32_t k, int32_t num_sms, int32_t bf16_weights, int32_t* out) {
    if (!out) return RT_E_INVAL;
    const rt::GemmPlan p = rt::gemm_q4k_plan(m, n, k, num_sms, bf16_weights != 0, true);
    if (p.bm == 0) return RT_E_SHAPE;
    out[0] = p.bm;
    out[1] = p.splits;
    out[2] = p.arows;
    out[3] = p.kps;
    return RT_OK;
}

int rt_gemv_bench(rt_ctx* ctx, int fmt, const rt_w* const* ws, int nw, const float* x, float* y, int launches,
                  int ctas_per_sm, int reps, float* us_per_gemv) {
    if (!ctx || !ws || nw < 1 || !x || !y || !us_per_gemv) return fail(ctx, RT_E_INVAL, "rt_gemv_bench: null argument");
    if (fmt != RT_FMT_Q4K && fmt != RT_FMT_BF16) return fail(ctx, RT_E_FORMAT, "rt_gemv_bench: fmt %d", fmt);
    if (launches < 1 || launches > 4096 || reps < 1 || (ctas_per_sm != 1 && ctas_per_sm != 2))
        return fail(ctx, RT_E_INVAL, "rt_gemv_bench: launches 1..4096, reps >= 1, ctas_per_sm 1 or 2");
    if ((reinterpret_cast<uintptr_t>(x) & 15) || (reinterpret_cast<uintptr_t>(y) & 15))
        return fail(ctx, RT_E_INVAL, "rt_gemv_bench: x and y must be 16-byte aligned device pointers");
    for (int i = 0; i < nw; ++i)
        if (!ws[i] || ws[i]->fmt != fmt || ws[i]->rows != ws[0]->rows || ws[i]->cols != ws[0]->cols)
            return fail(ctx, RT_E_SHAPE, "rt_gemv_bench: weight %d differs in format or shape", i);
    const int kind = fmt == RT_FMT_Q4K ? rt::kQ4K : rt::kBF16;
    const int64_t rows = ws[0]->rows;
    const int K = static_cast<int>(ws[0]->cols);
    RT_CHECK_CUDA(ctx, cudaSetDevice(ctx->device));
    // Q4_K with ctas_per_sm 1: the cluster kernel of rt_gemv_q4k; otherwise the
    // generic kernel at the requested CTAs per SM (kept for comparison)
    const bool cluster = kind == rt::kQ4K && ctas_per_sm == 1;
    const rt::GemvPlan p = cluster ? rt::gemv_cluster_plan(rows, K, ctx->num_sms)
                                   : rt::gemv_plan(kind, rows, K, 1, rt::kProPlain, rt::kEpiPlain, ctx->num_sms, ctas_per_sm);
    if (p.warps == 0) return fail(ctx, RT_E_SHAPE, "rt_gemv_bench: no launch geometry for cols %d", K);
    std::vector<CUtensorMap> tm(nw);
    for (int i = 0; i < nw; ++i)
        if (!rt::gemv_make_tmap(kind, ws[i]->d, rows, K, p, &tm[i]))
            return fail(ctx, RT_E_CUDA, "rt_gemv_bench: TMA descriptor rejected");
    if (int rc = ensure_gemv_scratch(ctx, p); rc != RT_OK) return rc;
    RT_CHECK_CUDA(ctx, cudaStreamSynchronize(ctx->stream));
    cudaGraph_t graph = nullptr;
    cudaGraphExec_t exec = nullptr;
    cudaEvent_t e0 = nullptr, e1 = nullptr;
    cudaError_t e = cudaStreamBeginCapture(ctx->stream, cudaStreamCaptureModeThreadLocal);
    for (int i = 0; e == cudaSuccess && i < launches; ++i) {
        rt::GemvArgs a = {};
        a.w = static_cast<const uint8_t*>(ws[i % nw]->d);
        a.rows = rows;
        a.K = K;
        a.x = x;
        a.y = y;
        a.part = ctx->gemv_part;
        a.tile_cnt = ctx->gemv_cnt;
        a.err = ctx->d_err;
        e = cluster ? rt::gemv_cluster_launch(a, tm[i % nw], p, ctx->stream, i > 0)
                    : rt::gemv_launch(kind, rt::kProPlain, rt::kEpiPlain, a, tm[i % nw], p, ctx->stream, i > 0);
    }
    const cudaError_t ec = cudaStreamEndCapture(ctx->stream, &graph);
    if (e == cudaSuccess) e = ec;
    if (e == cudaSuccess) e = cudaGraphInstantiate(&exec, graph, 0);
    if (e == cudaSuccess) e = cudaEventCreate(&e0);
    if (e == cudaSuccess) e = cudaEventCreate(&e1);
    if (e == cudaSuccess) e = cudaGraphLaunch(exec, ctx->stream);  // warm-up
    if (e == cudaSuccess) e = cudaEventRecord(e0, ctx->stream);
    for (int r = 0; e == cudaSuccess && r < reps; ++r) e = cudaGraphLaunch(exec, ctx->stream);
    if (e == cudaSuccess) e = cudaEventRecord(e1, ctx->stream);
    if (e == cudaSuccess) e = cudaEventSynchronize(e1);
    float ms = 0.f;
    if (e == cudaSuccess) e = cudaEventElapsedTime(&ms, e0, e1);
    if (exec) cudaGraphExecDestroy(exec);
    if (graph) cudaGraphDestroy(graph);
    if (e0) cudaEventDestroy(e0);
    if (e1) cudaEventDestroy(e1);
    RT_CHECK_CUDA(ctx, e);
    *us_per_gemv = ms * 1000.f / static_cast<float>(reps * launches);
    return rt_sync(ctx);
}

int rt_convert_q4_0_to_q4k(rt_ctx* ctx, const void* q4_0, int64_t rows, int64_t cols, int flags, rt_w** out) {
    if (!ctx || !q4_0 || !out) return fail(ctx, RT_E_INVAL, "rt_convert_q4_0_to_q4k: null argument");
    *out = nullptr;
    if (flags != RT_HOST && flags != RT_DEVICE) return fail(ctx, RT_E_INVAL, "rt_convert_q4_0_to_q4k: bad flags");
    if (rows <= 0 || cols <= 0 || cols % 256)
        return fail(ctx, RT_E_SHAPE, "rt_convert_q4_0_to_q4k: cols must be a positive multiple of 256");
    RT_CHECK_CUDA(ctx, cudaSetDevice(ctx->device));
    const uint64_t in_bytes = rt::weight_bytes(RT_FMT_Q4_0, rows, cols);
    const uint64_t out_bytes = rt::weight_bytes(RT_FMT_Q4K, rows, cols);
    const uint8_t* src = static_cast<const uint8_t*>(q4_0);
    void* staged = nullptr;
    if (flags == RT_HOST) {
        int rc = rt::dev_alloc(ctx, &staged, in_bytes, "q4_0 staging");
        if (rc != RT_OK) return rc;
        cudaError_t e = cudaMemcpyAsync(staged, q4_0, in_bytes, cudaMemcpyHostToDevice, ctx->stream);
        if (e != cudaSuccess) {
            cudaFree(staged);
            return fail(ctx, RT_E_CUDA, "rt_convert_q4_0_to_q4k: %s", cudaGetErrorString(e));
        }
        src = static_cast<const uint8_t*>(staged);
    }
    rt_w* w = new rt_w();
    w->fmt = RT_FMT_Q4K;
    w->rows = rows;
    w->cols = cols;
    w->bytes = out_bytes;
    int rc = rt::dev_alloc(ctx, &w->d, out_bytes, "q4_k weight");
    if (rc == RT_OK) {
        cudaError_t e = rt::q4_0_to_q4k_launch(src, rows * (cols / 256), static_cast<uint8_t*>(w->d), ctx->stream);
        if (e == cudaSuccess) e = cudaStreamSynchronize(ctx->stream);
        if (e != cudaSuccess) rc = fail(ctx, RT_E_CUDA, "rt_convert_q4_0_to_q4k: %s", cudaGetErrorString(e));
    }
    cudaFree(staged);
    if (rc != RT_OK) {
        cudaFree(w->d);
        delete w;
        return rc;
    }
    *out = w;
    return RT_OK;
}

int rt_convert_q6k_to_bf16(rt_ctx* ctx, const void* q6k, int64_t rows, int64_t cols, int flags, rt_w** out) {
    if (!ctx || !q6k || !out) return fail(ctx, RT_E_INVAL, "rt_convert_q6k_to_bf16: null argument");
    *out = nullptr;
    if (flags != RT_HOST && flags != RT_DEVICE) return fail(ctx, RT_E_INVAL, "rt_convert_q6k_to_bf16: bad flags");
    if (rows <= 0 || cols <= 0 || cols % 256)
        return fail(ctx, RT_E_SHAPE, "rt_convert_q6k_to_bf16: cols must be a positive multiple of 256");
    RT_CHECK_CUDA(ctx, cudaSetDevice(ctx->device));
    const uint64_t in_bytes = rt::weight_bytes(RT_FMT_Q6K, rows, cols);
    const uint64_t out_bytes = rt::weight_bytes(RT_FMT_BF16, rows, cols);
    const uint8_t* src = static_cast<const uint8_t*>(q6k);
    void* staged = nullptr;
    if (flags == RT_HOST) {
        int rc = rt::dev_alloc(ctx, &staged, in_bytes, "q6_k staging");
        if (rc != RT_OK) return rc;
        cudaError_t e = cudaMemcpyAsync(staged, q6k, in_bytes, cudaMemcpyHostToDevice, ctx->stream);
        if (e != cudaSuccess) {
            cudaFree(staged);
            return fail(ctx, RT_E_CUDA, "rt_convert_q6k_to_bf16: %s", cudaGetErrorString(e));
        }
        src = static_cast<const uint8_t*>(staged);
    }
    rt_w* w = new rt_w();
    w->fmt = RT_FMT_BF16;
    w->rows = rows;
    w->cols = cols;
    w->bytes = out_bytes;
    int rc = rt::dev_alloc(ctx, &w->d, out_bytes, "bf16 weight");
    if (rc == RT_OK) {
        cudaError_t e = rt::q6k_to_bf16_launch(src, rows * cols, static_cast<uint16_t*>(w->d), ctx->stream);
        if (e == cudaSuccess) e = cudaStreamSynchronize(ctx->stream);
        if (e != cudaSuccess) rc = fail(ctx, RT_E_CUDA, "rt_convert_q6k_to_bf16: %s", cudaGetErrorString(e));
    }
    cudaFree(staged);
    if (rc != RT_OK) {
        cudaFree(w->d);
        delete w;
        return rc;
    }
    *out = w;
    return RT_OK;
}

}  // extern "C"
