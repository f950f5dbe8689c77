// rt_internal.h -- library-private definitions behind include/rt_cuda.h.
#pragma once

#include <cuda_runtime.h>
#include <stdarg.h>
#include <stdint.h>
#include <stdio.h>

#include <map>
#include <string>
#include <tuple>

#include "../../include/rt_cuda.h"
#include "gemv.cuh"

struct rt_ctx {
    int device = 0;
    int num_sms = 0;
    cudaStream_t stream = nullptr;
    std::string err;
    // Scratch for the host-pointer GEMV entry points (x in, y out).
    float* scratch = nullptr;
    size_t scratch_floats = 0;
    int* d_err = nullptr;  // device error word written by kernels
    // Split-tile scratch of the standalone GEMVs (counters zeroed on allocation;
    // every completed launch leaves them at zero).
    float* gemv_part = nullptr;
    uint32_t* gemv_cnt = nullptr;
    int64_t gemv_part_floats = 0, gemv_cnt_words = 0;
    // Device copies of host-pointer inputs and outputs of rt_qlinear_forward
    // (kept apart from `scratch`, which the GEMV and GEMM use for their own
    // intermediates).
    float* io = nullptr;
    size_t io_floats = 0;
};

struct rt_w {
    int fmt = 0;
    int64_t rows = 0, cols = 0;
    uint64_t bytes = 0;
    void* d = nullptr;
    // Launch plan and TMA descriptor of the standalone GEMV, made on first use.
    bool gemv_ready = false;
    rt::GemvPlan plan;
    CUtensorMap tmap;
};

namespace rt {

// Record an error message on ctx (if any) and return `code`.
int fail(rt_ctx* ctx, int code, const char* fmt, ...);

// Device allocation through one place, so tests can inject an allocation
// failure from the host: RT_FAULT_INJECT_ALLOC=N makes the N-th allocation
// (1-based, counted per process) fail with RT_E_NOMEM.
int dev_alloc(rt_ctx* ctx, void** p, size_t bytes, const char* what);

// Q4_K / BF16 storage size of a [rows, cols] matrix, 0 if the shape is invalid.
uint64_t weight_bytes(int fmt, int64_t rows, int64_t cols);

// Host-side helpers of the synthetic generator that other files reuse.
void rope_table(float theta, float freq_scale, int head_dim, int cap, float* cos_out, float* sin_out);

}  // namespace rt

#define RT_CHECK_CUDA(ctx, call)                                                                    \
    do {                                                                                            \
        cudaError_t e_ = (call);                                                                    \
        if (e_ != cudaSuccess) return rt::fail((ctx), RT_E_CUDA, "%s: %s", #call, cudaGetErrorString(e_)); \
    } while (0)
