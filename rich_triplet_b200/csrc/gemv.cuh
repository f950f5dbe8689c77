// gemv.cuh -- row-streaming GEMV for Q4_K and BF16 weight matrices on the
// tensor cores (mma.sync), for sm_100a.
//
// y[r] = sum_k W[r, k] * x[k] for a [rows, K] row-major matrix whose rows are
// contiguous in HBM.  One kernel serves the standalone GEMV entry points
// (rt_gemv_q4k / rt_gemv_bf16) and every projection of the fused decode step,
// where a prologue builds x in shared memory (RMSNorm of the residual stream,
// embedding lookup) and an epilogue fuses the GELU gate or the greedy argmax.
#pragma once

#include <stdint.h>

#include <cuda.h>  // CUtensorMap (the encoder is fetched from the driver at run time)
#include <cuda_runtime.h>

namespace rt {

enum WeightKind : int { kQ4K = 0, kBF16 = 1 };

// How the kernel obtains its input vector x.
enum Prologue : int {
    kProPlain = 0,      // x read from global memory (written by the previous kernel)
    kProResidNorm = 1,  // resid_out = resid_in + rmsnorm(src)*(1+g_post);  x = rmsnorm(resid_out)*(1+g_pre)
    kProEmbedNorm = 2,  // resid_out = bf16(embed[token]) * embed_scale;    x = rmsnorm(resid_out)*(1+g_pre)
};

// What the kernel does with the row sums.
enum Epilogue : int {
    kEpiPlain = 0,     // y[r] = sum
    kEpiGeluPair = 1,  // rows interleaved (gate, up): y[r/2] = gelu_tanh(gate) * up
    kEpiArgmax = 2,    // y[r] = sum, plus the greedy token (max, ties to higher index)
};

struct GemvArgs {
    const uint8_t* w;   // weight rows, row_bytes each, 16-byte aligned
    int64_t rows;       // rows of W computed by this launch
    int32_t K;          // columns
    int32_t nseg;       // ceil(K / 256): 256-column segments per row
    int32_t seg_bytes;  // 144 (Q4_K block) or 512 (BF16)
    int32_t row_bytes;  // bytes of one row
    // geometry chosen by gemv_plan()
    int32_t spst;         // 256-column segments per stage (a stage is 16 rows x spst segments)
    int32_t srow;         // shared-memory row stride of a stage, = 64 mod 128 bytes
    int32_t nbuf;         // shared-memory stage buffers
    int32_t stage_bytes;  // bytes of one stage buffer (16 * srow)
    int32_t pair;         // 2 for kEpiGeluPair (row ranges start on even rows)
    int32_t x_smem;       // plain prologue: 1 = copy x into shared memory first, 0 = read it in place
    // prologue inputs
    const float* x;
    const float* src;
    const float* resid_in;
    float* resid_out;
    const float* g_post;
    const float* g_pre;
    const uint16_t* embed;
    const int32_t* token;
    float embed_scale;
    float eps;
    // outputs
    float* y;
    float* am_val;         // [gridDim.x] per-CTA best logit
    int32_t* am_idx;       // [gridDim.x] per-CTA best index
    uint32_t* am_counter;  // zero before the launch; the last CTA resets it
    int32_t* token_out;    // greedy token written by the last CTA
    int32_t* pos_inout;    // incremented by the last CTA (device-side decode loop)
    int32_t* token_hist;   // token_hist[pos] = greedy token of the step at pos (may be null)
    int* err;              // error word (kErr*), may be null
};

struct GemvPlan {
    int warps = 0;
    int spst = 0;
    int srow = 0;
    int nbuf = 0;
    int stage_bytes = 0;
    int x_smem = 1;
    int grid = 0;
    size_t smem = 0;
};

// Raise the dynamic shared-memory limit of every kernel instantiation on the
// current device.  Call once per device before planning or capturing.
void gemv_prepare();

// Choose warps / stage geometry / grid for a [rows, K] GEMV.
GemvPlan gemv_plan(int kind, int64_t rows, int K, int pair, int prologue, int epilogue, int num_sms,
                   int max_ctas_per_sm);

// TMA descriptor of a [rows, K] weight matrix at `w` for plan `p`: 8-byte
// elements, box = one stage (16 rows x srow bytes; bytes past the row end and
// rows past the matrix read as zero).  Returns false if the driver refuses.
bool gemv_make_tmap(int kind, const void* w, int64_t rows, int K, const GemvPlan& p, CUtensorMap* out);

// Fill the geometry fields of `a` from `p` and launch.  `pdl` attaches the
// programmatic-stream-serialization attribute (used inside the decode graph).
cudaError_t gemv_launch(int kind, int prologue, int epilogue, GemvArgs a, const CUtensorMap& tmap, const GemvPlan& p,
                        cudaStream_t stream, bool pdl);

// Algorithmic bytes of one launch: weights + x + y (+ prologue vectors).
uint64_t gemv_algorithmic_bytes(int kind, int64_t rows, int K, int prologue, int epilogue);

}  // namespace rt
