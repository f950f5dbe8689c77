// gemv.cuh -- weight-streaming GEMV for Q4_K and BF16 matrices on the sm_100a
// tensor cores (mma.sync).
//
// y[r] = sum_k W[r, k] * x[k] for a [rows, K] row-major matrix whose rows are
// contiguous in HBM.  One kernel serves the standalone GEMV entry points
// (rt_gemv_q4k / rt_gemv_bf16) and every projection of the fused decode step,
// where a prologue builds x (RMSNorm of the residual stream, embedding lookup)
// and an epilogue fuses the GELU gate or the greedy argmax.
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
    kEpiArgmax = 2,    // y[r] = sum, plus the greedy token (GreedySlot)
};

// Per-CTA state of the greedy epilogue, combined by the last CTA to finish.
// sample_token at temperature 0 (src/transformer4.rs:3036-3091) takes the
// LAST index of the largest softmax probability p_i = exp(y_i - M) / S:
//   m   the CTA's largest y (M is the maximum over the CTAs' m);
//   s   sum over the CTA's rows of exp(y - m) (so S = sum_c s_c exp(m_c - M));
//   idx the CTA's row of m (ties to the higher row);
//   lo, hi  the lowest and highest row the CTA emitted: the rows the last CTA
//       re-reads for near-ties when m is within kGreedyTau of M;
//   failed  a bounded wait of the CTA gave up: the launch has no token, and
//       the last CTA returns the launch's counters to zero.
struct GreedySlot {
    float m;
    float s;
    int32_t idx;
    int32_t lo;
    int32_t hi;
    int32_t failed;
    int32_t pad[2];
};

struct GemvArgs {
    const uint8_t* w;  // weight rows, 16-byte aligned
    int64_t rows;      // rows of W
    int32_t K;         // columns
    // geometry (filled by gemv_launch from the plan)
    int32_t nseg;        // column segments per row (256 Q4_K / 128 BF16 columns each)
    int32_t nb;          // copies in flight per warp
    int32_t unit_bytes;  // shared-memory bytes of one unit (16 rows x one segment, padded)
    // split-tile scratch: tiles shared by several warps are summed here
    float* part;        // [gridDim.x * warps * 2 * 16] partial row sums
    uint32_t* tile_cnt; // [ceil(rows / 16)] units arrived per split tile; zero before, zero after
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
    GreedySlot* am_slot;   // [gridDim.x] per-CTA greedy state
    uint32_t* am_counter;  // zero before the launch; the last CTA resets it
    int32_t* token_out;    // greedy token written by the last CTA
    int32_t* pos_inout;    // incremented by the last CTA (device-side decode loop)
    int32_t* token_hist;   // token_hist[pos] = greedy token of the step at pos (may be null)
    int* err;              // error word (kErr*), may be null
    int32_t fail_token;    // 1: a launch whose bounded wait gave up writes token_out = -1
    uint32_t wait_iters;   // poll limit of the weight-stream waits (0: the default bound)
};

struct GemvPlan {
    int warps = 0;       // warps per CTA (0: shape not supported)
    int nb = 0;          // copies in flight per warp
    int unit_bytes = 0;  // shared-memory bytes of one unit
    int box_x = 0;       // TMA box inner extent, 8-byte elements
    int grid = 0;
    size_t smem = 0;
    int64_t part_floats = 0;  // split-tile scratch this plan needs (GemvArgs::part)
    int64_t cnt_words = 0;    // and GemvArgs::tile_cnt, zeroed once by the owner
};

// cuTensorMapEncodeTiled, fetched from the driver once per process (thread-safe);
// null if the driver does not provide it.
using TmapEncodeFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                  const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                  CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);
TmapEncodeFn tmap_encoder();

// Raise the dynamic shared-memory limit of every kernel instantiation on the
// current device.  Call once per device before planning or capturing.
void gemv_prepare();

// Choose warps / ring depth / grid for a [rows, K] GEMV: one CTA per SM.
// ctas_per_sm is 1 (the CTA takes the whole SM) or 2 (a half-size CTA, so a
// CTA of the next kernel in a PDL chain can be resident beside it).
GemvPlan gemv_plan(int kind, int64_t rows, int K, int pair, int prologue, int epilogue, int num_sms,
                   int ctas_per_sm);

// TMA descriptor of a [rows, K] weight matrix at `w` for plan `p`: 8-byte
// elements, box = one unit (box_x elements x 16 rows; bytes past the row end
// and rows past the matrix read as zero).  Returns false if the driver refuses.
bool gemv_make_tmap(int kind, const void* w, int64_t rows, int K, const GemvPlan& p, CUtensorMap* out);

// Fill the geometry fields of `a` from `p` and launch.  `pdl` attaches the
// programmatic-stream-serialization attribute (used inside the decode graph).
cudaError_t gemv_launch(int kind, int prologue, int epilogue, GemvArgs a, const CUtensorMap& tmap, const GemvPlan& p,
                        cudaStream_t stream, bool pdl);

// The Q4_K GEMV of the standalone entry points (gemv_cluster.cu): plain x,
// plain y, row-major weights; four-CTA clusters, two CTAs per SM where the
// shared memory allows.  The plan's tensor map is gemv_make_tmap's (box_x, 16).
GemvPlan gemv_cluster_plan(int64_t rows, int K, int num_sms);
cudaError_t gemv_cluster_prepare();
cudaError_t gemv_cluster_launch(GemvArgs a, const CUtensorMap& tmap, const GemvPlan& p, cudaStream_t stream, bool pdl);

// Algorithmic bytes of one launch: weights + x + y (+ prologue vectors).
uint64_t gemv_algorithmic_bytes(int kind, int64_t rows, int K, int prologue, int epilogue);

}  // namespace rt
