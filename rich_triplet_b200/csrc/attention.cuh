// attention.cuh -- single-token GQA attention for the Gemma 3 decode step.
#pragma once

#include <stdint.h>

#include <cuda_runtime.h>

#include "gemv.cuh"

namespace rt {

// 16-byte aligned (and so a multiple of 16 bytes): the decode-step kernel
// brings a layer's entry into shared memory with one bulk copy.
struct alignas(16) AttnArgs {
    const float* qkv;       // raw projections of this token: [nq*D | nkv*D | nkv*D]
    const float* q_norm;    // [D]  gamma of the per-head q norm
    const float* k_norm;    // [D]
    float* kcache;          // this layer's K cache, [nkv][cap][D] f32
    float* vcache;          // this layer's V cache
    const float* rope_cos;  // [cap][D/2] cos for this layer's theta / scale
    const float* rope_sin;  // [cap][D/2]
    const int32_t* pos;     // absolute position of the token (device scalar)
    int32_t cap;            // cache positions
    int32_t nq, nkv, D;
    int32_t window;         // sliding window (0 = attend to every cached position)
    int32_t nsplit;         // context splits per KV head (gridDim.x)
    float scale;            // 1 / sqrt(query_pre_attn_scalar)
    float eps;              // RMSNorm epsilon
    float* part;            // [nkv][nsplit][G][attn_part_stride(D)] per-split (unnormalised out, m, l)
    uint32_t* counter;      // [nkv], zero before the launch; the combining CTA resets it
    float* out;             // [nq*D]
    int* err;
    // Tagged-word form (decode-step kernel): q/k/v read from qkv_ll, the merged
    // output written to out_ll, when the caller passes nonzero tags.
    const uint64_t* qkv_ll = nullptr;
    uint64_t* out_ll = nullptr;
    uint64_t* part_ll = nullptr;  // the per-split partials as tagged words (layout of `part`)
    // Several sequences in one launch (grid z = sequence b): b's qkv, caches,
    // partials and output sit these many floats after sequence 0's, its
    // position at pos[b] and its counters at counter[b * nkv].  Unused with one.
    int64_t seq_qkv = 0, seq_kv = 0, seq_part = 0, seq_out = 0;
};

constexpr int kAttnTile = 32;     // cached positions per shared-memory tile
constexpr int kAttnThreads = 256;

// Floats per (split, query head) row of the attention partials: D outputs,
// then m and l; padded to a multiple of 4 so every row starts 16-byte aligned.
__host__ __device__ constexpr int attn_part_stride(int D) { return D + 4; }

size_t attention_smem_bytes(int D, int G);
// Set kernel attributes; call once per device before the first launch / capture.
cudaError_t attention_prepare();
cudaError_t attention_launch(const AttnArgs& a, cudaStream_t s, bool pdl);
// The same for `nseq` sequences (AttnArgs::seq_* strides), one grid plane each.
cudaError_t attention_launch_batch(const AttnArgs& a, int nseq, cudaStream_t s);
// Algorithmic bytes at context length L (positions attended) for one layer.
uint64_t attention_algorithmic_bytes(int nq, int nkv, int D, int64_t L);

}  // namespace rt
