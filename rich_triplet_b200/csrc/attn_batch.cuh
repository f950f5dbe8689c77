// attn_batch.cuh -- decode attention over many rows at once: each row is one
// query token with its own position, reading either its own KV cache (many
// sequences, one token each) or one cache that all rows share (the prompt
// tokens of one sequence, causal).
//
// Two kernels per layer:
//   prep   per row: the per-head q/k RMSNorm and NeoX RoPE of the raw
//          projections (apply_per_head_norm, src/transformer4.rs:2485-2510;
//          apply_rope_at_offset, :2742-2772); the row's K and V are appended
//          to its cache at its position (Gemma3LayerKvCache::append,
//          :1813-1823) and its rotated queries stored.
//   chunk  attention of every (row, KV head) over its attended positions
//          [max(0, pos + 1 - window), pos] (gqa_attention_cached with
//          t_q == 1, src/transformer4.rs:2806-2880), split into chunks of
//          kAttnChunk positions, each with an online softmax; a merge kernel
//          combines the chunks of rows that span several.
#pragma once

#include <stddef.h>
#include <stdint.h>

#include <cuda_runtime.h>

namespace rt {

constexpr int kAttnChunk = 256;  // cached positions per work item

struct AttnRowsArgs {
    const float* qkv;                 // [B][qkv_stride]: row b's [nq*D | nkv*D | nkv*D] raw projections
    int64_t qkv_stride;
    int parts;                        // split-K parts at qkv + q * part_stride, added in part order (<= 1: one)
    int64_t part_stride;
    const float* q_norm;              // [D] gamma of the per-head q norm
    const float* k_norm;              // [D]
    const float* rope_cos;            // [cap][D/2] for this layer's theta / scale
    const float* rope_sin;
    const int32_t* pos;               // [B] position of each row
    float* kcache;                    // row 0's K cache of this layer, [nkv][cap][D]
    float* vcache;
    int64_t seq_kv;                   // floats between consecutive rows' caches (0: one shared cache)
    int cap, nq, nkv, D;
    float eps;
    float* q_out;                     // [B][nq][D] rotated queries
};

struct AttnChunkArgs {
    const float* q;                   // [B][nq][D] from the prep kernel
    const float* kcache;              // row 0's caches, [nkv][cap][D]
    const float* vcache;
    int64_t seq_kv;                   // as AttnRowsArgs
    const int32_t* pos;               // [B]
    int B, nq, nkv, D, cap;
    int window;                       // sliding window (0: every position up to pos)
    int nchunk;                       // attn_chunk_count(cap, window)
    float scale;                      // 1 / sqrt(query_pre_attn_scalar)
    float* part;                      // attn_chunk_part_floats(...) floats of per-chunk states
    float* out;                       // [B][nq][D]
    int* err;                         // error word (kErrMbarTimeout on a wait that gave up)
};

// Chunks per (row, KV head) at most: ceil(min(cap, window) / kAttnChunk).
int attn_chunk_count(int cap, int window);
size_t attn_chunk_part_floats(int B, int nkv, int nchunk, int G, int D);
// True if the chunk kernel handles head_dim D with G query heads per KV head.
bool attn_chunk_supported(int D, int G);
cudaError_t attn_chunk_prepare();  // shared-memory limits, once per device, outside capture
cudaError_t attn_rows_prep_launch(const AttnRowsArgs& a, int B, cudaStream_t s);
// The chunk kernel, then (nchunk > 1) the merge kernel.
cudaError_t attn_chunk_launch(const AttnChunkArgs& a, int num_sms, cudaStream_t s);

}  // namespace rt
