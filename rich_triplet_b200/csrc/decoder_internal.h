// decoder_internal.h -- the single-sequence decode engine's state
// (decoder.cu), shared with the many-sequence engine (batch.cu), which runs on
// the same fused weights, norms and RoPE conventions.
#pragma once

#include <stdint.h>

#include <vector>

#include <cuda.h>
#include <cuda_runtime.h>

#include "gemv.cuh"
#include "rt_internal.h"
#include "step.cuh"

// Column parts of the step kernel's down projection (a divisor of FFN / 256).
constexpr int kMaxDownParts = rt::gcore::kMaxSrcParts;

struct rt_dec {
    rt_ctx* ctx = nullptr;
    rt_gemma3_cfg cfg{};
    int H = 0, D = 0, NQ = 0, NKV = 0, F = 0, V = 0, NL = 0, cap = 0;
    int qkv_rows = 0;
    // weights (device)
    std::vector<uint8_t*> w_qkv, w_o, w_gu, w_down;
    uint16_t* embed = nullptr;
    float* norms = nullptr;     // [NL][4][H]: attn, post_attn, pre_ffn, post_ffn
    float* qk_norms = nullptr;  // [NL][2][D]
    float* final_norm = nullptr;
    float* kcache = nullptr;  // [NL][NKV][cap][D]
    float* vcache = nullptr;
    float* rope = nullptr;  // [2 (local, global)][2 (cos, sin)][cap][D/2]
    // activations
    float* act = nullptr;  // one allocation, sliced below
    float *resid[2] = {nullptr, nullptr}, *qkv = nullptr, *attn = nullptr, *o_out = nullptr, *hbuf = nullptr,
          *down = nullptr, *logits = nullptr, *attn_part = nullptr;
    rt::GreedySlot* am_slot = nullptr;
    // The step kernel's vectors as tagged words (value + phase tag, 8 bytes each):
    // q/k/v, attention output, O, gated FFN hidden, down projection parts.
    uint64_t* ll = nullptr;
    uint64_t *qkv_ll = nullptr, *attn_ll = nullptr, *o_ll = nullptr, *h_ll = nullptr, *down_ll = nullptr,
             *part_ll = nullptr;
    size_t ll_words = 0;
    uint32_t* counters = nullptr;  // [NKV] attention + [1] argmax
    float* g_part = nullptr;       // GEMV split-tile partials (shared by the step's GEMVs, which run in order)
    uint32_t* g_cnt = nullptr;     // GEMV split-tile counters, zero between launches
    int64_t g_cnt_words = 0;
    int32_t* ctl = nullptr;        // [0] token, [1] position, [2..] token history [cap]
    int* h_err = nullptr;          // pinned copy of the context's error word
    // launch geometry
    rt::GemvPlan p_qkv, p_o, p_gu, p_down, p_lm;
    std::vector<CUtensorMap> t_qkv, t_o, t_gu, t_down;  // TMA descriptors of the weights
    CUtensorMap t_lm;
    int nsplit = 0;
    int down_parts = 1;  // column parts of the step kernel's down projection (partials in `down`)
    int final_resid = 0;
    int launches = 0;
    cudaGraph_t graph = nullptr;
    cudaGraphExec_t exec = nullptr;
    // The persistent step kernel (one cooperative launch per step), when the
    // shapes fit it; otherwise the captured graph of per-projection kernels.
    bool use_step = false;
    bool single = false;  // the single-sequence path (GEMV plans, step kernel or graph) exists
    int step_grid = 0;
    rt::StepGeom step_geom;
    rt::StepParams step_params{};
    uint64_t dev_bytes = 0;
    // Positions of this sequence several at a time (prefill, batched verify):
    // the many-sequence engine in rows mode on these caches, made at first use.
    rt_batch* rows = nullptr;
    std::vector<void*> allocs;
};

namespace rt {

// Config4::is_global_layer (src/transformer4.rs:141-143): every sixth layer.
inline bool is_global(int layer) { return layer % 6 == 5; }

// Norm weight `which` (0 attn, 1 post-attn, 2 pre-FFN, 3 post-FFN) of `layer`.
inline float* norm_ptr(rt_dec* d, int layer, int which) {
    return d->norms + (static_cast<size_t>(layer) * 4 + which) * d->H;
}

}  // namespace rt

namespace rt {
// Frees the rows engine of a decoder (batch.cu).
void rows_engine_free(rt_batch* t);
}  // namespace rt
