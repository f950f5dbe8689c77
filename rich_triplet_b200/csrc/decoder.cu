// decoder.cu -- Gemma 3 decode engine: one token = one CUDA graph launch.
//
// Replaces MetalDecodeContext (src/metal_decode.rs:971-2074, paths relative
// to the reference crate root), which encodes ~717 dispatches per token into
// one Metal command buffer.  Here one step is 5 kernels per layer plus the LM
// head, captured once into a CUDA graph whose kernels are chained with
// programmatic dependent launch, so each kernel's weight stream starts while
// its predecessor drains:
//
//   per layer l:
//     1. QKV GEMV    prologue: (l == 0) embedding * sqrt(H)  |  (l > 0) residual +=
//                    post-FFN-norm(down_{l-1});  then input RMSNorm.
//                    Rows of q, k, v are concatenated into one Q4_K matrix.
//     2. attention   per-head q/k RMSNorm + RoPE + KV append + split-context
//                    flash-decode + merge (attention.cu)
//     3. o GEMV
//     4. gate/up GEMV prologue: residual += post-attn-norm(o); pre-FFN RMSNorm.
//                    Rows of gate and up interleaved; epilogue gelu_tanh(g) * u.
//     5. down GEMV
//   LM head: prologue residual += post-FFN-norm(down_last); final RMSNorm;
//            BF16 GEMV over the tied embedding; epilogue greedy argmax.
//
// The residual stream lives in two ping-pong buffers: in a fused prologue
// every CTA reads the current one and CTA 0 writes the next, so no CTA can
// overwrite a value another CTA has yet to read.
//
// Device layout (all f32 unless stated): KV cache [layer][kv_head][cap][D];
// RoPE tables [cap][D/2] for local and global layers; activations sized for
// one token.  The token id and position live in device memory, so the same
// graph serves every step; rt_decoder_step writes them before each launch.
#include <math.h>
#include <stdlib.h>
#include <string.h>

#include <algorithm>
#include <vector>

#include "attention.cuh"
#include "convert.cuh"
#include "decoder_internal.h"
#include "gemv.cuh"
#include "rt_internal.h"
#include "step.cuh"

using rt::fail;
using rt::is_global;
using rt::norm_ptr;

namespace {

// Writes the step's token and position into device memory.  They travel as
// kernel arguments, so back-to-back asynchronous calls never share a host
// staging buffer.
__global__ void set_ctl_kernel(int32_t* ctl, int32_t token, int32_t pos) {
    ctl[0] = token;
    ctl[1] = pos;
}

cudaError_t set_ctl(rt_dec* d, int32_t token, int32_t pos);

int dalloc(rt_dec* d, void** p, size_t bytes, const char* what) {
    int rc = rt::dev_alloc(d->ctx, p, bytes, what);
    if (rc == RT_OK) {
        d->allocs.push_back(*p);
        d->dev_bytes += bytes;
    }
    return rc;
}

float* kc_layer(rt_dec* d, int layer) { return d->kcache + static_cast<size_t>(layer) * d->NKV * d->cap * d->D; }
float* vc_layer(rt_dec* d, int layer) { return d->vcache + static_cast<size_t>(layer) * d->NKV * d->cap * d->D; }

// Enqueue one decode step.  q4k_only: just the Q4_K GEMV launches (timing).
cudaError_t enqueue_step(rt_dec* d, cudaStream_t s, bool pdl, bool q4k_only, int32_t* n_launches, uint64_t* bytes) {
    const int H = d->H, D = d->D;
    int p = 0;  // index of the current residual buffer
    int n = 0;
    uint64_t b = 0;
    cudaError_t e = cudaSuccess;
    const float eps = d->cfg.rms_norm_eps;
    for (int l = 0; l < d->NL; ++l) {
        // 1. QKV
        {
            rt::GemvArgs a = {};
            a.part = d->g_part;
            a.tile_cnt = d->g_cnt;
            a.w = d->w_qkv[l];
            a.rows = d->qkv_rows;
            a.K = H;
            a.eps = eps;
            a.y = d->qkv;
            a.err = d->ctx->d_err;
            a.g_pre = norm_ptr(d, l, 0);
            int pro;
            if (l == 0) {
                pro = rt::kProEmbedNorm;
                a.embed = d->embed;
                a.token = d->ctl;
                a.embed_scale = sqrtf(static_cast<float>(H));
                a.resid_out = d->resid[0];
                p = 0;
            } else {
                pro = rt::kProResidNorm;
                a.src = d->down;
                a.resid_in = d->resid[p];
                a.resid_out = d->resid[1 - p];
                a.g_post = norm_ptr(d, l - 1, 3);
                p = 1 - p;
            }
            e = rt::gemv_launch(rt::kQ4K, pro, rt::kEpiPlain, a, d->t_qkv[l], d->p_qkv, s, pdl);
            if (e != cudaSuccess) return e;
            ++n;
            b += rt::gemv_algorithmic_bytes(rt::kQ4K, d->qkv_rows, H, pro, rt::kEpiPlain);
        }
        // 2. attention
        if (!q4k_only) {
            rt::AttnArgs a = {};
            a.qkv = d->qkv;
            a.q_norm = d->qk_norms + static_cast<size_t>(l) * 2 * D;
            a.k_norm = a.q_norm + D;
            a.kcache = kc_layer(d, l);
            a.vcache = vc_layer(d, l);
            const int gsel = is_global(l) ? 1 : 0;
            const size_t tab = static_cast<size_t>(d->cap) * (D / 2);
            a.rope_cos = d->rope + (static_cast<size_t>(gsel) * 2 + 0) * tab;
            a.rope_sin = d->rope + (static_cast<size_t>(gsel) * 2 + 1) * tab;
            a.pos = d->ctl + 1;
            a.cap = d->cap;
            a.nq = d->NQ;
            a.nkv = d->NKV;
            a.D = D;
            a.window = is_global(l) ? 0 : d->cfg.sliding_window;
            a.nsplit = d->nsplit;
            a.scale = 1.0f / sqrtf(d->cfg.query_pre_attn_scalar);
            a.eps = eps;
            a.part = d->attn_part;
            a.counter = d->counters;
            a.out = d->attn;
            a.err = d->ctx->d_err;
            e = rt::attention_launch(a, s, pdl);
            if (e != cudaSuccess) return e;
            ++n;
        }
        // 3. o projection
        {
            rt::GemvArgs a = {};
            a.part = d->g_part;
            a.tile_cnt = d->g_cnt;
            a.w = d->w_o[l];
            a.rows = H;
            a.K = d->NQ * D;
            a.x = d->attn;
            a.y = d->o_out;
            a.err = d->ctx->d_err;
            e = rt::gemv_launch(rt::kQ4K, rt::kProPlain, rt::kEpiPlain, a, d->t_o[l], d->p_o, s, pdl);
            if (e != cudaSuccess) return e;
            ++n;
            b += rt::gemv_algorithmic_bytes(rt::kQ4K, H, d->NQ * D, rt::kProPlain, rt::kEpiPlain);
        }
        // 4. gate / up with GELU gate
        {
            rt::GemvArgs a = {};
            a.part = d->g_part;
            a.tile_cnt = d->g_cnt;
            a.w = d->w_gu[l];
            a.rows = 2LL * d->F;
            a.K = H;
            a.eps = eps;
            a.src = d->o_out;
            a.resid_in = d->resid[p];
            a.resid_out = d->resid[1 - p];
            a.g_post = norm_ptr(d, l, 1);
            a.g_pre = norm_ptr(d, l, 2);
            a.y = d->hbuf;
            a.err = d->ctx->d_err;
            p = 1 - p;
            e = rt::gemv_launch(rt::kQ4K, rt::kProResidNorm, rt::kEpiGeluPair, a, d->t_gu[l], d->p_gu, s, pdl);
            if (e != cudaSuccess) return e;
            ++n;
            b += rt::gemv_algorithmic_bytes(rt::kQ4K, 2LL * d->F, H, rt::kProResidNorm, rt::kEpiGeluPair);
        }
        // 5. down projection
        {
            rt::GemvArgs a = {};
            a.part = d->g_part;
            a.tile_cnt = d->g_cnt;
            a.w = d->w_down[l];
            a.rows = H;
            a.K = d->F;
            a.x = d->hbuf;
            a.y = d->down;
            a.err = d->ctx->d_err;
            e = rt::gemv_launch(rt::kQ4K, rt::kProPlain, rt::kEpiPlain, a, d->t_down[l], d->p_down, s, pdl);
            if (e != cudaSuccess) return e;
            ++n;
            b += rt::gemv_algorithmic_bytes(rt::kQ4K, H, d->F, rt::kProPlain, rt::kEpiPlain);
        }
    }
    if (!q4k_only) {
        rt::GemvArgs a = {};
        a.part = d->g_part;
        a.tile_cnt = d->g_cnt;
        a.w = reinterpret_cast<const uint8_t*>(d->embed);
        a.rows = d->V;
        a.K = H;
        a.eps = eps;
        a.src = d->down;
        a.resid_in = d->resid[p];
        a.resid_out = d->resid[1 - p];
        a.g_post = norm_ptr(d, d->NL - 1, 3);
        a.g_pre = d->final_norm;
        a.y = d->logits;
        a.am_slot = d->am_slot;
        a.am_counter = d->counters + d->NKV;
        a.token_out = d->ctl;
        a.pos_inout = d->ctl + 1;
        a.token_hist = d->ctl + 2;
        a.err = d->ctx->d_err;
        d->final_resid = 1 - p;
        e = rt::gemv_launch(rt::kBF16, rt::kProResidNorm, rt::kEpiArgmax, a, d->t_lm, d->p_lm, s, pdl);
        if (e != cudaSuccess) return e;
        ++n;
    }
    if (n_launches) *n_launches = n;
    if (bytes) *bytes = b;
    return cudaSuccess;
}

int check_layer(rt_ctx* ctx, const rt_gemma3_cfg& c, const rt_gemma3_layer& L, int i) {
    const int64_t H = c.hidden_size, D = c.head_dim, q = static_cast<int64_t>(c.num_attention_heads) * D,
                  kv = static_cast<int64_t>(c.num_key_value_heads) * D, F = c.intermediate_size;
    struct {
        const rt_w* w;
        int64_t r, k;
        const char* n;
    } ws[7] = {{L.q, q, H, "q"},        {L.k, kv, H, "k"},       {L.v, kv, H, "v"},      {L.o, H, q, "o"},
               {L.gate, F, H, "gate"}, {L.up, F, H, "up"},     {L.down, H, F, "down"}};
    for (auto& w : ws) {
        if (!w.w) return fail(ctx, RT_E_INVAL, "layer %d: %s projection missing", i, w.n);
        if (w.w->fmt != RT_FMT_Q4K)
            return fail(ctx, RT_E_FORMAT, "layer %d: %s projection has format %d; the decode engine takes Q4_K", i, w.n,
                        w.w->fmt);
        if (w.w->rows != w.r || w.w->cols != w.k)
            return fail(ctx, RT_E_SHAPE, "layer %d: %s is [%lld, %lld], expected [%lld, %lld]", i, w.n,
                        static_cast<long long>(w.w->rows), static_cast<long long>(w.w->cols),
                        static_cast<long long>(w.r), static_cast<long long>(w.k));
    }
    if (!L.attn_norm || !L.post_attn_norm || !L.pre_ffn_norm || !L.post_ffn_norm || !L.q_norm || !L.k_norm)
        return fail(ctx, RT_E_INVAL, "layer %d: norm weights missing", i);
    return RT_OK;
}

// Job and attention tables of the persistent step kernel, mirroring the
// per-projection launches of enqueue_step (same buffers, same residual ping-pong).
int build_step(rt_dec* d) {
    rt_ctx* ctx = d->ctx;
    const int H = d->H, D = d->D, NL = d->NL;
    const int G = d->NQ / d->NKV;
    const int kp_max = std::max({H, d->NQ * D, d->F});
    d->step_geom = rt::step_geometry(H, kp_max, D, G, 4 * NL + 1);
    if (!d->step_geom.warps) return RT_OK;  // shapes outside the step kernel: keep the graph
    if (rt::step_prepare(d->step_geom) != cudaSuccess) {
        cudaGetLastError();
        return RT_OK;
    }
    const int grid = rt::step_max_grid(d->step_geom);
    const int nsplit = std::min(grid / d->NKV, d->nsplit);  // the partials buffer holds d->nsplit slices
    if (grid < ctx->num_sms || nsplit < 1) return RT_OK;
    const int njobs = 4 * NL + 1;
    std::vector<CUtensorMap> tm(njobs);
    for (int l = 0; l < NL; ++l) {
        tm[4 * l] = d->t_qkv[l];
        tm[4 * l + 1] = d->t_o[l];
        tm[4 * l + 2] = d->t_gu[l];
        tm[4 * l + 3] = d->t_down[l];
    }
    tm[4 * NL] = d->t_lm;
    CUtensorMap* d_tm = nullptr;
    rt::gcore::Job* d_jobs = nullptr;
    rt::AttnArgs* d_attn = nullptr;
    uint32_t* d_sync = nullptr;
    // Scratch indexed by CTA or by warp must cover the step kernel's own grid
    // (the per-projection plans may use fewer CTAs).
    float* s_part = nullptr;
    rt::GreedySlot* s_am_slot = nullptr;
    const int64_t part_floats = static_cast<int64_t>(grid) * d->step_geom.warps * 2 * 16;
    int rc;
    if ((rc = dalloc(d, reinterpret_cast<void**>(&s_part), sizeof(float) * part_floats, "step partials")) != RT_OK) return rc;
    if ((rc = dalloc(d, reinterpret_cast<void**>(&s_am_slot), sizeof(rt::GreedySlot) * grid, "step greedy slots")) != RT_OK) return rc;
    if ((rc = dalloc(d, reinterpret_cast<void**>(&d_tm), sizeof(CUtensorMap) * njobs, "step tensor maps")) != RT_OK) return rc;
    if ((rc = dalloc(d, reinterpret_cast<void**>(&d_jobs), sizeof(rt::gcore::Job) * njobs, "step jobs")) != RT_OK) return rc;
    if ((rc = dalloc(d, reinterpret_cast<void**>(&d_attn), sizeof(rt::AttnArgs) * NL, "step attention")) != RT_OK) return rc;
    if ((rc = dalloc(d, reinterpret_cast<void**>(&d_sync), 4 * sizeof(uint32_t), "step sync")) != RT_OK) return rc;
    {
        // Tagged-word vectors of the step kernel; each slice 32-byte aligned.
        const size_t nv[6] = {static_cast<size_t>(d->qkv_rows), static_cast<size_t>(d->NQ) * D, static_cast<size_t>(H),
                              static_cast<size_t>(d->F), static_cast<size_t>(d->down_parts) * H,
                              static_cast<size_t>(d->NKV) * nsplit * (d->NQ / d->NKV) * rt::attn_part_stride(D)};
        size_t words = 0;
        for (size_t n : nv) words += (n + 3) & ~size_t(3);
        if ((rc = dalloc(d, reinterpret_cast<void**>(&d->ll), sizeof(uint64_t) * words, "step tagged vectors")) != RT_OK)
            return rc;
        RT_CHECK_CUDA(ctx, cudaMemsetAsync(d->ll, 0, sizeof(uint64_t) * words, ctx->stream));  // tag 0: never current
        d->ll_words = words;
        uint64_t* q = d->ll;
        uint64_t** dst[6] = {&d->qkv_ll, &d->attn_ll, &d->o_ll, &d->h_ll, &d->down_ll, &d->part_ll};
        for (int i = 0; i < 6; ++i) {
            *dst[i] = q;
            q += (nv[i] + 3) & ~size_t(3);
        }
    }
    // Tile-major copies of the Q4_K projections: each warp's share of a
    // projection is then one contiguous byte range (1-D bulk copies).
    auto tile_major = [&](const uint8_t* w, int64_t rows, int K, int parts, const uint8_t** out) -> int {
        uint8_t* t = nullptr;
        const size_t bytes = static_cast<size_t>((rows + 15) / 16) * (K / 256) * 2304;
        int r = dalloc(d, reinterpret_cast<void**>(&t), bytes, "tile-major weight");
        if (r != RT_OK) return r;
        if (rt::q4k_tile_major_launch(w, rows, K / 256, parts, t, ctx->stream) != cudaSuccess)
            return fail(ctx, RT_E_CUDA, "tile-major weight copy");
        *out = t;
        return RT_OK;
    };
    std::vector<rt::gcore::Job> jobs(njobs);
    std::vector<rt::AttnArgs> attn(NL);
    const float eps = d->cfg.rms_norm_eps;
    auto q4k = [&](int idx, int64_t rows, int K) -> rt::gcore::Job& {
        rt::gcore::Job& j = jobs[idx];
        j = rt::gcore::Job{};
        j.tmap = d_tm + idx;
        j.kind = rt::kQ4K;
        j.K = K;
        j.nseg = K / 256;
        j.rows = rows;
        j.eps = eps;
        return j;
    };
    int p = 0;
    for (int l = 0; l < NL; ++l) {
        rt::gcore::Job& jq = q4k(4 * l, d->qkv_rows, H);
        jq.tile_split = 1;
        jq.g_pre = norm_ptr(d, l, 0);
        jq.y = d->qkv;
        jq.out_ll = d->qkv_ll;
        if (l == 0) {
            jq.embed = d->embed;
            jq.token = d->ctl;
            jq.embed_scale = sqrtf(static_cast<float>(H));
            jq.resid_out = d->resid[0];
            p = 0;
        } else {
            jq.src = d->down;
            jq.in_ll = d->down_ll;
            jq.src_parts = d->down_parts;
            jq.resid_in = d->resid[p];
            jq.resid_out = d->resid[1 - p];
            jq.g_post = norm_ptr(d, l - 1, 3);
            p = 1 - p;
        }
        rt::gcore::Job& jo = q4k(4 * l + 1, H, d->NQ * D);
        jo.x = d->attn;
        jo.y = d->o_out;
        jo.in_ll = d->attn_ll;
        jo.out_ll = d->o_ll;
        jo.tile_split = 1;
        rt::gcore::Job& jg = q4k(4 * l + 2, 2LL * d->F, H);
        jg.src = d->o_out;
        jg.in_ll = d->o_ll;
        jg.out_ll = d->h_ll;
        jg.resid_in = d->resid[p];
        jg.resid_out = d->resid[1 - p];
        jg.g_post = norm_ptr(d, l, 1);
        jg.g_pre = norm_ptr(d, l, 2);
        jg.y = d->hbuf;
        jg.tile_split = 1;
        p = 1 - p;
        // down: column split into down_parts GEMVs (the 160 tiles of a 2560-row
        // output would leave some CTAs twice the units of others)
        rt::gcore::Job& jd = q4k(4 * l + 3, static_cast<int64_t>(d->down_parts) * H, d->F);
        jd.nseg = d->F / 256 / d->down_parts;
        jd.kparts = d->down_parts;
        jd.ptiles = static_cast<int32_t>(H / 16);
        jd.x = d->hbuf;
        jd.y = d->down;
        jd.in_ll = d->h_ll;
        jd.out_ll = d->down_ll;
        jd.tile_split = 1;
        if ((rc = tile_major(d->w_qkv[l], d->qkv_rows, H, 1, &jq.wt)) != RT_OK ||
            (rc = tile_major(d->w_o[l], H, d->NQ * D, 1, &jo.wt)) != RT_OK ||
            (rc = tile_major(d->w_gu[l], 2LL * d->F, H, 1, &jg.wt)) != RT_OK ||
            (rc = tile_major(d->w_down[l], H, d->F, d->down_parts, &jd.wt)) != RT_OK)
            return rc;
        rt::AttnArgs& a = attn[l];
        a = rt::AttnArgs{};
        a.qkv = d->qkv;
        a.q_norm = d->qk_norms + static_cast<size_t>(l) * 2 * D;
        a.k_norm = a.q_norm + D;
        a.kcache = kc_layer(d, l);
        a.vcache = vc_layer(d, l);
        const int gsel = is_global(l) ? 1 : 0;
        const size_t tab = static_cast<size_t>(d->cap) * (D / 2);
        a.rope_cos = d->rope + (static_cast<size_t>(gsel) * 2 + 0) * tab;
        a.rope_sin = d->rope + (static_cast<size_t>(gsel) * 2 + 1) * tab;
        a.pos = d->ctl + 1;
        a.cap = d->cap;
        a.nq = d->NQ;
        a.nkv = d->NKV;
        a.D = D;
        a.window = is_global(l) ? 0 : d->cfg.sliding_window;
        a.nsplit = nsplit;
        a.scale = 1.0f / sqrtf(d->cfg.query_pre_attn_scalar);
        a.eps = eps;
        a.part = d->attn_part;
        a.counter = d->counters;
        a.out = d->attn;
        a.qkv_ll = d->qkv_ll;
        a.out_ll = d->attn_ll;
        a.part_ll = d->part_ll;
        a.err = ctx->d_err;
    }
    rt::gcore::Job& jl = jobs[4 * NL];
    jl = rt::gcore::Job{};
    jl.tmap = d_tm + 4 * NL;
    jl.kind = rt::kBF16;
    jl.K = H;
    jl.nseg = (H + 127) / 128;
    jl.rows = d->V;
    jl.eps = eps;
    jl.src = d->down;
    jl.in_ll = d->down_ll;
    jl.src_parts = d->down_parts;
    jl.resid_in = d->resid[p];
    jl.resid_out = d->resid[1 - p];
    jl.g_post = norm_ptr(d, NL - 1, 3);
    jl.g_pre = d->final_norm;
    jl.tile_split = 1;
    jl.y = d->logits;
    jl.am_slot = s_am_slot;
    jl.am_counter = d->counters + d->NKV;
    jl.token_out = d->ctl;
    jl.pos_inout = d->ctl + 1;
    jl.token_hist = d->ctl + 2;
    cudaStream_t s = ctx->stream;
    RT_CHECK_CUDA(ctx, cudaMemcpyAsync(d_tm, tm.data(), sizeof(CUtensorMap) * njobs, cudaMemcpyHostToDevice, s));
    RT_CHECK_CUDA(ctx, cudaMemcpyAsync(d_jobs, jobs.data(), sizeof(rt::gcore::Job) * njobs, cudaMemcpyHostToDevice, s));
    RT_CHECK_CUDA(ctx, cudaMemcpyAsync(d_attn, attn.data(), sizeof(rt::AttnArgs) * NL, cudaMemcpyHostToDevice, s));
    RT_CHECK_CUDA(ctx, cudaMemsetAsync(d_sync, 0, 4 * sizeof(uint32_t), s));
    RT_CHECK_CUDA(ctx, cudaStreamSynchronize(s));
    rt::StepParams& P = d->step_params;
    P.geom = d->step_geom;
    P.jobs = d_jobs;
    P.attn = d_attn;
    P.nlayers = NL;
    P.sync = d_sync;
    P.abort = reinterpret_cast<int*>(d_sync + 2);
    P.scratch = rt::gcore::SplitScratch{s_part, d->g_cnt};
    P.err = ctx->d_err;

    if ((rc = dalloc(d, reinterpret_cast<void**>(&P.trace), sizeof(uint64_t) * rt::kStepTraceLen, "step trace")) != RT_OK)
        return rc;
    RT_CHECK_CUDA(ctx, cudaMemset(P.trace, 0, sizeof(uint64_t) * rt::kStepTraceLen));
    d->step_grid = grid;
    d->use_step = getenv("RT_DECODER_GRAPH") == nullptr;
    if (d->use_step) d->launches = 1;
    return RT_OK;
}

int build_graph(rt_dec* d) {
    cudaStream_t s = d->ctx->stream;
    RT_CHECK_CUDA(d->ctx, cudaStreamBeginCapture(s, cudaStreamCaptureModeThreadLocal));
    int32_t n = 0;
    cudaError_t e = enqueue_step(d, s, true, false, &n, nullptr);
    cudaGraph_t g = nullptr;
    cudaError_t e2 = cudaStreamEndCapture(s, &g);
    if (e != cudaSuccess || e2 != cudaSuccess) {
        if (g) cudaGraphDestroy(g);
        cudaGetLastError();
        return fail(d->ctx, RT_E_CUDA, "graph capture failed: %s / %s", cudaGetErrorString(e), cudaGetErrorString(e2));
    }
    d->graph = g;
    d->launches = n;
    RT_CHECK_CUDA(d->ctx, cudaGraphInstantiate(&d->exec, g, 0));
    return RT_OK;
}

cudaError_t launch_one_step(rt_dec* d, cudaStream_t s) {
    if (d->use_step) return rt::step_launch(d->step_params, d->step_geom, d->step_grid, s);
    return cudaGraphLaunch(d->exec, s);
}

cudaError_t set_ctl(rt_dec* d, int32_t token, int32_t pos) {
    set_ctl_kernel<<<1, 1, 0, d->ctx->stream>>>(d->ctl, token, pos);
    return cudaGetLastError();
}

int post_launch_check(rt_dec* d) {
    if (*d->h_err) {
        const int w = *d->h_err;
        *d->h_err = 0;
        cudaMemsetAsync(d->ctx->d_err, 0, sizeof(int), d->ctx->stream);
        // Counters a failed launch can leave behind: attention merges and the
        // greedy arrivals, and the GEMVs' split-tile unit counts.
        cudaMemsetAsync(d->counters, 0, sizeof(uint32_t) * (d->NKV + 1), d->ctx->stream);
        if (d->g_cnt && d->g_cnt_words) cudaMemsetAsync(d->g_cnt, 0, sizeof(uint32_t) * d->g_cnt_words, d->ctx->stream);
        if (d->use_step) {
            // an aborted step kernel leaves its counters behind; with the launch
            // count back at zero, the tagged vectors are cleared too (tag 0 is
            // never current), so no word of the aborted launch can pass for new
            cudaMemsetAsync(d->step_params.sync, 0, 2 * sizeof(uint32_t), d->ctx->stream);
            cudaMemsetAsync(d->step_params.abort, 0, sizeof(int), d->ctx->stream);
            if (d->ll) cudaMemsetAsync(d->ll, 0, sizeof(uint64_t) * d->ll_words, d->ctx->stream);
        }
        cudaStreamSynchronize(d->ctx->stream);
        return fail(d->ctx, RT_E_TIMEOUT, "decode step: a kernel reported error word %d", w);
    }
    return RT_OK;
}

}  // namespace

extern "C" {

void rt_decoder_destroy(rt_dec* d) {
    if (!d) return;
    cudaSetDevice(d->ctx->device);
    cudaStreamSynchronize(d->ctx->stream);
    if (d->rows) rt::rows_engine_free(d->rows);
    if (d->exec) cudaGraphExecDestroy(d->exec);
    if (d->graph) cudaGraphDestroy(d->graph);
    for (void* p : d->allocs) cudaFree(p);
    if (d->h_err) cudaFreeHost(d->h_err);
    delete d;
}

int rt_decoder_create(rt_ctx* ctx, const rt_gemma3_cfg* cfg, const rt_gemma3_layer* layers, const rt_w* embed,
                      const float* final_norm, int32_t max_ctx, rt_dec** out) {
    if (!ctx || !cfg || !layers || !embed || !final_norm || !out) return fail(ctx, RT_E_INVAL, "rt_decoder_create: null argument");
    *out = nullptr;
    const rt_gemma3_cfg& c = *cfg;
    if (c.hidden_size <= 0 || c.hidden_size % 256 || c.intermediate_size <= 0 || c.intermediate_size % 256 ||
        c.head_dim <= 0 || c.head_dim % 32 || c.head_dim > 256 || c.num_attention_heads <= 0 ||
        c.num_key_value_heads <= 0 || c.num_attention_heads % c.num_key_value_heads ||
        (static_cast<int64_t>(c.num_attention_heads) * c.head_dim) % 256 || c.num_hidden_layers <= 0 ||
        c.vocab_size <= 0 || max_ctx <= 0)
        return fail(ctx, RT_E_SHAPE, "rt_decoder_create: unsupported config");
    const int G = c.num_attention_heads / c.num_key_value_heads;
    if (G != 1 && G != 2 && G != 4 && G != 8) return fail(ctx, RT_E_SHAPE, "rt_decoder_create: GQA group %d unsupported", G);
    if (embed->fmt != RT_FMT_BF16 || embed->rows != c.vocab_size || embed->cols != c.hidden_size)
        return fail(ctx, RT_E_SHAPE, "rt_decoder_create: embedding must be BF16 [vocab, hidden]");
    for (int i = 0; i < c.num_hidden_layers; ++i) {
        int rc = check_layer(ctx, c, layers[i], i);
        if (rc != RT_OK) return rc;
    }
    RT_CHECK_CUDA(ctx, cudaSetDevice(ctx->device));
    rt_dec* d = new rt_dec();
    d->ctx = ctx;
    d->cfg = c;
    d->H = c.hidden_size;
    d->D = c.head_dim;
    d->NQ = c.num_attention_heads;
    d->NKV = c.num_key_value_heads;
    d->F = c.intermediate_size;
    d->V = c.vocab_size;
    d->NL = c.num_hidden_layers;
    d->cap = max_ctx;
    d->qkv_rows = (d->NQ + 2 * d->NKV) * d->D;
    const int H = d->H, D = d->D, NL = d->NL;
    cudaStream_t s = ctx->stream;
    auto bail = [&](int rc) {
        rt_decoder_destroy(d);
        return rc;
    };
    int rc;
    // --- weights: fused QKV (rows q | k | v), interleaved gate/up, o, down ---
    const uint64_t row_h = static_cast<uint64_t>(H / 256) * 144;
    d->w_qkv.resize(NL);
    d->w_o.resize(NL);
    d->w_gu.resize(NL);
    d->w_down.resize(NL);
    for (int l = 0; l < NL; ++l) {
        const rt_gemma3_layer& L = layers[l];
        if ((rc = dalloc(d, reinterpret_cast<void**>(&d->w_qkv[l]), row_h * d->qkv_rows, "qkv weight")) != RT_OK) return bail(rc);
        uint8_t* dst = d->w_qkv[l];
        for (const rt_w* w : {L.q, L.k, L.v}) {
            if (cudaMemcpyAsync(dst, w->d, w->bytes, cudaMemcpyDeviceToDevice, s) != cudaSuccess)
                return bail(fail(ctx, RT_E_CUDA, "copy qkv"));
            dst += w->bytes;
        }
        if ((rc = dalloc(d, reinterpret_cast<void**>(&d->w_o[l]), L.o->bytes, "o weight")) != RT_OK) return bail(rc);
        if (cudaMemcpyAsync(d->w_o[l], L.o->d, L.o->bytes, cudaMemcpyDeviceToDevice, s) != cudaSuccess)
            return bail(fail(ctx, RT_E_CUDA, "copy o"));
        if ((rc = dalloc(d, reinterpret_cast<void**>(&d->w_gu[l]), 2 * L.gate->bytes, "gate/up weight")) != RT_OK) return bail(rc);
        // row 2j = gate row j, row 2j+1 = up row j
        if (cudaMemcpy2DAsync(d->w_gu[l], 2 * row_h, L.gate->d, row_h, row_h, d->F, cudaMemcpyDeviceToDevice, s) != cudaSuccess ||
            cudaMemcpy2DAsync(d->w_gu[l] + row_h, 2 * row_h, L.up->d, row_h, row_h, d->F, cudaMemcpyDeviceToDevice, s) != cudaSuccess)
            return bail(fail(ctx, RT_E_CUDA, "copy gate/up"));
        if ((rc = dalloc(d, reinterpret_cast<void**>(&d->w_down[l]), L.down->bytes, "down weight")) != RT_OK) return bail(rc);
        if (cudaMemcpyAsync(d->w_down[l], L.down->d, L.down->bytes, cudaMemcpyDeviceToDevice, s) != cudaSuccess)
            return bail(fail(ctx, RT_E_CUDA, "copy down"));
    }
    if ((rc = dalloc(d, reinterpret_cast<void**>(&d->embed), embed->bytes, "embedding")) != RT_OK) return bail(rc);
    if (cudaMemcpyAsync(d->embed, embed->d, embed->bytes, cudaMemcpyDeviceToDevice, s) != cudaSuccess)
        return bail(fail(ctx, RT_E_CUDA, "copy embedding"));
    // --- norms ---
    {
        std::vector<float> h(static_cast<size_t>(NL) * 4 * H);
        std::vector<float> hq(static_cast<size_t>(NL) * 2 * D);
        for (int l = 0; l < NL; ++l) {
            const float* src[4] = {layers[l].attn_norm, layers[l].post_attn_norm, layers[l].pre_ffn_norm,
                                   layers[l].post_ffn_norm};
            for (int w = 0; w < 4; ++w) memcpy(&h[(static_cast<size_t>(l) * 4 + w) * H], src[w], sizeof(float) * H);
            memcpy(&hq[static_cast<size_t>(l) * 2 * D], layers[l].q_norm, sizeof(float) * D);
            memcpy(&hq[static_cast<size_t>(l) * 2 * D + D], layers[l].k_norm, sizeof(float) * D);
        }
        if ((rc = dalloc(d, reinterpret_cast<void**>(&d->norms), h.size() * 4, "norms")) != RT_OK) return bail(rc);
        if ((rc = dalloc(d, reinterpret_cast<void**>(&d->qk_norms), hq.size() * 4, "qk norms")) != RT_OK) return bail(rc);
        if ((rc = dalloc(d, reinterpret_cast<void**>(&d->final_norm), sizeof(float) * H, "final norm")) != RT_OK) return bail(rc);
        if (cudaMemcpy(d->norms, h.data(), h.size() * 4, cudaMemcpyHostToDevice) != cudaSuccess ||
            cudaMemcpy(d->qk_norms, hq.data(), hq.size() * 4, cudaMemcpyHostToDevice) != cudaSuccess ||
            cudaMemcpy(d->final_norm, final_norm, sizeof(float) * H, cudaMemcpyHostToDevice) != cudaSuccess)
            return bail(fail(ctx, RT_E_CUDA, "upload norms"));
    }
    // --- KV cache and RoPE tables ---
    const size_t kv_elems = static_cast<size_t>(NL) * d->NKV * d->cap * D;
    if ((rc = dalloc(d, reinterpret_cast<void**>(&d->kcache), kv_elems * 4, "K cache")) != RT_OK) return bail(rc);
    if ((rc = dalloc(d, reinterpret_cast<void**>(&d->vcache), kv_elems * 4, "V cache")) != RT_OK) return bail(rc);
    cudaMemsetAsync(d->kcache, 0, kv_elems * 4, s);
    cudaMemsetAsync(d->vcache, 0, kv_elems * 4, s);
    {
        const size_t tab = static_cast<size_t>(d->cap) * (D / 2);
        std::vector<float> r(4 * tab);
        rt::rope_table(c.rope_theta_local, c.rope_freq_scale_local, D, d->cap, &r[0], &r[tab]);
        rt::rope_table(c.rope_theta_global, c.rope_freq_scale_global, D, d->cap, &r[2 * tab], &r[3 * tab]);
        if ((rc = dalloc(d, reinterpret_cast<void**>(&d->rope), r.size() * 4, "rope tables")) != RT_OK) return bail(rc);
        if (cudaMemcpy(d->rope, r.data(), r.size() * 4, cudaMemcpyHostToDevice) != cudaSuccess)
            return bail(fail(ctx, RT_E_CUDA, "upload rope tables"));
    }
    // --- plans ---
    rt::gemv_prepare();
    d->p_qkv = rt::gemv_plan(rt::kQ4K, d->qkv_rows, H, 1, rt::kProResidNorm, rt::kEpiPlain, ctx->num_sms, 1);
    d->p_o = rt::gemv_plan(rt::kQ4K, H, d->NQ * D, 1, rt::kProPlain, rt::kEpiPlain, ctx->num_sms, 1);
    d->p_gu = rt::gemv_plan(rt::kQ4K, 2LL * d->F, H, 2, rt::kProResidNorm, rt::kEpiGeluPair, ctx->num_sms, 1);
    d->p_down = rt::gemv_plan(rt::kQ4K, H, d->F, 1, rt::kProPlain, rt::kEpiPlain, ctx->num_sms, 1);
    d->p_lm = rt::gemv_plan(rt::kBF16, d->V, H, 1, rt::kProResidNorm, rt::kEpiArgmax, ctx->num_sms, 1);
    // Without GEMV geometry for these shapes the decoder holds the weights,
    // caches and tables for the GEMM-based engines (rows mode, many-sequence,
    // tensor-parallel shards) and refuses the single-sequence calls.
    d->single = d->p_qkv.warps && d->p_o.warps && d->p_gu.warps && d->p_down.warps && d->p_lm.warps;
    if (!d->single) {
        if (cudaMallocHost(reinterpret_cast<void**>(&d->h_err), sizeof(int) * 4) != cudaSuccess)
            return bail(fail(ctx, RT_E_NOMEM, "pinned staging"));
        *d->h_err = 0;
        if (cudaStreamSynchronize(s) != cudaSuccess) return bail(fail(ctx, RT_E_CUDA, "rt_decoder_create: set-up failed"));
        *out = d;
        return RT_OK;
    }
    d->t_qkv.resize(NL);
    d->t_o.resize(NL);
    d->t_gu.resize(NL);
    d->t_down.resize(NL);
    for (int l = 0; l < NL; ++l) {
        if (!rt::gemv_make_tmap(rt::kQ4K, d->w_qkv[l], d->qkv_rows, H, d->p_qkv, &d->t_qkv[l]) ||
            !rt::gemv_make_tmap(rt::kQ4K, d->w_o[l], H, d->NQ * D, d->p_o, &d->t_o[l]) ||
            !rt::gemv_make_tmap(rt::kQ4K, d->w_gu[l], 2LL * d->F, H, d->p_gu, &d->t_gu[l]) ||
            !rt::gemv_make_tmap(rt::kQ4K, d->w_down[l], H, d->F, d->p_down, &d->t_down[l]))
            return bail(fail(ctx, RT_E_CUDA, "rt_decoder_create: TMA descriptor rejected (layer %d)", l));
    }
    if (!rt::gemv_make_tmap(rt::kBF16, d->embed, d->V, H, d->p_lm, &d->t_lm))
        return bail(fail(ctx, RT_E_CUDA, "rt_decoder_create: TMA descriptor rejected (LM head)"));
    d->nsplit = std::max(1, std::min(64, (ctx->num_sms + d->NKV - 1) / d->NKV));
    // RT_STEP_ATTN_SPLITS overrides the context splits per KV head (tuning).
    if (const char* e = getenv("RT_STEP_ATTN_SPLITS")) d->nsplit = std::max(1, std::min(d->nsplit, atoi(e)));
    for (int parts = kMaxDownParts; parts >= 1; parts /= 2)
        if ((d->F / 256) % parts == 0) {
            d->down_parts = parts;
            break;
        }
    if (rt::attention_prepare() != cudaSuccess) return bail(fail(ctx, RT_E_CUDA, "attention kernel attributes"));
    // --- activations ---
    {
        const size_t G_ = static_cast<size_t>(G);
        const size_t n_act = 2 * static_cast<size_t>(H) + d->qkv_rows + static_cast<size_t>(d->NQ) * D + H + d->F +
                             static_cast<size_t>(kMaxDownParts) * H +
                             d->V + static_cast<size_t>(d->NKV) * d->nsplit * G_ * rt::attn_part_stride(D) + d->p_lm.grid + 10 * 64;
        if ((rc = dalloc(d, reinterpret_cast<void**>(&d->act), n_act * 4 + 1024, "activations")) != RT_OK) return bail(rc);
        cudaMemsetAsync(d->act, 0, n_act * 4 + 1024, s);
        // Every slice starts on a 256-byte boundary (the kernels move these
        // vectors with TMA bulk copies, which need 16-byte alignment).
        float* p = d->act;
        auto slice = [&](size_t n) {
            float* q = p;
            p += (n + 63) & ~size_t(63);
            return q;
        };
        d->resid[0] = slice(H);
        d->resid[1] = slice(H);
        d->qkv = slice(d->qkv_rows);
        d->attn = slice(static_cast<size_t>(d->NQ) * D);
        d->o_out = slice(H);
        d->hbuf = slice(d->F);
        d->down = slice(static_cast<size_t>(kMaxDownParts) * H);  // the step path keeps down_parts partials
        d->logits = slice(d->V);
        d->attn_part = slice(static_cast<size_t>(d->NKV) * d->nsplit * G_ * rt::attn_part_stride(D));
        if ((rc = dalloc(d, reinterpret_cast<void**>(&d->am_slot), sizeof(rt::GreedySlot) * d->p_lm.grid, "greedy slots")) != RT_OK) return bail(rc);
        if ((rc = dalloc(d, reinterpret_cast<void**>(&d->counters), sizeof(uint32_t) * (d->NKV + 1), "counters")) != RT_OK) return bail(rc);
        cudaMemsetAsync(d->counters, 0, sizeof(uint32_t) * (d->NKV + 1), s);
        int64_t part_floats = 0, cnt_words = 0;
        for (const rt::GemvPlan* gp : {&d->p_qkv, &d->p_o, &d->p_gu, &d->p_down, &d->p_lm}) {
            part_floats = std::max(part_floats, gp->part_floats);
            cnt_words = std::max(cnt_words, gp->cnt_words);
        }
        if ((rc = dalloc(d, reinterpret_cast<void**>(&d->g_part), sizeof(float) * part_floats, "gemv partials")) != RT_OK) return bail(rc);
        if ((rc = dalloc(d, reinterpret_cast<void**>(&d->g_cnt), sizeof(uint32_t) * cnt_words, "gemv counters")) != RT_OK) return bail(rc);
        d->g_cnt_words = cnt_words;
        cudaMemsetAsync(d->g_cnt, 0, sizeof(uint32_t) * cnt_words, s);
        if ((rc = dalloc(d, reinterpret_cast<void**>(&d->ctl), sizeof(int32_t) * (2 + d->cap), "control")) != RT_OK) return bail(rc);
        cudaMemsetAsync(d->ctl, 0, sizeof(int32_t) * (2 + d->cap), s);
    }
    if (cudaMallocHost(reinterpret_cast<void**>(&d->h_err), sizeof(int) * 4) != cudaSuccess)
        return bail(fail(ctx, RT_E_NOMEM, "pinned staging"));
    *d->h_err = 0;
    if (cudaStreamSynchronize(s) != cudaSuccess) return bail(fail(ctx, RT_E_CUDA, "rt_decoder_create: set-up failed"));
    if ((rc = build_graph(d)) != RT_OK) return bail(rc);
    if ((rc = build_step(d)) != RT_OK) return bail(rc);
    *out = d;
    return RT_OK;
}

int rt_decoder_load_kv(rt_dec* d, int32_t layer, const float* k, const float* v, int32_t seq_len) {
    if (!d || !k || !v) return fail(d ? d->ctx : nullptr, RT_E_INVAL, "rt_decoder_load_kv: null argument");
    if (layer < 0 || layer >= d->NL || seq_len < 0 || seq_len > d->cap)
        return fail(d->ctx, RT_E_SHAPE, "rt_decoder_load_kv: layer %d / seq_len %d out of range", layer, seq_len);
    if (seq_len == 0) return RT_OK;
    const size_t D = d->D, row = static_cast<size_t>(d->NKV) * D;
    for (int h = 0; h < d->NKV; ++h) {
        float* kd = kc_layer(d, layer) + static_cast<size_t>(h) * d->cap * D;
        float* vd = vc_layer(d, layer) + static_cast<size_t>(h) * d->cap * D;
        RT_CHECK_CUDA(d->ctx, cudaMemcpy2DAsync(kd, D * 4, k + h * D, row * 4, D * 4, seq_len, cudaMemcpyHostToDevice, d->ctx->stream));
        RT_CHECK_CUDA(d->ctx, cudaMemcpy2DAsync(vd, D * 4, v + h * D, row * 4, D * 4, seq_len, cudaMemcpyHostToDevice, d->ctx->stream));
    }
    RT_CHECK_CUDA(d->ctx, cudaStreamSynchronize(d->ctx->stream));
    return RT_OK;
}

int rt_decoder_read_kv(rt_dec* d, int32_t layer, float* k, float* v, int32_t seq_len) {
    if (!d || !k || !v) return fail(d ? d->ctx : nullptr, RT_E_INVAL, "rt_decoder_read_kv: null argument");
    if (layer < 0 || layer >= d->NL || seq_len < 0 || seq_len > d->cap)
        return fail(d->ctx, RT_E_SHAPE, "rt_decoder_read_kv: layer %d / seq_len %d out of range", layer, seq_len);
    if (seq_len == 0) return RT_OK;
    const size_t D = d->D, row = static_cast<size_t>(d->NKV) * D;
    for (int h = 0; h < d->NKV; ++h) {
        const float* kd = kc_layer(d, layer) + static_cast<size_t>(h) * d->cap * D;
        const float* vd = vc_layer(d, layer) + static_cast<size_t>(h) * d->cap * D;
        RT_CHECK_CUDA(d->ctx, cudaMemcpy2DAsync(k + h * D, row * 4, kd, D * 4, D * 4, seq_len, cudaMemcpyDeviceToHost, d->ctx->stream));
        RT_CHECK_CUDA(d->ctx, cudaMemcpy2DAsync(v + h * D, row * 4, vd, D * 4, D * 4, seq_len, cudaMemcpyDeviceToHost, d->ctx->stream));
    }
    RT_CHECK_CUDA(d->ctx, cudaStreamSynchronize(d->ctx->stream));
    return RT_OK;
}

int rt_decoder_step(rt_dec* d, int32_t token, int32_t position, float* logits) {
    if (!d) return RT_E_INVAL;
    if (!d->single) return fail(d->ctx, RT_E_SHAPE, "rt_decoder_step: no single-sequence path for these shapes");
    if (token < 0 || token >= d->V) return fail(d->ctx, RT_E_INVAL, "rt_decoder_step: token %d out of range", token);
    if (position < 0 || position >= d->cap)
        return fail(d->ctx, RT_E_STATE, "rt_decoder_step: position %d outside the %d-position cache", position, d->cap);
    cudaStream_t s = d->ctx->stream;
    RT_CHECK_CUDA(d->ctx, set_ctl(d, token, position));
    RT_CHECK_CUDA(d->ctx, launch_one_step(d, s));
    if (logits) RT_CHECK_CUDA(d->ctx, cudaMemcpyAsync(logits, d->logits, sizeof(float) * d->V, cudaMemcpyDeviceToHost, s));
    RT_CHECK_CUDA(d->ctx, cudaMemcpyAsync(d->h_err, d->ctx->d_err, sizeof(int), cudaMemcpyDeviceToHost, s));
    RT_CHECK_CUDA(d->ctx, cudaStreamSynchronize(s));
    return post_launch_check(d);
}

int rt_decoder_prefill(rt_dec* d, const int32_t* tokens, int32_t n, int32_t start_pos, float* last_logits) {
    if (!d || (!tokens && n > 0)) return fail(d ? d->ctx : nullptr, RT_E_INVAL, "rt_decoder_prefill: null argument");
    if (!d->single) return fail(d->ctx, RT_E_SHAPE, "rt_decoder_prefill: no single-sequence path for these shapes");
    if (n <= 0) return RT_OK;
    if (start_pos < 0 || static_cast<int64_t>(start_pos) + n > d->cap)
        return fail(d->ctx, RT_E_STATE, "rt_decoder_prefill: positions %d..%d outside the cache", start_pos, start_pos + n - 1);
    for (int i = 0; i < n; ++i)
        if (tokens[i] < 0 || tokens[i] >= d->V) return fail(d->ctx, RT_E_INVAL, "rt_decoder_prefill: token %d out of range", tokens[i]);
    cudaStream_t s = d->ctx->stream;
    for (int i = 0; i < n; ++i) {
        RT_CHECK_CUDA(d->ctx, set_ctl(d, tokens[i], start_pos + i));
        RT_CHECK_CUDA(d->ctx, launch_one_step(d, s));
    }
    if (last_logits) RT_CHECK_CUDA(d->ctx, cudaMemcpyAsync(last_logits, d->logits, sizeof(float) * d->V, cudaMemcpyDeviceToHost, s));
    RT_CHECK_CUDA(d->ctx, cudaMemcpyAsync(d->h_err, d->ctx->d_err, sizeof(int), cudaMemcpyDeviceToHost, s));
    RT_CHECK_CUDA(d->ctx, cudaStreamSynchronize(s));
    return post_launch_check(d);
}

int rt_decoder_generate(rt_dec* d, int32_t first_token, int32_t start_pos, int32_t n, int32_t* tokens_out, int flags) {
    if (!d) return RT_E_INVAL;
    if (!d->single) return fail(d->ctx, RT_E_SHAPE, "rt_decoder_generate: no single-sequence path for these shapes");
    if (flags != RT_HOST && flags != RT_DEVICE) return fail(d->ctx, RT_E_INVAL, "rt_decoder_generate: bad flags");
    if (flags == RT_DEVICE && tokens_out) return fail(d->ctx, RT_E_INVAL, "rt_decoder_generate: RT_DEVICE takes no tokens_out");
    if (first_token < 0 || first_token >= d->V) return fail(d->ctx, RT_E_INVAL, "rt_decoder_generate: token out of range");
    if (n <= 0) return RT_OK;
    if (start_pos < 0 || static_cast<int64_t>(start_pos) + n > d->cap)
        return fail(d->ctx, RT_E_STATE, "rt_decoder_generate: positions %d..%d outside the cache", start_pos, start_pos + n - 1);
    cudaStream_t s = d->ctx->stream;
    RT_CHECK_CUDA(d->ctx, set_ctl(d, first_token, start_pos));
    for (int i = 0; i < n; ++i) RT_CHECK_CUDA(d->ctx, launch_one_step(d, s));
    if (flags == RT_DEVICE) return RT_OK;
    if (tokens_out)
        RT_CHECK_CUDA(d->ctx, cudaMemcpyAsync(tokens_out, d->ctl + 2 + start_pos, sizeof(int32_t) * n, cudaMemcpyDeviceToHost, s));
    RT_CHECK_CUDA(d->ctx, cudaMemcpyAsync(d->h_err, d->ctx->d_err, sizeof(int), cudaMemcpyDeviceToHost, s));
    RT_CHECK_CUDA(d->ctx, cudaStreamSynchronize(s));
    return post_launch_check(d);
}

int rt_decoder_enqueue_q4k_gemvs(rt_dec* d, int32_t* n_launches, uint64_t* bytes) {
    if (!d) return RT_E_INVAL;
    if (!d->single) return fail(d->ctx, RT_E_SHAPE, "rt_decoder_enqueue_q4k_gemvs: no single-sequence path for these shapes");
    RT_CHECK_CUDA(d->ctx, enqueue_step(d, d->ctx->stream, false, true, n_launches, bytes));
    return RT_OK;
}

int rt_decoder_memory(const rt_dec* d, uint64_t* bytes) {
    if (!d || !bytes) return RT_E_INVAL;
    *bytes = d->dev_bytes;
    return RT_OK;
}

int rt_decoder_launches_per_step(const rt_dec* d, int32_t* n) {
    if (!d || !n) return RT_E_INVAL;
    *n = d->launches;
    return RT_OK;
}

int rt_decoder_read_activation(rt_dec* d, int32_t which, float* host, int64_t count) {
    if (!d || !host) return RT_E_INVAL;
    if (!d->single) return fail(d->ctx, RT_E_SHAPE, "rt_decoder_read_activation: no single-sequence path for these shapes");
    const float* src = nullptr;
    int64_t n = 0;
    if (which == 0) {
        src = d->resid[d->final_resid];
        n = d->H;
    } else if (which == 1) {
        src = d->logits;
        n = d->V;
    } else if (which >= 3 && which <= 7 && d->use_step) {
        // the step kernel keeps these vectors as tagged words (value in the low 32 bits);
        // the down projection as its column parts, added here in part order
        uint64_t* v[5] = {d->qkv_ll, d->attn_ll, d->o_ll, d->h_ll, d->down_ll};
        const int64_t nv[5] = {d->qkv_rows, static_cast<int64_t>(d->NQ) * d->D, d->H, d->F, d->H};
        const int64_t nn = nv[which - 3];
        const int parts = which == 7 ? d->down_parts : 1;
        if (count < 0 || count > nn) return fail(d->ctx, RT_E_SHAPE, "rt_decoder_read_activation: count %lld > %lld",
                                                 static_cast<long long>(count), static_cast<long long>(nn));
        std::vector<uint64_t> w(static_cast<size_t>(parts) * nn);
        RT_CHECK_CUDA(d->ctx, cudaMemcpyAsync(w.data(), v[which - 3], sizeof(uint64_t) * w.size(), cudaMemcpyDeviceToHost,
                                              d->ctx->stream));
        RT_CHECK_CUDA(d->ctx, cudaStreamSynchronize(d->ctx->stream));
        auto val = [](uint64_t x) {
            const uint32_t b = static_cast<uint32_t>(x);
            float f;
            memcpy(&f, &b, 4);
            return f;
        };
        for (int64_t i = 0; i < count; ++i) {
            float a = val(w[static_cast<size_t>(i)]);
            for (int q = 1; q < parts; ++q) a += val(w[static_cast<size_t>(q) * nn + i]);
            host[i] = a;
        }
        return RT_OK;
    } else if (which == 7 && d->use_step && d->down_parts > 1) {
        // the step kernel leaves the down projection as column-part partials
        if (count < 0 || count > d->H) return fail(d->ctx, RT_E_SHAPE, "rt_decoder_read_activation: count %lld > %lld",
                                                   static_cast<long long>(count), static_cast<long long>(d->H));
        std::vector<float> parts(static_cast<size_t>(d->down_parts) * d->H);
        RT_CHECK_CUDA(d->ctx, cudaMemcpyAsync(parts.data(), d->down, sizeof(float) * parts.size(), cudaMemcpyDeviceToHost,
                                              d->ctx->stream));
        RT_CHECK_CUDA(d->ctx, cudaStreamSynchronize(d->ctx->stream));
        for (int64_t i = 0; i < count; ++i) {
            float v = parts[i];
            for (int q = 1; q < d->down_parts; ++q) v += parts[static_cast<size_t>(q) * d->H + i];
            host[i] = v;
        }
        return RT_OK;
    } else if (which >= 3 && which <= 7) {
        // the last layer's intermediate vectors: qkv, attention output, O
        // projection, GELU-gated FFN hidden, down projection
        const float* v[5] = {d->qkv, d->attn, d->o_out, d->hbuf, d->down};
        const int64_t nv[5] = {d->qkv_rows, static_cast<int64_t>(d->NQ) * d->D, d->H, d->F, d->H};
        src = v[which - 3];
        n = nv[which - 3];
    } else if (which == 2 && d->use_step) {
        // phase timeline of the last step kernel: kStepTraceLen u64 as 2x f32 each
        src = reinterpret_cast<const float*>(d->step_params.trace);
        n = 2 * rt::kStepTraceLen;
    } else {
        return fail(d->ctx, RT_E_INVAL, "rt_decoder_read_activation: unknown vector %d", which);
    }
    if (count < 0 || count > n) return fail(d->ctx, RT_E_SHAPE, "rt_decoder_read_activation: count %lld > %lld",
                                            static_cast<long long>(count), static_cast<long long>(n));
    RT_CHECK_CUDA(d->ctx, cudaMemcpyAsync(host, src, sizeof(float) * count, cudaMemcpyDeviceToHost, d->ctx->stream));
    RT_CHECK_CUDA(d->ctx, cudaStreamSynchronize(d->ctx->stream));
    return RT_OK;
}

}  // extern "C"
