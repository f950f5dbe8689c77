// qwen35.cu -- Qwen 3.5 decode engine (rt_qwen35_*): the hybrid Gated
// DeltaNet / full-attention model of src/transformer_qwen35.rs, one token per
// call, every projection on this library's Q4_K GEMV (gemv_cluster.cu) and the
// tied BF16 LM head on the BF16 GEMV.  The Metal engine it stands in for is
// MetalDecodeContextQwen35 (src/metal_decode_qwen35.rs).
//
// Per layer (Qwen35Block::forward_cached, src/transformer_qwen35.rs:905-924):
//   xn = rmsnorm(x) (1 + input_norm)                         resid_norm_kernel
//   DeltaNet layer (Qwen35DeltaNet::forward_cached, :315-456):
//     [qkv | z | a | b] = W_in xn                             one fused GEMV
//     conv = silu(causal depthwise conv1d(qkv, state))        dn_conv_kernel
//     per value head: l2-normalised q, k (key head h / (nv / nk)), q / sqrt(kd);
//       S = exp(g) S;  S += k (beta (v - S^T k))^T;  o = S^T q;
//       out = rmsnorm(o) * norm_weight * silu(z)              dn_heads_kernel
//     y = W_out out                                           GEMV
//   full-attention layer (Qwen35FullAttention::forward_cached, :663-724):
//     [q, gate per head | k | v] = W_qkv xn                   one fused GEMV
//     per-head RMSNorm (1 + gamma), partial RoPE, K/V append  fa_prep_kernel
//     softmax attention over the cache, times sigmoid(gate)   fa_attn_kernel
//     y = W_o out                                             GEMV
//   x += y;  xn = rmsnorm(x) (1 + post_norm)                  resid_norm_kernel
//   x += W_down (silu(W_gate xn) * W_up xn)                   GEMV, silu_mul_kernel, GEMV
// then rmsnorm(x) (1 + final_norm) and the LM head.
//
// State lives in HBM: each DeltaNet layer's recurrent matrices ([nv][kd][vd]
// f32) and conv1d history ([qkv_dim][kernel - 1]), each full-attention
// layer's f32 K/V cache ([max_tokens][nkv][head_dim]).
#include <math.h>

#include <algorithm>
#include <vector>

#include "../../include/rt_cuda.h"
#include "common.cuh"
#include "gemv.cuh"
#include "rt_internal.h"

using rt::fail;

namespace {

constexpr int kQThreads = 256;
constexpr int kQWide = 1024;  // threads of the row-norm and DeltaNet head kernels (short per-thread chains)

__device__ __forceinline__ float sigmoid_f(float x) { return 1.0f / (1.0f + expf(-x)); }
__device__ __forceinline__ float silu_f(float x) { return x * sigmoid_f(x); }
__device__ __forceinline__ float softplus_f(float x) { return x > 20.0f ? x : logf(1.0f + expf(x)); }

// Sum of v over the block (up to 1024 threads), the same value in every thread.
__device__ __forceinline__ float qblock_sum(float v, float* red) {
    v = rt::block_sum(v, red);
    __syncthreads();  // red is reused by the next reduction
    return v;
}

// out = embed[token] as f32 (Qwen35Model::embed_token, src/transformer_qwen35.rs:1170-1181);
// tokpos = {token, position} of this step.
__global__ void q_embed_kernel(const uint16_t* __restrict__ embed, const int32_t* __restrict__ tokpos, int H,
                               float* __restrict__ x) {
    const int token = tokpos[0];
    for (int c = threadIdx.x; c < H; c += blockDim.x)
        x[c] = rt::bf16_bits_to_f32(embed[static_cast<int64_t>(token) * H + c]);
}

// x += add (if any); xn = x / sqrt(mean(x^2) + eps) * (1 + gamma)
// (RmsNorm2::forward_gemma3, the zero-centred variant the blocks use).
__global__ void __launch_bounds__(kQWide) q_resid_norm_kernel(float* __restrict__ x, const float* __restrict__ add,
                                                                 const float* __restrict__ gamma, float eps, int H,
                                                                 float* __restrict__ xn) {
    __shared__ float red[32];
    rt::pdl_launch_dependents();  // the next GEMV may start streaming its weights now
    float ss = 0.f;
    for (int c = threadIdx.x; c < H; c += blockDim.x) {
        float v = x[c];
        if (add) {
            v += add[c];
            x[c] = v;
        }
        ss += v * v;
    }
    ss = qblock_sum(ss, red);
    const float r = 1.0f / sqrtf(ss * (1.0f / static_cast<float>(H)) + eps);
    for (int c = threadIdx.x; c < H; c += blockDim.x) xn[c] = (x[c] * r) * (1.0f + gamma[c]);
}

// Causal depthwise conv1d + SiLU over the qkv channels, history shifted
// (Qwen35DeltaNet::apply_conv1d, src/transformer_qwen35.rs:589-617).
__global__ void q_dn_conv_kernel(const float* __restrict__ in, const float* __restrict__ w, float* __restrict__ state,
                                 int C, int KS, float* __restrict__ out) {
    const int hist = KS - 1;
    for (int c = blockIdx.x * blockDim.x + threadIdx.x; c < C; c += gridDim.x * blockDim.x) {
        const float* wc = w + static_cast<int64_t>(c) * KS;
        float* sc = state + static_cast<int64_t>(c) * hist;
        float v = 0.f;
        for (int t = 0; t < hist; ++t) v += wc[t] * sc[t];
        v += wc[hist] * in[c];
        out[c] = silu_f(v);
        for (int t = 0; t + 1 < hist; ++t) sc[t] = sc[t + 1];
        if (hist > 0) sc[hist - 1] = in[c];
    }
}

struct DnHeadArgs {
    const float* conv;   // [2 nk kd + nv vd]: q | k | v after the conv
    const float* zab;    // [nv vd + 2 nv]: z | a | b (the in-projection rows after qkv)
    const float* a_log;  // [nv]
    const float* dt_bias;
    const float* norm_w;  // [vd]
    float* S;             // [nv][kd][vd]
    float* out;           // [nv vd]
    int nk, nv, kd, vd;
};

// One CTA of kQWide threads per value head h (src/transformer_qwen35.rs:339-453).
// Thread t owns column j = t % vd of the head's state and rows i = p, p + P,
// ... (P = kQWide / vd row groups, p = t / vd), at most kDnMaxRows of them, in
// registers.
constexpr int kDnMaxRows = 16;

__global__ void __launch_bounds__(kQWide) q_dn_heads_kernel(const DnHeadArgs a) {
    __shared__ float red[32];
    rt::pdl_launch_dependents();
    __shared__ float qs[256], ks[256];  // this head's q (scaled) and k, kd <= 256
    __shared__ float part[kQWide];
    __shared__ float col[256];          // kv_mem, then the output column values
    const int h = blockIdx.x, t = threadIdx.x;
    const int kd = a.kd, vd = a.vd, P = kQWide / vd;
    const int g = h / (a.nv / a.nk);  // key head of this value head
    const float* q = a.conv + g * kd;
    const float* k = a.conv + a.nk * kd + g * kd;
    const float* v = a.conv + 2 * a.nk * kd + h * vd;
    // l2_normalize_heads (src/transformer_qwen35.rs:1756-1766), then q / sqrt(kd)
    float sq = 0.f, sk = 0.f;
    for (int i = t; i < kd; i += kQWide) {
        sq += q[i] * q[i];
        sk += k[i] * k[i];
    }
    sq = qblock_sum(sq, red);
    sk = qblock_sum(sk, red);
    const float nq = fmaxf(sqrtf(sq), 1e-12f), nk = fmaxf(sqrtf(sk), 1e-12f);
    const float qscale = 1.0f / sqrtf(static_cast<float>(kd));
    for (int i = t; i < kd; i += kQWide) {
        qs[i] = (q[i] / nq) * qscale;
        ks[i] = k[i] / nk;
    }
    // gates: beta = sigmoid(b), decay = exp(-exp(A_log) softplus(a + dt_bias))
    const float* z = a.zab + h * vd;
    const float av = a.zab[a.nv * vd + h], bv = a.zab[a.nv * vd + a.nv + h];
    const float beta = sigmoid_f(bv);
    const float decay = expf(-expf(a.a_log[h]) * softplus_f(av + a.dt_bias[h]));
    __syncthreads();
    const int j = t % vd, p = t / vd;
    const bool active = p < P;
    const int nr = active ? (kd - p + P - 1) / P : 0;  // rows i = p + P r, r < nr
    float* Sh = a.S + static_cast<int64_t>(h) * kd * vd;
    float s[kDnMaxRows];
#pragma unroll
    for (int r = 0; r < kDnMaxRows; ++r)
        if (r < nr) s[r] = Sh[static_cast<int64_t>(p + P * r) * vd + j] * decay;
    // kv_mem[j] = sum_i S[i][j] k[i]
    float acc = 0.f;
#pragma unroll
    for (int r = 0; r < kDnMaxRows; ++r)
        if (r < nr) acc += s[r] * ks[p + P * r];
    part[t] = acc;
    __syncthreads();
    if (t < vd) {
        float kv = 0.f;
        for (int pp = 0; pp < P; ++pp) kv += part[pp * vd + t];
        col[t] = kv;
    }
    __syncthreads();
    // delta = (v - kv_mem) beta;  S += k delta^T;  o[j] = sum_i S[i][j] q[i]
    const float delta = active ? (v[j] - col[j]) * beta : 0.f;
    acc = 0.f;
#pragma unroll
    for (int r = 0; r < kDnMaxRows; ++r)
        if (r < nr) {
            s[r] += ks[p + P * r] * delta;
            acc += s[r] * qs[p + P * r];
            Sh[static_cast<int64_t>(p + P * r) * vd + j] = s[r];
        }
    __syncthreads();  // every col[] read above is done
    part[t] = acc;
    __syncthreads();
    float o = 0.f;
    if (t < vd) {
        for (int pp = 0; pp < P; ++pp) o += part[pp * vd + t];
    }
    // gated RMSNorm over the head: o / rms * norm_weight * silu(z), eps 1e-6
    const float ss = qblock_sum(t < vd ? o * o : 0.f, red);
    const float rms = sqrtf(ss / static_cast<float>(vd) + 1e-6f);
    if (t < vd) a.out[h * vd + t] = ((o / rms) * a.norm_w[t]) * silu_f(z[t]);
}

struct FaArgs {
    const float* qkv;     // [nq (2 d) | nkv d | nkv d]: per head query then gate, then k, then v
    const float* q_norm;  // [d]
    const float* k_norm;
    const float* rope_cos;  // [max_tokens][rope_dim / 2]
    const float* rope_sin;
    float* kcache;  // [max_tokens][nkv][d]
    float* vcache;
    float* q_rot;   // [nq][d]
    float* out;     // [nq][d]
    const int32_t* tokpos;  // {token, position}: the position is read on the device
    int nq, nkv, d, rope_dim;
    float eps, scale;
};

// One CTA per head (nq query heads, then nkv key heads): per-head RMSNorm with
// (1 + gamma) (apply_per_head_norm_raw, src/transformer_qwen35.rs:1768-1781),
// partial RoPE on the first rope_dim dims, pairs (i, i + rope_dim / 2)
// (apply_partial_rope, :1783-1812); keys and values appended at pos.
__global__ void __launch_bounds__(kQThreads) q_fa_prep_kernel(const FaArgs a) {
    __shared__ float red[32];
    __shared__ float row[512];
    const int hd = blockIdx.x, t = threadIdx.x, d = a.d, pos = a.tokpos[1];
    const bool is_q = hd < a.nq;
    const int h = is_q ? hd : hd - a.nq;
    const float* src = is_q ? a.qkv + static_cast<int64_t>(h) * 2 * d : a.qkv + static_cast<int64_t>(a.nq) * 2 * d + h * d;
    const float* gm = is_q ? a.q_norm : a.k_norm;
    float ss = 0.f;
    for (int j = t; j < d; j += kQThreads) ss += src[j] * src[j];
    ss = qblock_sum(ss, red);
    const float rms = sqrtf(ss / static_cast<float>(d) + a.eps);
    for (int j = t; j < d; j += kQThreads) row[j] = (src[j] / rms) * (1.0f + gm[j]);
    __syncthreads();
    const int half = a.rope_dim / 2;
    float* dst = is_q ? a.q_rot + static_cast<int64_t>(h) * d
                      : a.kcache + (static_cast<int64_t>(pos) * a.nkv + h) * d;
    for (int j = t; j < d; j += kQThreads) {
        float v = row[j];
        if (j < half) {
            const float c = a.rope_cos[static_cast<int64_t>(pos) * half + j];
            const float s = a.rope_sin[static_cast<int64_t>(pos) * half + j];
            v = row[j] * c - row[j + half] * s;
        } else if (j < 2 * half) {
            const float c = a.rope_cos[static_cast<int64_t>(pos) * half + j - half];
            const float s = a.rope_sin[static_cast<int64_t>(pos) * half + j - half];
            v = row[j] * c + row[j - half] * s;
        }
        dst[j] = v;
    }
    if (!is_q) {
        const float* vs = a.qkv + static_cast<int64_t>(a.nq) * 2 * d + static_cast<int64_t>(a.nkv) * d + h * d;
        for (int j = t; j < d; j += kQThreads) a.vcache[(static_cast<int64_t>(pos) * a.nkv + h) * d + j] = vs[j];
    }
}

// One CTA per query head: softmax(q . K / sqrt(d)) over positions 0..pos, the
// weighted sum of V (gqa_attention_cached, src/transformer_qwen35.rs:1814-1869),
// times sigmoid(gate).  Scores live in dynamic shared memory (max_tokens floats).
__global__ void __launch_bounds__(kQThreads) q_fa_attn_kernel(const FaArgs a) {
    extern __shared__ float sc[];
    __shared__ float red[32];
    rt::pdl_launch_dependents();
    __shared__ float qv[512];
    const int h = blockIdx.x, t = threadIdx.x, lane = t & 31, warp = t >> 5, d = a.d;
    const int kvh = h / (a.nq / a.nkv), L = a.tokpos[1] + 1;
    for (int j = t; j < d; j += kQThreads) qv[j] = a.q_rot[static_cast<int64_t>(h) * d + j];
    __syncthreads();
    for (int p = warp; p < L; p += kQThreads / 32) {
        const float* kr = a.kcache + (static_cast<int64_t>(p) * a.nkv + kvh) * d;
        float dot = 0.f;
        for (int j = lane; j < d; j += 32) dot += qv[j] * kr[j];
        dot = rt::warp_sum(dot);
        if (lane == 0) sc[p] = dot * a.scale;
    }
    __syncthreads();
    float m = -INFINITY;
    for (int p = t; p < L; p += kQThreads) m = fmaxf(m, sc[p]);
    m = rt::block_max(m, red);
    __syncthreads();
    float sum = 0.f;
    for (int p = t; p < L; p += kQThreads) {
        const float e = expf(sc[p] - m);
        sc[p] = e;
        sum += e;
    }
    sum = qblock_sum(sum, red);
    const float inv = 1.0f / sum;
    for (int j = t; j < d; j += kQThreads) {
        float o = 0.f;
        for (int p = 0; p < L; ++p) o += (sc[p] * inv) * a.vcache[(static_cast<int64_t>(p) * a.nkv + kvh) * d + j];
        const float gate = a.qkv[static_cast<int64_t>(h) * 2 * d + d + j];
        a.out[static_cast<int64_t>(h) * d + j] = o * sigmoid_f(gate);
    }
}

// h[j] = silu(gate[j]) * up[j] from [gate (F) | up (F)] (Qwen35Mlp::forward, :864-869).
__global__ void q_silu_mul_kernel(const float* __restrict__ gu, int F, float* __restrict__ out) {
    rt::pdl_launch_dependents();
    for (int j = blockIdx.x * blockDim.x + threadIdx.x; j < F; j += gridDim.x * blockDim.x)
        out[j] = silu_f(gu[j]) * gu[F + j];
}

// A Q4_K projection of the engine: rows stacked from one or more source
// matrices, with its GEMV plan and tensor map.
struct QProj {
    void* d = nullptr;
    int64_t rows = 0;
    int K = 0;
    rt::GemvPlan plan;
    CUtensorMap tmap;
};

}  // namespace

struct rt_qwen35 {
    rt_ctx* ctx = nullptr;
    rt_qwen35_cfg cfg{};
    int max_tokens = 0;
    int H = 0, qkv_dim = 0, value_dim = 0, nl = 0;
    std::vector<void*> allocs;
    struct Layer {
        bool full = false;
        QProj in, out, gu, down;  // in: [qkv | z | a | b] or [q, gate | k | v]; out: out_proj or o_proj
        float *in_norm = nullptr, *post_norm = nullptr;
        float *conv_w = nullptr, *a_log = nullptr, *dt_bias = nullptr, *norm_w = nullptr;  // DeltaNet
        float *S = nullptr, *conv_state = nullptr;
        float *q_norm = nullptr, *k_norm = nullptr;  // full attention
        float *kcache = nullptr, *vcache = nullptr;
    };
    std::vector<Layer> layers;
    float* final_norm = nullptr;
    const uint16_t* embed = nullptr;  // the caller's BF16 [vocab, hidden] rt_w (kept alive by the caller)
    rt::GemvPlan lm_plan;
    CUtensorMap lm_tmap;
    float *rope_cos = nullptr, *rope_sin = nullptr;
    // activations
    float *x = nullptr, *xn = nullptr, *y = nullptr, *big = nullptr, *conv = nullptr, *mix = nullptr, *q_rot = nullptr,
          *hbuf = nullptr, *logits = nullptr;
    float* part = nullptr;  // LM head split-tile scratch
    uint32_t* cnt = nullptr;
    // One step as a CUDA graph (captured at the first step); the token and the
    // position reach it through tokpos, copied in from pinned h_tokpos.
    int32_t* tokpos = nullptr;
    int32_t* h_tokpos = nullptr;
    cudaGraph_t graph = nullptr;
    cudaGraphExec_t exec = nullptr;
};

namespace {

int qalloc(rt_qwen35* e, void** p, size_t bytes, const char* what) {
    int rc = rt::dev_alloc(e->ctx, p, bytes, what);
    if (rc == RT_OK) e->allocs.push_back(*p);
    return rc;
}

int upload_f32(rt_qwen35* e, float** dst, const float* src, size_t n, const char* what) {
    if (!src) return fail(e->ctx, RT_E_INVAL, "rt_qwen35_create: missing %s", what);
    int rc = qalloc(e, reinterpret_cast<void**>(dst), n * 4, what);
    if (rc != RT_OK) return rc;
    if (cudaMemcpy(*dst, src, n * 4, cudaMemcpyHostToDevice) != cudaSuccess)
        return fail(e->ctx, RT_E_CUDA, "rt_qwen35_create: upload %s", what);
    return RT_OK;
}

// Stack Q4_K matrices with K columns row-wise into one projection.
int make_proj(rt_qwen35* e, QProj* p, std::initializer_list<std::pair<const rt_w*, int64_t>> parts, int K,
              const char* what) {
    int64_t rows = 0;
    for (const auto& pr : parts) {
        const rt_w* w = pr.first;
        if (!w || w->fmt != RT_FMT_Q4K || w->cols != K || w->rows != pr.second)
            return fail(e->ctx, RT_E_SHAPE, "rt_qwen35_create: %s: expected Q4_K [%lld, %d]", what,
                        static_cast<long long>(pr.second), K);
        rows += w->rows;
    }
    const uint64_t row_bytes = static_cast<uint64_t>(K / 256) * 144;
    int rc = qalloc(e, &p->d, rows * row_bytes, what);
    if (rc != RT_OK) return rc;
    uint64_t off = 0;
    for (const auto& pr : parts) {
        if (cudaMemcpy(static_cast<uint8_t*>(p->d) + off, pr.first->d, pr.first->rows * row_bytes,
                       cudaMemcpyDeviceToDevice) != cudaSuccess)
            return fail(e->ctx, RT_E_CUDA, "rt_qwen35_create: copy %s", what);
        off += pr.first->rows * row_bytes;
    }
    p->rows = rows;
    p->K = K;
    p->plan = rt::gemv_cluster_plan(rows, K, e->ctx->num_sms);
    if (p->plan.warps == 0) return fail(e->ctx, RT_E_SHAPE, "rt_qwen35_create: %s: no GEMV geometry", what);
    if (!rt::gemv_make_tmap(rt::kQ4K, p->d, rows, K, p->plan, &p->tmap))
        return fail(e->ctx, RT_E_CUDA, "rt_qwen35_create: %s: TMA descriptor rejected", what);
    return RT_OK;
}

cudaError_t gemv(rt_qwen35* e, const QProj& p, const float* x, float* y) {
    rt::GemvArgs a = {};
    a.w = static_cast<const uint8_t*>(p.d);
    a.rows = p.rows;
    a.K = p.K;
    a.x = x;
    a.y = y;
    a.err = e->ctx->d_err;
    // programmatic dependent launch: the GEMV's CTAs start, and copy their
    // weights, while the kernel before it (which triggers at entry) runs; they
    // read its output only after griddepcontrol.wait
    return rt::gemv_cluster_launch(a, p.tmap, p.plan, e->ctx->stream, true);
}

}  // namespace

namespace {

// Enqueue one step (every kernel of it) on the context stream; the caller
// captures it into the engine's graph.
cudaError_t enqueue_step(rt_qwen35* e) {
#define QCHECK(call)                      \
    do {                                  \
        const cudaError_t r_ = (call);    \
        if (r_ != cudaSuccess) return r_; \
    } while (0)
    const rt_qwen35_cfg& c = e->cfg;
    cudaStream_t s = e->ctx->stream;
    const int H = e->H, nv = c.linear_num_value_heads, nq = c.num_attention_heads, D = c.head_dim;
    const int F = c.intermediate_size;
    q_embed_kernel<<<1, kQThreads, 0, s>>>(e->embed, e->tokpos, H, e->x);
    QCHECK(cudaGetLastError());
    const float* add = nullptr;  // the previous block's MLP output, added before the next norm
    for (int l = 0; l < e->nl; ++l) {
        rt_qwen35::Layer& L = e->layers[l];
        q_resid_norm_kernel<<<1, kQWide, 0, s>>>(e->x, add, L.in_norm, c.rms_norm_eps, H, e->xn);
        QCHECK(gemv(e, L.in, e->xn, e->big));
        if (!L.full) {
            q_dn_conv_kernel<<<(e->qkv_dim + 255) / 256, 256, 0, s>>>(e->big, L.conv_w, L.conv_state, e->qkv_dim,
                                                                       c.linear_conv_kernel_dim, e->conv);
            DnHeadArgs a;
            a.conv = e->conv;
            a.zab = e->big + e->qkv_dim;
            a.a_log = L.a_log;
            a.dt_bias = L.dt_bias;
            a.norm_w = L.norm_w;
            a.S = L.S;
            a.out = e->mix;
            a.nk = c.linear_num_key_heads;
            a.nv = nv;
            a.kd = c.linear_key_head_dim;
            a.vd = c.linear_value_head_dim;
            q_dn_heads_kernel<<<nv, kQWide, 0, s>>>(a);
        } else {
            FaArgs a;
            a.qkv = e->big;
            a.q_norm = L.q_norm;
            a.k_norm = L.k_norm;
            a.rope_cos = e->rope_cos;
            a.rope_sin = e->rope_sin;
            a.kcache = L.kcache;
            a.vcache = L.vcache;
            a.q_rot = e->q_rot;
            a.out = e->mix;
            a.nq = nq;
            a.nkv = c.num_key_value_heads;
            a.d = D;
            a.rope_dim = c.rope_dim;
            a.tokpos = e->tokpos;
            a.eps = c.rms_norm_eps;
            a.scale = 1.0f / sqrtf(static_cast<float>(D));
            q_fa_prep_kernel<<<nq + a.nkv, kQThreads, 0, s>>>(a);
            q_fa_attn_kernel<<<nq, kQThreads, sizeof(float) * e->max_tokens, s>>>(a);
        }
        QCHECK(cudaGetLastError());
        QCHECK(gemv(e, L.out, e->mix, e->y));
        q_resid_norm_kernel<<<1, kQWide, 0, s>>>(e->x, e->y, L.post_norm, c.rms_norm_eps, H, e->xn);
        QCHECK(gemv(e, L.gu, e->xn, e->big));
        q_silu_mul_kernel<<<(F + 255) / 256, 256, 0, s>>>(e->big, F, e->hbuf);
        QCHECK(cudaGetLastError());
        QCHECK(gemv(e, L.down, e->hbuf, e->y));
        add = e->y;
    }
    q_resid_norm_kernel<<<1, kQWide, 0, s>>>(e->x, add, e->final_norm, c.rms_norm_eps, H, e->xn);
    QCHECK(cudaGetLastError());
    rt::GemvArgs a = {};
    a.w = reinterpret_cast<const uint8_t*>(e->embed);
    a.rows = c.vocab_size;
    a.K = H;
    a.x = e->xn;
    a.y = e->logits;
    a.part = e->part;
    a.tile_cnt = e->cnt;
    a.err = e->ctx->d_err;
    QCHECK(rt::gemv_launch(rt::kBF16, rt::kProPlain, rt::kEpiPlain, a, e->lm_tmap, e->lm_plan, s, true));
    return cudaSuccess;
#undef QCHECK
}

}  // namespace

extern "C" {

int rt_qwen35_create(rt_ctx* ctx, const rt_qwen35_cfg* cfg, const rt_qwen35_layer* layers, const rt_w* embed,
                     const float* final_norm, int32_t max_tokens, rt_qwen35** out) {
    if (!ctx || !cfg || !layers || !embed || !final_norm || !out) return fail(ctx, RT_E_INVAL, "rt_qwen35_create: null argument");
    *out = nullptr;
    const rt_qwen35_cfg& c = *cfg;
    const int H = c.hidden_size, nk = c.linear_num_key_heads, nv = c.linear_num_value_heads;
    const int kd = c.linear_key_head_dim, vd = c.linear_value_head_dim, KS = c.linear_conv_kernel_dim;
    const int nq = c.num_attention_heads, nkv = c.num_key_value_heads, D = c.head_dim, F = c.intermediate_size;
    if (H <= 0 || H % 256 || F % 256 || c.num_hidden_layers <= 0 || nk <= 0 || nv % nk || kd > 256 || vd <= 0 ||
        vd > 256 || kQWide % vd || kd > kDnMaxRows * (kQWide / vd) || KS < 1 || nq <= 0 || nkv <= 0 || nq % nkv || D > 512 ||
        (nq * D) % 256 || (nv * vd) % 256 || c.rope_dim % 2 || c.rope_dim > D || c.full_attention_interval <= 0 ||
        max_tokens <= 0 || max_tokens > 40000 || c.vocab_size <= 0)
        return fail(ctx, RT_E_SHAPE, "rt_qwen35_create: unsupported configuration");
    if (embed->fmt != RT_FMT_BF16 || embed->rows != c.vocab_size || embed->cols != H)
        return fail(ctx, RT_E_SHAPE, "rt_qwen35_create: embed must be BF16 [vocab, hidden]");
    RT_CHECK_CUDA(ctx, cudaSetDevice(ctx->device));
    rt_qwen35* e = new rt_qwen35();
    e->ctx = ctx;
    e->cfg = c;
    e->max_tokens = max_tokens;
    e->H = H;
    e->nl = c.num_hidden_layers;
    e->qkv_dim = 2 * nk * kd + nv * vd;
    e->value_dim = nv * vd;
    auto bail = [&](int rc) {
        rt_qwen35_destroy(e);
        return rc;
    };
    int rc = RT_OK;
    e->layers.resize(e->nl);
    size_t big = static_cast<size_t>(2) * F;
    for (int l = 0; l < e->nl; ++l) {
        const rt_qwen35_layer& L = layers[l];
        rt_qwen35::Layer& E = e->layers[l];
        E.full = (l + 1) % c.full_attention_interval == 0;  // ConfigQwen35::is_full_attention_layer
        if ((rc = upload_f32(e, &E.in_norm, L.input_norm, H, "input_norm")) != RT_OK ||
            (rc = upload_f32(e, &E.post_norm, L.post_attn_norm, H, "post_attn_norm")) != RT_OK ||
            (rc = make_proj(e, &E.gu, {{L.gate, F}, {L.up, F}}, H, "gate/up")) != RT_OK ||
            (rc = make_proj(e, &E.down, {{L.down, H}}, F, "down")) != RT_OK)
            return bail(rc);
        if (E.full) {
            if ((rc = make_proj(e, &E.in, {{L.q, 2LL * nq * D}, {L.k, static_cast<int64_t>(nkv) * D}, {L.v, static_cast<int64_t>(nkv) * D}},
                                H, "q/k/v")) != RT_OK ||
                (rc = make_proj(e, &E.out, {{L.o, H}}, nq * D, "o")) != RT_OK ||
                (rc = upload_f32(e, &E.q_norm, L.q_norm, D, "q_norm")) != RT_OK ||
                (rc = upload_f32(e, &E.k_norm, L.k_norm, D, "k_norm")) != RT_OK ||
                (rc = qalloc(e, reinterpret_cast<void**>(&E.kcache), sizeof(float) * max_tokens * nkv * D, "k cache")) != RT_OK ||
                (rc = qalloc(e, reinterpret_cast<void**>(&E.vcache), sizeof(float) * max_tokens * nkv * D, "v cache")) != RT_OK)
                return bail(rc);
            big = std::max(big, static_cast<size_t>(2) * nq * D + 2 * nkv * D);
        } else {
            if ((rc = make_proj(e, &E.in, {{L.in_qkv, e->qkv_dim}, {L.in_z, e->value_dim}, {L.in_a, nv}, {L.in_b, nv}}, H,
                                "DeltaNet in-projections")) != RT_OK ||
                (rc = make_proj(e, &E.out, {{L.out_proj, H}}, e->value_dim, "out_proj")) != RT_OK ||
                (rc = upload_f32(e, &E.conv_w, L.conv1d_weight, static_cast<size_t>(e->qkv_dim) * KS, "conv1d_weight")) != RT_OK ||
                (rc = upload_f32(e, &E.a_log, L.a_log, nv, "a_log")) != RT_OK ||
                (rc = upload_f32(e, &E.dt_bias, L.dt_bias, nv, "dt_bias")) != RT_OK ||
                (rc = upload_f32(e, &E.norm_w, L.norm_weight, vd, "norm_weight")) != RT_OK ||
                (rc = qalloc(e, reinterpret_cast<void**>(&E.S), sizeof(float) * nv * kd * vd, "DeltaNet state")) != RT_OK ||
                (rc = qalloc(e, reinterpret_cast<void**>(&E.conv_state), sizeof(float) * e->qkv_dim * std::max(1, KS - 1),
                             "conv1d state")) != RT_OK)
                return bail(rc);
            big = std::max(big, static_cast<size_t>(e->qkv_dim) + e->value_dim + 2 * nv);
        }
    }
    if ((rc = upload_f32(e, &e->final_norm, final_norm, H, "final_norm")) != RT_OK) return bail(rc);
    e->embed = static_cast<const uint16_t*>(embed->d);
    e->lm_plan = rt::gemv_plan(rt::kBF16, c.vocab_size, H, 1, rt::kProPlain, rt::kEpiPlain, ctx->num_sms, 1);
    if (e->lm_plan.warps == 0 || !rt::gemv_make_tmap(rt::kBF16, embed->d, c.vocab_size, H, e->lm_plan, &e->lm_tmap))
        return bail(fail(ctx, RT_E_SHAPE, "rt_qwen35_create: no LM-head GEMV"));
    // RoPE tables in f32 as apply_partial_rope forms them: freq = 1 / theta^(2i / rope_dim), angle = pos * freq
    const int half = c.rope_dim / 2;
    std::vector<float> hc(static_cast<size_t>(max_tokens) * std::max(1, half)), hs(hc.size());
    for (int p = 0; p < max_tokens; ++p)
        for (int i = 0; i < half; ++i) {
            const float freq = 1.0f / std::pow(c.rope_theta, 2.0f * static_cast<float>(i) / static_cast<float>(c.rope_dim));
            const float ang = static_cast<float>(p) * freq;
            hc[static_cast<size_t>(p) * half + i] = std::cos(ang);
            hs[static_cast<size_t>(p) * half + i] = std::sin(ang);
        }
    const size_t act = static_cast<size_t>(std::max<int64_t>({H, F, e->value_dim, static_cast<int64_t>(nq) * D}));
    if ((rc = upload_f32(e, &e->rope_cos, hc.data(), hc.size(), "rope cos")) != RT_OK ||
        (rc = upload_f32(e, &e->rope_sin, hs.data(), hs.size(), "rope sin")) != RT_OK ||
        (rc = qalloc(e, reinterpret_cast<void**>(&e->x), sizeof(float) * H, "residual")) != RT_OK ||
        (rc = qalloc(e, reinterpret_cast<void**>(&e->xn), sizeof(float) * H, "normed")) != RT_OK ||
        (rc = qalloc(e, reinterpret_cast<void**>(&e->y), sizeof(float) * H, "block output")) != RT_OK ||
        (rc = qalloc(e, reinterpret_cast<void**>(&e->big), sizeof(float) * big, "projection output")) != RT_OK ||
        (rc = qalloc(e, reinterpret_cast<void**>(&e->conv), sizeof(float) * e->qkv_dim, "conv output")) != RT_OK ||
        (rc = qalloc(e, reinterpret_cast<void**>(&e->mix), sizeof(float) * act, "mixer output")) != RT_OK ||
        (rc = qalloc(e, reinterpret_cast<void**>(&e->q_rot), sizeof(float) * nq * D, "rotated queries")) != RT_OK ||
        (rc = qalloc(e, reinterpret_cast<void**>(&e->hbuf), sizeof(float) * F, "MLP hidden")) != RT_OK ||
        (rc = qalloc(e, reinterpret_cast<void**>(&e->logits), sizeof(float) * c.vocab_size, "logits")) != RT_OK ||
        (rc = qalloc(e, reinterpret_cast<void**>(&e->tokpos), 2 * sizeof(int32_t), "token and position")) != RT_OK ||
        (rc = qalloc(e, reinterpret_cast<void**>(&e->part), sizeof(float) * std::max<int64_t>(1, e->lm_plan.part_floats),
                     "LM-head scratch")) != RT_OK ||
        (rc = qalloc(e, reinterpret_cast<void**>(&e->cnt), sizeof(uint32_t) * std::max<int64_t>(1, e->lm_plan.cnt_words),
                     "LM-head counters")) != RT_OK)
        return bail(rc);
    if (cudaMemset(e->cnt, 0, sizeof(uint32_t) * std::max<int64_t>(1, e->lm_plan.cnt_words)) != cudaSuccess ||
        cudaFuncSetAttribute(q_fa_attn_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, 160 * 1024) != cudaSuccess)
        return bail(fail(ctx, RT_E_CUDA, "rt_qwen35_create: set-up"));
    if (cudaMallocHost(reinterpret_cast<void**>(&e->h_tokpos), 2 * sizeof(int32_t)) != cudaSuccess)
        return bail(fail(ctx, RT_E_NOMEM, "rt_qwen35_create: pinned token buffer"));
    if ((rc = rt_qwen35_reset(e)) != RT_OK) return bail(rc);
    *out = e;
    return RT_OK;
}

void rt_qwen35_destroy(rt_qwen35* e) {
    if (!e) return;
    if (e->exec) cudaGraphExecDestroy(e->exec);
    if (e->graph) cudaGraphDestroy(e->graph);
    if (e->h_tokpos) cudaFreeHost(e->h_tokpos);
    for (void* p : e->allocs) cudaFree(p);
    delete e;
}

int rt_qwen35_reset(rt_qwen35* e) {
    if (!e) return RT_E_INVAL;
    rt_ctx* ctx = e->ctx;
    RT_CHECK_CUDA(ctx, cudaSetDevice(ctx->device));
    const rt_qwen35_cfg& c = e->cfg;
    for (auto& L : e->layers) {
        if (L.full) continue;
        RT_CHECK_CUDA(ctx, cudaMemsetAsync(L.S, 0,
                                           sizeof(float) * c.linear_num_value_heads * c.linear_key_head_dim *
                                               c.linear_value_head_dim,
                                           ctx->stream));
        RT_CHECK_CUDA(ctx, cudaMemsetAsync(L.conv_state, 0,
                                           sizeof(float) * e->qkv_dim * std::max(1, c.linear_conv_kernel_dim - 1),
                                           ctx->stream));
    }
    return rt_sync(ctx);
}

int rt_qwen35_step(rt_qwen35* e, int32_t token, int32_t position, float* logits) {
    if (!e) return RT_E_INVAL;
    rt_ctx* ctx = e->ctx;
    const rt_qwen35_cfg& c = e->cfg;
    if (token < 0 || token >= c.vocab_size) return fail(ctx, RT_E_INVAL, "rt_qwen35_step: token %d", token);
    if (position < 0 || position >= e->max_tokens)
        return fail(ctx, RT_E_STATE, "rt_qwen35_step: position %d outside the %d-token cache", position, e->max_tokens);
    RT_CHECK_CUDA(ctx, cudaSetDevice(ctx->device));
    cudaStream_t s = ctx->stream;
    e->h_tokpos[0] = token;
    e->h_tokpos[1] = position;
    RT_CHECK_CUDA(ctx, cudaMemcpyAsync(e->tokpos, e->h_tokpos, 2 * sizeof(int32_t), cudaMemcpyHostToDevice, s));
    if (!e->exec) {
        RT_CHECK_CUDA(ctx, cudaStreamBeginCapture(s, cudaStreamCaptureModeThreadLocal));
        const cudaError_t ce = enqueue_step(e);
        cudaGraph_t g = nullptr;
        const cudaError_t ee = cudaStreamEndCapture(s, &g);
        if (ce != cudaSuccess || ee != cudaSuccess || !g) {
            if (g) cudaGraphDestroy(g);
            cudaGetLastError();
            return fail(ctx, RT_E_CUDA, "rt_qwen35_step: capture: %s", cudaGetErrorString(ce != cudaSuccess ? ce : ee));
        }
        e->graph = g;
        RT_CHECK_CUDA(ctx, cudaGraphInstantiate(&e->exec, g, 0));
    }
    RT_CHECK_CUDA(ctx, cudaGraphLaunch(e->exec, s));
    if (logits)
        RT_CHECK_CUDA(ctx, cudaMemcpyAsync(logits, e->logits, sizeof(float) * c.vocab_size, cudaMemcpyDeviceToHost, s));
    return rt_sync(ctx);  // also keeps h_tokpos untouched until its copy is done
}

int rt_qwen35_logits_device(rt_qwen35* e, const float** out) {
    if (!e || !out) return RT_E_INVAL;
    *out = e->logits;
    return RT_OK;
}

}  // extern "C"
