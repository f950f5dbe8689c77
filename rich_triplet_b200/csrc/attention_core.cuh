// attention_core.cuh -- device side of the fused per-head QK-norm + NeoX RoPE +
// KV append + split-context flash-decode attention for one query token
// (Gemma 3, GQA), shared by the standalone attention kernel (attention.cu) and
// the persistent decode-step kernel (step.cu).
//
// Reference semantics (paths relative to the reference crate root):
//   apply_per_head_norm      src/transformer4.rs:2485-2510 (rms_norm_gemma3 per head)
//   apply_rope_at_offset     src/transformer4.rs:2742-2772 (pairs (i, i + D/2))
//   Gemma3LayerKvCache::append + window selection  src/transformer4.rs:1813-1823, 1923-1929
//   gqa_attention_cached (t_q == 1)  src/transformer4.rs:2806-2880
//
// Work item (h, s): the s-th slice of the attended positions [k_start, pos] of
// KV head h, for all G query heads that share it.  Cached positions (< pos) do
// not depend on this step, so their first tile can be copied into shared
// memory (TMA bulk copy) before the projections of this step exist.  The item
// whose slice contains `pos` normalises and rotates the new K row, appends K
// and V to the cache and uses them from shared memory.  Each item keeps an
// online softmax (max m, sum l, unnormalised output) per query head and writes
// it to `part`; the last item of each KV head to finish (atomic counter, no
// waiting) merges the slices.  RoPE cos/sin come from host-built tables that
// evaluate the reference formula with the host libm, so the rotation matches
// it exactly.  All threads of the CTA take part (any multiple of 32 >= D).
#pragma once

#include "attention.cuh"
#include "common.cuh"

namespace rt {
namespace acore {

constexpr int kMaxHeadDim = 256;  // the decoder accepts head_dim <= 256, a multiple of 32

struct AttnSmem {
    uint64_t* bar;
    float* red;    // [32]
    float* m_run;  // [G]
    float* l_run;  // [G]
    float* corr;   // [G]
    int* flag;     // [4]
    float* qv;     // [G][D]
    float* sc;     // [G][T]
    float* knew;   // [D]
    float* vnew;   // [D]
    float* kt;     // [T][D]
    float* vt;     // [T][D]
};

// Shared-memory layout for G query heads per KV head and tiles of T positions.
__host__ __device__ inline size_t attn_carve(uint8_t* base, int D, int G, int T, AttnSmem* S) {
    size_t off = 0;
    auto take = [&](size_t bytes, size_t align) -> uint8_t* {
        off = (off + align - 1) / align * align;
        uint8_t* p = base + off;
        off += bytes;
        return p;
    };
    uint8_t* bar = take(16, 16);
    uint8_t* red = take(32 * 4, 16);
    uint8_t* m = take(G * 4, 16);
    uint8_t* l = take(G * 4, 16);
    uint8_t* cr = take(G * 4, 16);
    uint8_t* fl = take(16, 16);
    uint8_t* qv = take(static_cast<size_t>(G) * D * 4, 16);
    uint8_t* sc = take(static_cast<size_t>(G) * T * 4, 16);
    uint8_t* kn = take(static_cast<size_t>(D) * 4, 16);
    uint8_t* vn = take(static_cast<size_t>(D) * 4, 16);
    // K and V tiles, one region (after the tile loop it holds the warps'
    // partial outputs while they are combined)
    uint8_t* kt = take(2 * static_cast<size_t>(T) * D * 4, 128);
    uint8_t* vt = kt + static_cast<size_t>(T) * D * 4;
    if (S) {
        S->bar = reinterpret_cast<uint64_t*>(bar);
        S->red = reinterpret_cast<float*>(red);
        S->m_run = reinterpret_cast<float*>(m);
        S->l_run = reinterpret_cast<float*>(l);
        S->corr = reinterpret_cast<float*>(cr);
        S->flag = reinterpret_cast<int*>(fl);
        S->qv = reinterpret_cast<float*>(qv);
        S->sc = reinterpret_cast<float*>(sc);
        S->knew = reinterpret_cast<float*>(kn);
        S->vnew = reinterpret_cast<float*>(vn);
        S->kt = reinterpret_cast<float*>(kt);
        S->vt = reinterpret_cast<float*>(vt);
    }
    return off;
}

// One warp: dst[D] = rope(rmsnorm(raw) * (1 + gamma)) -- the per-head norm
// (rms_norm_gemma3 per head, src/transformer4.rs:2485-2510) and the NeoX
// rotation of pairs (j, j + D/2) (src/transformer4.rs:2742-2772).
// LL: the row is read from tagged words at raw_ll (polled until every word
// carries `tag`); false if that wait gave up.  Otherwise from raw.
template <bool LL>
__device__ __forceinline__ bool head_load_warp(const float* raw, const uint64_t* raw_ll, uint32_t tag, int D,
                                               const int* abort, float (&x)[kMaxHeadDim / 32]) {
    constexpr int kMaxPer = kMaxHeadDim / 32;
    const int lane = threadIdx.x & 31;
    if constexpr (!LL) {
#pragma unroll
        for (int i = 0; i < kMaxPer; ++i) {  // every load of the row in flight at once
            const int j = lane + 32 * i;
            x[i] = j < D ? raw[j] : 0.f;
        }
        return true;
    }
    LLPoll pl;
    pl.init(abort);
    for (;;) {
        bool ready = true;
#pragma unroll
        for (int i = 0; i < kMaxPer; ++i) {
            const int j = lane + 32 * i;
            const uint64_t w = j < D ? ll_load(raw_ll + j) : ll_word(0.f, tag);
            x[i] = ll_val(w);
            ready &= ll_has(w, tag);
        }
        if (__all_sync(0xffffffffu, ready)) return true;
        if (!pl.again()) return false;
    }
}

template <bool LL>
__device__ __forceinline__ bool head_prep_warp(const float* raw, const uint64_t* raw_ll, uint32_t tag,
                                               const float* gamma, const float* cs, const float* sn, int D, float eps,
                                               float* dst, const int* abort) {
    constexpr int kMaxPer = kMaxHeadDim / 32;
    const int lane = threadIdx.x & 31, half = D / 2;
    float x[kMaxPer];
    float ss = 0.f;
    if (!head_load_warp<LL>(raw, raw_ll, tag, D, abort, x)) return false;
#pragma unroll
    for (int i = 0; i < kMaxPer; ++i) {
        const int j = lane + 32 * i;
        if (j < D) dst[j] = x[i];
        ss += x[i] * x[i];
    }
    ss = warp_sum(ss);
    __syncwarp();  // the row is in dst for the pairs other lanes own
    const float r = 1.0f / sqrtf(ss * (1.0f / static_cast<float>(D)) + eps);
    #pragma unroll 1
    for (int j = lane; j < half; j += 32) {
        const float x0 = __fmul_rn(__fmul_rn(dst[j], r), __fadd_rn(1.0f, gamma[j]));
        const float x1 = __fmul_rn(__fmul_rn(dst[j + half], r), __fadd_rn(1.0f, gamma[j + half]));
        const float c = cs[j], s = sn[j];
        dst[j] = __fsub_rn(__fmul_rn(x0, c), __fmul_rn(x1, s));
        dst[j + half] = __fadd_rn(__fmul_rn(x0, s), __fmul_rn(x1, c));
    }
    return true;
}

template <int G, int T>
__device__ __forceinline__ void attend_tile(const AttnSmem& S, const float* K, const float* V, int nt, int D,
                                            float scale, float (&acc)[G]) {
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5, nw = blockDim.x >> 5;
    #pragma unroll 1
    for (int j = warp; j < nt; j += nw) {
        const float* kr = K + static_cast<size_t>(j) * D;
#pragma unroll
        for (int g = 0; g < G; ++g) {
            const float* q = S.qv + g * D;
            float dot = 0.f;
            #pragma unroll 1
            for (int d = lane; d < D; d += 32) dot += q[d] * kr[d];
            dot = warp_sum(dot);
            if (lane == 0) S.sc[g * T + j] = dot * scale;
        }
    }
    __syncthreads();
    if (warp == 0) {
#pragma unroll
        for (int g = 0; g < G; ++g) {
            const float v = lane < nt ? S.sc[g * T + lane] : -INFINITY;
            const float tmax = warp_max(v);
            const float mold = S.m_run[g];
            const float mnew = fmaxf(mold, tmax);
            const float p = lane < nt ? expf(v - mnew) : 0.f;
            const float psum = warp_sum(p);
            if (lane < T) S.sc[g * T + lane] = p;
            __syncwarp();
            if (lane == 0) {
                const float cr = expf(mold - mnew);
                S.corr[g] = cr;
                S.l_run[g] = S.l_run[g] * cr + psum;
                S.m_run[g] = mnew;
            }
            __syncwarp();
        }
    }
    __syncthreads();
    if (tid < D) {
#pragma unroll
        for (int g = 0; g < G; ++g) {
            float v = acc[g] * S.corr[g];
            const float* p = S.sc + g * T;
            #pragma unroll 2
            for (int j = 0; j < nt; ++j) v += p[j] * V[static_cast<size_t>(j) * D + tid];
            acc[g] = v;
        }
    }
    __syncthreads();
}

// Positions per split below which the context uses fewer splits: the merge
// reads every split's partial, so splits cost more than they save when short.
constexpr int kMinPerSplit = 16;

// Attended positions of item (h, s) (window selection, src/transformer4.rs:1923-1929).
struct AttnRange {
    int pos;
    int nsplit;   // splits in use at this context length (<= a.nsplit)
    bool active;  // s < nsplit
    int p0;
    int ncached;  // cached positions of the slice (excluding the new one)
    int ntiles;
    bool has_new;
    size_t head_base;
};

__device__ __forceinline__ AttnRange attn_range(const AttnArgs& a, int h, int s, int T, int pos = -1) {
    AttnRange R;
    R.pos = pos >= 0 ? pos : *a.pos;
    const int L = R.pos + 1;
    const int kstart = a.window > 0 ? max(0, L - a.window) : 0;
    const int n = L - kstart;
    R.nsplit = max(1, min(a.nsplit, (n + kMinPerSplit - 1) / kMinPerSplit));
    R.active = s < R.nsplit;
    const int chunk = (n + R.nsplit - 1) / R.nsplit;
    R.p0 = min(L, kstart + s * chunk);
    const int p1 = min(L, R.p0 + chunk);
    R.has_new = R.p0 <= R.pos && R.pos < p1;
    R.ncached = max(0, (R.has_new ? R.pos : p1) - R.p0);
    R.ntiles = (R.ncached + T - 1) / T;
    R.head_base = static_cast<size_t>(h) * a.cap;
    return R;
}

// Thread 0: copy cached tile t of the item into shared memory, completing on S.bar.
__device__ __forceinline__ void attn_issue(const AttnArgs& a, const AttnRange& R, const AttnSmem& S, int t, int T) {
    const int r0 = R.p0 + t * T;
    const int nt = min(T, R.p0 + R.ncached - r0);
    const uint32_t bytes = static_cast<uint32_t>(nt) * a.D * 4;
    mbar_arrive_expect_tx(S.bar, 2 * bytes);
    bulk_g2s_nohint(S.kt, a.kcache + (R.head_base + r0) * a.D, bytes, S.bar);
    bulk_g2s_nohint(S.vt, a.vcache + (R.head_base + r0) * a.D, bytes, S.bar);
}

// exp(mx - m) for the rescaling of a partial state whose running max is mx
// (an empty state, mx = -inf, weighs 0).
__device__ __forceinline__ float lse_scale(float mx, float m) { return mx == -INFINITY ? 0.f : expf(mx - m); }

// Merge of the nsplit partial states of KV head h (the CTA that finished last;
// all threads).  Per query head: M = max m_q, w_q = exp(m_q - M),
// out = sum w_q acc_q / sum w_q l_q.  Thread (c, k), k = tid % kg, takes
// float4 column c of the G*D outputs and splits k, k + kg, ... (kBatch loads
// in flight, running max rescaled per batch); the kg states of a column sit
// in adjacent lanes and are combined by a butterfly, so every load of the
// merge is issued in one round for nsplit <= kg * kBatch.
template <int G>
__device__ __forceinline__ void attn_merge(const AttnArgs& a, int h, int nsplit, uint32_t out_tag) {
    constexpr int kBatch = 12;
    const int D = a.D, stride = attn_part_stride(D);
    const int Q = G * D / 4;  // float4 columns
    int kg = 1;
    while (kg < 32 && 2 * kg * Q <= static_cast<int>(blockDim.x)) kg *= 2;
    const int tid = threadIdx.x, per_pass = static_cast<int>(blockDim.x) / kg;
    const int k = tid % kg;
    for (int c0 = 0; c0 < Q; c0 += per_pass) {
        const int c = c0 + tid / kg;
        const bool col = c < Q;
        const int g = col ? 4 * c / D : 0, d = col ? 4 * c - g * D : 0;
        const float* base = a.part + (static_cast<size_t>(h) * a.nsplit * G + g) * stride;
        float M = -INFINITY, den = 0.f;
        float4 num = make_float4(0.f, 0.f, 0.f, 0.f);
        for (int q0 = k; col && q0 < nsplit; q0 += kg * kBatch) {
            float2 ml[kBatch];
            float4 v[kBatch];
#pragma unroll
            for (int i = 0; i < kBatch; ++i) {
                const int q = q0 + i * kg;
                if (q < nsplit) {
                    const float* row = base + static_cast<size_t>(q) * G * stride;
                    ml[i] = __ldcg(reinterpret_cast<const float2*>(row + D));
                    v[i] = __ldcg(reinterpret_cast<const float4*>(row + d));
                } else {
                    ml[i] = make_float2(-INFINITY, 0.f);
                    v[i] = make_float4(0.f, 0.f, 0.f, 0.f);
                }
            }
            float bm = M;
#pragma unroll
            for (int i = 0; i < kBatch; ++i) bm = fmaxf(bm, ml[i].x);
            const float cr = lse_scale(M, bm);
            den *= cr;
            num.x *= cr;
            num.y *= cr;
            num.z *= cr;
            num.w *= cr;
#pragma unroll
            for (int i = 0; i < kBatch; ++i) {
                const float w = lse_scale(ml[i].x, bm);
                den += w * ml[i].y;
                num.x += w * v[i].x;
                num.y += w * v[i].y;
                num.z += w * v[i].z;
                num.w += w * v[i].w;
            }
            M = bm;
        }
        // Butterfly over the kg lanes of column c (aligned groups of a warp).
        #pragma unroll 1
        for (int o = 1; o < kg; o <<= 1) {
            const float oM = __shfl_xor_sync(0xffffffffu, M, o);
            const float oden = __shfl_xor_sync(0xffffffffu, den, o);
            float4 on;
            on.x = __shfl_xor_sync(0xffffffffu, num.x, o);
            on.y = __shfl_xor_sync(0xffffffffu, num.y, o);
            on.z = __shfl_xor_sync(0xffffffffu, num.z, o);
            on.w = __shfl_xor_sync(0xffffffffu, num.w, o);
            const float nm = fmaxf(M, oM);
            const float sa = lse_scale(M, nm), sb = lse_scale(oM, nm);
            den = den * sa + oden * sb;
            num.x = num.x * sa + on.x * sb;
            num.y = num.y * sa + on.y * sb;
            num.z = num.z * sa + on.z * sb;
            num.w = num.w * sa + on.w * sb;
            M = nm;
        }
        if (col && k == 0) {
            const size_t o = static_cast<size_t>(h * G + g) * D + d;
            if (out_tag) {
                ll_store2(a.out_ll + o, num.x / den, num.y / den, out_tag);
                ll_store2(a.out_ll + o + 2, num.z / den, num.w / den, out_tag);
            } else {
                *reinterpret_cast<float4*>(a.out + o) = make_float4(num.x / den, num.y / den, num.z / den, num.w / den);
            }
        }
    }
}

// Merge of KV head h's partials, spread over the head's active items: item s
// of ns takes the float4 quads [s Q / ns, (s+1) Q / ns) of the G*D outputs
// (Q = G*D/4), one warp per quad.  Lane j polls splits j and j + 32 (ns <= 64):
// their outputs at the quad and their (m, l), published by the items as
// tagged words (part_tag); it merges its splits online, and a butterfly over
// the warp combines the lanes in a fixed order.  The quad's four outputs go
// to a.out_ll as tagged words (out_tag).  Each item reads about ns * 48 bytes
// per quad, instead of one CTA reading every split's partial.  False (on
// every thread) if a poll gave up.
template <int G>
__device__ __forceinline__ bool attn_merge_slice_ll(const AttnArgs& a, int h, int s, int ns, uint32_t part_tag,
                                                    uint32_t out_tag, const int* abort) {
    const int D = a.D, stride = attn_part_stride(D);
    const int Q = G * D / 4;
    const int q0 = s * Q / ns, q1 = (s + 1) * Q / ns;
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nw = blockDim.x >> 5;
    bool ok = true;
    #pragma unroll 1
    for (int qd = q0 + warp; qd < q1 && ok; qd += nw) {
        const int g = 4 * qd / D, d = 4 * qd - g * D;
        const uint64_t* base = a.part_ll + (static_cast<size_t>(h) * a.nsplit * G + g) * stride;
        ulonglong2 w[2][3];
        LLPoll pl;
        pl.init(abort);
        for (;;) {
            bool ready = true;
#pragma unroll
            for (int i = 0; i < 2; ++i) {
                const int q = lane + 32 * i;
                if (q < ns) {
                    const uint64_t* row = base + static_cast<size_t>(q) * G * stride;
                    w[i][0] = ll_load2(row + d);
                    w[i][1] = ll_load2(row + d + 2);
                    w[i][2] = ll_load2(row + D);
#pragma unroll
                    for (int k = 0; k < 3; ++k) ready &= ll_has(w[i][k].x, part_tag) && ll_has(w[i][k].y, part_tag);
                }
            }
            if (__all_sync(0xffffffffu, ready)) break;
            if (!pl.again()) {
                ok = false;
                break;
            }
        }
        if (!__all_sync(0xffffffffu, ok)) {
            ok = false;
            break;
        }
        float M = -INFINITY, den = 0.f;
        float4 num = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
        for (int i = 0; i < 2; ++i) {
            if (lane + 32 * i >= ns) continue;
            const float m = ll_val(w[i][2].x), l = ll_val(w[i][2].y);
            const float nm = fmaxf(M, m);
            const float sa = lse_scale(M, nm), sb = lse_scale(m, nm);
            den = den * sa + l * sb;
            num.x = num.x * sa + ll_val(w[i][0].x) * sb;
            num.y = num.y * sa + ll_val(w[i][0].y) * sb;
            num.z = num.z * sa + ll_val(w[i][1].x) * sb;
            num.w = num.w * sa + ll_val(w[i][1].y) * sb;
            M = nm;
        }
        #pragma unroll 1
        for (int o = 1; o < 32; o <<= 1) {
            const float oM = __shfl_xor_sync(0xffffffffu, M, o);
            const float oden = __shfl_xor_sync(0xffffffffu, den, o);
            float4 on;
            on.x = __shfl_xor_sync(0xffffffffu, num.x, o);
            on.y = __shfl_xor_sync(0xffffffffu, num.y, o);
            on.z = __shfl_xor_sync(0xffffffffu, num.z, o);
            on.w = __shfl_xor_sync(0xffffffffu, num.w, o);
            const float nm = fmaxf(M, oM);
            const float sa = lse_scale(M, nm), sb = lse_scale(oM, nm);
            den = den * sa + oden * sb;
            num.x = num.x * sa + on.x * sb;
            num.y = num.y * sa + on.y * sb;
            num.z = num.z * sa + on.z * sb;
            num.w = num.w * sa + on.w * sb;
            M = nm;
        }
        if (lane == 0) {
            uint64_t* out = a.out_ll + static_cast<size_t>(h * G + g) * D + d;
            ll_store2(out, num.x / den, num.y / den, out_tag);
            ll_store2(out + 2, num.z / den, num.w / den, out_tag);
        }
    }
    return !__syncthreads_or(!ok);
}

// Thread 0: initialise the tile barrier.  An initialised mbarrier owns its 8
// bytes until it is invalidated: ordinary stores to them are undefined (on
// B200 they do not stick), so the barrier must not live in memory that other
// phases of the same kernel reuse.
__device__ __forceinline__ void attn_bar_init(const AttnSmem& S) {
    mbar_init(S.bar, 1);
    fence_mbar_init();
}

// Thread 0, before the projections of this step exist: start the first cached
// tile (S.bar initialised; its next phase is the one attn_run waits on first).
__device__ __forceinline__ void attn_prefetch(const AttnArgs& a, const AttnRange& R, const AttnSmem& S, int T) {
    fence_proxy_async_smem();  // the region may have been written by ordinary stores before
    if (R.active && R.ntiles > 0) attn_issue(a, R, S, 0, T);
}

// The item itself (all threads).  LL (decode-step kernel): q/k/v of this step
// come from the tagged words a.qkv_ll (polled until they carry in_tag), the
// item publishes its partial as tagged words (a.part_ll, part_tag) and then
// merges its slice of the head's outputs (attn_merge_slice_ll) into a.out_ll
// (out_tag).  Otherwise q/k/v come from a.qkv and the last item of the head to
// finish (atomic counter) merges every split into a.out.  `ph0`: parity of the
// tile barrier's next phase (phases it completed before, mod 2); the item
// completes R.ntiles phases.  Returns false if a bounded wait gave up (after
// waiting, bounded, for the copy in flight); `a.err` is then set.
template <int G, int T, bool LL>
__device__ __forceinline__ bool attn_run(const AttnArgs& a, int h, int s, const AttnRange& R, const AttnSmem& S,
                                         uint32_t ph0, uint32_t in_tag = 0, uint32_t out_tag = 0,
                                         const int* abort = nullptr, uint32_t part_tag = 0) {
    if (!R.active) return true;
    const int D = a.D;
    const int tid = threadIdx.x;
    // Query heads h*G .. h*G+G-1 (kvh = qh / group, src/transformer4.rs:2819):
    // warp g < G prepares query head g, warp G the new K row, warp G + 1
    // copies the new V row.
    const float* cs = a.rope_cos + static_cast<size_t>(R.pos) * (D / 2);
    const float* sn = a.rope_sin + static_cast<size_t>(R.pos) * (D / 2);
    const int warp = tid >> 5;
    bool got = true;
    if (warp < G || (warp == G && R.has_new)) {
        // one call site for the query heads and the new K row (smaller code)
        const bool qh = warp < G;
        const size_t o = static_cast<size_t>(qh ? h * G + warp : a.nq + h) * D;
        got = head_prep_warp<LL>(a.qkv + o, a.qkv_ll + o, in_tag, qh ? a.q_norm : a.k_norm, cs, sn, D, a.eps,
                                 qh ? S.qv + warp * D : S.knew, abort);
    } else if (warp == G + 1 && R.has_new) {
        const size_t o = static_cast<size_t>(a.nq + a.nkv + h) * D;
        float v[kMaxHeadDim / 32];
        got = head_load_warp<LL>(a.qkv + o, a.qkv_ll + o, in_tag, D, abort, v);
#pragma unroll
        for (int i = 0; i < kMaxHeadDim / 32; ++i) {
            const int d = (tid & 31) + 32 * i;
            if (d < D) S.vnew[d] = v[i];
        }
    }
    if (tid < G) {
        S.m_run[tid] = -INFINITY;
        S.l_run[tid] = 0.f;
    }
    if (__syncthreads_or(!got)) {
        // the inputs never came: the prefetched tile must still land (bounded)
        // before this shared memory is reused
        if (tid == 0) {
            if (a.err) atomicExch(a.err, kErrGridTimeout);
            if (R.ntiles > 0) (void)mbar_wait(S.bar, ph0 & 1u);
        }
        __syncthreads();
        return false;
    }
    if (R.has_new) {
        float* kdst = a.kcache + (R.head_base + R.pos) * D;
        float* vdst = a.vcache + (R.head_base + R.pos) * D;
        #pragma unroll 1
        for (int d = tid; d < D; d += blockDim.x) {
            kdst[d] = S.knew[d];
            vdst[d] = S.vnew[d];
        }
    }

    // Per-warp online softmax.  Lane l owns the float4 columns c = l + 32 f
    // (dims 4c..4c+3) of every row, so each warp-wide float4 load of a row
    // reads 512 contiguous bytes; warp w takes positions w, w + nw, ... of each
    // tile, and one warp the new row.  Every warp keeps its own running max,
    // sum and output per query head, with no block-wide step per position; the
    // warps' states are combined once at the end.
    constexpr int kNF = kMaxHeadDim / 128;
    const int lane = tid & 31, nw = static_cast<int>(blockDim.x >> 5);
    const int nc4 = D / 4;
    float4 q4[G][kNF];
#pragma unroll
    for (int g = 0; g < G; ++g)
#pragma unroll
        for (int f = 0; f < kNF; ++f) {
            const int c = lane + 32 * f;
            q4[g][f] = c < nc4 ? reinterpret_cast<const float4*>(S.qv + g * D)[c] : make_float4(0.f, 0.f, 0.f, 0.f);
        }
    float m[G], l[G];
    float4 acc[G][kNF];
#pragma unroll
    for (int g = 0; g < G; ++g) {
        m[g] = -INFINITY;
        l[g] = 0.f;
#pragma unroll
        for (int f = 0; f < kNF; ++f) acc[g][f] = make_float4(0.f, 0.f, 0.f, 0.f);
    }
    // One position: scores q . k * scale, then the online update with v.
    auto visit = [&](const float* kr, const float* vr) {
        float4 k4[kNF], v4[kNF];
#pragma unroll
        for (int f = 0; f < kNF; ++f) {
            const int c = lane + 32 * f;
            k4[f] = c < nc4 ? reinterpret_cast<const float4*>(kr)[c] : make_float4(0.f, 0.f, 0.f, 0.f);
            v4[f] = c < nc4 ? reinterpret_cast<const float4*>(vr)[c] : make_float4(0.f, 0.f, 0.f, 0.f);
        }
        float sc[G];
#pragma unroll
        for (int g = 0; g < G; ++g) {
            float d = 0.f;
#pragma unroll
            for (int f = 0; f < kNF; ++f)
                d += q4[g][f].x * k4[f].x + q4[g][f].y * k4[f].y + q4[g][f].z * k4[f].z + q4[g][f].w * k4[f].w;
            sc[g] = d;
        }
#pragma unroll
        for (int o = 16; o > 0; o >>= 1)
#pragma unroll
            for (int g = 0; g < G; ++g) sc[g] += __shfl_xor_sync(0xffffffffu, sc[g], o);
#pragma unroll
        for (int g = 0; g < G; ++g) {
            const float x = sc[g] * a.scale;
            const float mn = fmaxf(m[g], x);
            const float cr = expf(m[g] - mn);  // 0 for the first position (m = -inf)
            const float p = expf(x - mn);
            l[g] = l[g] * cr + p;
#pragma unroll
            for (int f = 0; f < kNF; ++f) {
                acc[g][f].x = acc[g][f].x * cr + p * v4[f].x;
                acc[g][f].y = acc[g][f].y * cr + p * v4[f].y;
                acc[g][f].z = acc[g][f].z * cr + p * v4[f].z;
                acc[g][f].w = acc[g][f].w * cr + p * v4[f].w;
            }
            m[g] = mn;
        }
    };
#pragma unroll 1
    for (int t = 0; t < R.ntiles; ++t) {
        const bool ok = mbar_wait(S.bar, (ph0 + static_cast<uint32_t>(t)) & 1u);
        if (__syncthreads_or(!ok)) {
            if (tid == 0) {
                if (a.err) atomicExch(a.err, kErrMbarTimeout);
                // the one outstanding copy must land (bounded) before shared memory is reused
                (void)mbar_wait(S.bar, (ph0 + static_cast<uint32_t>(t)) & 1u);
            }
            __syncthreads();
            return false;
        }
        const int nt = min(T, R.ncached - t * T);
#pragma unroll 1
        for (int j = warp; j < nt; j += nw) visit(S.kt + static_cast<size_t>(j) * D, S.vt + static_cast<size_t>(j) * D);
        __syncthreads();  // every warp is done with the tile before the next copy overwrites it
        if (tid == 0 && t + 1 < R.ntiles) {
            fence_proxy_async_smem();
            attn_issue(a, R, S, t + 1, T);
        }
    }
    if (R.has_new && warp == R.ncached % nw) visit(S.knew, S.vnew);
    // Every warp has read q from S.qv (which the states below overwrite) and
    // finished its positions; with no cached tile there was no barrier yet.
    __syncthreads();

    // Combine the warps' states.  Per query head g: M = max_w m_w, weight
    // e_w = exp(m_w - M), l = sum_w e_w l_w, output = sum_w e_w acc_w (the
    // item's partial: unnormalised output, M, l).  S.qv (q is in registers now)
    // holds the warps' m and l, S.sc the weights; the K/V tile region holds
    // the warps' outputs, gpp query heads per pass.
    float* wm = S.qv;
    float* wl = S.qv + nw * G;
    if (lane == 0) {
#pragma unroll
        for (int g = 0; g < G; ++g) {
            wm[warp * G + g] = m[g];
            wl[warp * G + g] = l[g];
        }
    }
    __syncthreads();
    if (warp < G) {
        const float mv = lane < nw ? wm[lane * G + warp] : -INFINITY;
        const float M = warp_max(mv);
        const float e = lane < nw && mv != -INFINITY ? expf(mv - M) : 0.f;
        const float den = warp_sum(lane < nw ? e * wl[lane * G + warp] : 0.f);
        if (lane < nw) S.sc[lane * G + warp] = e;
        if (lane == 0) {
            S.m_run[warp] = M;
            S.l_run[warp] = den;
        }
    }
    const int stride = attn_part_stride(D);
    const int gpp = max(1, 2 * T / nw);  // query heads per pass: nw * gpp * D floats fit the tile region
    float4* wacc = reinterpret_cast<float4*>(S.kt);
#pragma unroll 1
    for (int g0 = 0; g0 < G; g0 += gpp) {
        __syncthreads();  // the region's previous users (tile loop, previous pass) are done
#pragma unroll
        for (int g = 0; g < G; ++g) {
            if (g < g0 || g >= g0 + gpp) continue;
#pragma unroll
            for (int f = 0; f < kNF; ++f) {
                const int c = lane + 32 * f;
                if (c < nc4) wacc[(warp * gpp + (g - g0)) * nc4 + c] = acc[g][f];
            }
        }
        __syncthreads();
#pragma unroll 1
        for (int k = tid; k < gpp * nc4; k += blockDim.x) {
            const int gg = k / nc4, c = k - gg * nc4, g = g0 + gg;
            if (g >= G) continue;
            float4 o = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll 4
            for (int w = 0; w < nw; ++w) {
                const float e = S.sc[w * G + g];
                const float4 v = wacc[(w * gpp + gg) * nc4 + c];
                o.x += e * v.x;
                o.y += e * v.y;
                o.z += e * v.z;
                o.w += e * v.w;
            }
            const size_t row = (static_cast<size_t>(h * a.nsplit + s) * G + g) * stride;
            if constexpr (LL) {
                ll_store2(a.part_ll + row + 4 * c, o.x, o.y, part_tag);
                ll_store2(a.part_ll + row + 4 * c + 2, o.z, o.w, part_tag);
                if (c == 0) ll_store2(a.part_ll + row + D, S.m_run[g], S.l_run[g], part_tag);
            } else {
                *reinterpret_cast<float4*>(a.part + row + 4 * c) = o;
                if (c == 0) {
                    a.part[row + D] = S.m_run[g];
                    a.part[row + D + 1] = S.l_run[g];
                }
            }
        }
    }
    if constexpr (LL) {
        return attn_merge_slice_ll<G>(a, h, s, R.nsplit, part_tag, out_tag, abort);
    } else {
        __threadfence();
        __syncthreads();
        if (tid == 0) {
            const uint32_t prev = atomicAdd(&a.counter[h], 1u);
            S.flag[0] = prev == static_cast<uint32_t>(R.nsplit - 1);
        }
        __syncthreads();
        if (!S.flag[0]) return true;
        __threadfence();
        // The counter is reset before the merged output is published: a later
        // layer's items of this head (which can only start after consumers saw the
        // output) must find it at zero.
        if (tid == 0) {
            a.counter[h] = 0u;
            __threadfence();
        }
        __syncthreads();
        attn_merge<G>(a, h, R.nsplit, out_tag);
        return true;
    }
}

}  // namespace acore
}  // namespace rt
