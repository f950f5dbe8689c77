// attention.cu -- fused per-head QK-norm + NeoX RoPE + KV append + split-context
// flash-decode attention for one query token (Gemma 3, GQA), sm_100a.
//
// Reference semantics (paths relative to the reference crate root):
//   apply_per_head_norm      src/transformer4.rs:2485-2510 (rms_norm_gemma3 per head)
//   apply_rope_at_offset     src/transformer4.rs:2742-2772 (pairs (i, i + D/2))
//   Gemma3LayerKvCache::append + window selection  src/transformer4.rs:1813-1823, 1923-1929
//   gqa_attention_cached (t_q == 1)  src/transformer4.rs:2806-2880
//
// Grid (nsplit, nkv).  CTA (s, h) takes the s-th slice of the attended
// positions [k_start, pos] of KV head h and all G query heads that share it.
// Cached positions (< pos) do not depend on this step, so the CTA starts their
// TMA bulk copy into shared memory before griddepcontrol.wait.  The CTA whose
// slice contains `pos` normalises and rotates the new K row, appends K and V to
// the cache and uses them from shared memory.  Each CTA keeps an online
// softmax (max m, sum l, unnormalised output) per query head and writes it to
// `part`; the last CTA of each KV head (atomic counter, no waiting) merges the
// slices.  RoPE cos/sin come from host-built tables that evaluate the
// reference formula with the host libm, so the rotation matches it exactly.
#include <algorithm>

#include "attention.cuh"
#include "common.cuh"

namespace rt {

namespace {

struct AttnSmem {
    uint64_t* bar;
    float* red;    // [32]
    float* m_run;  // [G]
    float* l_run;  // [G]
    float* corr;   // [G]
    int* flag;     // [4]
    float* qv;     // [G][D]
    float* sc;     // [G][kAttnTile]
    float* knew;   // [D]
    float* vnew;   // [D]
    float* kt;     // [kAttnTile][D]
    float* vt;     // [kAttnTile][D]
};

__host__ __device__ inline size_t attn_carve(uint8_t* base, int D, int G, AttnSmem* S) {
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
    uint8_t* sc = take(static_cast<size_t>(G) * kAttnTile * 4, 16);
    uint8_t* kn = take(static_cast<size_t>(D) * 4, 16);
    uint8_t* vn = take(static_cast<size_t>(D) * 4, 16);
    uint8_t* kt = take(static_cast<size_t>(kAttnTile) * D * 4, 128);
    uint8_t* vt = take(static_cast<size_t>(kAttnTile) * D * 4, 128);
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

// In-place per-head RMSNorm (1 + gamma) of `v[D]` in shared memory.
__device__ __forceinline__ void head_norm(float* v, const float* gamma, int D, float eps, float* red) {
    float ss = 0.f;
    for (int d = threadIdx.x; d < D; d += blockDim.x) ss += v[d] * v[d];
    ss = block_sum(ss, red);
    const float r = 1.0f / sqrtf(ss * (1.0f / static_cast<float>(D)) + eps);
    for (int d = threadIdx.x; d < D; d += blockDim.x) v[d] = __fmul_rn(__fmul_rn(v[d], r), __fadd_rn(1.0f, gamma[d]));
    __syncthreads();
}

// In-place NeoX rotation of `v[D]`: (x0, x1) = (v[j], v[j + D/2]).
__device__ __forceinline__ void head_rope(float* v, const float* cs, const float* sn, int D) {
    const int half = D / 2;
    for (int j = threadIdx.x; j < half; j += blockDim.x) {
        const float x0 = v[j], x1 = v[j + half], c = cs[j], s = sn[j];
        v[j] = __fsub_rn(__fmul_rn(x0, c), __fmul_rn(x1, s));
        v[j + half] = __fadd_rn(__fmul_rn(x0, s), __fmul_rn(x1, c));
    }
    __syncthreads();
}

template <int G>
__device__ __forceinline__ void attend_tile(const AttnSmem& S, const float* K, const float* V, int nt, int D,
                                            float scale, float (&acc)[G]) {
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5, nw = blockDim.x >> 5;
    for (int j = warp; j < nt; j += nw) {
        const float* kr = K + static_cast<size_t>(j) * D;
#pragma unroll
        for (int g = 0; g < G; ++g) {
            const float* q = S.qv + g * D;
            float dot = 0.f;
            for (int d = lane; d < D; d += 32) dot += q[d] * kr[d];
            dot = warp_sum(dot);
            if (lane == 0) S.sc[g * kAttnTile + j] = dot * scale;
        }
    }
    __syncthreads();
    if (warp == 0) {
#pragma unroll
        for (int g = 0; g < G; ++g) {
            const float v = lane < nt ? S.sc[g * kAttnTile + lane] : -INFINITY;
            const float tmax = warp_max(v);
            const float mold = S.m_run[g];
            const float mnew = fmaxf(mold, tmax);
            const float p = lane < nt ? expf(v - mnew) : 0.f;
            const float psum = warp_sum(p);
            S.sc[g * kAttnTile + lane] = p;
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
            const float* p = S.sc + g * kAttnTile;
            for (int j = 0; j < nt; ++j) v += p[j] * V[static_cast<size_t>(j) * D + tid];
            acc[g] = v;
        }
    }
    __syncthreads();
}

template <int G>
__global__ void __launch_bounds__(kAttnThreads) attention_kernel(const AttnArgs a) {
    extern __shared__ __align__(128) uint8_t smem[];
    AttnSmem S;
    attn_carve(smem, a.D, G, &S);
    const int D = a.D;
    const int h = blockIdx.y, s = blockIdx.x;
    const int tid = threadIdx.x;

    // Attended positions (window selection, src/transformer4.rs:1923-1929).
    const int pos = *a.pos;
    const int L = pos + 1;
    const int kstart = a.window > 0 ? max(0, L - a.window) : 0;
    const int n = L - kstart;
    const int chunk = (n + a.nsplit - 1) / a.nsplit;
    const int p0 = min(L, kstart + s * chunk);
    const int p1 = min(L, p0 + chunk);
    const bool has_new = p0 <= pos && pos < p1;
    const int ncached = max(0, (has_new ? pos : p1) - p0);
    const int ntiles = (ncached + kAttnTile - 1) / kAttnTile;
    const size_t head_base = static_cast<size_t>(h) * a.cap;

    auto issue = [&](int t) {
        const int r0 = p0 + t * kAttnTile;
        const int nt = min(kAttnTile, p0 + ncached - r0);
        const uint32_t bytes = static_cast<uint32_t>(nt) * D * 4;
        mbar_arrive_expect_tx(S.bar, 2 * bytes);
        bulk_g2s_nohint(S.kt, a.kcache + (head_base + r0) * D, bytes, S.bar);
        bulk_g2s_nohint(S.vt, a.vcache + (head_base + r0) * D, bytes, S.bar);
    };
    if (tid == 0) {
        mbar_init(S.bar, 1);
        fence_mbar_init();
    }
    __syncthreads();
    if (tid == 0 && ntiles > 0) issue(0);  // cached K/V: independent of this step
    pdl_launch_dependents();
    pdl_wait();

    // Query heads h*G .. h*G+G-1 (kvh = qh / group, src/transformer4.rs:2819).
    const float* qraw = a.qkv + static_cast<size_t>(h) * G * D;
    for (int i = tid; i < G * D; i += blockDim.x) S.qv[i] = qraw[i];
    if (tid < G) {
        S.m_run[tid] = -INFINITY;
        S.l_run[tid] = 0.f;
    }
    __syncthreads();
    const float* cs = a.rope_cos + static_cast<size_t>(pos) * (D / 2);
    const float* sn = a.rope_sin + static_cast<size_t>(pos) * (D / 2);
#pragma unroll
    for (int g = 0; g < G; ++g) {
        head_norm(S.qv + g * D, a.q_norm, D, a.eps, S.red);
        head_rope(S.qv + g * D, cs, sn, D);
    }
    if (has_new) {
        const float* kraw = a.qkv + static_cast<size_t>(a.nq) * D + static_cast<size_t>(h) * D;
        const float* vraw = a.qkv + static_cast<size_t>(a.nq + a.nkv) * D + static_cast<size_t>(h) * D;
        for (int d = tid; d < D; d += blockDim.x) {
            S.knew[d] = kraw[d];
            S.vnew[d] = vraw[d];
        }
        __syncthreads();
        head_norm(S.knew, a.k_norm, D, a.eps, S.red);
        head_rope(S.knew, cs, sn, D);
        float* kdst = a.kcache + (head_base + pos) * D;
        float* vdst = a.vcache + (head_base + pos) * D;
        for (int d = tid; d < D; d += blockDim.x) {
            kdst[d] = S.knew[d];
            vdst[d] = S.vnew[d];
        }
    }

    float acc[G];
#pragma unroll
    for (int g = 0; g < G; ++g) acc[g] = 0.f;
    bool timed_out = false;
    int t_fail = 0;
    for (int t = 0; t < ntiles; ++t) {
        const bool ok = mbar_wait(S.bar, static_cast<uint32_t>(t) & 1u);
        if (__syncthreads_or(!ok)) {
            timed_out = true;
            t_fail = t;
            break;
        }
        const int nt = min(kAttnTile, ncached - t * kAttnTile);
        attend_tile<G>(S, S.kt, S.vt, nt, D, a.scale, acc);
        if (tid == 0 && t + 1 < ntiles) issue(t + 1);
    }
    if (timed_out) {
        if (tid == 0) {
            if (a.err) atomicExch(a.err, kErrMbarTimeout);
            // the one outstanding copy must land (bounded) before shared memory goes
            (void)mbar_wait(S.bar, static_cast<uint32_t>(t_fail) & 1u);
        }
        __syncthreads();
        return;
    }
    if (has_new) attend_tile<G>(S, S.knew, S.vnew, 1, D, a.scale, acc);

    // Per-split partial state.
    const int stride = D + 2;
#pragma unroll
    for (int g = 0; g < G; ++g) {
        float* pp = a.part + (static_cast<size_t>(h * a.nsplit + s) * G + g) * stride;
        if (tid < D) pp[tid] = acc[g];
        if (tid == 0) {
            pp[D] = S.m_run[g];
            pp[D + 1] = S.l_run[g];
        }
    }
    __threadfence();
    __syncthreads();
    if (tid == 0) {
        const uint32_t prev = atomicAdd(&a.counter[h], 1u);
        S.flag[0] = prev == static_cast<uint32_t>(a.nsplit - 1);
    }
    __syncthreads();
    if (!S.flag[0]) return;
    __threadfence();
    if (tid < D) {
#pragma unroll
        for (int g = 0; g < G; ++g) {
            float M = -INFINITY;
            for (int q = 0; q < a.nsplit; ++q) {
                const float* pp = a.part + (static_cast<size_t>(h * a.nsplit + q) * G + g) * stride;
                M = fmaxf(M, __ldcg(pp + D));
            }
            float num = 0.f, den = 0.f;
            for (int q = 0; q < a.nsplit; ++q) {
                const float* pp = a.part + (static_cast<size_t>(h * a.nsplit + q) * G + g) * stride;
                const float w = expf(__ldcg(pp + D) - M);
                den += w * __ldcg(pp + D + 1);
                num += w * __ldcg(pp + tid);
            }
            a.out[static_cast<size_t>(h * G + g) * D + tid] = num / den;
        }
    }
    if (tid == 0) a.counter[h] = 0u;
}

template <int G>
cudaError_t launch_g(const AttnArgs& a, cudaStream_t s, bool pdl) {
    return rt_launch(attention_kernel<G>, dim3(a.nsplit, a.nkv), dim3(kAttnThreads), attention_smem_bytes(a.D, G), s,
                     pdl, a);
}

}  // namespace

size_t attention_smem_bytes(int D, int G) { return attn_carve(nullptr, D, G, nullptr) + 128; }

cudaError_t attention_prepare() {
    // Raise the dynamic shared-memory limit once, outside any stream capture.
    cudaError_t e = cudaFuncSetAttribute(attention_kernel<1>, cudaFuncAttributeMaxDynamicSharedMemorySize, 200 * 1024);
    if (e == cudaSuccess) e = cudaFuncSetAttribute(attention_kernel<2>, cudaFuncAttributeMaxDynamicSharedMemorySize, 200 * 1024);
    if (e == cudaSuccess) e = cudaFuncSetAttribute(attention_kernel<4>, cudaFuncAttributeMaxDynamicSharedMemorySize, 200 * 1024);
    if (e == cudaSuccess) e = cudaFuncSetAttribute(attention_kernel<8>, cudaFuncAttributeMaxDynamicSharedMemorySize, 200 * 1024);
    return e;
}

cudaError_t attention_launch(const AttnArgs& a, cudaStream_t s, bool pdl) {
    if (a.D > kAttnThreads || a.D % 32 != 0 || a.nq % a.nkv != 0) return cudaErrorInvalidValue;
    switch (a.nq / a.nkv) {
        case 1: return launch_g<1>(a, s, pdl);
        case 2: return launch_g<2>(a, s, pdl);
        case 4: return launch_g<4>(a, s, pdl);
        case 8: return launch_g<8>(a, s, pdl);
        default: return cudaErrorInvalidValue;
    }
}

uint64_t attention_algorithmic_bytes(int nq, int nkv, int D, int64_t L) {
    // K and V rows read (the new row is written once and read from registers),
    // plus q/k/v in and the output.
    return static_cast<uint64_t>(2) * nkv * D * 4 * static_cast<uint64_t>(L) +
           static_cast<uint64_t>(nq + 2 * nkv) * D * 4 + static_cast<uint64_t>(nq) * D * 4;
}

}  // namespace rt
