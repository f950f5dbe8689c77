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
#include "attention_core.cuh"
#include "common.cuh"

namespace rt {

namespace {

using namespace acore;

// Grid (nsplit, nkv, sequences): CTA (s, h, b) runs item (h, s) of sequence b.
template <int G>
__global__ void __launch_bounds__(kAttnThreads) attention_kernel(const AttnArgs a0) {
    // Each of sequence b's pointers is formed from the parameter itself.  (A
    // conditional in-place update of the copy, `if (b) a.qkv += ...`, built
    // with nvcc 12.9 -O3, left a.qkv at sequence 0's rows while the other
    // members moved: every plane then attended with sequence 0's q/k/v.)
    AttnArgs a = a0;
    const int64_t b = blockIdx.z;
    a.qkv = a0.qkv + b * a0.seq_qkv;
    a.kcache = a0.kcache + b * a0.seq_kv;
    a.vcache = a0.vcache + b * a0.seq_kv;
    a.part = a0.part + b * a0.seq_part;
    a.out = a0.out + b * a0.seq_out;
    a.pos = a0.pos + b;
    a.counter = a0.counter + b * a0.nkv;
    extern __shared__ __align__(128) uint8_t smem[];
    AttnSmem S;
    attn_carve(smem, a.D, G, kAttnTile, &S);
    const int h = blockIdx.y, s = blockIdx.x;
    const AttnRange R = attn_range(a, h, s, kAttnTile);
    if (threadIdx.x == 0) {
        attn_bar_init(S);
        attn_prefetch(a, R, S, kAttnTile);  // cached K/V: independent of this step
    }
    __syncthreads();
    pdl_launch_dependents();
    pdl_wait();
    (void)attn_run<G, kAttnTile, false>(a, h, s, R, S, 0u);
}

template <int G>
cudaError_t launch_g(const AttnArgs& a, cudaStream_t s, bool pdl, int nseq = 1) {
    return rt_launch(attention_kernel<G>, dim3(a.nsplit, a.nkv, nseq), dim3(kAttnThreads), attention_smem_bytes(a.D, G), s,
                     pdl, a);
}

}  // namespace

size_t attention_smem_bytes(int D, int G) { return attn_carve(nullptr, D, G, kAttnTile, nullptr) + 128; }

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

cudaError_t attention_launch_batch(const AttnArgs& a, int nseq, cudaStream_t s) {
    if (a.D > kAttnThreads || a.D % 32 != 0 || a.nq % a.nkv != 0 || nseq < 1 || nseq > 65535) return cudaErrorInvalidValue;
    switch (a.nq / a.nkv) {
        case 1: return launch_g<1>(a, s, false, nseq);
        case 2: return launch_g<2>(a, s, false, nseq);
        case 4: return launch_g<4>(a, s, false, nseq);
        case 8: return launch_g<8>(a, s, false, nseq);
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
