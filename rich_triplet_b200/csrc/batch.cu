// batch.cu -- many-sequence Gemma 3 decode: one step
// advances B independent sequences, each with its own KV cache and position.
//
// The reference decodes one sequence at a time (MetalDecodeContext::
// decode_step, src/metal_decode.rs:2028-2074; its decode_step_batch,
// :2079-2579, batches the positions of ONE sequence).  Per step here, the
// weights are read once for all B sequences: every projection is the tcgen05
// GEMM with M = B (gemm.cu), fp16 activations (each row scaled by a power of
// two into fp16's range, undone on the f32 product) and f32 accumulation,
// split across K when B alone leaves SMs idle.  Per layer l:
//   rows    residual += post-FFN-norm(down_{l-1}) (embedding * sqrt(H) at l = 0);
//           x = RMSNorm(residual) -> fp16                      (Gemma3Block, src/transformer4.rs:1954-1964)
//   GEMM    qkv = x . Wqkv^T
//   attn    per sequence: q/k norm + RoPE and KV append; then per (sequence,
//           KV head, 256-position chunk) flash decode (attn_batch.cu)
//   GEMM    o = fp16(attn) . Wo^T
//   rows    residual += post-attn-norm(o); x = pre-FFN RMSNorm -> fp16
//   GEMM    gu = x . Wgu^T  (gate/up rows interleaved)
//   rows    h = gelu_tanh(gate) * up -> fp16
//   GEMM    down = h . Wdown^T
// then the final norm, the LM head as a GEMM over the tied bf16
// embedding, and a per-sequence greedy argmax (ties to the higher index, as
// sample_token, src/transformer4.rs:3084-3091) that also advances each
// sequence's position.  One step is captured once as a CUDA graph; tokens and
// positions live in device memory, so generation is graph launches alone.
//
// Weights, norms and the RoPE conventions are the single-sequence engine's
// (decoder_internal.h); this engine adds the B KV caches and its activations.
#include <math.h>
#include <string.h>

#include <cooperative_groups.h>

#include <algorithm>
#include <vector>

#include "attention.cuh"
#include "attn_batch.cuh"
#include "common.cuh"
#include "decoder_internal.h"
#include "gemm.cuh"
#include "gemv_core.cuh"
#include "nccl_dl.h"
#include "rt_internal.h"

using rt::fail;
namespace cg = cooperative_groups;

namespace {

// Peer all-reduce of the tensor-parallel step (rt_tp_peer_open).
constexpr int kMaxRanks = 8;
constexpr int kArCtas = 16;          // CTAs of one all-reduce; CTA c owns slice c of the vector
constexpr int64_t kArFlagBytes = 4096;  // [2 parities][kMaxRanks][kArCtas] u32 flags, then the receive areas

// Every rank's symmetric buffer, as this rank addresses it (its own: local).
struct PeerBufs {
    uint8_t* base[kMaxRanks];
};

struct BatchGemm {
    rt::GemmPlan p;
    CUtensorMap ta, tw;
    const float* ascale = nullptr;  // row scales of A
    const uint16_t* a = nullptr;    // fp16 rows of A (the multi-row GEMV reads them directly)
    const float* a32 = nullptr;     // f32 rows of A for the multi-row GEMV (RowsPlan::f32_rows)
    int64_t m = 0, n = 0;
    int k = 0;
};

// GEMM launches of one step over m rows; the LM head covers rows
// [lm_row0, lm_row0 + lm_rows) (none if lm_rows == 0).
struct RowsPlan {
    int m = 0, lm_row0 = 0, lm_rows = 0;
    // Every projection runs the multi-row GEMV, which reads f32 rows: the row
    // kernels then write f32 GEMM inputs (no fp16 row scale) and the
    // attention output feeds the o projection as it is.
    bool f32_rows = false;
    std::vector<BatchGemm> qkv, o, gu, down;
    BatchGemm lm;
    int64_t part_floats = 0;  // split-K outputs the plan needs
};

}  // namespace

struct rt_batch {
    rt_dec* dec = nullptr;
    rt_ctx* ctx = nullptr;
    int B = 0, cap = 0, H = 0, D = 0, NQ = 0, NKV = 0, F = 0, V = 0, NL = 0, qkv_rows = 0, nsplit = 0;
    // KV caches: layer l's K of row b at kv_k0 + l * kv_lstride + b * seq_kv
    // ([NKV][cap][D]), V likewise from kv_v0.  Many-sequence mode owns
    // kv = [B][NL][2 (K, V)][NKV][cap][D]; rows mode (positions of one
    // sequence) uses the decoder's caches with seq_kv = 0.
    bool rows_mode = false;
    int64_t seq_kv = 0;
    int64_t kv_lstride = 0;
    float* kv = nullptr;
    float* kv_k0 = nullptr;
    float* kv_v0 = nullptr;
    float* rope = nullptr;       // [2 (local, global)][2 (cos, sin)][cap][D/2] (the decoder's in rows mode)
    uint16_t* xa = nullptr;      // fp16 [B][K] input of the next GEMM, row b scaled by 1 / xscale[b]
    float* xa32 = nullptr;       // f32 [min(B, kRowsMaxM)][K] input of the next multi-row GEMV
    float* xscale = nullptr;     // [B] power-of-two row scales of xa
    float* parts = nullptr;      // GEMM outputs [splits][rows][N]
    int64_t part_cap = 0;        // floats allocated at `parts`
    float* qkv = nullptr;        // [B][qkv_rows]
    float* attn = nullptr;       // [B][NQ * D]
    float* resid[2] = {nullptr, nullptr};  // [B][H], ping-pong
    float* logits = nullptr;     // [logit_rows][V]
    int logit_rows = 0;
    float* attn_part = nullptr;  // per-chunk (or per-split) attention states
    float* q_rot = nullptr;      // [B][NQ][D] rotated queries (chunk path)
    bool chunk_path = false;     // attn_batch.cu kernels (false: attention.cu, one grid plane per sequence)
    uint32_t* counters = nullptr;  // [B][NKV], zero between launches
    int32_t* tokens = nullptr;   // [B] input token of the next step
    int32_t* pos = nullptr;      // [B] position of the next step
    int* h_err = nullptr;        // pinned copy of the context's error word
    RowsPlan plan;               // the captured step's (many-sequence mode)
    // Rows mode: a plan and a captured graph per (rows, logit rows) met so far.
    struct RowsGraph {
        RowsPlan plan;
        cudaGraph_t graph = nullptr;
        cudaGraphExec_t exec = nullptr;
    };
    std::vector<RowsGraph*> rows_graphs;
    // Tensor parallelism (nranks > 1): the decoder holds this rank's shard
    // (its query / KV heads and FFN columns); the o and down outputs are
    // summed over the ranks (NCCL all-reduce) and the LM head covers vocab
    // rows [v0, v0 + vr), the greedy token coming from an all-gather of every
    // rank's best (value, index).
    int nranks = 1, rank = 0, v0 = 0, vr = 0;
    const rt::NcclApi* nccl = nullptr;
    ncclComm_t comm = nullptr;
    float* ar_buf = nullptr;      // [B][H] summed projection
    // Peer all-reduce (after rt_tp_peer_open; NCCL's before): this rank's
    // symmetric buffer [flags][2][nranks][B*H] (exported through CUDA IPC),
    // every rank's buffer as mapped here, and the step counter that tags the
    // flags.
    bool p2p = false;
    uint8_t* ar_sym = nullptr;
    PeerBufs peers{};
    void* opened[kMaxRanks] = {};
    int32_t* step_ctr = nullptr;
    uint32_t* am_send = nullptr;  // [slices][rows][kTpWords] this rank's greedy records of each row
    uint32_t* am_recv = nullptr;  // [nranks][slices][rows][kTpWords]
    cudaGraph_t graph = nullptr;
    cudaGraphExec_t exec = nullptr;
    int launches = 0;
    uint64_t dev_bytes = 0;
    std::vector<void*> allocs;
};

namespace {

// ---- row kernels (one CTA per sequence row) ----

constexpr int kMaxParts = 8;  // split-K partial products a row kernel adds (gemm_q4k_plan caps splits at 8)
constexpr int kRowsMax = 512;            // rows mode: positions per call (longer prompts run in pieces)
constexpr int kRowsMaxLogitRows = 64;    // rows mode: rows whose logits one call can return

// Row kernels.  One sequence row is split over a thread-block cluster of
// `cl` CTAs (cluster rank q: columns [q * chunk, (q + 1) * chunk), chunk a
// multiple of 4, float4 accesses); the row's sums and maxima are block
// reductions combined over the cluster through distributed shared memory, the
// CTAs' partials added in cluster-rank order, so every CTA gets the same bits.
// Dynamic shared memory: chunk floats (the CTA's slice of the row).
constexpr int kRowCta = 256;

struct RowSlice {
    int64_t base;  // row start (elements)
    int c0, c1;    // this CTA's columns
    int chunk;     // columns per CTA (the dynamic shared memory holds multiples of it)
};

__device__ __forceinline__ RowSlice row_slice(int n) {
    cg::cluster_group cl = cg::this_cluster();
    const int q = static_cast<int>(cl.block_rank()), csize = static_cast<int>(cl.num_blocks());
    const int chunk = (n + 4 * csize - 1) / (4 * csize) * 4;
    const int b = blockIdx.x / csize;
    return RowSlice{static_cast<int64_t>(b) * n, min(n, q * chunk), min(n, (q + 1) * chunk), chunk};
}

// Sum (kMax false) or maximum (kMax true) of v over the cluster's threads.
// `slot` is a shared float used by this reduction alone: its CTA's partial,
// read by the other CTAs after the cluster barrier.
template <bool kMax>
__device__ __forceinline__ float cluster_reduce(float v, float* red, float* slot) {
    cg::cluster_group cl = cg::this_cluster();
    v = kMax ? rt::block_max(v, red) : rt::block_sum(v, red);
    if (threadIdx.x == 0) *slot = v;
    cl.sync();
    const int csize = static_cast<int>(cl.num_blocks());
    float t = *cl.map_shared_rank(slot, 0);
    for (int r = 1; r < csize; ++r) {
        const float x = *cl.map_shared_rank(slot, r);
        t = kMax ? fmaxf(t, x) : t + x;
    }
    return t;
}

// src[i..i+4) + src[stride + i..] + ... (`parts` <= kMaxParts terms, in part
// order), every load issued before the first add.
__device__ __forceinline__ float4 ld_parts4(const float* src, int parts, int64_t stride, int64_t i) {
    float4 w[kMaxParts];
#pragma unroll
    for (int q = 0; q < kMaxParts; ++q)
        w[q] = q < parts ? *reinterpret_cast<const float4*>(src + q * stride + i) : make_float4(0.f, 0.f, 0.f, 0.f);
    float4 v = w[0];
#pragma unroll
    for (int q = 1; q < kMaxParts; ++q)
        if (q < parts) v = make_float4(v.x + w[q].x, v.y + w[q].y, v.z + w[q].z, v.w + w[q].w);
    return v;
}

__device__ __forceinline__ float abs_max4(float m, float4 v) {
    return fmaxf(fmaxf(m, fmaxf(fabsf(v.x), fabsf(v.y))), fmaxf(fabsf(v.z), fabsf(v.w)));
}

// The slice row[0..c1-c0) as fp16 GEMM input: out = fp16(v * 2^-e), oscale =
// 2^e, e from the row's maximum |v| (`mx`, this thread's part of it), then a
// last cluster barrier: no CTA leaves while another still reads its slots.
__device__ __forceinline__ void store_f16_slice(const float* row, RowSlice rs, float mx, float* red, float* slot,
                                                uint16_t* out, float* oscale) {
    mx = cluster_reduce<true>(mx, red, slot);
    float inv, sc;
    rt::row_scale_f16(mx, &inv, &sc);
    for (int c = rs.c0 + 4 * threadIdx.x; c < rs.c1; c += 4 * blockDim.x) {
        const float4 v = *reinterpret_cast<const float4*>(row + (c - rs.c0));
        const __half2 lo = __floats2half2_rn(v.x * inv, v.y * inv), hi = __floats2half2_rn(v.z * inv, v.w * inv);
        uint2 pk;
        pk.x = *reinterpret_cast<const uint32_t*>(&lo);
        pk.y = *reinterpret_cast<const uint32_t*>(&hi);
        *reinterpret_cast<uint2*>(out + rs.base + c) = pk;
    }
    if (threadIdx.x == 0 && cg::this_cluster().block_rank() == 0) *oscale = sc;
    cg::this_cluster().sync();
}

// Residual update and RMSNorm of one row (the fused prologues of the
// single-sequence engine, in the same operation order per element):
//   embed != null: r = bf16(embed[tokens[b]]) * embed_scale   (src/transformer4.rs:2360-2364)
//   else:          s = src parts added in order; r = resid_in + s * rms(s) * (1 + gpost)
//   resid_out = r;  x = r * rms(r) * (1 + gpre)                 (rms_norm_gemma3, src/autograd2.rs:3477-3496)
// and x goes out as an fp16 GEMM row with its scale (or, out32 != null, as f32
// for the multi-row GEMV).  Rows of H (a multiple of 4).
__global__ void __launch_bounds__(kRowCta) resid_norm_rows_kernel(
    const uint16_t* embed, const int32_t* tokens, float embed_scale, const float* src, int src_parts,
    int64_t part_stride, const float* resid_in, float* resid_out, const float* gpost, const float* gpre, float eps, int H,
    uint16_t* out, float* oscale, float* out32) {
    // This CTA's slice of the row, then of resid_in, gpost and gpre: every
    // global load is issued in the first pass, before the first reduction.
    extern __shared__ float4 row4[];
    float* row = reinterpret_cast<float*>(row4);
    __shared__ float red[32];
    __shared__ float slot[4];
    const RowSlice rs = row_slice(H);
    float* rin = row + rs.chunk;
    float* gpo = rin + rs.chunk;
    float* gpr = gpo + rs.chunk;
    const int b = static_cast<int>(rs.base / H), tid = threadIdx.x, step = 4 * blockDim.x;
    const float inv_d = 1.0f / static_cast<float>(H);
    float ss = 0.f;
    if (embed) {
        const uint16_t* er = embed + static_cast<int64_t>(tokens[b]) * H;
        for (int c = rs.c0 + 4 * tid; c < rs.c1; c += step) {
            const uint2 raw = *reinterpret_cast<const uint2*>(er + c);
            const float4 v = make_float4(__fmul_rn(rt::bf16_bits_to_f32(raw.x & 0xFFFFu), embed_scale),
                                         __fmul_rn(rt::bf16_bits_to_f32(raw.x >> 16), embed_scale),
                                         __fmul_rn(rt::bf16_bits_to_f32(raw.y & 0xFFFFu), embed_scale),
                                         __fmul_rn(rt::bf16_bits_to_f32(raw.y >> 16), embed_scale));
            *reinterpret_cast<float4*>(row + (c - rs.c0)) = v;
            *reinterpret_cast<float4*>(gpr + (c - rs.c0)) = *reinterpret_cast<const float4*>(gpre + c);
            *reinterpret_cast<float4*>(resid_out + rs.base + c) = v;
            ss += v.x * v.x + v.y * v.y + v.z * v.z + v.w * v.w;
        }
    } else {
        for (int c = rs.c0 + 4 * tid; c < rs.c1; c += step) {
            const float4 v = ld_parts4(src, src_parts, part_stride, rs.base + c);
            const float4 ri = *reinterpret_cast<const float4*>(resid_in + rs.base + c);
            const float4 g1 = *reinterpret_cast<const float4*>(gpost + c);
            const float4 g2 = *reinterpret_cast<const float4*>(gpre + c);
            *reinterpret_cast<float4*>(row + (c - rs.c0)) = v;
            *reinterpret_cast<float4*>(rin + (c - rs.c0)) = ri;
            *reinterpret_cast<float4*>(gpo + (c - rs.c0)) = g1;
            *reinterpret_cast<float4*>(gpr + (c - rs.c0)) = g2;
            ss += v.x * v.x + v.y * v.y + v.z * v.z + v.w * v.w;
        }
        ss = cluster_reduce<false>(ss, red, &slot[0]);
        const float r1 = 1.0f / sqrtf(ss * inv_d + eps);
        ss = 0.f;
        for (int c = rs.c0 + 4 * tid; c < rs.c1; c += step) {
            const float4 v = *reinterpret_cast<const float4*>(row + (c - rs.c0));
            const float4 ri = *reinterpret_cast<const float4*>(rin + (c - rs.c0));
            const float4 g = *reinterpret_cast<const float4*>(gpo + (c - rs.c0));
            const float4 nv = make_float4(__fadd_rn(ri.x, __fmul_rn(__fmul_rn(v.x, r1), __fadd_rn(1.0f, g.x))),
                                          __fadd_rn(ri.y, __fmul_rn(__fmul_rn(v.y, r1), __fadd_rn(1.0f, g.y))),
                                          __fadd_rn(ri.z, __fmul_rn(__fmul_rn(v.z, r1), __fadd_rn(1.0f, g.z))),
                                          __fadd_rn(ri.w, __fmul_rn(__fmul_rn(v.w, r1), __fadd_rn(1.0f, g.w))));
            *reinterpret_cast<float4*>(row + (c - rs.c0)) = nv;
            *reinterpret_cast<float4*>(resid_out + rs.base + c) = nv;
            ss += nv.x * nv.x + nv.y * nv.y + nv.z * nv.z + nv.w * nv.w;
        }
    }
    ss = cluster_reduce<false>(ss, red, &slot[1]);
    const float r2 = 1.0f / sqrtf(ss * inv_d + eps);
    float mx = 0.f;
    for (int c = rs.c0 + 4 * tid; c < rs.c1; c += step) {
        const float4 v = *reinterpret_cast<const float4*>(row + (c - rs.c0));
        const float4 g = *reinterpret_cast<const float4*>(gpr + (c - rs.c0));
        const float4 x = make_float4(__fmul_rn(__fmul_rn(v.x, r2), __fadd_rn(1.0f, g.x)),
                                     __fmul_rn(__fmul_rn(v.y, r2), __fadd_rn(1.0f, g.y)),
                                     __fmul_rn(__fmul_rn(v.z, r2), __fadd_rn(1.0f, g.z)),
                                     __fmul_rn(__fmul_rn(v.w, r2), __fadd_rn(1.0f, g.w)));
        if (out32) {
            *reinterpret_cast<float4*>(out32 + rs.base + c) = x;
        } else {
            *reinterpret_cast<float4*>(row + (c - rs.c0)) = x;
            mx = abs_max4(mx, x);
        }
    }
    if (out32) {
        cg::this_cluster().sync();  // no CTA leaves while another still reads its slots
        return;
    }
    store_f16_slice(row, rs, mx, red, &slot[2], out, oscale + b);
}

// h[b][j] = gelu_tanh(gate) * up from the interleaved gate/up GEMM output
// (column 2j gate, 2j + 1 up), its split parts added in order; h goes out as an
// fp16 GEMM row with its scale (or, out32 != null, as f32).  Rows of F outputs
// (a multiple of 4).
__global__ void __launch_bounds__(kRowCta) gelu_rows_kernel(const float* c, int parts, int64_t part_stride, int F,
                                                           uint16_t* out, float* oscale, float* out32) {
    extern __shared__ float4 h4[];
    float* h = reinterpret_cast<float*>(h4);
    __shared__ float red[32];
    __shared__ float slot[1];
    const RowSlice rs = row_slice(F);
    const int b = static_cast<int>(rs.base / F);
    const int64_t in = 2 * rs.base;  // row b of the [B][2F] input
    float mx = 0.f;
    for (int j = rs.c0 + 4 * threadIdx.x; j < rs.c1; j += 4 * blockDim.x) {
        const float4 a = ld_parts4(c, parts, part_stride, in + 2 * j);      // g0 u0 g1 u1
        const float4 e = ld_parts4(c, parts, part_stride, in + 2 * j + 4);  // g2 u2 g3 u3
        const float4 v = make_float4(__fmul_rn(rt::gcore::gelu_tanh_dev(a.x), a.y),
                                     __fmul_rn(rt::gcore::gelu_tanh_dev(a.z), a.w),
                                     __fmul_rn(rt::gcore::gelu_tanh_dev(e.x), e.y),
                                     __fmul_rn(rt::gcore::gelu_tanh_dev(e.z), e.w));
        if (out32) {
            *reinterpret_cast<float4*>(out32 + rs.base + j) = v;
        } else {
            *reinterpret_cast<float4*>(h + (j - rs.c0)) = v;
            mx = abs_max4(mx, v);
        }
    }
    if (!out32) store_f16_slice(h, rs, mx, red, &slot[0], out, oscale + b);
}

// Row b of `in` ([B][n] f32, n a multiple of 4) as an fp16 GEMM row with its
// scale.
__global__ void __launch_bounds__(kRowCta) f16_rows_kernel(const float* in, int n, uint16_t* out, float* oscale) {
    extern __shared__ float4 v4[];
    float* v = reinterpret_cast<float*>(v4);
    __shared__ float red[32];
    __shared__ float slot[1];
    const RowSlice rs = row_slice(n);
    float mx = 0.f;
    for (int c = rs.c0 + 4 * threadIdx.x; c < rs.c1; c += 4 * blockDim.x) {
        const float4 x = *reinterpret_cast<const float4*>(in + rs.base + c);
        *reinterpret_cast<float4*>(v + (c - rs.c0)) = x;
        mx = abs_max4(mx, x);
    }
    store_f16_slice(v, rs, mx, red, &slot[0], out, oscale + rs.base / n);
}

// CTAs per row: enough CTAs in flight for small batches, at most 8 (the
// portable cluster size), and a slice that fits 48 KB of shared memory.
int row_cluster(int rows, int n) {
    int cl = rows >= 128 ? 2 : rows >= 32 ? 4 : 8;
    while (cl < 8 && (n + 4 * cl - 1) / (4 * cl) * 4 * sizeof(float) > 48 * 1024) cl *= 2;
    return cl;
}

// kSlices: how many chunk-sized float arrays the kernel keeps in dynamic
// shared memory.
template <int kSlices = 1, typename... KArgs, typename... Args>
cudaError_t launch_rows(void (*k)(KArgs...), int rows, int n, cudaStream_t s, Args... args) {
    const int cl = row_cluster(rows, n);
    cudaLaunchConfig_t cfg{};
    cfg.gridDim = dim3(static_cast<unsigned>(rows * cl));
    cfg.blockDim = dim3(kRowCta);
    cfg.dynamicSmemBytes = sizeof(float) * kSlices * ((n + 4 * cl - 1) / (4 * cl) * 4);
    cfg.stream = s;
    cudaLaunchAttribute at[1];
    at[0].id = cudaLaunchAttributeClusterDimension;
    at[0].val.clusterDim.x = static_cast<unsigned>(cl);
    at[0].val.clusterDim.y = 1;
    at[0].val.clusterDim.z = 1;
    cfg.attrs = at;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, k, static_cast<KArgs>(args)...);
}

// Greedy sampling (sample_token at temperature 0: the last index of the
// largest softmax probability, see kGreedyTau in gemv_core.cuh) over rows of
// logits split into vocab slices, each slice taken by one CTA.  The record of
// a slice: words [0] m (its largest logit, bits), [1] s (sum of exp(y - m)
// over the slice, bits), [2] the number of its logits within kGreedyTau of
// m, [3] unused, then up to kTpCand (value bits, vocab index) pairs of those
// logits, highest indices first.  The merge (argmax_merge_kernel) combines the
// records of a row in vocab order: every candidate of the global maximum is
// in them unless a slice holds more than kTpCand logits within kGreedyTau of
// its own maximum (word 2).  On one GPU the merge then rescans that slice; a
// tensor-parallel merge, whose other slices live on other ranks, decides
// among the kTpCand highest of them.
constexpr int kTpCand = 4;
constexpr int kTpWords = 4 + 2 * kTpCand;
constexpr int kGreedySlices = 32;  // vocab slices per row and rank (CTAs per row)
constexpr int kGreedyThreads = 256;

// CTA (b, p) of a (rows, slices) grid: the record of columns [p W, (p + 1) W)
// of row b of `logits` ([rows][V], this rank's vocab rows v0..v0+V).
// Launched with kGreedyThreads threads.
__global__ void __launch_bounds__(kGreedyThreads) argmax_local_kernel(const float* logits, int V, int W, int v0,
                                                                      uint32_t* out) {
    __shared__ float sm[32], ss[32];
    __shared__ long long si[32];
    __shared__ int sbest, ncand;
    __shared__ int cand[kTpCand];
    using rt::gcore::Greedy;
    const int b = blockIdx.x, p = blockIdx.y, tid = threadIdx.x, lane = tid & 31, warp = tid >> 5, nw = blockDim.x >> 5;
    const int c0 = p * W;
    const float* r = logits + static_cast<int64_t>(b) * V + c0;
    V = max(0, min(W, V - c0));  // this slice's columns
    v0 += c0;
    Greedy g;
    g.init();
    // This thread's elements tid, tid + 256, ... in order, loaded 8 at a time
    // ahead of the (branchy) state updates.
    constexpr int kBatch = 8;
    for (int i0 = tid; i0 < V; i0 += kBatch * kGreedyThreads) {
        float v[kBatch];
#pragma unroll
        for (int j = 0; j < kBatch; ++j) {
            const int i = i0 + j * kGreedyThreads;
            v[j] = i < V ? r[i] : 0.f;
        }
#pragma unroll
        for (int j = 0; j < kBatch; ++j)
            if (i0 + j * kGreedyThreads < V) g.add(v[j], i0 + j * kGreedyThreads);
    }
    const float my_m = g.m;
    g.warp_merge();
    if (lane == 0) {
        sm[warp] = g.m;
        ss[warp] = g.s;
        si[warp] = g.i;
    }
    if (tid == 0) {
        sbest = -1;
        ncand = 0;
    }
    __syncthreads();
    Greedy c;
    c.init();
    for (int w = 0; w < nw; ++w) c.merge(sm[w], ss[w], si[w], 0, 0);
    const float lim = c.m - rt::gcore::kGreedyTau;
    // Candidates of this slice: the kTpCand highest indices within kGreedyTau
    // of its maximum, found one at a time from the top (a few passes at most,
    // by the few threads that hold any).
    int below = V;  // next candidate must have a lower index
    for (int k = 0; k < kTpCand; ++k) {
        int best = -1, cnt = 0;
        if (my_m >= lim)
            for (int i0 = tid; i0 < V; i0 += kBatch * kGreedyThreads) {
                float v[kBatch];
#pragma unroll
                for (int j = 0; j < kBatch; ++j) {
                    const int i = i0 + j * kGreedyThreads;
                    v[j] = i < V ? r[i] : -INFINITY;
                }
#pragma unroll
                for (int j = 0; j < kBatch; ++j) {
                    const int i = i0 + j * kGreedyThreads;
                    if (v[j] >= lim) {
                        if (i < below) best = i;
                        ++cnt;
                    }
                }
            }
        if (best >= 0) atomicMax(&sbest, best);
        if (k == 0 && cnt) atomicAdd(&ncand, cnt);
        __syncthreads();
        const int found = sbest;
        __syncthreads();
        if (found < 0) break;
        if (tid == 0) {
            cand[k] = found;
            sbest = -1;
        }
        below = found;
        __syncthreads();
    }
    if (tid == 0) {
        uint32_t* o = out + (static_cast<int64_t>(p) * gridDim.x + b) * kTpWords;
        o[0] = __float_as_uint(c.m);
        o[1] = __float_as_uint(c.s);
        o[2] = static_cast<uint32_t>(ncand);
        o[3] = 0u;
        const int n = min(ncand, kTpCand);
        for (int k = 0; k < kTpCand; ++k) {
            o[4 + 2 * k] = __float_as_uint(k < n ? r[cand[k]] : -INFINITY);
            o[5 + 2 * k] = k < n ? static_cast<uint32_t>(v0 + cand[k]) : 0xFFFFFFFFu;
        }
    }
}

// The greedy token of each row from its nrec slice records ([nrec][B], in
// vocab order): M = max m_r, S = sum_r s_r exp(m_r - M) in record order, then
// the highest candidate index whose probability equals the maximum's; then
// tokens[b] = it and pos[b] += 1.  logits != null: the records are this GPU's
// slices of width W of logits ([B][V]), and a slice with more candidates than
// its record holds is rescanned.
__global__ void argmax_merge_kernel(const uint32_t* recs, int nrec, int B, int32_t* tokens, int32_t* pos,
                                    const float* logits, int V, int W) {
    const int b = blockIdx.x * blockDim.x + threadIdx.x;
    if (b >= B) return;
    auto rec = [&](int r) { return recs + (static_cast<int64_t>(r) * B + b) * kTpWords; };
    float M = -INFINITY;
    for (int r = 0; r < nrec; ++r) M = fmaxf(M, __uint_as_float(rec(r)[0]));
    float S = 0.f;
    for (int r = 0; r < nrec; ++r) {
        const uint32_t* o = rec(r);
        if (o[1] != 0u) S += __uint_as_float(o[1]) * expf(__uint_as_float(o[0]) - M);  // empty slice: s = 0, m = -inf
    }
    const float q = __fdiv_rn(1.0f, S), lim = M - rt::gcore::kGreedyTau;
    int best = -1;
    for (int r = 0; r < nrec; ++r) {
        const uint32_t* o = rec(r);
        if (__uint_as_float(o[0]) < lim) continue;
        if (logits && o[2] > static_cast<uint32_t>(kTpCand)) {
            const int c1 = min(V, (r + 1) * W);
            for (int i = r * W; i < c1; ++i) {
                const float v = logits[static_cast<int64_t>(b) * V + i];
                if (v >= lim && i > best && rt::gcore::greedy_ties_max(v, M, S, q)) best = i;
            }
            continue;
        }
        for (int k = 0; k < kTpCand; ++k) {
            const float v = __uint_as_float(o[4 + 2 * k]);
            const int i = static_cast<int>(o[5 + 2 * k]);
            if (i >= 0 && v >= lim && i > best && rt::gcore::greedy_ties_max(v, M, S, q)) best = i;
        }
    }
    tokens[b] = best;
    pos[b] += 1;
}

// Sum over the ranks of this rank's partial into buf[0..count), through the
// ranks' symmetric buffers.  The partial is src's `parts` split-K parts
// (stride count) added in part order, as sum_parts_launch adds them; src may
// be buf itself (one part).  CTA c stores its slice of the partial into
// every rank's receive area of this rank (NVLink stores), fences at system
// scope and raises its flag there with `tag`; then it waits (bounded) for the
// flag of every rank's CTA c in its own buffer and adds the ranks' slices in
// rank order, so every rank gets the same bits.  Two receive areas alternate
// between consecutive calls (`parity`): a rank cannot reach call s + 2 before
// every rank has finished call s, so no area or flag is rewritten while it is
// read.  After a wait gives up (err set) later calls no longer wait.
__global__ void __launch_bounds__(256) peer_allreduce_kernel(const float* src, int parts, float* buf, int64_t count,
                                                             int64_t cap_count, PeerBufs pb,
                                                             int nranks, int rank, int parity, uint32_t call,
                                                             const int32_t* step_ctr, int* err) {
    const int c = blockIdx.x, tid = threadIdx.x;
    const int64_t per = (count + 4 * kArCtas - 1) / (4 * kArCtas) * 4;
    const int64_t i0 = c * per, i1 = min(count, i0 + per);
    const uint32_t tag = static_cast<uint32_t>(*step_ctr) * 256u + call + 1u;
    const bool broken = *reinterpret_cast<volatile int*>(err) != 0;
    auto recv = [&](int owner, int src) {
        return reinterpret_cast<float*>(pb.base[owner] + kArFlagBytes) + static_cast<int64_t>(parity * nranks + src) * cap_count;
    };
    auto flag = [&](int owner, int src) {
        return reinterpret_cast<uint32_t*>(pb.base[owner]) + (parity * kMaxRanks + src) * kArCtas + c;
    };
    for (int64_t i = i0 + 4 * tid; i < i1; i += 4 * blockDim.x) {
        float4 v = *reinterpret_cast<const float4*>(src + i);
        for (int z = 1; z < parts; ++z) {
            const float4 w = *reinterpret_cast<const float4*>(src + z * count + i);
            v = make_float4(v.x + w.x, v.y + w.y, v.z + w.z, v.w + w.w);
        }
        for (int r = 0; r < nranks; ++r) *reinterpret_cast<float4*>(recv(r, rank) + i) = v;
    }
    __threadfence_system();
    __syncthreads();
    if (tid < nranks)
        asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(flag(tid, rank)), "r"(tag) : "memory");
    if (tid < nranks && !broken) {
        const uint32_t* f = flag(rank, tid);
        uint64_t t0 = 0;
        for (uint32_t it = 1;; ++it) {
            uint32_t v;
            asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(f) : "memory");
            if (v == tag) break;
            if ((it & 1023u) == 0u) {
                uint64_t t;
                asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
                if (it == 1024u) t0 = t;
                else if (t - t0 > 2000000000ull) {
                    atomicExch(err, rt::kErrGridTimeout);
                    break;
                }
            }
        }
    }
    __syncthreads();
    for (int64_t i = i0 + 4 * tid; i < i1; i += 4 * blockDim.x) {
        float4 a = __ldcg(reinterpret_cast<const float4*>(recv(rank, 0) + i));
        for (int r = 1; r < nranks; ++r) {
            const float4 b = __ldcg(reinterpret_cast<const float4*>(recv(rank, r) + i));
            a = make_float4(a.x + b.x, a.y + b.y, a.z + b.z, a.w + b.w);
        }
        *reinterpret_cast<float4*>(buf + i) = a;
    }
}

__global__ void tick_kernel(int32_t* ctr) { *ctr += 1; }

// Synthetic cache contents for benchmarks: a hash of (seed, index) mapped to
// a uniform value of unit variance.
__global__ void synth_kv_kernel(float* kv, int64_t n, uint64_t seed) {
    const int64_t stride = static_cast<int64_t>(gridDim.x) * blockDim.x;
    for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < n; i += stride) {
        uint64_t z = seed + static_cast<uint64_t>(i) * 0x9E3779B97F4A7C15ull;
        z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
        z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
        z ^= z >> 31;
        kv[i] = (static_cast<float>(z >> 40) * (1.0f / 16777216.0f) - 0.5f) * 3.4641016f;
    }
}

__global__ void fill_i32_kernel(int32_t* p, int n, int32_t v) {
    const int i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i < n) p[i] = v;
}

int balloc(rt_batch* t, void** p, size_t bytes, const char* what) {
    int rc = rt::dev_alloc(t->ctx, p, bytes, what);
    if (rc == RT_OK) {
        t->allocs.push_back(*p);
        t->dev_bytes += bytes;
    }
    return rc;
}

void drop_rows_graphs(rt_batch* t) {
    for (rt_batch::RowsGraph* r : t->rows_graphs) {
        if (r->exec) cudaGraphExecDestroy(r->exec);
        if (r->graph) cudaGraphDestroy(r->graph);
        delete r;
    }
    t->rows_graphs.clear();
}

void release(rt_batch* t) {
    if (!t) return;
    drop_rows_graphs(t);
    if (t->exec) cudaGraphExecDestroy(t->exec);
    if (t->graph) cudaGraphDestroy(t->graph);
    if (t->comm && t->nccl) t->nccl->comm_destroy(t->comm);  // after the graphs that hold its calls
    for (void* p : t->opened)
        if (p) cudaIpcCloseMemHandle(p);
    for (void* p : t->allocs) cudaFree(p);
    if (t->h_err) cudaFreeHost(t->h_err);
    delete t;
}

float* k_layer(rt_batch* t, int l) { return t->kv_k0 + static_cast<int64_t>(l) * t->kv_lstride; }
float* v_layer(rt_batch* t, int l) { return t->kv_v0 + static_cast<int64_t>(l) * t->kv_lstride; }

// C[m, n] = rows [row0, row0 + m) of xa (K = k) . W^T.
bool make_gemm(rt_batch* t, int m, int row0, const void* w, int64_t n, int k, bool wbf16, bool allow_split, BatchGemm* g) {
    g->m = m;
    g->n = n;
    g->k = k;
    g->ascale = t->xscale + row0;
    g->a = t->xa + static_cast<int64_t>(row0) * k;
    g->p = rt::gemm_q4k_plan(m, n, k, t->ctx->num_sms, wbf16, allow_split);
    if (g->p.bm == 0 || g->p.splits > kMaxParts) return false;
    return rt::gemm_q4k_tmaps(t->xa + static_cast<int64_t>(row0) * k, m, w, n, k, g->p, &g->ta, &g->tw);
}

bool build_plan(rt_batch* t, int m, int lm_row0, int lm_rows, RowsPlan* pl) {
    rt_dec* d = t->dec;
    const int H = t->H;
    pl->m = m;
    pl->lm_row0 = lm_row0;
    pl->lm_rows = lm_rows;
    pl->qkv.assign(t->NL, BatchGemm{});
    pl->o.assign(t->NL, BatchGemm{});
    pl->gu.assign(t->NL, BatchGemm{});
    pl->down.assign(t->NL, BatchGemm{});
    pl->part_floats = 0;
    for (int l = 0; l < t->NL; ++l) {
        if (!make_gemm(t, m, 0, d->w_qkv[l], t->qkv_rows, H, false, true, &pl->qkv[l]) ||
            !make_gemm(t, m, 0, d->w_o[l], H, t->NQ * t->D, false, true, &pl->o[l]) ||
            !make_gemm(t, m, 0, d->w_gu[l], 2LL * t->F, H, false, true, &pl->gu[l]) ||
            !make_gemm(t, m, 0, d->w_down[l], H, t->F, false, true, &pl->down[l]))
            return false;
        for (const BatchGemm* g : {&pl->qkv[l], &pl->o[l], &pl->gu[l], &pl->down[l]})
            pl->part_floats = std::max<int64_t>(pl->part_floats, static_cast<int64_t>(g->p.splits) * m * g->n);
    }
    pl->f32_rows = m <= rt::kRowsMaxM && t->xa32 != nullptr;
    for (int l = 0; l < t->NL; ++l)
        for (const BatchGemm* g : {&pl->qkv[l], &pl->o[l], &pl->gu[l], &pl->down[l]})
            pl->f32_rows = pl->f32_rows && g->p.rows_nt > 0;
    if (pl->f32_rows)
        for (int l = 0; l < t->NL; ++l) {
            pl->qkv[l].a32 = pl->gu[l].a32 = pl->down[l].a32 = t->xa32;
            pl->o[l].a32 = t->attn;
        }
    return lm_rows == 0 ||
           make_gemm(t, lm_rows, lm_row0, d->embed + static_cast<int64_t>(t->v0) * H, t->vr, H, true, false, &pl->lm);
}

// Enqueue one step over pl.m rows (all launches of it) on `s`; `argmax`: the
// greedy token of every row, which also advances its position.
cudaError_t enqueue(rt_batch* t, const RowsPlan& pl, cudaStream_t s, bool argmax) {
    rt_dec* d = t->dec;
    const int B = pl.m, H = t->H, D = t->D, G = t->NQ / t->NKV;
    const float eps = d->cfg.rms_norm_eps;
    int p = 0;
    int n = 0;
    cudaError_t e = cudaSuccess;
    auto ok = [&](cudaError_t r) {
        if (e == cudaSuccess) e = r;
        ++n;
        return e == cudaSuccess;
    };
    auto gemm = [&](const BatchGemm& g, float* c) {
        if (g.a32) return ok(rt::gemm_rows_launch(g.tw, nullptr, nullptr, c, g.m, g.n, g.k, g.p, t->ctx->d_err, s, g.a32));
        return ok(rt::gemm_q4k_launch(g.ta, g.tw, g.ascale, c, g.m, g.n, g.k, g.p, t->ctx->d_err, s, g.a));
    };
    float* const x32 = pl.f32_rows ? t->xa32 : nullptr;  // the row kernels' f32 output, if any
    auto nccl_ok = [&](ncclResult_t r) { return ok(r == ncclSuccess ? cudaSuccess : cudaErrorUnknown); };
    uint32_t ar_call = 0;  // peer all-reduces of this step so far
    // A row-split projection's output as a row kernel reads it: (source,
    // split parts, part stride).  With several ranks the parts are added and
    // the sum is all-reduced over the ranks into ar_buf.
    struct Proj {
        const float* src = nullptr;
        int parts = 1;
        int64_t stride = 0;
    };
    auto project = [&](const BatchGemm& g) -> Proj {
        const int64_t count = static_cast<int64_t>(B) * g.n;
        if (t->nranks == 1) return gemm(g, t->parts) ? Proj{t->parts, g.p.splits, count} : Proj{};
        if (!gemm(g, g.p.splits > 1 ? t->parts : t->ar_buf)) return Proj{};
        if (t->p2p) {  // split-K sum and all-reduce in one kernel
            const bool split = g.p.splits > 1;
            peer_allreduce_kernel<<<kArCtas, 256, 0, s>>>(split ? t->parts : t->ar_buf, split ? g.p.splits : 1, t->ar_buf,
                                                        count, static_cast<int64_t>(t->B) * t->H, t->peers, t->nranks,
                                                        t->rank, static_cast<int>(ar_call & 1), ar_call, t->step_ctr,
                                                        t->ctx->d_err);
            ++ar_call;
            if (!ok(cudaGetLastError())) return Proj{};
            return Proj{t->ar_buf, 1, count};
        }
        if (g.p.splits > 1 && !ok(rt::sum_parts_launch(t->parts, g.p.splits, count, t->ar_buf, t->ctx->num_sms, s)))
            return Proj{};
        if (!nccl_ok(t->nccl->all_reduce(t->ar_buf, t->ar_buf, static_cast<size_t>(count), ncclFloat32, ncclSum,
                                                t->comm, s))) {
            return Proj{};
        }
        return Proj{t->ar_buf, 1, count};
    };
    Proj pdown;  // the previous layer's down projection
    for (int l = 0; l < t->NL && e == cudaSuccess; ++l) {
        // residual update (or embedding) + attention RMSNorm -> x
        if (l == 0) {
            if (!ok(launch_rows<4>(resid_norm_rows_kernel, B, H, s, d->embed, t->tokens, sqrtf(static_cast<float>(H)),
                                nullptr, 0, int64_t{0}, nullptr, t->resid[0], nullptr, rt::norm_ptr(d, 0, 0), eps, H,
                                t->xa, t->xscale, x32)))
                break;
        } else {
            if (!ok(launch_rows<4>(resid_norm_rows_kernel, B, H, s, nullptr, nullptr, 0.f, pdown.src, pdown.parts,
                                pdown.stride, t->resid[p], t->resid[1 - p], rt::norm_ptr(d, l - 1, 3),
                                rt::norm_ptr(d, l, 0), eps, H, t->xa, t->xscale, x32)))
                break;
            p = 1 - p;
        }
        // qkv
        const BatchGemm& gq = pl.qkv[l];
        const bool qkv_parts = t->chunk_path && gq.p.splits > 1;  // the prep kernel adds the parts
        if (qkv_parts) {
            if (!gemm(gq, t->parts)) break;
        } else if (gq.p.splits > 1) {
            if (!gemm(gq, t->parts)) break;
            if (!ok(rt::sum_parts_launch(t->parts, gq.p.splits, static_cast<int64_t>(B) * t->qkv_rows, t->qkv,
                                         t->ctx->num_sms, s)))
                break;
        } else if (!gemm(gq, t->qkv)) {
            break;
        }
        // attention
        const size_t tab = static_cast<size_t>(t->cap) * (D / 2);
        const int gsel = rt::is_global(l) ? 1 : 0;
        const float* rope_cos = t->rope + (static_cast<size_t>(gsel) * 2 + 0) * tab;
        const float* rope_sin = t->rope + (static_cast<size_t>(gsel) * 2 + 1) * tab;
        const int window = rt::is_global(l) ? 0 : d->cfg.sliding_window;
        if (t->chunk_path) {
            rt::AttnRowsArgs pr{};
            pr.qkv = qkv_parts ? t->parts : t->qkv;
            pr.qkv_stride = t->qkv_rows;
            pr.parts = qkv_parts ? gq.p.splits : 1;
            pr.part_stride = static_cast<int64_t>(B) * t->qkv_rows;
            pr.q_norm = d->qk_norms + static_cast<size_t>(l) * 2 * D;
            pr.k_norm = pr.q_norm + D;
            pr.rope_cos = rope_cos;
            pr.rope_sin = rope_sin;
            pr.pos = t->pos;
            pr.kcache = k_layer(t, l);
            pr.vcache = v_layer(t, l);
            pr.seq_kv = t->seq_kv;
            pr.cap = t->cap;
            pr.nq = t->NQ;
            pr.nkv = t->NKV;
            pr.D = D;
            pr.eps = eps;
            pr.q_out = t->q_rot;
            if (!ok(rt::attn_rows_prep_launch(pr, B, s))) break;
            rt::AttnChunkArgs ca{};
            ca.q = t->q_rot;
            ca.kcache = k_layer(t, l);
            ca.vcache = v_layer(t, l);
            ca.seq_kv = t->seq_kv;
            ca.pos = t->pos;
            ca.B = B;
            ca.nq = t->NQ;
            ca.nkv = t->NKV;
            ca.D = D;
            ca.cap = t->cap;
            ca.window = window;
            ca.nchunk = rt::attn_chunk_count(t->cap, window);
            ca.scale = 1.0f / sqrtf(d->cfg.query_pre_attn_scalar);
            ca.part = t->attn_part;
            ca.out = t->attn;
            ca.err = t->ctx->d_err;
            if (!ok(rt::attn_chunk_launch(ca, t->ctx->num_sms, s))) break;
            if (ca.nchunk > 1) ++n;  // the merge kernel launched with it
        } else {
            rt::AttnArgs a{};
            a.qkv = t->qkv;
            a.q_norm = d->qk_norms + static_cast<size_t>(l) * 2 * D;
            a.k_norm = a.q_norm + D;
            a.kcache = k_layer(t, l);
            a.vcache = v_layer(t, l);
            a.rope_cos = rope_cos;
            a.rope_sin = rope_sin;
            a.pos = t->pos;
            a.cap = t->cap;
            a.nq = t->NQ;
            a.nkv = t->NKV;
            a.D = D;
            a.window = window;
            a.nsplit = t->nsplit;
            a.scale = 1.0f / sqrtf(d->cfg.query_pre_attn_scalar);
            a.eps = eps;
            a.part = t->attn_part;
            a.counter = t->counters;
            a.out = t->attn;
            a.err = t->ctx->d_err;
            a.seq_qkv = t->qkv_rows;
            a.seq_kv = t->seq_kv;
            a.seq_part = static_cast<int64_t>(t->NKV) * t->nsplit * G * rt::attn_part_stride(D);
            a.seq_out = static_cast<int64_t>(t->NQ) * D;
            if (!ok(rt::attention_launch_batch(a, B, s))) break;
        }
        if (!pl.f32_rows && !ok(launch_rows(f16_rows_kernel, B, t->NQ * D, s, t->attn, t->NQ * D, t->xa, t->xscale)))
            break;
        // o, then residual update + pre-FFN RMSNorm
        const Proj po = project(pl.o[l]);
        if (!po.src) break;
        if (!ok(launch_rows<4>(resid_norm_rows_kernel, B, H, s, nullptr, nullptr, 0.f, po.src, po.parts, po.stride,
                            t->resid[p], t->resid[1 - p], rt::norm_ptr(d, l, 1), rt::norm_ptr(d, l, 2), eps, H, t->xa,
                            t->xscale, x32)))
            break;
        p = 1 - p;
        // gate/up, GELU gate (in the multi-row GEMV's epilogue when K is one part)
        const BatchGemm& gg = pl.gu[l];
        if (gg.a32 && gg.p.splits == 1) {
            if (!ok(rt::gemm_rows_launch(gg.tw, nullptr, nullptr, t->xa32, gg.m, gg.n, gg.k, gg.p, t->ctx->d_err, s,
                                         gg.a32, rt::kRowsEpiGelu)))
                break;
        } else {
            if (!gemm(gg, t->parts)) break;
            if (!ok(launch_rows(gelu_rows_kernel, B, t->F, s, t->parts, gg.p.splits, static_cast<int64_t>(B) * 2 * t->F,
                                t->F, t->xa, t->xscale, x32)))
                break;
        }
        // down
        pdown = project(pl.down[l]);
        if (!pdown.src) break;
    }
    if (e == cudaSuccess && pl.lm_rows > 0) {
        // final residual update + norm, LM head, greedy tokens
        if (ok(launch_rows<4>(resid_norm_rows_kernel, B, H, s, nullptr, nullptr, 0.f, pdown.src, pdown.parts, pdown.stride,
                           t->resid[p], t->resid[1 - p], rt::norm_ptr(d, t->NL - 1, 3), d->final_norm, eps, H, t->xa,
                           t->xscale, static_cast<float*>(nullptr))) &&
            gemm(pl.lm, t->logits) && argmax) {
            const int W = (t->vr + kGreedySlices - 1) / kGreedySlices;
            argmax_local_kernel<<<dim3(pl.lm_rows, kGreedySlices), kGreedyThreads, 0, s>>>(t->logits, t->vr, W, t->v0,
                                                                                           t->am_send);
            const unsigned mb = static_cast<unsigned>((pl.lm_rows + 127) / 128);
            if (ok(cudaGetLastError()) && t->nranks == 1) {
                argmax_merge_kernel<<<mb, 128, 0, s>>>(t->am_send, kGreedySlices, pl.lm_rows, t->tokens, t->pos,
                                                       t->logits, t->vr, W);
                ok(cudaGetLastError());
            } else if (e == cudaSuccess &&
                       nccl_ok(t->nccl->all_gather(t->am_send, t->am_recv,
                                                   kTpWords * static_cast<size_t>(kGreedySlices) * pl.lm_rows, ncclUint32,
                                                   t->comm, s))) {
                argmax_merge_kernel<<<mb, 128, 0, s>>>(t->am_recv, t->nranks * kGreedySlices, pl.lm_rows, t->tokens,
                                                       t->pos, nullptr, 0, 0);
                ok(cudaGetLastError());
            }
        }
    }
    if (e == cudaSuccess && t->p2p) {  // the next step's peer all-reduces carry the next tag
        tick_kernel<<<1, 1, 0, s>>>(t->step_ctr);
        ok(cudaGetLastError());
    }
    t->launches = n;
    return e;
}

int check_error_word(rt_batch* t) {
    if (*t->h_err) {
        const int w = *t->h_err;
        *t->h_err = 0;
        cudaMemsetAsync(t->ctx->d_err, 0, sizeof(int), t->ctx->stream);
        cudaStreamSynchronize(t->ctx->stream);
        return fail(t->ctx, RT_E_TIMEOUT, "batch step: a kernel reported error word %d", w);
    }
    return RT_OK;
}

int grow_parts(rt_batch* t, int64_t floats) {
    if (floats <= t->part_cap) return RT_OK;
    if (t->parts) {
        cudaStreamSynchronize(t->ctx->stream);
        cudaFree(t->parts);
        t->allocs.erase(std::find(t->allocs.begin(), t->allocs.end(), static_cast<void*>(t->parts)));
        t->dev_bytes -= sizeof(float) * t->part_cap;
        t->parts = nullptr;
        t->part_cap = 0;
    }
    const int rc = balloc(t, reinterpret_cast<void**>(&t->parts), sizeof(float) * floats, "batch GEMM outputs");
    if (rc == RT_OK) t->part_cap = floats;
    return rc;
}

// (Re)capture the many-sequence step as t->graph / t->exec.
int capture_step(rt_batch* t) {
    rt_ctx* ctx = t->ctx;
    if (t->exec) cudaGraphExecDestroy(t->exec);
    if (t->graph) cudaGraphDestroy(t->graph);
    t->exec = nullptr;
    t->graph = nullptr;
    RT_CHECK_CUDA(ctx, cudaStreamSynchronize(ctx->stream));
    cudaStream_t s = ctx->stream;
    if (cudaStreamBeginCapture(s, cudaStreamCaptureModeThreadLocal) != cudaSuccess)
        return fail(ctx, RT_E_CUDA, "batch engine: begin capture");
    const cudaError_t ce = enqueue(t, t->plan, s, true);
    const cudaError_t ee = cudaStreamEndCapture(s, &t->graph);
    if (ce != cudaSuccess || ee != cudaSuccess || cudaGraphInstantiate(&t->exec, t->graph, 0) != cudaSuccess) {
        cudaGetLastError();
        return fail(ctx, RT_E_CUDA, "batch engine: step capture failed (%s)", cudaGetErrorString(ce != cudaSuccess ? ce : ee));
    }
    return RT_OK;
}

// Tensor-parallel set-up of a many-sequence engine (nranks 1: none).
struct TpInit {
    int nranks = 1, rank = 0;
    ncclUniqueId id{};
};

// Many-sequence mode: `rows` sequences with their own caches of `cap`
// positions and one captured step (on `tp->nranks` GPUs, this rank's shard).
// Rows mode: up to `rows` positions of the decoder's sequence per call, on
// the decoder's caches (cap = the decoder's), launched eagerly.
int create_engine(rt_dec* d, int rows, int cap, bool rows_mode, const TpInit* tp, rt_batch** out) {
    rt_ctx* ctx = d->ctx;
    RT_CHECK_CUDA(ctx, cudaSetDevice(ctx->device));
    rt_batch* t = new rt_batch;
    t->dec = d;
    t->ctx = ctx;
    t->rows_mode = rows_mode;
    t->B = rows;
    t->cap = rows_mode ? d->cap : cap;
    t->H = d->H;
    t->D = d->D;
    t->NQ = d->NQ;
    t->NKV = d->NKV;
    t->F = d->F;
    t->V = d->V;
    t->NL = d->NL;
    t->qkv_rows = d->qkv_rows;
    const int G = t->NQ / t->NKV;
    cap = t->cap;
    t->nranks = tp ? tp->nranks : 1;
    t->rank = tp ? tp->rank : 0;
    t->v0 = static_cast<int>(static_cast<int64_t>(t->V) * t->rank / t->nranks);
    t->vr = static_cast<int>(static_cast<int64_t>(t->V) * (t->rank + 1) / t->nranks) - t->v0;
    // Enough attention items to fill the SMs about four times over (attention.cu path).
    t->nsplit = std::max(1, std::min(64, (4 * ctx->num_sms + rows * t->NKV - 1) / (rows * t->NKV)));
    t->chunk_path = rt::attn_chunk_supported(t->D, G);
    auto bail = [&](int rc) {
        release(t);
        return rc;
    };
    if (t->H % 4 || t->F % 4 || (t->NQ * t->D) % 4)  // the row kernels' float4 slices
        return bail(fail(ctx, RT_E_SHAPE, "batch engine: hidden %d / FFN %d / heads x head_dim %d not multiples of 4",
                         t->H, t->F, t->NQ * t->D));
    if (rows_mode && !t->chunk_path)
        return bail(fail(ctx, RT_E_SHAPE, "rows engine: head_dim %d with %d query heads per KV head is not supported", t->D, G));
    int rc;
    if (rows_mode) {
        t->seq_kv = 0;
        t->kv_lstride = static_cast<int64_t>(t->NKV) * cap * t->D;
        t->kv_k0 = d->kcache;
        t->kv_v0 = d->vcache;
        t->rope = d->rope;
    } else {
        t->kv_lstride = 2LL * t->NKV * cap * t->D;
        t->seq_kv = static_cast<int64_t>(t->NL) * t->kv_lstride;
        if ((rc = balloc(t, reinterpret_cast<void**>(&t->kv), sizeof(float) * t->seq_kv * rows, "batch KV caches")) != RT_OK)
            return bail(rc);
        RT_CHECK_CUDA(ctx, cudaMemsetAsync(t->kv, 0, sizeof(float) * t->seq_kv * rows, ctx->stream));
        t->kv_k0 = t->kv;
        t->kv_v0 = t->kv + static_cast<int64_t>(t->NKV) * cap * t->D;
        const size_t tab = static_cast<size_t>(cap) * (t->D / 2);
        std::vector<float> r(4 * tab);
        const rt_gemma3_cfg& c = d->cfg;
        rt::rope_table(c.rope_theta_local, c.rope_freq_scale_local, t->D, cap, &r[0], &r[tab]);
        rt::rope_table(c.rope_theta_global, c.rope_freq_scale_global, t->D, cap, &r[2 * tab], &r[3 * tab]);
        if ((rc = balloc(t, reinterpret_cast<void**>(&t->rope), r.size() * 4, "batch rope tables")) != RT_OK) return bail(rc);
        if (cudaMemcpy(t->rope, r.data(), r.size() * 4, cudaMemcpyHostToDevice) != cudaSuccess)
            return bail(fail(ctx, RT_E_CUDA, "batch engine: upload rope tables"));
    }
    const int64_t B = rows;
    t->logit_rows = rows_mode ? std::min(rows, kRowsMaxLogitRows) : rows;
    const size_t part_floats_attn =
        t->chunk_path ? rt::attn_chunk_part_floats(rows, t->NKV, rt::attn_chunk_count(cap, 0), G, t->D)
                      : static_cast<size_t>(B) * t->NKV * t->nsplit * G * rt::attn_part_stride(t->D);
    const int64_t kmax = std::max<int64_t>({t->H, static_cast<int64_t>(t->NQ) * t->D, t->F});
    if ((rc = balloc(t, reinterpret_cast<void**>(&t->xa), sizeof(uint16_t) * B * kmax + 256, "batch GEMM input")) != RT_OK ||
        (rc = balloc(t, reinterpret_cast<void**>(&t->xscale), sizeof(float) * B, "batch GEMM row scales")) != RT_OK ||
        (rc = balloc(t, reinterpret_cast<void**>(&t->xa32), sizeof(float) * std::min<int64_t>(B, rt::kRowsMaxM) * kmax,
                     "batch GEMM input (f32)")) != RT_OK ||
        (rc = balloc(t, reinterpret_cast<void**>(&t->qkv), sizeof(float) * B * t->qkv_rows, "batch qkv")) != RT_OK ||
        (rc = balloc(t, reinterpret_cast<void**>(&t->attn), sizeof(float) * B * t->NQ * t->D, "batch attention")) != RT_OK ||
        (rc = balloc(t, reinterpret_cast<void**>(&t->resid[0]), sizeof(float) * B * t->H, "batch residual")) != RT_OK ||
        (rc = balloc(t, reinterpret_cast<void**>(&t->resid[1]), sizeof(float) * B * t->H, "batch residual")) != RT_OK ||
        (rc = balloc(t, reinterpret_cast<void**>(&t->logits), sizeof(float) * t->logit_rows * t->vr, "batch logits")) != RT_OK ||
        (rc = balloc(t, reinterpret_cast<void**>(&t->attn_part), sizeof(float) * part_floats_attn, "batch attention partials")) != RT_OK ||
        (t->chunk_path &&
         (rc = balloc(t, reinterpret_cast<void**>(&t->q_rot), sizeof(float) * B * t->NQ * t->D, "batch rotated queries")) != RT_OK) ||
        (rc = balloc(t, reinterpret_cast<void**>(&t->counters), sizeof(uint32_t) * B * t->NKV, "batch counters")) != RT_OK ||
        (rc = balloc(t, reinterpret_cast<void**>(&t->tokens), sizeof(int32_t) * B, "batch tokens")) != RT_OK ||
        (rc = balloc(t, reinterpret_cast<void**>(&t->pos), sizeof(int32_t) * B, "batch positions")) != RT_OK)
        return bail(rc);
    RT_CHECK_CUDA(ctx, cudaMemsetAsync(t->counters, 0, sizeof(uint32_t) * B * t->NKV, ctx->stream));
    RT_CHECK_CUDA(ctx, cudaMemsetAsync(t->tokens, 0, sizeof(int32_t) * B, ctx->stream));
    RT_CHECK_CUDA(ctx, cudaMemsetAsync(t->pos, 0, sizeof(int32_t) * B, ctx->stream));
    const int64_t rec_rows = std::max<int64_t>(B, t->logit_rows);  // rows a greedy pass covers
    if ((rc = balloc(t, reinterpret_cast<void**>(&t->am_send), sizeof(uint32_t) * kTpWords * kGreedySlices * rec_rows,
                     "greedy records")) != RT_OK)
        return bail(rc);
    if (cudaMallocHost(reinterpret_cast<void**>(&t->h_err), sizeof(int)) != cudaSuccess) return bail(fail(ctx, RT_E_NOMEM, "pinned error word"));
    *t->h_err = 0;
    if (t->nranks > 1) {
        const char* why = nullptr;
        if (!(t->nccl = rt::nccl_api(&why))) return bail(fail(ctx, RT_E_CUDA, "tensor parallel: NCCL unavailable (%s)", why));
        if ((rc = balloc(t, reinterpret_cast<void**>(&t->ar_buf), sizeof(float) * B * t->H, "tp all-reduce buffer")) != RT_OK ||
            (rc = balloc(t, reinterpret_cast<void**>(&t->am_recv), sizeof(uint32_t) * kTpWords * kGreedySlices * rec_rows * t->nranks,
                         "tp greedy records")) != RT_OK)
            return bail(rc);
        RT_CHECK_CUDA(ctx, cudaStreamSynchronize(ctx->stream));
        const ncclResult_t nr = t->nccl->comm_init_rank(&t->comm, t->nranks, tp->id, t->rank);
        if (nr != ncclSuccess) {
            t->comm = nullptr;
            return bail(fail(ctx, RT_E_CUDA, "tensor parallel: ncclCommInitRank: %s", t->nccl->error_string(nr)));
        }
    }
    if (rt::gemm_q4k_prepare() != cudaSuccess || rt::attention_prepare() != cudaSuccess ||
        rt::attn_chunk_prepare() != cudaSuccess)
        return bail(fail(ctx, RT_E_CUDA, "batch engine: kernel attributes"));
    auto smem_limit = [](auto kernel, size_t bytes) {
        return bytes <= 48 * 1024 ||
               cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(bytes)) == cudaSuccess;
    };
    if (!smem_limit(gelu_rows_kernel, sizeof(float) * t->F) || !smem_limit(f16_rows_kernel, sizeof(float) * t->NQ * t->D) ||
        !smem_limit(resid_norm_rows_kernel, sizeof(float) * 4 * t->H))
        return bail(fail(ctx, RT_E_CUDA, "batch engine: row kernel attributes"));
    if (!rows_mode) {
        // the step's GEMM plans and tensor maps (A is xa, read as [B][K]), then its capture
        if (!build_plan(t, rows, 0, rows, &t->plan)) return bail(fail(ctx, RT_E_SHAPE, "rt_batch_create: no GEMM geometry"));
        if ((rc = grow_parts(t, t->plan.part_floats)) != RT_OK) return bail(rc);
        if ((rc = capture_step(t)) != RT_OK) return bail(rc);
    }
    RT_CHECK_CUDA(ctx, cudaStreamSynchronize(ctx->stream));
    *out = t;
    return RT_OK;
}

// Rows mode: tokens[0..m) at positions start, start + 1, ... through every
// layer (their K/V appended to the decoder's caches); logits of the last
// `lm_rows` rows (0: none) to host `logits` ([lm_rows][V]).
int rows_run(rt_batch* t, const int32_t* tokens, int m, int start, int lm_rows, float* logits) {
    rt_ctx* ctx = t->ctx;
    cudaStream_t s = ctx->stream;
    std::vector<int32_t> pos(m);
    for (int i = 0; i < m; ++i) pos[i] = start + i;
    RT_CHECK_CUDA(ctx, cudaMemcpyAsync(t->tokens, tokens, sizeof(int32_t) * m, cudaMemcpyHostToDevice, s));
    RT_CHECK_CUDA(ctx, cudaMemcpyAsync(t->pos, pos.data(), sizeof(int32_t) * m, cudaMemcpyHostToDevice, s));
    rt_batch::RowsGraph* rg = nullptr;
    for (rt_batch::RowsGraph* r : t->rows_graphs)
        if (r->plan.m == m && r->plan.lm_rows == lm_rows) rg = r;
    if (!rg) {
        // a new shape: its plan, then one captured step replayed from now on
        auto* r = new rt_batch::RowsGraph;
        if (!build_plan(t, m, m - lm_rows, lm_rows, &r->plan)) {
            delete r;
            return fail(ctx, RT_E_SHAPE, "rows engine: no GEMM geometry for %d rows", m);
        }
        if (r->plan.part_floats > t->part_cap || t->rows_graphs.size() >= 32)
            drop_rows_graphs(t);  // the graphs hold the old split-K buffer
        const int rc = grow_parts(t, r->plan.part_floats);
        if (rc != RT_OK) {
            delete r;
            return rc;
        }
        cudaError_t ce = cudaStreamBeginCapture(s, cudaStreamCaptureModeThreadLocal);
        if (ce == cudaSuccess) {
            const cudaError_t ee = enqueue(t, r->plan, s, false);
            ce = cudaStreamEndCapture(s, &r->graph);
            if (ee != cudaSuccess) ce = ee;
        }
        if (ce == cudaSuccess) ce = cudaGraphInstantiate(&r->exec, r->graph, 0);
        if (ce != cudaSuccess) {
            cudaGetLastError();
            if (r->graph) cudaGraphDestroy(r->graph);
            delete r;
            return fail(ctx, RT_E_CUDA, "rows engine: step capture failed (%s)", cudaGetErrorString(ce));
        }
        t->rows_graphs.push_back(r);
        rg = r;
    }
    RT_CHECK_CUDA(ctx, cudaGraphLaunch(rg->exec, s));
    if (logits && lm_rows > 0)
        RT_CHECK_CUDA(ctx, cudaMemcpyAsync(logits, t->logits, sizeof(float) * lm_rows * t->vr, cudaMemcpyDeviceToHost, s));
    RT_CHECK_CUDA(ctx, cudaMemcpyAsync(t->h_err, ctx->d_err, sizeof(int), cudaMemcpyDeviceToHost, s));
    RT_CHECK_CUDA(ctx, cudaStreamSynchronize(s));
    return check_error_word(t);
}

int rows_engine(rt_dec* d, rt_batch** out) {
    if (!d->rows) {
        const int rc = create_engine(d, kRowsMax, 0, true, nullptr, &d->rows);
        if (rc != RT_OK) return rc;
    }
    *out = d->rows;
    return RT_OK;
}

int check_rows_args(rt_dec* d, const int32_t* tokens, int32_t n, int32_t start_pos, const char* who) {
    if (!tokens && n > 0) return fail(d->ctx, RT_E_INVAL, "%s: null tokens", who);
    if (start_pos < 0 || static_cast<int64_t>(start_pos) + n > d->cap)
        return fail(d->ctx, RT_E_STATE, "%s: positions %d..%d outside the %d-position cache", who, start_pos,
                    start_pos + n - 1, d->cap);
    for (int i = 0; i < n; ++i)
        if (tokens[i] < 0 || tokens[i] >= d->V) return fail(d->ctx, RT_E_INVAL, "%s: token %d out of range", who, tokens[i]);
    return RT_OK;
}

}  // namespace

namespace rt {
void rows_engine_free(rt_batch* t) { release(t); }
}  // namespace rt

extern "C" {

int rt_batch_create(rt_dec* d, int32_t nseq, int32_t cap, rt_batch** out) {
    if (!d || !out) return RT_E_INVAL;
    *out = nullptr;
    if (nseq < 1 || nseq > 1024 || cap < 1) return fail(d->ctx, RT_E_SHAPE, "rt_batch_create: nseq %d / cap %d", nseq, cap);
    return create_engine(d, nseq, cap, false, nullptr, out);
}

void rt_batch_destroy(rt_batch* t) {
    if (!t) return;
    cudaSetDevice(t->ctx->device);
    cudaStreamSynchronize(t->ctx->stream);
    release(t);
}

int rt_batch_set(rt_batch* t, const int32_t* tokens, const int32_t* positions) {
    if (!t || !tokens || !positions) return t ? fail(t->ctx, RT_E_INVAL, "rt_batch_set: null argument") : RT_E_INVAL;
    for (int b = 0; b < t->B; ++b) {
        if (tokens[b] < 0 || tokens[b] >= t->V) return fail(t->ctx, RT_E_INVAL, "rt_batch_set: token %d out of range", tokens[b]);
        if (positions[b] < 0 || positions[b] >= t->cap)
            return fail(t->ctx, RT_E_STATE, "rt_batch_set: position %d outside the cache", positions[b]);
    }
    RT_CHECK_CUDA(t->ctx, cudaMemcpyAsync(t->tokens, tokens, sizeof(int32_t) * t->B, cudaMemcpyHostToDevice, t->ctx->stream));
    RT_CHECK_CUDA(t->ctx, cudaMemcpyAsync(t->pos, positions, sizeof(int32_t) * t->B, cudaMemcpyHostToDevice, t->ctx->stream));
    RT_CHECK_CUDA(t->ctx, cudaStreamSynchronize(t->ctx->stream));
    return RT_OK;
}

int rt_batch_step(rt_batch* t, float* logits, int32_t* next_tokens) {
    if (!t) return RT_E_INVAL;
    cudaStream_t s = t->ctx->stream;
    RT_CHECK_CUDA(t->ctx, cudaGraphLaunch(t->exec, s));
    if (logits)
        RT_CHECK_CUDA(t->ctx, cudaMemcpyAsync(logits, t->logits, sizeof(float) * t->B * t->vr, cudaMemcpyDeviceToHost, s));
    if (next_tokens)
        RT_CHECK_CUDA(t->ctx, cudaMemcpyAsync(next_tokens, t->tokens, sizeof(int32_t) * t->B, cudaMemcpyDeviceToHost, s));
    RT_CHECK_CUDA(t->ctx, cudaMemcpyAsync(t->h_err, t->ctx->d_err, sizeof(int), cudaMemcpyDeviceToHost, s));
    RT_CHECK_CUDA(t->ctx, cudaStreamSynchronize(s));
    return check_error_word(t);
}

int rt_batch_generate(rt_batch* t, int32_t steps, int flags) {
    if (!t) return RT_E_INVAL;
    if (flags != RT_HOST && flags != RT_DEVICE) return fail(t->ctx, RT_E_INVAL, "rt_batch_generate: bad flags");
    for (int i = 0; i < steps; ++i) RT_CHECK_CUDA(t->ctx, cudaGraphLaunch(t->exec, t->ctx->stream));
    if (flags == RT_DEVICE) return RT_OK;
    RT_CHECK_CUDA(t->ctx, cudaMemcpyAsync(t->h_err, t->ctx->d_err, sizeof(int), cudaMemcpyDeviceToHost, t->ctx->stream));
    RT_CHECK_CUDA(t->ctx, cudaStreamSynchronize(t->ctx->stream));
    return check_error_word(t);
}

int rt_batch_synth_kv(rt_batch* t, uint64_t seed, int32_t seq_len) {
    if (!t) return RT_E_INVAL;
    if (seq_len < 0 || seq_len >= t->cap) return fail(t->ctx, RT_E_STATE, "rt_batch_synth_kv: length %d outside the cache", seq_len);
    const int64_t n = t->seq_kv * t->B;
    synth_kv_kernel<<<static_cast<unsigned>(std::min<int64_t>((n + 255) / 256, 65536)), 256, 0, t->ctx->stream>>>(t->kv, n, seed);
    fill_i32_kernel<<<(t->B + 255) / 256, 256, 0, t->ctx->stream>>>(t->pos, t->B, seq_len);
    RT_CHECK_CUDA(t->ctx, cudaGetLastError());
    RT_CHECK_CUDA(t->ctx, cudaStreamSynchronize(t->ctx->stream));
    return RT_OK;
}

int rt_batch_info(const rt_batch* t, uint64_t* bytes, int32_t* launches_per_step) {
    if (!t) return RT_E_INVAL;
    if (bytes) *bytes = t->dev_bytes;
    if (launches_per_step) *launches_per_step = t->launches;
    return RT_OK;
}

int rt_nccl_unique_id(void* id_out) {
    if (!id_out) return RT_E_INVAL;
    const char* why = nullptr;
    const rt::NcclApi* api = rt::nccl_api(&why);
    if (!api) return RT_E_CUDA;
    ncclUniqueId id;
    if (api->get_unique_id(&id) != ncclSuccess) return RT_E_CUDA;
    memcpy(id_out, &id, sizeof(id));
    return RT_OK;
}

int rt_tp_create(rt_dec* shard, const void* nccl_id, int32_t nranks, int32_t rank, int32_t nseq, int32_t cap,
                 rt_batch** out) {
    if (!shard || !out || (nranks > 1 && !nccl_id)) return shard ? fail(shard->ctx, RT_E_INVAL, "rt_tp_create: null argument") : RT_E_INVAL;
    *out = nullptr;
    if (nranks < 1 || rank < 0 || rank >= nranks || nseq < 1 || nseq > 1024 || cap < 1)
        return fail(shard->ctx, RT_E_SHAPE, "rt_tp_create: nranks %d rank %d nseq %d cap %d", nranks, rank, nseq, cap);
    TpInit tp;
    tp.nranks = nranks;
    tp.rank = rank;
    if (nranks > 1) memcpy(&tp.id, nccl_id, sizeof(tp.id));
    return create_engine(shard, nseq, cap, false, &tp, out);
}

int rt_tp_peer_handle(rt_batch* t, void* handle_out) {
    if (!t || !handle_out) return t ? fail(t->ctx, RT_E_INVAL, "rt_tp_peer_handle: null argument") : RT_E_INVAL;
    if (t->nranks < 2 || t->nranks > kMaxRanks || 2 * t->NL + 1 > 255)
        return fail(t->ctx, RT_E_SHAPE, "rt_tp_peer_handle: %d ranks, %d layers", t->nranks, t->NL);
    RT_CHECK_CUDA(t->ctx, cudaSetDevice(t->ctx->device));
    if (!t->ar_sym) {
        const size_t bytes = kArFlagBytes + sizeof(float) * 2 * t->nranks * static_cast<size_t>(t->B) * t->H;
        int rc = balloc(t, reinterpret_cast<void**>(&t->ar_sym), bytes, "tp peer all-reduce buffer");
        if (rc == RT_OK) rc = balloc(t, reinterpret_cast<void**>(&t->step_ctr), sizeof(int32_t), "tp step counter");
        if (rc != RT_OK) return rc;
        // zeroed flags before any peer can see the handle
        RT_CHECK_CUDA(t->ctx, cudaMemsetAsync(t->ar_sym, 0, bytes, t->ctx->stream));
        RT_CHECK_CUDA(t->ctx, cudaMemsetAsync(t->step_ctr, 0, sizeof(int32_t), t->ctx->stream));
        RT_CHECK_CUDA(t->ctx, cudaStreamSynchronize(t->ctx->stream));
    }
    cudaIpcMemHandle_t h;
    RT_CHECK_CUDA(t->ctx, cudaIpcGetMemHandle(&h, t->ar_sym));
    memcpy(handle_out, &h, sizeof(h));
    return RT_OK;
}

int rt_tp_peer_open(rt_batch* t, const void* handles) {
    if (!t || !handles) return t ? fail(t->ctx, RT_E_INVAL, "rt_tp_peer_open: null argument") : RT_E_INVAL;
    if (!t->ar_sym) return fail(t->ctx, RT_E_STATE, "rt_tp_peer_open: call rt_tp_peer_handle first");
    if (t->p2p) return RT_OK;
    RT_CHECK_CUDA(t->ctx, cudaSetDevice(t->ctx->device));
    const uint8_t* hb = static_cast<const uint8_t*>(handles);
    for (int r = 0; r < t->nranks; ++r) {
        if (r == t->rank) {
            t->peers.base[r] = t->ar_sym;
            continue;
        }
        cudaIpcMemHandle_t h;
        memcpy(&h, hb + r * sizeof(h), sizeof(h));
        void* p = nullptr;
        const cudaError_t e = cudaIpcOpenMemHandle(&p, h, cudaIpcMemLazyEnablePeerAccess);
        if (e != cudaSuccess) {
            cudaGetLastError();
            return fail(t->ctx, RT_E_CUDA, "rt_tp_peer_open: rank %d's buffer: %s", r, cudaGetErrorString(e));
        }
        t->opened[r] = p;
        t->peers.base[r] = static_cast<uint8_t*>(p);
    }
    t->p2p = true;
    const int rc = capture_step(t);
    if (rc != RT_OK) t->p2p = false;
    return rc;
}

int rt_batch_vocab_slice(const rt_batch* t, int32_t* v0, int32_t* vr) {
    if (!t) return RT_E_INVAL;
    if (v0) *v0 = t->v0;
    if (vr) *vr = t->vr;
    return RT_OK;
}

int rt_decoder_prefill_gemm(rt_dec* d, const int32_t* tokens, int32_t n, int32_t start_pos, float* last_logits) {
    if (!d) return RT_E_INVAL;
    int rc = check_rows_args(d, tokens, n, start_pos, "rt_decoder_prefill_gemm");
    if (rc != RT_OK || n <= 0) return n < 0 ? fail(d->ctx, RT_E_SHAPE, "rt_decoder_prefill_gemm: n = %d", n) : rc;
    rt_batch* t = nullptr;
    if ((rc = rows_engine(d, &t)) != RT_OK) return rc;
    for (int off = 0; off < n; off += kRowsMax) {
        const int m = std::min(kRowsMax, n - off);
        const bool last = off + m == n;
        rc = rows_run(t, tokens + off, m, start_pos + off, last && last_logits ? 1 : 0, last ? last_logits : nullptr);
        if (rc != RT_OK) return rc;
    }
    return RT_OK;
}

int rt_decoder_step_batch(rt_dec* d, const int32_t* tokens, int32_t m, int32_t start_pos, float* logits) {
    if (!d) return RT_E_INVAL;
    if (m < 1 || m > kRowsMaxLogitRows)
        return fail(d->ctx, RT_E_SHAPE, "rt_decoder_step_batch: %d positions (1..%d)", m, kRowsMaxLogitRows);
    int rc = check_rows_args(d, tokens, m, start_pos, "rt_decoder_step_batch");
    if (rc != RT_OK) return rc;
    rt_batch* t = nullptr;
    if ((rc = rows_engine(d, &t)) != RT_OK) return rc;
    return rows_run(t, tokens, m, start_pos, logits ? m : 0, logits);
}

// Test hook: the peer all-reduce kernel run by one process as rank 0 of two,
// the second rank's buffer a local zeroed allocation whose flag never rises.
// The first call's bounded wait must give up (error word kErrGridTimeout)
// and every later call must return without waiting.  Nothing faults and no
// wait is unbounded: the flag wait ends after 2 s of globaltimer.
int rt_test_peer_allreduce_lonely(rt_ctx* ctx, int* err_word, float* first_ms, float* second_ms) {
    if (!ctx || !err_word || !first_ms || !second_ms) return fail(ctx, RT_E_INVAL, "rt_test_peer_allreduce_lonely: null");
    RT_CHECK_CUDA(ctx, cudaSetDevice(ctx->device));
    const int64_t count = 4096;
    const size_t bytes = kArFlagBytes + sizeof(float) * 2 * kMaxRanks * count;
    void *b0 = nullptr, *b1 = nullptr, *src = nullptr, *out = nullptr, *ctr = nullptr, *err = nullptr;
    cudaEvent_t e0 = nullptr, e1 = nullptr, e2 = nullptr;
    cudaError_t e = cudaSuccess;
    auto chk = [&](cudaError_t r) {
        if (e == cudaSuccess) e = r;
        return e == cudaSuccess;
    };
    chk(cudaMalloc(&b0, bytes));
    chk(cudaMalloc(&b1, bytes));
    chk(cudaMalloc(&src, sizeof(float) * count));
    chk(cudaMalloc(&out, sizeof(float) * count));
    chk(cudaMalloc(&ctr, sizeof(int32_t)));
    chk(cudaMalloc(&err, sizeof(int)));
    if (e == cudaSuccess) {
        chk(cudaMemsetAsync(b0, 0, bytes, ctx->stream));
        chk(cudaMemsetAsync(b1, 0, bytes, ctx->stream));
        chk(cudaMemsetAsync(src, 0, sizeof(float) * count, ctx->stream));
        chk(cudaMemsetAsync(ctr, 0, sizeof(int32_t), ctx->stream));
        chk(cudaMemsetAsync(err, 0, sizeof(int), ctx->stream));
        chk(cudaEventCreate(&e0));
        chk(cudaEventCreate(&e1));
        chk(cudaEventCreate(&e2));
    }
    if (e == cudaSuccess) {
        PeerBufs pb = {};
        pb.base[0] = static_cast<uint8_t*>(b0);
        pb.base[1] = static_cast<uint8_t*>(b1);
        chk(cudaEventRecord(e0, ctx->stream));
        peer_allreduce_kernel<<<kArCtas, 256, 0, ctx->stream>>>(static_cast<const float*>(src), 1,
                                                                static_cast<float*>(out), count, count, pb, 2, 0, 0, 0u,
                                                                static_cast<const int32_t*>(ctr), static_cast<int*>(err));
        chk(cudaGetLastError());
        chk(cudaEventRecord(e1, ctx->stream));
        peer_allreduce_kernel<<<kArCtas, 256, 0, ctx->stream>>>(static_cast<const float*>(src), 1,
                                                                static_cast<float*>(out), count, count, pb, 2, 0, 1, 1u,
                                                                static_cast<const int32_t*>(ctr), static_cast<int*>(err));
        chk(cudaGetLastError());
        chk(cudaEventRecord(e2, ctx->stream));
        chk(cudaMemcpyAsync(err_word, err, sizeof(int), cudaMemcpyDeviceToHost, ctx->stream));
        chk(cudaStreamSynchronize(ctx->stream));
        chk(cudaEventElapsedTime(first_ms, e0, e1));
        chk(cudaEventElapsedTime(second_ms, e1, e2));
    }
    for (void* q : {b0, b1, src, out, ctr, err})
        if (q) cudaFree(q);
    for (cudaEvent_t ev : {e0, e1, e2})
        if (ev) cudaEventDestroy(ev);
    RT_CHECK_CUDA(ctx, e);
    return RT_OK;
}

}  // extern "C"
