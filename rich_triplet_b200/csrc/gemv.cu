// gemv.cu -- Q4_K / BF16 GEMV kernel for sm_100a.
//
// Work decomposition
//   * A CTA owns a contiguous range of rows.  Its rows are contiguous bytes in
//     HBM, so they are streamed into shared memory by 1-D TMA bulk copies
//     (cp.async.bulk, no tensor map, no multicast) of `rows_per_stage` rows,
//     through `nbuf` stage buffers completed on mbarriers.  The first copies are
//     issued before griddepcontrol.wait, so under programmatic dependent launch
//     the weight stream starts while the previous kernel is still finishing.
//   * Threads form groups of 4 lanes.  A group owns one 256-column segment of
//     every row (one Q4_K super-block, or 256 BF16 values); lane c of the group
//     owns columns [64c, 64c+64) of that segment, so it keeps those 64 values of
//     x in registers for the whole kernel and never re-reads x.
//     Groups with the same segment index ("row lanes") take alternate rows.
//   * Per (row, segment) the 4 lanes' partial sums are reduced with two shuffles
//     and stored to shared memory; after each stage one thread per row adds the
//     segment partials in a fixed order (deterministic) and runs the epilogue.
//
// Q4_K arithmetic (block layout: src/autograd2.rs:1003-1042; dot product:
// Q4KMat::dot_row, src/autograd2.rs:1637-1702)
//   A 4-bit quant q becomes the float 128 + q with one byte permute
//   (0x43000000 | q << 16), so sum (128+q) x = 128 sum x + sum q x, and
//   sum q x = acc - 128 * sum x, where sum x over each 32-column sub-block is
//   computed once per kernel.  The sub-block contribution is then
//   d*sc*(sum q x) - dmin*m*(sum x), the same factorisation dot_row uses.
//   Accumulation is in f32 with packed f32x2 FMAs.
#include <algorithm>
#include <cstdio>

#include "common.cuh"
#include "gemv.cuh"

namespace rt {

namespace {

constexpr int kMaxNbuf = 4;

__device__ __forceinline__ float gelu_tanh_dev(float x) {
    // TensorNode::gelu_tanh (src/autograd2.rs:3082-3091): x*0.5*(1+tanh(s*(x+c*x^3))),
    // evaluated without FMA contraction in the reference's operation order.
    const float kS = 0.7978845608028654f, kC = 0.044715f;
    float x3 = __fmul_rn(__fmul_rn(__fmul_rn(kC, x), x), x);
    float inner = __fmul_rn(kS, __fadd_rn(x, x3));
    return __fmul_rn(__fmul_rn(x, 0.5f), __fadd_rn(1.0f, tanhf(inner)));
}

// Quant nibble byte (0..15 in byte b of `v`) -> float 128 + q.
template <int B>
__device__ __forceinline__ float q_plus_128(uint32_t v) {
    return __uint_as_float(__byte_perm(v, 0x43000000u, 0x7044u | (B << 8)));
}

// Byte b (0..3) of v as an exact float.
__device__ __forceinline__ float byte_to_float(uint32_t v, uint32_t sel) {
    return __uint_as_float(__byte_perm(v, 0x4B000000u, sel)) - 8388608.0f;
}

struct SmemLayout {
    uint64_t* full;  // [nbuf]
    float* part;     // [2][rows_per_stage][nseg]
    float* xs;       // [K] (norm prologues)
    float* red;      // [32]
    int* flag;       // [4]
    uint8_t* stage;  // [nbuf][stage_bytes], 128-byte aligned
};

__device__ __forceinline__ SmemLayout carve(uint8_t* smem, const GemvArgs& a, bool need_xs) {
    SmemLayout L;
    size_t off = 0;
    L.full = reinterpret_cast<uint64_t*>(smem + off);
    off += sizeof(uint64_t) * kMaxNbuf;
    L.red = reinterpret_cast<float*>(smem + off);
    off += sizeof(float) * 32;
    L.flag = reinterpret_cast<int*>(smem + off);
    off += sizeof(int) * 4;
    L.part = reinterpret_cast<float*>(smem + off);
    off += sizeof(float) * 2 * a.rows_per_stage * a.nseg;
    off = (off + 15) & ~size_t(15);
    L.xs = reinterpret_cast<float*>(smem + off);
    if (need_xs) off += sizeof(float) * a.K;
    off = (off + 127) & ~size_t(127);
    L.stage = smem + off;
    return L;
}

template <int KIND, int PRO, int EPI>
__global__ void __launch_bounds__(512) gemv_kernel(const GemvArgs a) {
    extern __shared__ __align__(128) uint8_t smem[];
    constexpr bool kNeedXs = PRO != kProPlain;
    SmemLayout S = carve(smem, a, kNeedXs);

    const int tid = threadIdx.x;
    const int nthr = blockDim.x;
    const int gi = tid >> 2;
    const int c = tid & 3;
    const int seg = gi % a.nseg;
    const int rlane = gi / a.nseg;
    const bool active = rlane < a.rl;
    const uint32_t gmask = 0xFu << ((tid & 31) & ~3);

    // Contiguous, balanced row range of this CTA (in units of `pair` rows).
    const int64_t units = a.rows / a.pair;
    const int64_t r_begin = (units * blockIdx.x / gridDim.x) * a.pair;
    const int64_t r_end = (units * (blockIdx.x + 1) / gridDim.x) * a.pair;
    const int64_t nrows = r_end - r_begin;
    const int R = a.rows_per_stage;
    const int nst = static_cast<int>((nrows + R - 1) / R);

    if (tid == 0) {
        for (int b = 0; b < a.nbuf; ++b) mbar_init(&S.full[b], 1);
        fence_mbar_init();
        S.flag[0] = 0;
    }
    __syncthreads();

    const uint64_t pol = l2_evict_first_policy();
    int issued = 0;  // stages whose copy thread 0 has issued (thread 0 only)
    auto issue = [&](int st) {
        ++issued;
        const int64_t r0 = r_begin + static_cast<int64_t>(st) * R;
        const int64_t nr = min(static_cast<int64_t>(R), r_end - r0);
        const uint32_t bytes = static_cast<uint32_t>(nr * a.row_bytes);
        const int b = st % a.nbuf;
        uint8_t* dst = S.stage + static_cast<size_t>(b) * a.stage_bytes;
        mbar_arrive_expect_tx(&S.full[b], bytes);
        bulk_g2s(dst, a.w + r0 * a.row_bytes, bytes, &S.full[b], pol);
    };
    // Weights do not depend on the previous kernel: start streaming now.
    if (tid == 0) {
        for (int st = 0; st < min(a.nbuf, nst); ++st) issue(st);
    }
    pdl_launch_dependents();
    pdl_wait();

    // ---------------- prologue: build x ----------------
    const int K = a.K;
    if constexpr (PRO == kProResidNorm || PRO == kProEmbedNorm) {
        const float inv_d = 1.0f / static_cast<float>(K);
        float ss = 0.f;
        if constexpr (PRO == kProResidNorm) {
            // post-norm of the sub-layer output, then the residual add
            // (Gemma3Block::forward_cached, src/transformer4.rs:1954-1964)
            for (int i = tid; i < K; i += nthr) {
                float v = a.src[i];
                ss += v * v;
            }
            ss = block_sum(ss, S.red);
            const float r1 = 1.0f / sqrtf(ss * inv_d + a.eps);
            float ss2 = 0.f;
            for (int i = tid; i < K; i += nthr) {
                float t = __fmul_rn(__fmul_rn(a.src[i], r1), __fadd_rn(1.0f, a.g_post[i]));
                float n = __fadd_rn(a.resid_in[i], t);
                S.xs[i] = n;
                ss2 += n * n;
                if (blockIdx.x == 0) a.resid_out[i] = n;
            }
            ss = block_sum(ss2, S.red);
        } else {
            // embedding row * sqrt(hidden) (src/transformer4.rs:2360-2364)
            const int64_t tok = static_cast<int64_t>(*a.token);
            const uint16_t* erow = a.embed + tok * K;
            for (int i = tid; i < K; i += nthr) {
                float n = __fmul_rn(bf16_bits_to_f32(erow[i]), a.embed_scale);
                S.xs[i] = n;
                ss += n * n;
                if (blockIdx.x == 0) a.resid_out[i] = n;
            }
            ss = block_sum(ss, S.red);
        }
        // pre-norm producing the projection input (rms_norm_gemma3,
        // src/autograd2.rs:3477-3496)
        const float r2 = 1.0f / sqrtf(ss * inv_d + a.eps);
        for (int i = tid; i < K; i += nthr) S.xs[i] = __fmul_rn(__fmul_rn(S.xs[i], r2), __fadd_rn(1.0f, a.g_pre[i]));
        __syncthreads();
    }
    const float* xsrc = kNeedXs ? S.xs : a.x;

    // ---------------- this lane's 64 columns of x ----------------
    const int col0 = seg * 256 + c * 64;
    float2 xv[32];
    float sx_lo = 0.f, sx_hi = 0.f;
    int nvalid16 = 0;  // BF16: 16-byte chunks of this lane that hold real columns
    if (active) {
        if constexpr (KIND == kQ4K) {
#pragma unroll
            for (int j = 0; j < 16; ++j) xv[j] = make_float2(xsrc[col0 + 2 * j], xsrc[col0 + 2 * j + 1]);
#pragma unroll
            for (int j = 0; j < 16; ++j) xv[16 + j] = make_float2(xsrc[col0 + 32 + 2 * j], xsrc[col0 + 33 + 2 * j]);
#pragma unroll
            for (int j = 0; j < 16; ++j) sx_lo = sx_lo + xv[j].x + xv[j].y;
#pragma unroll
            for (int j = 0; j < 16; ++j) sx_hi = sx_hi + xv[16 + j].x + xv[16 + j].y;
        } else {
            const int nv = max(0, min(64, K - col0));
            nvalid16 = nv / 8;
#pragma unroll
            for (int j = 0; j < 32; ++j)
                xv[j] = (2 * j < nv) ? make_float2(xsrc[col0 + 2 * j], xsrc[col0 + 2 * j + 1]) : make_float2(0.f, 0.f);
        }
    }

    // ---------------- stream the rows ----------------
    float best_v = -INFINITY;
    int64_t best_i = -1;
    bool timed_out = false;
    int st_fail = 0;
    for (int st = 0; st < nst; ++st) {
        const int b = st % a.nbuf;
        const uint32_t parity = static_cast<uint32_t>(st / a.nbuf) & 1u;
        const bool ok = mbar_wait(&S.full[b], parity);
        if (__syncthreads_or(!ok)) {
            timed_out = true;
            st_fail = st;
            break;
        }
        const int64_t r0 = r_begin + static_cast<int64_t>(st) * R;
        const int rows_in = static_cast<int>(min(static_cast<int64_t>(R), r_end - r0));
        const uint8_t* sb = S.stage + static_cast<size_t>(b) * a.stage_bytes;
        float* pb = S.part + (st & 1) * R * a.nseg;

        if (active) {
            for (int r = rlane; r < rows_in; r += a.rl) {
                float p;
                if constexpr (KIND == kQ4K) {
                    const uint8_t* blk = sb + static_cast<size_t>(r) * a.row_bytes + seg * 144;
                    const uint4 h = *reinterpret_cast<const uint4*>(blk);
                    const uint4 qa = *reinterpret_cast<const uint4*>(blk + 16 + 32 * c);
                    const uint4 qb = *reinterpret_cast<const uint4*>(blk + 32 + 32 * c);
                    const uint32_t qw[8] = {qa.x, qa.y, qa.z, qa.w, qb.x, qb.y, qb.z, qb.w};
                    float2 accL = make_float2(0.f, 0.f), accH = make_float2(0.f, 0.f);
#pragma unroll
                    for (int k = 0; k < 8; ++k) {
                        const uint32_t lo = qw[k] & 0x0F0F0F0Fu;
                        const uint32_t hi = (qw[k] >> 4) & 0x0F0F0F0Fu;
                        accL = ffma2(make_float2(q_plus_128<0>(lo), q_plus_128<1>(lo)), xv[2 * k], accL);
                        accL = ffma2(make_float2(q_plus_128<2>(lo), q_plus_128<3>(lo)), xv[2 * k + 1], accL);
                        accH = ffma2(make_float2(q_plus_128<0>(hi), q_plus_128<1>(hi)), xv[16 + 2 * k], accH);
                        accH = ffma2(make_float2(q_plus_128<2>(hi), q_plus_128<3>(hi)), xv[16 + 2 * k + 1], accH);
                    }
                    // 6-bit scales / mins of sub-blocks 2c and 2c+1 (scale_min,
                    // src/autograd2.rs:1075-1085), four at a time per word.
                    const uint32_t S_ = (c < 2) ? (h.y & 0x3F3F3F3Fu)
                                                : ((h.w & 0x0F0F0F0Fu) | ((h.y >> 2) & 0x30303030u));
                    const uint32_t M_ = (c < 2) ? (h.z & 0x3F3F3F3Fu)
                                                : (((h.w >> 4) & 0x0F0F0F0Fu) | ((h.z >> 2) & 0x30303030u));
                    const uint32_t sel0 = 0x7540u | (2u * (c & 1));
                    const float s0 = byte_to_float(S_, sel0), s1 = byte_to_float(S_, sel0 + 1);
                    const float m0 = byte_to_float(M_, sel0), m1 = byte_to_float(M_, sel0 + 1);
                    const float d = f16_bits_to_f32(h.x & 0xFFFFu), dmin = f16_bits_to_f32(h.x >> 16);
                    const float tl = (accL.x + accL.y) - 128.0f * sx_lo;
                    const float th = (accH.x + accH.y) - 128.0f * sx_hi;
                    p = (d * s0) * tl - (dmin * m0) * sx_lo + (d * s1) * th - (dmin * m1) * sx_hi;
                } else {
                    const uint8_t* rp = sb + static_cast<size_t>(r) * a.row_bytes + seg * 512 + c * 128;
                    float2 acc0 = make_float2(0.f, 0.f), acc1 = make_float2(0.f, 0.f);
#pragma unroll
                    for (int k = 0; k < 8; ++k) {
                        if (k < nvalid16) {
                            const uint4 v = *reinterpret_cast<const uint4*>(rp + 16 * k);
                            acc0 = ffma2(make_float2(__uint_as_float(v.x << 16), __uint_as_float(v.x & 0xFFFF0000u)),
                                         xv[4 * k], acc0);
                            acc1 = ffma2(make_float2(__uint_as_float(v.y << 16), __uint_as_float(v.y & 0xFFFF0000u)),
                                         xv[4 * k + 1], acc1);
                            acc0 = ffma2(make_float2(__uint_as_float(v.z << 16), __uint_as_float(v.z & 0xFFFF0000u)),
                                         xv[4 * k + 2], acc0);
                            acc1 = ffma2(make_float2(__uint_as_float(v.w << 16), __uint_as_float(v.w & 0xFFFF0000u)),
                                         xv[4 * k + 3], acc1);
                        }
                    }
                    p = (acc0.x + acc0.y) + (acc1.x + acc1.y);
                }
                p += __shfl_xor_sync(gmask, p, 1);
                p += __shfl_xor_sync(gmask, p, 2);
                if (c == 0) pb[r * a.nseg + seg] = p;
            }
        }
        __syncthreads();
        if (tid == 0 && st + a.nbuf < nst) issue(st + a.nbuf);

        // ---------------- epilogue ----------------
        if constexpr (EPI == kEpiGeluPair) {
            if (tid < rows_in / 2) {
                const float* pg = pb + (2 * tid) * a.nseg;
                const float* pu = pg + a.nseg;
                float g = 0.f, u = 0.f;
                for (int s = 0; s < a.nseg; ++s) g += pg[s];
                for (int s = 0; s < a.nseg; ++s) u += pu[s];
                a.y[(r0 >> 1) + tid] = __fmul_rn(gelu_tanh_dev(g), u);
            }
        } else {
            if (tid < rows_in) {
                const float* pr = pb + tid * a.nseg;
                float v = 0.f;
                for (int s = 0; s < a.nseg; ++s) v += pr[s];
                a.y[r0 + tid] = v;
                if constexpr (EPI == kEpiArgmax) {
                    if (v > best_v || (v == best_v && r0 + tid > best_i)) {
                        best_v = v;
                        best_i = r0 + tid;
                    }
                }
            }
        }
    }

    if (timed_out) {
        // Record the failure, then wait (bounded) for every copy this CTA issued
        // before letting its shared memory go.
        if (tid == 0) {
            if (a.err) atomicExch(a.err, kErrMbarTimeout);
            for (int st = st_fail; st < issued; ++st) {
                if (!mbar_wait(&S.full[st % a.nbuf], static_cast<uint32_t>(st / a.nbuf) & 1u)) break;
            }
        }
        __syncthreads();
        return;
    }

    if constexpr (EPI == kEpiArgmax) {
        // Block argmax (largest value; ties to the higher row index).
        const int lane = tid & 31, warp = tid >> 5, nw = nthr >> 5;
        for (int o = 16; o > 0; o >>= 1) {
            const float ov = __shfl_xor_sync(0xffffffffu, best_v, o);
            const int64_t oi = __shfl_xor_sync(0xffffffffu, best_i, o);
            if (ov > best_v || (ov == best_v && oi > best_i)) {
                best_v = ov;
                best_i = oi;
            }
        }
        __shared__ float wv[32];
        __shared__ int64_t wi[32];
        __shared__ bool is_last;
        if (lane == 0) {
            wv[warp] = best_v;
            wi[warp] = best_i;
        }
        __syncthreads();
        if (tid == 0) {
            float bv = wv[0];
            int64_t bi = wi[0];
            for (int w = 1; w < nw; ++w)
                if (wv[w] > bv || (wv[w] == bv && wi[w] > bi)) {
                    bv = wv[w];
                    bi = wi[w];
                }
            a.am_val[blockIdx.x] = bv;
            a.am_idx[blockIdx.x] = static_cast<int32_t>(bi);
            __threadfence();
            const uint32_t prev = atomicAdd(a.am_counter, 1u);
            is_last = prev == gridDim.x - 1;
        }
        __syncthreads();
        if (is_last && tid == 0) {
            __threadfence();
            const volatile float* vv = a.am_val;
            const volatile int32_t* vi = a.am_idx;
            float bv = vv[0];
            int32_t bi = vi[0];
            for (unsigned g = 1; g < gridDim.x; ++g) {
                const float v = vv[g];
                const int32_t i = vi[g];
                if (v > bv || (v == bv && i > bi)) {
                    bv = v;
                    bi = i;
                }
            }
            if (a.token_out) *a.token_out = bi;
            if (a.pos_inout) {
                const int32_t p = *a.pos_inout;
                if (a.token_hist) a.token_hist[p] = bi;
                *a.pos_inout = p + 1;
            }
            *a.am_counter = 0u;
        }
    }
}

// Calls f(kernel) for the instantiation matching (kind, prologue, epilogue).
template <typename F>
bool dispatch(int kind, int pro, int epi, F&& f) {
#define RT_GEMV_CASE(K, P, E)                \
    if (kind == K && pro == P && epi == E) { \
        f(gemv_kernel<K, P, E>);             \
        return true;                         \
    }
    RT_GEMV_CASE(kQ4K, kProPlain, kEpiPlain)
    RT_GEMV_CASE(kQ4K, kProResidNorm, kEpiPlain)
    RT_GEMV_CASE(kQ4K, kProEmbedNorm, kEpiPlain)
    RT_GEMV_CASE(kQ4K, kProPlain, kEpiGeluPair)
    RT_GEMV_CASE(kQ4K, kProResidNorm, kEpiGeluPair)
    RT_GEMV_CASE(kBF16, kProPlain, kEpiPlain)
    RT_GEMV_CASE(kBF16, kProResidNorm, kEpiPlain)
    RT_GEMV_CASE(kBF16, kProEmbedNorm, kEpiPlain)
    RT_GEMV_CASE(kBF16, kProPlain, kEpiGeluPair)
    RT_GEMV_CASE(kBF16, kProResidNorm, kEpiGeluPair)
    RT_GEMV_CASE(kBF16, kProPlain, kEpiArgmax)
    RT_GEMV_CASE(kBF16, kProResidNorm, kEpiArgmax)
#undef RT_GEMV_CASE
    return false;
}

}  // namespace

GemvPlan gemv_plan(int kind, int64_t rows, int K, int pair, int prologue, int epilogue, int num_sms,
                   int max_ctas_per_sm) {
    GemvPlan best;
    const int nseg = (K + 255) / 256;
    const int row_bytes = kind == kQ4K ? nseg * 144 : K * 2;
    const int stage_cap = 24 * 1024;
    const int stage_hard = 64 * 1024;
    double best_score = -1.0;
    for (int w = 1; w <= 16; ++w) {
        const int groups = 8 * w;
        const int rl = groups / nseg;
        if (rl < 1) continue;
        if (static_cast<int64_t>(rl) * row_bytes > stage_hard) continue;
        const double eff = static_cast<double>(rl * nseg) / groups;
        const double score = eff * (1.0 - 0.03 * std::abs(w - 8));
        if (score > best_score + 1e-9) {
            best_score = score;
            best.warps = w;
            best.rl = rl;
        }
    }
    if (best.warps == 0) return best;  // K too large for one CTA
    int rps = best.rl * std::max(1, stage_cap / (best.rl * row_bytes));
    if (pair == 2 && (rps & 1)) rps += best.rl;  // stages hold whole (gate, up) pairs
    best.rows_per_stage = rps;
    best.stage_bytes = ((rps * row_bytes) + 127) & ~127;
    best.nbuf = 3;
    size_t smem = sizeof(uint64_t) * kMaxNbuf + sizeof(float) * 32 + sizeof(int) * 4 + sizeof(float) * 2 * rps * nseg;
    smem = (smem + 15) & ~size_t(15);
    if (prologue != kProPlain) smem += sizeof(float) * K;
    smem = (smem + 127) & ~size_t(127);
    smem += static_cast<size_t>(best.nbuf) * best.stage_bytes;
    best.smem = smem;
    // Raise the dynamic shared-memory limit of every instantiation here, outside
    // any stream capture (a plan made for one prologue also serves the others).
    for (int kd : {kQ4K, kBF16})
        for (int pr : {kProPlain, kProResidNorm, kProEmbedNorm})
            for (int ep : {kEpiPlain, kEpiGeluPair, kEpiArgmax})
                dispatch(kd, pr, ep, [&](auto k) {
                    cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, 200 * 1024);
                });
    int occ = 1;
    dispatch(kind, prologue, epilogue, [&](auto k) {
        if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&occ, k, best.warps * 32, smem) != cudaSuccess) occ = 1;
    });
    cudaGetLastError();
    const int cps = std::max(1, std::min(occ, max_ctas_per_sm));
    const int64_t units = rows / pair;
    const int64_t min_units_per_cta = std::max<int64_t>(1, rps / pair / 2);
    const int64_t grid = std::min<int64_t>(static_cast<int64_t>(num_sms) * cps,
                                           (units + min_units_per_cta - 1) / min_units_per_cta);
    best.grid = static_cast<int>(std::max<int64_t>(1, grid));
    return best;
}

cudaError_t gemv_launch(int kind, int prologue, int epilogue, GemvArgs a, const GemvPlan& p, cudaStream_t s, bool pdl) {
    a.nseg = (a.K + 255) / 256;
    a.seg_bytes = kind == kQ4K ? 144 : 512;
    a.row_bytes = kind == kQ4K ? a.nseg * 144 : a.K * 2;
    a.rl = p.rl;
    a.rows_per_stage = p.rows_per_stage;
    a.nbuf = p.nbuf;
    a.stage_bytes = p.stage_bytes;
    a.pair = epilogue == kEpiGeluPair ? 2 : 1;
    cudaError_t err = cudaErrorInvalidValue;
    // The dynamic shared-memory limit was raised by gemv_plan (not here: this
    // function also runs under stream capture).
    dispatch(kind, prologue, epilogue,
             [&](auto k) { err = rt_launch(k, dim3(p.grid), dim3(p.warps * 32), p.smem, s, pdl, a); });
    return err;
}

uint64_t gemv_algorithmic_bytes(int kind, int64_t rows, int K, int prologue, int epilogue) {
    const int nseg = (K + 255) / 256;
    uint64_t w = kind == kQ4K ? static_cast<uint64_t>(rows) * nseg * 144 : static_cast<uint64_t>(rows) * K * 2;
    uint64_t in = static_cast<uint64_t>(K) * 4;
    if (prologue == kProResidNorm) in = static_cast<uint64_t>(K) * 4 * 5;  // src, resid_in, 2 gammas, resid_out
    if (prologue == kProEmbedNorm) in = static_cast<uint64_t>(K) * (2 + 4 + 4);
    uint64_t out = static_cast<uint64_t>(epilogue == kEpiGeluPair ? rows / 2 : rows) * 4;
    return w + in + out;
}

}  // namespace rt
