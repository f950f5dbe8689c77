// gemv.cu -- Q4_K / BF16 GEMV on the sm_100a tensor cores (mma.sync).
//
// Streaming.  A CTA owns a contiguous range of 16-row tiles.  Each "stage" is
// one tile restricted to `spst` consecutive 256-column segments, copied HBM ->
// shared memory by one 2-D TMA tensor copy (8-byte elements, box = stage row
// stride x 16 rows, no multicast) into a row stride of 64 mod 128 bytes, so the
// fragment loads below are bank-conflict free.  The last warp of the CTA is the
// copy producer; `nbuf` stage buffers are completed on mbarriers and released
// by the compute warps on a second ring.  The first copies are issued before
// griddepcontrol.wait, so under programmatic dependent launch the weight stream
// starts while the previous kernel drains.  The 16 x 256 "units" of the stages
// are dealt round-robin over the compute warps in flat (stage, segment) order.
//
// Q4_K (block layout src/autograd2.rs:1003-1042; Q4KMat::dot_row
// src/autograd2.rs:1637-1702).  Per 32-column sub-block j of a row,
//     dot_j = d * sc_j * sum(q * x) - dmin * m_j * sum(x).
// The quants q (0..15) are the u8 A operand of mma.m16n8k32.u8.s8: a byte
// mask (and a shift for the high nibbles) turns four packed quants into four
// A bytes.  x is split once per launch, per sub-block, into three int8 planes
// x = s * (p0 + p1/128 + p2/16384) (|error| <= s/32768, s = max|x|/127), the s8
// B operand.  The MMA sums q * p exactly in s32; one k32 MMA covers 8 columns
// of 4 sub-blocks, and B is zero outside a column pair per sub-block, so lane
// t of every lane quad ends up holding the (p0, p1, p2) sums of one sub-block
// for two rows and all 32 lanes share the per-sub-block scale epilogue.
//
// BF16 (MatBf16::dot_row, src/autograd2.rs:861-888).  The weights are the A
// operand of mma.m16n8k16.bf16 as they sit in shared memory; x is split exactly
// into three bf16 planes x = hi + mid + lo (B columns 0..2), so the f32 sum of
// the three product columns is the f32 dot product.
//
// Each unit leaves one partial sum per row in shared memory; the warp that
// finishes the last unit of a tile (a shared-memory counter) adds the partials
// in segment order (deterministic) and runs the epilogue (store, GELU gate,
// greedy argmax).
#include <cudaTypedefs.h>  // PFN_cuTensorMapEncodeTiled

#include <algorithm>
#include <cstdio>

#include "common.cuh"
#include "gemv.cuh"

namespace rt {

namespace {

constexpr int kMaxNbuf = 6;
constexpr int kTile = 16;

__device__ __forceinline__ float gelu_tanh_dev(float x) {
    // TensorNode::gelu_tanh (src/autograd2.rs:3082-3091): x*0.5*(1+tanh(s*(x+c*x^3))),
    // evaluated without FMA contraction in the reference's operation order.
    const float kS = 0.7978845608028654f, kC = 0.044715f;
    float x3 = __fmul_rn(__fmul_rn(__fmul_rn(kC, x), x), x);
    float inner = __fmul_rn(kS, __fadd_rn(x, x3));
    return __fmul_rn(__fmul_rn(x, 0.5f), __fadd_rn(1.0f, tanhf(inner)));
}

// Byte selected by `sel` (0x7540 | b) of v, as an exact float.
__device__ __forceinline__ float byte_to_float(uint32_t v, uint32_t sel) {
    return __uint_as_float(__byte_perm(v, 0x4B000000u, sel)) - 8388608.0f;
}

__device__ __forceinline__ uint4 lds128(const void* p) { return *reinterpret_cast<const uint4*>(p); }

__device__ __forceinline__ void mma_u8s8(int (&c)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3, uint32_t b0,
                                         uint32_t b1) {
    asm("mma.sync.aligned.m16n8k32.row.col.s32.u8.s8.s32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};"
        : "+r"(c[0]), "+r"(c[1]), "+r"(c[2]), "+r"(c[3])
        : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

__device__ __forceinline__ void mma_bf16(float (&c)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                                         uint32_t b0, uint32_t b1) {
    asm("mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};"
        : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
        : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

__device__ __forceinline__ uint32_t word(const uint4& v, int i) {
    return i == 0 ? v.x : i == 1 ? v.y : i == 2 ? v.z : v.w;
}

constexpr int kSlots = kMaxNbuf + 2;  // tiles that can be in flight at once
constexpr int kMaxV = 6;               // float4 chunks per thread in the norm prologues

struct Smem {
    uint64_t* full;    // [kMaxNbuf] stage data landed
    uint64_t* empty;   // [kMaxNbuf] stage consumed by every compute warp
    uint64_t* pbar;    // prologue vectors landed
    float* red;        // [32]
    int* flags;        // [8]: 0 = error, 1 = stages issued
    uint32_t* tcnt;    // [kSlots] units finished per in-flight tile
    float* part;       // [kSlots][16][nseg] per-(row, segment) partial sums
    float* bv;         // [32] per-warp argmax value
    long long* bi;     // [32] per-warp argmax row
    uint8_t* zero;     // [16] zeros: B operand of columns a lane does not feed
    float* xs;         // [K] x (copied in, or built by a norm prologue)
    float* rs;         // [K] residual stream in (norm prologue) / embedding row (bf16)
    uint8_t* planes;   // Q4_K: [3][Kp] int8; BF16: [3][Kp] bf16
    float* sx;         // Q4_K: [Kp/32] sum of x over each sub-block
    uint8_t* stage;    // [nbuf][stage_bytes]
};

__host__ __device__ inline size_t carve(uint8_t* base, int kind, int K, int nseg, int nbuf, int stage_bytes,
                                        bool need_xs, bool x_smem, Smem* S) {
    size_t off = 0;
    auto take = [&](size_t bytes, size_t align) -> uint8_t* {
        off = (off + align - 1) / align * align;
        uint8_t* p = base + off;
        off += bytes;
        return p;
    };
    const size_t Kp = static_cast<size_t>(nseg) * 256;
    uint8_t* full = take(sizeof(uint64_t) * kMaxNbuf, 16);
    uint8_t* empty = take(sizeof(uint64_t) * kMaxNbuf, 16);
    uint8_t* pbar = take(sizeof(uint64_t), 16);
    uint8_t* red = take(32 * 4, 16);
    uint8_t* flags = take(8 * 4, 16);
    uint8_t* tcnt = take(4 * kSlots, 16);
    uint8_t* part = take(sizeof(float) * kSlots * kTile * nseg, 16);
    uint8_t* bv = take(4 * 32, 16);
    uint8_t* bi = take(8 * 32, 16);
    uint8_t* zero = take(16, 16);
    uint8_t* xs = take(need_xs || x_smem ? sizeof(float) * K : 0, 16);
    uint8_t* rs = take(need_xs ? sizeof(float) * K : 0, 16);
    uint8_t* planes = take(kind == kQ4K ? 3 * Kp : 3 * Kp * 2, 16);
    uint8_t* sx = take(kind == kQ4K ? sizeof(float) * (Kp / 32) : 0, 16);
    uint8_t* stage = take(static_cast<size_t>(nbuf) * stage_bytes, 128);
    if (S) {
        S->full = reinterpret_cast<uint64_t*>(full);
        S->empty = reinterpret_cast<uint64_t*>(empty);
        S->pbar = reinterpret_cast<uint64_t*>(pbar);
        S->red = reinterpret_cast<float*>(red);
        S->flags = reinterpret_cast<int*>(flags);
        S->tcnt = reinterpret_cast<uint32_t*>(tcnt);
        S->part = reinterpret_cast<float*>(part);
        S->bv = reinterpret_cast<float*>(bv);
        S->bi = reinterpret_cast<long long*>(bi);
        S->zero = zero;
        S->xs = reinterpret_cast<float*>(xs);
        S->rs = reinterpret_cast<float*>(rs);
        S->planes = planes;
        S->sx = reinterpret_cast<float*>(sx);
        S->stage = stage;
    }
    return off + 128;  // slack for the dynamic shared-memory base alignment
}

__device__ __forceinline__ float block_max(float v, float* red) {
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nw = blockDim.x >> 5;
    v = warp_max(v);
    __syncthreads();
    if (lane == 0) red[warp] = v;
    __syncthreads();
    float t = 0.f;
    for (int i = 0; i < nw; ++i) t = fmaxf(t, red[i]);
    return t;
}

// Round to the nearest integer (ties to even) without the XU pipe:
// adding 1.5 * 2^23 leaves the integer in the low mantissa bits (|y| < 2^22).
__device__ __forceinline__ int round_magic(float y, float* yr) {
    const float m = __fadd_rn(y, 12582912.0f);
    *yr = __fsub_rn(m, 12582912.0f);
    return __float_as_int(m) - 0x4B400000;
}

__device__ __forceinline__ uint32_t pack4(int a, int b, int c, int d) {
    return (static_cast<uint32_t>(a) & 0xFFu) | ((static_cast<uint32_t>(b) & 0xFFu) << 8) |
           ((static_cast<uint32_t>(c) & 0xFFu) << 16) | (static_cast<uint32_t>(d) << 24);
}

// f32 -> bf16 bits, round to nearest even (finite inputs).
__device__ __forceinline__ uint32_t bf16_rne(float x) {
    const uint32_t u = __float_as_uint(x);
    return (u + 0x7FFFu + ((u >> 16) & 1u)) >> 16;
}

template <int KIND, int PRO, int EPI>
__global__ void __launch_bounds__(544) gemv_kernel(const GemvArgs a, const __grid_constant__ CUtensorMap tmap) {
    extern __shared__ __align__(128) uint8_t smem[];
    constexpr bool kNeedXs = PRO != kProPlain;
    Smem S;
    carve(smem, KIND, a.K, a.nseg, a.nbuf, a.stage_bytes, kNeedXs, a.x_smem != 0, &S);

    const int tid = threadIdx.x, nthr = blockDim.x;
    const int lane = tid & 31, warp = tid >> 5, nw = nthr >> 5;
    const int nwc = nw - 1;  // compute warps; the last warp is the copy producer
    const bool producer = warp == nwc;
    const int K = a.K, nseg = a.nseg, spst = a.spst;
    const int Kp = nseg * 256;
    const int nsc = (nseg + spst - 1) / spst;  // segment chunks (stages) per tile

    // Contiguous, balanced range of 16-row tiles.
    const int64_t ntiles_all = (a.rows + kTile - 1) / kTile;
    const int64_t t_begin = ntiles_all * blockIdx.x / gridDim.x;
    const int64_t t_end = ntiles_all * (blockIdx.x + 1) / gridDim.x;
    const int64_t r_begin = t_begin * kTile;
    const int64_t r_end = min(a.rows, t_end * kTile);
    const int nst = static_cast<int>(t_end - t_begin) * nsc;

    if (tid == 0) {
        for (int b = 0; b < a.nbuf; ++b) {
            mbar_init(&S.full[b], 1);
            mbar_init(&S.empty[b], nwc);
        }
        mbar_init(S.pbar, 1);
        fence_mbar_init();
        S.flags[0] = 0;
        S.flags[1] = 0;
    }
    if (tid < kSlots) S.tcnt[tid] = 0u;
    if (tid < 4) reinterpret_cast<uint32_t*>(S.zero)[tid] = 0u;
    __syncthreads();

    const uint64_t pol = l2_evict_first_policy();
    // Producer: one 2-D tensor copy per stage (16 rows x one segment chunk);
    // the box's inner extent is the padded row stride.
    auto issue = [&](int st) {
        if (lane == 0) {
            const int tile = st / nsc, sc = st % nsc;
            const int64_t r0 = r_begin + static_cast<int64_t>(tile) * kTile;
            const int b = st % a.nbuf;
            mbar_arrive_expect_tx(&S.full[b], static_cast<uint32_t>(a.stage_bytes));
            tma_2d_g2s(S.stage + static_cast<size_t>(b) * a.stage_bytes, &tmap, sc * spst * a.seg_bytes / 8,
                       static_cast<int>(r0), &S.full[b], pol);
            S.flags[1] = st + 1;
        }
        __syncwarp();
    };
    if (producer) {
        for (int st = 0; st < min(a.nbuf, nst); ++st) issue(st);
    }
    // The norm weights are constants: load this thread's float4 chunks now,
    // before waiting for the previous kernel.
    const int K4 = K / 4;
    float4 gp[kMaxV], gq[kMaxV];
    if constexpr (PRO != kProPlain) {
#pragma unroll
        for (int k = 0; k < kMaxV; ++k) {
            const int i = tid + k * nthr;
            if (i < K4) {
                if constexpr (PRO == kProResidNorm) gp[k] = reinterpret_cast<const float4*>(a.g_post)[i];
                gq[k] = reinterpret_cast<const float4*>(a.g_pre)[i];
            }
        }
    }
    pdl_launch_dependents();
    pdl_wait();

    // ---------------- prologue: the input vectors, one bulk round trip ----------------
    const bool x_in_place = PRO == kProPlain && !a.x_smem;  // large K: planes read x from global
    if (tid == 0 && !x_in_place) {
        if constexpr (PRO == kProPlain) {
            mbar_arrive_expect_tx(S.pbar, static_cast<uint32_t>(K) * 4u);
            bulk_g2s_nohint(S.xs, a.x, static_cast<uint32_t>(K) * 4u, S.pbar);
        } else if constexpr (PRO == kProResidNorm) {
            mbar_arrive_expect_tx(S.pbar, static_cast<uint32_t>(K) * 8u);
            bulk_g2s_nohint(S.xs, a.src, static_cast<uint32_t>(K) * 4u, S.pbar);
            bulk_g2s_nohint(S.rs, a.resid_in, static_cast<uint32_t>(K) * 4u, S.pbar);
        } else {
            const int64_t tok = static_cast<int64_t>(*a.token);
            mbar_arrive_expect_tx(S.pbar, static_cast<uint32_t>(K) * 2u);
            bulk_g2s_nohint(S.rs, a.embed + tok * K, static_cast<uint32_t>(K) * 2u, S.pbar);
        }
    }
    if (!x_in_place && !mbar_wait(S.pbar, 0u) && lane == 0) atomicExch(&S.flags[0], 1);
    float4* xs4 = reinterpret_cast<float4*>(S.xs);
    if constexpr (PRO == kProResidNorm || PRO == kProEmbedNorm) {
        const float inv_d = 1.0f / static_cast<float>(K);
        float4* out4 = reinterpret_cast<float4*>(a.resid_out);
        float ss = 0.f;
        if constexpr (PRO == kProResidNorm) {
            // post-norm of the sub-layer output, then the residual add
            // (Gemma3Block::forward_cached, src/transformer4.rs:1954-1964)
            const float4* rs4 = reinterpret_cast<const float4*>(S.rs);
#pragma unroll
            for (int k = 0; k < kMaxV; ++k) {
                const int i = tid + k * nthr;
                if (i < K4) {
                    const float4 v = xs4[i];
                    ss += (v.x * v.x + v.y * v.y) + (v.z * v.z + v.w * v.w);
                }
            }
            ss = block_sum(ss, S.red);
            const float r1 = 1.0f / sqrtf(ss * inv_d + a.eps);
            float ss2 = 0.f;
#pragma unroll
            for (int k = 0; k < kMaxV; ++k) {
                const int i = tid + k * nthr;
                if (i < K4) {
                    const float4 v = xs4[i], r = rs4[i], g = gp[k];
                    float4 n;
                    n.x = __fadd_rn(r.x, __fmul_rn(__fmul_rn(v.x, r1), __fadd_rn(1.0f, g.x)));
                    n.y = __fadd_rn(r.y, __fmul_rn(__fmul_rn(v.y, r1), __fadd_rn(1.0f, g.y)));
                    n.z = __fadd_rn(r.z, __fmul_rn(__fmul_rn(v.z, r1), __fadd_rn(1.0f, g.z)));
                    n.w = __fadd_rn(r.w, __fmul_rn(__fmul_rn(v.w, r1), __fadd_rn(1.0f, g.w)));
                    xs4[i] = n;
                    ss2 += (n.x * n.x + n.y * n.y) + (n.z * n.z + n.w * n.w);
                    if (blockIdx.x == 0) out4[i] = n;
                }
            }
            ss = block_sum(ss2, S.red);
        } else {
            // embedding row * sqrt(hidden) (src/transformer4.rs:2360-2364)
            const uint2* e2 = reinterpret_cast<const uint2*>(S.rs);
#pragma unroll
            for (int k = 0; k < kMaxV; ++k) {
                const int i = tid + k * nthr;
                if (i < K4) {
                    const uint2 e = e2[i];
                    float4 n;
                    n.x = __fmul_rn(bf16_bits_to_f32(e.x & 0xFFFFu), a.embed_scale);
                    n.y = __fmul_rn(bf16_bits_to_f32(e.x >> 16), a.embed_scale);
                    n.z = __fmul_rn(bf16_bits_to_f32(e.y & 0xFFFFu), a.embed_scale);
                    n.w = __fmul_rn(bf16_bits_to_f32(e.y >> 16), a.embed_scale);
                    xs4[i] = n;
                    ss += (n.x * n.x + n.y * n.y) + (n.z * n.z + n.w * n.w);
                    if (blockIdx.x == 0) out4[i] = n;
                }
            }
            ss = block_sum(ss, S.red);
        }
        // pre-norm producing the projection input (rms_norm_gemma3,
        // src/autograd2.rs:3477-3496)
        const float r2 = 1.0f / sqrtf(ss * inv_d + a.eps);
#pragma unroll
        for (int k = 0; k < kMaxV; ++k) {
            const int i = tid + k * nthr;
            if (i < K4) {
                const float4 n = xs4[i], g = gq[k];
                float4 x;
                x.x = __fmul_rn(__fmul_rn(n.x, r2), __fadd_rn(1.0f, g.x));
                x.y = __fmul_rn(__fmul_rn(n.y, r2), __fadd_rn(1.0f, g.y));
                x.z = __fmul_rn(__fmul_rn(n.z, r2), __fadd_rn(1.0f, g.z));
                x.w = __fmul_rn(__fmul_rn(n.w, r2), __fadd_rn(1.0f, g.w));
                xs4[i] = x;
            }
        }
    }
    __syncthreads();
    const float* xsrc = x_in_place ? a.x : S.xs;

    // ---------------- x planes (the B operand) ----------------
    float xsc = 0.f;  // Q4_K: value of one unit of the combined plane integer
    if constexpr (KIND == kQ4K) {
        // One scale for the whole vector: x = s * (p0 + p1/128 + p2/16384),
        // |error| <= s / 32768 with s = max|x| / 127.
        float m = 0.f;
        for (int i = tid; i < K4; i += nthr) {
            const float4 v = reinterpret_cast<const float4*>(xsrc)[i];
            m = fmaxf(m, fmaxf(fmaxf(fabsf(v.x), fabsf(v.y)), fmaxf(fabsf(v.z), fabsf(v.w))));
        }
        m = block_max(m, S.red);
        const float s = m / 127.0f;
        const float inv = m > 0.f ? 127.0f / m : 0.f;
        const float s128 = s * (1.0f / 128.0f);
        const float inv128 = inv * 128.0f, inv16k = inv * 16384.0f;
        xsc = s * (1.0f / 16384.0f);
        uint32_t* P = reinterpret_cast<uint32_t*>(S.planes);
        for (int base = 0; base < K4; base += nthr) {
            const int i = base + tid;
            const bool valid = i < K4;
            const float4 v = valid ? reinterpret_cast<const float4*>(xsrc)[i] : make_float4(0.f, 0.f, 0.f, 0.f);
            const float xv[4] = {v.x, v.y, v.z, v.w};
            int q0[4], q1[4], q2[4];
#pragma unroll
            for (int e = 0; e < 4; ++e) {
                float f0, f1, f2;
                q0[e] = round_magic(xv[e] * inv, &f0);
                const float r1 = fmaf(-f0, s, xv[e]);
                q1[e] = round_magic(r1 * inv128, &f1);
                const float r2 = fmaf(-f1, s128, r1);
                q2[e] = round_magic(r2 * inv16k, &f2);
            }
            float sum = (v.x + v.y) + (v.z + v.w);
            sum += __shfl_xor_sync(0xffffffffu, sum, 1);
            sum += __shfl_xor_sync(0xffffffffu, sum, 2);
            sum += __shfl_xor_sync(0xffffffffu, sum, 4);
            if (valid) {
                P[i] = pack4(q0[0], q0[1], q0[2], q0[3]);
                P[Kp / 4 + i] = pack4(q1[0], q1[1], q1[2], q1[3]);
                P[Kp / 2 + i] = pack4(q2[0], q2[1], q2[2], q2[3]);
                if ((i & 7) == 0) S.sx[i >> 3] = sum;
            }
        }
    } else {
        uint2* P = reinterpret_cast<uint2*>(S.planes);
        for (int i = tid; i < Kp / 4; i += nthr) {
            const float4 v = i < K4 ? reinterpret_cast<const float4*>(xsrc)[i] : make_float4(0.f, 0.f, 0.f, 0.f);
            const float xv[4] = {v.x, v.y, v.z, v.w};
            uint32_t h[4], md[4], lo[4];
#pragma unroll
            for (int e = 0; e < 4; ++e) {
                h[e] = bf16_rne(xv[e]);
                const float r = xv[e] - __uint_as_float(h[e] << 16);
                md[e] = bf16_rne(r);
                lo[e] = bf16_rne(r - __uint_as_float(md[e] << 16));
            }
            P[i] = make_uint2(h[0] | (h[1] << 16), h[2] | (h[3] << 16));
            P[Kp / 4 + i] = make_uint2(md[0] | (md[1] << 16), md[2] | (md[3] << 16));
            P[Kp / 2 + i] = make_uint2(lo[0] | (lo[1] << 16), lo[2] | (lo[3] << 16));
        }
    }
    __syncthreads();

    float best_v = -INFINITY;
    long long best_i = -1;
    if (producer) {
        // Refill each buffer once every compute warp has released it.
        for (int st = a.nbuf; st < nst; ++st) {
            const int b = st % a.nbuf;
            const bool ok = mbar_wait(&S.empty[b], static_cast<uint32_t>(st / a.nbuf - 1) & 1u);
            if (!ok) {
                if (lane == 0) atomicExch(&S.flags[0], 1);
                break;
            }
            issue(st);
        }
    } else {
        const int g = lane >> 2, t = lane & 3;
        // Q4_K: the B column this lane feeds (see the header comment).
        const bool sel0 = (g >> 1) == (t >> 1);
        const bool sel1 = (g >> 1) == 2 + (t >> 1);
        const int j0 = 2 * (t & 1) + (t >> 1);  // sub-block (of each half block) whose sums this lane gets
        const uint32_t jsel = 0x7540u | static_cast<uint32_t>(j0);
        for (int st = 0; st < nst; ++st) {
            const int b = st % a.nbuf;
            if (!mbar_wait(&S.full[b], static_cast<uint32_t>(st / a.nbuf) & 1u)) {
                if (lane == 0) atomicExch(&S.flags[0], 1);
                break;
            }
            const int tile = st / nsc, sc = st % nsc;
            const int64_t r0 = r_begin + static_cast<int64_t>(tile) * kTile;
            const int nr = static_cast<int>(min(static_cast<int64_t>(kTile), r_end - r0));
            const int s0 = sc * spst;
            const int nus = min(nseg, s0 + spst) - s0;  // segments (units) in this stage
            const uint8_t* sbuf = S.stage + static_cast<size_t>(b) * a.stage_bytes;
            const int slot = tile % kSlots;
            float* pb = S.part + static_cast<size_t>(slot) * kTile * nseg;
            int mine = 0;
            // Units are dealt round-robin over the flat (stage, segment) order, so
            // the compute warps spread over every stage that has landed.
            const int u0 = ((warp - (st * spst) % nwc) % nwc + nwc) % nwc;
            for (int u = u0; u < nus; u += nwc) {
                ++mine;
                const int seg = s0 + u;
                float vg = 0.f, vg8 = 0.f;
                if constexpr (KIND == kQ4K) {
                    const uint8_t* rg = sbuf + g * a.srow + u * 144;
                    const uint8_t* rg8 = rg + 8 * a.srow;
                    const uint4 h0 = lds128(rg), h1 = lds128(rg8);
                    uint4 A0[2], A1[2], Ba0[2], Ba1[2], Bb0[2], Bb1[2];
#pragma unroll
                    for (int G = 0; G < 2; ++G) {
                        // This lane's quants: chunk 2G + (t >> 1), bytes 16 (t & 1) .. +16;
                        // low nibbles feed a0 / a1 (sub-block sb0), high nibbles a2 / a3 (sb0 + 1).
                        const int aoff = 16 + 32 * (2 * G + (t >> 1)) + 16 * (t & 1);
                        A0[G] = lds128(rg + aoff);
                        A1[G] = lds128(rg8 + aoff);
                        const int eoff = seg * 256 + 32 * (4 * G + 2 * (t >> 1)) + 16 * (t & 1);
                        const uint8_t* zp = S.zero;
                        Ba0[G] = lds128(sel0 ? S.planes + (g & 1) * Kp + eoff : zp);
                        Ba1[G] = lds128(sel1 ? S.planes + (g & 1) * Kp + eoff + 32 : zp);
                        Bb0[G] = lds128((sel0 && !(g & 1)) ? S.planes + 2 * Kp + eoff : zp);
                        Bb1[G] = lds128((sel1 && !(g & 1)) ? S.planes + 2 * Kp + eoff + 32 : zp);
                    }
                    int ca[2][4] = {{0, 0, 0, 0}, {0, 0, 0, 0}}, cbb[2][4] = {{0, 0, 0, 0}, {0, 0, 0, 0}};
#pragma unroll
                    for (int s = 0; s < 4; ++s) {
#pragma unroll
                        for (int G = 0; G < 2; ++G) {
                            const uint32_t w0 = word(A0[G], s), w1 = word(A1[G], s);
                            const uint32_t a0 = w0 & 0x0F0F0F0Fu, a2 = (w0 >> 4) & 0x0F0F0F0Fu;
                            const uint32_t a1 = w1 & 0x0F0F0F0Fu, a3 = (w1 >> 4) & 0x0F0F0F0Fu;
                            mma_u8s8(ca[G], a0, a1, a2, a3, word(Ba0[G], s), word(Ba1[G], s));
                            mma_u8s8(cbb[G], a0, a1, a2, a3, word(Bb0[G], s), word(Bb1[G], s));
                        }
                    }
                    // Lane (g, t) now holds sub-blocks j0 (G = 0) and j0 + 4 (G = 1):
                    // ca[G] = {P0, P1} of row g (regs 0, 1) and row g+8 (regs 2, 3);
                    // cbb[G][0] / cbb[G][2] = P2 of rows g / g+8.
                    const float sx0 = S.sx[seg * 8 + j0], sx1 = S.sx[seg * 8 + j0 + 4];
#pragma unroll
                    for (int half = 0; half < 2; ++half) {
                        const uint4 h = half ? h1 : h0;
                        const float d = f16_bits_to_f32(h.x & 0xFFFFu), dmin = f16_bits_to_f32(h.x >> 16);
                        // scale_min (src/autograd2.rs:1075-1085), four 6-bit fields per word
                        const uint32_t s_lo = h.y & 0x3F3F3F3Fu, m_lo = h.z & 0x3F3F3F3Fu;
                        const uint32_t s_hi = (h.w & 0x0F0F0F0Fu) | ((h.y >> 2) & 0x30303030u);
                        const uint32_t m_hi = ((h.w >> 4) & 0x0F0F0F0Fu) | ((h.z >> 2) & 0x30303030u);
                        const float sc0 = byte_to_float(s_lo, jsel), mn0 = byte_to_float(m_lo, jsel);
                        const float sc1 = byte_to_float(s_hi, jsel), mn1 = byte_to_float(m_hi, jsel);
                        const int i0 = 2 * half;
                        const float T0 = static_cast<float>(ca[0][i0] * 16384 + ca[0][i0 + 1] * 128 + cbb[0][i0]);
                        const float T1 = static_cast<float>(ca[1][i0] * 16384 + ca[1][i0 + 1] * 128 + cbb[1][i0]);
                        const float v = d * ((sc0 * T0 + sc1 * T1) * xsc) - dmin * (mn0 * sx0 + mn1 * sx1);
                        if (half) vg8 = v;
                        else vg = v;
                    }
                } else {
                    const uint8_t* rg = sbuf + g * a.srow + u * 512 + 16 * t;
                    const uint8_t* rg8 = rg + 8 * a.srow;
                    const uint8_t* pbp = g < 3 ? S.planes + static_cast<size_t>(g) * Kp * 2 + seg * 512 + 16 * t : S.zero;
                    const int pstep = g < 3 ? 64 : 0;
                    const int valid = K - seg * 256;  // columns of this segment inside the row (multiple of 8)
                    float c[4][4];
#pragma unroll
                    for (int q = 0; q < 4; ++q)
#pragma unroll
                        for (int i = 0; i < 4; ++i) c[q][i] = 0.f;
#pragma unroll
                    for (int p = 0; p < 8; ++p) {
                        uint4 A0 = lds128(rg + 64 * p), A1 = lds128(rg8 + 64 * p);
                        const uint4 B = lds128(pbp + pstep * p);
                        if (32 * p + 8 * t >= valid) A0 = A1 = make_uint4(0, 0, 0, 0);
                        mma_bf16(c[(2 * p) & 3], A0.x, A1.x, A0.y, A1.y, B.x, B.y);
                        mma_bf16(c[(2 * p + 1) & 3], A0.z, A1.z, A0.w, A1.w, B.z, B.w);
                    }
                    vg = ((c[0][0] + c[1][0]) + (c[2][0] + c[3][0])) + ((c[0][1] + c[1][1]) + (c[2][1] + c[3][1]));
                    vg8 = ((c[0][2] + c[1][2]) + (c[2][2] + c[3][2])) + ((c[0][3] + c[1][3]) + (c[2][3] + c[3][3]));
                }
                vg += __shfl_xor_sync(0xffffffffu, vg, 1);
                vg += __shfl_xor_sync(0xffffffffu, vg, 2);
                vg8 += __shfl_xor_sync(0xffffffffu, vg8, 1);
                vg8 += __shfl_xor_sync(0xffffffffu, vg8, 2);
                if (t == 0) {
                    pb[g * nseg + seg] = vg;
                    pb[(g + 8) * nseg + seg] = vg8;
                }
            }
            // Count this warp's units of the tile; the warp that completes the
            // tile sums its partials (fixed order) and runs the epilogue.
            __syncwarp();
            int last = 0;
            if (lane == 0 && mine) {
                __threadfence_block();
                const uint32_t prev = atomicAdd(&S.tcnt[slot], static_cast<uint32_t>(mine));
                last = prev + mine == static_cast<uint32_t>(nseg);
            }
            last = __shfl_sync(0xffffffffu, last, 0);
            if (last) {
                __threadfence_block();
                if constexpr (EPI == kEpiGeluPair) {
                    if (lane < nr / 2) {
                        float gsum = 0.f, usum = 0.f;
                        for (int s2 = 0; s2 < nseg; ++s2) gsum += pb[(2 * lane) * nseg + s2];
                        for (int s2 = 0; s2 < nseg; ++s2) usum += pb[(2 * lane + 1) * nseg + s2];
                        a.y[(r0 >> 1) + lane] = __fmul_rn(gelu_tanh_dev(gsum), usum);
                    }
                } else {
                    if (lane < nr) {
                        float v = 0.f;
                        for (int s2 = 0; s2 < nseg; ++s2) v += pb[lane * nseg + s2];
                        a.y[r0 + lane] = v;
                        if constexpr (EPI == kEpiArgmax) {
                            if (v > best_v || (v == best_v && r0 + lane > best_i)) {
                                best_v = v;
                                best_i = r0 + lane;
                            }
                        }
                    }
                }
                __syncwarp();
                if (lane == 0) S.tcnt[slot] = 0u;
            }
            __syncwarp();
            if (lane == 0) mbar_arrive(&S.empty[b]);
        }
    }
    __syncthreads();

    if (S.flags[0]) {
        // A bounded wait gave up: record it, then wait (bounded) for every copy
        // this CTA issued before letting its shared memory go.
        if (tid == 0) {
            if (a.err) atomicExch(a.err, kErrMbarTimeout);
            const int issued = S.flags[1];
            for (int st = max(0, issued - a.nbuf); st < issued; ++st) {
                if (!mbar_wait(&S.full[st % a.nbuf], static_cast<uint32_t>(st / a.nbuf) & 1u)) break;
            }
        }
        __syncthreads();
        return;
    }

    if constexpr (EPI == kEpiArgmax) {
        // Block argmax (largest value; ties to the higher row index).
        __shared__ bool is_last;
        for (int o = 16; o > 0; o >>= 1) {
            const float ov = __shfl_xor_sync(0xffffffffu, best_v, o);
            const long long oi = __shfl_xor_sync(0xffffffffu, best_i, o);
            if (ov > best_v || (ov == best_v && oi > best_i)) {
                best_v = ov;
                best_i = oi;
            }
        }
        if (lane == 0) {
            S.bv[warp] = best_v;
            S.bi[warp] = best_i;
        }
        __syncthreads();
        if (tid == 0) {
            float bv = S.bv[0];
            long long bi = S.bi[0];
            for (int w = 1; w < nw; ++w)
                if (S.bv[w] > bv || (S.bv[w] == bv && S.bi[w] > bi)) {
                    bv = S.bv[w];
                    bi = S.bi[w];
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
            for (unsigned q = 1; q < gridDim.x; ++q) {
                const float v = vv[q];
                const int32_t i = vi[q];
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

// Largest divisor of n that is <= cap, or cap itself when that divisor would
// leave stages less than half full.
int pick_spst(int n, int cap) {
    if (n <= cap) return n;
    int best = 1;
    for (int d = 1; d <= cap; ++d)
        if (n % d == 0) best = d;
    return best * 2 >= cap ? best : cap;
}

}  // namespace

void gemv_prepare() {
    // Raise the dynamic shared-memory limit of every instantiation, outside any
    // stream capture.
    for (int kd : {kQ4K, kBF16})
        for (int pr : {kProPlain, kProResidNorm, kProEmbedNorm})
            for (int ep : {kEpiPlain, kEpiGeluPair, kEpiArgmax})
                dispatch(kd, pr, ep, [&](auto k) {
                    cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, 220 * 1024);
                });
    cudaGetLastError();
}

GemvPlan gemv_plan(int kind, int64_t rows, int K, int pair, int prologue, int epilogue, int num_sms,
                   int max_ctas_per_sm) {
    GemvPlan p;
    const int nseg = (K + 255) / 256;
    const int seg_bytes = kind == kQ4K ? 144 : 512;
    // A stage row (plus padding) is one TMA box row: at most 256 8-byte elements.
    const int spst = pick_spst(nseg, kind == kQ4K ? 10 : 3);
    int srow = (spst * seg_bytes + 15) & ~15;
    srow += ((64 - srow % 128) + 128) % 128;  // = 64 (mod 128): conflict-free fragment loads
    p.spst = spst;
    p.srow = srow;
    p.stage_bytes = kTile * srow;
    p.warps = 16 + 1;  // compute warps + the copy-producer warp
    const bool need_xs = prologue != kProPlain;
    if (need_xs && K / 4 > kMaxV * p.warps * 32) {
        p.warps = 0;  // norm prologue holds at most kMaxV float4 per thread
        return p;
    }
    // As many stage buffers as fit next to the rest (one CTA per SM).
    const size_t budget = 200 * 1024;
    p.x_smem = static_cast<size_t>(K) * 4 <= 48 * 1024 ? 1 : 0;
    p.nbuf = 2;
    size_t smem = carve(nullptr, kind, K, nseg, p.nbuf, p.stage_bytes, need_xs, p.x_smem, nullptr);
    while (p.nbuf < kMaxNbuf && smem + p.stage_bytes <= budget) {
        ++p.nbuf;
        smem = carve(nullptr, kind, K, nseg, p.nbuf, p.stage_bytes, need_xs, p.x_smem, nullptr);
    }
    if (smem > 220 * 1024) {
        p.warps = 0;  // does not fit: the caller reports RT_E_SHAPE
        return p;
    }
    p.smem = smem;
    int occ = 1;
    dispatch(kind, prologue, epilogue, [&](auto k) {
        if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&occ, k, p.warps * 32, smem) != cudaSuccess) occ = 1;
    });
    cudaGetLastError();
    const int cps = std::max(1, std::min(occ, max_ctas_per_sm));
    (void)pair;  // tiles are 16 rows, so (gate, up) pairs never straddle CTAs
    const int64_t tiles = (rows + kTile - 1) / kTile;
    p.grid = static_cast<int>(std::max<int64_t>(1, std::min<int64_t>(static_cast<int64_t>(num_sms) * cps, tiles)));
    return p;
}

bool gemv_make_tmap(int kind, const void* w, int64_t rows, int K, const GemvPlan& p, CUtensorMap* out) {
    static PFN_cuTensorMapEncodeTiled_v12000 encode = nullptr;
    if (!encode) {
        cudaDriverEntryPointQueryResult q;
        void* fn = nullptr;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &fn, cudaEnableDefault, &q) != cudaSuccess ||
            q != cudaDriverEntryPointSuccess || !fn) {
            cudaGetLastError();
            return false;
        }
        encode = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(fn);
    }
    const int nseg = (K + 255) / 256;
    const uint64_t row_bytes = kind == kQ4K ? static_cast<uint64_t>(nseg) * 144 : static_cast<uint64_t>(K) * 2;
    const cuuint64_t dims[2] = {row_bytes / 8, static_cast<cuuint64_t>(rows)};
    const cuuint64_t strides[1] = {row_bytes};
    const cuuint32_t box[2] = {static_cast<cuuint32_t>(p.srow / 8), static_cast<cuuint32_t>(kTile)};
    const cuuint32_t estr[2] = {1, 1};
    const CUresult r = encode(out, CU_TENSOR_MAP_DATA_TYPE_UINT64, 2, const_cast<void*>(w), dims, strides, box, estr,
                              CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE,
                              CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    return r == CUDA_SUCCESS;
}

cudaError_t gemv_launch(int kind, int prologue, int epilogue, GemvArgs a, const CUtensorMap& tmap, const GemvPlan& p,
                        cudaStream_t s, bool pdl) {
    a.nseg = (a.K + 255) / 256;
    a.seg_bytes = kind == kQ4K ? 144 : 512;
    a.row_bytes = kind == kQ4K ? a.nseg * 144 : a.K * 2;
    a.spst = p.spst;
    a.srow = p.srow;
    a.nbuf = p.nbuf;
    a.stage_bytes = p.stage_bytes;
    a.pair = epilogue == kEpiGeluPair ? 2 : 1;
    a.x_smem = p.x_smem;
    cudaError_t err = cudaErrorInvalidValue;
    // The dynamic shared-memory limit is raised by gemv_prepare (not here: this
    // function also runs under stream capture).
    dispatch(kind, prologue, epilogue,
             [&](auto k) { err = rt_launch(k, dim3(p.grid), dim3(p.warps * 32), p.smem, s, pdl, a, tmap); });
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
