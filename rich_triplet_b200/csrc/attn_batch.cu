// attn_batch.cu -- decode attention over many rows (attn_batch.cuh).
//
// Chunk kernel: persistent, one CTA per SM, work items (row b, KV head h,
// chunk c) dealt round-robin.  Warp 8 (lane 0) streams the item's cached K
// and V rows into a ring of 16 shared-memory stages with bulk copies (one
// tile = 4 KB of K rows + 4 KB of V rows, 1024 / D positions), running ahead
// across items.  Tile g of the CTA's stream goes to stage g % 16 and consumer
// warp g % 8, so every stage has one consumer warp that takes its phases in
// order; each warp keeps its own online softmax (max m, sum l, unnormalised
// output) for the G query heads of KV head h.  Lane l owns the dims
// 128 f + 4 l .. + 3 of every row, so each shared-memory load of a warp reads
// 512 contiguous bytes.  Scores: each lane
// forms partial dot products for all G x T (query head, position) pairs of a
// tile, and a transposing butterfly (one shuffle per score) leaves each lane
// with one full score.  At the end of an item the eight warp states are
// combined in shared memory (two combine areas, alternating between items,
// so one named barrier per item suffices); an item that covers all attended
// positions writes the output, otherwise it writes its state to `part`, and
// the merge kernel (one CTA per row and KV head) combines the chunks.
//
// Every wait gives up after a second (globaltimer), records kErrMbarTimeout
// and lets the CTA run to its end without further copies.
#include <math.h>

#include <algorithm>

#include "attention_core.cuh"
#include "attn_batch.cuh"
#include "common.cuh"

namespace rt {

namespace {

constexpr int kCWarps = 8;                        // consumer warps
constexpr int kChunkThreads = (kCWarps + 1) * 32;  // + the producer warp
constexpr int kRingStages = 2 * kCWarps;         // stage s is consumed by warp s % kCWarps only
constexpr int kTileBytes = 4096;                   // K (or V) rows of one tile

template <int D, int G>
struct ChunkCfg {
    static constexpr int T = kTileBytes / (D * 4);  // positions per tile
    static constexpr int NV = G * T;                // scores per tile
    static constexpr int REP = 32 / NV;             // lanes holding each score
    static constexpr int NF4 = D / 128;             // float4 groups per lane and row
    static constexpr int CS = D + 4;                // floats per combine row: D outputs, m, l, pad (16-byte rows)
    static constexpr int kStageBytes = 2 * kTileBytes;
    static constexpr int kCombFloats = kCWarps * G * CS;
    static constexpr int kOffComb = kRingStages * kStageBytes;               // [2][kCWarps][G][CS] floats
    static constexpr int kOffBar = kOffComb + 2 * kCombFloats * 4;           // full[], empty[]
    static constexpr int kOffFlag = kOffBar + 2 * kRingStages * 8;
    static constexpr int kSmem = kOffFlag + 16;
    static_assert(D % 128 == 0 && NV <= 32 && 32 % NV == 0, "tile shape");
    static_assert(kOffBar % 8 == 0 && kSmem <= 227 * 1024, "shared memory");
};

__device__ __forceinline__ void named_sync_consumers() { asm volatile("bar.sync 1, %0;" ::"n"(kCWarps * 32) : "memory"); }

// In lane l: the sum over the warp of v[l / (32 / NV)] (a transposing
// butterfly: at each of the first log2(NV) steps a lane keeps half of its
// values, selected by one bit of its lane index, and adds its partner's copy
// of that half; the remaining steps add plainly).
template <int NV>
__device__ __forceinline__ float transpose_reduce(float (&v)[NV], int lane) {
#pragma unroll
    for (int st = 0; st < 5; ++st) {
        const int o = 16 >> st;
        const int n = NV >> st;
        if (n > 1) {
            const bool up = (lane & o) != 0;
#pragma unroll
            for (int i = 0; i < n / 2; ++i) {
                const float keep = up ? v[i + n / 2] : v[i];
                const float send = up ? v[i] : v[i + n / 2];
                v[i] = keep + __shfl_xor_sync(0xffffffffu, send, o);
            }
        } else {
            v[0] += __shfl_xor_sync(0xffffffffu, v[0], o);
        }
    }
    return v[0];
}

struct Item {
    int b, h, c;
    int nch;     // chunks of (b, h) in use
    int p0, p1;  // cached positions [p0, p1) of this chunk
    bool empty;
};

__device__ __forceinline__ Item decode_item(const AttnChunkArgs& a, int item) {
    Item it;
    it.c = item % a.nchunk;
    it.h = (item / a.nchunk) % a.nkv;
    it.b = item / (a.nchunk * a.nkv);
    const int L = a.pos[it.b] + 1;
    const int kstart = a.window > 0 ? max(0, L - a.window) : 0;
    const int n = L - kstart;
    it.nch = (n + kAttnChunk - 1) / kAttnChunk;
    it.p0 = kstart + it.c * kAttnChunk;
    it.p1 = min(L, it.p0 + kAttnChunk);
    it.empty = it.c >= it.nch;
    return it;
}

__device__ __forceinline__ float lse_w(float m, float M) { return m == -INFINITY ? 0.f : expf(m - M); }

template <int D, int G>
__global__ void __launch_bounds__(kChunkThreads, 1) attn_chunk_kernel(const AttnChunkArgs a) {
    using C = ChunkCfg<D, G>;
    constexpr int T = C::T, NV = C::NV, REP = C::REP, NF4 = C::NF4, CS = C::CS;
    extern __shared__ __align__(128) uint8_t smem[];
    float* comb = reinterpret_cast<float*>(smem + C::kOffComb);
    uint64_t* full = reinterpret_cast<uint64_t*>(smem + C::kOffBar);
    uint64_t* empty = full + kRingStages;
    volatile int* flag = reinterpret_cast<volatile int*>(smem + C::kOffFlag);  // [0] abort
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int nitems = a.B * a.nkv * a.nchunk;
    if (threadIdx.x == 0) {
        for (int s = 0; s < kRingStages; ++s) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], 1);
        }
        flag[0] = 0;
        fence_mbar_init();
    }
    __syncthreads();

    if (warp == kCWarps) {
        // ---- producer ----
        if (lane == 0) {
            uint32_t gt = 0;
            for (int item = blockIdx.x; item < nitems && !flag[0]; item += gridDim.x) {
                const Item it = decode_item(a, item);
                if (it.empty) continue;
                const float* kc = a.kcache + it.b * a.seq_kv + static_cast<int64_t>(it.h) * a.cap * D;
                const float* vc = a.vcache + it.b * a.seq_kv + static_cast<int64_t>(it.h) * a.cap * D;
                for (int r0 = it.p0; r0 < it.p1; r0 += T, ++gt) {
                    const int s = static_cast<int>(gt % kRingStages);
                    if (gt >= kRingStages && !mbar_wait_timed(&empty[s], (gt / kRingStages - 1) & 1u)) {
                        flag[0] = 1;
                        if (a.err) atomicExch(a.err, kErrMbarTimeout);
                        break;
                    }
                    if (flag[0]) break;
                    const uint32_t bytes = static_cast<uint32_t>(min(T, it.p1 - r0)) * D * 4;
                    uint8_t* st = smem + s * C::kStageBytes;
                    mbar_arrive_expect_tx(&full[s], 2 * bytes);
                    bulk_g2s_nohint(st, kc + static_cast<int64_t>(r0) * D, bytes, &full[s]);
                    bulk_g2s_nohint(st + kTileBytes, vc + static_cast<int64_t>(r0) * D, bytes, &full[s]);
                }
            }
            // The last copies into each stage must land before the CTA exits.
            for (uint32_t i = gt > kRingStages ? gt - kRingStages : 0; i < gt; ++i)
                (void)mbar_wait_timed(&full[i % kRingStages], (i / kRingStages) & 1u);
        }
        return;
    }

    // ---- consumers ----
    uint32_t gt_base = 0;  // ring index of the item's first tile
    int cpar = 0;          // combine area of this item
    for (int item = blockIdx.x; item < nitems; item += gridDim.x) {
        const Item it = decode_item(a, item);
        if (it.empty) continue;
        float* const cbuf = comb + cpar * C::kCombFloats;
        cpar ^= 1;
        const int ntiles = (it.p1 - it.p0 + T - 1) / T;
        // this warp's queries, lane-owned dims
        float q[G][4 * NF4];
        const float* qb = a.q + (static_cast<int64_t>(it.b) * a.nq + it.h * G) * D;
#pragma unroll
        for (int g = 0; g < G; ++g)
#pragma unroll
            for (int f = 0; f < NF4; ++f) {
                const float4 v = *reinterpret_cast<const float4*>(qb + g * D + 128 * f + 4 * lane);
                q[g][4 * f] = v.x;
                q[g][4 * f + 1] = v.y;
                q[g][4 * f + 2] = v.z;
                q[g][4 * f + 3] = v.w;
            }
        float acc[G][4 * NF4];
#pragma unroll
        for (int g = 0; g < G; ++g)
#pragma unroll
            for (int i = 0; i < 4 * NF4; ++i) acc[g][i] = 0.f;
        const int jl = (lane / REP) % T;         // position (within the tile) of the score this lane holds
        float m_mine = -INFINITY, l_mine = 0.f;  // state of this lane's query head, (lane / REP) / T
        const int first = static_cast<int>((static_cast<uint32_t>(warp) + kCWarps - gt_base % kCWarps) % kCWarps);
        for (int t = first; t < ntiles; t += kCWarps) {
            const uint32_t gt = gt_base + static_cast<uint32_t>(t);  // gt % kCWarps == warp
            const int s = static_cast<int>(gt % kRingStages);
            const int nt = min(T, it.p1 - (it.p0 + t * T));
            bool ok = !flag[0];
            if (ok && !mbar_wait_timed(&full[s], (gt / kRingStages) & 1u)) {
                flag[0] = 1;
                if (a.err) atomicExch(a.err, kErrMbarTimeout);
                ok = false;
            }
            if (ok) {
                const float* kt = reinterpret_cast<const float*>(smem + s * C::kStageBytes);
                const float* vt = kt + kTileBytes / 4;
                float part[NV];
#pragma unroll
                for (int j = 0; j < T; ++j) {
                    if (j < nt) {
                        float4 kk[NF4];
#pragma unroll
                        for (int f = 0; f < NF4; ++f) kk[f] = *reinterpret_cast<const float4*>(kt + j * D + 128 * f + 4 * lane);
#pragma unroll
                        for (int g = 0; g < G; ++g) {
                            float d = 0.f;
#pragma unroll
                            for (int f = 0; f < NF4; ++f)
                                d += q[g][4 * f] * kk[f].x + q[g][4 * f + 1] * kk[f].y + q[g][4 * f + 2] * kk[f].z +
                                     q[g][4 * f + 3] * kk[f].w;
                            part[g * T + j] = d;
                        }
                    } else {
#pragma unroll
                        for (int g = 0; g < G; ++g) part[g * T + j] = 0.f;
                    }
                }
                float sc = transpose_reduce<NV>(part, lane);
                sc = jl < nt ? sc * a.scale : -INFINITY;
                float tmax = sc;
#pragma unroll
                for (int o = REP; o < T * REP; o <<= 1) tmax = fmaxf(tmax, __shfl_xor_sync(0xffffffffu, tmax, o));
                const float mnew = fmaxf(m_mine, tmax);
                const float p = jl < nt ? expf(sc - mnew) : 0.f;
                const float corr = lse_w(m_mine, mnew);
                float psum = p;
#pragma unroll
                for (int o = REP; o < T * REP; o <<= 1) psum += __shfl_xor_sync(0xffffffffu, psum, o);
                l_mine = l_mine * corr + psum;
                m_mine = mnew;
#pragma unroll
                for (int g = 0; g < G; ++g) {
                    const float cg = __shfl_sync(0xffffffffu, corr, g * T * REP);
#pragma unroll
                    for (int i = 0; i < 4 * NF4; ++i) acc[g][i] *= cg;
                }
#pragma unroll
                for (int j = 0; j < T; ++j) {
                    if (j < nt) {
                        float4 vv[NF4];
#pragma unroll
                        for (int f = 0; f < NF4; ++f) vv[f] = *reinterpret_cast<const float4*>(vt + j * D + 128 * f + 4 * lane);
#pragma unroll
                        for (int g = 0; g < G; ++g) {
                            const float pg = __shfl_sync(0xffffffffu, p, (g * T + j) * REP);
#pragma unroll
                            for (int f = 0; f < NF4; ++f) {
                                acc[g][4 * f] += pg * vv[f].x;
                                acc[g][4 * f + 1] += pg * vv[f].y;
                                acc[g][4 * f + 2] += pg * vv[f].z;
                                acc[g][4 * f + 3] += pg * vv[f].w;
                            }
                        }
                    }
                }
            }
            __syncwarp();
            if (lane == 0) mbar_arrive(&empty[s]);
        }
        gt_base += static_cast<uint32_t>(ntiles);

        // ---- combine the warps' states; write the output or this chunk's state ----
#pragma unroll
        for (int g = 0; g < G; ++g) {
            float* cw = cbuf + (warp * G + g) * CS;
#pragma unroll
            for (int f = 0; f < NF4; ++f)
                *reinterpret_cast<float4*>(cw + 128 * f + 4 * lane) =
                    make_float4(acc[g][4 * f], acc[g][4 * f + 1], acc[g][4 * f + 2], acc[g][4 * f + 3]);
            const float mg = __shfl_sync(0xffffffffu, m_mine, g * T * REP);
            const float lg = __shfl_sync(0xffffffffu, l_mine, g * T * REP);
            if (lane == 0) {
                cw[D] = mg;
                cw[D + 1] = lg;
            }
        }
        named_sync_consumers();
        const int tid = threadIdx.x;
        const int64_t bh = static_cast<int64_t>(it.b) * a.nkv + it.h;
        float* out = a.out + (static_cast<int64_t>(it.b) * a.nq + it.h * G) * D;
        const int stride = D + 4;
        for (int idx = tid; idx < G * D; idx += kCWarps * 32) {
            const int g = idx / D, d = idx % D;
            float M = -INFINITY;
#pragma unroll
            for (int w = 0; w < kCWarps; ++w) M = fmaxf(M, cbuf[(w * G + g) * CS + D]);
            float Ls = 0.f, A = 0.f;
#pragma unroll
            for (int w = 0; w < kCWarps; ++w) {
                const float* cw = cbuf + (w * G + g) * CS;
                const float e = lse_w(cw[D], M);
                Ls += cw[D + 1] * e;
                A += cw[d] * e;
            }
            if (it.nch == 1) {
                out[g * D + d] = A / Ls;
            } else {
                float* pp = a.part + ((bh * a.nchunk + it.c) * G + g) * stride;
                pp[d] = A;
                if (d == 0) {
                    pp[D] = M;
                    pp[D + 1] = Ls;
                }
            }
        }
    }
}

// Chunk states of (row b, KV head h) -> output, for rows with more than one
// chunk.  One CTA per (b, h): the chunks' (m, l) pairs and weights
// exp(m - M) go through shared memory; each thread adds its (g, d) outputs over
// the chunks in chunk order.
template <int G>
__global__ void __launch_bounds__(256) attn_merge_kernel(const AttnChunkArgs a) {
    extern __shared__ float wsm[];  // [nchunk][G] weights, then [G] sums
    const int bh = blockIdx.x, b = bh / a.nkv, h = bh % a.nkv;
    const int D = a.D, stride = D + 4;
    const int L = a.pos[b] + 1;
    const int kstart = a.window > 0 ? max(0, L - a.window) : 0;
    const int nch = (L - kstart + kAttnChunk - 1) / kAttnChunk;
    if (nch <= 1) return;
    const float* pb = a.part + static_cast<int64_t>(bh) * a.nchunk * G * stride;
    float* lsum = wsm + a.nchunk * G;
    if (threadIdx.x < G) {
        const int g = threadIdx.x;
        float M = -INFINITY;
        for (int c = 0; c < nch; ++c) M = fmaxf(M, pb[(c * G + g) * stride + D]);
        float Ls = 0.f;
        for (int c = 0; c < nch; ++c) {
            const float e = lse_w(pb[(c * G + g) * stride + D], M);
            wsm[c * G + g] = e;
            Ls += pb[(c * G + g) * stride + D + 1] * e;
        }
        lsum[g] = Ls;
    }
    __syncthreads();
    float* out = a.out + (static_cast<int64_t>(b) * a.nq + h * G) * D;
    for (int idx = threadIdx.x; idx < G * D; idx += blockDim.x) {
        const int g = idx / D, d = idx % D;
        float A = 0.f;
        for (int c = 0; c < nch; ++c) A += pb[(c * G + g) * stride + d] * wsm[c * G + g];
        out[g * D + d] = A / lsum[g];
    }
}

// One warp: dst[D] = rope(rmsnorm(raw) * (1 + gamma)), the arithmetic of
// acore::head_prep_warp in the same order, with the NeoX pairs (j, j + D/2)
// taken from registers: for D a multiple of 64 both halves of a pair belong
// to the same lane (element j is lane j % 32's value D/32-slot j / 32).
// raw[0] + raw[stride] + ... (`parts` <= 8 terms, added in part order as the
// split-K sum kernel adds them), every load issued before the first add.
__device__ __forceinline__ float ld_parts(const float* raw, int parts, int64_t stride) {
    constexpr int kMax = 8;  // the GEMM plan's split cap
    float w[kMax];
#pragma unroll
    for (int q = 0; q < kMax; ++q) w[q] = q < parts ? raw[q * stride] : 0.f;
    float v = w[0];
#pragma unroll
    for (int q = 1; q < kMax; ++q)
        if (q < parts) v += w[q];
    return v;
}

__device__ __forceinline__ void head_prep_reg(const float* raw, int parts, int64_t stride, const float* gamma,
                                              const float* cs, const float* sn, int D, float eps, float* dst) {
    constexpr int kMaxPer = acore::kMaxHeadDim / 32;
    const int lane = threadIdx.x & 31, per = D / 32, hp = per / 2;
    float x[kMaxPer];
    float ss = 0.f;
#pragma unroll
    for (int i = 0; i < kMaxPer; ++i) {
        const int j = lane + 32 * i;
        x[i] = i < per ? ld_parts(raw + j, parts, stride) : 0.f;
    }
#pragma unroll
    for (int i = 0; i < kMaxPer; ++i) ss += x[i] * x[i];
    ss = warp_sum(ss);
    const float r = 1.0f / sqrtf(ss * (1.0f / static_cast<float>(D)) + eps);
#pragma unroll
    for (int i = 0; i < kMaxPer / 2; ++i) {
        if (i < hp) {
            const int j = lane + 32 * i, jh = j + D / 2;
            const float x0 = __fmul_rn(__fmul_rn(x[i], r), __fadd_rn(1.0f, gamma[j]));
            const float x1 = __fmul_rn(__fmul_rn(x[i + hp], r), __fadd_rn(1.0f, gamma[jh]));
            const float c = cs[j], s = sn[j];
            dst[j] = __fsub_rn(__fmul_rn(x0, c), __fmul_rn(x1, s));
            dst[jh] = __fadd_rn(__fmul_rn(x0, s), __fmul_rn(x1, c));
        }
    }
}

__global__ void attn_rows_prep_kernel(const AttnRowsArgs a) {
    const int b = blockIdx.x, head = blockIdx.y, lane = threadIdx.x;
    const int D = a.D;
    const int p = a.pos[b];
    const int parts = a.parts > 1 ? a.parts : 1;
    const float* row = a.qkv + static_cast<int64_t>(b) * a.qkv_stride;
    const float* cs = a.rope_cos + static_cast<int64_t>(p) * (D / 2);
    const float* sn = a.rope_sin + static_cast<int64_t>(p) * (D / 2);
    if (head < a.nq) {
        head_prep_reg(row + static_cast<int64_t>(head) * D, parts, a.part_stride, a.q_norm, cs, sn, D, a.eps,
                      a.q_out + (static_cast<int64_t>(b) * a.nq + head) * D);
    } else {
        const int h = head - a.nq;
        const int64_t off = b * a.seq_kv + (static_cast<int64_t>(h) * a.cap + p) * D;
        head_prep_reg(row + static_cast<int64_t>(a.nq + h) * D, parts, a.part_stride, a.k_norm, cs, sn, D, a.eps,
                      a.kcache + off);
        const float* vr = row + static_cast<int64_t>(a.nq + a.nkv + h) * D;
        for (int d = lane; d < D; d += 32) a.vcache[off + d] = ld_parts(vr + d, parts, a.part_stride);
    }
}

template <int D, int G>
cudaError_t launch_chunk(const AttnChunkArgs& a, int num_sms, cudaStream_t s) {
    const int nitems = a.B * a.nkv * a.nchunk;
    const int grid = std::max(1, std::min(nitems, num_sms > 0 ? num_sms : 148));
    attn_chunk_kernel<D, G><<<grid, kChunkThreads, ChunkCfg<D, G>::kSmem, s>>>(a);
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess || a.nchunk == 1) return e;
    attn_merge_kernel<G><<<a.B * a.nkv, 256, sizeof(float) * (a.nchunk + 1) * G, s>>>(a);
    return cudaGetLastError();
}

}  // namespace

int attn_chunk_count(int cap, int window) {
    const int n = window > 0 ? std::min(cap, window) : cap;
    return std::max(1, (n + kAttnChunk - 1) / kAttnChunk);
}

size_t attn_chunk_part_floats(int B, int nkv, int nchunk, int G, int D) {
    return static_cast<size_t>(B) * nkv * nchunk * G * (D + 4);
}

bool attn_chunk_supported(int D, int G) {
    return (D == 256 && (G == 1 || G == 2 || G == 4)) || (D == 128 && (G == 1 || G == 2));
}

cudaError_t attn_chunk_prepare() {
    cudaError_t e = cudaSuccess;
    auto set = [&](auto kernel, int bytes) {
        if (e == cudaSuccess) e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes);
    };
    set(attn_chunk_kernel<256, 1>, ChunkCfg<256, 1>::kSmem);
    set(attn_chunk_kernel<256, 2>, ChunkCfg<256, 2>::kSmem);
    set(attn_chunk_kernel<256, 4>, ChunkCfg<256, 4>::kSmem);
    set(attn_chunk_kernel<128, 1>, ChunkCfg<128, 1>::kSmem);
    set(attn_chunk_kernel<128, 2>, ChunkCfg<128, 2>::kSmem);
    return e;
}

cudaError_t attn_rows_prep_launch(const AttnRowsArgs& a, int B, cudaStream_t s) {
    if (B < 1 || a.nq + a.nkv > 65535 || a.D > acore::kMaxHeadDim || a.D % 64 != 0)
        return cudaErrorInvalidValue;
    attn_rows_prep_kernel<<<dim3(static_cast<unsigned>(B), static_cast<unsigned>(a.nq + a.nkv)), 32, 0, s>>>(a);
    return cudaGetLastError();
}

cudaError_t attn_chunk_launch(const AttnChunkArgs& a, int num_sms, cudaStream_t s) {
    if (a.nq % a.nkv != 0 || a.B < 1 || a.nchunk < 1) return cudaErrorInvalidValue;
    const int G = a.nq / a.nkv;
    if (a.D == 256 && G == 1) return launch_chunk<256, 1>(a, num_sms, s);
    if (a.D == 256 && G == 2) return launch_chunk<256, 2>(a, num_sms, s);
    if (a.D == 256 && G == 4) return launch_chunk<256, 4>(a, num_sms, s);
    if (a.D == 128 && G == 1) return launch_chunk<128, 1>(a, num_sms, s);
    if (a.D == 128 && G == 2) return launch_chunk<128, 2>(a, num_sms, s);
    return cudaErrorInvalidValue;
}

}  // namespace rt
