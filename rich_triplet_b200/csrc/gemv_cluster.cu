// gemv_cluster.cu -- the Q4_K GEMV of the standalone entry points
// (rt_gemv_q4k, rt_gemv_bench): y = W x for a row-major [rows, K] Q4_K matrix
// (Q4KMat::gemv_mt, src/autograd2.rs:1953-2035; Metal gemv_q4k_t,
// src/metal_decode.rs:368-425).
//
// Built for a GEMV that is one launch of a chain (a PDL chain or a CUDA graph
// of GEMVs), where the cost to beat is latency, not arithmetic:
//  * A CTA is 8 warps with about 110 KB of shared memory, so a CTA of the next
//    GEMV in the chain fits on the same SM and starts streaming its weights
//    (TMA, before its griddepcontrol.wait) while this one finishes.
//  * Every warp's units (16 rows x 256 columns, one 2-D TMA box of the
//    row-major blocks) are copied into a private ring that holds most or all
//    of its share, all issued at launch.
//  * Two CTAs (on SMs of one GPC) form a thread-block cluster that owns whole
//    16-row tiles; its 16 warps split the cluster's units evenly.  A tile shared by several
//    warps is summed through distributed shared memory (each warp stores its
//    16 row sums into the cluster's CTA 0, one cluster barrier, CTA 0 adds
//    them in warp order), so there is no global scratch, atomic or fence.
//  * The planes of x (gemv_core.cuh) are built once per cluster: CTA r
//    quantises segments r, r + 2, ... and stores them into both CTAs' shared
//    memory.
// The unit arithmetic is gemv_core's (IMMA on three int8 planes of x, the
// scales applied per row and sub-block), so results match the other GEMV
// kernels' to rounding.
//
// Every wait is bounded: mbarrier waits by iteration count (GemvArgs::
// wait_iters, or the default); a warp whose wait gave up records kErrMbarTimeout,
// waits (bounded) for its copies in flight and still takes part in the cluster
// barriers: every thread of every CTA arrives at each of the three, and every
// thread of CTA 0 (the other CTA: the first two) waits on it.
#include <algorithm>

#include "common.cuh"
#include "gemv.cuh"
#include "gemv_core.cuh"

namespace rt {

namespace {

using namespace gcore;

constexpr int kCW = 8;             // warps per CTA
constexpr int kCC = 2;             // CTAs per cluster (clusters of 4 do not all fit at one CTA per SM:
                                   // a GPC holds 18-19 SMs, so only 33 of 37 are resident)
constexpr int kCWarps = kCW * kCC;  // warps per cluster
constexpr int kCMaxNb = 8;          // ring slots per warp, at most
constexpr size_t kCSmemCap = 112 * 1024;  // two CTAs per SM (the next GEMV's beside this one)

struct CSmem {
    uint64_t* full;  // [kCW][nb] unit landed
    int* flags;      // [4]: 0 = a wait gave up
    float* pieces;   // [kCWarps][2][16] row sums of split tiles (read in the cluster's CTA 0)
    uint8_t* planes;
    float2* xsx;     // + the zero line
    uint8_t* ring;   // [kCW][nb][kQ4KUnit]
};

__host__ __device__ inline size_t c_carve(uint8_t* base, int Kp, int nb, CSmem* S) {
    size_t off = 0;
    auto take = [&](size_t bytes, size_t align) -> uint8_t* {
        off = (off + align - 1) / align * align;
        uint8_t* p = base + off;
        off += bytes;
        return p;
    };
    uint8_t* full = take(sizeof(uint64_t) * kCW * nb, 16);
    uint8_t* flags = take(16, 16);
    uint8_t* pieces = take(sizeof(float) * kCWarps * 2 * kTile, 16);
    uint8_t* planes = take(planes_bytes(kQ4K, Kp), 128);
    uint8_t* xsx = take(xsx_bytes(kQ4K, Kp), 16);
    uint8_t* ring = take(static_cast<size_t>(kCW) * nb * kQ4KUnit, 128);
    if (S) {
        S->full = reinterpret_cast<uint64_t*>(full);
        S->flags = reinterpret_cast<int*>(flags);
        S->pieces = reinterpret_cast<float*>(pieces);
        S->planes = planes;
        S->xsx = reinterpret_cast<float2*>(xsx);
        S->ring = ring;
    }
    return off;
}

__device__ __forceinline__ uint32_t cluster_rank() {
    uint32_t r;
    asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
    return r;
}

// Every thread of every CTA of the cluster; orders earlier shared-memory
// stores (local and remote) before later accesses.
__device__ __forceinline__ void cluster_sync() {
    asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}
// The same without ordering: only that every CTA of the cluster is running.
__device__ __forceinline__ void cluster_sync_relaxed() {
    asm volatile("barrier.cluster.arrive.relaxed.aligned;\n\tbarrier.cluster.wait.aligned;" ::: "memory");
}
// Arrival alone (release: this thread's earlier remote stores become visible
// to the threads that wait on the barrier).
__device__ __forceinline__ void cluster_arrive() {
    asm volatile("barrier.cluster.arrive.release.aligned;" ::: "memory");
}
__device__ __forceinline__ void cluster_wait() {
    asm volatile("barrier.cluster.wait.acquire.aligned;" ::: "memory");
}

// Address of `local` (this CTA's shared memory) in CTA `rank` of the cluster.
__device__ __forceinline__ uint32_t map_rank(const void* local, uint32_t rank) {
    uint32_t r;
    asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(smem_u32(local)), "r"(rank));
    return r;
}

__device__ __forceinline__ void st_cluster_u32(uint32_t addr, uint32_t v) {
    asm volatile("st.shared::cluster.u32 [%0], %1;" ::"r"(addr), "r"(v) : "memory");
}

// The planes of one 256-column segment (lane l holds elements 8l..8l+7),
// quantised once and stored into the planes / xsx of all kCC CTAs: the same
// bytes, at the same offsets, as q4k_segment_planes writes.
__device__ __forceinline__ void segment_planes_cluster(const float (&xv)[8], int seg, int lane, int pstride,
                                                       uint8_t* planes, float2* xsx2) {
    float m = 0.f, sum = 0.f;
#pragma unroll
    for (int e = 0; e < 8; ++e) {
        m = fmaxf(m, fabsf(xv[e]));
        sum += xv[e];
    }
    sum += __shfl_xor_sync(0xffffffffu, sum, 1);
    sum += __shfl_xor_sync(0xffffffffu, sum, 2);
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
    const float s = m * (1.0f / 127.0f);
    const float inv = m > 1e-30f ? __fdividef(127.0f, m) : 0.f;
    const float s254 = s * (1.0f / 254.0f);
    const float inv254 = inv * 254.0f, inv254sq = inv * 64516.0f;
    uint32_t b0[8], b1[8], b2[8];
#pragma unroll
    for (int e = 0; e < 8; ++e) {
        const float f0 = round_clamp127(xv[e] * inv, &b0[e]);
        const float r1 = fmaf(-f0, s, xv[e]);
        const float f1 = round_clamp127(r1 * inv254, &b1[e]);
        const float r2 = fmaf(-f1, s254, r1);
        (void)round_clamp127(r2 * inv254sq, &b2[e]);
    }
    const int j = lane >> 2;
    const int par = j & 1, jj = j >> 1, q = lane & 3;
    const int t0 = 2 * (q & 1), hi = q >> 1;
    const int o0 = seg * 256 + (jj >> 1) * 128 + (par * 4 + t0) * 16 + (jj & 1) * 8 + hi * 4;
    const int o1 = o0 + 16;
    const uint32_t w[6] = {pack4_low(b0[0], b0[1], b0[2], b0[3]), pack4_low(b0[4], b0[5], b0[6], b0[7]),
                           pack4_low(b1[0], b1[1], b1[2], b1[3]), pack4_low(b1[4], b1[5], b1[6], b1[7]),
                           pack4_low(b2[0], b2[1], b2[2], b2[3]), pack4_low(b2[4], b2[5], b2[6], b2[7])};
    const int off[6] = {o0, o1, pstride + o0, pstride + o1, 2 * pstride + o0, 2 * pstride + o1};
    float* xf = reinterpret_cast<float*>(xsx2) + seg * kQ4KXsxFloats;
#pragma unroll
    for (uint32_t r = 0; r < kCC; ++r) {
        const uint32_t pb = map_rank(planes, r);
#pragma unroll
        for (int k = 0; k < 6; ++k) st_cluster_u32(pb + off[k], w[k]);
        if (q == 0) st_cluster_u32(map_rank(xf + par * 4 + jj, r), __float_as_uint(sum));
        if (lane == 0) st_cluster_u32(map_rank(xf + 8, r), __float_as_uint(s * (1.0f / 64516.0f)));
    }
}

__global__ void __cluster_dims__(kCC, 1, 1) __launch_bounds__(kCW * 32, 2)
    gemv_q4k_cluster_kernel(const GemvArgs a, const __grid_constant__ CUtensorMap tmap) {
    extern __shared__ __align__(128) uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 127) & ~uintptr_t{127});
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int nseg = a.nseg, nb = a.nb, K = a.K;
    const int Kp = nseg * kQ4KSegCols;
    const int pstride = q4k_pstride(Kp);
    CSmem S;
    c_carve(smem, Kp, nb, &S);
    const uint32_t rank = cluster_rank();
    const uint32_t cid = blockIdx.x / kCC, ncl = gridDim.x / kCC;
    const uint32_t cw = rank * kCW + warp;  // this warp's index in the cluster
    // The cluster's whole tiles and units; the warps' equal shares of them.
    const int64_t rows = a.rows;
    const uint32_t ntiles = static_cast<uint32_t>((rows + kTile - 1) / kTile);
    Split ct;
    ct.init(ntiles, ncl);
    const uint32_t tb = ct.start(cid), te = ct.start(cid + 1);
    const uint32_t u0 = tb * nseg, n = (te - tb) * nseg;
    const uint32_t us = u0 + n * cw / kCWarps, ue = u0 + n * (cw + 1) / kCWarps;
    const uint64_t pol = l2_evict_first_policy();

    // ---- launch: the warp's weight copies, before the wait on the previous kernel ----
    uint64_t* full = S.full + warp * nb;
    uint8_t* ring = S.ring + static_cast<size_t>(warp) * nb * kQ4KUnit;
    uint32_t iu = us;  // next unit to copy
    auto issue = [&](int slot) {
        const uint32_t t = iu / nseg, sg = iu - t * nseg;
        mbar_arrive_expect_tx(&full[slot], static_cast<uint32_t>(kQ4KUnit));
        tma_2d_g2s(ring + static_cast<size_t>(slot) * kQ4KUnit, &tmap, static_cast<int>(sg) * box_step(kQ4K),
                   static_cast<int>(t * kTile), &full[slot], pol);
        ++iu;
    };
    if (lane == 0) {
        for (int k = 0; k < nb; ++k) mbar_init(&full[k], 1);
        fence_mbar_init();
        for (int k = 0; k < nb && iu < ue; ++k) issue(k);
    }
    if (tid == 0) S.flags[0] = 0;
    cluster_sync_relaxed();  // #1: every CTA of the cluster is running (its shared memory may be written)
    pdl_launch_dependents();
    pdl_wait();

    // ---- planes of x, each segment quantised by one CTA and stored in all four ----
#pragma unroll 1
    for (int sg = static_cast<int>(rank) + kCC * warp; sg < nseg; sg += kCC * kCW) {
        float4 lo, hi;
        load8(a.x, sg * kQ4KSegCols + lane * 8, K, lo, hi);
        const float xv[8] = {lo.x, lo.y, lo.z, lo.w, hi.x, hi.y, hi.z, hi.w};
        segment_planes_cluster(xv, sg, lane, pstride, S.planes, S.xsx);
    }
    q4k_zero_line(S.xsx, Kp);
    cluster_sync();  // #2: the planes are complete in every CTA

    // ---- the warp's units ----
    const int g = lane >> 2, t = lane & 3;
    const int ldsm_off = ((lane & 7) + ((lane >> 3) & 1) * 8) * kQ4KPitch + 16 + ((lane >> 4) & 1) * 16;
    const int bpar = g >> 2, bpl = g & 3;
    const int lane_b = bpl * pstride + (bpar * 4 + t) * 16;
    const uint8_t* zline = reinterpret_cast<const uint8_t*>(S.xsx) + static_cast<size_t>(nseg) * kQ4KXsxFloats * 4;
    const bool feeds_lo = bpl < 3 && bpar == 0, feeds_hi = bpl < 3 && bpar == 1;
    const float* xsf = reinterpret_cast<const float*>(S.xsx);
    const uint32_t first_tile = us / nseg;
    float acc0 = 0.f, acc1 = 0.f;  // this lane's share of rows g and g+8 of the current tile
    int pu = 0;                     // units of the current tile piece
    bool ok = true;
    int slot = 0;
    uint32_t ph = 0;
    uint32_t u = us;
#pragma unroll 1
    for (; u < ue; ++u) {
        const bool landed = mbar_wait_n(&full[slot], ph, a.wait_iters);
        if (__any_sync(0xffffffffu, !landed)) {
            ok = false;
            break;
        }
        const uint32_t tile = u / nseg, sg = u - tile * nseg;
        const uint8_t* ub = ring + static_cast<size_t>(slot) * kQ4KUnit;
        const uint8_t* real = S.planes + lane_b + sg * 256;
        const float* xf = xsf + sg * kQ4KXsxFloats;
        const float v = q4k_unit_value(ub, feeds_lo ? real : zline, feeds_hi ? real : zline, g, t, xf[8],
                                       *reinterpret_cast<const float4*>(xf + (t >> 1) * 4), ldsm_off);
        if (t & 1) acc1 += v;
        else acc0 += v;
        ++pu;
        // Release the slot to this warp's next unit.  Every lane's reads of it
        // (ldmatrix, header) completed into registers that the MMAs and the
        // epilogue already consumed, so the copy that overwrites it needs no
        // cross-proxy fence (the CUTLASS TMA pipelines recycle their stages
        // the same way).
        __syncwarp();
        if (lane == 0 && iu < ue) issue(slot);
        if (++slot == nb) {
            slot = 0;
            ph ^= 1u;
        }
        if (sg == static_cast<uint32_t>(nseg) - 1u || u + 1 == ue) {
            // row sums of this piece: quad reduction, then lane L < 16 takes row L
            float s0 = acc0 + __shfl_xor_sync(0xffffffffu, acc0, 1);
            s0 += __shfl_xor_sync(0xffffffffu, s0, 2);
            float s1 = acc1 + __shfl_xor_sync(0xffffffffu, acc1, 1);
            s1 += __shfl_xor_sync(0xffffffffu, s1, 2);
            const float ra = __shfl_sync(0xffffffffu, s0, 4 * (lane & 7));
            const float rb = __shfl_sync(0xffffffffu, s1, 4 * (lane & 7));
            const float rowv = (lane & 8) ? rb : ra;
            const int64_t r = static_cast<int64_t>(tile) * kTile + lane;
            if (pu == nseg) {
                if (lane < kTile && r < rows) a.y[r] = rowv;
            } else if (lane < kTile) {
                // a piece of a shared tile: into the cluster's CTA 0
                const int pslot = tile == first_tile ? 0 : 1;
                st_cluster_u32(map_rank(S.pieces + (cw * 2 + pslot) * kTile + lane, 0), __float_as_uint(rowv));
            }
            acc0 = acc1 = 0.f;
            pu = 0;
        }
    }
    if (!ok && lane == 0) {
        // Bounded wait for this warp's copies in flight (issued, not consumed)
        // before the CTA can leave: the k-th sits in slot (slot + k) % nb, one
        // phase later when it wrapped around the ring.
        S.flags[0] = 1;
        const uint32_t inflight = (iu - us) - (u - us);
        for (uint32_t k = 0; k < inflight; ++k) {
            const uint32_t sk = static_cast<uint32_t>(slot) + k;
            (void)mbar_wait(&full[sk % static_cast<uint32_t>(nb)], (ph ^ ((sk / static_cast<uint32_t>(nb)) & 1u)) & 1u);
        }
    }
    __syncwarp();
    // #3: every piece is in CTA 0.  Only CTA 0 waits: the other CTA's shared
    // memory is not read by anyone after #2, so it may leave once it arrived.
    if (tid == 0 && S.flags[0] && a.err) atomicExch(a.err, kErrMbarTimeout);
    cluster_arrive();
    if (rank != 0) return;
    cluster_wait();
    if (n == 0) return;
    // ---- CTA 0: the shared tiles, pieces added in warp order ----
    auto wstart = [&](uint32_t w) { return n * w / kCWarps; };
    auto owner = [&](uint32_t uu) {  // warp whose share holds cluster unit uu
        const uint32_t w = (kCWarps * (uu + 1) + n - 1) / n - 1;
        return w < kCWarps ? w : kCWarps - 1;
    };
#pragma unroll 1
    for (uint32_t T = tb + warp; T < te; T += kCW) {
        const uint32_t a0 = (T - tb) * nseg, a1 = a0 + nseg - 1;
        const uint32_t wa = owner(a0), wb = owner(a1);
        if (wa == wb) continue;  // one warp had the whole tile: already stored
        float v = 0.f;
        for (uint32_t w = wa; w <= wb; ++w) {
            const uint32_t s0 = wstart(w);
            if (wstart(w + 1) <= s0) continue;  // a warp without units
            if (lane < kTile) v += S.pieces[(w * 2 + (s0 < a0 ? 1 : 0)) * kTile + lane];
        }
        const int64_t r = static_cast<int64_t>(T) * kTile + lane;
        if (lane < kTile && r < rows) a.y[r] = v;
    }
}

}  // namespace

GemvPlan gemv_cluster_plan(int64_t rows, int K, int num_sms) {
    GemvPlan p;
    if (rows <= 0 || K <= 0 || K % 256 != 0 || num_sms < kCC) return p;
    const int nseg = K / 256;
    const int64_t U = ((rows + kTile - 1) / kTile) * nseg;
    if (U >= (int64_t{1} << 31) / kCWarps) return p;
    p.grid = num_sms / kCC * kCC;
    p.warps = kCW;
    p.unit_bytes = kQ4KUnit;
    p.box_x = kQ4KPitch / 8;
    // Ring depth: the warp's whole share if it fits beside the planes within
    // the two-CTAs-per-SM budget, else as many slots as fit (at least 2).
    const int64_t per_warp = (U + static_cast<int64_t>(p.grid) * kCW - 1) / (static_cast<int64_t>(p.grid) * kCW);
    const int want = static_cast<int>(std::min<int64_t>(kCMaxNb, std::max<int64_t>(2, per_warp)));
    for (int nb = want; nb >= 2; --nb) {
        const size_t smem = c_carve(nullptr, K, nb, nullptr) + 128;
        if (smem <= kCSmemCap) {
            p.nb = nb;
            p.smem = smem;
            break;
        }
    }
    if (p.nb == 0) {
        // wide rows: one CTA per SM
        const size_t smem = c_carve(nullptr, K, 2, nullptr) + 128;
        if (smem > 226 * 1024) {
            p.warps = 0;
            return p;
        }
        p.nb = 2;
        p.smem = smem;
    }
    return p;
}

cudaError_t gemv_cluster_prepare() {
    return cudaFuncSetAttribute(gemv_q4k_cluster_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, 226 * 1024);
}

cudaError_t gemv_cluster_launch(GemvArgs a, const CUtensorMap& tmap, const GemvPlan& p, cudaStream_t s, bool pdl) {
    a.nseg = a.K / 256;
    a.nb = p.nb;
    a.unit_bytes = kQ4KUnit;
    return rt_launch(gemv_q4k_cluster_kernel, dim3(p.grid), dim3(p.warps * 32), p.smem, s, pdl, a, tmap);
}

}  // namespace rt
