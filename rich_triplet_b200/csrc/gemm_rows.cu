// gemm_rows.cu -- the Q4_K product at small M as a multi-row GEMV:
// C[M, N] = diag(ascale) . A[M, K] . dequant(W[N, K])^T for M <= 16 rows of A
// (fp16 with a power-of-two scale per row, or f32) and a row-major Q4_K weight W, every
// weight byte streamed once and used for all M rows.  Matmul_q4k_t
// (src/autograd2.rs:1437-1457) is the product's definition; the reference's
// batched GEMV (gemv_q4k_t_batch, src/metal_decode.rs:460-524) computes it
// for its verify step the same way, one pass over W for several rows.
//
// At M <= 16 the product is a weight stream (0.5625 bytes per weight for 2 M
// FLOPs).  This kernel widens the GEMV core's unit arithmetic (gemv_core.cuh)
// to several rows of A:
//  * A row's 256-column segment is split into two int8 planes,
//    a = s (p0 + p1 / 254) with s = max|a| / 127 over the segment (error at
//    most s / 508 per element: 1.6e-5 of the segment's largest magnitude,
//    below the fp16 rounding of A itself).
//  * One mma.sync.m16n8k32.u8.s8 multiplies the nibbles of one sub-block (32
//    columns) of 16 weight rows by 4 rows of A x 2 planes (B column 2 r + p);
//    the low and high nibbles of a 32-byte chunk are two sub-blocks, two
//    MMAs.  Each A fragment feeds M/4 MMAs.
//  * The 6-bit sub-block scales multiply the MMAs' integer sums in int32
//    (exact: at most 8 * 63 * 32 * 240 * 127 < 2^31); each lane then holds,
//    per n8 tile, the two plane sums of rows g and g + 8 of W for row t of A,
//    so the value d * s / 16 * (P0 + P1 / 254) - dmin * sum_j m_j sum(a_j)
//    needs no shuffle.
//  * The min term sum_j m_j sum(a_j) is one more MMA per n8 tile: the 6-bit
//    mins of the 16 rows (A, k = sub-block) times the sub-block sums of A,
//    themselves split into two int8 planes (scale max_j |sum(a_j)| / 127).
//  * The planes sit in shared memory in the MMA's B-fragment order (lane l's
//    16 bytes of a chunk are consecutive), one 16-byte load per chunk and n8
//    tile, no bank conflict.
// Work: K is cut into `parts` column ranges (p.splits, each written as one
// partial product for the caller to add) so that one range's planes fit in
// shared memory beside the weight rings; the CTAs of a part own whole 16-row
// tiles, and their 16 warps split the CTA's units (16 rows x 256 columns)
// evenly.  Each warp streams its units through a private ring of 2-D TMA
// copies (16 rows x 144 bytes); a tile shared by several warps is added in
// warp order in shared memory, so results are deterministic.
// Every wait is bounded: a warp whose wait gives up records kErrMbarTimeout,
// waits (bounded) for its own copies in flight and still reaches the CTA's
// barrier.
#include <algorithm>

#include "common.cuh"
#include "gemm.cuh"
#include "gemv_core.cuh"

namespace rt {

namespace {

using namespace gcore;

constexpr int kRW = 16;               // warps per CTA (one CTA per SM)
constexpr int kRNbMin = 2, kRNbMax = 6;  // ring slots per warp (the plan takes as many as fit)
constexpr int kRTilePlane = 2048;     // B-fragment bytes per segment and n8 tile: 4 chunks x 32 lanes x 16
constexpr size_t kRSmemMax = 227 * 1024;

struct RowsArgs {
    const uint16_t* a;     // fp16 [m][k] (when a32 is null)
    const float* a32;      // or f32 [m][k], no row scale
    const float* ascale;   // [m] or null
    float* c;              // [parts][m][n]
    int* err;
    int64_t n;
    int m, k, nseg, spp, parts, cpp, nb;
};

struct RowsSmem {
    uint64_t* full;   // [kRW][nb] unit landed
    int* flags;       // [4]: 0 = a wait gave up
    float* pieces;    // [kRW][2][4 NT][16] split-tile pieces
    uint8_t* planes;  // [spp][NT][4 chunks][32 lanes][16 bytes]
    uint32_t* splanes;  // [spp][NT][32 lanes]: B fragment of the sub-block sums' planes
    float* useg;      // [spp][4 NT][2]: s / 16, and the sums' plane unit
    uint8_t* ring;    // [kRW][nb][kQ4KUnit]
};

__host__ __device__ inline size_t rows_carve(uint8_t* base, int nt, int spp, int nb, RowsSmem* S) {
    size_t off = 0;
    auto take = [&](size_t bytes, size_t align) -> uint8_t* {
        off = (off + align - 1) / align * align;
        uint8_t* p = base + off;
        off += bytes;
        return p;
    };
    uint8_t* full = take(sizeof(uint64_t) * kRW * nb, 16);
    uint8_t* flags = take(16, 16);
    uint8_t* pieces = take(sizeof(float) * kRW * 2 * 4 * nt * kTile, 16);
    uint8_t* planes = take(static_cast<size_t>(spp) * nt * kRTilePlane, 128);
    uint8_t* splanes = take(sizeof(uint32_t) * spp * nt * 32, 16);
    uint8_t* useg = take(sizeof(float) * spp * 4 * nt * 2, 16);
    uint8_t* ring = take(static_cast<size_t>(kRW) * nb * kQ4KUnit, 128);
    if (S) {
        S->full = reinterpret_cast<uint64_t*>(full);
        S->flags = reinterpret_cast<int*>(flags);
        S->pieces = reinterpret_cast<float*>(pieces);
        S->planes = planes;
        S->splanes = reinterpret_cast<uint32_t*>(splanes);
        S->useg = reinterpret_cast<float*>(useg);
        S->ring = ring;
    }
    return off;
}

// The two planes of row r of A over segment s of the part (lane l holds
// elements 8l..8l+7 of it), stored in B-fragment order: the record of
// (column n = 2 (r % 4) + p, k-quad t') of chunk c holds bytes 4t'..4t'+3 and
// 16+4t'..16+4t'+3 of sub-block 2c, then the same of sub-block 2c+1.
template <int NT>
__device__ __forceinline__ void rows_segment_planes(const float (&xv)[8], int r, int s, int lane, const RowsSmem& S) {
    float m = 0.f, sum = 0.f;
#pragma unroll
    for (int e = 0; e < 8; ++e) {
        m = fmaxf(m, fabsf(xv[e]));
        sum += xv[e];
    }
    sum += __shfl_xor_sync(0xffffffffu, sum, 1);  // a sub-block is 4 lanes
    sum += __shfl_xor_sync(0xffffffffu, sum, 2);
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
    // Each residual is taken against the stored scale s, so the reciprocal
    // only has to be close: |x inv| and |r1 inv 254| stay below 127.5.
    const float sc = m * (1.0f / 127.0f);
    const float inv = m > 1e-30f ? __fdividef(127.0f, m) : 0.f;
    const float inv254 = inv * 254.0f;
    uint32_t b0[8], b1[8];
#pragma unroll
    for (int e = 0; e < 8; ++e) {
        const float f0 = round_clamp127(xv[e] * inv, &b0[e]);
        const float r1 = fmaf(-f0, sc, xv[e]);
        (void)round_clamp127(r1 * inv254, &b1[e]);
    }
    const int j = lane >> 2, q = lane & 3;  // sub-block j, its elements 8q..8q+7
    const int t0 = 2 * (q & 1);              // k-quad of elements 8q..8q+3 (8q+4..: t0 + 1)
    const int col0 = 2 * (r & 3);            // B column of plane 0 (plane 1: col0 + 1)
    uint8_t* base = S.planes + static_cast<size_t>(s * NT + (r >> 2)) * kRTilePlane + (j >> 1) * 512 + (j & 1) * 8 +
                    (q >> 1) * 4;
    *reinterpret_cast<uint32_t*>(base + (col0 * 4 + t0) * 16) = pack4_low(b0[0], b0[1], b0[2], b0[3]);
    *reinterpret_cast<uint32_t*>(base + (col0 * 4 + t0 + 1) * 16) = pack4_low(b0[4], b0[5], b0[6], b0[7]);
    *reinterpret_cast<uint32_t*>(base + ((col0 + 1) * 4 + t0) * 16) = pack4_low(b1[0], b1[1], b1[2], b1[3]);
    *reinterpret_cast<uint32_t*>(base + ((col0 + 1) * 4 + t0 + 1) * 16) = pack4_low(b1[4], b1[5], b1[6], b1[7]);
    // The sub-block sums (every lane holds its sub-block's) as two int8
    // planes over the segment: sum_j = s2 (q0_j + q1_j / 254).
    float m2 = fabsf(sum);
    m2 = fmaxf(m2, __shfl_xor_sync(0xffffffffu, m2, 4));
    m2 = fmaxf(m2, __shfl_xor_sync(0xffffffffu, m2, 8));
    m2 = fmaxf(m2, __shfl_xor_sync(0xffffffffu, m2, 16));
    const float s2 = m2 * (1.0f / 127.0f);
    const float inv2 = m2 > 1e-30f ? __fdividef(127.0f, m2) : 0.f;
    uint32_t c0, c1;
    const float g0 = round_clamp127(sum * inv2, &c0);
    (void)round_clamp127(fmaf(-g0, s2, sum) * (inv2 * 254.0f), &c1);
    // B fragment of the min MMA: lane (column n, k-quad t') holds the planes
    // of sub-blocks 4t'..4t'+3 (t' < 2; k 8..31 are zero); lanes 0 and 16
    // gather sub-blocks 0..3 and 4..7 (held by lanes 4j).
    const int src = (lane & 16);
    const uint32_t p00 = __shfl_sync(0xffffffffu, c0, src), p01 = __shfl_sync(0xffffffffu, c0, src + 4),
                   p02 = __shfl_sync(0xffffffffu, c0, src + 8), p03 = __shfl_sync(0xffffffffu, c0, src + 12);
    const uint32_t p10 = __shfl_sync(0xffffffffu, c1, src), p11 = __shfl_sync(0xffffffffu, c1, src + 4),
                   p12 = __shfl_sync(0xffffffffu, c1, src + 8), p13 = __shfl_sync(0xffffffffu, c1, src + 12);
    uint32_t* sp = S.splanes + static_cast<size_t>(s * NT + (r >> 2)) * 32;
    if ((lane & 15) == 0) {
        const int tq = lane >> 4;
        sp[col0 * 4 + tq] = pack4_low(p00, p01, p02, p03);
        sp[(col0 + 1) * 4 + tq] = pack4_low(p10, p11, p12, p13);
    } else if ((lane & 15) == 1) {
        const int tq = 2 + (lane >> 4);
        sp[col0 * 4 + tq] = 0u;
        sp[(col0 + 1) * 4 + tq] = 0u;
    }
    if (lane == 0) {
        S.useg[(s * 4 * NT + r) * 2] = sc * 0.0625f;  // the high nibbles are seen as 16 q
        S.useg[(s * 4 * NT + r) * 2 + 1] = s2 * (1.0f / 254.0f);
    }
}

// One unit (16 rows of W at shared-memory address ub x one segment): adds to
// acc[nt][0 / 1] this lane's values of W rows g / g + 8 for row 4 nt + t of A.
// pl: this lane's B records of the segment; sp: its B fragments of the
// sub-block sums; us: the segment's plane units.
template <int NT>
__device__ __forceinline__ void rows_unit(const uint8_t* ub, const uint8_t* pl, const uint32_t* sp, const float* us,
                                          int g, int t, int ldsm_off, float (&acc)[NT][2]) {
    const uint4 h0 = lds128(ub + g * kQ4KPitch), h1 = lds128(ub + (g + 8) * kQ4KPitch);
    // scale_min (src/autograd2.rs:1075-1085): sub-blocks 0..3 in the low
    // words, 4..7 in the high words, one byte each
    const uint32_t s0l = h0.y & 0x3F3F3F3Fu, s0h = (h0.w & 0x0F0F0F0Fu) | ((h0.y >> 2) & 0x30303030u);
    const uint32_t s1l = h1.y & 0x3F3F3F3Fu, s1h = (h1.w & 0x0F0F0F0Fu) | ((h1.y >> 2) & 0x30303030u);
    int R[NT][4];
#pragma unroll
    for (int nt = 0; nt < NT; ++nt) R[nt][0] = R[nt][1] = R[nt][2] = R[nt][3] = 0;
#pragma unroll
    for (int c = 0; c < 4; ++c) {
        uint32_t a0, a1, a2, a3;
        ldsm_x4(ub + ldsm_off + 32 * c, a0, a1, a2, a3);
        const uint32_t l0 = a0 & 0x0F0F0F0Fu, l1 = a1 & 0x0F0F0F0Fu, l2 = a2 & 0x0F0F0F0Fu, l3 = a3 & 0x0F0F0F0Fu;
        const uint32_t q0 = sub_on_fma(a0, l0), q1 = sub_on_fma(a1, l1), q2 = sub_on_fma(a2, l2),
                       q3 = sub_on_fma(a3, l3);  // the high nibbles in place: 16 q
        // sub-blocks 2c (low nibbles) and 2c + 1: bytes 2 (c & 1) and 2 (c & 1) + 1
        const uint32_t w0 = c < 2 ? s0l : s0h, w1 = c < 2 ? s1l : s1h;
        const uint32_t sl = 0x4440u | static_cast<uint32_t>(2 * (c & 1)), sh = sl + 1u;
        const int lo0 = static_cast<int>(__byte_perm(w0, 0u, sl)) << 4, hi0 = static_cast<int>(__byte_perm(w0, 0u, sh));
        const int lo1 = static_cast<int>(__byte_perm(w1, 0u, sl)) << 4, hi1 = static_cast<int>(__byte_perm(w1, 0u, sh));
#pragma unroll
        for (int nt = 0; nt < NT; ++nt) {
            const uint4 B = lds128(pl + nt * kRTilePlane + c * 512);
            int cl[4], ch[4];
            mma_u8s8_z(cl, l0, l1, l2, l3, B.x, B.y);
            mma_u8s8_z(ch, q0, q1, q2, q3, B.z, B.w);
            R[nt][0] += lo0 * cl[0] + hi0 * ch[0];
            R[nt][1] += lo0 * cl[1] + hi0 * ch[1];
            R[nt][2] += lo1 * cl[2] + hi1 * ch[2];
            R[nt][3] += lo1 * cl[3] + hi1 * ch[3];
        }
    }
    const float d0 = f16_bits_to_f32(h0.x & 0xFFFFu), dm0 = f16_bits_to_f32(h0.x >> 16);
    const float d1 = f16_bits_to_f32(h1.x & 0xFFFFu), dm1 = f16_bits_to_f32(h1.x >> 16);
    // the min MMA's A: row g's mins of sub-blocks 4t..4t+3 (t < 2), k 8..31 zero
    const uint32_t m0l = h0.z & 0x3F3F3F3Fu, m0h = ((h0.w >> 4) & 0x0F0F0F0Fu) | ((h0.z >> 2) & 0x30303030u);
    const uint32_t m1l = h1.z & 0x3F3F3F3Fu, m1h = ((h1.w >> 4) & 0x0F0F0F0Fu) | ((h1.z >> 2) & 0x30303030u);
    const uint32_t ma0 = t == 0 ? m0l : t == 1 ? m0h : 0u, ma1 = t == 0 ? m1l : t == 1 ? m1h : 0u;
#pragma unroll
    for (int nt = 0; nt < NT; ++nt) {
        const int r = 4 * nt + t;
        int cm[4];
        mma_u8s8_z(cm, ma0, ma1, 0u, 0u, sp[nt * 32], 0u);
        const float2 u = *reinterpret_cast<const float2*>(us + 2 * r);
        const float T0 = fmaf(static_cast<float>(R[nt][1]), 1.0f / 254.0f, static_cast<float>(R[nt][0]));
        const float T1 = fmaf(static_cast<float>(R[nt][3]), 1.0f / 254.0f, static_cast<float>(R[nt][2]));
        const float V0 = fmaf(static_cast<float>(cm[0]), 254.0f, static_cast<float>(cm[1]));
        const float V1 = fmaf(static_cast<float>(cm[2]), 254.0f, static_cast<float>(cm[3]));
        acc[nt][0] += d0 * (T0 * u.x) - dm0 * (V0 * u.y);
        acc[nt][1] += d1 * (T1 * u.x) - dm1 * (V1 * u.y);
    }
}

template <int NT, int EPI>
__global__ void __launch_bounds__(kRW * 32, 1) gemm_rows_q4k_kernel(const RowsArgs a, const __grid_constant__ CUtensorMap tmw) {
    extern __shared__ __align__(128) uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 127) & ~uintptr_t{127});
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    RowsSmem S;
    const int nb = a.nb;
    rows_carve(smem, NT, a.spp, nb, &S);
    const int part = static_cast<int>(blockIdx.x) / a.cpp, ci = static_cast<int>(blockIdx.x) - part * a.cpp;
    const int seg0 = part * a.spp, nsp = min(a.spp, a.nseg - seg0);
    const int64_t n = a.n;
    // this CTA's whole tiles [tb, te) of the part; its warps' equal shares of their units
    Split ct;
    ct.init(static_cast<uint32_t>((n + kTile - 1) / kTile), static_cast<uint32_t>(a.cpp));
    const uint32_t tb = ct.start(ci), te = ct.start(ci + 1);
    const uint32_t un = (te - tb) * static_cast<uint32_t>(nsp);
    const uint32_t us = un * warp / kRW, ue = un * (warp + 1) / kRW;
    const uint64_t pol = l2_evict_first_policy();

    uint64_t* full = S.full + warp * nb;
    uint8_t* ring = S.ring + static_cast<size_t>(warp) * nb * kQ4KUnit;
    uint32_t iu = us;  // next unit to copy: tile row y0 + 16 itl, segment seg0 + isg
    int itl = static_cast<int>(us / nsp), isg = static_cast<int>(us) - itl * nsp;
    const int y0 = static_cast<int>(tb) * kTile;
    auto issue = [&](int slot) {
        mbar_arrive_expect_tx(&full[slot], static_cast<uint32_t>(kQ4KUnit));
        tma_2d_g2s(ring + static_cast<size_t>(slot) * kQ4KUnit, &tmw, (seg0 + isg) * box_step(kQ4K), y0 + itl * kTile,
                   &full[slot], pol);
        ++iu;
        if (++isg == nsp) {
            isg = 0;
            ++itl;
        }
    };
    if (lane == 0) {
        for (int k = 0; k < nb; ++k) mbar_init(&full[k], 1);
        fence_mbar_init();
        for (int k = 0; k < nb && iu < ue; ++k) issue(k);
    }
    if (tid == 0) S.flags[0] = 0;

    // ---- the planes of the part's rows of A (rows m..4 NT-1 are zero) ----
    const int m = a.m;
#pragma unroll 1
    for (int task = warp; task < 4 * NT * nsp; task += kRW) {
        const int r = task % (4 * NT), s = task / (4 * NT);
        float xv[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
        const int64_t off = static_cast<int64_t>(r) * a.k + (seg0 + s) * kQ4KSegCols + lane * 8;
        if (r < m && a.a32) {
            const float4 lo = __ldg(reinterpret_cast<const float4*>(a.a32 + off));
            const float4 hi = __ldg(reinterpret_cast<const float4*>(a.a32 + off + 4));
            xv[0] = lo.x, xv[1] = lo.y, xv[2] = lo.z, xv[3] = lo.w;
            xv[4] = hi.x, xv[5] = hi.y, xv[6] = hi.z, xv[7] = hi.w;
        } else if (r < m) {
            const uint4 v = __ldg(reinterpret_cast<const uint4*>(a.a + off));
            const uint32_t w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
            for (int e = 0; e < 4; ++e) {
                xv[2 * e] = f16_bits_to_f32(w[e] & 0xFFFFu);
                xv[2 * e + 1] = f16_bits_to_f32(w[e] >> 16);
            }
        }
        rows_segment_planes<NT>(xv, r, s, lane, S);
    }
    __syncthreads();

    // ---- the warp's units ----
    const int g = lane >> 2, t = lane & 3;
    const int ldsm_off = ((lane & 7) + ((lane >> 3) & 1) * 8) * kQ4KPitch + 16 + ((lane >> 4) & 1) * 16;
    float as[NT];  // row scale of row 4 nt + t of A
#pragma unroll
    for (int nt = 0; nt < NT; ++nt) {
        const int r = 4 * nt + t;
        as[nt] = r < m ? (a.ascale && !a.a32 ? a.ascale[r] : 1.f) : 0.f;
    }
    float* cpart = a.c + static_cast<int64_t>(part) * m * n;
    constexpr bool gelu = EPI == kRowsEpiGelu;
    auto store = [&](int r, int64_t row, float v) {
        if (r < m && row < n) cpart[static_cast<int64_t>(r) * n + row] = v;
    };
    // GELU gate: weight rows 2j (gate) and 2j + 1 (up) give output column j
    // (src/autograd2.rs:3082-3091, the product not contracted into an FMA).
    auto store_h = [&](int r, int64_t row, float gate, float up) {
        if (r < m && row + 1 < n) cpart[static_cast<int64_t>(r) * (n >> 1) + (row >> 1)] = __fmul_rn(gelu_tanh_dev(gate), up);
    };
    float acc[NT][2];
#pragma unroll
    for (int nt = 0; nt < NT; ++nt) acc[nt][0] = acc[nt][1] = 0.f;
    const uint32_t first_tile = us / nsp;
    uint32_t tl = first_tile;                                  // current unit: tile tb + tl,
    int sg = static_cast<int>(us) - static_cast<int>(tl) * nsp;  // segment sg of the part
    int pu = 0;  // units of the current tile piece
    bool ok = true;
    int slot = 0;
    uint32_t ph = 0;
    uint32_t u = us;
#pragma unroll 1
    for (; u < ue; ++u) {
        const bool landed = mbar_wait_timed(&full[slot], ph);
        if (__any_sync(0xffffffffu, !landed)) {
            ok = false;
            break;
        }
        const uint8_t* ub = ring + static_cast<size_t>(slot) * kQ4KUnit;
        rows_unit<NT>(ub, S.planes + static_cast<size_t>(sg) * NT * kRTilePlane + lane * 16,
                      S.splanes + sg * NT * 32 + lane, S.useg + sg * 4 * NT * 2, g, t, ldsm_off, acc);
        ++pu;
        // Release the slot to this warp's next unit: every lane's reads of it
        // completed into registers the MMAs already consumed.
        __syncwarp();
        if (lane == 0 && iu < ue) issue(slot);
        if (++slot == nb) {
            slot = 0;
            ph ^= 1u;
        }
        if (sg == nsp - 1 || u + 1 == ue) {
            const int64_t row0 = static_cast<int64_t>(tb + tl) * kTile + g;
            if (pu == nsp) {
#pragma unroll
                for (int nt = 0; nt < NT; ++nt) {
                    const float v0 = acc[nt][0] * as[nt], v1 = acc[nt][1] * as[nt];
                    if constexpr (gelu) {  // the up row of a pair sits in lane + 4 (g + 1)
                        const float u0 = __shfl_down_sync(0xffffffffu, v0, 4), u1 = __shfl_down_sync(0xffffffffu, v1, 4);
                        if (!(g & 1)) {
                            store_h(4 * nt + t, row0, v0, u0);
                            store_h(4 * nt + t, row0 + 8, v1, u1);
                        }
                    } else {
                        store(4 * nt + t, row0, v0);
                        store(4 * nt + t, row0 + 8, v1);
                    }
                }
            } else {
                float* pc = S.pieces + (warp * 2 + (tl == first_tile ? 0 : 1)) * 4 * NT * kTile;
#pragma unroll
                for (int nt = 0; nt < NT; ++nt) {
                    pc[(4 * nt + t) * kTile + g] = acc[nt][0];
                    pc[(4 * nt + t) * kTile + g + 8] = acc[nt][1];
                }
            }
#pragma unroll
            for (int nt = 0; nt < NT; ++nt) acc[nt][0] = acc[nt][1] = 0.f;
            pu = 0;
        }
        if (++sg == nsp) {
            sg = 0;
            ++tl;
        }
    }
    if (!ok && lane == 0) {
        // Bounded wait for this warp's copies in flight (issued, not consumed):
        // the k-th sits in slot (slot + k) % nb, one phase later when it
        // wrapped around the ring.
        S.flags[0] = 1;
        const uint32_t inflight = iu - u;
        for (uint32_t k = 0; k < inflight; ++k) {
            const uint32_t sk = static_cast<uint32_t>(slot) + k;
            (void)mbar_wait(&full[sk % static_cast<uint32_t>(nb)], (ph ^ ((sk / static_cast<uint32_t>(nb)) & 1u)) & 1u);
        }
    }
    __syncthreads();
    if (tid == 0 && S.flags[0] && a.err) atomicExch(a.err, kErrMbarTimeout);
    if (un == 0) return;
    // ---- the shared tiles: pieces added in warp order ----
    auto wstart = [&](uint32_t w) { return un * w / kRW; };
    auto owner = [&](uint32_t uu) {  // warp whose share holds unit uu
        const uint32_t w = (kRW * (uu + 1) + un - 1) / un - 1;
        return w < static_cast<uint32_t>(kRW) ? w : static_cast<uint32_t>(kRW) - 1;
    };
#pragma unroll 1
    for (uint32_t T = tb + warp; T < te; T += kRW) {
        const uint32_t a0 = (T - tb) * nsp, a1 = a0 + nsp - 1;
        const uint32_t wa = owner(a0), wb = owner(a1);
        if (wa == wb) continue;  // one warp had the whole tile: already stored
        auto piece_sum = [&](int r, int row) {
            float v = 0.f;
            for (uint32_t w = wa; w <= wb; ++w) {
                const uint32_t s0 = wstart(w);
                if (wstart(w + 1) <= s0) continue;  // a warp without units
                v += S.pieces[((w * 2 + (s0 < a0 ? 1 : 0)) * 4 * NT + r) * kTile + row];
            }
            return v * (a.ascale && !a.a32 ? a.ascale[r] : 1.f);
        };
        const int per = gelu ? 2 : 1;  // rows per output
#pragma unroll 1
        for (int idx = lane; idx < 4 * NT * kTile / per; idx += 32) {
            const int r = idx / (kTile / per), row = (idx - r * (kTile / per)) * per;
            if (r >= m) continue;
            if constexpr (gelu) store_h(r, static_cast<int64_t>(T) * kTile + row, piece_sum(r, row), piece_sum(r, row + 1));
            else store(r, static_cast<int64_t>(T) * kTile + row, piece_sum(r, row));
        }
    }
}

}  // namespace

bool gemm_rows_plan(int64_t m, int64_t n, int k, int num_sms, int max_parts, int force_parts, GemmPlan* p) {
    if (m < 1 || m > kRowsMaxM || n < 1 || k < 256 || k % 256 != 0 || num_sms < 1) return false;
    const int nt = m <= 4 ? 1 : m <= 8 ? 2 : 4;
    const int nseg = k / 256;
    const int64_t ntiles = (n + kTile - 1) / kTile;
    if (ntiles >= (int64_t{1} << 26)) return false;
    int spp_max = 0;
    while (spp_max < nseg && rows_carve(nullptr, nt, spp_max + 1, kRNbMin, nullptr) + 128 <= kRSmemMax) ++spp_max;
    if (spp_max == 0) return false;
    // Parts: as few as the planes allow, more while they balance the CTAs'
    // whole tiles better.  Estimated cost in units per CTA: its units, the
    // planes it builds, and the partial products of several parts (written,
    // then read again by their consumer) as units of streamed bytes.
    double best = 1e300;
    int best_parts = 0, best_spp = 0, best_cpp = 0;
    const double uc = 1.0 + 0.5 * (nt - 1);  // a unit's arithmetic grows with the n8 tiles
    const int min_parts = (nseg + spp_max - 1) / spp_max;
    int lo = min_parts, hi = std::min(nseg, max_parts);
    if (force_parts > 0) lo = hi = std::max(min_parts, std::min(force_parts, nseg));
    for (int parts = lo; parts <= hi; ++parts) {
        const int spp = (nseg + parts - 1) / parts;
        const int real_parts = (nseg + spp - 1) / spp;
        const int cpp = num_sms / real_parts;
        if (cpp < 1) break;
        const int64_t tiles_per_cta = (ntiles + cpp - 1) / cpp;
        // (an extra part also costs the pass that adds the parts: about 3 us,
        // some 40 units' time, measured on the 27B and 4B projections)
        const double cost = spp * (static_cast<double>(tiles_per_cta) * uc + 1.2 * nt) +
                            (real_parts > 1 ? 40.0 + 8.0 * m * n * real_parts / kQ4KUnit / num_sms : 0.0);
        if (cost < best * 0.98) {
            best = cost;
            best_parts = real_parts;
            best_spp = spp;
            best_cpp = cpp;
        }
    }
    if (best_parts == 0) return false;
    p->rows_nt = nt;
    p->splits = best_parts;
    p->kps = best_spp * 256;
    p->rows_cpp = best_cpp;
    p->bm = kTile;
    p->bn = kTile;  // the W tensor map's box: 16 rows x one 144-byte block
    p->arows = kTile;
    p->wbf16 = false;
    p->grid = dim3(static_cast<unsigned>(best_parts * best_cpp));
    // the deepest ring that fits beside the part's planes
    int nb = kRNbMin;
    while (nb < kRNbMax && rows_carve(nullptr, nt, best_spp, nb + 1, nullptr) + 128 <= kRSmemMax) ++nb;
    p->rows_nb = nb;
    p->smem = rows_carve(nullptr, nt, best_spp, nb, nullptr) + 128;
    return true;
}

cudaError_t gemm_rows_prepare() {
    cudaError_t e = cudaSuccess;
    auto set = [&](auto kernel) {
        if (e == cudaSuccess) e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, kRSmemMax);
    };
    set(gemm_rows_q4k_kernel<1, kRowsEpiPlain>);
    set(gemm_rows_q4k_kernel<2, kRowsEpiPlain>);
    set(gemm_rows_q4k_kernel<4, kRowsEpiPlain>);
    set(gemm_rows_q4k_kernel<1, kRowsEpiGelu>);
    set(gemm_rows_q4k_kernel<2, kRowsEpiGelu>);
    set(gemm_rows_q4k_kernel<4, kRowsEpiGelu>);
    return e;
}

cudaError_t gemm_rows_launch(const CUtensorMap& tm_w, const uint16_t* a, const float* ascale, float* c, int64_t m,
                             int64_t n, int k, const GemmPlan& p, int* err, cudaStream_t s, const float* a32, int epi) {
    const uintptr_t src = a32 ? reinterpret_cast<uintptr_t>(a32) : reinterpret_cast<uintptr_t>(a);
    if (!src || p.rows_nt == 0 || m < 1 || m > kRowsMaxM || (src & 15)) return cudaErrorInvalidValue;
    if (epi == kRowsEpiGelu && (p.splits != 1 || (n & 1))) return cudaErrorInvalidValue;
    RowsArgs ra;
    ra.a = a;
    ra.a32 = a32;
    ra.ascale = ascale;
    ra.c = c;
    ra.err = err;
    ra.n = n;
    ra.m = static_cast<int>(m);
    ra.k = k;
    ra.nseg = k / 256;
    ra.spp = p.kps / 256;
    ra.parts = p.splits;
    ra.cpp = p.rows_cpp;
    ra.nb = p.rows_nb;
    const dim3 block(kRW * 32);
#define RT_ROWS_LAUNCH(NTT, EP) gemm_rows_q4k_kernel<NTT, EP><<<p.grid, block, p.smem, s>>>(ra, tm_w)
    const bool g = epi == kRowsEpiGelu;
    if (p.rows_nt == 1) g ? RT_ROWS_LAUNCH(1, kRowsEpiGelu) : RT_ROWS_LAUNCH(1, kRowsEpiPlain);
    else if (p.rows_nt == 2) g ? RT_ROWS_LAUNCH(2, kRowsEpiGelu) : RT_ROWS_LAUNCH(2, kRowsEpiPlain);
    else if (p.rows_nt == 4) g ? RT_ROWS_LAUNCH(4, kRowsEpiGelu) : RT_ROWS_LAUNCH(4, kRowsEpiPlain);
    else return cudaErrorInvalidValue;
#undef RT_ROWS_LAUNCH
    return cudaGetLastError();
}

}  // namespace rt
