// gemv_core.cuh -- device side of the weight-streaming GEMV, shared by the
// standalone GEMV kernel (gemv.cu) and the persistent decode-step kernel
// (step.cu).
//
// Work split.  A matrix is cut into units of 16 rows x one column segment
// (256 Q4_K columns = one 144-byte block per row, or 128 BF16 columns).  Units
// are numbered tile-major (a tile is 16 rows) and every warp of the grid takes
// one contiguous, equal share of that sequence, so all warps stream the same
// number of bytes whatever the shape.  A warp copies its units HBM -> shared
// memory itself: lane 0 issues one 2-D TMA tensor copy per unit (8-byte
// elements, box = unit width x 16 rows, one destination CTA) into a private ring of
// `nb` buffers, each completed on its own mbarrier (bounded waits).  A warp's
// stream runs through a list of GEMVs ("jobs") back to back: the copies of the
// next job's first units are issued as soon as ring slots free up, before that
// job's input vector exists.  No warp ever waits for another warp inside a
// job's stream.
//
// Row sums.  A warp accumulates the units of one tile in registers.  A tile it
// covers whole goes straight to the epilogue; a tile shared with neighbouring
// warps (at most two per warp) leaves a 16-row partial in global scratch, and
// the warp that brings the tile's unit count to a full row (an atomic counter
// per split tile) adds the partials in warp order -- a fixed order, so results
// are deterministic -- and runs the epilogue (store, GELU gate, greedy argmax).
//
// Q4_K (block layout src/autograd2.rs:1003-1042; Q4KMat::dot_row
// src/autograd2.rs:1637-1702).  Per 32-column sub-block j of a row,
//     dot_j = d * sc_j * sum(q * x) - dmin * m_j * sum(x).
// ldmatrix hands each lane the A fragment of one 32-byte quant chunk c for 16
// rows; a byte mask keeps the low nibbles (sub-block 2c) or the high nibbles
// (sub-block 2c+1, as 16 q) as the u8 A operand of mma.m16n8k32.u8.s8.  x is
// split once per job, per 256-column segment, into three int8 planes
// x = s * (p0 + p1/254 + p2/254^2) (|error| <= s/129032, s = max|x|/127 over
// the segment), the s8 B operand.  One MMA per sub-block: its planes sit in
// B columns 4 (j&1) + 0..2, zero elsewhere (lanes feeding the other parity
// read a zero line instead of masking), and the two MMAs of a chunk share an
// accumulator, so eight MMAs cover a 16-row unit.  Two shuffles per chunk
// pair up each row's three plane sums; with one x scale per segment, every
// lane weights them by its row's 6-bit sub-block scales in integer
// arithmetic and converts once per unit.  (Two planes would halve the B
// columns but leave errors near 3e-5 of rms(y): the dot product of K terms
// accumulates the 16-bit rounding of x.)
//
// BF16 (MatBf16::dot_row, src/autograd2.rs:861-888).  The weights, loaded by
// ldmatrix, are the A operand of mma.m16n8k16.bf16; x is split exactly into
// three bf16 planes x = hi + mid + lo (B columns 0..2), so the f32 sum of the
// three product columns is the f32 dot product.  The unit box is 272 bytes wide
// (128 columns + 16 bytes of the next unit), which puts consecutive rows 16
// bytes apart modulo 128 and keeps ldmatrix free of bank conflicts.
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

#include "common.cuh"
#include "gemv.cuh"


namespace rt {
namespace gcore {

constexpr int kTile = 16;
constexpr int kMaxWarps = 16;
constexpr int kQ4KSegCols = 256;
constexpr int kBF16SegCols = 128;
constexpr int kQ4KPitch = 144;   // one Q4_K block per row of a unit
constexpr int kBF16Pitch = 272;  // 128 BF16 columns + 16 bytes
constexpr int kQ4KUnit = kTile * kQ4KPitch;
constexpr int kBF16Unit = kTile * kBF16Pitch;

__host__ __device__ constexpr int seg_cols(int kind) { return kind == kQ4K ? kQ4KSegCols : kBF16SegCols; }
__host__ __device__ constexpr int unit_bytes(int kind) { return kind == kQ4K ? kQ4KUnit : kBF16Unit; }
__host__ __device__ constexpr int box_x(int kind) { return kind == kQ4K ? kQ4KPitch / 8 : kBF16Pitch / 8; }
// TMA x coordinate advance per segment (8-byte elements).
__host__ __device__ constexpr int box_step(int kind) { return kind == kQ4K ? kQ4KPitch / 8 : kBF16SegCols * 2 / 8; }

// Shared-memory plane layout.
//  Q4_K: plane p (0..2) at p * pstride bytes; per 256-column segment 256 bytes.
//  For the four sub-blocks j = 2 jj + par of one parity, lane t of the lane
//  group feeding B column 4 par + p needs, per sub-block, the B fragment (b0,
//  b1) = (elements 4t..4t+3, elements 16+4t..19+4t) of plane p: byte
//      seg*256 + (jj >> 1)*128 + (par*4 + t)*16 + (jj & 1)*8 + (e >= 16)*4 + (e & 3)
//  holds element e of sub-block j, t = (e & 15) >> 2, so that lane fetches
//  its fragments for all four sub-blocks in two 16-byte loads, and the 24
//  lanes that feed B read whole 128-byte lines per plane.  Per
//  segment and parity the four {unit, sum} of xsx sit together (xsx index
//  (seg*2 + par)*4 + jj), so a lane fetches its four in two 16-byte loads.
//  BF16: plane p (hi, mid, lo) at p * pstride bytes, u16 elements; per 16
//  columns, lane t's B fragment (columns 2t, 2t+1, 8+2t, 9+2t) is 8 bytes at 8t.
__host__ __device__ inline int q4k_pstride(int Kp) { return Kp + 64; }       // = 64 mod 128: no bank conflicts
__host__ __device__ inline int bf16_pstride(int Kp) { return Kp * 2 + 32; }  // = 32 mod 128
__host__ __device__ inline size_t planes_bytes(int kind, int Kp) {
    return kind == kQ4K ? 3 * static_cast<size_t>(q4k_pstride(Kp)) : 3 * static_cast<size_t>(bf16_pstride(Kp));
}
// Q4_K: per 256-column segment 12 floats (48 bytes): the sums of x over the
// segment's eight sub-blocks, those of parity 0 first ([parity][jj], sub-block
// 2 jj + parity), then the segment's plane unit s / 64516 and three unused;
// after the last segment a zero line (kQ4KZeroBytes) that lanes read in place
// of B fragments they must not feed.
constexpr int kQ4KXsxFloats = 12;
constexpr int kQ4KZeroBytes = 144;
__host__ __device__ inline size_t xsx_bytes(int kind, int Kp) {
    return kind == kQ4K ? static_cast<size_t>(Kp / 256) * kQ4KXsxFloats * 4 + kQ4KZeroBytes + 16 : 0;
}

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
__device__ __forceinline__ uint2 lds64(const void* p) { return *reinterpret_cast<const uint2*>(p); }

__device__ __forceinline__ void mma_u8s8(int (&c)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3, uint32_t b0,
                                         uint32_t b1) {
    asm("mma.sync.aligned.m16n8k32.row.col.s32.u8.s8.s32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};"
        : "+r"(c[0]), "+r"(c[1]), "+r"(c[2]), "+r"(c[3])
        : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

// The same with a zero accumulator: d = A . B (no register to clear first).
__device__ __forceinline__ void mma_u8s8_z(int (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3, uint32_t b0,
                                           uint32_t b1) {
    asm("mma.sync.aligned.m16n8k32.row.col.s32.u8.s8.s32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%10,%10,%10,%10};"
        : "=r"(d[0]), "=r"(d[1]), "=r"(d[2]), "=r"(d[3])
        : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1), "r"(0));
}

__device__ __forceinline__ void mma_bf16(float (&c)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                                         uint32_t b0, uint32_t b1) {
    asm("mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};"
        : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
        : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

// round(y) for |y| <= 127.5, as a float; *bits gets the integer in its low
// byte (two's complement), from the same magic-number sum.  The quantiser
// below only passes values within that range (|x / s| <= 127 up to a few
// ulps, and each residual is at most half a step of the plane above), so no
// clamp is needed.
__device__ __forceinline__ float round_clamp127(float y, uint32_t* bits) {
    const float t = __fadd_rn(y, 12582912.0f);
    *bits = __float_as_uint(t);
    return __fsub_rn(t, 12582912.0f);
}

// Bytes 0 of a, b, c, d -> one word (a lowest).
__device__ __forceinline__ uint32_t pack4_low(uint32_t a, uint32_t b, uint32_t c, uint32_t d) {
    return __byte_perm(__byte_perm(a, b, 0x0040), __byte_perm(c, d, 0x0040), 0x5410);
}

// f32 -> bf16 bits, round to nearest even (finite inputs).
__device__ __forceinline__ uint32_t bf16_rne(float x) {
    const uint32_t u = __float_as_uint(x);
    return (u + 0x7FFFu + ((u >> 16) & 1u)) >> 16;
}

__device__ __forceinline__ float ldcg_f32(const float* p) {
    float v;
    asm volatile("ld.global.cg.f32 %0, [%1];" : "=f"(v) : "l"(p) : "memory");
    return v;
}

// Q4_K planes of one 256-column segment: lane l of the calling warp holds
// elements 8l..8l+7 of it (zeros past K).  Writes the three planes, the
// sub-block sums and the segment's plane unit (xsx layout above).
__device__ __forceinline__ void q4k_segment_planes(const float (&xv)[8], int seg, int lane, int pstride,
                                                   uint8_t* planes, float2* xsx2) {
    float m = 0.f, sum = 0.f;
#pragma unroll
    for (int e = 0; e < 8; ++e) {
        m = fmaxf(m, fabsf(xv[e]));
        sum += xv[e];
    }
    // a sub-block is 4 lanes; the scale covers the whole segment
    sum += __shfl_xor_sync(0xffffffffu, sum, 1);
    sum += __shfl_xor_sync(0xffffffffu, sum, 2);
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
    // x = s (p0 + p1/254 + p2/254^2) with one s = max|x| / 127 per segment:
    // each residual spans the full int8 range, |error| <= s / (2 * 254^2).
    // Each residual is taken against the stored scale s, so the reciprocal
    // only has to be close (|x inv| stays below 127.5).  A segment whose
    // largest magnitude is below 1e-30 quantises to zero.  One scale per
    // segment (not per sub-block) lets the dot products apply the weights'
    // 6-bit sub-block scales in integer arithmetic (q4k_unit_value).
    const float s = m * (1.0f / 127.0f);
    const float inv = m > 1e-30f ? __fdividef(127.0f, m) : 0.f;
    const float s254 = s * (1.0f / 254.0f);
    const float inv254 = inv * 254.0f, inv254sq = inv * 64516.0f;
    uint32_t b0[8], b1[8], b2[8];  // low byte: the plane value (two's complement)
#pragma unroll
    for (int e = 0; e < 8; ++e) {
        const float f0 = round_clamp127(xv[e] * inv, &b0[e]);
        const float r1 = fmaf(-f0, s, xv[e]);
        const float f1 = round_clamp127(r1 * inv254, &b1[e]);
        const float r2 = fmaf(-f1, s254, r1);
        (void)round_clamp127(r2 * inv254sq, &b2[e]);
    }
    const int j = lane >> 2;  // sub-block of this lane's elements (8(lane&3)..8(lane&3)+7 of it)
    const int par = j & 1, jj = j >> 1, q = lane & 3;
    const int t0 = 2 * (q & 1), hi = q >> 1;  // elements 8q..8q+3: t = t0; 8q+4..8q+7: t = t0 + 1
    const int o0 = seg * 256 + (jj >> 1) * 128 + (par * 4 + t0) * 16 + (jj & 1) * 8 + hi * 4;
    const int o1 = o0 + 16;
    uint8_t* P0 = planes;
    uint8_t* P1 = planes + pstride;
    uint8_t* P2 = planes + 2 * pstride;
    *reinterpret_cast<uint32_t*>(P0 + o0) = pack4_low(b0[0], b0[1], b0[2], b0[3]);
    *reinterpret_cast<uint32_t*>(P0 + o1) = pack4_low(b0[4], b0[5], b0[6], b0[7]);
    *reinterpret_cast<uint32_t*>(P1 + o0) = pack4_low(b1[0], b1[1], b1[2], b1[3]);
    *reinterpret_cast<uint32_t*>(P1 + o1) = pack4_low(b1[4], b1[5], b1[6], b1[7]);
    *reinterpret_cast<uint32_t*>(P2 + o0) = pack4_low(b2[0], b2[1], b2[2], b2[3]);
    *reinterpret_cast<uint32_t*>(P2 + o1) = pack4_low(b2[4], b2[5], b2[6], b2[7]);
    float* xf = reinterpret_cast<float*>(xsx2) + seg * kQ4KXsxFloats;
    if (q == 0) xf[par * 4 + jj] = sum;
    if (lane == 0) xf[8] = s * (1.0f / 64516.0f);
}

// Threads 0..8 of the block: clear the zero line after the xsx of Kp columns.
__device__ __forceinline__ void q4k_zero_line(float2* xsx2, int Kp) {
    if (threadIdx.x < kQ4KZeroBytes / 16) {
        uint8_t* z = reinterpret_cast<uint8_t*>(xsx2) + static_cast<size_t>(Kp / 256) * kQ4KXsxFloats * 4;
        reinterpret_cast<uint4*>(z)[threadIdx.x] = make_uint4(0u, 0u, 0u, 0u);
    }
}

// BF16 planes of 8 consecutive columns 8q..8q+7 (zeros past K).
__device__ __forceinline__ void bf16_chunk_planes(const float (&xv)[8], int q, int pstride, uint8_t* planes) {
    uint32_t h[8], md[8], lo[8];
#pragma unroll
    for (int e = 0; e < 8; ++e) {
        h[e] = bf16_rne(xv[e]);
        const float r = xv[e] - __uint_as_float(h[e] << 16);
        md[e] = bf16_rne(r);
        lo[e] = bf16_rne(r - __uint_as_float(md[e] << 16));
    }
    // 16-column block b = q >> 1, half hf = q & 1: element 8hf + i sits at slot
    // 4(i >> 1) + 2hf + (i & 1), i.e. pair i>>1 is 32-bit word 2(i>>1) + hf.
    const int b = q >> 1, hf = q & 1;
    uint32_t* P0 = reinterpret_cast<uint32_t*>(planes) + b * 8 + hf;
    uint32_t* P1 = reinterpret_cast<uint32_t*>(planes + pstride) + b * 8 + hf;
    uint32_t* P2 = reinterpret_cast<uint32_t*>(planes + 2 * pstride) + b * 8 + hf;
#pragma unroll
    for (int k = 0; k < 4; ++k) {
        P0[2 * k] = h[2 * k] | (h[2 * k + 1] << 16);
        P1[2 * k] = md[2 * k] | (md[2 * k + 1] << 16);
        P2[2 * k] = lo[2 * k] | (lo[2 * k + 1] << 16);
    }
}

// The unit split: warp w (grid-wide index) owns units [start(w), start(w+1))
// with start(w) = floor(U * w / NW); U < 2^31 and NW < 2^16 keep all of it in
// 32-bit arithmetic.
struct Split {
    uint32_t U;
    uint32_t q;  // U / NW
    uint32_t r;  // U % NW
    uint32_t NW;
    float w_per_u;  // NW / U
    __device__ __forceinline__ void init(uint32_t units, uint32_t nwarps) {
        U = units;
        NW = nwarps;
        q = U / NW;
        r = U - q * NW;
        w_per_u = static_cast<float>(NW) / static_cast<float>(U);
    }
    __device__ __forceinline__ uint32_t start(uint32_t w) const { return q * w + (r * w) / NW; }
    // The warp whose range holds unit u (a float estimate, then exact steps).
    __device__ __forceinline__ uint32_t owner(uint32_t u) const {
        uint32_t w = min(NW - 1, static_cast<uint32_t>(static_cast<float>(u) * w_per_u));
        while (w + 1 < NW && start(w + 1) <= u) ++w;
        while (w > 0 && start(w) > u) --w;
        return w;
    }
};

// Q4_K units per copy when W is stored tile-major (see Job::wt).
constexpr int kTileMajorUnitsPerCopy = 2;

// Partial vectors a residual-update prologue can add (Job::src_parts).
constexpr int kMaxSrcParts = 4;

// Greedy sampling (sample_token at temperature 0, src/transformer4.rs:3036-3091):
// the token is the LAST index of the largest softmax probability
// p_i = expf(y_i - M) / S, M = max y, S = sum_i expf(y_i - M).  exp(y_i - M) is
// at most 1, reached by the maximum itself, so only rows whose exp rounds to
// within one quotient ulp of 1 can share its probability: exp(y_i - M) >=
// 1 - 2^-23, i.e. y_i >= M - 2^-23 (a little more for the rounding of exp).
// Rows within kGreedyTau = 2^-21 of M are therefore the only candidates; for
// them p_i is formed as the reference does (f32 difference, exp rounded to
// f32, one f32 division by S) and the highest candidate row whose p_i equals
// 1/S wins.  Distinct logits tie exactly when exp(y_i - M) rounds to 1 (|y_i -
// M| < 2^-25: logits of magnitude below ~0.25 one ulp apart).  The one value
// in between, exp = 1 - 2^-24, ties or not depending on the last bits of S,
// whose summation order differs from the reference's sequential sum.
constexpr float kGreedyTau = 4.76837158203125e-07f;  // 2^-21

// Running greedy state of one lane, warp or CTA: the largest value m, the sum
// s of exp(y - m) over the rows seen (online rescaling), the row of m (ties to
// the higher row) and the range of rows seen.
struct Greedy {
    float m;
    float s;
    long long i;
    int lo, hi;
    __device__ __forceinline__ void init() {
        m = -INFINITY;
        s = 0.f;
        i = -1;
        lo = 0x7fffffff;
        hi = -1;
    }
    __device__ __forceinline__ void add(float v, long long r) {
        if (v > m) {
            s = s * expf(m - v) + 1.0f;  // exp(-inf) = 0 for the first row
            m = v;
            i = r;
        } else {
            s += expf(v - m);
            if (v == m && r > i) i = r;
        }
        lo = min(lo, static_cast<int>(r));
        hi = max(hi, static_cast<int>(r));
    }
    __device__ __forceinline__ void merge(float om, float os, long long oi, int olo, int ohi) {
        if (oi < 0) return;
        if (i < 0) {
            m = om;
            s = os;
            i = oi;
            lo = olo;
            hi = ohi;
            return;
        }
        const float M = fmaxf(m, om);
        s = s * expf(m - M) + os * expf(om - M);
        if (om > m || (om == m && oi > i)) i = oi;
        m = M;
        lo = min(lo, olo);
        hi = max(hi, ohi);
    }
    // Butterfly over the warp: every lane ends with the warp's state.
    __device__ __forceinline__ void warp_merge() {
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) {
            const float om = __shfl_xor_sync(0xffffffffu, m, o);
            const float os = __shfl_xor_sync(0xffffffffu, s, o);
            const long long oi = __shfl_xor_sync(0xffffffffu, i, o);
            const int olo = __shfl_xor_sync(0xffffffffu, lo, o);
            const int ohi = __shfl_xor_sync(0xffffffffu, hi, o);
            merge(om, os, oi, olo, ohi);
        }
    }
};

// Shared memory of the greedy epilogue's reductions.
struct GreedySmem {
    float m[32];
    float s[32];
    long long i[32];
    int lo[32];
    int hi[32];
    int cand[16];  // CTAs whose maximum is within kGreedyTau of the grid's
    int ncand;
    int best;
};

// p_i == p_max for a candidate row of value v (M the maximum, q = 1/S).
__device__ __forceinline__ bool greedy_ties_max(float v, float M, float S, float q) {
    const float x = __fsub_rn(v, M);
    const float e = static_cast<float>(exp(static_cast<double>(x)));  // exp correctly rounded to f32
    return __fdiv_rn(e, S) == q;
}

// One GEMV as the kernels see it.  16-byte aligned (and so a multiple of 16
// bytes), so that the decode-step kernel can bring a table entry into shared
// memory with one bulk copy.
struct alignas(16) Job {
    const void* tmap;   // CUtensorMap of W (parameter or global memory), row-major W
    const uint8_t* wt;  // Q4_K only, or null: W stored tile-major, unit (t, s) at
                        // ((t * nseg) + s) * 2304 bytes (16 rows x 144 bytes, rows
                        // past the matrix zero), so a warp's share of units is one
                        // contiguous byte range, copied by 1-D bulk copies
    int32_t kind;       // kQ4K / kBF16
    int32_t K;
    int32_t nseg;      // column segments per row
    int32_t pad;
    int64_t rows;
    int32_t tile_split;  // 1: each CTA takes whole tiles, its warps split them (combined by cta_combine)
    // Column split (0 or 1: none; needs `wt`).  With kparts = P the job is P
    // stacked GEMVs over consecutive column ranges of nseg segments each:
    // virtual tile p * ptiles + t covers rows 16t..16t+15 of the matrix over
    // x segments [p * nseg, (p + 1) * nseg), `rows` counts P * 16 * ptiles
    // virtual rows, and y holds P partial vectors [P][16 * ptiles] that the
    // consumer adds (src_parts).
    int32_t kparts;
    int32_t ptiles;
    int32_t src_parts;  // residual-update prologue: src is the sum of this many vectors of K (0 or 1: one;
                        // at most kMaxSrcParts)
    // prologue
    const float* x;
    const float* src;
    const float* resid_in;
    float* resid_out;
    const float* g_post;
    const float* g_pre;
    const uint16_t* embed;
    const int32_t* token;
    float embed_scale;
    float eps;
    // epilogue
    float* y;
    GreedySlot* am_slot;
    uint32_t* am_counter;
    int32_t* token_out;
    int32_t* pos_inout;
    int32_t* token_hist;
    // Tagged-word input and output (decode-step kernel): in_ll holds x, or the
    // src_parts vectors of a residual-update prologue; out_ll receives y.
    const uint64_t* in_ll;
    uint64_t* out_ll;
    int32_t fail_token;   // 1: a failed launch writes token_out = -1 (GemvArgs::fail_token)
    uint32_t wait_iters;  // poll limit of the weight-stream waits (0: default)
};

__device__ __forceinline__ uint32_t job_units(const Job& j) {
    return static_cast<uint32_t>((j.rows + kTile - 1) / kTile) * static_cast<uint32_t>(j.nseg);
}

// A warp's units [s, e) of a job.
struct Share {
    uint32_t s, e;
};

// Whole-grid split (tile_split == 0): every warp of the grid an equal,
// contiguous share of the tile-major unit sequence; tiles may straddle warps
// of different CTAs.  Tile split: CTA c takes whole tiles
// [floor(T c / G), floor(T (c+1) / G)) and its warps share those tiles' units
// equally, so no tile ever straddles CTAs.
__device__ __forceinline__ Share warp_share(const Job& j, uint32_t cta, uint32_t ncta, uint32_t warp, uint32_t nw) {
    const uint32_t nseg = static_cast<uint32_t>(j.nseg);
    const uint32_t ntiles = static_cast<uint32_t>((j.rows + kTile - 1) / kTile);
    if (j.tile_split) {
        Split ct;
        ct.init(ntiles, ncta);
        const uint32_t tb = ct.start(cta), te = ct.start(cta + 1);
        const uint32_t n = (te - tb) * nseg;
        if (n == 0) return Share{0, 0};
        Split wt;
        wt.init(n, nw);
        return Share{tb * nseg + wt.start(warp), tb * nseg + wt.start(warp + 1)};
    }
    Split sp;
    sp.init(ntiles * nseg, ncta * nw);
    const uint32_t gw = cta * nw + warp;
    return Share{sp.start(gw), sp.start(gw + 1)};
}

// Grid-wide scratch of the split tiles.
struct SplitScratch {
    float* part;         // [NW][2][16]
    uint32_t* tile_cnt;  // [tiles of the largest job], zero between jobs
};

// What a stream needs of one job, kept in shared memory by the decode-step
// kernel: the weight pointers, the kind and column segments, and this CTA's
// units [u0, u1) of a tile-split job (the warps share them equally, as
// warp_share does).
struct JobLite {
    const uint8_t* wt;
    const void* tmap;
    uint32_t u0, u1;
    int32_t nseg;
    int32_t kind;
    const float* g_post;  // norm weights of a norm prologue (prefetch_gammas)
    const float* g_pre;
    int32_t K;
    int32_t pad;
};

// This CTA's JobLite of job j (tile-split jobs; called by one thread per job).
__device__ __forceinline__ JobLite job_lite(const Job& j, uint32_t cta, uint32_t ncta) {
    JobLite L;
    L.wt = j.wt;
    L.tmap = j.tmap;
    L.nseg = j.nseg;
    L.kind = j.kind;
    L.g_post = j.g_post;
    L.g_pre = j.g_pre;
    L.K = j.K;
    L.pad = 0;
    Split ct;
    ct.init(static_cast<uint32_t>((j.rows + kTile - 1) / kTile), ncta);
    L.u0 = ct.start(cta) * static_cast<uint32_t>(j.nseg);
    L.u1 = ct.start(cta + 1) * static_cast<uint32_t>(j.nseg);
    return L;
}

// Per-warp weight stream over a list of jobs.  All lanes hold the same
// consumer state; the issue cursor is advanced by lane 0 only.
struct Stream {
    uint64_t* full;      // [nb] slot landed
    uint8_t* ring;       // [nb][slot_bytes]
    int nb;
    int slot_bytes;
    int jb;              // next slot to consume
    uint32_t ph;         // its phase parity
    uint64_t pol;
    const Job* jobs;
    const JobLite* jt;   // shared-memory table of the jobs (tile-split jobs only), or null
    int njobs;
    uint32_t cta, ncta, warp, nw;  // this warp's place in the grid
    // issue cursor
    int ij;              // job being issued (njobs: done)
    uint32_t iu, iend;   // next unit, end of this warp's share of job ij
    uint32_t itile;
    int iseg;
    int islot;           // slot the next copy goes to
    int issued;          // copies issued, all jobs
    int consumed;        // copies consumed, all jobs
    // Job ij's fields the copies need, loaded once by seek() (the Job table is
    // in global memory; reading it per copy would put its latency on the path
    // of every copy).
    const uint8_t* iwt;
    const void* itmap;
    int ikind;
    int inseg;
    // Move the cursor to the next job in which this warp has units.
    __device__ __forceinline__ void seek(int j) {
        if (jt) {
            // From the shared-memory table: no global read, no division.
#pragma unroll 1
            for (ij = j; ij < njobs; ++ij) {
                const JobLite L = jt[ij];
                const uint32_t n = L.u1 - L.u0;
                iu = L.u0 + n * warp / nw;
                iend = L.u0 + n * (warp + 1) / nw;
                if (iu < iend) {
                    inseg = L.nseg;
                    ikind = L.kind;
                    iwt = L.wt;
                    itmap = L.tmap;
                    const uint32_t ns = static_cast<uint32_t>(inseg);
                    itile = iu / ns;
                    iseg = static_cast<int>(iu - itile * ns);
                    return;
                }
            }
            return;
        }
#pragma unroll 1
        for (ij = j; ij < njobs; ++ij) {
            const Job& jo = jobs[ij];
            const Share sh = warp_share(jo, cta, ncta, warp, nw);
            iu = sh.s;
            iend = sh.e;
            if (iu < iend) {
                inseg = jo.nseg;
                ikind = jo.kind;
                iwt = jo.wt;
                itmap = jo.tmap;
                const uint32_t ns = static_cast<uint32_t>(inseg);
                itile = iu / ns;
                iseg = static_cast<int>(iu - itile * ns);
                return;
            }
        }
    }
    // lane 0: issue the next copy (one unit, or up to kTileMajorUnitsPerCopy
    // consecutive units of a tile-major W) into slot `islot`, if any is left.
    __device__ __forceinline__ bool issue() {
        if (ij >= njobs) return false;
        uint64_t* bar = &full[islot];
        uint8_t* dst = ring + static_cast<size_t>(islot) * slot_bytes;
        int k = 1;
        if (iwt) {
            k = min(static_cast<uint32_t>(kTileMajorUnitsPerCopy), iend - iu);
            const uint32_t bytes = static_cast<uint32_t>(k) * kQ4KUnit;
            mbar_arrive_expect_tx(bar, bytes);
            bulk_g2s(dst, iwt + static_cast<size_t>(iu) * kQ4KUnit, bytes, bar, pol);
        } else {
            mbar_arrive_expect_tx(bar, static_cast<uint32_t>(unit_bytes(ikind)));
            tma_2d_g2s(dst, itmap, iseg * box_step(ikind), static_cast<int>(itile * kTile), bar, pol);
        }
        if (++islot == nb) islot = 0;
        ++issued;
        iseg += k;
        while (iseg >= inseg) {
            iseg -= inseg;
            ++itile;
        }
        iu += static_cast<uint32_t>(k);
        if (iu == iend) seek(ij + 1);
        return true;
    }
};

// Set up the stream of warp `warp`; lane 0 initialises its barriers and
// issues the first copies.  The caller makes the barrier init visible
// (__syncthreads or __syncwarp) before any other lane waits on them.
__device__ __forceinline__ void stream_start(Stream& s, uint64_t* full, uint8_t* ring, int nb, int slot_bytes,
                                             const Job* jobs, int njobs, int lane, const JobLite* jt = nullptr) {
    s.jt = jt;
    s.full = full;
    s.ring = ring;
    s.nb = nb;
    s.slot_bytes = slot_bytes;
    s.jb = 0;
    s.ph = 0;
    s.pol = l2_evict_first_policy();
    s.jobs = jobs;
    s.njobs = njobs;
    s.cta = blockIdx.x;
    s.ncta = gridDim.x;
    s.warp = threadIdx.x >> 5;
    s.nw = blockDim.x >> 5;
    s.islot = 0;
    s.issued = 0;
    s.consumed = 0;
    s.seek(0);
    if (lane == 0) {
        for (int j = 0; j < nb; ++j) mbar_init(&full[j], 1);
        fence_mbar_init();
        for (int j = 0; j < nb; ++j)
            if (!s.issue()) break;
    }
}

// lane 0, after a failure: wait (bounded) for this warp's copies in flight.
__device__ __forceinline__ void stream_drain(Stream& s) {
    for (int k = s.consumed; k < s.issued; ++k)
        if (!mbar_wait(&s.full[k % s.nb], static_cast<uint32_t>(k / s.nb) & 1u)) break;
}

// Shared memory a job's prologue and epilogue use.
struct JobSmem {
    uint64_t* pbar;  // norm weights landed
    float* red;      // [32]
    int* flag;       // [4] block-wide flags: 0 = failure, 1 = last-CTA
    GreedySmem* gs;  // greedy epilogue reductions
    float* gpost;    // [K]
    float* gpre;     // [K]
    uint8_t* planes;
    float2* xsx;
    float* wpart;    // [warps][2][16] per-warp pieces of tiles shared within the CTA (cta_combine)
    uint2* wse;      // [warps] each warp's units [s, e) of the current tile-split job
    float* xs;       // [K] residual stream of a norm prologue (null if none)
    float* sub;      // [K] sub-layer output of the residual-update prologue; may share memory with
                     // `planes` (dead before the planes are written)
};

// Thread 0: fetch the norm weights (K floats each) of a norm prologue `pro`
// into gpost / gpre, completing one phase of pbar.
__device__ __forceinline__ void prefetch_gammas(int K, const float* g_post, const float* g_pre, int pro,
                                                const JobSmem& S) {
    if (pro == kProPlain) return;
    const uint32_t kb = static_cast<uint32_t>(K) * 4u;
    mbar_arrive_expect_tx(S.pbar, pro == kProResidNorm ? 2u * kb : kb);
    if (pro == kProResidNorm) bulk_g2s_nohint(S.gpost, g_post, kb, S.pbar);
    bulk_g2s_nohint(S.gpre, g_pre, kb, S.pbar);
}
__device__ __forceinline__ void prefetch_gammas(const Job& j, int pro, const JobSmem& S) {
    prefetch_gammas(j.K, j.g_post, j.g_pre, pro, S);
}

// Eight consecutive floats of x at column c0 (zeros at and past K; K is a
// multiple of 8).
__device__ __forceinline__ void load8(const float* x, int c0, int K, float4& lo, float4& hi) {
    if (c0 + 8 <= K) {
        lo = *reinterpret_cast<const float4*>(x + c0);
        hi = *reinterpret_cast<const float4*>(x + c0 + 4);
    } else {
        lo = hi = make_float4(0.f, 0.f, 0.f, 0.f);
    }
}

// Planes of one 8-column chunk (BF16: chunk q) or of one warp's 256-column
// segment (Q4_K: lane l holds its columns 8l..8l+7).
template <int KIND>
__device__ __forceinline__ void chunk_planes(const float4& lo, const float4& hi, int idx, int lane, int pstride,
                                             const JobSmem& S) {
    const float xv[8] = {lo.x, lo.y, lo.z, lo.w, hi.x, hi.y, hi.z, hi.w};
    if constexpr (KIND == kQ4K) q4k_segment_planes(xv, idx, lane, pstride, S.planes, S.xsx);
    else bf16_chunk_planes(xv, idx, pstride, S.planes);
}

// Planes of x read from global memory.  Q4_K: warp w takes segments w, w + nw,
// ...; BF16: thread t takes chunks t, t + nthr, ...  The next item's loads are
// issued before the current item is quantised, so the load latency is paid
// once, and the quantiser is compiled once.
template <int KIND>
__device__ __forceinline__ void planes_from_global(const float* x, int K, int Kp, int pstride, const JobSmem& S) {
    const int lane = threadIdx.x & 31;
    const int first = KIND == kQ4K ? static_cast<int>(threadIdx.x >> 5) : static_cast<int>(threadIdx.x);
    const int step = KIND == kQ4K ? static_cast<int>(blockDim.x >> 5) : static_cast<int>(blockDim.x);
    const int n = KIND == kQ4K ? Kp / kQ4KSegCols : Kp / 8;
    auto col = [&](int i) { return KIND == kQ4K ? i * kQ4KSegCols + lane * 8 : i * 8; };
    float4 lo, hi;
    if (first < n) load8(x, col(first), K, lo, hi);
#pragma unroll 1
    for (int i = first; i < n; i += step) {
        float4 nlo = make_float4(0.f, 0.f, 0.f, 0.f), nhi = nlo;
        if (i + step < n) load8(x, col(i + step), K, nlo, nhi);
        chunk_planes<KIND>(lo, hi, i, lane, pstride, S);
        lo = nlo;
        hi = nhi;
    }
}

// Planes of the pre-normed x: S.xs holds the residual stream (K floats), and
// x = xs * r * (1 + g_pre) (rms_norm_gemma3, src/autograd2.rs:3477-3496) is
// formed as it is read.
template <int KIND>
__device__ __forceinline__ void planes_from_smem(int K, int Kp, int pstride, float r, const JobSmem& S) {
    const int lane = threadIdx.x & 31;
    const int first = KIND == kQ4K ? static_cast<int>(threadIdx.x >> 5) : static_cast<int>(threadIdx.x);
    const int step = KIND == kQ4K ? static_cast<int>(blockDim.x >> 5) : static_cast<int>(blockDim.x);
    const int n = KIND == kQ4K ? Kp / kQ4KSegCols : Kp / 8;
#pragma unroll 1
    for (int i = first; i < n; i += step) {
        const int c0 = KIND == kQ4K ? i * kQ4KSegCols + lane * 8 : i * 8;
        float4 lo, hi, glo, ghi;
        load8(S.xs, c0, K, lo, hi);
        load8(S.gpre, c0, K, glo, ghi);
        auto nrm = [&](float v, float gm) { return __fmul_rn(__fmul_rn(v, r), __fadd_rn(1.0f, gm)); };
        lo = make_float4(nrm(lo.x, glo.x), nrm(lo.y, glo.y), nrm(lo.z, glo.z), nrm(lo.w, glo.w));
        hi = make_float4(nrm(hi.x, ghi.x), nrm(hi.y, ghi.y), nrm(hi.z, ghi.z), nrm(hi.w, ghi.w));
        chunk_planes<KIND>(lo, hi, i, lane, pstride, S);
    }
}

__device__ __forceinline__ float sumsq4(const float4& v) { return v.x * v.x + v.y * v.y + v.z * v.z + v.w * v.w; }

// Build the planes of x for job j in shared memory (all threads of the CTA).
// Norm prologues wait for gamma phase `pbar_phase` and stage the residual
// stream in S.xs (K floats; the residual-update prologue also stages the
// sub-layer output in S.sub).  Ends with __syncthreads.
template <int KIND, int PRO>
__device__ __forceinline__ void job_prologue(const Job& a, const JobSmem& S, uint32_t pbar_phase) {
    const int tid = threadIdx.x, nthr = blockDim.x;
    const int lane = tid & 31;
    const int K = a.K;
    const int Kp = (K + seg_cols(KIND) - 1) / seg_cols(KIND) * seg_cols(KIND);
    const int pstride = KIND == kQ4K ? q4k_pstride(Kp) : bf16_pstride(Kp);
    if constexpr (PRO == kProPlain) {
        planes_from_global<KIND>(a.x, K, Kp, pstride, S);
    } else {
        const float inv_d = 1.0f / static_cast<float>(K);
        float ss = 0.f;
        if constexpr (PRO == kProResidNorm) {
            // post-norm of the sub-layer output, then the residual add
            // (Gemma3Block::forward_cached, src/transformer4.rs:1954-1964)
            float* sub = S.sub;
#pragma unroll 2
            for (int c = tid * 4; c < K; c += nthr * 4) {
                // the column parts of a split GEMV, added in part order (loads all in flight)
                float4 t4[kMaxSrcParts];
#pragma unroll
                for (int q = 0; q < kMaxSrcParts; ++q)
                    t4[q] = q == 0 || q < a.src_parts ? *reinterpret_cast<const float4*>(a.src + static_cast<size_t>(q) * K + c)
                                                      : make_float4(0.f, 0.f, 0.f, 0.f);
                float4 s4 = t4[0];
#pragma unroll
                for (int q = 1; q < kMaxSrcParts; ++q)
                    if (q < a.src_parts) s4 = make_float4(s4.x + t4[q].x, s4.y + t4[q].y, s4.z + t4[q].z, s4.w + t4[q].w);
                const float4 r4 = *reinterpret_cast<const float4*>(a.resid_in + c);
                *reinterpret_cast<float4*>(sub + c) = s4;
                *reinterpret_cast<float4*>(S.xs + c) = r4;
                ss += sumsq4(s4);
            }
            ss = block_sum(ss, S.red);
            if (!mbar_wait(S.pbar, pbar_phase) && lane == 0) atomicExch(&S.flag[0], 1);
            const float r1 = 1.0f / sqrtf(ss * inv_d + a.eps);
            float ss2 = 0.f;
#pragma unroll 1
            for (int c = tid * 4; c < K; c += nthr * 4) {
                const float4 s4 = *reinterpret_cast<const float4*>(sub + c);
                const float4 r4 = *reinterpret_cast<const float4*>(S.xs + c);
                const float4 g4 = *reinterpret_cast<const float4*>(S.gpost + c);
                auto upd = [&](float rv, float sv, float gv) {
                    return __fadd_rn(rv, __fmul_rn(__fmul_rn(sv, r1), __fadd_rn(1.0f, gv)));
                };
                const float4 nv = make_float4(upd(r4.x, s4.x, g4.x), upd(r4.y, s4.y, g4.y), upd(r4.z, s4.z, g4.z),
                                              upd(r4.w, s4.w, g4.w));
                *reinterpret_cast<float4*>(S.xs + c) = nv;
                if (blockIdx.x == 0) *reinterpret_cast<float4*>(a.resid_out + c) = nv;
                ss2 += sumsq4(nv);
            }
            ss = block_sum(ss2, S.red);
        } else {
            // embedding row * sqrt(hidden) (src/transformer4.rs:2360-2364)
            const uint16_t* er = a.embed + static_cast<int64_t>(*a.token) * K;
#pragma unroll 2
            for (int c = tid * 4; c < K; c += nthr * 4) {
                const uint2 e = *reinterpret_cast<const uint2*>(er + c);
                const float4 v = make_float4(__fmul_rn(bf16_bits_to_f32(e.x & 0xFFFFu), a.embed_scale),
                                             __fmul_rn(bf16_bits_to_f32(e.x >> 16), a.embed_scale),
                                             __fmul_rn(bf16_bits_to_f32(e.y & 0xFFFFu), a.embed_scale),
                                             __fmul_rn(bf16_bits_to_f32(e.y >> 16), a.embed_scale));
                *reinterpret_cast<float4*>(S.xs + c) = v;
                if (blockIdx.x == 0) *reinterpret_cast<float4*>(a.resid_out + c) = v;
                ss += sumsq4(v);
            }
            ss = block_sum(ss, S.red);
            if (!mbar_wait(S.pbar, pbar_phase) && lane == 0) atomicExch(&S.flag[0], 1);
        }
        // pre-norm producing the projection input, applied as the planes are built
        planes_from_smem<KIND>(K, Kp, pstride, 1.0f / sqrtf(ss * inv_d + a.eps), S);
    }
    if constexpr (KIND == kQ4K) q4k_zero_line(S.xsx, Kp);
    __syncthreads();
}

// ---- Prologues over tagged-word inputs (decode-step kernel) ----------------
// The input vector is read straight from the producers' tagged words: a
// thread loads every word it needs at once and re-polls until each carries
// `tag`.  They return false (the same on every thread) if a wait gave up
// (LLPoll: about two seconds, or another CTA raised `abort`), and end with
// __syncthreads.

// Planes of x = a.in_ll[0 .. K) (K a multiple of 8), restricted to the
// column segments [seg_lo, seg_hi) this CTA's units read (a column-split job
// reads only its parts' segments).  Q4_K: warp w takes segments seg_lo + w,
// seg_lo + w + nw, ...; each lane loads its 8 values of every segment of the
// warp (up to kLLSegs at once).
constexpr int kLLSegs = 3;

// The column segments [lo, hi) of x that this CTA's units of job `a` read
// (tile split): all of them, or for a column-split job (kparts > 1) those of
// the parts its virtual tiles belong to.
__device__ __forceinline__ int2 cta_x_segments(const Job& a, const JobLite& L) {
    const int kseg = (a.K + kQ4KSegCols - 1) / kQ4KSegCols;
    if (a.kparts <= 1 || L.u1 <= L.u0) return make_int2(0, kseg);
    const uint32_t nseg = static_cast<uint32_t>(a.nseg), pt = static_cast<uint32_t>(a.ptiles);
    const int p0 = static_cast<int>(L.u0 / nseg / pt), p1 = static_cast<int>((L.u1 - 1) / nseg / pt);
    return make_int2(p0 * a.nseg, (p1 + 1) * a.nseg);
}

template <int KIND>
__device__ __forceinline__ bool ll_prologue_plain(const Job& a, const JobSmem& S, uint32_t tag, const int* abort,
                                                  int2 segs) {
    static_assert(KIND == kQ4K, "the step kernel's plain prologues are Q4_K projections");
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nw = blockDim.x >> 5;
    const int K = a.K;
    const int Kp = (K + kQ4KSegCols - 1) / kQ4KSegCols * kQ4KSegCols;
    const int pstride = q4k_pstride(Kp);
    const int nseg = segs.y;
    bool ok = true;
    const uint64_t* in_ll = a.in_ll;
#pragma unroll 1
    for (int s0 = segs.x + warp; s0 < nseg && ok; s0 += kLLSegs * nw) {
        ulonglong2 w[kLLSegs][4];
        // Words still to (re)load: a poll round reloads only the words that
        // did not carry the tag yet.
        uint32_t need = 0;
#pragma unroll
        for (int b = 0; b < kLLSegs; ++b) {
            const int seg = s0 + b * nw, c0 = seg * kQ4KSegCols + lane * 8;
#pragma unroll
            for (int h = 0; h < 4; ++h) {
                w[b][h] = make_ulonglong2(ll_word(0.f, tag), ll_word(0.f, tag));
                if (seg < nseg && c0 + 2 * h < K) need |= 1u << (b * 4 + h);
            }
        }
        LLPoll pl;
        pl.init(abort);
        for (;;) {
#pragma unroll
            for (int b = 0; b < kLLSegs; ++b) {
                const int c0 = (s0 + b * nw) * kQ4KSegCols + lane * 8;
#pragma unroll
                for (int h = 0; h < 4; ++h)
                    if (need & (1u << (b * 4 + h))) w[b][h] = ll_load2(in_ll + c0 + 2 * h);
            }
#pragma unroll
            for (int b = 0; b < kLLSegs; ++b)
#pragma unroll
                for (int h = 0; h < 4; ++h)
                    if (ll_has(w[b][h].x, tag) && ll_has(w[b][h].y, tag)) need &= ~(1u << (b * 4 + h));
            if (__all_sync(0xffffffffu, need == 0)) break;
            if (!pl.again()) {
                ok = false;
                break;
            }
        }
        if (!ok) break;
#pragma unroll
        for (int b = 0; b < kLLSegs; ++b) {
            const int seg = s0 + b * nw;
            if (seg >= nseg) break;
            const float4 lo = make_float4(ll_val(w[b][0].x), ll_val(w[b][0].y), ll_val(w[b][1].x), ll_val(w[b][1].y));
            const float4 hi = make_float4(ll_val(w[b][2].x), ll_val(w[b][2].y), ll_val(w[b][3].x), ll_val(w[b][3].y));
            chunk_planes<KIND>(lo, hi, seg, lane, pstride, S);
        }
    }
    q4k_zero_line(S.xsx, Kp);
    return !__syncthreads_or(!ok);
}

// The residual-update + RMSNorm prologue with the residual stream kept in
// S.xs between prologues (every CTA computes it identically, so no CTA reads
// it back from global memory): sub = sum of the a.src_parts vectors of K at
// a.in_ll (in part order), xs += rmsnorm(sub) * (1 + g_post), x = rmsnorm(xs) *
// (1 + g_pre) (Gemma3Block::forward_cached, src/transformer4.rs:1954-1964;
// rms_norm_gemma3, src/autograd2.rs:3477-3496).  CTA 0 also stores the new
// residual at a.resid_out when that is set.
constexpr int kLLPairs = 3;  // pairs of elements of the vector per thread and poll (K <= 6 * threads)

template <int KIND>
__device__ __forceinline__ bool ll_prologue_resid_norm(const Job& a, const JobSmem& S, uint32_t pbar_phase,
                                                       uint32_t tag, const int* abort) {
    const int tid = threadIdx.x, nthr = blockDim.x, lane = tid & 31;
    const int K = a.K;
    const int Kp = (K + seg_cols(KIND) - 1) / seg_cols(KIND) * seg_cols(KIND);
    const int pstride = KIND == kQ4K ? q4k_pstride(Kp) : bf16_pstride(Kp);
    const int parts = a.src_parts > 1 ? a.src_parts : 1;
    const float inv_d = 1.0f / static_cast<float>(K);
    float* sub = S.sub;
    bool ok = true;
    float ss = 0.f;
    const int npairs = K / 2;
    const uint64_t* in_ll = a.in_ll;
#pragma unroll 1
    for (int pb = tid; pb < npairs && ok; pb += kLLPairs * nthr) {
        ulonglong2 w[kLLPairs][kMaxSrcParts];
        // Words still to (re)load: a poll round reloads only the words that
        // did not carry the tag yet.
        uint32_t need = 0;
#pragma unroll
        for (int i = 0; i < kLLPairs; ++i) {
            const int c = 2 * (pb + i * nthr);
#pragma unroll
            for (int q = 0; q < kMaxSrcParts; ++q) {
                w[i][q] = make_ulonglong2(ll_word(0.f, tag), ll_word(0.f, tag));
                if (c < K && q < parts) need |= 1u << (i * kMaxSrcParts + q);
            }
        }
        LLPoll pl;
        pl.init(abort);
        for (;;) {
#pragma unroll
            for (int i = 0; i < kLLPairs; ++i) {
                const int c = 2 * (pb + i * nthr);
#pragma unroll
                for (int q = 0; q < kMaxSrcParts; ++q)
                    if (need & (1u << (i * kMaxSrcParts + q)))
                        w[i][q] = ll_load2(in_ll + static_cast<size_t>(q) * K + c);
            }
#pragma unroll
            for (int i = 0; i < kLLPairs; ++i)
#pragma unroll
                for (int q = 0; q < kMaxSrcParts; ++q)
                    if (ll_has(w[i][q].x, tag) && ll_has(w[i][q].y, tag)) need &= ~(1u << (i * kMaxSrcParts + q));
            if (need == 0) break;
            if (!pl.again()) {
                ok = false;
                break;
            }
        }
        if (!ok) break;
#pragma unroll
        for (int i = 0; i < kLLPairs; ++i) {
            const int c = 2 * (pb + i * nthr);
            if (c >= K) break;
            float2 s2 = make_float2(ll_val(w[i][0].x), ll_val(w[i][0].y));
#pragma unroll
            for (int q = 1; q < kMaxSrcParts; ++q)
                if (q < parts) s2 = make_float2(s2.x + ll_val(w[i][q].x), s2.y + ll_val(w[i][q].y));
            *reinterpret_cast<float2*>(sub + c) = s2;
            ss += s2.x * s2.x + s2.y * s2.y;
        }
    }
    if (__syncthreads_or(!ok)) return false;
    ss = block_sum(ss, S.red);
    if (!mbar_wait(S.pbar, pbar_phase) && lane == 0) atomicExch(&S.flag[0], 1);
    const float r1 = 1.0f / sqrtf(ss * inv_d + a.eps);
    float ss2 = 0.f;
#pragma unroll 1
    for (int c = tid * 4; c < K; c += nthr * 4) {
        const float4 s4 = *reinterpret_cast<const float4*>(sub + c);
        const float4 r4 = *reinterpret_cast<const float4*>(S.xs + c);
        const float4 g4 = *reinterpret_cast<const float4*>(S.gpost + c);
        auto upd = [&](float rv, float sv, float gv) {
            return __fadd_rn(rv, __fmul_rn(__fmul_rn(sv, r1), __fadd_rn(1.0f, gv)));
        };
        const float4 nv = make_float4(upd(r4.x, s4.x, g4.x), upd(r4.y, s4.y, g4.y), upd(r4.z, s4.z, g4.z),
                                      upd(r4.w, s4.w, g4.w));
        *reinterpret_cast<float4*>(S.xs + c) = nv;
        if (blockIdx.x == 0 && a.resid_out) *reinterpret_cast<float4*>(a.resid_out + c) = nv;
        ss2 += sumsq4(nv);
    }
    ss2 = block_sum(ss2, S.red);
    planes_from_smem<KIND>(K, Kp, pstride, 1.0f / sqrtf(ss2 * inv_d + a.eps), S);
    if constexpr (KIND == kQ4K) q4k_zero_line(S.xsx, Kp);
    __syncthreads();
    return true;
}

// a - b computed as a multiply-add (on the FMA pipe; the integer ALU pipe is
// the one the unit arithmetic saturates).
__device__ __forceinline__ uint32_t sub_on_fma(uint32_t a, uint32_t b) {
    uint32_t r;
    asm("mad.lo.u32 %0, %1, %2, %3;" : "=r"(r) : "r"(b), "r"(0xFFFFFFFFu), "r"(a));
    return r;
}

// This lane's share of one Q4_K unit (16 rows x one 256-column segment at
// shared-memory address ub): the value of row g + 8 (t & 1) over the four
// sub-blocks of parity t >> 1, scales applied.  blo / bhi: where this lane
// reads its B fragments for the low-nibble and high-nibble MMAs (its plane
// bytes, or the zero line when its columns belong to the other parity);
// useg: the segment's plane unit; xs4: the segment's sums of x over this
// lane's four sub-blocks.
__device__ __forceinline__ float q4k_unit_value(const uint8_t* ub, const uint8_t* blo, const uint8_t* bhi, int g,
                                                int t, float useg, const float4 xs4, int ldsm_off) {
    // One MMA per sub-block j (k = its 32 elements).  B column 4 par + p
    // holds plane p of x's sub-block j when j has parity par (lane group
    // g = 4 par + p feeds it); columns 3 and 7 stay zero.  The MMAs of chunk
    // c (sub-blocks 2c, 2c+1: low and high nibbles of the same 32 bytes) share
    // accumulator c: columns 0..2 the plane sums of 2c, columns 4..6 those of
    // 2c+1 (whose A operand is the high nibble in place, i.e. 16 q).
    const uint4 L0 = lds128(blo), L1 = lds128(blo + 128);
    const uint4 H0 = lds128(bhi), H1 = lds128(bhi + 128);
    const int lpar = t >> 1, odd = t & 1;
    const uint4 hd = lds128(ub + (g + 8 * odd) * kQ4KPitch);
    int acc[4][4];
#pragma unroll
    for (int c = 0; c < 4; ++c) {
        uint32_t a0, a1, a2, a3;
        ldsm_x4(ub + ldsm_off + 32 * c, a0, a1, a2, a3);
        const uint32_t l0 = a0 & 0x0F0F0F0Fu, l1 = a1 & 0x0F0F0F0Fu, l2 = a2 & 0x0F0F0F0Fu, l3 = a3 & 0x0F0F0F0Fu;
        const uint32_t lw0 = c == 0 ? L0.x : c == 1 ? L0.z : c == 2 ? L1.x : L1.z;
        const uint32_t lw1 = c == 0 ? L0.y : c == 1 ? L0.w : c == 2 ? L1.y : L1.w;
        const uint32_t hw0 = c == 0 ? H0.x : c == 1 ? H0.z : c == 2 ? H1.x : H1.z;
        const uint32_t hw1 = c == 0 ? H0.y : c == 1 ? H0.w : c == 2 ? H1.y : H1.w;
        mma_u8s8_z(acc[c], l0, l1, l2, l3, lw0, lw1);
        mma_u8s8(acc[c], sub_on_fma(a0, l0), sub_on_fma(a1, l1), sub_on_fma(a2, l2), sub_on_fma(a3, l3), hw0, hw1);
    }
    // Lane t even holds (p0, p1) of rows g and g+8, its odd neighbour (p2, 0).
    // Two shuffles give the even lane row g's p2 and the odd lane row g+8's
    // p0 and p1; every lane then weights its own and the received sums by
    // the 6-bit sub-block scales of its row in integer arithmetic (exact:
    // at most 4 * 63 * 32 * 240 * 127 < 2^31), and forms
    // T = 64516 P0 + 254 P1 + P2 once per unit.
    const float d = f16_bits_to_f32(hd.x & 0xFFFFu), dmin = f16_bits_to_f32(hd.x >> 16);
    // scale_min (src/autograd2.rs:1075-1085), four 6-bit fields per word
    const uint32_t s_lo = hd.y & 0x3F3F3F3Fu, m_lo = hd.z & 0x3F3F3F3Fu;
    const uint32_t s_hi = (hd.w & 0x0F0F0F0Fu) | ((hd.y >> 2) & 0x30303030u);
    const uint32_t m_hi = ((hd.w >> 4) & 0x0F0F0F0Fu) | ((hd.z >> 2) & 0x30303030u);
    // sub-block 2c + lpar: byte lpar (c even) or 2 + lpar (c odd) of the low
    // (c < 2) or high words; as an integer, or as an exact float
    const uint32_t isel_a = 0x4440u | static_cast<uint32_t>(lpar), isel_b = 0x4440u | static_cast<uint32_t>(2 + lpar);
    const uint32_t fsel_a = 0x7540u | static_cast<uint32_t>(lpar), fsel_b = 0x7540u | static_cast<uint32_t>(2 + lpar);
    int A0 = 0, A1 = 0, A2 = 0, AX = 0, AY = 0;
    float vm = 0.f;
#pragma unroll
    for (int c = 0; c < 4; ++c) {
        const int x = __shfl_xor_sync(0xffffffffu, odd ? acc[c][0] : acc[c][2], 1);
        const int y = __shfl_xor_sync(0xffffffffu, acc[c][3], 1);
        const uint32_t sw = c < 2 ? s_lo : s_hi, mw = c < 2 ? m_lo : m_hi;
        const int sc = static_cast<int>(__byte_perm(sw, 0u, (c & 1) ? isel_b : isel_a));
        A0 += sc * acc[c][0];
        A1 += sc * acc[c][1];
        A2 += sc * acc[c][2];
        AX += sc * x;
        AY += sc * y;
        const float xs = c == 0 ? xs4.x : c == 1 ? xs4.y : c == 2 ? xs4.z : xs4.w;
        vm = fmaf(byte_to_float(mw, (c & 1) ? fsel_b : fsel_a), xs, vm);
    }
    // even lane (row g): T = 64516 A0 + 254 A1 + AX; odd lane (row g+8): T = 64516 AX + 254 AY + A2
    const float wa = odd ? 0.f : 64516.0f, wb = odd ? 0.f : 254.0f, wc = odd ? 1.0f : 0.f;
    const float wx = odd ? 64516.0f : 1.0f, wy = odd ? 254.0f : 0.f;
    const float T = fmaf(static_cast<float>(A0), wa,
                         fmaf(static_cast<float>(A1), wb,
                              fmaf(static_cast<float>(A2), wc, fmaf(static_cast<float>(AX), wx, static_cast<float>(AY) * wy))));
    const float u = lpar ? useg * 0.0625f : useg;  // the high nibbles were seen as 16 q
    return d * (T * u) - dmin * vm;
}

// How the warps' shares of a job are laid out (Job::tile_split matches it).
enum SplitMode : int {
    kSplitGrid = 0,  // whole-grid warp split; shared tiles combined through global scratch
    kSplitTile = 1,  // CTAs own whole tiles; shared tiles combined in shared memory (cta_combine)
};

// Stream this warp's units of job `a` (whose planes are ready) through the
// epilogue.  Returns false if a wait gave up (the warp's stream is then
// abandoned; the caller drains it).  gr: this lane's running greedy state.
// out_tag != 0: rows go to a.out_ll as tagged words with that tag.
template <int KIND, int EPI, int SPLIT>
__device__ __forceinline__ bool job_units_run(const Job& a, Stream& st, const JobSmem& S, const SplitScratch& sc,
                                              Greedy& gr, uint32_t out_tag = 0) {
    const int lane = threadIdx.x & 31;
    const int g = lane >> 2, t = lane & 3;
    // The job's fields, read once: the Job table is in global memory, and every
    // asm statement with a memory clobber below would otherwise make the
    // compiler read them again.
    const int nseg = a.nseg;
    const int64_t rows = a.rows;
    const int kparts = a.kparts, ptiles = a.ptiles;
    const uint32_t wait_iters = a.wait_iters;
    uint64_t* const out_ll = a.out_ll;
    float* const yv = a.y;
    const bool tile_major = a.wt != nullptr;
    const int Kp = (a.K + seg_cols(KIND) - 1) / seg_cols(KIND) * seg_cols(KIND);
    const int pstride = KIND == kQ4K ? q4k_pstride(Kp) : bf16_pstride(Kp);
    const Share sh = warp_share(a, st.cta, st.ncta, st.warp, st.nw);
    const uint32_t u_begin = sh.s;
    const int n = static_cast<int>(sh.e - sh.s);
    if (SPLIT == kSplitTile && lane == 0) S.wse[st.warp] = make_uint2(sh.s, sh.e);

    // Row epilogue: lane L < 16 holds the sum of row r0 + L.
    auto emit_rows = [&](int64_t r0, float v) {
        const int64_t r = r0 + lane;
        if constexpr (EPI == kEpiGeluPair) {
            const float up = __shfl_down_sync(0xffffffffu, v, 1);
            if (lane < kTile && !(lane & 1) && r < rows) {
                const float h = __fmul_rn(gelu_tanh_dev(v), up);
                if (out_tag) ll_store(out_ll + (r >> 1), h, out_tag);
                else yv[r >> 1] = h;
            }
        } else {
            if (lane < kTile && r < rows) {
                if (out_tag) ll_store(out_ll + r, v, out_tag);
                else yv[r] = v;
                if constexpr (EPI == kEpiArgmax) gr.add(v, r);
            }
        }
    };

    // ldmatrix row address of this lane within a unit (matrix l/8: rows 0-7 or
    // 8-15, first or second 16 bytes of the 32-byte k slice)
    const int ldsm_off = KIND == kQ4K
                             ? ((lane & 7) + ((lane >> 3) & 1) * 8) * kQ4KPitch + 16 + ((lane >> 4) & 1) * 16
                             : ((lane & 7) + ((lane >> 3) & 1) * 8) * kBF16Pitch + ((lane >> 4) & 1) * 16;

    // Q4_K: this lane's B fragments (planes at lane_b + 256 xseg, or the zero
    // line) and its sub-block parity's sums of x.
    const int bpar = g >> 2, bpl = g & 3;
    const int lane_b = bpl * pstride + (bpar * 4 + t) * 16;
    const uint8_t* zline = reinterpret_cast<const uint8_t*>(S.xsx) + static_cast<size_t>(Kp / 256) * kQ4KXsxFloats * 4;
    const bool feeds_lo = bpl < 3 && bpar == 0, feeds_hi = bpl < 3 && bpar == 1;
    const float* xsf = reinterpret_cast<const float*>(S.xsx);
    auto unit_at = [&](const uint8_t* ub, int xs) {
        const uint8_t* real = S.planes + lane_b + xs * 256;
        const float* xf = xsf + xs * kQ4KXsxFloats;
        return q4k_unit_value(ub, feeds_lo ? real : zline, feeds_hi ? real : zline, g, t, xf[8],
                              *reinterpret_cast<const float4*>(xf + (t >> 1) * 4), ldsm_off);
    };

    float acc0 = 0.f, acc1 = 0.f;  // this lane's share of rows g and g+8 of the current tile
    uint32_t tile = u_begin / nseg;
    int seg = static_cast<int>(u_begin - tile * nseg);
    const uint32_t first_tile = tile;
    // first segment of x for the current tile (column-split jobs)
    auto part_base = [&](uint32_t tl) { return kparts > 1 ? static_cast<int>(tl / ptiles) * nseg : 0; };
    int xseg = part_base(tile) + seg;
    int pu = 0;  // units of the current tile piece
    const int upc = tile_major ? kTileMajorUnitsPerCopy : 1;
    int in_copy = 0, uic = 0;  // units left in / consumed from the current copy
    float cv0 = 0.f, cv1 = 0.f;  // Q4_K: this lane's values of the current copy's units
    for (int i = 0; i < n; ++i) {
        if (in_copy == 0) {
            const bool ok = mbar_wait_n(&st.full[st.jb], st.ph, wait_iters);
            if (__any_sync(0xffffffffu, !ok)) return false;
            in_copy = min(upc, n - i);
            uic = 0;
        }
        const uint8_t* ub = st.ring + static_cast<size_t>(st.jb) * st.slot_bytes + uic * unit_bytes(KIND);
        if constexpr (KIND == kQ4K) {
            // The units of a copy are computed together (independent chains, so
            // the scheduler can interleave them), then consumed one by one.
            if (uic == 0) {
                cv0 = unit_at(ub, xseg);
                if (in_copy > 1) {
                    const int xs1 = seg + 1 < nseg ? xseg + 1 : part_base(tile + 1);
                    cv1 = unit_at(ub + kQ4KUnit, xs1);
                }
            }
            const float v = uic == 0 ? cv0 : cv1;
            if (t & 1) acc1 += v;
            else acc0 += v;
        } else {
            // BF16: lanes g < 3 feed B column g (plane g); the rest feed zeros.
            const uint8_t* pb = S.planes + (g < 3 ? g : 0) * pstride + xseg * (kBF16SegCols * 2) + t * 8;
            float c[4][4];
#pragma unroll
            for (int k = 0; k < 4; ++k)
#pragma unroll
                for (int e = 0; e < 4; ++e) c[k][e] = 0.f;
#pragma unroll
            for (int s = 0; s < 8; ++s) {
                uint32_t a0, a1, a2, a3;
                ldsm_x4(ub + ldsm_off + 32 * s, a0, a1, a2, a3);
                const uint2 b = g < 3 ? lds64(pb + 32 * s) : make_uint2(0u, 0u);
                mma_bf16(c[s & 3], a0, a1, a2, a3, b.x, b.y);
            }
            acc0 += ((c[0][0] + c[1][0]) + (c[2][0] + c[3][0])) + ((c[0][1] + c[1][1]) + (c[2][1] + c[3][1]));
            acc1 += ((c[0][2] + c[1][2]) + (c[2][2] + c[3][2])) + ((c[0][3] + c[1][3]) + (c[2][3] + c[3][3]));
        }
        ++pu;
        ++uic;
        if (--in_copy == 0) {
            // Release the slot to the next copy of this warp's stream (any job).
            ++st.consumed;
            __syncwarp();
            if (lane == 0) {
                fence_proxy_async_smem();
                st.issue();
            }
            if (++st.jb == st.nb) {
                st.jb = 0;
                st.ph ^= 1u;
            }
        }
        ++xseg;
        const bool tile_end = ++seg == nseg;
        if (tile_end || i == n - 1) {
            // Row sums of this piece: quad reduction, then lane L < 16 takes row L.
            float s0 = acc0 + __shfl_xor_sync(0xffffffffu, acc0, 1);
            s0 += __shfl_xor_sync(0xffffffffu, s0, 2);
            float s1 = acc1 + __shfl_xor_sync(0xffffffffu, acc1, 1);
            s1 += __shfl_xor_sync(0xffffffffu, s1, 2);
            const float ra = __shfl_sync(0xffffffffu, s0, 4 * (lane & 7));
            const float rb = __shfl_sync(0xffffffffu, s1, 4 * (lane & 7));
            const float rowv = (lane & 8) ? rb : ra;
            const int64_t r0 = static_cast<int64_t>(tile) * kTile;
            if (pu == nseg) {
                emit_rows(r0, rowv);
            } else if constexpr (SPLIT == kSplitTile) {
                // Combined later by the CTA (cta_combine), in shared memory.
                const int slot = tile == first_tile ? 0 : 1;
                if (lane < kTile) S.wpart[((threadIdx.x >> 5) * 2 + slot) * kTile + lane] = rowv;
            } else {
                Split sp;  // the whole-grid split (owner lookups)
                sp.init(job_units(a), st.ncta * st.nw);
                const uint32_t gw = st.cta * st.nw + st.warp;
                // Lanes 16..31 (row = lane - 16) publish the piece.
                const int slot = tile == first_tile ? 0 : 1;
                const bool pub = lane >= kTile;
                const float rv = __shfl_sync(0xffffffffu, rowv, lane & (kTile - 1));
                if (pub) {
                    sc.part[(static_cast<int64_t>(gw) * 2 + slot) * kTile + (lane - kTile)] = rv;
                    __threadfence();
                }
                __syncwarp();
                int last = 0;
                if (lane == kTile)
                    last = atomicAdd(&sc.tile_cnt[tile], static_cast<uint32_t>(pu)) + static_cast<uint32_t>(pu) ==
                           static_cast<uint32_t>(nseg);
                last = __shfl_sync(0xffffffffu, last, kTile);
                if (last) {
                    if (pub) __threadfence();
                    const uint32_t u0 = tile * nseg;
                    const uint32_t w_first = sp.owner(u0), w_last = sp.owner(u0 + nseg - 1);
                    // Sum the pieces in warp order, eight loads in flight at a time.
                    float v = 0.f;
                    for (uint32_t wb = w_first; wb <= w_last; wb += 8) {
                        float pv[8];
#pragma unroll
                        for (int k = 0; k < 8; ++k) {
                            const uint32_t w = wb + k;
                            pv[k] = 0.f;
                            if (w <= w_last && pub) {
                                const uint32_t s_w = sp.start(w);
                                // a warp that began in an earlier tile keeps this one in slot 1
                                if (sp.start(w + 1) > s_w)
                                    pv[k] = ldcg_f32(sc.part + (static_cast<int64_t>(w) * 2 + (s_w < u0 ? 1 : 0)) * kTile +
                                                     (lane - kTile));
                            }
                        }
#pragma unroll
                        for (int k = 0; k < 8; ++k) v += pv[k];
                    }
                    emit_rows(r0, __shfl_sync(0xffffffffu, v, (lane & (kTile - 1)) + kTile));
                    if (lane == kTile) sc.tile_cnt[tile] = 0u;
                }
            }
            acc0 = acc1 = 0.f;
            pu = 0;
            if (tile_end) {
                seg = 0;
                ++tile;
                xseg = part_base(tile);
            }
        }
    }
    return true;
}

// After every warp of the CTA ran job_units_run on a job with tile_split set:
// add, in warp order, the pieces of the tiles this CTA's warps shared (one
// warp per tile, from shared memory) and run the epilogue on them.  All
// threads call it; it starts with __syncthreads.  The warps' unit ranges come
// from the table job_units_run filled (no division per piece).
template <int EPI>
__device__ __forceinline__ void cta_combine(const Job& a, const JobSmem& S, Greedy& gr, uint32_t out_tag = 0) {
    __syncthreads();
    const uint32_t nw = blockDim.x >> 5, warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;
    const uint32_t nseg = static_cast<uint32_t>(a.nseg);
    const uint32_t ntiles = static_cast<uint32_t>((a.rows + kTile - 1) / kTile);
    Split ct;
    ct.init(ntiles, gridDim.x);
    const uint32_t tb = ct.start(blockIdx.x), te = ct.start(blockIdx.x + 1);
    // lane -> row (or the first row of a GELU pair)
    constexpr int kPer = EPI == kEpiGeluPair ? kTile / 2 : kTile;
    const int row = EPI == kEpiGeluPair ? 2 * lane : lane;
    for (uint32_t T = tb + warp; T < te; T += nw) {
        const uint32_t u0 = T * nseg, u1 = u0 + nseg;
        float v0 = 0.f, v1 = 0.f;
        int pieces = 0;
        // All warps' table entries and pieces are loaded at once (unrolled,
        // predicated); the sum runs in warp order, adding zero for warps
        // without a piece of this tile.
#pragma unroll
        for (int w = 0; w < kMaxWarps; ++w) {
            const uint2 se = w < static_cast<int>(nw) ? S.wse[w] : make_uint2(0u, 0u);
            const bool in = se.x < se.y && se.x < u1 && se.y > u0;
            pieces += in ? 1 : 0;
            // a warp that began in an earlier tile keeps this one in slot 1
            const float* pw = S.wpart + (w * 2 + (se.x < u0 ? 1 : 0)) * kTile;
            const bool rd = in && lane < kPer;
            v0 += rd ? pw[row] : 0.f;
            if constexpr (EPI == kEpiGeluPair) v1 += rd ? pw[row + 1] : 0.f;
        }
        if (pieces < 2) continue;  // one warp had it all: already through the epilogue
        if (lane >= kPer) continue;
        const int64_t r = static_cast<int64_t>(T) * kTile + row;
        if (r >= a.rows) continue;
        if constexpr (EPI == kEpiGeluPair) {
            const float h = __fmul_rn(gelu_tanh_dev(v0), v1);
            if (out_tag) ll_store(a.out_ll + (r >> 1), h, out_tag);
            else a.y[r >> 1] = h;
        } else {
            if (out_tag) ll_store(a.out_ll + r, v0, out_tag);
            else a.y[r] = v0;
            if constexpr (EPI == kEpiArgmax) gr.add(v0, r);
        }
    }
}

// Greedy token over the grid (sample_token's rule, see kGreedyTau), after
// every warp of every CTA ran job_units_run: per CTA a GreedySlot; the last CTA
// to arrive combines them (M, S in a fixed order), re-reads the rows of the
// CTAs whose maximum is within kGreedyTau of M, writes the token (and advances
// the device-side decode position) and resets the counter.  All threads of
// the CTA call it, also when one of its bounded waits gave up (`failed`): the
// last CTA then writes no token (-1 with Job::fail_token), leaves the decode
// position alone and returns the split-tile counters to zero, so the next
// launch starts clean.
__device__ __forceinline__ void argmax_finish(const Job& a, const JobSmem& S, Greedy gr, bool failed,
                                              uint32_t* tile_cnt) {
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5, nw = blockDim.x >> 5, nthr = blockDim.x;
    GreedySmem& G = *S.gs;
    gr.warp_merge();
    if (lane == 0) {
        G.m[warp] = gr.m;
        G.s[warp] = gr.s;
        G.i[warp] = gr.i;
        G.lo[warp] = gr.lo;
        G.hi[warp] = gr.hi;
    }
    __syncthreads();
    if (tid == 0) {
        Greedy c;
        c.init();
        for (int w = 0; w < nw; ++w) c.merge(G.m[w], G.s[w], G.i[w], G.lo[w], G.hi[w]);
        GreedySlot sl;
        sl.m = c.m;
        sl.s = c.s;
        sl.idx = static_cast<int32_t>(c.i);
        sl.lo = c.lo;
        sl.hi = c.hi;
        sl.failed = failed ? 1 : 0;
        sl.pad[0] = sl.pad[1] = 0;
        a.am_slot[blockIdx.x] = sl;
        __threadfence();
        const uint32_t prev = atomicAdd(a.am_counter, 1u);
        S.flag[1] = prev == gridDim.x - 1;
        G.ncand = 0;
        G.best = -1;
    }
    __syncthreads();
    if (!S.flag[1]) return;
    __threadfence();
    // M, then S = sum_c s_c exp(m_c - M) in a fixed order; the CTAs that may
    // hold candidates.
    const int ncta = static_cast<int>(gridDim.x);
    const volatile GreedySlot* slots = a.am_slot;
    int any_failed = 0;
    for (int k = tid; k < ncta; k += nthr) any_failed |= slots[k].failed;
    if (__syncthreads_or(any_failed)) {
        // Units that never arrived left split tiles half-counted.
        if (tile_cnt) {
            const int64_t ntiles = (a.rows + kTile - 1) / kTile;
            for (int64_t t = tid; t < ntiles; t += nthr) tile_cnt[t] = 0u;
        }
        __syncthreads();
        if (tid == 0) {
            if (a.token_out && a.fail_token) *a.token_out = -1;
            __threadfence();
            *a.am_counter = 0u;
        }
        return;
    }
    float lm = -INFINITY;
    for (int k = tid; k < ncta; k += nthr)
        if (slots[k].idx >= 0) lm = fmaxf(lm, slots[k].m);
    const float M = block_max(lm, S.red);
    float ls = 0.f;
    for (int k = tid; k < ncta; k += nthr) {
        if (slots[k].idx < 0) continue;
        const float mk = slots[k].m;
        ls += slots[k].s * expf(mk - M);
        if (mk >= M - kGreedyTau) {
            const int n = atomicAdd(&G.ncand, 1);
            if (n < 16) G.cand[n] = k;
        }
    }
    const float Ssum = block_sum(ls, S.red);  // ends with every thread past a __syncthreads
    const float q = __fdiv_rn(1.0f, Ssum);
    const float lim = M - kGreedyTau;
    int best = -1;
    const volatile float* y = a.y;
    if (G.ncand <= 16) {
        for (int c = 0; c < G.ncand; ++c) {
            const int k = G.cand[c];
            const int lo = slots[k].lo, hi = slots[k].hi;
            for (int r = lo + tid; r <= hi; r += nthr) {
                const float v = y[r];
                if (v >= lim && r > best && greedy_ties_max(v, M, Ssum, q)) best = r;
            }
        }
    } else {  // many CTAs near the maximum: every row
        for (int r = tid; r < a.rows; r += nthr) {
            const float v = y[r];
            if (v >= lim && r > best && greedy_ties_max(v, M, Ssum, q)) best = r;
        }
    }
    if (best >= 0) atomicMax(&G.best, best);
    __syncthreads();
    if (tid == 0) {
        const int32_t bi = G.best;
        if (a.token_out) *a.token_out = bi;
        if (a.pos_inout) {
            const int32_t p = *a.pos_inout;
            if (a.token_hist) a.token_hist[p] = bi;
            *a.pos_inout = p + 1;
        }
        *a.am_counter = 0u;
    }
}

}  // namespace gcore
}  // namespace rt
