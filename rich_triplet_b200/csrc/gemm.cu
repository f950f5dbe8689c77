// gemm.cu -- Q4_K prefill GEMM on the tcgen05 tensor cores.
//
// C[M, N] = diag(ascale) . A[M, K] . dequant(W[N, K])^T, A fp16 with a
// power-of-two scale per row, W Q4_K (or bf16), f32 accumulate
// (Q4KMat::matmul_q4k_t, src/autograd2.rs:1437-1457).
//
// One CTA computes a 128 x 128 or 256 x 256 tile of C (one or two M128
// accumulators in tensor memory); K advances in blocks of 64 columns (one
// 128-byte swizzle row of bf16).  Warp roles:
//   warp 0, lane 0   TMA producer: the A tile of each K-block (2-D tensor
//                    copy, 128-byte swizzle) and, once per Q4_K super-block
//                    (four K-blocks), the 128 raw 144-byte blocks of W
//   warp 1, lane 0   MMA issuer: four tcgen05.mma (M128 N128/256 K16, fp16
//                    in, f32 accumulator in tensor memory) per K-block and
//                    accumulator, then a tcgen05.commit that frees the stage
//   warps 2..17      dequantisers, two groups of 8 taking alternate K-blocks
//                    (two K-blocks in flight): w = q * (d*sc) - dmin*m (the Q4_K block
//                    format, src/autograd2.rs:1003-1085) in fp16, stored in
//                    the swizzled K-major layout the MMA reads (bf16 W tiles
//                    are converted to fp16 in place instead); then they move
//                    the accumulators tensor memory -> registers -> C, times
//                    the row's scale
// Every mbarrier wait gives up after a second; a CTA that gives up records kErrMbarTimeout,
// waits (bounded) for its own copies and MMAs in flight, frees its tensor
// memory and returns.
//
// Precision: the MMA takes both operands in one 16-bit type.  fp16 keeps 11
// significant bits (bf16: 8), so each operand is within 2^-11 relative of its
// f32 value: about 3e-4 relative L2 on a product, against 2.5e-3 with bf16
// operands.  fp16's range is kept by scaling each row of A by a power of two
// (its largest magnitude lands in [2^14, 2^15)), undone exactly in the
// epilogue.  A dequantised weight is fma(q, fp16(d*sc), fp16(-dmin*m)) with
// one fp16 rounding; q is exact (0..15).  The result is the product of those
// fp16 operands up to f32 summation order.
#include <cudaTypedefs.h>  // PFN_cuTensorMapEncodeTiled
#include <stdlib.h>

#include <algorithm>

#include "common.cuh"
#include "gemm.cuh"
#include "gemv.cuh"

namespace rt {

namespace {

constexpr int kBK = 64;                 // K-block: one 128-byte swizzle row of 16-bit elements
constexpr int kBlockBytes = 144;        // one Q4_K super-block (256 columns) of one row
constexpr int kKBPerBlock = 256 / kBK;  // K-blocks per super-block
constexpr int kDeqGroups = 2;                    // dequantiser groups: group g takes K-blocks g, g + 2, ...
constexpr int kGroupWarps = 8;                   // warps per group (one stage is filled by one group)
constexpr int kDeqWarps = kDeqGroups * kGroupWarps;
constexpr int kThreads = (2 + kDeqWarps) * 32;

// Tile configuration: NACC accumulators of M128 x N=BN stacked along M (CTA
// tile 128 NACC x BN; NACC * BN tensor-memory columns).  Larger tiles read A
// fewer times (N / BN) and dequantise W fewer times (M / (128 NACC)).
// AROWS < 128 (one accumulator, M <= AROWS): the operands swap roles.  The
// dequantised W tile is the MMA's A operand (M = 128 weight rows) and the
// AROWS rows of activations its B operand (N = AROWS), so the accumulator is
// C^T (tensor-memory lane = weight row, column = activation row).  Each MMA
// then reads 4 KB of weights and AROWS x 32 bytes of activations from shared
// memory instead of 128 rows of each; at small M the product is bound by
// that shared-memory traffic.  The smaller A stages also buy a deeper ring.
template <int NACC, int BN, int AROWS = 128>
struct Cfg {
    static constexpr int kBM = 128 * NACC;
    static constexpr int kATileC = AROWS * kBK * 2;  // one accumulator's A stage
    static constexpr int kBTile = BN * kBK * 2;
    static constexpr int kRawTile = BN * kBlockBytes;
    // Swapped (small M): two CTAs per SM, so each gets about half of the
    // shared memory.
    static constexpr int kStages = AROWS == 16 ? 4 : AROWS == 64 ? 3 : (NACC * BN >= 512 ? 2 : 4);  // A / B ring
    static constexpr int kRawStages = (BN >= 256 || AROWS < 128) ? 2 : 4;  // raw W super-block ring
    static constexpr int kCtasPerSm = AROWS < 128 ? 2 : 1;
    static constexpr bool kSwap = AROWS < 128;
    static constexpr int kTmemCols = kSwap ? (AROWS < 32 ? 32 : AROWS) : NACC * BN;
    static constexpr int kTpr = 256 / BN;  // dequantiser threads per W row
    static constexpr int kOffA = 0;
    static constexpr int kOffB = kOffA + kStages * NACC * kATileC;
    static constexpr int kOffRaw = kOffB + kStages * kBTile;
    static constexpr int kOffBar = kOffRaw + kRawStages * kRawTile;
    static constexpr int kNumBars = 4 * kStages + 2 * kRawStages + 1;
    static constexpr int kOffMisc = kOffBar + kNumBars * 8;
    static constexpr int kSmemBytes = kOffMisc + 16 + 1024;  // + slack for the 1024-byte alignment of the tiles
    // Instruction descriptor (kind::f16): f32 accumulator (bits 4-5 = 1), fp16
    // A and B (bits 7-9 and 10-12 = 0), both K-major, N = BN, M = 128.
    // (Swapped: M = BN weight rows, N = AROWS activation rows.)
    static constexpr uint32_t kIdesc =
        (1u << 4) | (static_cast<uint32_t>((kSwap ? AROWS : BN) >> 3) << 17) |
        (static_cast<uint32_t>((kSwap ? BN : 128) >> 4) << 24);
    static_assert(kOffB % 1024 == 0 && kOffRaw % 1024 == 0 && kRawTile % 128 == 0 && kATileC % 1024 == 0, "tile alignment");
    static_assert(AROWS == 128 || (NACC == 1 && BN == 128 && AROWS % 16 == 0), "swapped operands: one M128 accumulator");
    static_assert(kTmemCols >= 32 && (kTmemCols & (kTmemCols - 1)) == 0 && kTmemCols <= 512, "tensor memory allocation");
    static_assert(kSmemBytes * kCtasPerSm <= 227 * 1024, "shared memory");
    static_assert(kTmemCols <= 512 && (BN == 128 || BN == 256), "tensor memory");
};

// Shared-memory matrix descriptor of a K-major tile of 64-element (128-byte)
// 16-bit rows in the 128-byte swizzle: 8-row groups 1024 bytes apart (stride
// byte offset), descriptor version 1, layout type 2.  `addr` is the start of
// the K16 slice (tile base + 32 bytes per slice; the tile base is 1024-aligned).
__device__ __forceinline__ uint64_t sw128_desc(uint32_t addr) {
    return static_cast<uint64_t>((addr & 0x3FFFFu) >> 4) | (uint64_t{1} << 16) | (uint64_t{1024 >> 4} << 32) |
           (uint64_t{1} << 46) | (uint64_t{2} << 61);
}

__device__ __forceinline__ void umma_f16(uint32_t d_tmem, uint64_t a, uint64_t b, uint32_t idesc, uint32_t accumulate) {
    const uint32_t z = 0;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, {%5, %6, %7, %8}, p;\n\t}"
        ::"r"(d_tmem), "l"(a), "l"(b), "r"(idesc), "r"(accumulate), "r"(z), "r"(z), "r"(z), "r"(z));
}

// Arrive on `bar` once every tcgen05 operation this thread issued has completed.
__device__ __forceinline__ void umma_commit(uint64_t* bar) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(bar))
                 : "memory");
}

__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

// 2-D tensor copy without a cache hint, completing on `bar`.
__device__ __forceinline__ void tma_load_2d(void* dst, const CUtensorMap* tm, int x, int y, uint64_t* bar) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];" ::"r"(
            smem_u32(dst)),
        "l"(reinterpret_cast<uint64_t>(tm)), "r"(x), "r"(y), "r"(smem_u32(bar))
        : "memory");
}

// 32 consecutive f32 columns of this thread's tensor-memory lane.
__device__ __forceinline__ void tmem_ld32(uint32_t taddr, uint32_t (&v)[32]) {
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, "
        "%15, %16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31}, [%32];"
        : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3]), "=r"(v[4]), "=r"(v[5]), "=r"(v[6]), "=r"(v[7]), "=r"(v[8]),
          "=r"(v[9]), "=r"(v[10]), "=r"(v[11]), "=r"(v[12]), "=r"(v[13]), "=r"(v[14]), "=r"(v[15]), "=r"(v[16]),
          "=r"(v[17]), "=r"(v[18]), "=r"(v[19]), "=r"(v[20]), "=r"(v[21]), "=r"(v[22]), "=r"(v[23]), "=r"(v[24]),
          "=r"(v[25]), "=r"(v[26]), "=r"(v[27]), "=r"(v[28]), "=r"(v[29]), "=r"(v[30]), "=r"(v[31])
        : "r"(taddr));
    asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
}

__device__ __forceinline__ uint4 ld_shared_128(const void* p) {
    uint4 v;
    asm volatile("ld.shared.v4.u32 {%0, %1, %2, %3}, [%4];" : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w) : "r"(smem_u32(p)));
    return v;
}

__device__ __forceinline__ void st_shared_128(void* p, uint32_t a, uint32_t b, uint32_t c, uint32_t d) {
    asm volatile("st.shared.v4.u32 [%0], {%1, %2, %3, %4};" ::"r"(smem_u32(p)), "r"(a), "r"(b), "r"(c), "r"(d)
                 : "memory");
}

__device__ __forceinline__ uint32_t h2_sub(uint32_t a, uint32_t b) {
    uint32_t r;
    asm("sub.rn.f16x2 %0, %1, %2;" : "=r"(r) : "r"(a), "r"(b));
    return r;
}

__device__ __forceinline__ uint32_t h2_fma(uint32_t a, uint32_t b, uint32_t c) {
    uint32_t r;
    asm("fma.rn.f16x2 %0, %1, %2, %3;" : "=r"(r) : "r"(a), "r"(b), "r"(c));
    return r;
}

// fp16 bits of x (round to nearest even), twice.
__device__ __forceinline__ uint32_t f16_pair(float x) {
    uint32_t r;
    asm("cvt.rn.f16x2.f32 %0, %1, %1;" : "=r"(r) : "f"(x));
    return r;
}

// Two bf16 values -> the same two values in fp16 (exact in fp16's normal range).
__device__ __forceinline__ uint32_t bf16x2_to_f16x2(uint32_t x) {
    uint32_t r;
    asm("cvt.rn.f16x2.f32 %0, %1, %2;" : "=r"(r) : "f"(__uint_as_float(x & 0xFFFF0000u)), "f"(__uint_as_float(x << 16)));
    return r;
}

// Sixteen weights from the 8 bytes w0, w1 (16 nibbles): lo[] gets the low
// nibbles of bytes 0..7 in order as fp16 pairs, w = q * d_lo - m_lo; hi[] the
// high nibbles, w = q * d_hi - m_hi (dd / nm: the fp16 scale and negated min,
// twice).  A byte spread into a 16-bit lane and OR-ed into the fp16 pattern of
// 1024 (ulp 1) holds 1024 + q for its low nibble; its high nibble (q << 4)
// OR-ed into 64 (ulp 1/16) holds 64 + q.  Subtracting 1024 / 64 is exact, so
// the one rounding is the fma's.
__device__ __forceinline__ void dequant16_f16(uint32_t w0, uint32_t w1, uint32_t d_lo, uint32_t nm_lo, uint32_t d_hi,
                                              uint32_t nm_hi, uint32_t (&lo)[4], uint32_t (&hi)[4]) {
    constexpr uint32_t k1024 = 0x64006400u, k64 = 0x54005400u;
    const uint32_t sp[4] = {__byte_perm(w0, 0u, 0x4140u), __byte_perm(w0, 0u, 0x4342u), __byte_perm(w1, 0u, 0x4140u),
                            __byte_perm(w1, 0u, 0x4342u)};
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        lo[i] = h2_fma(h2_sub((sp[i] & 0x000F000Fu) | k1024, k1024), d_lo, nm_lo);
        hi[i] = h2_fma(h2_sub((sp[i] & 0x00F000F0u) | k64, k64), d_hi, nm_hi);
    }
}

// Wait for phase `parity` of `bar`, giving up after about one second
// (globaltimer, first read after 1024 polls so that short waits never pay
// for it): a CTA that stalls ends within seconds, with its error recorded.
__device__ __forceinline__ bool wait_phase(uint64_t* bar, uint32_t parity) {
    const uint32_t addr = smem_u32(bar);
    uint64_t t0 = 0;
    for (uint32_t it = 1;; ++it) {
        uint32_t done;
        asm volatile(
            "{\n\t.reg .pred p;\n\t"
            "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
            "selp.u32 %0, 1, 0, p;\n\t}"
            : "=r"(done)
            : "r"(addr), "r"(parity)
            : "memory");
        if (done) return true;
        if ((it & 1023u) == 0u) {
            uint64_t t;
            asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
            if (it == 1024u) t0 = t;
            else if (t - t0 > 1000000000ull) return false;
        }
    }
}

// True if phase `parity` of `bar` has completed (no waiting).
__device__ __forceinline__ bool test_phase(uint64_t* bar, uint32_t parity) {
    uint32_t done;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.test_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(done)
        : "r"(smem_u32(bar)), "r"(parity)
        : "memory");
    return done != 0;
}

__device__ __forceinline__ void fail(int* abort_flag, int* err) {
    atomicExch(abort_flag, 1);
    if (err) atomicExch(err, kErrMbarTimeout);
}

// WB: W is bf16 [N, K] (copied by TMA into the B tiles, then converted to
// fp16 in place).  ascale: row m of the product is multiplied by ascale[m]
// (null: 1).  Split-K: CTA z of the grid's third dimension takes columns
// [z kps, (z+1) kps) of K and writes its partial product to c + z M N.
template <int NACC, int BN, bool WB, int AROWS>
__global__ void __launch_bounds__(kThreads, Cfg<NACC, BN, AROWS>::kCtasPerSm)
    gemm_q4k_kernel(const __grid_constant__ CUtensorMap tm_a, const __grid_constant__ CUtensorMap tm_w,
                    const float* __restrict__ ascale, float* __restrict__ c, int64_t M, int64_t N, int K, int kps,
                    int* err) {
    using C = Cfg<NACC, BN, AROWS>;
    constexpr int kStages = C::kStages, kRawStages = C::kRawStages;
    extern __shared__ __align__(1024) uint8_t smem_raw[];
    uint8_t* sm = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t{1023});
    uint8_t* sA = sm + C::kOffA;
    uint8_t* sB = sm + C::kOffB;
    uint8_t* sRaw = sm + C::kOffRaw;
    uint64_t* bars = reinterpret_cast<uint64_t*>(sm + C::kOffBar);
    uint64_t* a_full = bars;
    uint64_t* b_full = a_full + kStages;
    uint64_t* empty = b_full + kStages;
    uint64_t* w_full = empty + kStages;  // WB: the bf16 W tile of the stage has landed
    uint64_t* raw_full = w_full + kStages;
    uint64_t* raw_empty = raw_full + kRawStages;
    uint64_t* tmem_full = raw_empty + kRawStages;
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(sm + C::kOffMisc);
    int* abort_flag = reinterpret_cast<int*>(sm + C::kOffMisc + 4);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int k0 = static_cast<int>(blockIdx.z) * kps;
    const int nkb = (min(K, k0 + kps) - k0) / kBK;
    c += static_cast<int64_t>(blockIdx.z) * M * N;
    const int m0 = static_cast<int>(blockIdx.y) * C::kBM, n0 = static_cast<int>(blockIdx.x) * BN;

    if (threadIdx.x == 0) {
        for (int s = 0; s < kStages; ++s) {
            mbar_init(&a_full[s], 1);
            mbar_init(&b_full[s], kGroupWarps);
            mbar_init(&empty[s], 1);
            mbar_init(&w_full[s], 1);
        }
        for (int r = 0; r < kRawStages; ++r) {
            mbar_init(&raw_full[r], 1);
            mbar_init(&raw_empty[r], kDeqWarps);
        }
        mbar_init(tmem_full, 1);
        *abort_flag = 0;
        fence_mbar_init();
    }
    __syncwarp();
    if (warp == 0) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_slot)),
                     "r"(C::kTmemCols)
                     : "memory");
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;

    if (warp == 0) {
        if (lane == 0) {
            // ---- TMA producer ----
            // Raw W super-blocks run ahead of the A/B stages as far as their
            // ring allows: the one a K-block needs is waited for, the next
            // ones are issued whenever a ring slot has been released.
            int kb_issued = 0;  // K-blocks whose A (and bf16 W) copies were issued
            const int nsb = WB ? 0 : nkb / kKBPerBlock;
            int sb_next = 0;  // next raw super-block to issue
            auto issue_raw = [&](bool block) -> int {  // 1 issued, 0 slot busy, -1 gave up
                const int r = sb_next % kRawStages;
                if (sb_next >= kRawStages) {
                    const uint32_t par = static_cast<uint32_t>(sb_next / kRawStages - 1) & 1u;
                    if (!block && !test_phase(&raw_empty[r], par)) return 0;
                    if (block && !wait_phase(&raw_empty[r], par)) return -1;
                }
                mbar_arrive_expect_tx(&raw_full[r], C::kRawTile);
                tma_load_2d(sRaw + r * C::kRawTile, &tm_w, (k0 / 256 + sb_next) * (kBlockBytes / 8), n0, &raw_full[r]);
                ++sb_next;
                return 1;
            };
            for (int kb = 0; kb < nkb; ++kb) {
                if (*reinterpret_cast<volatile int*>(abort_flag)) break;
                const int s = kb % kStages;
                if (!WB) {
                    bool gave_up = false;
                    while (sb_next <= kb / kKBPerBlock)
                        if (issue_raw(true) < 0) {
                            gave_up = true;
                            break;
                        }
                    if (gave_up) {
                        fail(abort_flag, err);
                        break;
                    }
                    while (sb_next < nsb && issue_raw(false) > 0) {
                    }
                }
                if (kb >= kStages && !wait_phase(&empty[s], static_cast<uint32_t>(kb / kStages - 1) & 1u)) {
                    fail(abort_flag, err);
                    break;
                }
                mbar_arrive_expect_tx(&a_full[s], NACC * C::kATileC);
#pragma unroll
                for (int ac = 0; ac < NACC; ++ac)
                    tma_load_2d(sA + (s * NACC + ac) * C::kATileC, &tm_a, k0 + kb * kBK, m0 + 128 * ac, &a_full[s]);
                if constexpr (WB) {
                    mbar_arrive_expect_tx(&w_full[s], C::kBTile);
                    tma_load_2d(sB + s * C::kBTile, &tm_w, k0 + kb * kBK, n0, &w_full[s]);
                }
                ++kb_issued;
            }
            // No copy of this CTA may still be landing when it exits: the last
            // copy into each stage (K-block / super-block i of a ring of n
            // slots completes phase i / n of slot i % n).
            for (int i = kb_issued > kStages ? kb_issued - kStages : 0; i < kb_issued; ++i) {
                (void)wait_phase(&a_full[i % kStages], static_cast<uint32_t>(i / kStages) & 1u);
                if (WB) (void)wait_phase(&w_full[i % kStages], static_cast<uint32_t>(i / kStages) & 1u);
            }
            for (int i = sb_next > kRawStages ? sb_next - kRawStages : 0; i < sb_next; ++i)
                (void)wait_phase(&raw_full[i % kRawStages], static_cast<uint32_t>(i / kRawStages) & 1u);
        }
    } else if (warp == 1) {
        if (lane == 0) {
            // ---- MMA issuer: accumulator ac in tensor-memory columns [ac * BN, (ac + 1) * BN) ----
            for (int kb = 0; kb < nkb; ++kb) {
                const int s = kb % kStages;
                const uint32_t par = static_cast<uint32_t>(kb / kStages) & 1u;
                if (!wait_phase(&a_full[s], par) || !wait_phase(&b_full[s], par)) {
                    fail(abort_flag, err);
                    break;
                }
                tc_fence_after();
                const uint32_t b_addr = smem_u32(sB + s * C::kBTile);
                if constexpr (C::kSwap) {
                    const uint32_t x_addr = smem_u32(sA + s * C::kATileC);
#pragma unroll
                    for (int k16 = 0; k16 < kBK / 16; ++k16)
                        umma_f16(tmem, sw128_desc(b_addr + 32 * k16), sw128_desc(x_addr + 32 * k16), C::kIdesc,
                                 (kb | k16) != 0);
                }
#pragma unroll
                for (int ac = 0; ac < (C::kSwap ? 0 : NACC); ++ac) {
                    const uint32_t a_addr = smem_u32(sA + (s * NACC + ac) * C::kATileC);
#pragma unroll
                    for (int k16 = 0; k16 < kBK / 16; ++k16)
                        umma_f16(tmem + static_cast<uint32_t>(ac * BN), sw128_desc(a_addr + 32 * k16),
                                  sw128_desc(b_addr + 32 * k16), C::kIdesc, (kb | k16) != 0);
                }
                umma_commit(&empty[s]);
            }
            umma_commit(tmem_full);  // also on failure: arrives once every MMA above has completed
        }
    } else {
        // ---- dequantisers: W row n of the tile; halves h0.. of each 64-column K-block ----
        const int dgrp = (warp - 2) / kGroupWarps;
        const int d = threadIdx.x - 64 - dgrp * kGroupWarps * 32;  // thread of the group
        const int n = d / C::kTpr;
        const int h_first = C::kTpr == 2 ? (d & 1) : 0, h_count = C::kTpr == 2 ? 1 : 2;
        if constexpr (WB) {
            // bf16 W tile -> fp16 in place (the swizzled layout is the same for
            // both types).  The stage's previous MMA is waited for first: with
            // an odd ring (3 stages) a stage alternates between the two groups,
            // and without that wait a group could test w_full[s] while the
            // previous K-block's copy into the stage had not landed, so that
            // its parity matched the phase two back.
            for (int kb = dgrp; kb < nkb; kb += kDeqGroups) {
                if (*reinterpret_cast<volatile int*>(abort_flag)) break;
                const int s = kb % kStages;
                if (kb >= kStages && !wait_phase(&empty[s], static_cast<uint32_t>(kb / kStages - 1) & 1u)) {
                    fail(abort_flag, err);
                    break;
                }
                if (!wait_phase(&w_full[s], static_cast<uint32_t>(kb / kStages) & 1u)) {
                    fail(abort_flag, err);
                    break;
                }
                uint8_t* tile = sB + s * C::kBTile;
                for (int ci = d; ci < C::kBTile / 16; ci += kGroupWarps * 32) {
                    const uint4 v = ld_shared_128(tile + 16 * ci);
                    st_shared_128(tile + 16 * ci, bf16x2_to_f16x2(v.x), bf16x2_to_f16x2(v.y), bf16x2_to_f16x2(v.z),
                                  bf16x2_to_f16x2(v.w));
                }
                fence_proxy_async_smem();
                __syncwarp();
                if (lane == 0) mbar_arrive(&b_full[s]);
            }
        }
        for (int kb = dgrp; kb < (WB ? 0 : nkb); kb += kDeqGroups) {
            if (*reinterpret_cast<volatile int*>(abort_flag)) break;
            const int s = kb % kStages, sb = kb / kKBPerBlock, ch = kb % kKBPerBlock, r = sb % kRawStages;
            // the group's first K-block of a super-block waits for its raw tile
            if (ch == dgrp && !wait_phase(&raw_full[r], static_cast<uint32_t>(sb / kRawStages) & 1u)) {
                fail(abort_flag, err);
                break;
            }
            if (kb >= kStages && !wait_phase(&empty[s], static_cast<uint32_t>(kb / kStages - 1) & 1u)) {
                fail(abort_flag, err);
                break;
            }
            const uint8_t* row = sRaw + r * C::kRawTile + n * kBlockBytes;
            const uint4 hdr = ld_shared_128(row);  // d, dmin, 12 bytes of scales/mins
            const float dd = f16_bits_to_f32(hdr.x & 0xFFFFu), dmin = f16_bits_to_f32(hdr.x >> 16);
            // scale_min of sub-blocks 2ch (low nibbles) and 2ch + 1 (high nibbles)
            // (Q4KMat::scale_min, src/autograd2.rs:1075-1085)
            auto scb = [&](int b) -> uint32_t {
                const uint32_t wd = b < 4 ? hdr.y : (b < 8 ? hdr.z : hdr.w);
                return (wd >> (8 * (b & 3))) & 0xFFu;
            };
            auto scale_min = [&](int j, float& d1, float& m1) {
                uint32_t sc, mn;
                if (j < 4) {
                    sc = scb(j) & 63u;
                    mn = scb(j + 4) & 63u;
                } else {
                    sc = (scb(j + 4) & 0xFu) | ((scb(j - 4) >> 6) << 4);
                    mn = (scb(j + 4) >> 4) | ((scb(j) >> 6) << 4);
                }
                d1 = __fmul_rn(dd, static_cast<float>(sc));
                m1 = __fmul_rn(dmin, static_cast<float>(mn));
            };
            float d_lo, m_lo, d_hi, m_hi;
            scale_min(2 * ch, d_lo, m_lo);
            scale_min(2 * ch + 1, d_hi, m_hi);
            const uint32_t hd_lo = f16_pair(d_lo), hm_lo = f16_pair(-m_lo), hd_hi = f16_pair(d_hi), hm_hi = f16_pair(-m_hi);
            uint8_t* tile = sB + s * C::kBTile + (n >> 3) * 1024 + (n & 7) * 128;
            const int sw = n & 7;
            for (int hh = 0; hh < h_count; ++hh) {
                const int h = h_first + hh;
                const uint4 qs = ld_shared_128(row + 16 + 32 * ch + 16 * h);
                const uint32_t q[4] = {qs.x, qs.y, qs.z, qs.w};
#pragma unroll
                for (int part = 0; part < 2; ++part) {  // 8 bytes: columns 16h + 8part.. (low), 32 + .. (high)
                    uint32_t lo[4], hi[4];
                    dequant16_f16(q[2 * part], q[2 * part + 1], hd_lo, hm_lo, hd_hi, hm_hi, lo, hi);
                    const int c_lo = 2 * h + part, c_hi = 4 + 2 * h + part;  // 16-byte chunks of the 128-byte row
                    st_shared_128(tile + ((c_lo ^ sw) << 4), lo[0], lo[1], lo[2], lo[3]);
                    st_shared_128(tile + ((c_hi ^ sw) << 4), hi[0], hi[1], hi[2], hi[3]);
                }
            }
            fence_proxy_async_smem();  // the MMA (async proxy) reads these stores; the raw reads precede the TMA refill
            __syncwarp();
            if (lane == 0) {
                mbar_arrive(&b_full[s]);
                if (ch >= kKBPerBlock - kDeqGroups) mbar_arrive(&raw_empty[r]);  // the group's last K-block of it
            }
        }
        // ---- epilogue: warp w owns tensor-memory lanes 32 (w % 4) .. +31; the
        // warps of a lane quarter split the (accumulator, 32-column) chunks ----
        const int quad = warp & 3, grp = (warp - 2) >> 2;
        constexpr int kEpiGroups = kDeqWarps / 4;
        const bool ok = wait_phase(tmem_full, 0u);
        if (!ok) fail(abort_flag, err);
        if (ok && !*reinterpret_cast<volatile int*>(abort_flag) && C::kSwap) {
            // lane = weight row n0 + 32 quad + lane; columns = activation rows
            tc_fence_after();
            const int64_t col = static_cast<int64_t>(n0) + 32 * quad + lane;
            for (int cc = grp; cc < (AROWS + 31) / 32; cc += kEpiGroups) {
                uint32_t v[32];
                tmem_ld32(tmem + (static_cast<uint32_t>(32 * quad) << 16) + static_cast<uint32_t>(32 * cc), v);
#pragma unroll
                for (int i = 0; i < 32; ++i) {
                    const int64_t row = 32 * cc + i;  // m0 = 0: one row tile
                    if (row < M && row < AROWS && col < N)
                        c[row * N + col] = __uint_as_float(v[i]) * (ascale ? ascale[row] : 1.0f);
                }
            }
        } else if (ok && !*reinterpret_cast<volatile int*>(abort_flag)) {
            tc_fence_after();
            for (int item = grp; item < NACC * (BN / 32); item += kEpiGroups) {
                const int ac = item / (BN / 32), cc = item % (BN / 32);
                uint32_t v[32];
                tmem_ld32(tmem + (static_cast<uint32_t>(32 * quad) << 16) + static_cast<uint32_t>(ac * BN + 32 * cc), v);
                const int64_t rowi = static_cast<int64_t>(m0) + 128 * ac + 32 * quad + lane;
                const int64_t col0 = n0 + 32 * cc;
                if (rowi < M) {
                    float* crow = c + rowi * N;
                    const float rs = ascale ? ascale[rowi] : 1.0f;
#pragma unroll
                    for (int i = 0; i < 32; ++i) v[i] = __float_as_uint(__uint_as_float(v[i]) * rs);
                    if (col0 + 32 <= N && (N & 3) == 0) {
#pragma unroll
                        for (int i = 0; i < 8; ++i)
                            *reinterpret_cast<float4*>(crow + col0 + 4 * i) =
                                make_float4(__uint_as_float(v[4 * i]), __uint_as_float(v[4 * i + 1]),
                                            __uint_as_float(v[4 * i + 2]), __uint_as_float(v[4 * i + 3]));
                    } else {
                        for (int i = 0; i < 32; ++i)
                            if (col0 + i < N) crow[col0 + i] = __uint_as_float(v[i]);
                    }
                }
            }
        }
    }
    // ---- teardown: every tensor-memory access done, then warp 0 frees it ----
    tc_fence_before();
    __syncthreads();
    if (warp == 0) {
        tc_fence_after();
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(C::kTmemCols) : "memory");
    }
}

}  // namespace

GemmPlan gemm_q4k_plan(int64_t m, int64_t n, int k, int num_sms, bool wbf16, bool allow_split) {
    GemmPlan p;
    if (m <= 0 || n <= 0 || k <= 0 || k % 256 != 0 || m > 0x7FFFFFFF || n > 0x7FFFFFFF) return p;
    // Q4_K at M <= 16: the multi-row GEMV streams the weights several times
    // faster than the tensor-memory kernel's per-K-block chain.  RT_GEMM_ROWS=0
    // or a forced tile (RT_GEMM_TILE) keeps the tcgen05 kernel; RT_GEMM_SPLITS
    // forces either kernel's K split (tests and tuning).
    const char* rows_env = getenv("RT_GEMM_ROWS");
    const char* splits_env = getenv("RT_GEMM_SPLITS");
    if (!wbf16 && m <= kRowsMaxM && !(rows_env && atoi(rows_env) == 0) && !getenv("RT_GEMM_TILE") &&
        gemm_rows_plan(m, n, k, num_sms > 0 ? num_sms : 148, allow_split ? 8 : 1,
                       allow_split && splits_env ? atoi(splits_env) : 0, &p))
        return p;
    // The 256 x 256 tile streams A half as often and dequantises W half as
    // often as the 128 x 128 tile, at about half the cost per FLOP (measured);
    // estimated time: waves of CTAs x per-tile cost (2 units big, 1 small).
    const int64_t small = ((m + 127) / 128) * ((n + 127) / 128), big = ((m + 255) / 256) * ((n + 255) / 256);
    const int64_t sms = num_sms > 0 ? num_sms : 148;
    bool use_big = ((big + sms - 1) / sms) * 2 <= (small + sms - 1) / sms;
    // At M <= 64 the product is a weight stream, and the swapped 128 tile (two
    // CTAs per SM) streams faster than the 256 tile that the estimate picks
    // for wide N (measured: BF16 262144 x 5376 at M = 1 / 8 886 / 926 -> 446 /
    // 454 us, 262144 x 2560 at M = 64 426 -> 262 us; Q4_K 20480 x 2560 at
    // M = 1 / 8 / 64 51.3 / 43.0 / 47.5 -> 39.1 / 40.3 / 43.4 us).
    if (m <= 64) use_big = false;
    // RT_GEMM_TILE=128 or 256 forces the tile (tests and tuning).
    if (const char* t = getenv("RT_GEMM_TILE")) {
        if (atoi(t) == 128) use_big = false;
        else if (atoi(t) == 256) use_big = true;
    }
    p.bm = use_big ? 256 : 128;
    p.bn = use_big ? 256 : 128;
    p.wbf16 = wbf16;
    const int64_t gx = (n + p.bn - 1) / p.bn, gy = (m + p.bm - 1) / p.bm;
    if (gx > 0x7FFFFFFF || gy > 65535) return GemmPlan{};
    // Split K (in whole 256-column super-blocks) while the tiles leave SMs idle.
    const int nsb = k / 256;
    // Split K only while the product is a weight stream (M <= 128): then
    // filling the SMs pays (measured at M = 64: 101 -> 30 us for a 10240-column
    // down projection); at larger M the partial products' traffic costs more.
    int splits = 1;
    // Resident CTAs: two per SM for the swapped small-M tiles; only at M <= 16
    // do the extra splits pay (measured: M = 8 down projection 87 -> 67 us, M =
    // 64 projections 10-30% slower from the partial sums).
    const int64_t slots = sms * ((!use_big && m <= 16) ? 2 : 1);
    if (allow_split && m <= 128) splits = static_cast<int>(std::max<int64_t>(1, std::min<int64_t>(std::min(nsb, 8), slots / (gx * gy))));
    // Q4_K tiles that alone fill half a wave to two waves of the small-M slots
    // leave the last wave's SMs idle; 3 splits above one wave, 4 below, give
    // them work when K is long (measured, M = 1 and 8: 27B gate/up N = 43008
    // 117 -> 103 us, its 2-rank shard N = 21504 91 -> 84 us; with K = 2560,
    // 10 super-blocks, splitting is slower, so K needs 16 or more).
    if (allow_split && !wbf16 && m <= 16 && splits == 1 && nsb >= 16 && 2 * gx * gy >= slots && gx * gy < 2 * slots)
        splits = gx * gy > slots ? 3 : 4;
    if (const char* t = getenv("RT_GEMM_SPLITS")) splits = std::max(1, std::min(nsb, atoi(t)));  // tests
    const int per = (nsb + splits - 1) / splits;
    p.kps = per * 256;
    p.splits = (nsb + per - 1) / per;
    p.grid = dim3(static_cast<unsigned>(gx), static_cast<unsigned>(gy), static_cast<unsigned>(p.splits));
    p.arows = use_big ? 128 : (m <= 16 ? 16 : m <= 64 ? 64 : 128);
    p.smem = use_big ? Cfg<2, 256>::kSmemBytes
                     : (p.arows == 16 ? Cfg<1, 128, 16>::kSmemBytes
                                      : p.arows == 64 ? Cfg<1, 128, 64>::kSmemBytes : Cfg<1, 128>::kSmemBytes);
    return p;
}

cudaError_t gemm_q4k_prepare() {
    cudaError_t e = cudaSuccess;
    auto set = [&](auto kernel, int bytes) {
        if (e == cudaSuccess) e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes);
    };
    set(gemm_q4k_kernel<1, 128, false, 128>, Cfg<1, 128>::kSmemBytes);
    set(gemm_q4k_kernel<1, 128, false, 64>, Cfg<1, 128, 64>::kSmemBytes);
    set(gemm_q4k_kernel<1, 128, false, 16>, Cfg<1, 128, 16>::kSmemBytes);
    set(gemm_q4k_kernel<2, 256, false, 128>, Cfg<2, 256>::kSmemBytes);
    set(gemm_q4k_kernel<1, 128, true, 128>, Cfg<1, 128>::kSmemBytes);
    set(gemm_q4k_kernel<1, 128, true, 64>, Cfg<1, 128, 64>::kSmemBytes);
    set(gemm_q4k_kernel<1, 128, true, 16>, Cfg<1, 128, 16>::kSmemBytes);
    set(gemm_q4k_kernel<2, 256, true, 128>, Cfg<2, 256>::kSmemBytes);
    if (e == cudaSuccess) e = gemm_rows_prepare();
    return e;
}

bool gemm_q4k_tmaps(const void* a, int64_t m, const void* w, int64_t n, int k, const GemmPlan& p, CUtensorMap* tm_a,
                    CUtensorMap* tm_w) {
    const TmapEncodeFn encode = tmap_encoder();
    if (!encode) return false;
    const cuuint32_t estr[2] = {1, 1};
    auto map16 = [&](CUtensorMap* out, CUtensorMapDataType dt, const void* base, int64_t rows, int box_rows) {
        const cuuint64_t dims[2] = {static_cast<cuuint64_t>(k), static_cast<cuuint64_t>(rows)};
        const cuuint64_t strides[1] = {static_cast<cuuint64_t>(k) * 2};
        const cuuint32_t box[2] = {kBK, static_cast<cuuint32_t>(box_rows)};
        return encode(out, dt, 2, const_cast<void*>(base), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                      CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                      CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
    };
    if (!map16(tm_a, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, a, m, p.arows)) return false;
    if (p.wbf16) return map16(tm_w, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, w, n, p.bn);
    const uint64_t row_bytes = static_cast<uint64_t>(k / 256) * kBlockBytes;
    const cuuint64_t dims[2] = {row_bytes / 8, static_cast<cuuint64_t>(n)};
    const cuuint64_t strides[1] = {row_bytes};
    const cuuint32_t box[2] = {kBlockBytes / 8, static_cast<cuuint32_t>(p.bn)};
    return encode(tm_w, CU_TENSOR_MAP_DATA_TYPE_UINT64, 2, const_cast<void*>(w), dims, strides, box, estr,
                  CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                  CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

cudaError_t gemm_q4k_launch(const CUtensorMap& tm_a, const CUtensorMap& tm_w, const float* ascale, float* c, int64_t m,
                            int64_t n, int k, const GemmPlan& p, int* err, cudaStream_t s, const uint16_t* a) {
    if (p.rows_nt > 0) return gemm_rows_launch(tm_w, a, ascale, c, m, n, k, p, err, s);
    const dim3 g = p.grid;
#define RT_GEMM_LAUNCH(NA, BNN, WBB, AR) \
    gemm_q4k_kernel<NA, BNN, WBB, AR><<<g, kThreads, p.smem, s>>>(tm_a, tm_w, ascale, c, m, n, k, p.kps, err)
    if (p.bm == 256 && !p.wbf16) RT_GEMM_LAUNCH(2, 256, false, 128);
    else if (p.bm == 256) RT_GEMM_LAUNCH(2, 256, true, 128);
    else if (p.bm == 128 && !p.wbf16 && p.arows == 16) RT_GEMM_LAUNCH(1, 128, false, 16);
    else if (p.bm == 128 && !p.wbf16 && p.arows == 64) RT_GEMM_LAUNCH(1, 128, false, 64);
    else if (p.bm == 128 && !p.wbf16) RT_GEMM_LAUNCH(1, 128, false, 128);
    else if (p.bm == 128 && p.arows == 16) RT_GEMM_LAUNCH(1, 128, true, 16);
    else if (p.bm == 128 && p.arows == 64) RT_GEMM_LAUNCH(1, 128, true, 64);
    else if (p.bm == 128) RT_GEMM_LAUNCH(1, 128, true, 128);
#undef RT_GEMM_LAUNCH
    else return cudaErrorInvalidValue;
    return cudaGetLastError();
}

namespace {
// One CTA per row: out = fp16(a * 2^-e), scale[row] = 2^e (row_scale_f16).
__global__ void a_to_f16_rows_kernel(const uint16_t* __restrict__ a, int k, uint16_t* __restrict__ out,
                                     float* __restrict__ scale) {
    __shared__ float red[32];
    const int64_t base = static_cast<int64_t>(blockIdx.x) * k;
    float mx = 0.f;
    for (int c = threadIdx.x; c < k; c += blockDim.x) mx = fmaxf(mx, fabsf(bf16_bits_to_f32(a[base + c])));
    mx = block_max(mx, red);
    float inv, sc;
    row_scale_f16(mx, &inv, &sc);
    for (int c = threadIdx.x; c < k; c += blockDim.x)
        out[base + c] = __half_as_ushort(__float2half_rn(bf16_bits_to_f32(a[base + c]) * inv));
    if (threadIdx.x == 0) scale[blockIdx.x] = sc;
}

// The same from f32 rows.
__global__ void a_f32_to_f16_rows_kernel(const float* __restrict__ a, int k, uint16_t* __restrict__ out,
                                         float* __restrict__ scale) {
    __shared__ float red[32];
    const int64_t base = static_cast<int64_t>(blockIdx.x) * k;
    float mx = 0.f;
    for (int c = threadIdx.x; c < k; c += blockDim.x) mx = fmaxf(mx, fabsf(a[base + c]));
    mx = block_max(mx, red);
    float inv, sc;
    row_scale_f16(mx, &inv, &sc);
    for (int c = threadIdx.x; c < k; c += blockDim.x) out[base + c] = __half_as_ushort(__float2half_rn(a[base + c] * inv));
    if (threadIdx.x == 0) scale[blockIdx.x] = sc;
}

// y[r][c] += bias[c] over m rows of n (add_bias_rows, src/qlinear.rs:49-61).
__global__ void bias_rows_kernel(float* __restrict__ y, int64_t m, int64_t n, const float* __restrict__ bias) {
    const int64_t total = m * n, stride = static_cast<int64_t>(gridDim.x) * blockDim.x;
    for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < total; i += stride)
        y[i] += bias[i % n];
}

// out[i] = sum over z < parts of in[z * count + i], in part order.
__global__ void sum_parts_kernel(const float* __restrict__ in, int parts, int64_t count, float* __restrict__ out) {
    const int64_t stride = static_cast<int64_t>(gridDim.x) * blockDim.x;
    for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < count; i += stride) {
        float v = in[i];
        for (int z = 1; z < parts; ++z) v += in[z * count + i];
        out[i] = v;
    }
}
}  // namespace

cudaError_t a_to_f16_launch(const uint16_t* a_bf16, int64_t m, int k, uint16_t* out, float* scale, cudaStream_t s) {
    if (m <= 0) return cudaSuccess;
    if (m > 0x7FFFFFFF) return cudaErrorInvalidValue;
    a_to_f16_rows_kernel<<<static_cast<unsigned>(m), 256, 0, s>>>(a_bf16, k, out, scale);
    return cudaGetLastError();
}

cudaError_t a_f32_to_f16_launch(const float* a, int64_t m, int k, uint16_t* out, float* scale, cudaStream_t s) {
    if (m <= 0) return cudaSuccess;
    if (m > 0x7FFFFFFF) return cudaErrorInvalidValue;
    a_f32_to_f16_rows_kernel<<<static_cast<unsigned>(m), 256, 0, s>>>(a, k, out, scale);
    return cudaGetLastError();
}

cudaError_t bias_rows_launch(float* y, int64_t m, int64_t n, const float* bias, int num_sms, cudaStream_t s) {
    if (m <= 0 || n <= 0) return cudaSuccess;
    const int64_t blocks = std::min<int64_t>((m * n + 255) / 256, static_cast<int64_t>(num_sms > 0 ? num_sms : 148) * 8);
    bias_rows_kernel<<<static_cast<unsigned>(blocks), 256, 0, s>>>(y, m, n, bias);
    return cudaGetLastError();
}

cudaError_t sum_parts_launch(const float* in, int parts, int64_t count, float* out, int num_sms, cudaStream_t s) {
    if (count <= 0) return cudaSuccess;
    const int64_t blocks = std::min<int64_t>((count + 255) / 256, static_cast<int64_t>(num_sms > 0 ? num_sms : 148) * 8);
    sum_parts_kernel<<<static_cast<unsigned>(blocks), 256, 0, s>>>(in, parts, count, out);
    return cudaGetLastError();
}

}  // namespace rt
