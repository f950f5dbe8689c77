// common.cuh -- sm_100a device helpers shared by the decode-path kernels:
// TMA bulk copies into shared memory completed on mbarriers (with bounded
// waits), programmatic dependent launch (PDL), packed f32x2 FMA, block
// reductions, and the launch helper that attaches the PDL attribute.
#pragma once

#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

namespace rt {

// Error words written by kernels into a device int (never trap).
enum : int {
    kErrNone = 0,
    kErrMbarTimeout = 1,  // an mbarrier wait exceeded its iteration limit
    kErrShape = 2,        // a kernel saw an argument it cannot handle
    kErrGridTimeout = 3,  // a grid-wide barrier of a persistent kernel timed out
};

// Iteration limit of every spin on an mbarrier.  Each try_wait may suspend the
// thread for a hardware-chosen interval, so this bounds the wait to well under
// a minute even in the worst case, while a healthy wait ends in microseconds.
constexpr uint32_t kMaxWaitIters = 1u << 24;

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
    return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}

// Make mbarrier initialisation visible to the async (TMA) proxy.
__device__ __forceinline__ void fence_mbar_init() {
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes)
                 : "memory");
}

// Bounded wait for phase `parity` of `bar`.  iters == 0: the default bound
// (mbar_wait).  iters > 0: at most `iters` non-blocking polls (test_wait, which
// never suspends the thread), so a small limit really does give up when the
// phase is not complete yet.  Returns false on timeout.
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity);
__device__ __forceinline__ bool mbar_wait_n(uint64_t* bar, uint32_t parity, uint32_t iters) {
    if (iters == 0) return mbar_wait(bar, parity);
    const uint32_t addr = smem_u32(bar);
    for (uint32_t it = 0; it < iters; ++it) {
        uint32_t done;
        asm volatile(
            "{\n\t.reg .pred p;\n\t"
            "mbarrier.test_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
            "selp.u32 %0, 1, 0, p;\n\t}"
            : "=r"(done)
            : "r"(addr), "r"(parity)
            : "memory");
        if (done) return true;
    }
    return false;
}

// Bounded wait for phase `parity` of `bar`.  Returns false on timeout.
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity) {
    uint32_t addr = smem_u32(bar);
    for (uint32_t it = 0; it < kMaxWaitIters; ++it) {
        uint32_t done;
        asm volatile(
            "{\n\t.reg .pred p;\n\t"
            "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
            "selp.u32 %0, 1, 0, p;\n\t}"
            : "=r"(done)
            : "r"(addr), "r"(parity)
            : "memory");
        if (done) return true;
    }
    return false;
}

// L2 policy for streamed-once data (weights): evict first, so the weight
// stream does not push activations and the KV cache out of L2.
// Wait for phase `parity` of `bar`, giving up after about one second of
// globaltimer (first read after 1024 polls, so that short waits never pay
// for it): false if it gave up.
__device__ __forceinline__ bool mbar_wait_timed(uint64_t* bar, uint32_t parity) {
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

__device__ __forceinline__ uint64_t l2_evict_first_policy() {
    uint64_t pol;
    asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(pol));
    return pol;
}

// 1-D TMA bulk copy global -> shared, completing `bytes` on `bar`.
// dst, src 16-byte aligned; bytes a multiple of 16.
__device__ __forceinline__ void bulk_g2s(void* dst, const void* src, uint32_t bytes, uint64_t* bar,
                                         uint64_t policy) {
    asm volatile(
        "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint [%0], [%1], %2, [%3], %4;" ::"r"(
            smem_u32(dst)),
        "l"(src), "r"(bytes), "r"(smem_u32(bar)), "l"(policy)
        : "memory");
}

// 2-D tiled TMA load (tensor map in the kernel's parameter space) completing on `bar`.
// Into this CTA's shared memory only.  x is the innermost coordinate in elements of the map.
__device__ __forceinline__ void tma_2d_g2s(void* dst, const void* tmap, int x, int y, uint64_t* bar, uint64_t policy) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint [%0], [%1, {%2, %3}], [%4], %5;" ::"r"(
            smem_u32(dst)),
        "l"(reinterpret_cast<uint64_t>(tmap)), "r"(x), "r"(y), "r"(smem_u32(bar)), "l"(policy)
        : "memory");
}

__device__ __forceinline__ void bulk_g2s_nohint(void* dst, const void* src, uint32_t bytes, uint64_t* bar) {
    asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
                     smem_u32(dst)),
                 "l"(src), "r"(bytes), "r"(smem_u32(bar))
                 : "memory");
}

// Order this thread's earlier generic-proxy accesses of shared memory (plain
// loads, ldmatrix) before later async-proxy (TMA) writes to the same bytes.
__device__ __forceinline__ void fence_proxy_async_smem() {
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

// Four 8x8 b16 matrices from shared memory; lane l gives the row address of
// matrix l/8, row l%8 (16-byte aligned) and receives word (l%4) of row l/4 of
// each matrix.
__device__ __forceinline__ void ldsm_x4(const void* p, uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3) {
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0, %1, %2, %3}, [%4];"
                 : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
                 : "r"(smem_u32(p))
                 : "memory");
}

// Programmatic dependent launch: let the next kernel in the stream start its
// prologue now, and wait until every prerequisite grid has completed and its
// memory is visible.
__device__ __forceinline__ void pdl_launch_dependents() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }

// d = a * b + c on a pair of f32 lanes (sm_100 packed FMA).
__device__ __forceinline__ float2 ffma2(float2 a, float2 b, float2 c) {
    float2 d;
    asm("{\n\t.reg .b64 ra, rb, rc, rd;\n\t"
        "mov.b64 ra, {%2, %3};\n\t"
        "mov.b64 rb, {%4, %5};\n\t"
        "mov.b64 rc, {%6, %7};\n\t"
        "fma.rn.f32x2 rd, ra, rb, rc;\n\t"
        "mov.b64 {%0, %1}, rd;\n\t}"
        : "=f"(d.x), "=f"(d.y)
        : "f"(a.x), "f"(a.y), "f"(b.x), "f"(b.y), "f"(c.x), "f"(c.y));
    return d;
}

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}

__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
    return v;
}

// Maximum over the whole block; every thread gets it (`red` as for block_sum).
__device__ __forceinline__ float block_max(float v, float* red) {
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nw = blockDim.x >> 5;
    v = warp_max(v);
    __syncthreads();
    if (lane == 0) red[warp] = v;
    __syncthreads();
    return warp_max(lane < nw ? red[lane] : -INFINITY);
}

// Sum over the whole block; every thread gets the result.  `red` must hold
// 32 floats of shared memory; blockDim.x is a multiple of 32.  The per-warp
// sums are added by an xor butterfly in every warp: a fixed order (so the
// result is deterministic) in which each addition pairs the same two values
// on every lane, so every thread of the block, and every CTA that reduces the
// same values, gets the same bits.  Five shuffles instead of a chain of 16
// dependent shared-memory loads.
__device__ __forceinline__ float block_sum(float v, float* red) {
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nw = blockDim.x >> 5;
    v = warp_sum(v);
    __syncthreads();
    if (lane == 0) red[warp] = v;
    __syncthreads();
    return warp_sum(lane < nw ? red[lane] : 0.f);
}

// ---- Tagged words ("LL" words, after NCCL's low-latency protocol) ----------
// A 32-bit value and the 32-bit tag of the phase that wrote it, stored as one
// naturally aligned 64-bit word, so a reader sees either the old pair or the
// new one, never a mix.  A consumer polls the words it needs until each
// carries the tag it expects: the data itself says it is ready, with no
// barrier or flag between producer and consumer.
__device__ __forceinline__ uint64_t ll_word(float v, uint32_t tag) {
    return (static_cast<uint64_t>(tag) << 32) | __float_as_uint(v);
}
__device__ __forceinline__ void ll_store(uint64_t* p, float v, uint32_t tag) {
    asm volatile("st.relaxed.gpu.global.u64 [%0], %1;" ::"l"(p), "l"(ll_word(v, tag)) : "memory");
}
// Two consecutive words at p (16-byte aligned).
__device__ __forceinline__ void ll_store2(uint64_t* p, float a, float b, uint32_t tag) {
    asm volatile("st.relaxed.gpu.global.v2.u64 [%0], {%1, %2};" ::"l"(p), "l"(ll_word(a, tag)), "l"(ll_word(b, tag))
                 : "memory");
}
__device__ __forceinline__ ulonglong2 ll_load2(const uint64_t* p) {
    ulonglong2 r;
    asm volatile("ld.relaxed.gpu.global.v2.u64 {%0, %1}, [%2];" : "=l"(r.x), "=l"(r.y) : "l"(p) : "memory");
    return r;
}
__device__ __forceinline__ uint64_t ll_load(const uint64_t* p) {
    uint64_t r;
    asm volatile("ld.relaxed.gpu.global.u64 %0, [%1];" : "=l"(r) : "l"(p) : "memory");
    return r;
}
__device__ __forceinline__ float ll_val(uint64_t w) { return __uint_as_float(static_cast<uint32_t>(w)); }
__device__ __forceinline__ bool ll_has(uint64_t w, uint32_t tag) { return static_cast<uint32_t>(w >> 32) == tag; }

// Bound of a poll on tagged words: about two seconds of globaltimer (first
// read after 32 polls), and an early stop when another CTA raised `abort`.
struct LLPoll {
    const int* abort;
    uint64_t t0;
    uint32_t it;
    __device__ __forceinline__ void init(const int* ab) {
        abort = ab;
        t0 = 0;
        it = 0;
    }
    // After a poll that found some word not ready: false when the wait must stop.
    __device__ __forceinline__ bool again() {
        if ((++it & 31u) == 0u) {
            if (abort && *reinterpret_cast<const volatile int*>(abort)) return false;
            uint64_t t;
            asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
            if (it == 32u) t0 = t;
            else if (t - t0 > 2000000000ull) return false;
        }
        return true;
    }
};

__device__ __forceinline__ float bf16_bits_to_f32(uint32_t b) { return __uint_as_float(b << 16); }

__device__ __forceinline__ float f16_bits_to_f32(uint32_t h) {
    return __half2float(__ushort_as_half(static_cast<unsigned short>(h)));
}

}  // namespace rt

// Host-side launch helper: cudaLaunchKernelEx with optional PDL attribute.
template <typename... KArgs, typename... Args>
static inline cudaError_t rt_launch(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem,
                                    cudaStream_t stream, bool pdl, Args&&... args) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.dynamicSmemBytes = smem;
    cfg.stream = stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = pdl ? 1 : 0;
    return cudaLaunchKernelEx(&cfg, kernel, std::forward<Args>(args)...);
}
