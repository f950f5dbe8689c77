// step.cu -- the persistent Gemma 3 decode-step kernel.
//
// One cooperative launch runs a whole decode step: for every layer the QKV
// projection (with the fused residual/RMSNorm prologue), attention, the O
// projection, gate/up with the GELU gate and the down projection, then the LM
// head with the greedy argmax (Gemma3Block::forward_cached,
// src/transformer4.rs:1954-1964, and MetalDecodeContext::decode_step,
// src/metal_decode.rs:1930-2074).  One CTA per SM, all resident at once.
//
// No grid-wide barrier: every vector a phase produces (q/k/v, the attention
// output, O, the gated FFN hidden, the down projection's column parts) is
// published as tagged words (common.cuh), and the next phase's prologue polls
// exactly the words it needs until they carry this launch's tag for that
// vector.  A CTA that finishes a phase early starts the next one as soon as
// its inputs exist, and the data itself says when that is, so there is no
// separate arrival round trip.  Every CTA keeps the residual stream in its
// own shared memory (each computes it identically), so it is never read back.
//
// What this buys over one launch per projection: every warp's weight stream
// (gemv_core.cuh) runs through all the step's projections back to back, so
// the copies of the next projection's weights are already in flight, or in
// shared memory, while the CTA waits for its input; and there is no kernel
// launch, no first-copy latency and no drain between projections.  The GEMV
// and attention arithmetic is the same code the standalone kernels run.
//
// Every wait is bounded: mbarrier waits by iteration count, tagged-word polls
// by time (globaltimer, about 2 s).  A CTA that gives up raises `abort`; the
// others see it in their polls, wait (bounded) for their own copies in
// flight, and leave.
#include <algorithm>

#include "attention_core.cuh"
#include "common.cuh"
#include "gemv_core.cuh"
#include "step.cuh"

namespace rt {

namespace {

using namespace gcore;

constexpr int kStepWarps = 16;
constexpr int kStepNb = 2;           // 32 copies in flight per SM
constexpr int kSlotBytes =  // a ring slot holds a BF16 unit or a copy of tile-major Q4_K units
    kBF16Unit > kTileMajorUnitsPerCopy * kQ4KUnit ? kBF16Unit : kTileMajorUnitsPerCopy * kQ4KUnit;
constexpr int kAttnT = 16;           // cached positions per attention tile

__device__ __forceinline__ uint64_t gtimer() {
    uint64_t t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}

struct StepSmem {
    uint64_t* full;  // [warps][nb]
    uint64_t* jbar;  // [2] job copies landed (jbuf)
    uint64_t* cbar;  // attention arguments landed (abuf)
    Job* jbuf;       // [2] the current and the next projection's Job (bulk copies of the table entries)
    AttnArgs* abuf;  // the current layer's attention arguments
    uint64_t* pbar;
    uint64_t* abar;  // attention tile barrier (kept out of `uni`: see attn_bar_init)
    float* red;
    int* flags;      // 0: this CTA failed, 1: last CTA (argmax), 2: unused, 3: attention copy pending
    GreedySmem* gs;
    float* gpost;    // [hidden]
    float* gpre;     // [hidden]
    float* xs;       // [hidden] residual stream (norm prologues)
    float* wpart;    // [warps][2][16]
    uint2* wse;      // [warps]
    uint8_t* uni;    // planes + xsx of a projection (first the sub-layer output of a norm
                     // prologue), or an attention item
    float2* xsx;
    JobLite* jt;     // [njobs] this CTA's view of every projection (its weight streams' cursor)
    uint8_t* ring;   // [warps][nb][kSlotBytes]
};

__host__ __device__ inline size_t step_carve(uint8_t* base, const StepGeom& g, StepSmem* S) {
    size_t off = 0;
    auto take = [&](size_t bytes, size_t align) -> uint8_t* {
        off = (off + align - 1) / align * align;
        uint8_t* p = base + off;
        off += bytes;
        return p;
    };
    uint8_t* full = take(sizeof(uint64_t) * g.warps * g.nb, 16);
    uint8_t* jbar = take(2 * sizeof(uint64_t), 16);
    uint8_t* cbar = take(sizeof(uint64_t), 16);
    uint8_t* jbuf = take(2 * sizeof(Job), 16);
    uint8_t* abuf = take(sizeof(AttnArgs), 16);
    uint8_t* pbar = take(sizeof(uint64_t), 16);
    uint8_t* abar = take(sizeof(uint64_t), 16);
    uint8_t* red = take(32 * 4, 16);
    uint8_t* flags = take(4 * 4, 16);
    uint8_t* gs = take(sizeof(GreedySmem), 16);
    uint8_t* gpost = take(sizeof(float) * g.hidden, 16);
    uint8_t* gpre = take(sizeof(float) * g.hidden, 16);
    uint8_t* xs = take(sizeof(float) * g.hidden, 16);
    uint8_t* wpart = take(sizeof(float) * g.warps * 2 * 16, 16);
    uint8_t* wse = take(sizeof(uint2) * g.warps, 16);
    const size_t q4 = (planes_bytes(kQ4K, g.kp_max) + 127) / 128 * 128;
    const size_t q4all = q4 + xsx_bytes(kQ4K, g.kp_max), bf = planes_bytes(kBF16, g.kp_lm);
    const size_t proj = q4all > bf ? q4all : bf;
    const size_t att = acore::attn_carve(nullptr, g.head_dim, g.group, kAttnT, nullptr);
    size_t un = proj > att ? proj : att;
    if (un < sizeof(float) * g.hidden) un = sizeof(float) * g.hidden;  // the sub-layer output of a norm prologue
    uint8_t* uni = take(un, 128);
    uint8_t* jt = take(sizeof(JobLite) * g.njobs, 16);
    uint8_t* ring = take(static_cast<size_t>(g.warps) * g.nb * kSlotBytes, 128);
    if (S) {
        S->full = reinterpret_cast<uint64_t*>(full);
        S->jbar = reinterpret_cast<uint64_t*>(jbar);
        S->cbar = reinterpret_cast<uint64_t*>(cbar);
        S->jbuf = reinterpret_cast<Job*>(jbuf);
        S->abuf = reinterpret_cast<AttnArgs*>(abuf);
        S->pbar = reinterpret_cast<uint64_t*>(pbar);
        S->abar = reinterpret_cast<uint64_t*>(abar);
        S->red = reinterpret_cast<float*>(red);
        S->flags = reinterpret_cast<int*>(flags);
        S->gs = reinterpret_cast<GreedySmem*>(gs);
        S->gpost = reinterpret_cast<float*>(gpost);
        S->gpre = reinterpret_cast<float*>(gpre);
        S->xs = reinterpret_cast<float*>(xs);
        S->wpart = reinterpret_cast<float*>(wpart);
        S->wse = reinterpret_cast<uint2*>(wse);
        S->uni = uni;
        S->xsx = reinterpret_cast<float2*>(uni + q4);
        S->jt = reinterpret_cast<JobLite*>(jt);
        S->ring = ring;
    }
    return off;
}

// Stream this warp's units of a projection; on failure drain the warp's copies
// and mark the CTA failed.
template <int KIND, int EPI>
__device__ __forceinline__ void run_units(const Job& j, Stream& st, const JobSmem& JS, const StepParams& P,
                                          int* flags, Greedy& gr, uint32_t out_tag) {
    if (!job_units_run<KIND, EPI, kSplitTile>(j, st, JS, P.scratch, gr, out_tag)) {
        if ((threadIdx.x & 31) == 0) {
            atomicExch(&flags[0], 1);
            if (P.err) atomicExch(P.err, kErrMbarTimeout);
            stream_drain(st);
        }
        __syncwarp();
    }
}

// Raise the grid's abort flag after a wait of this CTA gave up (thread 0).
__device__ __forceinline__ void step_fail(const StepParams& P, int code) {
    if (P.err) atomicCAS(P.err, 0, code);
    atomicExch(P.abort, 1);
}

// Tag of the vector phase k of layer l writes in this launch (never 0).
enum StepVec : int { kVecQkv = 0, kVecAttn = 1, kVecO = 2, kVecH = 3, kVecDown = 4, kVecAttnPart = 5 };

template <int G>
__global__ void __launch_bounds__(kStepWarps * 32, 1) step_kernel(const StepParams P) {
    extern __shared__ __align__(128) uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 127) & ~uintptr_t{127});
    StepSmem S;
    step_carve(smem, P.geom, &S);
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int nb = P.geom.nb;
    acore::AttnSmem AS;
    acore::attn_carve(S.uni, P.geom.head_dim, G, kAttnT, &AS);
    AS.bar = S.abar;
    if (tid == 0) {
        mbar_init(S.pbar, 1);
        mbar_init(&S.jbar[0], 1);
        mbar_init(&S.jbar[1], 1);
        mbar_init(S.cbar, 1);
        acore::attn_bar_init(AS);
        S.flags[0] = S.flags[1] = S.flags[2] = S.flags[3] = 0;
        // The first projection's Job; each phase brings in the next one.
        mbar_arrive_expect_tx(&S.jbar[0], sizeof(Job));
        bulk_g2s_nohint(&S.jbuf[0], &P.jobs[0], sizeof(Job), &S.jbar[0]);
    }
    const int njobs = 4 * P.nlayers + 1;
    // This CTA's table of the jobs, read by the weight streams' cursors (one
    // global read per job and launch instead of one per copy).
    for (int j = tid; j < njobs; j += blockDim.x) S.jt[j] = job_lite(P.jobs[j], blockIdx.x, gridDim.x);
    __syncthreads();
    const JobSmem JS{S.pbar, S.red, S.flags, S.gs, S.gpost, S.gpre, S.uni, S.xsx, S.wpart, S.wse, S.xs,
                     reinterpret_cast<float*>(S.uni)};
    // Every vector a phase produces is published as tagged words; the tag is
    // unique to (launch, layer, vector), so a consumer can tell this launch's
    // words from any earlier ones.  P.sync[0] counts completed launches.
    const uint32_t base = *reinterpret_cast<const volatile uint32_t*>(&P.sync[0]) << 10;
    auto tag_of = [&](int l, int v) { return base + static_cast<uint32_t>(l * 8 + v + 1); };
    const int pos = *P.attn[0].pos;  // this step's position (the same for every layer)
    Stream st;
    stream_start(st, S.full + warp * nb, S.ring + static_cast<size_t>(warp) * nb * kSlotBytes, nb, kSlotBytes, P.jobs,
                 njobs, lane, S.jt);
    if (tid == 0) prefetch_gammas(S.jt[0].K, S.jt[0].g_post, S.jt[0].g_pre, kProEmbedNorm, JS);
    uint32_t pph = 0;  // gamma barrier phase
    int jlast = 0;     // the last Job copy issued (jbuf), and the last attention-argument copy (abuf)
    int alast = -1;
    uint32_t aph = 0;  // attention barrier phases completed
    Greedy gr;
    gr.init();

    // Phase timeline of CTA 0 (tracing; a few stores per phase).
    const bool tr = P.trace && blockIdx.x == 0 && tid == 0;
    auto stamp = [&](int slot) {
        if (tr && slot < kStepTraceLen) P.trace[slot] = gtimer();
    };
    stamp(0);
    bool ok = true;
    // One pass per projection: per layer QKV (then attention), O, gate/up,
    // down.  No grid-wide barrier: each prologue polls the tagged words of
    // its input, which the previous phase's CTAs publish as they finish.  A
    // runtime loop over the phases keeps each stage variant compiled once (the
    // per-layer code path stays small enough for the instruction cache).
#pragma unroll 1
    for (int p = 0; p < 4 * P.nlayers && ok; ++p) {
        const int l = p >> 2, k = p & 3;  // k: 0 QKV, 1 O, 2 gate/up, 3 down
        // This projection's Job, copied into shared memory during the previous
        // phase (its table entry is read once, off the critical path); then
        // start the copy of the next one (its buffer's last reader was the
        // previous phase, which every thread has left).
        if (!mbar_wait(&S.jbar[p & 1], static_cast<uint32_t>(p >> 1) & 1u)) {
            if (tid == 0) step_fail(P, kErrMbarTimeout);
            ok = false;
            break;
        }
        const Job& j = S.jbuf[p & 1];
        if (tid == 0) {
            // the buffers' previous readers (generic proxy) finished before the
            // barrier that ended their phase; order them before the copies
            fence_proxy_async_smem();
            mbar_arrive_expect_tx(&S.jbar[(p + 1) & 1], sizeof(Job));
            bulk_g2s_nohint(&S.jbuf[(p + 1) & 1], &P.jobs[p + 1], sizeof(Job), &S.jbar[(p + 1) & 1]);
            if (k == 0) {
                // this layer's attention arguments (read after the QKV projection)
                mbar_arrive_expect_tx(S.cbar, sizeof(AttnArgs));
                bulk_g2s_nohint(S.abuf, &P.attn[l], sizeof(AttnArgs), S.cbar);
            }
        }
        jlast = p + 1;
        if (k == 0) alast = l;
        const int slot = 1 + 10 * l + 2 * k + (k ? 1 : 0);
        if (k == 0 && l == 0) {
            job_prologue<kQ4K, kProEmbedNorm>(j, JS, pph);  // the embedding row: no producer to wait for
        } else if (k == 0 || k == 2) {
            // residual update + attention / FFN RMSNorm over the previous down / O output
            ok = ll_prologue_resid_norm<kQ4K>(j, JS, pph, k == 0 ? tag_of(l - 1, kVecDown) : tag_of(l, kVecO), P.abort);
        } else {
            ok = ll_prologue_plain<kQ4K>(j, JS, k == 1 ? tag_of(l, kVecAttn) : tag_of(l, kVecH), P.abort,
                                         cta_x_segments(j, S.jt[p]));
        }
        if (k == 0 || k == 2) {
            pph ^= 1u;
            // the next norm prologue's weights: gate/up's, the next layer's QKV or the LM head's
            if (tid == 0) {
                const JobLite& jn = S.jt[p + 2];
                prefetch_gammas(jn.K, jn.g_post, jn.g_pre, kProResidNorm, JS);
            }
        }
        if (!ok) {
            if (tid == 0) step_fail(P, kErrGridTimeout);
            break;
        }
        stamp(slot);
        const uint32_t out_tag = tag_of(l, k == 0 ? kVecQkv : k == 1 ? kVecO : k == 2 ? kVecH : kVecDown);
        if (k == 2) {
            run_units<kQ4K, kEpiGeluPair>(j, st, JS, P, S.flags, gr, out_tag);
            cta_combine<kEpiGeluPair>(j, JS, gr, out_tag);
        } else {
            run_units<kQ4K, kEpiPlain>(j, st, JS, P, S.flags, gr, out_tag);
            cta_combine<kEpiPlain>(j, JS, gr, out_tag);
        }
        stamp(slot + 1);
        __syncthreads();  // every warp is done with the projection's planes (and S.flags[0] is final)
        if (S.flags[0]) {
            ok = false;
            if (tid == 0) atomicExch(P.abort, 1);
            break;
        }
        if (k != 0) continue;
        // ---- attention (item h, s of this CTA) over the QKV words as they arrive ----
        if (!mbar_wait(S.cbar, static_cast<uint32_t>(l) & 1u)) {
            if (tid == 0) step_fail(P, kErrMbarTimeout);
            ok = false;
            break;
        }
        const AttnArgs& at = *S.abuf;
        const int items = at.nkv * at.nsplit;
        const int h = blockIdx.x / at.nsplit, s = blockIdx.x % at.nsplit;
        if (static_cast<int>(blockIdx.x) < items) {
            const acore::AttnRange R = acore::attn_range(at, h, s, kAttnT, pos);
            if (tid == 0) {
                acore::attn_prefetch(at, R, AS, kAttnT);
                S.flags[3] = R.active && R.ntiles > 0;
            }
            __syncthreads();
            const bool done = acore::attn_run<G, kAttnT, true>(at, h, s, R, AS, aph & 1u, tag_of(l, kVecQkv),
                                                         tag_of(l, kVecAttn), P.abort, tag_of(l, kVecAttnPart));
            if (tid == 0) S.flags[3] = 0;
            if (R.active) aph += static_cast<uint32_t>(R.ntiles);
            if (!done) {
                ok = false;
                if (tid == 0) step_fail(P, kErrGridTimeout);
            }
        }
        __syncthreads();  // the attention item's shared memory is dead before the O planes
        stamp(slot + 2);
    }
    if (ok) {
        // ---- LM head: residual update + final norm, BF16 GEMV, greedy token ----
        const int pl = 4 * P.nlayers;
        const bool jok = mbar_wait(&S.jbar[pl & 1], static_cast<uint32_t>(pl >> 1) & 1u);
        const Job& jl = S.jbuf[pl & 1];
        ok = jok && ll_prologue_resid_norm<kBF16>(jl, JS, pph, tag_of(P.nlayers - 1, kVecDown), P.abort);
        if (!ok) {
            if (tid == 0) step_fail(P, jok ? kErrGridTimeout : kErrMbarTimeout);
        } else {
            run_units<kBF16, kEpiArgmax>(jl, st, JS, P, S.flags, gr, 0u);
            cta_combine<kEpiArgmax>(jl, JS, gr);
            stamp(kStepTraceLen - 2);
            __syncthreads();
            if (S.flags[0]) {
                ok = false;
                if (tid == 0) atomicExch(P.abort, 1);
            } else {
                argmax_finish(jl, JS, gr, false, nullptr);
                stamp(kStepTraceLen - 1);
            }
        }
    }
    if (!ok) {
        // Leaving early: no copy of this CTA may still be landing in shared memory.
        if (lane == 0) stream_drain(st);
        if (tid == 0 && S.flags[3]) (void)mbar_wait(AS.bar, aph & 1u);
        if (tid == 0) {
            // the last Job and attention-argument copies issued (bounded waits;
            // a copy already consumed completes them at once)
            (void)mbar_wait(&S.jbar[jlast & 1], static_cast<uint32_t>(jlast >> 1) & 1u);
            if (alast >= 0) (void)mbar_wait(S.cbar, static_cast<uint32_t>(alast) & 1u);
        }
        __syncthreads();
        return;
    }
    // The last CTA out counts the launch (the next launch's tags) and returns
    // the exit counter to zero.
    __syncthreads();
    if (tid == 0) {
        const uint32_t prev = atomicAdd(&P.sync[1], 1u);
        if (prev == gridDim.x - 1) {
            P.sync[1] = 0u;
            P.sync[0] = P.sync[0] + 1u;
        }
    }
}

template <typename F>
bool dispatch_g(int G, F&& f) {
    switch (G) {
        case 1: f(step_kernel<1>); return true;
        case 2: f(step_kernel<2>); return true;
        case 4: f(step_kernel<4>); return true;
        default: return false;
    }
}

}  // namespace

StepGeom step_geometry(int hidden, int kp_max, int head_dim, int group, int njobs) {
    StepGeom g;
    g.warps = kStepWarps;
    g.njobs = njobs;
    g.nb = kStepNb;
    g.hidden = hidden;
    g.kp_max = kp_max;
    g.kp_lm = (hidden + kBF16SegCols - 1) / kBF16SegCols * kBF16SegCols;
    g.head_dim = head_dim;
    g.group = group;
    // head_dim must fit one thread per column in the attention PV loop.
    const bool fits_threads = head_dim <= kStepWarps * 32 && head_dim % 32 == 0;
    const bool fits_group = group == 1 || group == 2 || group == 4;
    g.smem = step_carve(nullptr, g, nullptr) + 128;
    if (!fits_threads || !fits_group || g.smem > 226 * 1024) g.warps = 0;
    return g;
}

cudaError_t step_prepare(const StepGeom& g) {
    cudaError_t e = cudaErrorInvalidValue;
    dispatch_g(g.group, [&](auto k) {
        e = cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(g.smem));
    });
    return e;
}

int step_max_grid(const StepGeom& g) {
    int dev = 0, sms = 0, per_sm = 0;
    if (cudaGetDevice(&dev) != cudaSuccess) return 0;
    if (cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess) return 0;
    dispatch_g(g.group, [&](auto k) {
        if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, k, g.warps * 32, g.smem) != cudaSuccess) per_sm = 0;
    });
    cudaGetLastError();
    return sms * std::min(per_sm, 1);
}

cudaError_t step_launch(const StepParams& p, const StepGeom& g, int grid, cudaStream_t s) {
    cudaError_t err = cudaErrorInvalidValue;
    dispatch_g(g.group, [&](auto k) {
        cudaLaunchConfig_t cfg = {};
        cfg.gridDim = dim3(grid);
        cfg.blockDim = dim3(g.warps * 32);
        cfg.dynamicSmemBytes = g.smem;
        cfg.stream = s;
        cudaLaunchAttribute attr[1];
        attr[0].id = cudaLaunchAttributeCooperative;
        attr[0].val.cooperative = 1;
        cfg.attrs = attr;
        cfg.numAttrs = 1;
        err = cudaLaunchKernelEx(&cfg, k, p);
    });
    return err;
}

}  // namespace rt

