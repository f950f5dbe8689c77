// gemv.cu -- the standalone Q4_K / BF16 GEMV kernel (one job per launch) and
// its host-side planning.  The streaming, the tensor-core arithmetic and the
// epilogues live in gemv_core.cuh, shared with the decode-step kernel.
#include <cudaTypedefs.h>  // PFN_cuTensorMapEncodeTiled

#include <algorithm>
#include <cstdio>
#include <mutex>

#include "common.cuh"
#include "gemv.cuh"
#include "gemv_core.cuh"

namespace rt {

namespace {

using namespace gcore;

constexpr int kMaxNb = 8;
constexpr int kCopiesInFlight = 32;  // per SM

struct Smem {
    uint64_t* full;  // [warps][nb] unit landed
    uint64_t* pbar;  // norm weights landed
    float* red;      // [32]
    int* flags;      // [4]: 0 = a wait gave up, 1 = last CTA (argmax)
    GreedySmem* gs;  // greedy epilogue reductions
    Job* job;
    float* gpost;    // [K] post-norm weight (residual-norm prologue)
    float* gpre;     // [K] pre-norm weight (norm prologues)
    float* xs;       // [K] residual stream (norm prologues)
    float* sub;      // [K] sub-layer output (residual-update prologue)
    uint8_t* planes;
    float2* xsx;
    uint8_t* ring;   // [warps][nb][unit_bytes]
};

__host__ __device__ inline size_t carve(uint8_t* base, int kind, int K, int nseg, int warps, int nb, int pro, Smem* S) {
    size_t off = 0;
    auto take = [&](size_t bytes, size_t align) -> uint8_t* {
        off = (off + align - 1) / align * align;
        uint8_t* p = base + off;
        off += bytes;
        return p;
    };
    const int Kp = nseg * seg_cols(kind);
    uint8_t* full = take(sizeof(uint64_t) * warps * nb, 16);
    uint8_t* pbar = take(sizeof(uint64_t), 16);
    uint8_t* red = take(32 * 4, 16);
    uint8_t* flags = take(4 * 4, 16);
    uint8_t* gs = take(sizeof(GreedySmem), 16);
    uint8_t* job = take(sizeof(Job), 16);
    uint8_t* gpost = take(pro == kProResidNorm ? sizeof(float) * K : 0, 16);
    uint8_t* gpre = take(pro != kProPlain ? sizeof(float) * K : 0, 16);
    uint8_t* xs = take(pro == kProPlain ? 0 : sizeof(float) * K, 16);
    uint8_t* sub = take(pro == kProResidNorm ? sizeof(float) * K : 0, 16);
    uint8_t* planes = take(planes_bytes(kind, Kp), 128);
    uint8_t* xsx = take(xsx_bytes(kind, Kp), 16);
    uint8_t* ring = take(static_cast<size_t>(warps) * nb * unit_bytes(kind), 128);
    if (S) {
        S->full = reinterpret_cast<uint64_t*>(full);
        S->pbar = reinterpret_cast<uint64_t*>(pbar);
        S->red = reinterpret_cast<float*>(red);
        S->flags = reinterpret_cast<int*>(flags);
        S->gs = reinterpret_cast<GreedySmem*>(gs);
        S->job = reinterpret_cast<Job*>(job);
        S->gpost = reinterpret_cast<float*>(gpost);
        S->gpre = reinterpret_cast<float*>(gpre);
        S->xs = reinterpret_cast<float*>(xs);
        S->sub = reinterpret_cast<float*>(sub);
        S->planes = planes;
        S->xsx = reinterpret_cast<float2*>(xsx);
        S->ring = ring;
    }
    return off;
}

template <int KIND, int PRO, int EPI>
__global__ void __launch_bounds__(kMaxWarps * 32, 1)
    gemv_kernel(const GemvArgs a, const __grid_constant__ CUtensorMap tmap) {
    extern __shared__ __align__(128) uint8_t smem_raw[];
    // TMA destinations need 128-byte alignment (the plan reserves the slack).
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 127) & ~uintptr_t{127});
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5, nw = blockDim.x >> 5;
    Smem S;
    carve(smem, KIND, a.K, a.nseg, nw, a.nb, PRO, &S);
    if (tid == 0) {
        Job& j = *S.job;
        j = Job{};
        j.tmap = &tmap;
        j.wt = nullptr;  // row-major W, 2-D tensor copies
        j.kind = KIND;
        j.K = a.K;
        j.nseg = a.nseg;
        j.rows = a.rows;
        j.x = a.x;
        j.src = a.src;
        j.resid_in = a.resid_in;
        j.resid_out = a.resid_out;
        j.g_post = a.g_post;
        j.g_pre = a.g_pre;
        j.embed = a.embed;
        j.token = a.token;
        j.embed_scale = a.embed_scale;
        j.eps = a.eps;
        j.y = a.y;
        j.am_slot = a.am_slot;
        j.am_counter = a.am_counter;
        j.token_out = a.token_out;
        j.pos_inout = a.pos_inout;
        j.token_hist = a.token_hist;
        j.fail_token = a.fail_token;
        j.wait_iters = a.wait_iters;
        mbar_init(S.pbar, 1);
        fence_mbar_init();
        S.flags[0] = 0;
        S.flags[1] = 0;
    }
    __syncthreads();
    const Job& job = *S.job;
    JobSmem JS{S.pbar, S.red, S.flags, S.gs, S.gpost, S.gpre, S.planes, S.xsx, nullptr, nullptr, S.xs, S.sub};

    // Each warp's weight stream starts before the wait on the previous kernel
    // (weights are constants), and so do the norm weights.
    const int ubytes = unit_bytes(KIND);
    Stream st;
    stream_start(st, S.full + warp * a.nb, S.ring + static_cast<size_t>(warp) * a.nb * ubytes, a.nb, ubytes, S.job, 1,
                 lane);
    if (tid == 0) prefetch_gammas(job, PRO, JS);
    pdl_launch_dependents();
    pdl_wait();

    job_prologue<KIND, PRO>(job, JS, 0u);
    Greedy gr;
    gr.init();
    const bool ok = job_units_run<KIND, EPI, kSplitGrid>(job, st, JS, SplitScratch{a.part, a.tile_cnt}, gr);
    if (!ok) {
        // A bounded wait gave up: record it, then wait (bounded) for the copies
        // this warp still has in flight before its shared memory goes away.
        if (lane == 0) {
            atomicExch(&S.flags[0], 1);
            stream_drain(st);
        }
        __syncwarp();
    }
    __syncthreads();
    const bool failed = S.flags[0] != 0;
    if (failed && tid == 0 && a.err) atomicExch(a.err, kErrMbarTimeout);
    // The greedy epilogue runs also after a failure: every CTA must still
    // arrive so that the last one can reset the launch's counters.
    if constexpr (EPI == kEpiArgmax) argmax_finish(job, JS, gr, failed, a.tile_cnt);
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

// Dynamic shared memory a CTA may take: the 227 KiB opt-in limit less 1 KiB,
// which leaves room for the kernels' own static shared variables.
constexpr size_t kSmemLimit = 226 * 1024;

}  // namespace

void gemv_prepare() {
    // Raise the dynamic shared-memory limit of every instantiation, outside any
    // stream capture.
    for (int kd : {kQ4K, kBF16})
        for (int pr : {kProPlain, kProResidNorm, kProEmbedNorm})
            for (int ep : {kEpiPlain, kEpiGeluPair, kEpiArgmax})
                dispatch(kd, pr, ep, [&](auto k) {
                    cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(kSmemLimit));
                });
    cudaGetLastError();  // a failure here surfaces as a launch error
}

GemvPlan gemv_plan(int kind, int64_t rows, int K, int pair, int prologue, int epilogue, int num_sms, int ctas_per_sm) {
    GemvPlan p;
    (void)pair;  // tiles are 16 rows, so (gate, up) pairs never straddle tiles
    (void)epilogue;
    if (rows <= 0 || K <= 0 || num_sms <= 0) return p;
    if (kind == kQ4K ? (K % 256) != 0 : (K % 8) != 0) return p;
    const int seg_cols = kind == kQ4K ? kQ4KSegCols : kBF16SegCols;
    const int nseg = (K + seg_cols - 1) / seg_cols;
    const int cps = ctas_per_sm >= 2 ? 2 : 1;
    p.unit_bytes = kind == kQ4K ? kQ4KUnit : kBF16Unit;
    p.box_x = kind == kQ4K ? kQ4KPitch / 8 : kBF16Pitch / 8;
    p.warps = cps == 2 ? kMaxWarps / 2 : kMaxWarps;
    // Ring depth: about 32 TMA copies in flight per SM stream fastest (more
    // outstanding copies slow the stream down), within the CTA's share of
    // shared memory.
    const size_t budget = cps == 2 ? kSmemLimit / 2 : kSmemLimit;
    p.nb = 0;
    size_t smem = 0;
    for (int nb = std::max(2, std::min(kMaxNb, kCopiesInFlight / p.warps)); nb >= 2; --nb) {
        smem = carve(nullptr, kind, K, nseg, p.warps, nb, prologue, nullptr) + 128;
        if (smem <= budget) {
            p.nb = nb;
            break;
        }
    }
    if (p.nb == 0) {
        p.warps = 0;  // does not fit: the caller reports RT_E_SHAPE
        return p;
    }
    p.smem = smem;
    // Every warp gets at least one unit; the split indexes warps with 16 bits
    // and units with 31.  One CTA per SM either way: a half-size CTA leaves the
    // other half of the SM to the next kernel of a PDL chain.
    const int64_t U = ((rows + kTile - 1) / kTile) * nseg;
    if (U >= (int64_t{1} << 31)) {
        p.warps = 0;
        return p;
    }
    int64_t grid = num_sms;
    grid = std::min<int64_t>(grid, (U + p.warps - 1) / p.warps);
    grid = std::max<int64_t>(1, std::min<int64_t>(grid, 65535 / p.warps));
    p.grid = static_cast<int>(grid);
    p.part_floats = grid * p.warps * 2 * kTile;
    p.cnt_words = (rows + kTile - 1) / kTile;
    return p;
}

TmapEncodeFn tmap_encoder() {
    static std::once_flag once;
    static TmapEncodeFn encode = nullptr;
    std::call_once(once, [] {
        cudaDriverEntryPointQueryResult q;
        void* fn = nullptr;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &fn, cudaEnableDefault, &q) != cudaSuccess ||
            q != cudaDriverEntryPointSuccess || !fn) {
            cudaGetLastError();
            return;
        }
        PFN_cuTensorMapEncodeTiled_v12000 f = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(fn);
        encode = f;
    });
    return encode;
}

bool gemv_make_tmap(int kind, const void* w, int64_t rows, int K, const GemvPlan& p, CUtensorMap* out) {
    const TmapEncodeFn encode = tmap_encoder();
    if (!encode) return false;
    const uint64_t row_bytes = kind == kQ4K ? static_cast<uint64_t>(K / 256) * 144 : static_cast<uint64_t>(K) * 2;
    const cuuint64_t dims[2] = {row_bytes / 8, static_cast<cuuint64_t>(rows)};
    const cuuint64_t strides[1] = {row_bytes};
    const cuuint32_t box[2] = {static_cast<cuuint32_t>(p.box_x), static_cast<cuuint32_t>(kTile)};
    const cuuint32_t estr[2] = {1, 1};
    const CUresult r = encode(out, CU_TENSOR_MAP_DATA_TYPE_UINT64, 2, const_cast<void*>(w), dims, strides, box, estr,
                              CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE,
                              CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    return r == CUDA_SUCCESS;
}

cudaError_t gemv_launch(int kind, int prologue, int epilogue, GemvArgs a, const CUtensorMap& tmap, const GemvPlan& p,
                        cudaStream_t s, bool pdl) {
    const int seg_cols = kind == kQ4K ? kQ4KSegCols : kBF16SegCols;
    a.nseg = (a.K + seg_cols - 1) / seg_cols;
    a.nb = p.nb;
    a.unit_bytes = p.unit_bytes;
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
