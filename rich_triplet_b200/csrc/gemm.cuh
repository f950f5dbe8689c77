// gemm.cuh -- Q4_K prefill GEMM on the sm_100a tensor cores (tcgen05).
//
// C[M, N] (f32, row-major) = diag(ascale) . A[M, K] (fp16, row-major) .
// dequant(W[N, K])^T for a Q4_K weight W of N rows (K a multiple of 256), or a
// bf16 W [N, K]: Q4KMat::matmul_q4k_t
// (src/autograd2.rs:1437-1457; the reference's BLAS path matmul_q4k_t_exact,
// :1507-1625, computes the same product with f32 weights).
#pragma once

#include <stdint.h>

#include <cuda.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>

namespace rt {

struct GemmPlan {
    int bm = 0, bn = 0;  // CTA tile (0: the shape is not supported)
    bool wbf16 = false;  // W is bf16 [n, k] instead of Q4_K
    int splits = 1;      // K split across the grid's third dimension
    int kps = 0;         // K columns per split (a multiple of 256)
    int arows = 128;     // rows of an A stage (16 / 64 for M up to that: a deeper A/B ring)
    dim3 grid;
    size_t smem = 0;
    // Multi-row GEMV (gemm_rows.cu) instead of the tensor-memory kernel:
    // n8 tiles of A rows (1, 2 or 4; 0: the tcgen05 kernel), CTAs per K part,
    // ring slots per warp.
    int rows_nt = 0, rows_cpp = 0, rows_nb = 0;
};

// Largest M the multi-row GEMV takes.
constexpr int kRowsMaxM = 16;

// Tile and split for C[m, n] = A[m, k] . W[n, k]^T.  With splits > 1 the
// launch writes `splits` partial products [splits][m][n] for the caller to
// add (sum_parts_launch, or a consumer that adds them as it loads).
GemmPlan gemm_q4k_plan(int64_t m, int64_t n, int k, int num_sms, bool wbf16, bool allow_split);
// Raise the kernels' shared-memory limit on the current device (outside capture).
cudaError_t gemm_q4k_prepare();
// Tensor maps of A (fp16 [m, k], 128-row 128-byte swizzled tiles) and of W:
// raw Q4_K rows ([n, k/256 blocks] of 144 bytes, p.bn rows per copy) or bf16
// [n, k] rows (swizzled like A).  False if the driver refuses.
bool gemm_q4k_tmaps(const void* a, int64_t m, const void* w, int64_t n, int k, const GemmPlan& p, CUtensorMap* tm_a,
                    CUtensorMap* tm_w);
// c: [p.splits][m][n] f32; row r of every part is multiplied by ascale[r]
// (null: by 1).  a: the fp16 rows of A that tm_a maps (read directly by the
// multi-row GEMV, which plans with p.rows_nt > 0; 16-byte aligned).
cudaError_t gemm_q4k_launch(const CUtensorMap& tm_a, const CUtensorMap& tm_w, const float* ascale, float* c, int64_t m,
                            int64_t n, int k, const GemmPlan& p, int* err, cudaStream_t s, const uint16_t* a);
// The multi-row GEMV's plan for a Q4_K product with m <= kRowsMaxM (false if
// the shape does not fit it): at most max_parts K parts (p->splits), exactly
// force_parts if that is > 0 and fits.
bool gemm_rows_plan(int64_t m, int64_t n, int k, int num_sms, int max_parts, int force_parts, GemmPlan* p);
cudaError_t gemm_rows_prepare();
// Epilogues of the multi-row GEMV: C as computed, or (one K part, n even) the
// GELU gate of interleaved gate/up rows, c[r][j] = gelu_tanh(C[r][2j]) * C[r][2j+1]
// ([m][n / 2]).
constexpr int kRowsEpiPlain = 0, kRowsEpiGelu = 1;
// a32 != null: A is f32 rows [m][k] (no row scale; a and ascale unused).
cudaError_t gemm_rows_launch(const CUtensorMap& tm_w, const uint16_t* a, const float* ascale, float* c, int64_t m,
                             int64_t n, int k, const GemmPlan& p, int* err, cudaStream_t s, const float* a32 = nullptr,
                             int epi = kRowsEpiPlain);
// A rows for the GEMM from bf16 rows: out[r] = fp16(a[r] * 2^-e_r), scale[r] = 2^e_r.
cudaError_t a_to_f16_launch(const uint16_t* a_bf16, int64_t m, int k, uint16_t* out, float* scale, cudaStream_t s);
// The same from f32 rows.
cudaError_t a_f32_to_f16_launch(const float* a, int64_t m, int k, uint16_t* out, float* scale, cudaStream_t s);
// y[r][c] += bias[c] for m rows of n.
cudaError_t bias_rows_launch(float* y, int64_t m, int64_t n, const float* bias, int num_sms, cudaStream_t s);
// out[i] = in[i] + in[count + i] + ... (parts vectors of `count`, in order).
cudaError_t sum_parts_launch(const float* in, int parts, int64_t count, float* out, int num_sms, cudaStream_t s);

#ifdef __CUDACC__
// Power-of-two scale of a GEMM input row whose largest magnitude is `maxabs`:
// `inv` (= 2^-e) brings that magnitude into [2^14, 2^15), inside fp16's range
// with 11 significant bits for every element within 2^28 of it; `scale` = 2^e
// undoes it exactly.  A zero, non-finite or f32-subnormal maximum gets 1.
__device__ __forceinline__ void row_scale_f16(float maxabs, float* inv, float* scale) {
    const int e = static_cast<int>((__float_as_uint(maxabs) >> 23) & 0xFFu) - 127;  // floor(log2), normal maxabs
    if (!(maxabs > 0.f) || e == 128 || e == -127) {
        *inv = 1.f;
        *scale = 1.f;
        return;
    }
    const int up = min(14 - e, 126);  // 2^up and 2^-up stay normal f32
    *inv = __uint_as_float(static_cast<uint32_t>(127 + up) << 23);
    *scale = __uint_as_float(static_cast<uint32_t>(127 - up) << 23);
}
#endif

}  // namespace rt
