// gemm.cuh -- Q4_K prefill GEMM on the sm_100a tensor cores (tcgen05).
//
// C[M, N] (f32, row-major) = A[M, K] (bf16, row-major) . dequant(W[N, K])^T
// for a Q4_K weight W of N rows (K a multiple of 256): Q4KMat::matmul_q4k_t
// (src/autograd2.rs:1437-1457; the reference's BLAS path matmul_q4k_t_exact,
// :1507-1625, computes the same product with f32 weights).
#pragma once

#include <stdint.h>

#include <cuda.h>
#include <cuda_runtime.h>

namespace rt {

struct GemmPlan {
    int bm = 0, bn = 0;  // CTA tile (0: the shape is not supported)
    bool wbf16 = false;  // W is bf16 [n, k] instead of Q4_K
    int splits = 1;      // K split across the grid's third dimension
    int kps = 0;         // K columns per split (a multiple of 256)
    dim3 grid;
    size_t smem = 0;
};

// Tile and split for C[m, n] = A[m, k] . W[n, k]^T.  With splits > 1 the
// launch writes `splits` partial products [splits][m][n] for the caller to
// add (sum_parts_launch, or a consumer that adds them as it loads).
GemmPlan gemm_q4k_plan(int64_t m, int64_t n, int k, int num_sms, bool wbf16, bool allow_split);
// Raise the kernels' shared-memory limit on the current device (outside capture).
cudaError_t gemm_q4k_prepare();
// Tensor maps of A (bf16 [m, k], 128-row 128-byte swizzled tiles) and of W:
// raw Q4_K rows ([n, k/256 blocks] of 144 bytes, p.bn rows per copy) or bf16
// [n, k] rows (swizzled like A).  False if the driver refuses.
bool gemm_q4k_tmaps(const void* a, int64_t m, const void* w, int64_t n, int k, const GemmPlan& p, CUtensorMap* tm_a,
                    CUtensorMap* tm_w);
// c: [p.splits][m][n] f32.
cudaError_t gemm_q4k_launch(const CUtensorMap& tm_a, const CUtensorMap& tm_w, float* c, int64_t m, int64_t n, int k,
                            const GemmPlan& p, int* err, cudaStream_t s);
// out[i] = in[i] + in[count + i] + ... (parts vectors of `count`, in order).
cudaError_t sum_parts_launch(const float* in, int parts, int64_t count, float* out, int num_sms, cudaStream_t s);

}  // namespace rt
