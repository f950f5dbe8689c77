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
    dim3 grid;
    size_t smem = 0;
};

GemmPlan gemm_q4k_plan(int64_t m, int64_t n, int k, int num_sms);
// Raise the kernel's shared-memory limit on the current device (outside capture).
cudaError_t gemm_q4k_prepare();
// Tensor maps of A (bf16 [m, k], 128-row 128-byte swizzled tiles) and of the
// raw Q4_K rows of W ([n, k/256 blocks] of 144 bytes, p.bn rows per copy).
// False if the driver refuses.
bool gemm_q4k_tmaps(const void* a, int64_t m, const void* w, int64_t n, int k, const GemmPlan& p, CUtensorMap* tm_a,
                    CUtensorMap* tm_w);
cudaError_t gemm_q4k_launch(const CUtensorMap& tm_a, const CUtensorMap& tm_w, float* c, int64_t m, int64_t n, int k,
                            const GemmPlan& p, int* err, cudaStream_t s);

}  // namespace rt
