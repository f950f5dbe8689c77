// convert.cuh -- load-time weight conversion kernels (bit-exact with the
// reference CPU code; see convert.cu).
#pragma once

#include <stdint.h>

#include <cuda_runtime.h>

namespace rt {

// GGUF Q4_0 bytes (18 per 32 elements) -> Q4_K blocks (144 per 256 elements).
cudaError_t q4_0_to_q4k_launch(const uint8_t* q40, int64_t n_q4k_blocks, uint8_t* out, cudaStream_t s);
// GGUF Q6_K bytes (210 per 256 elements) -> BF16.
cudaError_t q6k_to_bf16_launch(const uint8_t* q6, int64_t n_elem, uint16_t* out, cudaStream_t s);
// Row-major Q4_K [rows, nseg blocks] -> tile-major, column parts first: with
// nsp = nseg / parts, unit (part p, tile t, block j) = 16 rows x the 144-byte
// block p * nsp + j, at ((p * ntiles + t) * nsp + j) * 2304; rows past `rows`
// are zero.  parts = 1 is the plain tile-major order (unit (t, s) at
// (t * nseg + s) * 2304).  `out` holds ceil(rows / 16) * nseg * 2304 bytes.
// A layout change only.
cudaError_t q4k_tile_major_launch(const uint8_t* in, int64_t rows, int nseg, int parts, uint8_t* out, cudaStream_t s);

}  // namespace rt
