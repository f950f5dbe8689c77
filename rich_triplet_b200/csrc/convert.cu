// convert.cu -- load-time weight conversions on the GPU, bit-exact with the
// reference crate's CPU code (paths relative to the reference crate root):
//
//   Q4_0 -> Q4_K : GgufFile::decode_q4_0_to_q4mat (src/gguf_loader.rs:282-350),
//                  Q4Mat::dequantize_row_into     (src/autograd2.rs:2390-2410),
//                  Q4KMat::from_q4mat / quantize_block (src/autograd2.rs:1291-1320, 1171-1246)
//   Q6_K -> BF16 : GgufFile::decode_q6k_to_f32   (src/gguf_loader.rs:482-533),
//                  MatBf16::f32_to_bf16            (src/autograd2.rs:709-719)
//
// Bit-exactness rules: every f32 multiply / add / divide is written with the
// explicitly rounded intrinsics (__fmul_rn, __fadd_rn, __fdiv_rn), so no FMA
// contraction happens and each operation rounds once, as in Rust.  Min / max
// reductions are exact in any order.  f16 encoding truncates the mantissa, as
// Q4KMat::f32_to_f16 does; Rust's saturating `as u8` is restated exactly.
#include <stdint.h>

#include "common.cuh"
#include "convert.cuh"

namespace rt {

namespace {

__device__ __forceinline__ float f16_bits_to_f32_exact(uint32_t bits) {
    // IEEE half -> float is exact (gguf_loader f16_to_f32, src/gguf_loader.rs:947-976).
    return __half2float(__ushort_as_half(static_cast<unsigned short>(bits)));
}

// Q4KMat::f32_to_f16 (src/autograd2.rs:1090-1115): mantissa truncated.
__device__ __forceinline__ uint32_t f32_to_f16_trunc(float val) {
    const uint32_t bits = __float_as_uint(val);
    const uint32_t sign = (bits >> 16) & 0x8000u;
    const int exp = static_cast<int>((bits >> 23) & 0xFFu);
    const uint32_t mant = bits & 0x7FFFFFu;
    if (exp == 0xFF) return sign | 0x7C00u | (mant >> 13);
    const int new_exp = exp - 127 + 15;
    if (new_exp >= 0x1F) return sign | 0x7C00u;
    if (new_exp <= 0) {
        if (new_exp < -10) return sign;
        const uint32_t m = mant | 0x800000u;
        const uint32_t shift = static_cast<uint32_t>(1 - new_exp) + 13u;
        return sign | (m >> shift);
    }
    return sign | (static_cast<uint32_t>(new_exp) << 10) | (mant >> 13);
}

// Rust `x as u8` for f32: NaN -> 0, saturating, truncation toward zero.
__device__ __forceinline__ uint32_t rust_as_u8(float x) {
    if (x != x) return 0u;
    if (x <= 0.0f) return 0u;
    if (x >= 255.0f) return 255u;
    return __float2uint_rz(x);
}

// MatBf16::f32_to_bf16 (src/autograd2.rs:709-719).
__device__ __forceinline__ uint16_t f32_to_bf16_rne(float v) {
    const uint32_t bits = __float_as_uint(v);
    if (v != v) return static_cast<uint16_t>((bits >> 16) | 0x0040u);
    const uint32_t bias = 0x7FFFu + ((bits >> 16) & 1u);
    return static_cast<uint16_t>((bits + bias) >> 16);
}

// One warp per 256-element Q4_K block.  Lane l holds elements 8l .. 8l+7,
// i.e. 8 values of sub-block j = l / 4.
__global__ void __launch_bounds__(256) q4_0_to_q4k_kernel(const uint8_t* __restrict__ q40, int64_t n_blocks,
                                                        uint8_t* __restrict__ out) {
    const int lane = threadIdx.x & 31;
    const int64_t blk = static_cast<int64_t>(blockIdx.x) * (blockDim.x >> 5) + (threadIdx.x >> 5);
    if (blk >= n_blocks) return;  // warp-uniform

    // --- Q4_0 decode + Q4Mat dequant of this lane's 8 values ---
    // Flat element e = blk*256 + 8*lane + t lies in Q4_0 block e/32 at offset e%32:
    // offsets < 16 are the low nibble of qs[offset], >= 16 the high nibble of
    // qs[offset-16].  The remapped signed nibble (v-8) times the f16 scale.
    const int64_t qb = blk * 8 + lane / 4;
    const uint8_t* src = q40 + qb * 18;
    const float scale = f16_bits_to_f32_exact(static_cast<uint32_t>(src[0]) | (static_cast<uint32_t>(src[1]) << 8));
    float v[8];
    const int off0 = 8 * (lane & 3);
#pragma unroll
    for (int t = 0; t < 8; ++t) {
        const int o = off0 + t;
        const uint32_t byte = src[2 + (o & 15)];
        const uint32_t nib = o < 16 ? (byte & 0x0Fu) : ((byte >> 4) & 0x0Fu);
        const uint32_t enc = (nib - 8u) & 0x0Fu;                 // two's complement nibble
        const int q = enc >= 8u ? static_cast<int>(enc) - 16 : static_cast<int>(enc);
        v[t] = __fmul_rn(static_cast<float>(q), scale);
    }

    // --- quantize_block step 1: per-sub-block min / max ---
    float smin = INFINITY, smax = -INFINITY;
#pragma unroll
    for (int t = 0; t < 8; ++t) {
        if (v[t] < smin) smin = v[t];
        if (v[t] > smax) smax = v[t];
    }
#pragma unroll
    for (int o = 1; o <= 2; o <<= 1) {
        smin = fminf(smin, __shfl_xor_sync(0xffffffffu, smin, o));
        smax = fmaxf(smax, __shfl_xor_sync(0xffffffffu, smax, o));
    }
    float sub_scale, sub_min;
    if (smin >= 0.0f) {
        sub_min = 0.0f;
        sub_scale = smax > 0.0f ? __fdiv_rn(smax, 15.0f) : 0.0f;
    } else {
        sub_min = smin;
        sub_scale = smax > smin ? __fdiv_rn(__fsub_rn(smax, smin), 15.0f) : 0.0f;
    }
    // --- step 2: super-block d, dmin (fold(0.0, f32::max)) ---
    float max_scale = fmaxf(0.0f, sub_scale), max_min = fmaxf(0.0f, -sub_min);
#pragma unroll
    for (int o = 4; o <= 16; o <<= 1) {
        max_scale = fmaxf(max_scale, __shfl_xor_sync(0xffffffffu, max_scale, o));
        max_min = fmaxf(max_min, __shfl_xor_sync(0xffffffffu, max_min, o));
    }
    const float d = max_scale > 0.0f ? __fdiv_rn(max_scale, 63.0f) : 0.0f;
    const float dmin = max_min > 0.0f ? __fdiv_rn(max_min, 63.0f) : 0.0f;
    // --- step 3: 6-bit scale / min of this lane's sub-block ---
    uint32_t sv = 0, mv = 0;
    if (d > 0.0f) {
        const float inv_d = __fdiv_rn(1.0f, d);
        sv = min(rust_as_u8(__fadd_rn(__fmul_rn(sub_scale, inv_d), 0.5f)), 63u);
    }
    if (dmin > 0.0f) {
        const float inv_dmin = __fdiv_rn(1.0f, dmin);
        mv = min(rust_as_u8(__fadd_rn(__fmul_rn(-sub_min, inv_dmin), 0.5f)), 63u);
    }
    // --- step 4: f16 d / dmin; step 6 uses the f16-rounded values ---
    const uint32_t d16 = f32_to_f16_trunc(d), dmin16 = f32_to_f16_trunc(dmin);
    const float d_val = f16_bits_to_f32_exact(d16), dmin_val = f16_bits_to_f32_exact(dmin16);
    const float sc = __fmul_rn(d_val, static_cast<float>(sv));
    const float mn = __fmul_rn(dmin_val, static_cast<float>(mv));
    // --- step 6: 4-bit quants ---
    uint32_t q[8];
#pragma unroll
    for (int t = 0; t < 8; ++t) {
        q[t] = sc > 0.0f ? min(rust_as_u8(__fadd_rn(__fdiv_rn(__fadd_rn(v[t], mn), sc), 0.5f)), 15u) : 0u;
    }
    // Byte qs[32c + p] = low nibble from sub-block 2c | high nibble from 2c+1.
    // Sub-block 2c+1 sits 4 lanes above sub-block 2c.
    uint32_t hi[8];
#pragma unroll
    for (int t = 0; t < 8; ++t) hi[t] = __shfl_down_sync(0xffffffffu, q[t], 4);
    uint8_t* ob = out + blk * 144;
    const int j = lane / 4;
    if ((j & 1) == 0) {
        const int cchunk = j / 2;
        uint8_t* qs = ob + 16 + 32 * cchunk + 8 * (lane & 3);
#pragma unroll
        for (int t = 0; t < 8; ++t) qs[t] = static_cast<uint8_t>(q[t] | (hi[t] << 4));
    }
    // --- step 5: header (pack_scales, src/autograd2.rs:1119-1132) ---
    uint32_t svs[8], mvs[8];
#pragma unroll
    for (int k = 0; k < 8; ++k) {
        svs[k] = __shfl_sync(0xffffffffu, sv, 4 * k);
        mvs[k] = __shfl_sync(0xffffffffu, mv, 4 * k);
    }
    if (lane == 0) {
        ob[0] = static_cast<uint8_t>(d16 & 0xFF);
        ob[1] = static_cast<uint8_t>(d16 >> 8);
        ob[2] = static_cast<uint8_t>(dmin16 & 0xFF);
        ob[3] = static_cast<uint8_t>(dmin16 >> 8);
#pragma unroll
        for (int k = 0; k < 4; ++k) {
            ob[4 + k] = static_cast<uint8_t>((svs[k] & 0x3F) | ((svs[k + 4] & 0x30) << 2));
            ob[8 + k] = static_cast<uint8_t>((mvs[k] & 0x3F) | ((mvs[k + 4] & 0x30) << 2));
            ob[12 + k] = static_cast<uint8_t>((svs[k + 4] & 0x0F) | ((mvs[k + 4] & 0x0F) << 4));
        }
    }
}

// One thread per (block, half, l): the four outputs of one iteration of the
// reference's inner loop.
__global__ void __launch_bounds__(256) q6k_to_bf16_kernel(const uint8_t* __restrict__ q6, int64_t n_elem,
                                                        uint16_t* __restrict__ out) {
    const int64_t tid = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
    const int64_t n_blocks = (n_elem + 255) / 256;
    if (tid >= n_blocks * 64) return;
    const int64_t b = tid / 64;
    const int j = static_cast<int>((tid % 64) / 32);
    const int l = static_cast<int>(tid % 32);
    const uint8_t* blk = q6 + b * 210;
    const uint8_t* ql = blk + j * 64;
    const uint8_t* qh = blk + 128 + j * 32;
    const uint8_t* sc = blk + 192 + j * 8;
    const float d = f16_bits_to_f32_exact(static_cast<uint32_t>(blk[208]) | (static_cast<uint32_t>(blk[209]) << 8));
    const int is = l / 16;
    const int q1 = static_cast<int>((ql[l] & 0x0F) | (((qh[l] >> 0) & 3) << 4)) - 32;
    const int q2 = static_cast<int>((ql[l + 32] & 0x0F) | (((qh[l] >> 2) & 3) << 4)) - 32;
    const int q3 = static_cast<int>((ql[l] >> 4) | (((qh[l] >> 4) & 3) << 4)) - 32;
    const int q4 = static_cast<int>((ql[l + 32] >> 4) | (((qh[l] >> 6) & 3) << 4)) - 32;
    const float s0 = __fmul_rn(d, static_cast<float>(static_cast<int8_t>(sc[is])));
    const float s1 = __fmul_rn(d, static_cast<float>(static_cast<int8_t>(sc[is + 2])));
    const float s2 = __fmul_rn(d, static_cast<float>(static_cast<int8_t>(sc[is + 4])));
    const float s3 = __fmul_rn(d, static_cast<float>(static_cast<int8_t>(sc[is + 6])));
    const int64_t y = b * 256 + j * 128 + l;
    if (y < n_elem) out[y] = f32_to_bf16_rne(__fmul_rn(s0, static_cast<float>(q1)));
    if (y + 32 < n_elem) out[y + 32] = f32_to_bf16_rne(__fmul_rn(s1, static_cast<float>(q2)));
    if (y + 64 < n_elem) out[y + 64] = f32_to_bf16_rne(__fmul_rn(s2, static_cast<float>(q3)));
    if (y + 96 < n_elem) out[y + 96] = f32_to_bf16_rne(__fmul_rn(s3, static_cast<float>(q4)));
}

}  // namespace

cudaError_t q4_0_to_q4k_launch(const uint8_t* q40, int64_t n_q4k_blocks, uint8_t* out, cudaStream_t s) {
    if (n_q4k_blocks <= 0) return cudaSuccess;
    const int warps = 8;
    const int64_t grid = (n_q4k_blocks + warps - 1) / warps;
    q4_0_to_q4k_kernel<<<static_cast<unsigned>(grid), warps * 32, 0, s>>>(q40, n_q4k_blocks, out);
    return cudaGetLastError();
}

cudaError_t q6k_to_bf16_launch(const uint8_t* q6, int64_t n_elem, uint16_t* out, cudaStream_t s) {
    if (n_elem <= 0) return cudaSuccess;
    const int64_t threads = (n_elem + 255) / 256 * 64;
    q6k_to_bf16_kernel<<<static_cast<unsigned>((threads + 255) / 256), 256, 0, s>>>(q6, n_elem, out);
    return cudaGetLastError();
}

namespace {

// One warp per 16-row x 144-byte unit, 16-byte words.
__global__ void q4k_tile_major_kernel(const uint4* in, int64_t rows, int nseg, int parts, uint4* out, int64_t nunits) {
    const int64_t u = (static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x) >> 5;
    const int lane = threadIdx.x & 31;
    if (u >= nunits) return;
    // u = (p * ntiles + t) * nsp + j  ->  block (t, p * nsp + j) of the source
    const int nsp = nseg / parts;
    const int64_t ntiles = (rows + 15) / 16;
    const int64_t v = u / nsp;
    const int j = static_cast<int>(u - v * nsp);
    const int64_t p = v / ntiles, t = v - p * ntiles;
    const int s = static_cast<int>(p) * nsp + j;
    for (int k = lane; k < 16 * 9; k += 32) {
        const int i = k / 9, c = k - 9 * (k / 9);
        const int64_t r = t * 16 + i;
        out[u * 144 + k] = r < rows ? in[(r * nseg + s) * 9 + c] : make_uint4(0u, 0u, 0u, 0u);
    }
}

}  // namespace

cudaError_t q4k_tile_major_launch(const uint8_t* in, int64_t rows, int nseg, int parts, uint8_t* out, cudaStream_t s) {
    if (parts < 1 || nseg % parts != 0) return cudaErrorInvalidValue;
    const int64_t nunits = (rows + 15) / 16 * nseg;
    if (nunits <= 0) return cudaSuccess;
    const int threads = 256;
    const int64_t blocks = (nunits * 32 + threads - 1) / threads;
    q4k_tile_major_kernel<<<static_cast<unsigned>(blocks), threads, 0, s>>>(reinterpret_cast<const uint4*>(in), rows, nseg,
                                                                          parts, reinterpret_cast<uint4*>(out), nunits);
    return cudaGetLastError();
}

}  // namespace rt
