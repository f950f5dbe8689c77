// synth.cpp -- deterministic synthetic inputs (host) and the RoPE tables.
//
// Every value is a pure function of (seed, stream, index) through the
// SplitMix64 finaliser, so the bytes do not depend on how the work is split
// across threads, and the same call always reproduces the same tensor.
// Built with -ffp-contract=off: the RoPE angle is evaluated exactly as the
// reference's f32 expression (no fused multiply-add).
#include <math.h>
#include <stdint.h>
#include <string.h>

#include <algorithm>
#include <thread>
#include <vector>

#include "../../include/rt_cuda.h"

namespace {

inline uint64_t mix64(uint64_t z) {
    z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
    z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
    return z ^ (z >> 31);
}

inline uint64_t key_of(uint64_t seed, uint64_t stream) {
    return mix64(seed * 0x9E3779B97F4A7C15ull + mix64(stream + 0x632BE59BD9B4E019ull));
}

inline uint64_t draw(uint64_t key, uint64_t i) { return mix64(key + (i + 1) * 0x9E3779B97F4A7C15ull); }

// Uniform in [0, 1) with 24 random bits.
inline float unit(uint64_t r) { return static_cast<float>(r >> 40) * (1.0f / 16777216.0f); }

// Q4KMat::f32_to_f16 (truncating), the encoder of the reference's Q4_K producer.
uint16_t f32_to_f16_trunc(float val) {
    uint32_t bits;
    memcpy(&bits, &val, 4);
    uint32_t sign = (bits >> 16) & 0x8000u;
    int exp = static_cast<int>((bits >> 23) & 0xFFu);
    uint32_t mant = bits & 0x7FFFFFu;
    if (exp == 0xFF) return static_cast<uint16_t>(sign | 0x7C00u | (mant >> 13));
    int new_exp = exp - 127 + 15;
    if (new_exp >= 0x1F) return static_cast<uint16_t>(sign | 0x7C00u);
    if (new_exp <= 0) {
        if (new_exp < -10) return static_cast<uint16_t>(sign);
        uint32_t m = mant | 0x800000u;
        uint32_t shift = static_cast<uint32_t>(1 - new_exp) + 13u;
        return static_cast<uint16_t>(sign | (m >> shift));
    }
    return static_cast<uint16_t>(sign | (static_cast<uint32_t>(new_exp) << 10) | (mant >> 13));
}

uint16_t f32_to_bf16(float v) {
    uint32_t bits;
    memcpy(&bits, &v, 4);
    if (v != v) return static_cast<uint16_t>((bits >> 16) | 0x0040u);
    return static_cast<uint16_t>((bits + 0x7FFFu + ((bits >> 16) & 1u)) >> 16);
}

template <typename F>
void parallel_for(int64_t n, F&& f) {
    const int64_t min_chunk = 1 << 14;
    unsigned hw = std::thread::hardware_concurrency();
    int64_t nt = std::min<int64_t>(hw ? hw : 1, std::max<int64_t>(1, n / min_chunk));
    if (nt <= 1) {
        f(0, n);
        return;
    }
    std::vector<std::thread> th;
    const int64_t chunk = (n + nt - 1) / nt;
    for (int64_t t = 0; t < nt; ++t) {
        const int64_t a = t * chunk, b = std::min(n, a + chunk);
        if (a >= b) break;
        th.emplace_back([&f, a, b] { f(a, b); });
    }
    for (auto& t : th) t.join();
}

// Standard normal from two uniforms (Box-Muller in double, rounded to f32).
inline float normal_at(uint64_t key, uint64_t i) {
    const uint64_t r1 = draw(key, 2 * i), r2 = draw(key, 2 * i + 1);
    const double u1 = (static_cast<double>(r1 >> 11) + 1.0) * (1.0 / 9007199254740992.0);  // (0, 1]
    const double u2 = static_cast<double>(r2 >> 11) * (1.0 / 9007199254740992.0);
    return static_cast<float>(sqrt(-2.0 * log(u1)) * cos(6.283185307179586 * u2));
}

// Block `blk` (row-major block index of the whole matrix) of the seeded Q4_K
// matrix: BASELINE config 0's distributions.
void synth_q4k_block(uint64_t key, int64_t blk, uint8_t* o) {
    const uint64_t base = static_cast<uint64_t>(blk) * 20;
    const uint64_t r0 = draw(key, base);
    const float d = 1e-3f + 9e-3f * unit(r0);
    const float dmin = 5e-3f * unit(draw(key, base + 1));
    const uint16_t d16 = f32_to_f16_trunc(d), m16 = f32_to_f16_trunc(dmin);
    o[0] = static_cast<uint8_t>(d16 & 0xFF);
    o[1] = static_cast<uint8_t>(d16 >> 8);
    o[2] = static_cast<uint8_t>(m16 & 0xFF);
    o[3] = static_cast<uint8_t>(m16 >> 8);
    // 8 scales + 8 mins, 6 bits each, then pack_scales (src/autograd2.rs:1119-1132).
    const uint64_t r2 = draw(key, base + 2), r3 = draw(key, base + 3);
    uint8_t sv[8], mv[8];
    for (int j = 0; j < 8; ++j) {
        sv[j] = static_cast<uint8_t>((r2 >> (6 * j)) & 63u);
        mv[j] = static_cast<uint8_t>((r3 >> (6 * j)) & 63u);
    }
    for (int j = 0; j < 4; ++j) {
        o[4 + j] = static_cast<uint8_t>((sv[j] & 0x3F) | ((sv[j + 4] & 0x30) << 2));
        o[8 + j] = static_cast<uint8_t>((mv[j] & 0x3F) | ((mv[j + 4] & 0x30) << 2));
        o[12 + j] = static_cast<uint8_t>((sv[j + 4] & 0x0F) | ((mv[j + 4] & 0x0F) << 4));
    }
    for (int w = 0; w < 16; ++w) {
        const uint64_t r = draw(key, base + 4 + w);
        memcpy(o + 16 + 8 * w, &r, 8);
    }
}

}  // namespace

extern "C" {

void rt_synth_q4k(uint64_t seed, uint64_t stream, int64_t rows, int64_t cols, uint8_t* out) {
    const int64_t nblk = rows * (cols / 256);
    const uint64_t key = key_of(seed, stream);
    parallel_for(nblk, [&](int64_t a, int64_t b) {
        for (int64_t blk = a; blk < b; ++blk) synth_q4k_block(key, blk, out + blk * 144);
    });
}

// Rows [row0, row0 + nrows) x columns [col0, col0 + ncols) (multiples of 256)
// of the matrix rt_synth_q4k(seed, stream, rows, cols) makes, as a Q4_K
// matrix of its own: the same bytes as slicing the whole one.
void rt_synth_q4k_slice(uint64_t seed, uint64_t stream, int64_t rows, int64_t cols, int64_t row0, int64_t nrows,
                        int64_t col0, int64_t ncols, uint8_t* out) {
    (void)rows;
    const int64_t nb = cols / 256, b0 = col0 / 256, nbs = ncols / 256;
    const uint64_t key = key_of(seed, stream);
    parallel_for(nrows * nbs, [&](int64_t a, int64_t b) {
        for (int64_t i = a; i < b; ++i) {
            const int64_t r = row0 + i / nbs, c = b0 + i % nbs;
            synth_q4k_block(key, r * nb + c, out + i * 144);
        }
    });
}

void rt_synth_normal_f32(uint64_t seed, uint64_t stream, int64_t n, float mean, float stddev, float* out) {
    const uint64_t key = key_of(seed, stream);
    parallel_for(n, [&](int64_t a, int64_t b) {
        for (int64_t i = a; i < b; ++i) out[i] = mean + stddev * normal_at(key, static_cast<uint64_t>(i));
    });
}

void rt_synth_normal_bf16(uint64_t seed, uint64_t stream, int64_t n, float mean, float stddev, uint16_t* out) {
    const uint64_t key = key_of(seed, stream);
    parallel_for(n, [&](int64_t a, int64_t b) {
        for (int64_t i = a; i < b; ++i) out[i] = f32_to_bf16(mean + stddev * normal_at(key, static_cast<uint64_t>(i)));
    });
}

void rt_synth_tokens(uint64_t seed, uint64_t stream, int64_t n, int32_t vocab, int32_t* out) {
    const uint64_t key = key_of(seed, stream);
    for (int64_t i = 0; i < n; ++i) out[i] = static_cast<int32_t>(draw(key, static_cast<uint64_t>(i)) % static_cast<uint64_t>(vocab));
}

void rt_synth_bytes(uint64_t seed, uint64_t stream, int64_t n, uint8_t* out) {
    const uint64_t key = key_of(seed, stream);
    parallel_for((n + 7) / 8, [&](int64_t a, int64_t b) {
        for (int64_t i = a; i < b; ++i) {
            const uint64_t r = draw(key, static_cast<uint64_t>(i));
            const int64_t m = std::min<int64_t>(8, n - 8 * i);
            memcpy(out + 8 * i, &r, static_cast<size_t>(m));
        }
    });
}

}  // extern "C"

namespace rt {

// cos / sin of angle = (pos * freq_scale) / theta^(2i / head_dim), evaluated in
// f32 with the host libm exactly as apply_rope_at_offset does
// (src/transformer4.rs:2742-2772).  Tables are [cap][head_dim / 2].
void rope_table(float theta, float freq_scale, int head_dim, int cap, float* cos_out, float* sin_out) {
    const int half = head_dim / 2;
    std::vector<float> denom(half);
    for (int i = 0; i < half; ++i) denom[i] = powf(theta, 2.0f * static_cast<float>(i) / static_cast<float>(head_dim));
    for (int p = 0; p < cap; ++p) {
        for (int i = 0; i < half; ++i) {
            const float angle = (static_cast<float>(p) * freq_scale) / denom[i];
            cos_out[static_cast<size_t>(p) * half + i] = cosf(angle);
            sin_out[static_cast<size_t>(p) * half + i] = sinf(angle);
        }
    }
}

}  // namespace rt
