// Host-side arithmetic of the MAIVS index build: randomised Hadamard rotation, 1-bit codes,
// FastScan block packing and the exact-order dot products the build uses.
//
// Every routine here reproduces the reference's floating-point evaluation order bit for bit,
// because the index the GPU searches must be the index the reference would have built:
//   * dot products are 8-lane FMA chains closed by the fixed AVX2 horizontal-sum tree
//     (src/index.rs:58-65 hsum_ps, :136-152 dot_f32_avx2, :278-294 dot_f32_u8_avx2);
//   * every other sum is a plain sequential left fold with separate multiply and add
//     (Rust never contracts a*b+c), so this file must be compiled with -ffp-contract=off.
#pragma once

#include <immintrin.h>

#include <cmath>
#include <cstddef>
#include <cstdint>
#include <cstring>
#include <vector>

namespace maivs {

// ---- rotation (src/quantize.rs:32-163) ---------------------------------------------------------

constexpr int kRounds = 2;  // quantize.rs:34 ROUNDS

// Next power of two >= n, at least 64 (quantize.rs:38-40).
inline size_t pad_dim(size_t n) {
    size_t p = 1;
    while (p < n) p <<= 1;
    return p < 64 ? 64 : p;
}

// Code length in 64-bit words (quantize.rs:50-53).
inline size_t code_words(size_t code_bits, size_t dim_pad) {
    size_t b = code_bits == 0 ? dim_pad : (code_bits < dim_pad ? code_bits : dim_pad);
    size_t w = b / 64;
    return w < 1 ? 1 : w;
}

// +/-1 sign vectors from splitmix64, ROUNDS x dim_pad, row-major (quantize.rs:132-148).
inline std::vector<float> make_signs(size_t dim_pad, uint64_t seed) {
    std::vector<float> out(kRounds * dim_pad);
    uint64_t state = seed;
    for (size_t i = 0; i < out.size(); ++i) {
        state += 0x9E3779B97F4A7C15ull;
        uint64_t z = state;
        z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
        z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
        z ^= z >> 31;
        out[i] = (z & 1) == 0 ? 1.0f : -1.0f;
    }
    return out;
}

// Normalised fast Walsh-Hadamard transform, levels h = 1, 2, 4, ..., n/2, then x *= 1/sqrt(n)
// (quantize.rs:71-126). Each level is a full pass of independent butterflies, so any execution
// order within a level gives the same bits.
inline void fht_inplace(float* a, size_t n) {
    for (size_t h = 1; h < n; h <<= 1) {
        for (size_t i = 0; i < n; i += h << 1) {
            for (size_t j = i; j < i + h; ++j) {
                float x = a[j], y = a[j + h];
                a[j] = x + y;
                a[j + h] = x - y;
            }
        }
    }
    float s = 1.0f / std::sqrt((float)n);
    for (size_t i = 0; i < n; ++i) a[i] *= s;
}

// rotate(): zero-pad, then ROUNDS x (multiply by signs, FHT) (quantize.rs:152-163).
inline void rotate(const float* v, size_t dim, const float* signs, size_t dim_pad, float* out) {
    std::memcpy(out, v, dim * sizeof(float));
    for (size_t i = dim; i < dim_pad; ++i) out[i] = 0.0f;
    for (int r = 0; r < kRounds; ++r) {
        const float* s = signs + (size_t)r * dim_pad;
        for (size_t i = 0; i < dim_pad; ++i) out[i] *= s[i];
        fht_inplace(out, dim_pad);
    }
}

// Sign bits of the first nw*64 rotated coordinates, bit = (x < 0) (quantize.rs:57-67).
inline void pack_signs_trunc(const float* rot, size_t dim_pad, uint64_t* out, size_t nw) {
    for (size_t w = 0; w < nw; ++w) out[w] = 0;
    size_t bits = nw * 64 < dim_pad ? nw * 64 : dim_pad;
    for (size_t i = 0; i < bits; ++i)
        if (rot[i] < 0.0f) out[i >> 6] |= 1ull << (i & 63);
}

inline uint32_t hamming(const uint64_t* a, const uint64_t* b, size_t nw) {
    uint32_t s = 0;
    for (size_t i = 0; i < nw; ++i) s += (uint32_t)__builtin_popcountll(a[i] ^ b[i]);
    return s;
}

// ---- exact-order dot products (src/index.rs:41-343) --------------------------------------------

// ((v0+v4)+(v2+v6)) + ((v1+v5)+(v3+v7)), the hsum_ps tree of index.rs:58-65.
inline float hsum8(__m256 v) {
    __m128 lo = _mm256_castps256_ps128(v);
    __m128 hi = _mm256_extractf128_ps(v, 1);
    __m128 s = _mm_add_ps(lo, hi);
    s = _mm_add_ps(s, _mm_movehl_ps(s, s));
    s = _mm_add_ss(s, _mm_shuffle_ps(s, s, 0x55));
    return _mm_cvtss_f32(s);
}

// dot_f32_avx2 (index.rs:136-152).
inline float dot_f32(const float* a, const float* b, size_t n) {
    __m256 acc = _mm256_setzero_ps();
    size_t i = 0;
    for (; i + 8 <= n; i += 8) acc = _mm256_fmadd_ps(_mm256_loadu_ps(a + i), _mm256_loadu_ps(b + i), acc);
    float s = hsum8(acc);
    for (; i < n; ++i) s += a[i] * b[i];
    return s;
}

// dot_f32_u8_avx2 (index.rs:278-294): f32 weights times unsigned bytes.
inline float dot_f32_u8(const float* qs, const uint8_t* v, size_t n) {
    __m256 acc = _mm256_setzero_ps();
    size_t i = 0;
    for (; i + 8 <= n; i += 8) {
        __m128i b = _mm_loadl_epi64((const __m128i*)(v + i));
        __m256 vf = _mm256_cvtepi32_ps(_mm256_cvtepu8_epi32(b));
        acc = _mm256_fmadd_ps(_mm256_loadu_ps(qs + i), vf, acc);
    }
    float s = hsum8(acc);
    for (; i < n; ++i) s += qs[i] * (float)v[i];
    return s;
}

// dot_f32_i8_avx2 (index.rs:161-177): f32 query times signed bytes.
inline float dot_f32_i8(const float* q, const int8_t* v, size_t n) {
    __m256 acc = _mm256_setzero_ps();
    size_t i = 0;
    for (; i + 8 <= n; i += 8) {
        __m128i b = _mm_loadl_epi64((const __m128i*)(v + i));
        __m256 vf = _mm256_cvtepi32_ps(_mm256_cvtepi8_epi32(b));
        acc = _mm256_fmadd_ps(_mm256_loadu_ps(q + i), vf, acc);
    }
    float s = hsum8(acc);
    for (; i < n; ++i) s += q[i] * (float)v[i];
    return s;
}

// Sequential sum of squares, sqrt, divide in place if > 1e-12 (tree.rs:166-173, index.rs:2787-2794).
inline void normalize(float* v, size_t n) {
    float s = 0.0f;
    for (size_t i = 0; i < n; ++i) s += v[i] * v[i];
    s = std::sqrt(s);
    if (s > 1e-12f)
        for (size_t i = 0; i < n; ++i) v[i] /= s;
}

// Rust f32::round is half away from zero, then clamp and a saturating cast.
inline uint8_t quant_u8(float x) {
    float r = std::round(x);
    if (r < 0.0f) r = 0.0f;
    if (r > 255.0f) r = 255.0f;
    return (uint8_t)r;
}

inline int8_t quant_i8(float x) {
    float r = std::round(x);
    if (r < -127.0f) r = -127.0f;
    if (r > 127.0f) r = 127.0f;
    return (int8_t)r;
}

// ---- FastScan layout (src/quantize.rs:222-265) -------------------------------------------------

constexpr size_t kFsBlock = 32;  // quantize.rs:222 FS_BLOCK

inline size_t fs_block_bytes(size_t nw) { return nw * 64 * kFsBlock / 8; }

inline uint8_t nib(const uint64_t* code, size_t j) { return (uint8_t)((code[j >> 4] >> ((j & 15) * 4)) & 0xF); }

// Interleave up to 32 codes into one block: byte [p*32 + half*16 + i] holds nibble 2p+half of
// lane i (low) and lane i+16 (high); missing lanes are zero (quantize.rs:238-250).
inline void fs_pack_block(const uint64_t* const* codes, size_t ncodes, size_t nw, uint8_t* out) {
    size_t npos = nw * 16;
    for (size_t p = 0; p < npos / 2; ++p)
        for (size_t half = 0; half < 2; ++half) {
            size_t j = 2 * p + half;
            for (size_t i = 0; i < 16; ++i) {
                uint8_t lo = i < ncodes ? nib(codes[i], j) : 0;
                uint8_t hi = i + 16 < ncodes ? nib(codes[i + 16], j) : 0;
                out[p * 32 + half * 16 + i] = (uint8_t)(lo | (hi << 4));
            }
        }
}

}  // namespace maivs
