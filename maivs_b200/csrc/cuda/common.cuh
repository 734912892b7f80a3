// Device helpers shared by the MAIVS query kernels (sm_100a).
//
// The whole library is compiled with -fmad=false: the reference never fuses a*b+c (Rust does not
// contract), so every fused multiply-add below is written out with __fmaf_rn exactly where the
// reference's AVX2 kernels use _mm256_fmadd_ps, and nowhere else.
#pragma once

#include <cstdint>
#include <cuda_runtime.h>

namespace maivs {
namespace dev {

constexpr int kWarp = 32;
constexpr uint32_t kNoCell = 0xFFFFFFFFu;

// Orderable key of a float: larger float -> larger unsigned key (NaN-free inputs).
__device__ __forceinline__ uint32_t float_key(float f) {
    uint32_t u = __float_as_uint(f);
    return (u & 0x80000000u) ? ~u : (u | 0x80000000u);
}
__device__ __forceinline__ float key_float(uint32_t k) {
    uint32_t u = (k & 0x80000000u) ? (k & 0x7FFFFFFFu) : ~k;
    return __uint_as_float(u);
}

// Close an 8-lane accumulator the way the reference's hsum_ps does (src/index.rs:58-65):
// ((a0+a4)+(a2+a6)) + ((a1+a5)+(a3+a7)). `l8` is the lane within an aligned group of 8 threads;
// the result is valid in l8 == 0. All 8 lanes of the group must call it.
__device__ __forceinline__ float hsum8_group(float acc, unsigned mask) {
    float s = __fadd_rn(acc, __shfl_xor_sync(mask, acc, 4));
    float t = __fadd_rn(s, __shfl_xor_sync(mask, s, 2));
    return __fadd_rn(t, __shfl_xor_sync(mask, t, 1));
}

// Exact dot_f32_avx2 (src/index.rs:136-152) over n floats by a group of 8 lanes: lane l8 runs the
// FMA chain of SIMD lane l8 (elements l8, l8+8, ...); the scalar tail is a non-fused sequential
// loop in lane 0. Result valid in l8 == 0.
__device__ __forceinline__ float dot_f32_g8(const float* __restrict__ a, const float* __restrict__ b, int n, int l8,
                                            unsigned mask) {
    int full = n & ~7;
    float acc = 0.0f;
    for (int i = l8; i < full; i += 8) acc = __fmaf_rn(a[i], __ldg(b + i), acc);
    float s = hsum8_group(acc, mask);
    if (l8 == 0)
        for (int i = full; i < n; ++i) s = __fadd_rn(s, __fmul_rn(a[i], __ldg(b + i)));
    return s;
}

// Exact dot_f32_u8_avx2 (src/index.rs:278-294): f32 weights x unsigned bytes.
__device__ __forceinline__ float dot_f32_u8_g8(const float* __restrict__ qs, const uint8_t* __restrict__ v, int n,
                                               int l8, unsigned mask) {
    int full = n & ~7;
    float acc = 0.0f;
    for (int i = l8; i < full; i += 8) acc = __fmaf_rn(qs[i], (float)__ldg(v + i), acc);
    float s = hsum8_group(acc, mask);
    if (l8 == 0)
        for (int i = full; i < n; ++i) s = __fadd_rn(s, __fmul_rn(qs[i], (float)__ldg(v + i)));
    return s;
}

// Exact dot_f32_i8_avx2 (src/index.rs:161-177): f32 query x signed bytes.
__device__ __forceinline__ float dot_f32_i8_g8(const float* __restrict__ q, const int8_t* __restrict__ v, int n, int l8,
                                               unsigned mask) {
    int full = n & ~7;
    float acc = 0.0f;
    for (int i = l8; i < full; i += 8) acc = __fmaf_rn(q[i], (float)__ldg(v + i), acc);
    float s = hsum8_group(acc, mask);
    if (l8 == 0)
        for (int i = full; i < n; ++i) s = __fadd_rn(s, __fmul_rn(q[i], (float)__ldg(v + i)));
    return s;
}

// FsQuery::estimate (src/quantize.rs:317-319): delta * sum + bias, not fused.
__device__ __forceinline__ float fs_estimate(float delta, float bias, uint32_t sum) {
    return __fadd_rn(__fmul_rn(delta, (float)sum), bias);
}

__device__ __forceinline__ float clampf(float x, float lo, float hi) { return x < lo ? lo : (x > hi ? hi : x); }

// Reachability bound of one probed cell, cos(max(acos(cs) - r_bound, 0)) (src/index.rs:2176-2180,
// :1482-1486). Each single-precision intermediate is rounded once from a double-precision
// evaluation of the exact function, which is the correctly rounded f32 value except within a few
// ulps of a rounding boundary; the host oracle evaluates the same expression with libm acosf/cosf.
__device__ __forceinline__ float cell_bound(float cs, float r_bound) {
    float ang = (float)acos((double)clampf(cs, -1.0f, 1.0f));
    float diff = __fsub_rn(ang, r_bound);
    float m = diff > 0.0f ? diff : 0.0f;
    return (float)cos((double)m);
}

// sqrt(2 * dim_pad / pi) in f32, as the reference evaluates it (src/index.rs:2172).
__device__ __forceinline__ float fs_norm(int dim_pad) {
    return __fsqrt_rn(__fdiv_rn(__fmul_rn(2.0f, (float)dim_pad), 3.14159274101257324f));
}

}  // namespace dev
}  // namespace maivs
