// The exact rerank (index.rs rerank_exact :1309-1378 with the dots of :136-152, :278-294): the
// streamed f32 kernel, the flattened register gather for byte rows, the top-k selections, the
// merge of cell-range shards' best-k lists, and the centroid re-order dots that share the gather.
#include "dev_common.cuh"
#include "umma.cuh"

namespace maivs {
namespace dev {

namespace {

// ---- exact rerank + top-k (index.rs:1309-1378) --------------------------------------------------------

constexpr int kRerankChunk = 1024;

__device__ __forceinline__ bool better(float sa, uint64_t ia, float sb, uint64_t ib) {
    return sa > sb || (sa == sb && ia < ib);
}

// The 8 SIMD-lane accumulators of the reference's AVX2 dots, kept by one thread, closed with the
// hsum_ps tree (src/index.rs:58-65).
__device__ __forceinline__ float close8(const float a[8]) {
    float s0 = __fadd_rn(a[0], a[4]), s1 = __fadd_rn(a[1], a[5]), s2 = __fadd_rn(a[2], a[6]),
          s3 = __fadd_rn(a[3], a[7]);
    return __fadd_rn(__fadd_rn(s0, s2), __fadd_rn(s1, s3));
}

// dot_f32 (index.rs:136-152) of the shared-memory query with one f32 row, 32 bytes per step.
__device__ __forceinline__ float row_dot_f32(const float* qv, const float* __restrict__ row, int dim) {
    float a[8] = {0, 0, 0, 0, 0, 0, 0, 0};
    const int full = dim & ~7;
    if ((dim & 3) == 0) {
        const float4* r4 = reinterpret_cast<const float4*>(row);
        const float4* q4 = reinterpret_cast<const float4*>(qv);
#pragma unroll 4
        for (int g = 0; g < full / 8; ++g) {
            float4 x0 = __ldg(r4 + 2 * g), x1 = __ldg(r4 + 2 * g + 1);
            float4 y0 = q4[2 * g], y1 = q4[2 * g + 1];
            a[0] = __fmaf_rn(y0.x, x0.x, a[0]);
            a[1] = __fmaf_rn(y0.y, x0.y, a[1]);
            a[2] = __fmaf_rn(y0.z, x0.z, a[2]);
            a[3] = __fmaf_rn(y0.w, x0.w, a[3]);
            a[4] = __fmaf_rn(y1.x, x1.x, a[4]);
            a[5] = __fmaf_rn(y1.y, x1.y, a[5]);
            a[6] = __fmaf_rn(y1.z, x1.z, a[6]);
            a[7] = __fmaf_rn(y1.w, x1.w, a[7]);
        }
    } else {
        for (int i = 0; i < full; ++i) a[i & 7] = __fmaf_rn(qv[i], __ldg(row + i), a[i & 7]);
    }
    float s = close8(a);
    for (int i = full; i < dim; ++i) s = __fadd_rn(s, __fmul_rn(qv[i], __ldg(row + i)));
    return s;
}

// dot_f32_u8 / dot_f32_i8 (index.rs:278-294, :161-177) of the shared-memory weights with one
// byte row, 8 bytes per step.
template <bool kSigned>
__device__ __forceinline__ float row_dot_bytes(const float* qv, const uint8_t* __restrict__ row, int dim) {
    float a[8] = {0, 0, 0, 0, 0, 0, 0, 0};
    const int full = dim & ~7;
    auto cvt = [](uint32_t w, int b) -> float {
        uint32_t v = (w >> (8 * b)) & 0xFFu;
        return kSigned ? (float)(int8_t)v : (float)v;
    };
    if ((dim & 7) == 0) {
        const uint2* r2 = reinterpret_cast<const uint2*>(row);
        const float4* q4 = reinterpret_cast<const float4*>(qv);
#pragma unroll 4
        for (int g = 0; g < full / 8; ++g) {
            uint2 w = __ldg(r2 + g);
            float4 y0 = q4[2 * g], y1 = q4[2 * g + 1];
            a[0] = __fmaf_rn(y0.x, cvt(w.x, 0), a[0]);
            a[1] = __fmaf_rn(y0.y, cvt(w.x, 1), a[1]);
            a[2] = __fmaf_rn(y0.z, cvt(w.x, 2), a[2]);
            a[3] = __fmaf_rn(y0.w, cvt(w.x, 3), a[3]);
            a[4] = __fmaf_rn(y1.x, cvt(w.y, 0), a[4]);
            a[5] = __fmaf_rn(y1.y, cvt(w.y, 1), a[5]);
            a[6] = __fmaf_rn(y1.z, cvt(w.y, 2), a[6]);
            a[7] = __fmaf_rn(y1.w, cvt(w.y, 3), a[7]);
        }
    } else {
        for (int i = 0; i < full; ++i) a[i & 7] = __fmaf_rn(qv[i], cvt(__ldg(row + i), 0), a[i & 7]);
    }
    float s = close8(a);
    for (int i = full; i < dim; ++i) s = __fadd_rn(s, __fmul_rn(qv[i], cvt(__ldg(row + i), 0)));
    return s;
}

// One CTA per query, one thread per candidate row; the best k by (score desc, external id asc)
// are kept across chunks of 1024 candidates by a bitonic sort in shared memory.
__global__ void __launch_bounds__(kBS) k_rerank(IndexView ix, const float* __restrict__ Q, QueryEnc e,
                                                const uint32_t* __restrict__ cand, const uint32_t* __restrict__ cand_n,
                                                int cand_cap, int k, int P, uint64_t* ids, float* scores,
                                                uint32_t* out_n) {
    extern __shared__ uint64_t rsm[];
    uint64_t* sid = rsm;                                   // P ids
    float* ssc = reinterpret_cast<float*>(sid + P);        // P scores
    float* qv = ssc + P;                                   // dim (16-byte aligned: P is a power of two >= 1024)
    const int q = blockIdx.x, dim = ix.dim;
    const int n = (int)cand_n[q];
    const float* qsrc = ix.rerank_mode == 1 ? e.rqs + (size_t)q * dim : Q + (size_t)q * dim;
    for (int t = threadIdx.x; t < dim; t += kBS) qv[t] = qsrc[t];
    for (int i = threadIdx.x; i < k; i += kBS) {
        sid[i] = ~0ull;
        ssc[i] = -INFINITY;
    }
    const float base = ix.rerank_mode == 1 ? e.rbase[q] : 0.0f;
    const uint32_t* cq = cand + (size_t)q * cand_cap;
    for (int c0 = 0; c0 < n; c0 += kRerankChunk) {
        const int cn = min(kRerankChunk, n - c0);
        const int Pe = next_pow2(k + cn);
        for (int i = k + threadIdx.x; i < Pe; i += kBS) {
            sid[i] = ~0ull;
            ssc[i] = -INFINITY;
        }
        __syncthreads();
        for (int i = threadIdx.x; i < cn; i += kBS) {
            const uint32_t slot = cq[c0 + i];
            float s;
            if (ix.rerank_mode == 0)
                s = row_dot_f32(qv, ix.vecs_f32 + (size_t)slot * dim, dim);
            else if (ix.rerank_mode == 1)
                s = __fadd_rn(base, row_dot_bytes<false>(qv, ix.rr_u8 + (size_t)slot * dim, dim));
            else
                s = row_dot_bytes<true>(qv, ix.rr_u8 + (size_t)slot * dim, dim);
            sid[k + i] = ix.ext_ids[slot];
            ssc[k + i] = s;
        }
        __syncthreads();
        // bitonic sort of the Pe (score, id) pairs, best first
        for (int kk = 2; kk <= Pe; kk <<= 1) {
            for (int j = kk >> 1; j > 0; j >>= 1) {
                for (int i = threadIdx.x; i < Pe; i += kBS) {
                    int ixj = i ^ j;
                    if (ixj > i) {
                        float sa = ssc[i], sb = ssc[ixj];
                        uint64_t ia = sid[i], ib = sid[ixj];
                        bool first = (i & kk) == 0;
                        bool sw = first ? better(sb, ib, sa, ia) : better(sa, ia, sb, ib);
                        if (sw) {
                            ssc[i] = sb;
                            ssc[ixj] = sa;
                            sid[i] = ib;
                            sid[ixj] = ia;
                        }
                    }
                }
                __syncthreads();
            }
        }
    }
    __syncthreads();
    const int m = min(k, n);
    for (int i = threadIdx.x; i < k; i += kBS) {
        bool v = i < m;
        ids[(size_t)q * k + i] = v ? sid[i] : ~0ull;
        scores[(size_t)q * k + i] = v ? ssc[i] : -INFINITY;
    }
    if (threadIdx.x == 0) out_n[q] = (uint32_t)m;
}

// Best k of each query's scored candidates by (score desc, external id asc), chunks of 1024
// merged by a bitonic sort in shared memory (same order rule as k_rerank).
__global__ void __launch_bounds__(kBS) k_topk(IndexView ix, const uint32_t* __restrict__ cand,
                                              const uint32_t* __restrict__ cand_n, const float* __restrict__ sc_in,
                                              int cand_cap, int k, int P, uint64_t* ids, float* scores,
                                              uint32_t* out_n) {
    extern __shared__ uint64_t tsh[];
    uint64_t* sid = tsh;
    float* ssc = reinterpret_cast<float*>(sid + P);
    const int q = blockIdx.x;
    const int n = (int)cand_n[q];
    for (int i = threadIdx.x; i < k; i += kBS) {
        sid[i] = ~0ull;
        ssc[i] = -INFINITY;
    }
    for (int c0 = 0; c0 < n; c0 += kRerankChunk) {
        const int cn = min(kRerankChunk, n - c0);
        const int Pe = next_pow2(k + cn);
        for (int i = threadIdx.x; i < Pe - k; i += kBS) {
            const bool v = i < cn;
            sid[k + i] = v ? ix.ext_ids[cand[(size_t)q * cand_cap + c0 + i]] : ~0ull;
            ssc[k + i] = v ? sc_in[(size_t)q * cand_cap + c0 + i] : -INFINITY;
        }
        __syncthreads();
        for (int kk = 2; kk <= Pe; kk <<= 1) {
            for (int j = kk >> 1; j > 0; j >>= 1) {
                for (int i = threadIdx.x; i < Pe; i += kBS) {
                    int ixj = i ^ j;
                    if (ixj > i) {
                        float sa = ssc[i], sb = ssc[ixj];
                        uint64_t ia = sid[i], ib = sid[ixj];
                        bool first = (i & kk) == 0;
                        bool sw = first ? better(sb, ib, sa, ia) : better(sa, ia, sb, ib);
                        if (sw) {
                            ssc[i] = sb;
                            ssc[ixj] = sa;
                            sid[i] = ib;
                            sid[ixj] = ia;
                        }
                    }
                }
                __syncthreads();
            }
        }
    }
    const int m = min(k, n);
    for (int i = threadIdx.x; i < k; i += kBS) {
        bool v = i < m;
        ids[(size_t)q * k + i] = v ? sid[i] : ~0ull;
        scores[(size_t)q * k + i] = v ? ssc[i] : -INFINITY;
    }
    if (threadIdx.x == 0) out_n[q] = (uint32_t)m;
}

// Insert (s, id) into the warp's sorted list (lane j < k holds the j-th best).
__device__ __forceinline__ void warp_insert(float& ms, uint64_t& mid, float s, uint64_t id, int k) {
    const int lane = threadIdx.x & 31;
    const unsigned ahead = __ballot_sync(0xFFFFFFFFu, lane < k && better(ms, mid, s, id));
    const int p = __popc(ahead);
    const float us = __shfl_up_sync(0xFFFFFFFFu, ms, 1);
    const uint64_t uid = __shfl_up_sync(0xFFFFFFFFu, mid, 1);
    if (p < k) {
        if (lane == p) {
            ms = s;
            mid = id;
        } else if (lane > p && lane < k) {
            ms = us;
            mid = uid;
        }
    }
}

// ---- exact rerank: flattened gather into registers ----------------------------------------------
// The candidates of all queries are cut into items of R consecutive rows of one query (R = 16
// for f32 rows, 32 for byte rows); k_rerank_items numbers them (exclusive prefix of
// ceil(cand_n / R) per query) and every warp of a persistent grid takes an equal contiguous run
// of items. Rows are read straight into registers with 128-bit loads at full occupancy, which is
// what a random gather of ~1.5 KB rows needs to run at HBM speed; the warp keeps its query's
// vector in shared memory and prefetches the next item's slots while it scores the current one.
// f32 rows: two lanes per row, lane h running SIMD lanes 4h..4h+3 of the reference's 8-lane FMA
// dot (elements 8i + 4h .. 8i + 4h + 3 at step i), the pair closing it with the hsum_ps tree
// ((a0+a4)+(a2+a6))+((a1+a5)+(a3+a7)). Byte rows: one lane per row running all eight SIMD
// lanes, 16 elements (two steps) per load. The scalar tail is added sequentially, then the SQ8
// base. Scores go to score_out[q * cand_cap + r]; k_topk_warp (k <= 32) or k_topk picks the best
// k of each query.
__global__ void __launch_bounds__(1024) k_rerank_items(const uint32_t* __restrict__ cand_n, int nq, int rows,
                                                       uint32_t* __restrict__ item_off) {
    __shared__ uint32_t wsum[32];
    __shared__ uint32_t carry;
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    if (threadIdx.x == 0) carry = 0;
    __syncthreads();
    for (int q0 = 0; q0 < nq; q0 += 1024) {
        const int q = q0 + threadIdx.x;
        const uint32_t v = q < nq ? (cand_n[q] + rows - 1) / rows : 0u;
        uint32_t x = v;
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
            const uint32_t y = __shfl_up_sync(0xFFFFFFFFu, x, o);
            if (lane >= o) x += y;
        }
        if (lane == 31) wsum[warp] = x;
        __syncthreads();
        if (warp == 0) {
            uint32_t w = wsum[lane];
#pragma unroll
            for (int o = 1; o < 32; o <<= 1) {
                const uint32_t y = __shfl_up_sync(0xFFFFFFFFu, w, o);
                if (lane >= o) w += y;
            }
            wsum[lane] = w;
        }
        __syncthreads();
        const uint32_t before = carry + (warp ? wsum[warp - 1] : 0u) + x - v;
        if (q < nq) item_off[q] = before;
        __syncthreads();
        if (threadIdx.x == 1023) carry = before + v;
        __syncthreads();
    }
    if (threadIdx.x == 0) item_off[nq] = carry;
}

__host__ __device__ constexpr int gather_rows(int mode) { return mode == 0 ? 16 : 32; }


// Rows scored by row_dots: queries (nq x dim, f32), an optional per-query base added after the dot
// (SQ8 rows), and the rows themselves (f32 or bytes).
struct RowSrc {
    int dim;
    const float* qsrc;
    const float* qbase;
    const float* rows_f32;
    const uint8_t* rows_u8;
};

template <int kMode>  // 0: f32 rows, 1: unsigned byte rows + base, 2: signed byte rows
__device__ __forceinline__ void row_dots(const RowSrc& src, const uint32_t* __restrict__ cand,
                                         const uint32_t* __restrict__ cand_n, const uint32_t* __restrict__ item_off,
                                         int nq, int cand_cap, float* __restrict__ score_out) {
    constexpr int R = gather_rows(kMode);
    extern __shared__ __align__(16) float gsm[];
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int dim = src.dim, full8 = dim & ~7, n8 = full8 >> 3;
    float* sq = gsm + (size_t)warp * ((dim + 3) & ~3);
    const long long total = item_off[nq];
    const long long tw = (long long)gridDim.x * (blockDim.x >> 5), gw = (long long)blockIdx.x * (blockDim.x >> 5) + warp;
    const uint32_t i0 = (uint32_t)(total * gw / tw), i1 = (uint32_t)(total * (gw + 1) / tw);
    if (i0 >= i1) return;

    // the query owning item i0: last q with item_off[q] <= i0
    int lo = 0, hi = nq - 1;
    while (lo < hi) {
        const int mid = (lo + hi + 1) >> 1;
        if (item_off[mid] <= i0) lo = mid; else hi = mid - 1;
    }
    int lq = lo;
    uint32_t lq_end = item_off[lq + 1];
    auto advance = [&](uint32_t it, int& q, int& r0) {
        while (it >= lq_end) {
            ++lq;
            lq_end = item_off[lq + 1];
        }
        q = lq;
        r0 = (int)(it - item_off[lq]) * R;
    };
    const int j = kMode == 0 ? lane >> 1 : lane;  // this lane's row within the item
    const int h = lane & 1;
    auto slot_of = [&](int q, int r0) -> uint32_t {
        const int r = r0 + j;
        return r < (int)__ldg(cand_n + q) ? __ldg(cand + (size_t)q * cand_cap + r) : ~0u;
    };
    int q_a, r_a;
    advance(i0, q_a, r_a);
    uint32_t s_a = slot_of(q_a, r_a);
    int cur_q = -1;
    for (uint32_t it = i0; it < i1; ++it) {
        int q_n = 0, r_n = 0;
        uint32_t s_n = ~0u;
        if (it + 1 < i1) {
            advance(it + 1, q_n, r_n);
            s_n = slot_of(q_n, r_n);
        }
        const int q = q_a;
        if (q != cur_q) {  // warp-uniform: stage this query's vector
            __syncwarp();
            const float* qv = src.qsrc + (size_t)q * dim;
            for (int i = lane; i < dim; i += 32) sq[i] = __ldg(qv + i);
            __syncwarp();
            cur_q = q;
        }
        const bool valid = s_a != ~0u;
        float sc = 0.0f;
        if (kMode == 0) {
            const float* row = src.rows_f32 + (size_t)(valid ? s_a : 0u) * dim;
            float a0 = 0.0f, a1 = 0.0f, a2 = 0.0f, a3 = 0.0f;
            if (valid) {
                const float4* rp = reinterpret_cast<const float4*>(row) + h;
                const float4* qp = reinterpret_cast<const float4*>(sq) + h;
#pragma unroll 8
                for (int i = 0; i < n8; ++i) {
                    const float4 xx = __ldg(rp + 2 * i);
                    const float4 qq = qp[2 * i];
                    a0 = __fmaf_rn(qq.x, xx.x, a0);
                    a1 = __fmaf_rn(qq.y, xx.y, a1);
                    a2 = __fmaf_rn(qq.z, xx.z, a2);
                    a3 = __fmaf_rn(qq.w, xx.w, a3);
                }
            }
            const float s0 = __fadd_rn(a0, __shfl_xor_sync(0xFFFFFFFFu, a0, 1));
            const float s1 = __fadd_rn(a1, __shfl_xor_sync(0xFFFFFFFFu, a1, 1));
            const float s2 = __fadd_rn(a2, __shfl_xor_sync(0xFFFFFFFFu, a2, 1));
            const float s3 = __fadd_rn(a3, __shfl_xor_sync(0xFFFFFFFFu, a3, 1));
            sc = __fadd_rn(__fadd_rn(s0, s2), __fadd_rn(s1, s3));
            if (valid && h == 0) {
                for (int i = full8; i < dim; ++i) sc = __fadd_rn(sc, __fmul_rn(sq[i], __ldg(row + i)));
                score_out[(size_t)q * cand_cap + r_a + j] = sc;
            }
        } else if (valid) {
            constexpr bool sgn = kMode == 2;
            const uint8_t* row = src.rows_u8 + (size_t)s_a * dim;
            const uint4* rp = reinterpret_cast<const uint4*>(row);
            const float4* qp = reinterpret_cast<const float4*>(sq);
            float a0 = 0.0f, a1 = 0.0f, a2 = 0.0f, a3 = 0.0f, a4 = 0.0f, a5 = 0.0f, a6 = 0.0f, a7 = 0.0f;
            const int m2 = n8 >> 1;
#pragma unroll 4
            for (int m = 0; m < m2; ++m) {
                const uint4 w = __ldg(rp + m);
                const float4 q0 = qp[4 * m], q1 = qp[4 * m + 1], q2 = qp[4 * m + 2], q3 = qp[4 * m + 3];
                a0 = __fmaf_rn(q0.x, byte_val(w.x, 0, sgn), a0);
                a1 = __fmaf_rn(q0.y, byte_val(w.x, 1, sgn), a1);
                a2 = __fmaf_rn(q0.z, byte_val(w.x, 2, sgn), a2);
                a3 = __fmaf_rn(q0.w, byte_val(w.x, 3, sgn), a3);
                a4 = __fmaf_rn(q1.x, byte_val(w.y, 0, sgn), a4);
                a5 = __fmaf_rn(q1.y, byte_val(w.y, 1, sgn), a5);
                a6 = __fmaf_rn(q1.z, byte_val(w.y, 2, sgn), a6);
                a7 = __fmaf_rn(q1.w, byte_val(w.y, 3, sgn), a7);
                a0 = __fmaf_rn(q2.x, byte_val(w.z, 0, sgn), a0);
                a1 = __fmaf_rn(q2.y, byte_val(w.z, 1, sgn), a1);
                a2 = __fmaf_rn(q2.z, byte_val(w.z, 2, sgn), a2);
                a3 = __fmaf_rn(q2.w, byte_val(w.z, 3, sgn), a3);
                a4 = __fmaf_rn(q3.x, byte_val(w.w, 0, sgn), a4);
                a5 = __fmaf_rn(q3.y, byte_val(w.w, 1, sgn), a5);
                a6 = __fmaf_rn(q3.z, byte_val(w.w, 2, sgn), a6);
                a7 = __fmaf_rn(q3.w, byte_val(w.w, 3, sgn), a7);
            }
            for (int i = 2 * m2; i < n8; ++i) {  // an odd last step (not reached with 16-byte rows)
                const float* qs = sq + 8 * i;
                const uint8_t* xs = row + 8 * i;
                a0 = __fmaf_rn(qs[0], sgn ? (float)(int8_t)xs[0] : (float)xs[0], a0);
                a1 = __fmaf_rn(qs[1], sgn ? (float)(int8_t)xs[1] : (float)xs[1], a1);
                a2 = __fmaf_rn(qs[2], sgn ? (float)(int8_t)xs[2] : (float)xs[2], a2);
                a3 = __fmaf_rn(qs[3], sgn ? (float)(int8_t)xs[3] : (float)xs[3], a3);
                a4 = __fmaf_rn(qs[4], sgn ? (float)(int8_t)xs[4] : (float)xs[4], a4);
                a5 = __fmaf_rn(qs[5], sgn ? (float)(int8_t)xs[5] : (float)xs[5], a5);
                a6 = __fmaf_rn(qs[6], sgn ? (float)(int8_t)xs[6] : (float)xs[6], a6);
                a7 = __fmaf_rn(qs[7], sgn ? (float)(int8_t)xs[7] : (float)xs[7], a7);
            }
            sc = __fadd_rn(__fadd_rn(__fadd_rn(a0, a4), __fadd_rn(a2, a6)), __fadd_rn(__fadd_rn(a1, a5), __fadd_rn(a3, a7)));
            for (int i = full8; i < dim; ++i)
                sc = __fadd_rn(sc, __fmul_rn(sq[i], sgn ? (float)(int8_t)row[i] : (float)row[i]));
            if (kMode == 1) sc = __fadd_rn(__ldg(src.qbase + q), sc);
            score_out[(size_t)q * cand_cap + r_a + j] = sc;
        }
        q_a = q_n;
        r_a = r_n;
        s_a = s_n;
    }
}


// Exact rerank rows (index.rs:1309-1378): score_out[q * cand_cap + r] for every candidate.
template <int kMode>
__global__ void __launch_bounds__(256) k_rerank_gather(RowSrc src, const uint32_t* __restrict__ cand,
                                                       const uint32_t* __restrict__ cand_n,
                                                       const uint32_t* __restrict__ item_off, int nq, int cand_cap,
                                                       float* __restrict__ score_out) {
    row_dots<kMode>(src, cand, cand_n, item_off, nq, cand_cap, score_out);
}

// ---- exact f32 rerank, streamed through shared memory --------------------------------------------
// Each CTA walks a contiguous range of the flattened candidate items (k_rerank_items numbering,
// 16 rows an item) in stages of two items (32 rows). Lanes 0-3 of every warp each move one row of
// a stage with a bulk copy (cp.async.bulk, completion counted on the stage's mbarrier), so the
// gather is issued by the copy engine as whole rows, kS stages in flight. Then 8 threads own a
// row: thread c runs the chain of elements c, c + 8, c + 16, ... (the eight FMA chains of
// row_dots, same order, the query's chain held in registers) and shuffles combine them as
// ((c0 + c4) + (c2 + c6)) + ((c1 + c5) + (c3 + c7)). Every mbarrier wait is bounded: on a timeout
// the CTA sets *err, waits (bounded) for the copies it has in flight and returns.
constexpr int kStreamRows = 32;
constexpr size_t kStreamSmemMax = 222 * 1024;
constexpr size_t kStreamSmemSM = 228 * 1024;  // shared memory of one SM (per CTA: 1 KB reserved, 1.25 KB static)

__device__ __forceinline__ void bulk_row_copy(void* smem_dst, const void* gsrc, uint32_t bytes, uint64_t* bar) {
    asm volatile(
        "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];\n" ::"r"(
            umma::smem_addr(smem_dst)),
        "l"(gsrc), "r"(bytes), "r"(umma::smem_addr(bar))
        : "memory");
}
__device__ __forceinline__ void bar_arrive_expect(uint64_t* bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;\n" ::"r"(umma::smem_addr(bar)), "r"(bytes)
                 : "memory");
}

// The query holding item `it`: the last q with item_off[q] <= it (queries without items are
// skipped because the next one starts at the same offset).
__device__ __forceinline__ int query_of_item(const uint32_t* item_off, int nq, uint32_t it) {
    int lo = 0, hi = nq - 1;
    while (lo < hi) {
        const int mid = (lo + hi + 1) >> 1;
        if (item_off[mid] <= it) lo = mid; else hi = mid - 1;
    }
    return lo;
}

// Exclusive prefix over queries of ceil(cand_n / 16) into out[0..nq], out[nq] the total (the
// numbering of k_rerank_items), computed by one 256-thread CTA.
__device__ void block_items_prefix(const uint32_t* __restrict__ cand_n, int nq, uint32_t* out) {
    using BS = cub::BlockScan<uint32_t, 256>;
    __shared__ typename BS::TempStorage tmp;
    __shared__ uint32_t carry;
    if (threadIdx.x == 0) carry = 0;
    __syncthreads();
    for (int base = 0; base < nq; base += 256) {
        const int q = base + (int)threadIdx.x;
        const uint32_t v = q < nq ? (__ldg(cand_n + q) + 15u) / 16u : 0u;
        uint32_t ex, agg;
        BS(tmp).ExclusiveSum(v, ex, agg);
        const uint32_t c = carry;
        if (q < nq) out[q] = c + ex;
        __syncthreads();
        if (threadIdx.x == 0) carry = c + agg;
        __syncthreads();
    }
    if (threadIdx.x == 0) out[nq] = carry;
    __syncthreads();
}

template <int kS, int N8>
__global__ void __launch_bounds__(256, 1) k_rerank_stream(RowSrc src, const uint32_t* __restrict__ cand,
                                                          const uint32_t* __restrict__ cand_n,
                                                          const uint32_t* item_off_g, int nq, int cand_cap,
                                                          int rstride, float* __restrict__ score_out, uint32_t* err) {
    extern __shared__ __align__(128) float rbuf[];
    __shared__ __align__(8) uint64_t full[kS];
    constexpr int R = 16;  // rows an item
    constexpr int dim = N8 * 8;
    constexpr uint32_t row_bytes = dim * 4;
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const size_t stage_floats = (size_t)kStreamRows * rstride;
    // the item numbering: from k_rerank_items, or (item_off_g null) computed here after the stages
    const uint32_t* item_off = item_off_g;
    if (!item_off_g) {
        uint32_t* s_io = reinterpret_cast<uint32_t*>(rbuf + (size_t)kS * stage_floats);
        block_items_prefix(cand_n, nq, s_io);
        item_off = s_io;
    }
    const uint32_t items = item_off[nq];
    const uint32_t nst = (items + 1) >> 1;
    const uint32_t s0 = (uint32_t)((unsigned long long)nst * blockIdx.x / gridDim.x);
    const uint32_t s1 = (uint32_t)((unsigned long long)nst * (blockIdx.x + 1) / gridDim.x);
    if (s0 >= s1) return;
    if (tid == 0) {
#pragma unroll
        for (int i = 0; i < kS; ++i) umma::bar_init(&full[i], 32);  // lanes 0-3 of the 8 warps
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    __syncthreads();
    const int half = tid >> 7;  // this thread's item of a stage (its copy row and its compute row)
    // monotone cursors over the queries: one for the copies (kS stages ahead), one for compute
    int qm = query_of_item(item_off, nq, min(2 * s0 + half, items - 1));
    int qc = qm;
    auto advance = [&](int& q, uint32_t it) {
        while (item_off[q + 1] <= it) ++q;
    };
    const bool issuer = lane < 4;
    const int crow = warp * 4 + lane;  // the row an issuing lane copies
    // the slot of this lane's row of stage `stg` (~0 where there is no row)
    auto slot_for = [&](uint32_t stg) -> uint32_t {
        const uint32_t it = 2 * stg + half;
        if (!issuer || stg >= s1 || it >= items) return ~0u;
        advance(qm, it);
        const int q = qm;
        const int r = (int)(it - item_off[q]) * R + (crow & (R - 1));
        return r < (int)__ldg(cand_n + q) ? __ldg(cand + (size_t)q * cand_cap + r) : ~0u;
    };
    auto copy = [&](uint32_t stg, uint32_t sl) {
        if (!issuer || stg >= s1) return;
        const int b = (int)((stg - s0) % kS);
        bar_arrive_expect(&full[b], sl != ~0u ? row_bytes : 0u);
        if (sl != ~0u)
            bulk_row_copy(rbuf + (size_t)b * stage_floats + (size_t)crow * rstride,
                          src.rows_f32 + (size_t)sl * dim, row_bytes, &full[b]);
    };
    uint32_t issued = s0;  // stages [s0, issued) have their copies issued
#pragma unroll
    for (int i = 0; i < kS - 1; ++i) copy(s0 + i, slot_for(s0 + i));
    issued = min(s1, s0 + kS - 1);
    uint32_t pslot = slot_for(s0 + kS - 1);
    const int row = tid >> 3, c = tid & 7;
    float qreg[N8];  // this thread's chain of the current query: q[c + 8k]
    int qcur = -1;
    bool bad = false;
    uint32_t st = s0;
    for (; st < s1; ++st) {
        copy(st + kS - 1, pslot);       // its slot was loaded during the previous stage
        if (st + kS - 1 < s1) issued = st + kS;
        pslot = slot_for(st + kS);      // in flight while this stage is summed
        const int b = (int)((st - s0) % kS);
        if (!umma::bar_wait(&full[b], ((st - s0) / kS) & 1u)) bad = true;
        const uint32_t it = 2 * st + half;
        bool valid = false;
        int q = 0, r = 0;
        if (!bad && it < items) {
            advance(qc, it);
            q = qc;
            r = (int)(it - item_off[q]) * R + (row & (R - 1));
            valid = r < (int)__ldg(cand_n + q);
        }
        if (valid && q != qcur) {
            const float* qv = src.qsrc + (size_t)q * dim + c;
#pragma unroll
            for (int k = 0; k < N8; ++k) qreg[k] = __ldg(qv + 8 * k);
            qcur = q;
        }
        float acc = 0.0f;
        if (valid) {
            const float* sr = rbuf + (size_t)b * stage_floats + (size_t)row * rstride + c;
#pragma unroll
            for (int k = 0; k < N8; ++k) acc = __fmaf_rn(qreg[k], sr[8 * k], acc);
        }
        float v = __fadd_rn(acc, __shfl_xor_sync(0xFFFFFFFFu, acc, 4));
        v = __fadd_rn(v, __shfl_xor_sync(0xFFFFFFFFu, v, 2));
        v = __fadd_rn(v, __shfl_xor_sync(0xFFFFFFFFu, v, 1));
        if (valid && c == 0) score_out[(size_t)q * cand_cap + r] = v;
        // every thread is done with this stage's buffer before the next copy into it
        if (__syncthreads_or(bad)) break;
    }
    if (st < s1) {  // a wait ran out: report, then let the copies in flight land before leaving
        if (tid == 0) atomicAdd(err, 1u);
        // from stage st itself: its copies may still be in flight (a completed phase returns at once)
        for (uint32_t t = st; t < issued; ++t) umma::bar_wait(&full[(t - s0) % kS], ((t - s0) / kS) & 1u);
    }
}

// Centroid re-order scores of the routing shortlist (index.rs:1931-1977, :782-800): SQ8 rows with
// the query's base, or f32 rows; the same exact dot as the rerank.
template <int kMode>
__global__ void __launch_bounds__(256) k_rescore_dots(RowSrc src, const uint32_t* __restrict__ cells,
                                                      const uint32_t* __restrict__ cells_n,
                                                      const uint32_t* __restrict__ item_off, int nq, int cap,
                                                      float* __restrict__ score_out) {
    row_dots<kMode>(src, cells, cells_n, item_off, nq, cap, score_out);
}

// Best k (k <= 32) of each query's scored candidates, one warp per query. A chunk of up to 512
// scores is held in registers (16 per lane); the warp finds the k-th largest score key of the
// chunk by a bitwise search over the 32-bit order-preserving keys, loads the external ids of the
// few candidates at or above it (and at or above the running list's k-th), and inserts them into
// the sorted list (lane j holds the j-th best). Order: score desc, external id asc (as k_topk).
__global__ void __launch_bounds__(256) k_topk_warp(IndexView ix, const uint32_t* __restrict__ cand,
                                                   const uint32_t* __restrict__ cand_n,
                                                   const float* __restrict__ sc_in, int nq, int cand_cap, int k,
                                                   uint64_t* ids, float* scores, uint32_t* out_n) {
    constexpr int T = 16;
    const int lane = threadIdx.x & 31;
    const int q = blockIdx.x * (int)(blockDim.x >> 5) + (int)(threadIdx.x >> 5);
    if (q >= nq) return;  // warp-uniform
    const int n = (int)cand_n[q];
    const float* sp = sc_in + (size_t)q * cand_cap;
    const uint32_t* cq = cand + (size_t)q * cand_cap;
    float ms = -INFINITY;
    uint64_t mid = ~0ull;
    int filled = 0;
    for (int c0 = 0; c0 < n; c0 += 32 * T) {
        float s[T];
        uint32_t key[T];
#pragma unroll
        for (int t = 0; t < T; ++t) {
            const int r = c0 + 32 * t + lane;
            s[t] = r < n ? __ldg(sp + r) : -INFINITY;
        }
#pragma unroll
        for (int t = 0; t < T; ++t) {
            const int r = c0 + 32 * t + lane;
            key[t] = r < n ? float_key(s[t] == 0.0f ? 0.0f : s[t]) : 0u;
        }
        uint32_t thr = 0;
        for (int bit = 31; bit >= 0; --bit) {
            const uint32_t c = thr | (1u << bit);
            int cnt = 0;
#pragma unroll
            for (int t = 0; t < T; ++t) cnt += key[t] >= c ? 1 : 0;
            if (__reduce_add_sync(0xFFFFFFFFu, cnt) >= k) thr = c;
        }
        if (filled >= k) {
            const float ts = __shfl_sync(0xFFFFFFFFu, ms, k - 1);
            thr = max(thr, float_key(ts == 0.0f ? 0.0f : ts));
        }
        uint64_t id[T];
#pragma unroll
        for (int t = 0; t < T; ++t) {
            const int r = c0 + 32 * t + lane;
            id[t] = (r < n && key[t] >= thr) ? ix.ext_ids[__ldg(cq + r)] : ~0ull;
        }
#pragma unroll
        for (int t = 0; t < T; ++t) {
            const int r = c0 + 32 * t + lane;
            unsigned m = __ballot_sync(0xFFFFFFFFu, r < n && key[t] >= thr);
            while (m) {
                const int src = __ffs(m) - 1;
                m &= m - 1;
                const float cs = __shfl_sync(0xFFFFFFFFu, s[t], src);
                const uint64_t ci = __shfl_sync(0xFFFFFFFFu, id[t], src);
                warp_insert(ms, mid, cs, ci, k);
                ++filled;
            }
        }
    }
    const int got = min(k, n);
    if (lane < k) {
        const bool v = lane < got;
        ids[(size_t)q * k + lane] = v ? mid : ~0ull;
        scores[(size_t)q * k + lane] = v ? ms : -INFINITY;
    }
    if (lane == 0) out_n[q] = (uint32_t)got;
}

// Cell-range shards: merge the W shards' best-k lists of each query (rank r's block: nq x k ids,
// nq x k scores, nq counts) into the global best k, by score desc, external id asc.
__host__ __device__ inline size_t shard_topk_bytes(int nq, int k) {
    return (((size_t)nq * k * 12 + (size_t)nq * 4) + 15) & ~(size_t)15;
}

__global__ void __launch_bounds__(128) k_merge_topk(const uint8_t* __restrict__ tall, size_t rank_bytes, int W,
                                                    int nq, int k, int P, uint64_t* ids, float* scores,
                                                    uint32_t* out_n) {
    extern __shared__ uint64_t msh[];
    uint64_t* sid = msh;
    float* ssc = reinterpret_cast<float*>(sid + P);
    const int q = blockIdx.x;
    for (int i = threadIdx.x; i < P; i += blockDim.x) {
        sid[i] = ~0ull;
        ssc[i] = -INFINITY;
    }
    __syncthreads();
    unsigned got = 0;
    for (int r = 0; r < W; ++r) {
        const uint8_t* blk = tall + (size_t)r * rank_bytes;
        const uint64_t* ri = reinterpret_cast<const uint64_t*>(blk) + (size_t)q * k;
        const float* rs = reinterpret_cast<const float*>(blk + (size_t)nq * k * 8) + (size_t)q * k;
        const int n = min((int)reinterpret_cast<const uint32_t*>(blk + (size_t)nq * k * 12)[q], k);
        got += (unsigned)n;
        for (int j = threadIdx.x; j < n; j += blockDim.x) {
            sid[r * k + j] = ri[j];
            ssc[r * k + j] = rs[j];
        }
    }
    __syncthreads();
    for (int kk = 2; kk <= P; kk <<= 1) {
        for (int j = kk >> 1; j > 0; j >>= 1) {
            for (int i = threadIdx.x; i < P; i += blockDim.x) {
                const int ixj = i ^ j;
                if (ixj > i) {
                    const float sa = ssc[i], sb = ssc[ixj];
                    const uint64_t ia = sid[i], ib = sid[ixj];
                    const bool first = (i & kk) == 0;
                    if (first ? better(sb, ib, sa, ia) : better(sa, ia, sb, ib)) {
                        ssc[i] = sb;
                        ssc[ixj] = sa;
                        sid[i] = ib;
                        sid[ixj] = ia;
                    }
                }
            }
            __syncthreads();
        }
    }
    const int m = min(k, (int)got);
    for (int i = threadIdx.x; i < k; i += blockDim.x) {
        const bool v = i < m;
        ids[(size_t)q * k + i] = v ? sid[i] : ~0ull;
        scores[(size_t)q * k + i] = v ? ssc[i] : -INFINITY;
    }
    if (threadIdx.x == 0) out_n[q] = (uint32_t)m;
}

}  // namespace

// ---- launchers ----------------------------------------------------------------------------------------

void launch_rescore_dots(const IndexView& ix, const QueryEnc& e, const float* Q, int nq, const uint32_t* sl,
                         const uint32_t* sl_n, int sl_cap, bool use_sq8, float* rs_scores, uint32_t* rs_items,
                         cudaStream_t st) {
    const int mode = use_sq8 ? 1 : 0;
    const void* fn = mode == 1 ? (const void*)k_rescore_dots<1> : (const void*)k_rescore_dots<0>;
    const size_t smem = (size_t)8 * ((ix.dim + 3) & ~3) * sizeof(float);
    set_smem(fn, smem);
    const int sms = sm_count(), per_sm = blocks_per_sm(fn, 256, smem);
    const RowSrc src{ix.dim, use_sq8 ? e.cqs : Q, e.cqbase, ix.cent_f32, ix.cent_sq8};
    {
        Tick tk(kKRerankItems, st);
        k_rerank_items<<<1, 1024, 0, st>>>(sl_n, nq, gather_rows(mode), rs_items);
    }
    {
        Tick tk(kKRescoreDots, st);
        if (mode == 1)
            k_rescore_dots<1><<<sms * per_sm, 256, smem, st>>>(src, sl, sl_n, rs_items, nq, sl_cap, rs_scores);
        else
            k_rescore_dots<0><<<sms * per_sm, 256, smem, st>>>(src, sl, sl_n, rs_items, nq, sl_cap, rs_scores);
    }
}

// ---- centroid re-order over every live cell, as a tiled product ---------------------------------
// With neither a tree nor two-stage codes, route_query scores every live cell (index.rs:1260-1270),
// so every query of the batch has the same shortlist. A CTA takes kRaQ queries x kRaC cells with
// both operands staged in shared memory; each thread owns 2 queries x 4 cells and, for every pair,
// the eight FMA chains of the exact dot (element i on chain i % 8, elements in order), closed as
// ((c0 + c4) + (c2 + c6)) + ((c1 + c5) + (c3 + c7)), the tail added in order, then the SQ8 base:
// the value row_dots computes for the pair. Row strides are padded so the 16 rows a warp reads at
// once fall on distinct banks.
constexpr int kRaQ = 32, kRaC = 64;

template <int kMode>  // 0: f32 centroids with the raw query, 1: SQ8 centroids with the pre-scaled query + base
__global__ void __launch_bounds__(256) k_rescore_all(RowSrc src, const uint32_t* __restrict__ live_list, int nl,
                                                     int nq, int cap, float* __restrict__ score_out) {
    extern __shared__ __align__(16) uint8_t ra_sh[];
    const int dim = src.dim, full8 = dim & ~7, n8 = full8 >> 3;
    const int qs = ((dim + 3) & ~3) + 8;                                   // floats per staged query
    const int rs = kMode == 0 ? (((dim + 3) & ~3) + 8) * 4 : dim + 8;      // bytes per staged row
    float* sq = reinterpret_cast<float*>(ra_sh);
    uint8_t* sr = ra_sh + (size_t)kRaQ * qs * 4;
    const int q0 = blockIdx.x * kRaQ, c0 = blockIdx.y * kRaC;
    const int nqb = min(kRaQ, nq - q0), ncb = min(kRaC, nl - c0);
    for (int i = threadIdx.x; i < kRaQ * dim; i += 256) {
        const int j = i / dim, t = i - j * dim;
        sq[j * qs + t] = j < nqb ? __ldg(src.qsrc + (size_t)(q0 + j) * dim + t) : 0.0f;
    }
    if (kMode == 0) {
        const int w4 = dim >> 2;  // float4 per row
        for (int i = threadIdx.x; i < kRaC * w4; i += 256) {
            const int r = i / w4, t = i - r * w4;
            float4 v = make_float4(0.f, 0.f, 0.f, 0.f);
            if (r < ncb) v = __ldg(reinterpret_cast<const float4*>(src.rows_f32 + (size_t)__ldg(live_list + c0 + r) * dim) + t);
            *reinterpret_cast<float4*>(sr + (size_t)r * rs + 16 * t) = v;
        }
    } else {
        const int w16 = dim >> 4;  // 16-byte words per row
        for (int i = threadIdx.x; i < kRaC * w16; i += 256) {
            const int r = i / w16, t = i - r * w16;
            uint4 v = make_uint4(0u, 0u, 0u, 0u);
            if (r < ncb) v = __ldg(reinterpret_cast<const uint4*>(src.rows_u8 + (size_t)__ldg(live_list + c0 + r) * dim) + t);
            uint2* d = reinterpret_cast<uint2*>(sr + (size_t)r * rs + 16 * t);
            d[0] = make_uint2(v.x, v.y);
            d[1] = make_uint2(v.z, v.w);
        }
    }
    __syncthreads();
    const int qa = 2 * (threadIdx.x >> 4), cb = threadIdx.x & 15;  // queries qa, qa + 1; cells cb + 16 u
    float acc[2][4][8];
#pragma unroll
    for (int a = 0; a < 2; ++a)
#pragma unroll
        for (int u = 0; u < 4; ++u)
#pragma unroll
            for (int l = 0; l < 8; ++l) acc[a][u][l] = 0.0f;
    for (int m = 0; m < n8; ++m) {
        float qv[2][8];
#pragma unroll
        for (int a = 0; a < 2; ++a) {
            const float4 x = *reinterpret_cast<const float4*>(sq + (qa + a) * qs + 8 * m);
            const float4 y = *reinterpret_cast<const float4*>(sq + (qa + a) * qs + 8 * m + 4);
            qv[a][0] = x.x; qv[a][1] = x.y; qv[a][2] = x.z; qv[a][3] = x.w;
            qv[a][4] = y.x; qv[a][5] = y.y; qv[a][6] = y.z; qv[a][7] = y.w;
        }
#pragma unroll
        for (int u = 0; u < 4; ++u) {
            float rv[8];
            const uint8_t* rp = sr + (size_t)(cb + 16 * u) * rs;
            if (kMode == 0) {
                const float4 x = *reinterpret_cast<const float4*>(rp + 32 * m);
                const float4 y = *reinterpret_cast<const float4*>(rp + 32 * m + 16);
                rv[0] = x.x; rv[1] = x.y; rv[2] = x.z; rv[3] = x.w;
                rv[4] = y.x; rv[5] = y.y; rv[6] = y.z; rv[7] = y.w;
            } else {
                const uint2 w = *reinterpret_cast<const uint2*>(rp + 8 * m);
#pragma unroll
                for (int l = 0; l < 4; ++l) {
                    rv[l] = byte_val(w.x, l, false);
                    rv[4 + l] = byte_val(w.y, l, false);
                }
            }
#pragma unroll
            for (int a = 0; a < 2; ++a)
#pragma unroll
                for (int l = 0; l < 8; ++l) acc[a][u][l] = __fmaf_rn(qv[a][l], rv[l], acc[a][u][l]);
        }
    }
#pragma unroll
    for (int a = 0; a < 2; ++a) {
        const int q = qa + a;
        if (q >= nqb) continue;
#pragma unroll
        for (int u = 0; u < 4; ++u) {
            const int c = cb + 16 * u;
            if (c >= ncb) continue;
            const float* v = acc[a][u];
            float sc = __fadd_rn(__fadd_rn(__fadd_rn(v[0], v[4]), __fadd_rn(v[2], v[6])),
                                 __fadd_rn(__fadd_rn(v[1], v[5]), __fadd_rn(v[3], v[7])));
            const uint8_t* rp = sr + (size_t)c * rs;
            for (int i = full8; i < dim; ++i) {
                const float x = kMode == 0 ? reinterpret_cast<const float*>(rp)[i] : (float)rp[i];
                sc = __fadd_rn(sc, __fmul_rn(sq[q * qs + i], x));
            }
            if (kMode == 1) sc = __fadd_rn(__ldg(src.qbase + q0 + q), sc);
            score_out[(size_t)(q0 + q) * cap + c0 + c] = sc;
        }
    }
}

bool launch_rescore_all(const IndexView& ix, const QueryEnc& e, const float* Q, int nq, bool use_sq8, int cap,
                        float* rs_scores, cudaStream_t st) {
    const int dim = ix.dim, nl = ix.n_live_cells;
    if (nq <= 0 || nl <= 0) return false;
    if (use_sq8 ? dim % 16 != 0 : dim % 4 != 0) return false;
    const size_t qb = (size_t)kRaQ * (((dim + 3) & ~3) + 8) * 4;
    const size_t rb = (size_t)kRaC * (use_sq8 ? dim + 8 : (((dim + 3) & ~3) + 8) * 4);
    const size_t smem = qb + rb;
    if (smem > 220 * 1024) return false;
    const void* fn = use_sq8 ? (const void*)k_rescore_all<1> : (const void*)k_rescore_all<0>;
    set_smem(fn, smem);
    const RowSrc src{dim, use_sq8 ? e.cqs : Q, e.cqbase, ix.cent_f32, ix.cent_sq8};
    const dim3 grid((nq + kRaQ - 1) / kRaQ, (nl + kRaC - 1) / kRaC);
    Tick tk(kKRescoreDots, st);
    if (use_sq8)
        k_rescore_all<1><<<grid, 256, smem, st>>>(src, ix.live_list, nl, nq, cap, rs_scores);
    else
        k_rescore_all<0><<<grid, 256, smem, st>>>(src, ix.live_list, nl, nq, cap, rs_scores);
    return true;
}

void launch_merge_topk(const uint8_t* tall, size_t rank_bytes, int W, int nq, int k, uint64_t* ids, float* scores,
                       uint32_t* out_n, cudaStream_t st) {
    if (nq <= 0) return;
    const int P = next_pow2(std::max(W * k, 2));
    const size_t smem = (size_t)P * (sizeof(uint64_t) + sizeof(float));
    set_smem((const void*)k_merge_topk, smem);
    Tick tk(kKMergeTopk, st);
    k_merge_topk<<<nq, 128, smem, st>>>(tall, rank_bytes, W, nq, k, P, ids, scores, out_n);
}

size_t shard_topk_block_bytes(int nq, int k) { return shard_topk_bytes(nq, k); }

void launch_rerank(const IndexView& ix, const float* Q, const QueryEnc& e, int nq, const uint32_t* cand,
                   const uint32_t* cand_n, int cand_cap, int k, uint64_t* ids, float* scores, uint32_t* out_n,
                   float* score_scratch, uint32_t* item_scratch, uint32_t* err, cudaStream_t st) {
    if (nq <= 0) return;
    const int row_bytes = ix.rerank_mode == 0 ? ix.dim * 4 : ix.dim;
    if (row_bytes % 16 == 0 && score_scratch && item_scratch && k <= 4096) {
        const void* fn = ix.rerank_mode == 0   ? (const void*)k_rerank_gather<0>
                         : ix.rerank_mode == 1 ? (const void*)k_rerank_gather<1>
                                               : (const void*)k_rerank_gather<2>;
        const size_t smem = (size_t)8 * ((ix.dim + 3) & ~3) * sizeof(float);
        set_smem(fn, smem);
        const int sms = sm_count();
        const int grid = sms * blocks_per_sm(fn, 256, smem);
        const RowSrc src{ix.dim, ix.rerank_mode == 1 ? e.rqs : Q, e.rbase, ix.vecs_f32, ix.rr_u8};
        // f32 rows of 384 or 768 dimensions: the streamed kernel (the query chain in registers)
        const int rstride = ix.dim + ((8 - ix.dim % 32) + 32) % 32;  // rows of a warp on distinct banks
        const size_t stage_bytes = (size_t)kStreamRows * rstride * sizeof(float);
        const void* sf = nullptr;
        int stages = 0;
        int per_sm = 1;  // CTAs of the streamed kernel per SM
        if (ix.rerank_mode == 0 && ix.dim == 384) {
            // two CTAs per SM of two stages each: one CTA's sums overlap the other's copies
            sf = (const void*)k_rerank_stream<2, 48>;
            stages = 2;
            per_sm = 2;
        } else if (ix.rerank_mode == 0 && ix.dim == 768) {
            sf = (const void*)k_rerank_stream<2, 96>;
            stages = 2;
        }
        // the item numbering goes into the stream kernel's shared memory when it fits beside the stages
        // (of per_sm CTAs on one SM)
        const size_t items_bytes = ((size_t)nq + 1) * sizeof(uint32_t);
        const bool local_items =
            sf && (size_t)per_sm * ((size_t)stages * stage_bytes + items_bytes + 2560) <= kStreamSmemSM;
        if (!local_items) {
            Tick tk(kKRerankItems, st);
            k_rerank_items<<<1, 1024, 0, st>>>(cand_n, nq, gather_rows(ix.rerank_mode), item_scratch);
        }
        if (sf && (size_t)stages * stage_bytes <= kStreamSmemMax) {
            const size_t ssm = (size_t)stages * stage_bytes + (local_items ? items_bytes : 0);
            const uint32_t* io = local_items ? nullptr : item_scratch;
            set_smem(sf, ssm);
            Tick tk(kKRerank, st);
            if (ix.dim == 384)
                k_rerank_stream<2, 48><<<per_sm * sms, 256, ssm, st>>>(src, cand, cand_n, io, nq, cand_cap,
                                                                       rstride, score_scratch, err);
            else
                k_rerank_stream<2, 96><<<sms, 256, ssm, st>>>(src, cand, cand_n, io, nq, cand_cap, rstride,
                                                              score_scratch, err);
        } else {
            Tick tk(kKRerank, st);
            if (ix.rerank_mode == 0)
                k_rerank_gather<0><<<grid, 256, smem, st>>>(src, cand, cand_n, item_scratch, nq, cand_cap,
                                                            score_scratch);
            else if (ix.rerank_mode == 1)
                k_rerank_gather<1><<<grid, 256, smem, st>>>(src, cand, cand_n, item_scratch, nq, cand_cap,
                                                            score_scratch);
            else
                k_rerank_gather<2><<<grid, 256, smem, st>>>(src, cand, cand_n, item_scratch, nq, cand_cap,
                                                            score_scratch);
        }
        if (k <= 32) {
            Tick tk(kKTopk, st);
            // two queries (warps) a CTA: the CTAs spread over every SM even for small batches
            k_topk_warp<<<(nq + 1) / 2, 64, 0, st>>>(ix, cand, cand_n, score_scratch, nq, cand_cap, k, ids, scores,
                                                     out_n);
            return;
        }
        const int P = next_pow2(k + kRerankChunk);
        const size_t tsm = (size_t)P * (sizeof(uint64_t) + sizeof(float));
        set_smem((const void*)k_topk, tsm);
        Tick tk(kKTopk, st);
        k_topk<<<nq, kBS, tsm, st>>>(ix, cand, cand_n, score_scratch, cand_cap, k, P, ids, scores, out_n);
        return;
    }
    // rows that are not 16-byte multiples (odd dimensions): one CTA per query, rows read in place
    int P = next_pow2(k + kRerankChunk);
    size_t smem = (size_t)P * (sizeof(uint64_t) + sizeof(float)) + (size_t)ix.dim * sizeof(float);
    set_smem((const void*)k_rerank, smem);
    Tick tk(kKRerank, st);
    k_rerank<<<nq, kBS, smem, st>>>(ix, Q, e, cand, cand_n, cand_cap, k, P, ids, scores, out_n);
}

}  // namespace dev
}  // namespace maivs
