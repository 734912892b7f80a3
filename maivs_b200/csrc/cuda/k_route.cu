// Query encoding and routing (src/quantize.rs rotate / pack / FsQuery; index.rs route_batch
// :1873-1980 and route_query :1168-1305): the FWHT encoder, the flat Hamming shortlist with its
// counting cut-off, the centroid-tree beam descent and the exact SQ8 / f32 re-order with the
// nucleus cut.
#include "dev_common.cuh"

namespace maivs {
namespace dev {

namespace {

// ---- K1: query encoding ---------------------------------------------------------------------------

__global__ void __launch_bounds__(kBS) k_encode(IndexView ix, const float* __restrict__ Q, QueryEnc e, int want_cqs,
                                                int want_rqs) {
    extern __shared__ float sm[];
    float* rot = sm;
    float* mins = rot + ix.dim_pad;
    const int q = blockIdx.x, dp = ix.dim_pad, dim = ix.dim, npos = ix.npos;
    const float* x = Q + (size_t)q * dim;
    for (int i = threadIdx.x; i < dp; i += kBS) rot[i] = i < dim ? x[i] : 0.0f;
    __syncthreads();
    // rotate(): ROUNDS x (sign flip, normalised FWHT) (quantize.rs:152-163, :71-126)
    const float scale = __fdiv_rn(1.0f, __fsqrt_rn((float)dp));
    for (int r = 0; r < 2; ++r) {
        const float* s = ix.signs + (size_t)r * dp;
        for (int i = threadIdx.x; i < dp; i += kBS) rot[i] = __fmul_rn(rot[i], s[i]);
        __syncthreads();
        for (int h = 1; h < dp; h <<= 1) {
            for (int bt = threadIdx.x; bt < dp / 2; bt += kBS) {
                int i = (bt / h) * (2 * h) + (bt % h);
                float u = rot[i], v = rot[i + h];
                rot[i] = __fadd_rn(u, v);
                rot[i + h] = __fsub_rn(u, v);
            }
            __syncthreads();
        }
        for (int i = threadIdx.x; i < dp; i += kBS) rot[i] = __fmul_rn(rot[i], scale);
        __syncthreads();
    }
    // pack_signs_trunc (quantize.rs:57-67)
    for (int w = threadIdx.x; w < ix.nw; w += kBS) {
        uint64_t bits = 0;
        for (int t = 0; t < 64; ++t) {
            int i = w * 64 + t;
            if (i < dp && rot[i] < 0.0f) bits |= 1ull << t;
        }
        e.qbits[(size_t)q * ix.nw + w] = bits;
    }
    // FsQuery::new (quantize.rs:279-313); npos <= kBS, one position per thread
    float raw[16];
    float lo = INFINITY, hi = -INFINITY;
    const int j = threadIdx.x;
    if (j < npos) {
#pragma unroll
        for (int ev = 0; ev < 16; ++ev) {
            float v = 0.0f;
#pragma unroll
            for (int t = 0; t < 4; ++t) {
                float xv = rot[4 * j + t];
                v = ((ev >> t) & 1) ? __fsub_rn(v, xv) : __fadd_rn(v, xv);
            }
            raw[ev] = v;
            lo = fminf(lo, v);
            hi = fmaxf(hi, v);
        }
        mins[j] = lo;
    }
    float rj = j < npos ? __fsub_rn(hi, lo) : 0.0f;
    using BR = cub::BlockReduce<float, kBS>;
    __shared__ typename BR::TempStorage red;
    float range = BR(red).Reduce(rj, [](float a, float b) { return fmaxf(a, b); });
    __shared__ float s_range;
    if (threadIdx.x == 0) s_range = fmaxf(0.0f, range);
    __syncthreads();
    const float delta = fmaxf(__fdiv_rn(s_range, 255.0f), 1e-12f);
    if (j < npos) {
        uint32_t wv[4] = {0, 0, 0, 0};
#pragma unroll
        for (int ev = 0; ev < 16; ++ev) {
            float qv = roundf(__fdiv_rn(__fsub_rn(raw[ev], lo), delta));
            qv = clampf(qv, 0.0f, 255.0f);
            wv[ev >> 2] |= ((uint32_t)qv) << (8 * (ev & 3));
        }
        uint4* dst = reinterpret_cast<uint4*>(e.lut + ((size_t)q * npos + j) * 16);
        *dst = make_uint4(wv[0], wv[1], wv[2], wv[3]);
    }
    // Sequential sums, each in its own warp: bias (quantize.rs:312), the centroid SQ8 pre-scale
    // base (index.rs:1184-1186) and the rerank SQ8 base (index.rs:1324-1327).
    if (threadIdx.x == 0) {
        float b = 0.0f;
        for (int t = 0; t < npos; ++t) b = __fadd_rn(b, mins[t]);
        e.fs_delta[q] = delta;
        e.fs_bias[q] = b;
    }
    if (want_cqs && threadIdx.x == 32) {
        float b = 0.0f;
#pragma unroll 16
        for (int t = 0; t < dim; ++t) b = __fadd_rn(b, __fmul_rn(__ldg(x + t), __ldg(ix.csq_min + t)));
        e.cqbase[q] = b;
    }
    if (want_rqs && threadIdx.x == 64) {
        float b = 0.0f;
#pragma unroll 16
        for (int t = 0; t < dim; ++t) b = __fadd_rn(b, __fmul_rn(__ldg(x + t), __ldg(ix.sq_min + t)));
        e.rbase[q] = b;
    }
    if (want_cqs)
        for (int t = threadIdx.x; t < dim; t += kBS) e.cqs[(size_t)q * dim + t] = __fmul_rn(x[t], ix.csq_step[t]);
    if (want_rqs)
        for (int t = threadIdx.x; t < dim; t += kBS) e.rqs[(size_t)q * dim + t] = __fmul_rn(x[t], ix.sq_step[t]);
}

// Rotation layout: E = dim_pad / 32 rotated coordinates per lane of warp 0 (lane l holds l*E ..
// l*E+E-1); butterflies of the FWHT with h < E stay inside a lane, h >= E pair lane l with l ^ (h / E),
// every level applying the reference's butterflies (quantize.rs:71-126), so the bits are the same.
// Query encoding with four warps per query: warp 0 rotates (two rounds of sign flip + FWHT in
// registers and shuffles) and packs the sign bits while warps 1 and 2 compute the SQ8 pre-scales
// and their left-to-right base sums; then every thread builds the FastScan table entries of its
// nibble positions (rotated values from shared memory), the range reduction runs over the block,
// and one thread adds the table minima in position order (quantize.rs:57-67, :152-163, :279-313;
// index.rs:1177-1187), every float operation in the reference's order.
template <int E>
__global__ void __launch_bounds__(128) k_encode4(IndexView ix, const float* __restrict__ Q, QueryEnc e, int want_cqs,
                                                int want_rqs) {
    __shared__ float s_v[32 * E];
    __shared__ float s_mins[256];
    __shared__ float s_red[4];
    __shared__ uint32_t s_mask[32];
    __shared__ float s_prod[2][32 * E];  // x[t] * min[t] of the two SQ8 bases
    const int q = blockIdx.x, warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int dp = ix.dim_pad, dim = ix.dim, npos = ix.npos;
    const float* x = Q + (size_t)q * dim;
    if (warp == 0) {
        float v[E];
#pragma unroll
        for (int t = 0; t < E; ++t) {
            const int i = lane * E + t;
            v[t] = i < dim ? __ldg(x + i) : 0.0f;
        }
        const float scale = __fdiv_rn(1.0f, __fsqrt_rn((float)dp));
#pragma unroll
        for (int r = 0; r < 2; ++r) {
            const float* sg = ix.signs + (size_t)r * dp + lane * E;
#pragma unroll
            for (int t = 0; t < E; ++t) v[t] = __fmul_rn(v[t], __ldg(sg + t));
#pragma unroll
            for (int h = 1; h < E; h <<= 1) {
#pragma unroll
                for (int t = 0; t < E; ++t) {
                    if ((t & h) == 0) {
                        const float a = v[t], b = v[t + h];
                        v[t] = __fadd_rn(a, b);
                        v[t + h] = __fsub_rn(a, b);
                    }
                }
            }
            for (int hl = 1; hl < 32; hl <<= 1) {  // h = hl * E
#pragma unroll
                for (int t = 0; t < E; ++t) {
                    const float o = __shfl_xor_sync(0xFFFFFFFFu, v[t], hl);
                    v[t] = (lane & hl) ? __fsub_rn(o, v[t]) : __fadd_rn(v[t], o);
                }
            }
#pragma unroll
            for (int t = 0; t < E; ++t) v[t] = __fmul_rn(v[t], scale);
        }
        uint32_t m = 0;
#pragma unroll
        for (int t = 0; t < E; ++t) {
            s_v[lane * E + t] = v[t];
            if (v[t] < 0.0f) m |= 1u << t;
        }
        s_mask[lane] = m;
        __syncwarp();
        if (lane < ix.nw) {
            uint64_t w = 0;
            const int per = 64 / E;  // lanes per word
            for (int u = 0; u < per; ++u) w |= (uint64_t)s_mask[lane * per + u] << (u * E);
            e.qbits[(size_t)q * ix.nw + lane] = w;
        }
    } else if (warp == 1 || warp == 2) {
        // SQ8 pre-scales x * step and the products x * min (warp 1: centroid re-order, warp 2:
        // rerank); then lanes 0 and 1 of warp 1 fold the two bases sum(x * min) in dimension order,
        // side by side on one instruction stream (the products are the same rounded values the
        // fold would compute inline)
        const int which = warp - 1;
        const bool want = which == 0 ? want_cqs : want_rqs;
        if (want) {
            const float* mn = which == 0 ? ix.csq_min : ix.sq_min;
            const float* stp = which == 0 ? ix.csq_step : ix.sq_step;
            float* dst = (which == 0 ? e.cqs : e.rqs) + (size_t)q * dim;
            for (int t = lane; t < dim; t += 32) {
                const float xv = __ldg(x + t);
                dst[t] = __fmul_rn(xv, __ldg(stp + t));
                s_prod[which][t] = __fmul_rn(xv, __ldg(mn + t));
            }
        }
        asm volatile("bar.sync 1, 64;" ::: "memory");  // warps 1 and 2
        if (warp == 1 && lane < 2 && (lane == 0 ? want_cqs : want_rqs)) {
            const float* pr = s_prod[lane];
            float b = 0.0f;
#pragma unroll 8
            for (int t = 0; t < dim; ++t) b = __fadd_rn(b, pr[t]);
            (lane == 0 ? e.cqbase : e.rbase)[q] = b;
        }
    }
    __syncthreads();
    // FsQuery::new (quantize.rs:279-313): positions j = threadIdx.x + 128 u
    constexpr int PU = (8 * E + 127) / 128;  // positions per thread (npos <= 8 E)
    float raw[PU][16], lo[PU];
    float range = 0.0f;
#pragma unroll
    for (int u = 0; u < PU; ++u) {
        const int j = threadIdx.x + 128 * u;
        lo[u] = INFINITY;
        if (j < npos) {
            float hi = -INFINITY;
            const float v0 = s_v[4 * j], v1 = s_v[4 * j + 1], v2 = s_v[4 * j + 2], v3 = s_v[4 * j + 3];
#pragma unroll
            for (int ev = 0; ev < 16; ++ev) {
                float a = 0.0f;
                a = (ev & 1) ? __fsub_rn(a, v0) : __fadd_rn(a, v0);
                a = (ev & 2) ? __fsub_rn(a, v1) : __fadd_rn(a, v1);
                a = (ev & 4) ? __fsub_rn(a, v2) : __fadd_rn(a, v2);
                a = (ev & 8) ? __fsub_rn(a, v3) : __fadd_rn(a, v3);
                raw[u][ev] = a;
                lo[u] = fminf(lo[u], a);
                hi = fmaxf(hi, a);
            }
            range = fmaxf(range, __fsub_rn(hi, lo[u]));
            s_mins[j] = lo[u];
        }
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) range = fmaxf(range, __shfl_xor_sync(0xFFFFFFFFu, range, o));
    if (lane == 0) s_red[warp] = range;
    __syncthreads();
    range = fmaxf(fmaxf(s_red[0], s_red[1]), fmaxf(s_red[2], s_red[3]));
    const float delta = fmaxf(__fdiv_rn(range, 255.0f), 1e-12f);
#pragma unroll
    for (int u = 0; u < PU; ++u) {
        const int j = threadIdx.x + 128 * u;
        if (j >= npos) continue;
        uint32_t wv[4] = {0, 0, 0, 0};
#pragma unroll
        for (int ev = 0; ev < 16; ++ev) {
            float qv = clampf(roundf(__fdiv_rn(__fsub_rn(raw[u][ev], lo[u]), delta)), 0.0f, 255.0f);
            wv[ev >> 2] |= ((uint32_t)qv) << (8 * (ev & 3));
        }
        *reinterpret_cast<uint4*>(e.lut + ((size_t)q * npos + j) * 16) = make_uint4(wv[0], wv[1], wv[2], wv[3]);
    }
    if (threadIdx.x == 96) {  // bias: the table minima in position order
        float b = 0.0f;
        for (int t = 0; t < npos; ++t) b = __fadd_rn(b, s_mins[t]);
        e.fs_delta[q] = delta;
        e.fs_bias[q] = b;
    }
}

// ---- K2: flat Hamming shortlist ------------------------------------------------------------------

__device__ __forceinline__ uint32_t ham_row(const uint64_t* qb, const uint64_t* __restrict__ code, int nw) {
    uint32_t h = 0;
    for (int w = 0; w < nw; ++w) h += __popcll(qb[w] ^ __ldg(code + w));
    return h;
}

// Smallest t with prefix(t) >= want over hist[0..bits] (the counting cut-off of index.rs:86-104);
// bits when never reached. Warp 0 computes it.
constexpr int kRouteQB = 4;  // queries per CTA of the flat router (one warp each in pass 2)
constexpr int kRouteSmemH = 160 * 1024;  // Hamming rows kept in shared memory up to this size

// Pass 1: every centroid code is loaded once per CTA and scored against kRouteQB queries; the
// Hamming values (0xFFFF for empty cells) go to shared memory, or to the `hs` scratch (nq x M)
// when M is too large, plus a per-query histogram. Pass 2: warp j finds query j's counting
// cut-off and compacts its shortlist in cell order with ballots.
// Hamming distances of one centroid code to the CTA's queries; NW > 0: that many words, unrolled
// and read 16 bytes at a time (rows of NW words are 16-byte aligned for even NW); NW = 0: any nw.
template <int NW>
__device__ __forceinline__ void ham_rows(const uint64_t (*qb)[16], const uint64_t* __restrict__ code, int nw,
                                         uint32_t (&h)[kRouteQB]) {
#pragma unroll
    for (int j = 0; j < kRouteQB; ++j) h[j] = 0;
    if (NW > 0) {
        uint64_t cw[NW > 0 ? NW : 1];
#pragma unroll
        for (int w = 0; w < NW; w += 2) {
            const ulonglong2 v = __ldg(reinterpret_cast<const ulonglong2*>(code + w));
            cw[w] = v.x;
            cw[w + 1] = v.y;
        }
#pragma unroll
        for (int w = 0; w < NW; ++w)
#pragma unroll
            for (int j = 0; j < kRouteQB; ++j) h[j] += __popcll(qb[j][w] ^ cw[w]);
    } else {
        for (int w = 0; w < nw; ++w) {
            const uint64_t cw = __ldg(code + w);
#pragma unroll
            for (int j = 0; j < kRouteQB; ++j) h[j] += __popcll(qb[j][w] ^ cw);
        }
    }
}

template <int NW>
__global__ void __launch_bounds__(kBS) k_route_flat(IndexView ix, QueryEnc e, int nq, int want_c, int all,
                                                    int h_in_smem, uint16_t* hs, uint32_t* sl, uint32_t* sl_n,
                                                    int sl_cap) {
    extern __shared__ uint32_t rsh[];
    __shared__ uint64_t qb[kRouteQB][16];
    const int q0 = blockIdx.x * kRouteQB, nw = ix.nw, bits = nw * 64, M = ix.M;
    const int nqb = min(kRouteQB, nq - q0);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    uint32_t* hist = rsh;                                                     // kRouteQB x (bits + 1)
    uint16_t* hrow = h_in_smem ? reinterpret_cast<uint16_t*>(rsh + kRouteQB * (bits + 1))
                               : hs + (size_t)q0 * M;                         // kRouteQB x M
    if (!all) {
        for (int i = threadIdx.x; i < kRouteQB * 16; i += kBS) {
            int j = i / 16, w = i % 16;
            qb[j][w] = (j < nqb && w < nw) ? e.qbits[(size_t)(q0 + j) * nw + w] : 0ull;
        }
        for (int i = threadIdx.x; i < kRouteQB * (bits + 1); i += kBS) hist[i] = 0;
        __syncthreads();
        for (int c = threadIdx.x; c < M; c += kBS) {
            uint32_t h[kRouteQB];
            const bool lv = ix.live[c] != 0;
            if (lv) ham_rows<NW>(qb, ix.cent_bits + (size_t)c * nw, nw, h);
#pragma unroll
            for (int j = 0; j < kRouteQB; ++j) {
                if (j < nqb) {
                    hrow[(size_t)j * M + c] = lv ? (uint16_t)h[j] : (uint16_t)0xFFFF;
                    if (lv) atomicAdd(&hist[j * (bits + 1) + h[j]], 1u);
                }
            }
        }
        __syncthreads();
    }
    if (warp >= nqb) return;
    const int q = q0 + warp;
    int cut = bits;
    if (!all) cut = want_c == 0 ? 0 : warp_hist_cut(hist + warp * (bits + 1), bits, want_c);
    const uint16_t* hq = hrow + (size_t)warp * M;
    uint32_t count = 0;
    for (int base = 0; base < M; base += 128) {
        bool f[4];
#pragma unroll
        for (int u = 0; u < 4; ++u) {
            const int c = base + u * 32 + lane;
            f[u] = c < M && (all ? ix.live[c] != 0 : hq[c] <= (uint16_t)cut);
        }
#pragma unroll
        for (int u = 0; u < 4; ++u) {
            const int c = base + u * 32 + lane;
            unsigned m = __ballot_sync(0xFFFFFFFFu, f[u]);
            uint32_t pos = count + (uint32_t)__popc(m & ((1u << lane) - 1u));
            if (f[u] && pos < (uint32_t)sl_cap) sl[(size_t)q * sl_cap + pos] = (uint32_t)c;
            count += (uint32_t)__popc(m);
        }
    }
    if (lane == 0) sl_n[q] = count;
}

// ---- tree descent ---------------------------------------------------------------------------------

// keep_smallest (tree.rs:120-159) on n (h, id) pairs: the `keep` smallest h, ties at the cut-off
// in encounter order; stable compaction from (h_in, id_in) to id_out. Returns the kept count.
__device__ int block_keep_smallest(const uint32_t* h_in, const uint32_t* id_in, int n, int keep, int bits,
                                   uint32_t* id_out, uint32_t* hist) {
    using BS = cub::BlockScan<uint32_t, kBS>;
    __shared__ typename BS::TempStorage scan;
    __shared__ int s_t;
    __shared__ long long s_need;
    __shared__ uint32_t s_off, s_eq;
    if (keep >= n) {
        for (int i = threadIdx.x; i < n; i += kBS) id_out[i] = id_in[i];
        __syncthreads();
        return n;
    }
    for (int i = threadIdx.x; i <= bits; i += kBS) hist[i] = 0;
    __syncthreads();
    for (int i = threadIdx.x; i < n; i += kBS) atomicAdd(&hist[h_in[i]], 1u);
    __syncthreads();
    if (threadIdx.x < 32) {
        int t = warp_hist_cut(hist, bits, keep);
        if (threadIdx.x == 0) {
            long long below = 0;
            for (int i = 0; i < t; ++i) below += hist[i];
            s_t = t;
            s_need = keep - below;
            s_off = 0;
            s_eq = 0;
        }
    }
    __syncthreads();
    const uint32_t t = (uint32_t)s_t;
    const long long need = s_need;
    for (int base = 0; base < n; base += kBS) {
        int i = base + threadIdx.x;
        uint32_t h = i < n ? h_in[i] : 0xFFFFFFFFu;
        uint32_t eq = (i < n && h == t) ? 1u : 0u;
        uint32_t eq_rank, eq_agg;
        BS(scan).ExclusiveSum(eq, eq_rank, eq_agg);
        __syncthreads();
        uint32_t eq0 = s_eq;
        uint32_t kf = (i < n && (h < t || (eq && (long long)(eq0 + eq_rank) < need))) ? 1u : 0u;
        uint32_t pos, agg;
        BS(scan).ExclusiveSum(kf, pos, agg);
        uint32_t off = s_off;
        if (kf) id_out[off + pos] = id_in[i];
        __syncthreads();
        if (threadIdx.x == 0) {
            s_off = off + agg;
            s_eq = eq0 + eq_agg;
        }
        __syncthreads();
    }
    return (int)s_off;
}

struct Beams {
    int b[kMaxTreeLevels];
};

__global__ void __launch_bounds__(kBS) k_route_tree(IndexView ix, QueryEnc e, Beams bm, int want, uint32_t* scratch,
                                                    int cap, uint32_t* sl, uint32_t* sl_n, int sl_cap) {
    extern __shared__ uint32_t hist[];
    __shared__ uint64_t qb[16];
    __shared__ uint32_t s_n;
    using BS = cub::BlockScan<uint32_t, kBS>;
    __shared__ typename BS::TempStorage scan;
    const int q = blockIdx.x, nw = ix.nw, bits = nw * 64;
    uint32_t* fa = scratch + (size_t)q * 3 * cap;  // frontier
    uint32_t* fb = fa + cap;                      // survivors
    uint32_t* hh = fb + cap;                      // Hamming of the frontier
    if (threadIdx.x < nw) qb[threadIdx.x] = e.qbits[(size_t)q * nw + threadIdx.x];
    int nf = ix.tree_n[0];
    for (int i = threadIdx.x; i < nf; i += kBS) fa[i] = (uint32_t)i;
    __syncthreads();
    for (int li = 0; li < ix.tree_depth; ++li) {
        const uint64_t* codes = ix.tree_codes[li];
        for (int i = threadIdx.x; i < nf; i += kBS) hh[i] = ham_row(qb, codes + (size_t)fa[i] * nw, nw);
        __syncthreads();
        int keep = min(bm.b[li], nf);
        if (keep == 0) {
            nf = 0;
            break;
        }
        int ns = block_keep_smallest(hh, fa, nf, keep, bits, fb, hist);
        // expand kept nodes' children, in kept order (child_idx is the identity after compact_layout)
        const uint32_t* cst = ix.tree_child_start[li];
        const uint32_t* cln = ix.tree_child_len[li];
        if (threadIdx.x == 0) s_n = 0;
        __syncthreads();
        for (int base = 0; base < ns; base += kBS) {
            int i = base + threadIdx.x;
            uint32_t len = i < ns ? cln[fb[i]] : 0u;
            uint32_t pos, agg;
            BS(scan).ExclusiveSum(len, pos, agg);
            uint32_t off = s_n;
            if (i < ns) {
                uint32_t st = cst[fb[i]];
                for (uint32_t r = 0; r < len; ++r) fa[off + pos + r] = st + r;
            }
            __syncthreads();
            if (threadIdx.x == 0) s_n = off + agg;
            __syncthreads();
        }
        nf = (int)s_n;
        __syncthreads();
    }
    // final scan over candidate leaves
    for (int i = threadIdx.x; i < nf; i += kBS) hh[i] = ham_row(qb, ix.leaf_codes + (size_t)fa[i] * nw, nw);
    __syncthreads();
    int keep = min(want, nf);
    int ns = keep > 0 ? block_keep_smallest(hh, fa, nf, keep, bits, fb, hist) : 0;
    // leaf ids, live cells only (index.rs:1199-1209)
    if (threadIdx.x == 0) s_n = 0;
    __syncthreads();
    for (int base = 0; base < ns; base += kBS) {
        int i = base + threadIdx.x;
        uint32_t c = i < ns ? ix.leaf_ids[fb[i]] : 0u;
        uint32_t f = (i < ns && ix.live[c]) ? 1u : 0u;
        uint32_t pos, agg;
        BS(scan).ExclusiveSum(f, pos, agg);
        uint32_t off = s_n;
        if (f && off + pos < (uint32_t)sl_cap) sl[(size_t)q * sl_cap + off + pos] = c;
        __syncthreads();
        if (threadIdx.x == 0) s_n = off + agg;
        __syncthreads();
    }
    if (threadIdx.x == 0) sl_n[q] = s_n;
}

// ---- K3: exact re-order of the shortlist + nucleus -----------------------------------------------

__global__ void __launch_bounds__(kBS) k_rescore_select(IndexView ix, QueryEnc e, const float* __restrict__ Q,
                                                        const uint32_t* __restrict__ sl, const uint32_t* __restrict__ sl_n,
                                                        int sl_cap, int nprobe, float tc, float beta, int use_sq8,
                                                        uint32_t* chosen, float* cscore, uint32_t* nch, uint32_t* err) {
    extern __shared__ uint64_t keys[];
    const int q = blockIdx.x, dim = ix.dim;
    const int n = (int)sl_n[q];
    if (n > kSortCap || n > sl_cap) {
        if (threadIdx.x == 0) {
            nch[q] = 0;
            atomicAdd(err, 1u);
        }
        return;
    }
    const int P = next_pow2(max(n, 1));
    float* qv = reinterpret_cast<float*>(keys + P);
    const float* src = use_sq8 ? e.cqs + (size_t)q * dim : Q + (size_t)q * dim;
    for (int t = threadIdx.x; t < dim; t += kBS) qv[t] = src[t];
    for (int i = n + threadIdx.x; i < P; i += kBS) keys[i] = ~0ull;
    __syncthreads();
    const float base = use_sq8 ? e.cqbase[q] : 0.0f;
    const int l8 = threadIdx.x & 7;
    const unsigned gmask = 0xFFu << ((threadIdx.x & 31) & ~7);
    for (int i = threadIdx.x >> 3; i < n; i += kBS / 8) {
        uint32_t c = sl[(size_t)q * sl_cap + i];
        float s;
        if (use_sq8)
            s = __fadd_rn(dot_f32_u8_g8(qv, ix.cent_sq8 + (size_t)c * dim, dim, l8, gmask), base);
        else
            s = dot_f32_g8(qv, ix.cent_f32 + (size_t)c * dim, dim, l8, gmask);
        if (l8 == 0) keys[i] = ((uint64_t)(~float_key(s)) << 32) | c;
    }
    __syncthreads();
    block_bitonic_u64(keys, P);
    const int cap = min(nprobe, n);
    for (int i = threadIdx.x; i < cap; i += kBS) {
        uint64_t k = keys[i];
        chosen[(size_t)q * nprobe + i] = (uint32_t)k;
        cscore[(size_t)q * nprobe + i] = key_float(~(uint32_t)(k >> 32));
    }
    if (threadIdx.x == 0) {
        int m = cap;
        if (cap > 0 && tc < 1.0f) {
            // nucleus over the capped, sorted candidates (index.rs:1289-1300)
            float max_s = key_float(~(uint32_t)(keys[0] >> 32));
            float z = 0.0f;
            for (int i = 0; i < cap; ++i) {
                float s = key_float(~(uint32_t)(keys[i] >> 32));
                z = __fadd_rn(z, (float)exp((double)__fmul_rn(__fsub_rn(s, max_s), beta)));
            }
            float cum = 0.0f;
            m = 0;
            for (int i = 0; i < cap; ++i) {
                float s = key_float(~(uint32_t)(keys[i] >> 32));
                ++m;
                float p = __fdiv_rn((float)exp((double)__fmul_rn(__fsub_rn(s, max_s), beta)), __fadd_rn(z, 1e-9f));
                cum = __fadd_rn(cum, p);
                if (cum >= tc) break;
            }
        }
        nch[q] = (uint32_t)m;
    }
}

// The kth smallest (1-based) of n 64-bit keys given by key(i), by radix selection on all 8 bytes.
// All threads of the block call it; `hist` is 256 shared words.
template <typename KeyFn>
__device__ uint64_t block_select_kth_fn(KeyFn key, int n, int kth, uint32_t* hist) {
    __shared__ uint64_t s_prefix;
    __shared__ int s_rem;
    if (threadIdx.x == 0) {
        s_prefix = 0;
        s_rem = kth;
    }
    __syncthreads();
    uint64_t mask = 0;
    for (int by = 7; by >= 0; --by) {
        for (int i = threadIdx.x; i < 256; i += blockDim.x) hist[i] = 0;
        __syncthreads();
        const uint64_t prefix = s_prefix;
        const int shift = by * 8;
        for (int i = threadIdx.x; i < n; i += blockDim.x) {
            const uint64_t k = key(i);
            if ((k & mask) == prefix) atomicAdd(&hist[(k >> shift) & 255], 1u);
        }
        __syncthreads();
        if (threadIdx.x == 0) {
            int rem = s_rem, digit = 255;
            for (int t = 0; t < 256; ++t) {
                if ((int)hist[t] >= rem) {
                    digit = t;
                    break;
                }
                rem -= (int)hist[t];
            }
            s_rem = rem;
            s_prefix = prefix | ((uint64_t)digit << shift);
        }
        mask |= 0xFFull << shift;
        __syncthreads();
    }
    const uint64_t r = s_prefix;
    __syncthreads();
    return r;
}

// Probe selection after k_rescore_dots: the nprobe best shortlist cells by (score desc, cell asc),
// best first, then the nucleus cut (index.rs:1931-1977, :1283-1301). Up to `small` entries are
// sorted whole in shared memory; longer shortlists first select the nprobe-th key by radix and sort
// only the keys at or before it.
__global__ void __launch_bounds__(kBS) k_probe_select(const uint32_t* __restrict__ sl,
                                                      const uint32_t* __restrict__ sl_n,
                                                      const float* __restrict__ sc, int sl_cap, int nprobe, int small,
                                                      float tc, float beta, uint32_t* chosen, float* cscore,
                                                      uint32_t* nch, uint32_t* err) {
    extern __shared__ uint64_t pk[];
    __shared__ uint32_t hist[256];
    __shared__ uint32_t s_cnt;
    const int q = blockIdx.x;
    const int n = (int)sl_n[q];
    const int cap = min(nprobe, n);
    if (n > sl_cap || cap > small) {
        if (threadIdx.x == 0) {
            nch[q] = 0;
            atomicAdd(err, 1u);
        }
        return;
    }
    const uint32_t* cq = sl + (size_t)q * sl_cap;
    const float* sq = sc + (size_t)q * sl_cap;
    auto key = [&](int i) -> uint64_t { return ((uint64_t)(~float_key(__ldg(sq + i))) << 32) | __ldg(cq + i); };
    int m = n;  // keys to sort
    if (n <= small) {
        for (int i = threadIdx.x; i < n; i += kBS) pk[i] = key(i);
    } else {
        const uint64_t kk = block_select_kth_fn(key, n, cap, hist);
        if (threadIdx.x == 0) s_cnt = 0;
        __syncthreads();
        for (int base = 0; base < n; base += kBS) {
            const int i = base + threadIdx.x;
            const uint64_t k = i < n ? key(i) : ~0ull;
            const bool take = i < n && k <= kk;
            const uint32_t p = warp_append(take, &s_cnt);
            if (take) pk[p] = k;
        }
        __syncthreads();
        m = cap;
    }
    const int P = next_pow2(max(m, 1));
    for (int i = m + threadIdx.x; i < P; i += kBS) pk[i] = ~0ull;
    __syncthreads();
    block_bitonic_u64(pk, P);
    for (int i = threadIdx.x; i < cap; i += kBS) {
        const uint64_t k = pk[i];
        chosen[(size_t)q * nprobe + i] = (uint32_t)k;
        cscore[(size_t)q * nprobe + i] = key_float(~(uint32_t)(k >> 32));
    }
    if (threadIdx.x == 0) {
        int mm = cap;
        if (cap > 0 && tc < 1.0f) {
            // nucleus over the capped, sorted candidates (index.rs:1289-1300)
            float max_s = key_float(~(uint32_t)(pk[0] >> 32));
            float z = 0.0f;
            for (int i = 0; i < cap; ++i) {
                float s = key_float(~(uint32_t)(pk[i] >> 32));
                z = __fadd_rn(z, (float)exp((double)__fmul_rn(__fsub_rn(s, max_s), beta)));
            }
            float cum = 0.0f;
            mm = 0;
            for (int i = 0; i < cap; ++i) {
                float s = key_float(~(uint32_t)(pk[i] >> 32));
                ++mm;
                float p = __fdiv_rn((float)exp((double)__fmul_rn(__fsub_rn(s, max_s), beta)), __fadd_rn(z, 1e-9f));
                cum = __fadd_rn(cum, p);
                if (cum >= tc) break;
            }
        }
        nch[q] = (uint32_t)mm;
    }
}

// One lane's exact dot of a query (shared memory, dim floats) with one row: the reference's 8-lane
// FMA order (lane l takes elements l, l+8, ...), the hsum_ps tree, then the sequential tail.
// Byte rows are read 16 bytes (two steps) at a time; `row` must be 16-byte aligned with dim % 16 == 0
// for bytes and dim % 4 == 0 for f32.
template <bool kBytes>
__device__ __forceinline__ float lane_row_dot(const float* __restrict__ qs, const void* row, int dim) {
    const int full8 = dim & ~7, n8 = full8 >> 3;
    float a0 = 0.0f, a1 = 0.0f, a2 = 0.0f, a3 = 0.0f, a4 = 0.0f, a5 = 0.0f, a6 = 0.0f, a7 = 0.0f;
    const float4* qp = reinterpret_cast<const float4*>(qs);
    if (kBytes) {
        const uint4* rp = reinterpret_cast<const uint4*>(row);
#pragma unroll 4
        for (int m = 0; m < (n8 >> 1); ++m) {
            const uint4 w = __ldg(rp + m);
            const float4 q0 = qp[4 * m], q1 = qp[4 * m + 1], q2 = qp[4 * m + 2], q3 = qp[4 * m + 3];
            a0 = __fmaf_rn(q0.x, byte_val(w.x, 0, false), a0);
            a1 = __fmaf_rn(q0.y, byte_val(w.x, 1, false), a1);
            a2 = __fmaf_rn(q0.z, byte_val(w.x, 2, false), a2);
            a3 = __fmaf_rn(q0.w, byte_val(w.x, 3, false), a3);
            a4 = __fmaf_rn(q1.x, byte_val(w.y, 0, false), a4);
            a5 = __fmaf_rn(q1.y, byte_val(w.y, 1, false), a5);
            a6 = __fmaf_rn(q1.z, byte_val(w.y, 2, false), a6);
            a7 = __fmaf_rn(q1.w, byte_val(w.y, 3, false), a7);
            a0 = __fmaf_rn(q2.x, byte_val(w.z, 0, false), a0);
            a1 = __fmaf_rn(q2.y, byte_val(w.z, 1, false), a1);
            a2 = __fmaf_rn(q2.z, byte_val(w.z, 2, false), a2);
            a3 = __fmaf_rn(q2.w, byte_val(w.z, 3, false), a3);
            a4 = __fmaf_rn(q3.x, byte_val(w.w, 0, false), a4);
            a5 = __fmaf_rn(q3.y, byte_val(w.w, 1, false), a5);
            a6 = __fmaf_rn(q3.z, byte_val(w.w, 2, false), a6);
            a7 = __fmaf_rn(q3.w, byte_val(w.w, 3, false), a7);
        }
    } else {
        const float4* rp = reinterpret_cast<const float4*>(row);
#pragma unroll 4
        for (int i = 0; i < n8; ++i) {
            const float4 x0 = __ldg(rp + 2 * i), x1 = __ldg(rp + 2 * i + 1);
            const float4 q0 = qp[2 * i], q1 = qp[2 * i + 1];
            a0 = __fmaf_rn(q0.x, x0.x, a0);
            a1 = __fmaf_rn(q0.y, x0.y, a1);
            a2 = __fmaf_rn(q0.z, x0.z, a2);
            a3 = __fmaf_rn(q0.w, x0.w, a3);
            a4 = __fmaf_rn(q1.x, x1.x, a4);
            a5 = __fmaf_rn(q1.y, x1.y, a5);
            a6 = __fmaf_rn(q1.z, x1.z, a6);
            a7 = __fmaf_rn(q1.w, x1.w, a7);
        }
    }
    float sc = __fadd_rn(__fadd_rn(__fadd_rn(a0, a4), __fadd_rn(a2, a6)), __fadd_rn(__fadd_rn(a1, a5), __fadd_rn(a3, a7)));
    for (int i = full8; i < dim; ++i) {
        const float x = kBytes ? (float)reinterpret_cast<const uint8_t*>(row)[i] : reinterpret_cast<const float*>(row)[i];
        sc = __fadd_rn(sc, __fmul_rn(qs[i], x));
    }
    return sc;
}

// Small shortlists (the re-order of index.rs:1931-1977 when nprobe x multiplier is small): one warp
// per query scores up to kSmallShortlist cells, one lane per centroid row, then sorts the keys
// (score desc, cell asc) in its slice of shared memory and takes the best nprobe, then the nucleus.
constexpr int kSmallShortlist = 1024;
constexpr int kSmallQ = 4;  // queries (warps) per CTA
template <bool kBytes>
__global__ void __launch_bounds__(32 * kSmallQ) k_rescore_small(IndexView ix, const float* __restrict__ qsrc,
                                                               const float* __restrict__ qbase,
                                                               const uint32_t* __restrict__ sl,
                                                               const uint32_t* __restrict__ sl_n, int sl_cap, int nq,
                                                               int nprobe, float tc, float beta, uint32_t* chosen,
                                                               float* cscore, uint32_t* nch, uint32_t* err) {
    extern __shared__ __align__(16) uint8_t ssm[];
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, dim = ix.dim;
    const int q = blockIdx.x * kSmallQ + warp;
    const int qstride = (dim + 3) & ~3;
    float* qs = reinterpret_cast<float*>(ssm) + (size_t)warp * qstride;
    uint64_t* keys = reinterpret_cast<uint64_t*>(ssm + (size_t)kSmallQ * qstride * 4) + (size_t)warp * kSmallShortlist;
    if (q >= nq) return;  // warp-uniform
    const int n = (int)sl_n[q];
    if (n > kSmallShortlist || n > sl_cap) {
        if (lane == 0) {
            nch[q] = 0;
            atomicAdd(err, 1u);
        }
        return;
    }
    for (int i = lane; i < dim; i += 32) qs[i] = qsrc[(size_t)q * dim + i];
    __syncwarp();
    const float base = kBytes ? qbase[q] : 0.0f;
    const uint32_t* cq = sl + (size_t)q * sl_cap;
    for (int i = lane; i < n; i += 32) {
        const uint32_t c = __ldg(cq + i);
        const void* row = kBytes ? (const void*)(ix.cent_sq8 + (size_t)c * dim) : (const void*)(ix.cent_f32 + (size_t)c * dim);
        float s = lane_row_dot<kBytes>(qs, row, dim);
        if (kBytes) s = __fadd_rn(s, base);
        keys[i] = ((uint64_t)(~float_key(s)) << 32) | c;
    }
    const int P = next_pow2(max(n, 1));
    for (int i = n + lane; i < P; i += 32) keys[i] = ~0ull;
    __syncwarp();
    for (int kk = 2; kk <= P; kk <<= 1) {
        for (int j = kk >> 1; j > 0; j >>= 1) {
            for (int i = lane; i < P; i += 32) {
                const int ixj = i ^ j;
                if (ixj > i) {
                    const uint64_t a = keys[i], b = keys[ixj];
                    if ((a > b) == ((i & kk) == 0)) {
                        keys[i] = b;
                        keys[ixj] = a;
                    }
                }
            }
            __syncwarp();
        }
    }
    const int cap = min(nprobe, n);
    for (int i = lane; i < cap; i += 32) {
        const uint64_t k = keys[i];
        chosen[(size_t)q * nprobe + i] = (uint32_t)k;
        cscore[(size_t)q * nprobe + i] = key_float(~(uint32_t)(k >> 32));
    }
    if (lane == 0) {
        int mm = cap;
        if (cap > 0 && tc < 1.0f) {
            // nucleus over the capped, sorted candidates (index.rs:1289-1300)
            float max_s = key_float(~(uint32_t)(keys[0] >> 32));
            float z = 0.0f;
            for (int i = 0; i < cap; ++i) {
                float s = key_float(~(uint32_t)(keys[i] >> 32));
                z = __fadd_rn(z, (float)exp((double)__fmul_rn(__fsub_rn(s, max_s), beta)));
            }
            float cum = 0.0f;
            mm = 0;
            for (int i = 0; i < cap; ++i) {
                float s = key_float(~(uint32_t)(keys[i] >> 32));
                ++mm;
                float p = __fdiv_rn((float)exp((double)__fmul_rn(__fsub_rn(s, max_s), beta)), __fadd_rn(z, 1e-9f));
                cum = __fadd_rn(cum, p);
                if (cum >= tc) break;
            }
        }
        nch[q] = (uint32_t)mm;
    }
}

}  // namespace

// ---- launchers ----------------------------------------------------------------------------------------

void launch_encode(const IndexView& ix, const float* Q, int nq, const QueryEnc& e, bool want_cqs, bool want_rqs,
                   cudaStream_t st) {
    if (nq <= 0) return;
    Tick tk(kKEncode, st);
    const int wc = want_cqs ? 1 : 0, wr = want_rqs ? 1 : 0;
    switch (ix.dim_pad) {
        case 64: k_encode4<2><<<nq, 128, 0, st>>>(ix, Q, e, wc, wr); return;
        case 128: k_encode4<4><<<nq, 128, 0, st>>>(ix, Q, e, wc, wr); return;
        case 256: k_encode4<8><<<nq, 128, 0, st>>>(ix, Q, e, wc, wr); return;
        case 512: k_encode4<16><<<nq, 128, 0, st>>>(ix, Q, e, wc, wr); return;
        case 1024: k_encode4<32><<<nq, 128, 0, st>>>(ix, Q, e, wc, wr); return;
        default: break;
    }
    size_t smem = (size_t)(ix.dim_pad + ix.npos) * sizeof(float);
    k_encode<<<nq, kBS, smem, st>>>(ix, Q, e, wc, wr);
}

void launch_route_flat(const IndexView& ix, const QueryEnc& e, int nq, int want_c, uint16_t* hs, uint32_t* sl,
                       uint32_t* sl_n, int sl_cap, cudaStream_t st) {
    if (nq <= 0) return;
    const size_t hist_b = (size_t)kRouteQB * (ix.nw * 64 + 1) * sizeof(uint32_t);
    const size_t h_b = (size_t)kRouteQB * ix.M * sizeof(uint16_t);
    const int in_smem = h_b <= (size_t)kRouteSmemH ? 1 : 0;
    const size_t smem = hist_b + (in_smem ? h_b : 0);
    const int grid = (nq + kRouteQB - 1) / kRouteQB;
    const void* fn = ix.nw == 8    ? (const void*)k_route_flat<8>
                     : ix.nw == 4  ? (const void*)k_route_flat<4>
                     : ix.nw == 2  ? (const void*)k_route_flat<2>
                     : ix.nw == 12 ? (const void*)k_route_flat<12>
                     : ix.nw == 16 ? (const void*)k_route_flat<16>
                                   : (const void*)k_route_flat<0>;
    set_smem(fn, smem);
    Tick tk(kKRouteFlat, st);
    switch (ix.nw) {
        case 8: k_route_flat<8><<<grid, kBS, smem, st>>>(ix, e, nq, want_c, 0, in_smem, hs, sl, sl_n, sl_cap); break;
        case 4: k_route_flat<4><<<grid, kBS, smem, st>>>(ix, e, nq, want_c, 0, in_smem, hs, sl, sl_n, sl_cap); break;
        case 2: k_route_flat<2><<<grid, kBS, smem, st>>>(ix, e, nq, want_c, 0, in_smem, hs, sl, sl_n, sl_cap); break;
        case 12: k_route_flat<12><<<grid, kBS, smem, st>>>(ix, e, nq, want_c, 0, in_smem, hs, sl, sl_n, sl_cap); break;
        case 16: k_route_flat<16><<<grid, kBS, smem, st>>>(ix, e, nq, want_c, 0, in_smem, hs, sl, sl_n, sl_cap); break;
        default: k_route_flat<0><<<grid, kBS, smem, st>>>(ix, e, nq, want_c, 0, in_smem, hs, sl, sl_n, sl_cap); break;
    }
}

// Every live cell, in cell order, as every query's shortlist (route_query with neither tree nor
// two-stage codes scores all live cells, index.rs:1260-1270): a copy of the list built at upload.
__global__ void k_route_all(IndexView ix, int nq, uint32_t* __restrict__ sl, uint32_t* __restrict__ sl_n, int sl_cap) {
    const int n = ix.n_live_cells;
    const size_t total = (size_t)nq * n;
    for (size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x; i < total; i += (size_t)gridDim.x * blockDim.x) {
        const size_t q = i / n, j = i - q * n;
        if (j < (size_t)sl_cap) sl[q * sl_cap + j] = __ldg(ix.live_list + j);
        if (j == 0) sl_n[q] = (uint32_t)n;
    }
}

void launch_route_all(const IndexView& ix, int nq, uint32_t* sl, uint32_t* sl_n, int sl_cap, cudaStream_t st) {
    if (nq <= 0) return;
    const size_t total = (size_t)nq * std::max(ix.n_live_cells, 1);
    const int grid = (int)std::min<size_t>((total + kBS - 1) / kBS, 148 * 16);
    Tick tk(kKRouteFlat, st);
    k_route_all<<<grid, kBS, 0, st>>>(ix, nq, sl, sl_n, sl_cap);
}

void launch_route_tree(const IndexView& ix, const QueryEnc& e, int nq, const int* beams, int want, uint32_t* scratch,
                       int scratch_cap, uint32_t* sl, uint32_t* sl_n, int sl_cap, cudaStream_t st) {
    if (nq <= 0) return;
    Beams bm{};
    for (int i = 0; i < ix.tree_depth && i < kMaxTreeLevels; ++i) bm.b[i] = beams[i];
    size_t smem = (size_t)(ix.nw * 64 + 1) * sizeof(uint32_t);
    Tick tk(kKRouteTree, st);
    k_route_tree<<<nq, kBS, smem, st>>>(ix, e, bm, want, scratch, scratch_cap, sl, sl_n, sl_cap);
}

void launch_rescore_select(const IndexView& ix, const QueryEnc& e, const float* Q, int nq, const uint32_t* sl,
                           const uint32_t* sl_n, int sl_cap, int nprobe, float tc, float beta, bool use_sq8,
                           uint32_t* chosen, float* cscore, uint32_t* nch, uint32_t* err, float* rs_scores,
                           uint32_t* rs_items, int expect_n, bool all_live, cudaStream_t st) {
    if (nq <= 0) return;
    const int row_bytes = use_sq8 ? ix.dim : ix.dim * 4;
    if (expect_n <= 128 && row_bytes % 16 == 0 && nprobe <= kSmallShortlist) {
        // small shortlists: one launch, one warp per query
        const size_t smem = (size_t)kSmallQ * (((ix.dim + 3) & ~3) * sizeof(float) + kSmallShortlist * sizeof(uint64_t));
        const int grid = (nq + kSmallQ - 1) / kSmallQ;
        Tick tk(kKRescore, st);
        if (use_sq8) {
            set_smem((const void*)k_rescore_small<true>, smem);
            k_rescore_small<true><<<grid, 32 * kSmallQ, smem, st>>>(ix, e.cqs, e.cqbase, sl, sl_n, sl_cap, nq, nprobe,
                                                                     tc, beta, chosen, cscore, nch, err);
        } else {
            set_smem((const void*)k_rescore_small<false>, smem);
            k_rescore_small<false><<<grid, 32 * kSmallQ, smem, st>>>(ix, Q, e.cqbase, sl, sl_n, sl_cap, nq, nprobe,
                                                                      tc, beta, chosen, cscore, nch, err);
        }
        return;
    }
    const int small = std::max(next_pow2(std::max(nprobe, 1)), 1024);
    if (rs_scores && rs_items && small <= kSortCap && all_live &&
        launch_rescore_all(ix, e, Q, nq, use_sq8, sl_cap, rs_scores, st)) {
        // every shortlist is the live-cell list: the tiled product scored it, then the selection
        const size_t psm = (size_t)small * sizeof(uint64_t);
        set_smem((const void*)k_probe_select, psm);
        Tick tk(kKProbeSelect, st);
        k_probe_select<<<nq, kBS, psm, st>>>(sl, sl_n, rs_scores, sl_cap, nprobe, small, tc, beta, chosen, cscore, nch,
                                             err);
        return;
    }
    if (rs_scores && rs_items && row_bytes % 16 == 0) {
        // scores of every (query, shortlist cell) pair by the flattened register gather, then a
        // per-query selection
        launch_rescore_dots(ix, e, Q, nq, sl, sl_n, sl_cap, use_sq8, rs_scores, rs_items, st);
        if (small <= kSortCap) {
            const size_t psm = (size_t)small * sizeof(uint64_t);
            set_smem((const void*)k_probe_select, psm);
            Tick tk(kKProbeSelect, st);
            k_probe_select<<<nq, kBS, psm, st>>>(sl, sl_n, rs_scores, sl_cap, nprobe, small, tc, beta, chosen,
                                                 cscore, nch, err);
            return;
        }
    }
    int P = next_pow2(std::min(std::max(sl_cap, 1), kSortCap));
    size_t smem = (size_t)P * sizeof(uint64_t) + (size_t)ix.dim * sizeof(float);
    set_smem((const void*)k_rescore_select, smem);
    Tick tk(kKRescore, st);
    k_rescore_select<<<nq, kBS, smem, st>>>(ix, e, Q, sl, sl_n, sl_cap, nprobe, tc, beta, use_sq8 ? 1 : 0, chosen,
                                            cscore, nch, err);
}

}  // namespace dev
}  // namespace maivs
