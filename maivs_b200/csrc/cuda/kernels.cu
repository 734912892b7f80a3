// MAIVS query kernels for sm_100a: query encoding, routing, seed + adaptive prune, cell-major
// inversion and scan, per-query scan with the sequential stop rule, exact cut and rerank.
//
// Integer work (codes, table sums, distances, cut-offs) is exact by construction. Floating-point
// work follows the reference's evaluation order (see common.cuh), so scores are bit-identical to
// the reference's CPU path on the same inputs.
#include <cub/block/block_reduce.cuh>
#include <atomic>
#include <cub/block/block_scan.cuh>

#include "common.cuh"
#include "kernels.cuh"
#include "umma.cuh"

namespace maivs {
namespace dev {

namespace {

constexpr int kBS = 256;

// ---- block utilities ----------------------------------------------------------------------------

// prmt.b32 in its generic mode: byte i of the result is byte (sel nibble i) & 7 of {b, a}; every
// selector here keeps bit 3 of its nibbles clear (copy, no sign replication).
__device__ __forceinline__ uint32_t prmt(uint32_t a, uint32_t b, uint32_t sel) {
    uint32_t d;
    asm("prmt.b32 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(sel));
    return d;
}

// FastScan table lookups of one code word: nibble b of w (member b of the group) selects entry
// nib of the 16-byte table t. r0 holds members 0-3 and r1 members 4-7, one byte each. The byte
// selectors of both halves come from one mask and one shift of w.
__device__ __forceinline__ void lut16x8(uint4 t, uint32_t w, uint32_t& r0, uint32_t& r1) {
    const uint32_t s3 = w & 0x77777777u;                         // entry within the 8-byte half
    const uint32_t pk = ((w >> 1) & 0x44444444u) | 0x32103210u;  // pick the half by bit 3
    r0 = prmt(prmt(t.x, t.y, s3), prmt(t.z, t.w, s3), pk);
    const uint32_t s3h = s3 >> 16, pkh = pk >> 16;
    r1 = prmt(prmt(t.x, t.y, s3h), prmt(t.z, t.w, s3h), pkh);
}

// Running sums of a group's 8 members without widening every byte: `all` adds the four looked-up
// bytes as one 32-bit word (bytes 1 and 3 carry into their neighbours, modulo 2^32) and `odd`
// adds bytes 1 and 3 widened to 16-bit halves. Because every member's total stays below 2^16
// (255 x npos with npos <= 256), all - (odd << 8) is exactly bytes 0 and 2 widened, modulo 2^32.
struct GroupAcc {
    uint32_t all0 = 0, odd0 = 0, all1 = 0, odd1 = 0;
    __device__ __forceinline__ void add(uint4 t, uint32_t w) {
        uint32_t r0, r1;
        lut16x8(t, w, r0, r1);
        all0 += r0;
        odd0 += prmt(r0, 0, 0x4341);
        all1 += r1;
        odd1 += prmt(r1, 0, 0x4341);
    }
    // acc[b >> 1] holds member b's sum in half (b & 1)
    __device__ __forceinline__ void finish(uint32_t acc[4]) const {
        const uint32_t e0 = all0 - (odd0 << 8), e1 = all1 - (odd1 << 8);  // members 0|2, 4|6
        acc[0] = prmt(e0, odd0, 0x5410);
        acc[1] = prmt(e0, odd0, 0x7632);
        acc[2] = prmt(e1, odd1, 0x5410);
        acc[3] = prmt(e1, odd1, 0x7632);
    }
};

// Sum of each lane's 8 FastScan table sums of group g over npos positions. Word (j, g) of the
// cell holds nibble j of members 8g..8g+7; `lut` is npos x 16 bytes (layout of
// src/quantize.rs:303-311: entry e of position j at byte 16j + e). acc[b>>1] holds member b's
// 16-bit sum in half (b & 1). Sums never exceed 255 * npos <= 65280.
__device__ __forceinline__ void group_sums(const uint32_t* __restrict__ codes, int ng, int g, bool active,
                                           const uint8_t* lut, int npos, uint32_t acc[4]) {
    GroupAcc a;
    const uint4* T = reinterpret_cast<const uint4*>(lut);
    // npos is a multiple of 16; eight independent code-word loads are issued before their lookups
    uint32_t off = (uint32_t)g;
    for (int j0 = 0; j0 < npos; j0 += 8) {
        uint32_t w[8];
#pragma unroll
        for (int u = 0; u < 8; ++u) w[u] = active ? __ldg(codes + off + (uint32_t)u * (uint32_t)ng) : 0u;
        off += 8u * (uint32_t)ng;
#pragma unroll
        for (int u = 0; u < 8; ++u) a.add(T[j0 + u], w[u]);
    }
    a.finish(acc);
}

// group_sums over positions [p0, p1) only (the packed 16-bit partial sums of a position slice).
__device__ __forceinline__ void group_sums_range(const uint32_t* __restrict__ codes, int ng, int g, bool active,
                                                 const uint8_t* lut, int p0, int p1, uint32_t acc[4]) {
    GroupAcc a;
    const uint4* T = reinterpret_cast<const uint4*>(lut);
    int j0 = p0;
    uint32_t off = (uint32_t)p0 * (uint32_t)ng + (uint32_t)g;
    for (; j0 + 8 <= p1; j0 += 8) {
        uint32_t w[8];
#pragma unroll
        for (int u = 0; u < 8; ++u) w[u] = active ? __ldg(codes + off + (uint32_t)u * (uint32_t)ng) : 0u;
        off += 8u * (uint32_t)ng;
#pragma unroll
        for (int u = 0; u < 8; ++u) a.add(T[j0 + u], w[u]);
    }
    for (; j0 < p1; ++j0, off += (uint32_t)ng) a.add(T[j0], active ? __ldg(codes + off) : 0u);
    a.finish(acc);
}

__device__ __forceinline__ uint32_t member_sum(const uint32_t acc[4], int b) {
    return (acc[b >> 1] >> (16 * (b & 1))) & 0xFFFFu;
}

// Appends `key` for every lane whose `valid` is set with one atomic per warp: returns the slot
// index for this lane (undefined when !valid). All 32 lanes must call it.
__device__ __forceinline__ uint32_t warp_append(bool valid, uint32_t* counter) {
    const unsigned mask = __ballot_sync(0xFFFFFFFFu, valid);
    const int lane = threadIdx.x & 31;
    uint32_t base = 0;
    if (mask) {
        const int leader = __ffs(mask) - 1;
        if (lane == leader) base = atomicAdd(counter, (uint32_t)__popc(mask));
        base = __shfl_sync(0xFFFFFFFFu, base, leader);
    }
    return base + (uint32_t)__popc(mask & ((1u << lane) - 1u));
}

// Exactly-once rule of the cell-major join: a multi-home vector is scored only at its lowest-id
// probed home (index.rs:2036-2045).
// A probed-bitmap word. A kernel that wrote the bitmap itself reads it through L2 (kFresh): the
// read-only path may hold a line of it cached before the writes.
template <bool kFresh = false>
__device__ __forceinline__ uint64_t probed_word(const uint64_t* probed, uint32_t cell) {
    return kFresh ? __ldcg(probed + (cell >> 6)) : __ldg(probed + (cell >> 6));
}

template <bool kFresh = false>
__device__ __forceinline__ bool canonical_cm(const IndexView& ix, uint32_t slot, uint32_t c, const uint64_t* probed) {
    // branch-free over the homes so the loads of several members can be in flight together
    const uint32_t* h = ix.slot_cells + (size_t)slot * ix.ma;
    bool ok = true;
    for (int j = 0; j < ix.ma; ++j) {
        const uint32_t hc = __ldg(h + j);
        const bool lower = hc != kNoCell && hc < c;
        const uint64_t word = lower ? probed_word<kFresh>(probed, hc) : 0ull;
        ok = ok && !(lower && ((word >> (hc & 63)) & 1ull));
    }
    return ok;
}

// Byte b of w as a float (signed or unsigned).
__device__ __forceinline__ float byte_val(uint32_t w, int b, bool sgn) {
    const uint32_t v = (w >> (8 * b)) & 0xFFu;
    return sgn ? (float)(int8_t)v : (float)v;
}

// canonical_cm for a member entry whose lower home is precomputed (IndexView::cell_lower).
template <bool kFresh = false>
__device__ __forceinline__ bool canonical_lower(uint32_t lower, const uint64_t* probed) {
    return lower == kNoCell || !((probed_word<kFresh>(probed, lower) >> (lower & 63)) & 1ull);
}

// canonical_cm against a bitmap in shared memory.
__device__ __forceinline__ bool canonical_cm_bits(const IndexView& ix, uint32_t slot, uint32_t c,
                                                  const uint64_t* bits) {
    const uint32_t* h = ix.slot_cells + (size_t)slot * ix.ma;
    bool ok = true;
    for (int j = 0; j < ix.ma; ++j) {
        const uint32_t hc = __ldg(h + j);
        const bool lower = hc != kNoCell && hc < c;
        ok = ok && !(lower && ((bits[hc >> 6] >> (hc & 63)) & 1ull));
    }
    return ok;
}

// The kth smallest (1-based) of up to two key segments, by radix selection on bytes [lo_byte,
// hi_byte] of the 64-bit keys (higher bytes must be zero). Returns the selected key with the
// unselected low bytes zero. All threads of the block must call it; `hist` is 256 shared words.
__device__ uint64_t block_select_kth(const uint64_t* a, int na, const uint64_t* b, int nb, int kth, int hi_byte,
                                     int lo_byte, uint32_t* hist) {
    __shared__ uint64_t s_prefix;
    __shared__ int s_rem;
    if (threadIdx.x == 0) {
        s_prefix = 0;
        s_rem = kth;
    }
    __syncthreads();
    uint64_t mask = 0;
    for (int by = hi_byte; by >= lo_byte; --by) {
        for (int i = threadIdx.x; i < 256; i += blockDim.x) hist[i] = 0;
        __syncthreads();
        uint64_t prefix = s_prefix;
        int shift = by * 8;
        for (int i = threadIdx.x; i < na + nb; i += blockDim.x) {
            uint64_t k = i < na ? a[i] : b[i - na];
            if ((k & mask) == prefix) atomicAdd(&hist[(k >> shift) & 255], 1u);
        }
        __syncthreads();
        if (threadIdx.x < 32) {
            // warp scan over 256 bins, 8 per lane: the digit where the running count reaches rem
            const int lane = threadIdx.x;
            const int rem = s_rem;
            int local = 0;
#pragma unroll
            for (int t = 0; t < 8; ++t) local += (int)hist[lane * 8 + t];
            int inc = local;
#pragma unroll
            for (int o = 1; o < 32; o <<= 1) {
                int v = __shfl_up_sync(0xFFFFFFFFu, inc, o);
                if (lane >= o) inc += v;
            }
            const int excl = inc - local;
            const unsigned hit = __ballot_sync(0xFFFFFFFFu, excl < rem && inc >= rem);
            const int src = hit ? __ffs(hit) - 1 : 31;
            if (lane == src) {
                int r = rem - excl, digit = lane * 8 + 7;
                for (int t = 0; t < 8; ++t) {
                    int hv = (int)hist[lane * 8 + t];
                    if (hv >= r) {
                        digit = lane * 8 + t;
                        break;
                    }
                    r -= hv;
                }
                s_rem = r;
                s_prefix = prefix | ((uint64_t)digit << shift);
            }
        }
        mask |= 0xFFull << shift;
        __syncthreads();
    }
    uint64_t r = s_prefix;
    __syncthreads();
    return r;
}

// Warp 0 (all its lanes): the bin of `hist` (256 counts) where the running count reaches rem
// (1-based); *rem_out = rem less the counts of the bins before it. Nothing else is synchronised.
__device__ __forceinline__ void hist_find_warp0(const uint32_t* hist, int rem, uint32_t* bin_out, int* rem_out) {
    const int lane = threadIdx.x;
    int local = 0;
#pragma unroll
    for (int t = 0; t < 8; ++t) local += (int)hist[lane * 8 + t];
    int inc = local;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
        const int v = __shfl_up_sync(0xFFFFFFFFu, inc, o);
        if (lane >= o) inc += v;
    }
    const int excl = inc - local;
    const unsigned hit = __ballot_sync(0xFFFFFFFFu, excl < rem && inc >= rem);
    const int src = hit ? __ffs(hit) - 1 : 31;
    if (lane == src) {
        int r = rem - excl, bin = lane * 8 + 7;
        for (int t = 0; t < 8; ++t) {
            const int hv = (int)hist[lane * 8 + t];
            if (hv >= r) {
                bin = lane * 8 + t;
                break;
            }
            r -= hv;
        }
        *bin_out = (uint32_t)bin;
        *rem_out = r;
    }
}

// The kth smallest (1-based, kth <= na + nb) distance d = key >> 32 of up to two key segments,
// d < 2^16. Three passes over the keys: the block's smallest and largest d; a histogram of
// (d - lo) >> s, s the fewest bits that fit the range in 256 bins; and a histogram of the low s
// bits of the keys in the bin that holds the kth. Bins over the keys' own range spread the
// shared-memory atomics (fixed byte digits would pile most distances onto a few bins). All
// threads of the block call it; `hist` is 256 shared words.
__device__ uint32_t block_select_d(const uint64_t* a, int na, const uint64_t* b, int nb, int kth, uint32_t* hist) {
    __shared__ uint32_t s_lo, s_hi, s_bin;
    __shared__ int s_rem;
    const int n = na + nb;
    uint32_t lo = 0xFFFFFFFFu, hi = 0;
    for (int i = threadIdx.x; i < n; i += blockDim.x) {
        const uint32_t d = (uint32_t)((i < na ? a[i] : b[i - na]) >> 32);
        lo = min(lo, d);
        hi = max(hi, d);
    }
    lo = __reduce_min_sync(0xFFFFFFFFu, lo);
    hi = __reduce_max_sync(0xFFFFFFFFu, hi);
    if (threadIdx.x == 0) {
        s_lo = 0xFFFFFFFFu;
        s_hi = 0;
        s_rem = kth;
    }
    for (int i = threadIdx.x; i < 256; i += blockDim.x) hist[i] = 0;
    __syncthreads();
    if ((threadIdx.x & 31) == 0) {
        atomicMin(&s_lo, lo);
        atomicMax(&s_hi, hi);
    }
    __syncthreads();
    lo = s_lo;
    const uint32_t range = s_hi - lo;
    int sh = 0;
    while ((range >> sh) > 255u) ++sh;
    for (int i = threadIdx.x; i < n; i += blockDim.x) {
        const uint32_t d = (uint32_t)((i < na ? a[i] : b[i - na]) >> 32);
        atomicAdd(&hist[(d - lo) >> sh], 1u);
    }
    __syncthreads();
    if (threadIdx.x < 32) hist_find_warp0(hist, s_rem, &s_bin, &s_rem);
    __syncthreads();
    const uint32_t bin = s_bin;
    if (sh == 0) {
        __syncthreads();
        return lo + bin;
    }
    for (int i = threadIdx.x; i < 256; i += blockDim.x) hist[i] = 0;
    __syncthreads();
    const uint32_t mask = (1u << sh) - 1u;
    for (int i = threadIdx.x; i < n; i += blockDim.x) {
        const uint32_t d = (uint32_t)((i < na ? a[i] : b[i - na]) >> 32) - lo;
        if ((d >> sh) == bin) atomicAdd(&hist[d & mask], 1u);
    }
    __syncthreads();
    if (threadIdx.x < 32) hist_find_warp0(hist, s_rem, &s_bin, &s_rem);
    __syncthreads();
    const uint32_t v = lo + (bin << sh) + s_bin;
    __syncthreads();
    return v;
}

// ---- the rest scan's falling cut-off (index.rs:2231-2275) ----------------------------------------
// The reference scans the rest cells against a per-query cut-off shared by its workers: a worker
// holding `target` entries of a query publishes their target-th smallest distance with
// AtomicU32::fetch_min (index.rs:2266-2269) and later cells are tested against the lower value.
// Here one CTA scans one cell for all its queries and never holds `target` entries of one query, so
// the lower bound is proven by counting. For each query k_seed sets rungs e_0 > e_1 > ... below the
// seed cut-off tau, with s_l = the query's seed survivors at or below e_l; the scans count the
// canonical rest survivors at or below each rung (c_l), and once s_l + c_l >= target there are
// `target` distinct entries at or below e_l, so the exact target-th smallest distance is at most
// e_l and atomicMin lowers the query's cut-off gtau[q] to it. Entries above gtau can no longer be
// in the exact cut of k_final_cm (ties at the cut are kept, as before), so the result is unchanged
// while fewer entries are appended. Rungs sit near ranks m (3/4)^(l+1), m = min(seed survivors,
// target), rounded up to the edge of a 256-bin histogram over [lowest seed distance, tau].

// Writes the rungs of one query from its seed entries (keys[0..n), only d <= tau counted): per
// rung its distance, the count still needed (target - s_l, 0 when the seed alone has target) and a
// zeroed counter. All threads of the block call it; `hist` is 256 shared words.
__device__ void build_ladder(const uint64_t* keys, int n, uint32_t tau, int target, uint32_t* lad,
                             uint32_t* hist) {
    __shared__ uint32_t s_lo, s_cnt;
    __shared__ uint32_t s_bin[kLad];
    __shared__ int s_rem[kLad];
    uint32_t lo = 0xFFFFFFFFu, cnt = 0;
    for (int i = threadIdx.x; i < n; i += blockDim.x) {
        const uint32_t d = (uint32_t)(keys[i] >> 32);
        if (d <= tau) {
            lo = min(lo, d);
            ++cnt;
        }
    }
    lo = __reduce_min_sync(0xFFFFFFFFu, lo);
    cnt = __reduce_add_sync(0xFFFFFFFFu, cnt);
    if (threadIdx.x == 0) {
        s_lo = 0xFFFFFFFFu;
        s_cnt = 0;
    }
    for (int i = threadIdx.x; i < 256; i += blockDim.x) hist[i] = 0;
    __syncthreads();
    if ((threadIdx.x & 31) == 0) {
        atomicMin(&s_lo, lo);
        atomicAdd(&s_cnt, cnt);
    }
    __syncthreads();
    lo = s_lo;
    const int m = (int)s_cnt;
    if (m == 0) {  // no seed survivors: the rungs can never be proven
        if (threadIdx.x < kLad) {
            lad[threadIdx.x] = 0;
            lad[kLad + threadIdx.x] = 0xFFFFFFFFu;
            lad[2 * kLad + threadIdx.x] = 0;
        }
        __syncthreads();
        return;
    }
    int sh = 0;
    while (((tau - lo) >> sh) > 255u) ++sh;
    for (int i = threadIdx.x; i < n; i += blockDim.x) {
        const uint32_t d = (uint32_t)(keys[i] >> 32);
        if (d <= tau) atomicAdd(&hist[(d - lo) >> sh], 1u);
    }
    __syncthreads();
    const int mm = min(m, target);
    if (threadIdx.x < 32) {  // one warp scan of the bins serves every rung
        const int lane = threadIdx.x;
        int local = 0;
#pragma unroll
        for (int t = 0; t < 8; ++t) local += (int)hist[lane * 8 + t];
        int inc = local;
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
            const int v = __shfl_up_sync(0xFFFFFFFFu, inc, o);
            if (lane >= o) inc += v;
        }
        const int excl = inc - local;
        int r = mm;
        for (int l = 0; l < kLad; ++l) {
            r = max((r * 3) >> 2, 1);
            const unsigned hit = __ballot_sync(0xFFFFFFFFu, excl < r && inc >= r);
            if (lane == (hit ? __ffs(hit) - 1 : 31)) {
                int rr = r - excl, bin = lane * 8 + 7;
                for (int t = 0; t < 8; ++t) {
                    const int hv = (int)hist[lane * 8 + t];
                    if (hv >= rr) {
                        bin = lane * 8 + t;
                        break;
                    }
                    rr -= hv;
                }
                s_bin[l] = (uint32_t)bin;
                s_rem[l] = rr;
            }
        }
    }
    __syncthreads();
    if (threadIdx.x < kLad) {
        const int l = threadIdx.x;
        int r = mm;
        for (int t = 0; t <= l; ++t) r = max((r * 3) >> 2, 1);
        const uint32_t bin = s_bin[l];
        const uint32_t below = (uint32_t)(r - s_rem[l]) + hist[bin];  // seed survivors in bins <= bin
        const uint32_t e = min(lo + (bin << sh) + ((1u << sh) - 1u), tau);
        lad[l] = e;
        lad[kLad + l] = below >= (uint32_t)target ? 0u : (uint32_t)target - below;
        lad[2 * kLad + l] = 0;
    }
    __syncthreads();
}

// Adds a tile's counts (two u16 per word, zeroed here) to query q's rungs and lowers its cut-off
// to the lowest rung proven. Loads and atomics are independent so that they overlap.
__device__ __forceinline__ void ladder_flush(const CellMajorBufs& b, uint32_t q, uint32_t* packed) {
    uint32_t v[kLad];
    bool any = false;
#pragma unroll
    for (int w = 0; w < kLad / 2; ++w) {
        const uint32_t pair = packed[w];
        packed[w] = 0;
        v[2 * w] = pair & 0xFFFFu;
        v[2 * w + 1] = pair >> 16;
        any |= pair != 0;
    }
    if (!any) return;
    uint32_t* lq = b.lad + (size_t)q * kLadStride;
    const uint32_t g = *reinterpret_cast<volatile const uint32_t*>(b.gtau + q);
    uint32_t e[kLad], need[kLad], old[kLad];
#pragma unroll
    for (int l = 0; l < kLad; ++l) {
        e[l] = lq[l];
        need[l] = lq[kLad + l];
    }
#pragma unroll
    for (int l = 0; l < kLad; ++l) old[l] = (v[l] && e[l] < g) ? atomicAdd(lq + 2 * kLad + l, v[l]) : 0u;
    uint32_t best = g;
#pragma unroll
    for (int l = 0; l < kLad; ++l)
        if (v[l] && e[l] < g && old[l] + v[l] >= need[l]) best = min(best, e[l]);
    if (best < g) atomicMin(b.gtau + q, best);
}

// Adds v rest survivors at or below rung l of query q; lowers the query's cut-off once the rung is
// proven. Skips rungs at or above the current cut-off.
__device__ __forceinline__ void ladder_add(const CellMajorBufs& b, uint32_t q, int l, uint32_t v) {
    uint32_t* lq = b.lad + (size_t)q * kLadStride;
    const uint32_t e = lq[l];
    if (e >= *reinterpret_cast<volatile const uint32_t*>(b.gtau + q)) return;
    const uint32_t old = atomicAdd(lq + 2 * kLad + l, v);
    if (old + v >= lq[kLad + l]) atomicMin(b.gtau + q, e);
}

// Bitonic sort, ascending, of P (power of two) 64-bit keys in shared memory.
__device__ void block_bitonic_u64(uint64_t* keys, int P) {
    for (int k = 2; k <= P; k <<= 1) {
        for (int j = k >> 1; j > 0; j >>= 1) {
            for (int i = threadIdx.x; i < P; i += blockDim.x) {
                int ixj = i ^ j;
                if (ixj > i) {
                    uint64_t a = keys[i], b = keys[ixj];
                    bool up = (i & k) == 0;
                    if ((a > b) == up) {
                        keys[i] = b;
                        keys[ixj] = a;
                    }
                }
            }
            __syncthreads();
        }
    }
}

__host__ __device__ inline int next_pow2(int n) {
    int p = 1;
    while (p < n) p <<= 1;
    return p;
}

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
__device__ int warp_hist_cut(const uint32_t* hist, int bits, long long want) {
    int lane = threadIdx.x & 31;
    int nb = bits + 1;
    int per = (nb + 31) / 32;
    int b0 = lane * per, b1 = min(b0 + per, nb);
    long long s = 0;
    for (int i = b0; i < b1; ++i) s += hist[i];
    long long inc = s;
    for (int o = 1; o < 32; o <<= 1) {
        long long v = __shfl_up_sync(0xFFFFFFFFu, inc, o);
        if (lane >= o) inc += v;
    }
    long long excl = inc - s;
    int found = (excl < want && inc >= want) ? 1 : 0;
    unsigned bal = __ballot_sync(0xFFFFFFFFu, found);
    int res = bits;
    if (bal) {
        int src = __ffs(bal) - 1;
        int t = bits;
        if (lane == src) {
            long long c = excl;
            for (int i = b0; i < b1; ++i) {
                c += hist[i];
                if (c >= want) {
                    t = i;
                    break;
                }
            }
        }
        res = __shfl_sync(0xFFFFFFFFu, t, src);
    }
    return res;
}

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

// ---- cell-major: seed + adaptive prune (index.rs:2126-2191) --------------------------------------

// ---- cell-range shards: distance lists exchanged between shards -----------------------------------
// A shard publishes, per query, how many entries it holds and the smallest min(count, xl) of their
// distances (any order). The kth smallest distance of the union of all shards is then exact for
// any kth <= xl: a shard holding kth or more entries at or below a value lists kth of them, and a
// shard holding fewer lists them all. Rank r's block of an all-gathered buffer holds nq counts
// (u32), then nq x xl distances (u16; distances are at most 255 x 256).

__host__ __device__ inline size_t shard_list_bytes(int nq, int xl) {
    return (((size_t)nq * 4 + (size_t)nq * xl * 2) + 15) & ~(size_t)15;
}

// Writes the smallest min(na + nb, L) distances (key >> 32) of two key segments to out.
__device__ void emit_smallest_d(const uint64_t* a, int na, const uint64_t* b, int nb, int L, uint16_t* out,
                                uint32_t* hist) {
    __shared__ uint32_t s_cnt;
    const int n = na + nb;
    uint32_t dl = 0xFFFFFFFFu;
    if (n > L) dl = block_select_d(a, na, b, nb, L, hist);
    if (threadIdx.x == 0) s_cnt = 0;
    __syncthreads();
    for (int base = 0; base < n; base += blockDim.x) {
        const int i = base + threadIdx.x;
        const uint64_t k = i < na ? a[i] : (i < n ? b[i - na] : ~0ull);
        const uint32_t d = (uint32_t)(k >> 32);
        const bool take = i < n && d < dl;
        const uint32_t p = warp_append(take, &s_cnt);
        if (take) out[p] = (uint16_t)d;
    }
    __syncthreads();
    const int m = min(n, L);
    for (int i = (int)s_cnt + threadIdx.x; i < m; i += blockDim.x) out[i] = (uint16_t)dl;  // ties at the Lth
    __syncthreads();
}

__device__ __forceinline__ uint32_t shard_count(const uint8_t* xall, size_t rank_bytes, int r, int q) {
    return reinterpret_cast<const uint32_t*>(xall + (size_t)r * rank_bytes)[q];
}
__device__ __forceinline__ const uint16_t* shard_list(const uint8_t* xall, size_t rank_bytes, int r, int nq, int q,
                                                      int xl) {
    return reinterpret_cast<const uint16_t*>(xall + (size_t)r * rank_bytes + (size_t)nq * 4) + (size_t)q * xl;
}

// The kth smallest (1-based) distance of the union of W shards' lists for query q.
__device__ uint32_t block_select_lists(const uint8_t* xall, size_t rank_bytes, int W, int nq, int q, int xl,
                                       int kth, uint32_t* hist) {
    __shared__ uint32_t s_digit;
    __shared__ int s_rem;
    if (threadIdx.x == 0) s_rem = kth;
    uint32_t hi = 0;
    for (int pass = 0; pass < 2; ++pass) {
        for (int i = threadIdx.x; i < 256; i += blockDim.x) hist[i] = 0;
        __syncthreads();
        for (int r = 0; r < W; ++r) {
            const int cnt = min((int)shard_count(xall, rank_bytes, r, q), xl);
            const uint16_t* lst = shard_list(xall, rank_bytes, r, nq, q, xl);
            for (int j = threadIdx.x; j < cnt; j += blockDim.x) {
                const uint32_t v = lst[j];
                if (pass == 0)
                    atomicAdd(&hist[v >> 8], 1u);
                else if ((v >> 8) == hi)
                    atomicAdd(&hist[v & 255u], 1u);
            }
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
            s_digit = (uint32_t)digit;
        }
        __syncthreads();
        if (pass == 0) hi = s_digit;
    }
    const uint32_t v = (hi << 8) | s_digit;
    __syncthreads();
    return v;
}

// ---- cell-major: the seed step (index.rs:2126-2191) --------------------------------------------------
constexpr int kSeedScanThreads = 128;
// Seed keys k_seed keeps in shared memory (32 KB: five 256-thread CTAs per SM, the register
// limit); a query whose seed cells hold more members keeps them in its global seed buffer.
constexpr int kSeedSmemKeys = 4096;
// Probed-cell bitmaps up to this many words (M <= 65,536 cells) are built in shared memory.
constexpr int kSeedSmemBitmapWords = 1024;

// Group prefix of the query's seed cells in shared memory: g[r] = groups of the seed cells
// before r, ng/woff/moff/nc of cell r. Warp 0 computes it; the caller synchronises.
struct SeedCells {
    int g[kSeedCells + 1];
    int ng[kSeedCells], nc[kSeedCells];
    uint32_t woff[kSeedCells], moff[kSeedCells], c[kSeedCells];
};
__device__ __forceinline__ void seed_cells_prefix(const IndexView& ix, const uint32_t* ch, int ns, SeedCells& sc) {
    if (threadIdx.x >= 32) return;
    const int lane = threadIdx.x;
    int ng = 0, nc = 0;
    uint32_t c = 0, m0 = 0, woff = 0;
    if (lane < ns) {
        c = ch[lane];
        m0 = ix.cell_moff[c];
        nc = (int)(ix.cell_moff[c + 1] - m0);
        ng = (nc + 7) >> 3;
        woff = ix.cell_woff[c];
    }
    int inc = ng;
#pragma unroll
    for (int o = 1; o < kSeedCells; o <<= 1) {
        const int v = __shfl_up_sync(0xFFFFFFFFu, inc, o);
        if (lane >= o) inc += v;
    }
    if (lane < kSeedCells) {
        sc.g[lane + 1] = inc;
        sc.ng[lane] = ng;
        sc.nc[lane] = nc;
        sc.woff[lane] = woff;
        sc.moff[lane] = m0;
        sc.c[lane] = c;
    }
    if (lane == 0) sc.g[0] = 0;
}
// The seed cell holding numbered group f (cells without members hold none).
__device__ __forceinline__ int seed_cell_of(const SeedCells& sc, int f) {
    int r = 0;
    while (r + 1 < kSeedCells && sc.g[r + 1] <= f) ++r;
    return r;
}

// FastScan sums of every member of a query's seed cells (the first kSeedCells probes,
// index.rs:2131-2148). The member groups of the seed cells are numbered consecutively, cell after
// cell, and dealt to the query's gridDim.y blocks, one group of 8 members per thread, so warps
// stay full whatever the cells' sizes. Member b of numbered group f gets its distance
// maxk - sum at seed_d[8 f + b] (members past the end of their cell get a value nobody reads).
__global__ void __launch_bounds__(kSeedScanThreads) k_seed_scan(IndexView ix, QueryEnc e,
                                                                const uint32_t* __restrict__ chosen,
                                                                const uint32_t* __restrict__ nch, int nprobe,
                                                                CellMajorBufs b) {
    extern __shared__ __align__(16) uint8_t lut_s[];  // npos x 16 LUT bytes
    __shared__ SeedCells sc;
    const int q = blockIdx.x, npos = ix.npos;
    const int ns = min(kSeedCells, (int)nch[q]);
    seed_cells_prefix(ix, chosen + (size_t)q * nprobe, ns, sc);
    __syncthreads();
    const int G = sc.g[kSeedCells];
    const int first = blockIdx.y * kSeedScanThreads;
    if (first >= G) return;
    {
        const uint4* src = reinterpret_cast<const uint4*>(e.lut + (size_t)q * npos * 16);
        uint4* dst = reinterpret_cast<uint4*>(lut_s);
        for (int i = threadIdx.x; i < npos; i += kSeedScanThreads) dst[i] = src[i];
    }
    __syncthreads();
    const uint32_t maxk = ix.maxk;
    uint4* out = reinterpret_cast<uint4*>(b.seed_d + (size_t)q * b.seed_dcap);
    for (int f = first + (int)threadIdx.x; f < G; f += (int)gridDim.y * kSeedScanThreads) {
        const int r = seed_cell_of(sc, f);
        uint32_t acc[4];
        group_sums(ix.cell_codes + sc.woff[r], sc.ng[r], f - sc.g[r], true, lut_s, npos, acc);
        uint32_t o[4];
#pragma unroll
        for (int i = 0; i < 4; ++i) o[i] = (maxk - (acc[i] & 0xFFFFu)) | ((maxk - (acc[i] >> 16)) << 16);
        out[f] = make_uint4(o[0], o[1], o[2], o[3]);
    }
}

// The seed step of the cell-major join (index.rs:2131-2191), one CTA per query, after
// k_seed_scan: keeps the canonical seed entries (the exactly-once rule against every probed cell,
// whose bitmap it builds, in shared memory when smem_bits, and stores for the rest scan), selects
// the seed cut-off tau = the target-th smallest seed distance (ties kept), retains d <= tau and
// finds the adaptive end of the rest probes. The entries stay in shared memory when the seed
// cells' members fit in `smem_keys` keys. With final_cand (no probe beyond the seed cells) the
// survivors are already the exact cut of index.rs:2277-2306 and their slots become the candidate
// list; a cell-range shard (xlist) publishes its smallest distances instead.
__global__ void __launch_bounds__(kBS) k_seed(IndexView ix, QueryEnc e, const uint32_t* __restrict__ chosen,
                                              const float* __restrict__ cscore, const uint32_t* __restrict__ nch,
                                              int nprobe, int target, int adaptive, float at_margin, CellMajorBufs b,
                                              int smem_keys, int smem_bits, int final_cand, uint16_t* xlist,
                                              uint32_t* xcnt, int xl) {
    extern __shared__ __align__(16) uint64_t key_s[];  // smem_keys keys, then (smem_bits) the bitmap
    __shared__ uint32_t hist[256];
    __shared__ uint32_t s_n;
    __shared__ int s_last;
    __shared__ SeedCells sc;
    const int q = blockIdx.x;
    const int n_ch = (int)nch[q];
    const int ns = min(kSeedCells, n_ch);
    const uint32_t* ch = chosen + (size_t)q * nprobe;
    // the probed-cell bitmap of the exactly-once rule: built in shared memory when it fits and
    // stored for the rest scan, else built in the global buffer and read back through L2
    uint64_t* probed = b.probed + (size_t)q * b.mwords;
    uint64_t* bits = smem_bits ? key_s + smem_keys : probed;
    if (ix.ma > 1) {
        for (int w = threadIdx.x; w < b.mwords; w += kBS) bits[w] = 0;
        __syncthreads();
        for (int i = threadIdx.x; i < n_ch; i += kBS) atomicOr((unsigned long long*)&bits[ch[i] >> 6], 1ull << (ch[i] & 63));
    }
    seed_cells_prefix(ix, ch, ns, sc);
    if (threadIdx.x == 0) {
        s_n = 0;
        s_last = -1;
    }
    __syncthreads();
    if (ix.ma > 1 && smem_bits)
        for (int w = threadIdx.x; w < b.mwords; w += kBS) probed[w] = bits[w];
    uint64_t* sbuf = b.seed_buf + (size_t)q * b.seed_cap;
    int members = 0;
    for (int r = 0; r < ns; ++r) members += sc.nc[r];
    // all canonical seed entries go to `keys`: shared memory when they fit, else the global buffer
    const bool keys_in_smem = members <= smem_keys;
    uint64_t* keys = keys_in_smem ? key_s : sbuf;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, nwarps = kBS / 32;
    const uint32_t maxk = ix.maxk;
    const uint16_t* sd = b.seed_d + (size_t)q * b.seed_dcap;
    const int nslots = 8 * sc.g[kSeedCells];
    constexpr int U = 4;  // member entries per thread and round: their loads are issued together
    int rcur = 0;         // a thread's slots rise, so the seed cell of the last one is a start
    for (int base = 0; base < nslots; base += kBS * U) {
        uint32_t slot[U], d[U], lw[U];
        int rr[U];
        bool valid[U];
#pragma unroll
        for (int u = 0; u < U; ++u) {
            const int i = base + u * kBS + (int)threadIdx.x;
            valid[u] = false;
            slot[u] = d[u] = 0;
            lw[u] = kNoCell;
            rr[u] = 0;
            if (i < nslots) {
                const int f = i >> 3;
                while (rcur + 1 < kSeedCells && sc.g[rcur + 1] <= f) ++rcur;
                const int r = rcur;
                const int pos = 8 * (f - sc.g[r]) + (i & 7);
                if (pos < sc.nc[r]) {
                    const uint32_t m = sc.moff[r] + (uint32_t)pos;
                    valid[u] = true;
                    rr[u] = r;
                    slot[u] = __ldg(ix.cell_slots + m);
                    d[u] = sd[i];
                    if (ix.ma > 1 && ix.cell_lower) lw[u] = __ldg(ix.cell_lower + m);
                }
            }
        }
#pragma unroll
        for (int u = 0; u < U; ++u) {
            if (valid[u] && ix.ma > 1) {
                if (smem_bits)
                    valid[u] = ix.cell_lower ? lw[u] == kNoCell || !((bits[lw[u] >> 6] >> (lw[u] & 63)) & 1ull)
                                             : canonical_cm_bits(ix, slot[u], sc.c[rr[u]], bits);
                else
                    valid[u] = ix.cell_lower ? canonical_lower<true>(lw[u], probed)
                                             : canonical_cm<true>(ix, slot[u], sc.c[rr[u]], probed);
            }
            const uint32_t p = warp_append(valid[u], &s_n);
            if (valid[u] && p < (uint32_t)b.seed_cap) keys[p] = ((uint64_t)d[u] << 32) | slot[u];
        }
    }
    __syncthreads();
    int n = (int)s_n;
    if (n > b.seed_cap) {
        if (threadIdx.x == 0) atomicAdd(b.overflow, 1u);
        n = b.seed_cap;
    }
    if (xlist) {  // cell-range shard: publish this shard's seed distances; k_seed_finish goes on
        emit_smallest_d(keys, n, nullptr, 0, xl, xlist + (size_t)q * xl, hist);
        if (threadIdx.x == 0) {
            xcnt[q] = (uint32_t)n;
            b.seed_n[q] = (uint32_t)n;
        }
        return;
    }
    uint32_t tau = maxk;
    if (n >= target) {
        tau = block_select_d(keys, n, nullptr, 0, target, hist);
    }
    // retain d <= tau (ties kept): warps append the survivors to the global seed buffer. With no
    // probes beyond the seed cells (final_cand) the survivors are the exact cut already (the
    // target-th smallest of all entries is tau) and their slots go straight to the candidate list.
    __shared__ uint32_t s_out;
    uint32_t* cand = b.cand + (size_t)q * b.cand_cap;
    if (keys_in_smem) {
        if (threadIdx.x == 0) s_out = 0;
        __syncthreads();
        const int per = (n + nwarps - 1) / nwarps;
        const int i0 = warp * per, i1 = min(n, i0 + per);
        for (int base = i0; base < i1; base += 32) {
            const int i = base + lane;
            const uint64_t key = i < i1 ? keys[i] : ~0ull;
            const bool keep = i < i1 && (uint32_t)(key >> 32) <= tau;
            const uint32_t p = warp_append(keep, &s_out);
            if (keep) {
                if (final_cand) cand[p] = (uint32_t)key;
                else sbuf[p] = key;
            }
        }
        __syncthreads();
        n = (int)s_out;
    } else if (n >= target) {
        using BS = cub::BlockScan<uint32_t, kBS>;
        __shared__ typename BS::TempStorage scan;
        if (threadIdx.x == 0) s_out = 0;
        __syncthreads();
        for (int base = 0; base < n; base += kBS) {
            int i = base + threadIdx.x;
            uint64_t key = i < n ? sbuf[i] : 0;
            uint32_t f = (i < n && (uint32_t)(key >> 32) <= tau) ? 1u : 0u;
            uint32_t pos, agg;
            BS(scan).ExclusiveSum(f, pos, agg);
            __syncthreads();
            uint32_t off = s_out;
            if (f) {
                if (final_cand) cand[off + pos] = (uint32_t)key;
                else sbuf[off + pos] = key;
            }
            __syncthreads();
            if (threadIdx.x == 0) s_out = off + agg;
            __syncthreads();
        }
        n = (int)s_out;
    } else if (final_cand) {
        for (int i = threadIdx.x; i < n; i += kBS) cand[i] = (uint32_t)sbuf[i];
    }
    if (final_cand) {
        if (threadIdx.x == 0) {
            b.tau[q] = tau;
            b.seed_n[q] = (uint32_t)n;
            b.rest_hi[q] = (uint32_t)ns;
            b.rest_n[q] = 0;
            b.cand_n[q] = (uint32_t)n;
        }
        return;
    }
    int rest_end = n_ch;
    if (adaptive && n >= target && ns < n_ch) {
        const float norm = fs_norm(ix.dim_pad);
        float thr = clampf(__fdiv_rn(fs_estimate(e.fs_delta[q], e.fs_bias[q], maxk - tau), norm), -1.0f, 1.0f);
        float X = __fsub_rn(thr, at_margin);
        for (int i = ns + threadIdx.x; i < n_ch; i += kBS) {
            float bnd = cell_bound(cscore[(size_t)q * nprobe + i], ix.r_bound[ch[i]]);
            if (bnd >= X) atomicMax(&s_last, i);
        }
        __syncthreads();
        rest_end = s_last >= 0 ? s_last + 1 : ns;
    }
    if (rest_end > ns) build_ladder(sbuf, n, tau, target, b.lad + (size_t)q * kLadStride, hist);
    if (threadIdx.x == 0) {
        b.tau[q] = tau;
        b.gtau[q] = tau;
        b.seed_n[q] = (uint32_t)n;
        b.rest_hi[q] = (uint32_t)rest_end;
        b.rest_n[q] = 0;
    }
}

// Cell-range shard, after the seed lists are all-gathered: the global seed cut-off tau (the
// target-th smallest seed distance over all shards, index.rs:2150-2160), this shard's seed
// survivors (d <= tau) and the adaptive end of the rest probes (index.rs:2162-2191), exactly as
// k_seed computes them on a whole index.
__global__ void __launch_bounds__(kBS) k_seed_finish(IndexView ix, QueryEnc e, const uint32_t* __restrict__ chosen,
                                                     const float* __restrict__ cscore,
                                                     const uint32_t* __restrict__ nch, int nprobe, int target,
                                                     int adaptive, float at_margin, CellMajorBufs b,
                                                     const uint8_t* __restrict__ xall, size_t rank_bytes, int W,
                                                     int nq, int xl) {
    __shared__ uint32_t hist[256];
    __shared__ int s_last;
    __shared__ uint32_t s_out;
    const int q = blockIdx.x;
    const int n_ch = (int)nch[q];
    const int ns = min(kSeedCells, n_ch);
    const uint32_t* ch = chosen + (size_t)q * nprobe;
    const uint32_t maxk = ix.maxk;
    unsigned long long ng = 0;
    for (int r = 0; r < W; ++r) ng += shard_count(xall, rank_bytes, r, q);
    const bool full = ng >= (unsigned long long)target;
    uint32_t tau = maxk;
    if (full) tau = block_select_lists(xall, rank_bytes, W, nq, q, xl, target, hist);
    uint64_t* sbuf = b.seed_buf + (size_t)q * b.seed_cap;
    int n = (int)b.seed_n[q];
    if (threadIdx.x == 0) {
        s_out = 0;
        s_last = -1;
    }
    __syncthreads();
    if (full) {
        using BS = cub::BlockScan<uint32_t, kBS>;
        __shared__ typename BS::TempStorage scan;
        for (int base = 0; base < n; base += kBS) {
            int i = base + threadIdx.x;
            uint64_t key = i < n ? sbuf[i] : 0;
            uint32_t f = (i < n && (uint32_t)(key >> 32) <= tau) ? 1u : 0u;
            uint32_t pos, agg;
            BS(scan).ExclusiveSum(f, pos, agg);
            __syncthreads();
            uint32_t off = s_out;
            if (f) sbuf[off + pos] = key;
            __syncthreads();
            if (threadIdx.x == 0) s_out = off + agg;
            __syncthreads();
        }
        n = (int)s_out;
    }
    int rest_end = n_ch;
    if (adaptive && full && ns < n_ch) {
        const float norm = fs_norm(ix.dim_pad);
        float thr = clampf(__fdiv_rn(fs_estimate(e.fs_delta[q], e.fs_bias[q], maxk - tau), norm), -1.0f, 1.0f);
        float X = __fsub_rn(thr, at_margin);
        for (int i = ns + threadIdx.x; i < n_ch; i += kBS) {
            float bnd = cell_bound(cscore[(size_t)q * nprobe + i], ix.r_bound[ch[i]]);
            if (bnd >= X) atomicMax(&s_last, i);
        }
        __syncthreads();
        rest_end = s_last >= 0 ? s_last + 1 : ns;
    }
    // the rungs count this shard's seed survivors only: fewer than the global ones, so a rung this
    // shard proves with them and its own rest survivors holds for the union too
    if (rest_end > ns) build_ladder(sbuf, n, tau, target, b.lad + (size_t)q * kLadStride, hist);
    if (threadIdx.x == 0) {
        b.tau[q] = tau;
        b.gtau[q] = tau;
        b.seed_n[q] = (uint32_t)n;
        b.rest_hi[q] = (uint32_t)rest_end;
        b.rest_n[q] = 0;
    }
}

// Cell-range shard, after its rest scan: publish the smallest distances of its survivors (seed and
// rest) for the global candidate cut.
__global__ void __launch_bounds__(kBS) k_local_list(CellMajorBufs b, uint16_t* xlist, uint32_t* xcnt, int xl) {
    __shared__ uint32_t hist[256];
    const int q = blockIdx.x;
    const int ns = (int)b.seed_n[q];
    int nr = (int)b.rest_n[q];
    if (nr > b.rest_cap) {
        if (threadIdx.x == 0) atomicAdd(b.overflow, 1u);
        nr = b.rest_cap;
    }
    emit_smallest_d(b.seed_buf + (size_t)q * b.seed_cap, ns, b.rest_buf + (size_t)q * b.rest_cap, nr, xl,
                    xlist + (size_t)q * xl, hist);
    if (threadIdx.x == 0) xcnt[q] = (uint32_t)(ns + nr);
}

// ---- cell-major: inversion (index.rs:2193-2213) ---------------------------------------------------

__global__ void k_inv_count(const uint32_t* __restrict__ chosen, const uint32_t* __restrict__ nch,
                            const uint32_t* __restrict__ rest_hi, int nq, int nprobe, uint32_t* cnt) {
    int q = blockIdx.x * (blockDim.x / 32) + (threadIdx.x >> 5);
    if (q >= nq) return;
    int lo = min(kSeedCells, (int)nch[q]), hi = (int)rest_hi[q];
    for (int i = lo + (threadIdx.x & 31); i < hi; i += 32) atomicAdd(&cnt[chosen[(size_t)q * nprobe + i]], 1u);
}

// Exclusive scan of cnt[0..M) in place, cnt[M] = total.
__global__ void __launch_bounds__(1024) k_inv_scan(uint32_t* cnt, int M) {
    using BS = cub::BlockScan<uint32_t, 1024>;
    __shared__ typename BS::TempStorage scan;
    __shared__ uint32_t s_run;
    if (threadIdx.x == 0) s_run = 0;
    __syncthreads();
    for (int base = 0; base < M; base += 1024) {
        int i = base + threadIdx.x;
        uint32_t v = i < M ? cnt[i] : 0u;
        uint32_t pos, agg;
        BS(scan).ExclusiveSum(v, pos, agg);
        uint32_t run = s_run;
        if (i < M) cnt[i] = run + pos;
        __syncthreads();
        if (threadIdx.x == 0) s_run = run + agg;
        __syncthreads();
    }
    if (threadIdx.x == 0) cnt[M] = s_run;
}

__global__ void k_inv_scatter(const uint32_t* __restrict__ chosen, const uint32_t* __restrict__ nch,
                              const uint32_t* __restrict__ rest_hi, int nq, int nprobe, const uint32_t* start,
                              uint32_t* fill, uint32_t* qof) {
    int q = blockIdx.x * (blockDim.x / 32) + (threadIdx.x >> 5);
    if (q >= nq) return;
    int lo = min(kSeedCells, (int)nch[q]), hi = (int)rest_hi[q];
    for (int i = lo + (threadIdx.x & 31); i < hi; i += 32) {
        uint32_t c = chosen[(size_t)q * nprobe + i];
        uint32_t p = start[c] + atomicAdd(&fill[c], 1u);
        qof[p] = (uint32_t)q;
    }
}

// ---- cell-major: the scan (index.rs:2231-2275) ------------------------------------------------------
// One CTA per cell; each warp scores one interested query against 32 member groups (256 members)
// at a time. A member survives when its distance is within the query's falling cut-off gtau (at
// most the seed cut-off tau, always at least the exact final cut, index.rs:2266-2269) and it is
// canonical. Each warp counts its survivors under the query's rungs and proves rungs as it goes.

__global__ void __launch_bounds__(kBS) k_scan_cm(IndexView ix, QueryEnc e, const uint32_t* __restrict__ start,
                                                 const uint32_t* __restrict__ qof, CellMajorBufs b, uint32_t max_q) {
    const uint32_t c = blockIdx.x;
    const uint32_t s0 = start[c], s1 = start[c + 1];
    if (s0 == s1 || s1 - s0 >= max_q) return;  // high-batch cells go to k_scan_mma
    const uint32_t moff = ix.cell_moff[c];
    const int nc = (int)(ix.cell_moff[c + 1] - moff);
    if (nc == 0) return;
    const int ng = (nc + 7) >> 3;
    const uint32_t* codes = ix.cell_codes + ix.cell_woff[c];
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, nwarps = kBS / 32;
    const int npos = ix.npos;
    const uint32_t maxk = ix.maxk;
    for (int chk = 0; chk * 32 < ng; ++chk) {
        const int g = chk * 32 + lane;
        const bool act = g < ng;
        for (uint32_t qi = s0 + warp; qi < s1; qi += nwarps) {
            const uint32_t q = qof[qi];
            const uint32_t t = *reinterpret_cast<volatile const uint32_t*>(b.gtau + q);
            const uint32_t rung = lane < kLad ? b.lad[(size_t)q * kLadStride + lane] : 0u;  // lane l: e_l
            uint32_t el[kLad];
#pragma unroll
            for (int l = 0; l < kLad; ++l) el[l] = __shfl_sync(0xFFFFFFFFu, rung, l);
            uint32_t acc[4];
            group_sums(codes, ng, g, act, e.lut + (size_t)q * npos * 16, npos, acc);
            uint32_t below[kLad] = {0, 0, 0, 0, 0, 0, 0, 0};
            bool any = false;
#pragma unroll
            for (int bb = 0; bb < 8; ++bb) {
                const int pos = 8 * g + bb;
                bool valid = act && pos < nc;
                uint32_t d = 0, slot = 0;
                if (valid) {
                    d = maxk - member_sum(acc, bb);
                    valid = d <= t;
                }
                if (valid) {
                    slot = ix.cell_slots[moff + pos];
                    if (ix.ma > 1)
                        valid = ix.cell_lower ? canonical_lower(__ldg(ix.cell_lower + moff + pos),
                                                                b.probed + (size_t)q * b.mwords)
                                              : canonical_cm(ix, slot, c, b.probed + (size_t)q * b.mwords);
                }
                uint32_t p = warp_append(valid, &b.rest_n[q]);
                if (valid && p < (uint32_t)b.rest_cap) b.rest_buf[(size_t)q * b.rest_cap + p] = ((uint64_t)d << 32) | slot;
                if (valid) {
                    any = true;
#pragma unroll
                    for (int l = 0; l < kLad; ++l) below[l] += (el[l] < t && d <= el[l]) ? 1u : 0u;
                }
            }
            if (__any_sync(0xFFFFFFFFu, any)) {
#pragma unroll
                for (int l = 0; l < kLad; ++l) {
                    const uint32_t v = __reduce_add_sync(0xFFFFFFFFu, below[l]);
                    if (lane == l && v) ladder_add(b, q, l, v);
                }
            }
        }
    }
}

// ---- cell-major: the scan of high-batch cells on the tensor cores -----------------------------------
// The FastScan sum of a (query, member) pair is sum_j LUT_q[16 j + nib_j(member)], i.e. the dot
// product of the query's u8 table row (K = 16 x npos bytes) with the one-hot expansion of the
// member's nibbles. For a cell that many queries probe this is a dense u8 x u8 -> s32 GEMM:
// M = 128 queries x N = 256 members per tile, K in chunks of 128 bytes (8 nibble positions). A
// (tables) is copied and B (one-hot nibbles) is built in shared memory in the K-major 128-byte
// swizzled layout, one elected thread issues four kind::i8 tcgen05.mma per chunk into a TMEM
// accumulator (128 lanes x 256 columns), two stages overlap building chunk k + 1 with the MMAs of
// chunk k, and the epilogue reads the sums with tcgen05.ld and applies k_scan_cm's rule
// (d = maxk - sum <= tau, canonical home) to append survivors. Sums are exact integers, so the
// survivors equal k_scan_cm's. Every mbarrier wait is bounded; a timeout sets *err and the CTA
// stops issuing MMAs.
constexpr int kMmaQ = 128, kMmaN = 256, kMmaTmemCols = 256;
constexpr uint32_t kMmaMinQueries = 16;  // cells probed by at least this many queries of the batch
constexpr int kHitCap = 256;  // survivors one warp collects before resolving them (>= 32 rows x 8 members)
constexpr size_t kMmaStageBytes = (size_t)kMmaQ * 128 + (size_t)kMmaN * 128;  // A + B per stage
constexpr size_t kMmaSmem = 2 * kMmaStageBytes + 1024;

__global__ void __launch_bounds__(256) k_scan_mma(IndexView ix, QueryEnc e, const uint32_t* __restrict__ start,
                                                  const uint32_t* __restrict__ qof, CellMajorBufs b, uint32_t min_q,
                                                  uint32_t* err) {
    const uint32_t c = blockIdx.x;
    const uint32_t s0 = start[c], s1 = start[c + 1];
    const uint32_t nqc = s1 - s0;
    if (nqc < min_q || nqc == 0) return;
    const uint32_t moff = ix.cell_moff[c];
    const int nc = (int)(ix.cell_moff[c + 1] - moff);
    if (nc == 0) return;
    extern __shared__ uint8_t mraw[];
    __shared__ uint64_t bar[2];
    __shared__ uint32_t s_tmem;
    __shared__ uint32_t s_q[kMmaQ];
    __shared__ uint32_t s_hit[8][kHitCap];
    __shared__ uint32_t s_lc[kMmaQ][kLad / 2];  // per row: survivors under each rung, two u16 per word
    __shared__ uint8_t s_r0[kMmaQ];             // per row: the first rung below its cut-off
    const uint32_t sbase = umma::smem_addr(mraw);
    uint8_t* tiles = mraw + (((sbase + 1023u) & ~1023u) - sbase);
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int npos = ix.npos, kchunks = npos >> 3, ng = (nc + 7) >> 3;
    const uint32_t* codes = ix.cell_codes + ix.cell_woff[c];
    const uint32_t maxk = ix.maxk;
    if (warp == 0) umma::tmem_alloc(&s_tmem, kMmaTmemCols);
    for (int i = tid; i < kMmaQ * (kLad / 2); i += 256) (&s_lc[0][0])[i] = 0;
    if (tid == 0) {
        umma::bar_init(&bar[0], 1);
        umma::bar_init(&bar[1], 1);
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    umma::fence_before_sync();
    __syncthreads();
    umma::fence_after_sync();
    const uint32_t tmem = s_tmem;
    const uint32_t idesc = umma::idesc_u8_s32(kMmaQ, kMmaN);
    uint32_t it = 0;  // chunks issued so far (stage = it & 1)
    bool ok = true;
    // Thread roles in the operand builds: A rows ra + 32u (u < 4) at 16-byte chunk ch; B member
    // group gl at position ch (the 8 lanes of a quarter-warp take the 8 positions of one group, so
    // under the swizzle each store instruction hits all 32 banks once per 128 bytes).
    const int ch = tid & 7, ra = tid >> 3, gl = tid >> 3;
    for (uint32_t qt = 0; qt < nqc && ok; qt += kMmaQ) {
        const int nq_t = (int)min((uint32_t)kMmaQ, nqc - qt);
        for (int mt = 0; mt < nc && ok; mt += kMmaN) {
            __syncthreads();  // the previous tile's epilogue is done with s_q and the accumulator
            if (tid < nq_t) s_q[tid] = qof[s0 + qt + tid];
            __syncthreads();
            const uint8_t* arow[4];
#pragma unroll
            for (int u = 0; u < 4; ++u) {
                const int r = ra + 32 * u;
                arow[u] = r < nq_t ? e.lut + (size_t)s_q[r] * npos * 16 + ch * 16 : nullptr;
            }
            const int g = (mt >> 3) + gl;
            const uint32_t* bword = 8 * g < nc ? codes + (size_t)ch * ng + g : nullptr;
            // operands of one chunk, loaded a chunk ahead of their use
            struct Ops {
                uint4 a[4];
                uint32_t w;
            };
            auto load = [&](Ops& o, int kc) {
#pragma unroll
                for (int u = 0; u < 4; ++u)
                    if (arow[u]) o.a[u] = __ldg(reinterpret_cast<const uint4*>(arow[u] + (size_t)kc * 128));
                if (bword) o.w = __ldg(bword + (size_t)kc * 8 * ng);
            };
            // writes chunk kc into its stage and issues its MMAs; false when a wait ran out
            auto step = [&](const Ops& o, Ops& nxt, int kc) -> bool {
                const int st = (int)(it & 1);
                bool good = true;
                if (it >= 2) good = umma::bar_wait(&bar[st], ((it >> 1) - 1) & 1);  // stage free again
                good = __syncthreads_and(good);
                if (!good) return false;
                umma::fence_after_sync();
                uint8_t* sA = tiles + (size_t)st * kMmaStageBytes;
                uint8_t* sB = sA + (size_t)kMmaQ * 128;
#pragma unroll
                for (int u = 0; u < 4; ++u)
                    if (arow[u]) *reinterpret_cast<uint4*>(sA + umma::sw128_offset(ra + 32 * u, ch)) = o.a[u];
                if (bword) {
#pragma unroll
                    for (int bb = 0; bb < 8; ++bb) {
                        const uint32_t nb = (o.w >> (4 * bb)) & 15u;
                        const unsigned long long one = 1ull << (8 * (nb & 7u));
                        ulonglong2 v;
                        v.x = nb < 8 ? one : 0ull;
                        v.y = nb < 8 ? 0ull : one;
                        *reinterpret_cast<ulonglong2*>(sB + umma::sw128_offset(8 * gl + bb, ch)) = v;
                    }
                }
                if (kc + 1 < kchunks) load(nxt, kc + 1);  // in flight while this chunk's MMAs run
                umma::fence_smem_to_async();
                __syncthreads();
                if (tid == 0) {
                    umma::fence_after_sync();
                    const uint32_t a0 = umma::smem_addr(sA), b0 = umma::smem_addr(sB);
#pragma unroll
                    for (int k = 0; k < 4; ++k)
                        umma::mma_i8(tmem, umma::desc_k_sw128(a0 + 32 * k), umma::desc_k_sw128(b0 + 32 * k), idesc,
                                     (kc > 0 || k > 0) ? 1u : 0u);
                    umma::mma_commit(&bar[st]);
                }
                ++it;
                return true;
            };
            Ops o0, o1;
            load(o0, 0);
            for (int kc = 0; kc < kchunks && ok; kc += 2) {
                ok = step(o0, o1, kc);
                if (ok && kc + 1 < kchunks) ok = step(o1, o0, kc + 1);
            }
            if (!ok) break;
            // epilogue: wait for the tile's last chunk, then every warp reads 32 queries x 128 members
            const int lq = warp & 3, half = warp >> 2;
            const int r = 32 * lq + lane;
            const bool vq = r < nq_t;
            const uint32_t t = vq ? *reinterpret_cast<volatile const uint32_t*>(b.gtau + s_q[r]) : 0u;
            if (vq && half == 0) {  // rungs at or above the cut-off are proven already: skip them
                const uint32_t* eq = b.lad + (size_t)s_q[r] * kLadStride;
                int r0 = 0;
#pragma unroll
                for (int l = 0; l < kLad; ++l) r0 += __ldg(eq + l) >= t ? 1 : 0;  // rungs descend
                s_r0[r] = (uint8_t)r0;
            }
            ok = umma::bar_wait(&bar[(it - 1) & 1], ((it - 1) >> 1) & 1);
            ok = __syncthreads_and(ok);
            if (!ok) break;
            umma::fence_after_sync();
            // Survivors (row, member, d) of the warp's 32 rows x 128 members are collected in its
            // shared list and resolved by all 32 lanes together: one chain of dependent loads
            // (slot, lower home, probed bit, counter) per batch instead of one per thread and block.
            uint32_t* hb = s_hit[warp];
            uint32_t cur = 0;  // entries in hb (warp-uniform)
            auto resolve = [&](uint32_t n) {
                __syncwarp();
                for (uint32_t i = lane; i < n; i += 32) {
                    const uint32_t en = hb[i];
                    const uint32_t rr = en >> 24, mm = (en >> 16) & 255u, d = en & 0xFFFFu;
                    const uint32_t qq = s_q[rr], mi = moff + (uint32_t)mt + mm;
                    const uint32_t slot = __ldg(ix.cell_slots + mi);
                    bool keep = true;
                    if (ix.ma > 1) {
                        const uint64_t* pq = b.probed + (size_t)qq * b.mwords;
                        keep = ix.cell_lower ? canonical_lower(__ldg(ix.cell_lower + mi), pq)
                                             : canonical_cm(ix, slot, c, pq);
                    }
                    if (keep) {
                        const uint32_t p = atomicAdd(&b.rest_n[qq], 1u);
                        if (p < (uint32_t)b.rest_cap) b.rest_buf[(size_t)qq * b.rest_cap + p] = ((uint64_t)d << 32) | slot;
                        const uint32_t* eq = b.lad + (size_t)qq * kLadStride;
                        for (int l = s_r0[rr]; l < kLad && d <= __ldg(eq + l); ++l)
                            atomicAdd(&s_lc[rr][l >> 1], 1u << (16 * (l & 1)));
                    }
                }
                __syncwarp();
            };
            for (int cb = 0; cb < 128; cb += 16) {
                uint32_t v[16];
                umma::tmem_ld16(tmem + ((uint32_t)(32 * lq) << 16) + (uint32_t)(128 * half + cb), v);
                umma::tmem_wait_ld();
                const int m0 = mt + 128 * half + cb;
#pragma unroll
                for (int hh = 0; hh < 2; ++hh) {  // 8 columns at a time: at most 256 survivors per batch
                    uint32_t hit = 0;
#pragma unroll
                    for (int j = 0; j < 8; ++j)
                        if (vq && m0 + 8 * hh + j < nc && maxk - v[8 * hh + j] <= t) hit |= 1u << j;
                    const uint32_t nh = (uint32_t)__popc(hit);
                    const uint32_t tot = __reduce_add_sync(0xFFFFFFFFu, nh);
                    if (tot == 0) continue;
                    if (cur + tot > (uint32_t)kHitCap) {
                        resolve(cur);
                        cur = 0;
                    }
                    uint32_t pre = nh;  // inclusive prefix over lanes
#pragma unroll
                    for (int o = 1; o < 32; o <<= 1) {
                        const uint32_t y = __shfl_up_sync(0xFFFFFFFFu, pre, o);
                        if (lane >= o) pre += y;
                    }
                    uint32_t pos = cur + pre - nh;
                    const uint32_t mbase = (uint32_t)(128 * half + cb + 8 * hh);
#pragma unroll
                    for (int j = 0; j < 8; ++j) {
                        if (!((hit >> j) & 1u)) continue;
                        hb[pos++] = ((uint32_t)r << 24) | ((mbase + j) << 16) | (maxk - v[8 * hh + j]);
                    }
                    cur += tot;
                }
            }
            resolve(cur);
            umma::fence_before_sync();
            // the tile's survivors under each rung go to the queries' counters (at most 256 per row
            // and rung, so two u16 counts share a word)
            __syncthreads();
            if (tid < nq_t) ladder_flush(b, s_q[tid], s_lc[tid]);
        }
    }
    if (!ok) {
        if (tid == 0) atomicAdd(err, 1u);
        // let MMAs still in flight finish (bounded) before the accumulator is released
        if (tid == 0 && it > 0) umma::bar_wait(&bar[(it - 1) & 1], ((it - 1) >> 1) & 1);
    }
    umma::fence_before_sync();
    __syncthreads();
    if (warp == 0) umma::tmem_free(tmem, kMmaTmemCols);
}

// ---- cell-major: merge + exact global cut, ties kept (index.rs:2277-2306) ---------------------------

// With W > 0 (cell-range shard) the cut comes from all shards: the target-th smallest distance of
// the all-gathered lists when the shards hold more than target entries together, else no cut
// (xall == nullptr: no rest scan ran, so every shard's seed survivors are already within it).
__global__ void __launch_bounds__(kBS) k_final_cm(CellMajorBufs b, int target, const uint8_t* __restrict__ xall,
                                                  size_t rank_bytes, int W, int nq, int xl) {
    __shared__ uint32_t hist[256];
    const int q = blockIdx.x;
    const uint64_t* sb = b.seed_buf + (size_t)q * b.seed_cap;
    const uint64_t* rb = b.rest_buf + (size_t)q * b.rest_cap;
    int ns = (int)b.seed_n[q];
    int nr = (int)b.rest_n[q];
    if (nr > b.rest_cap) {
        if (threadIdx.x == 0) atomicAdd(b.overflow, 1u);
        nr = b.rest_cap;
    }
    const int total = ns + nr;
    uint32_t D = 0xFFFFFFFFu;
    if (W == 0) {
        if (total > target) D = block_select_d(sb, ns, rb, nr, target, hist);
    } else if (xall) {
        unsigned long long tg = 0;
        for (int r = 0; r < W; ++r) tg += shard_count(xall, rank_bytes, r, q);
        if (tg > (unsigned long long)target) D = block_select_lists(xall, rank_bytes, W, nq, q, xl, target, hist);
    }
    using BS = cub::BlockScan<uint32_t, kBS>;
    __shared__ typename BS::TempStorage scan;
    __shared__ uint32_t s_off;
    if (threadIdx.x == 0) s_off = 0;
    __syncthreads();
    uint32_t* out = b.cand + (size_t)q * b.cand_cap;
    for (int base = 0; base < total; base += kBS) {
        int i = base + threadIdx.x;
        uint64_t key = i < ns ? sb[i] : (i < total ? rb[i - ns] : ~0ull);
        uint32_t f = (i < total && (uint32_t)(key >> 32) <= D) ? 1u : 0u;
        uint32_t pos, agg;
        BS(scan).ExclusiveSum(f, pos, agg);
        uint32_t off = s_off;
        if (f && off + pos < (uint32_t)b.cand_cap) out[off + pos] = (uint32_t)key;
        __syncthreads();
        if (threadIdx.x == 0) s_off = off + agg;
        __syncthreads();
    }
    if (threadIdx.x == 0) b.cand_n[q] = min(s_off, (uint32_t)b.cand_cap);
}

// ---- per-query path (index.rs:1381-1864, FastScan branch) -------------------------------------------

// Probe ranks and the entry segment of every chosen cell.
__global__ void __launch_bounds__(kBS) k_pq_prep(IndexView ix, const uint32_t* __restrict__ chosen,
                                                 const uint32_t* __restrict__ nch, int nprobe, PerQueryBufs b) {
    using BS = cub::BlockScan<uint32_t, kBS>;
    __shared__ typename BS::TempStorage scan;
    __shared__ uint32_t s_run;
    const int q = blockIdx.x, M = ix.M;
    const int n = (int)nch[q];
    uint32_t* crank = b.crank + (size_t)q * M;
    for (int c = threadIdx.x; c < M; c += kBS) crank[c] = kNoCell;
    if (threadIdx.x == 0) s_run = 0;
    __syncthreads();
    for (int i = threadIdx.x; i < n; i += kBS) crank[chosen[(size_t)q * nprobe + i]] = (uint32_t)i;
    uint32_t* so = b.seg_off + (size_t)q * (nprobe + 1);
    for (int base = 0; base < n; base += kBS) {
        int i = base + threadIdx.x;
        uint32_t len = 0;
        if (i < n) {
            uint32_t c = chosen[(size_t)q * nprobe + i];
            len = ix.cell_moff[c + 1] - ix.cell_moff[c];
        }
        uint32_t pos, agg;
        BS(scan).ExclusiveSum(len, pos, agg);
        uint32_t run = s_run;
        if (i < n) so[i] = run + pos;
        __syncthreads();
        if (threadIdx.x == 0) s_run = run + agg;
        __syncthreads();
    }
    if (threadIdx.x == 0) so[n] = s_run;
}

// Every member of every chosen cell: (d << 32 | slot) when canonical under the first-ranked-home
// rule (index.rs:1443-1460) and inside the tag filter (index.rs:1430-1439), else kInvalidEntry.
// One CTA per (probe, query). The query's FastScan table sits in shared memory; for each chunk of
// 32 member groups (256 members) the 8 warps sum disjoint slices of the nibble positions and
// combine their packed 16-bit partials in shared memory (exact: a member's total is at most
// 255 x npos), then every thread resolves one member (slot, tag filter, the per-query exactly-once
// rule against the probe ranks), so the members' dependent loads run side by side.
__global__ void __launch_bounds__(kBS) k_pq_scan(IndexView ix, QueryEnc e, const uint32_t* __restrict__ chosen,
                                                 const uint32_t* __restrict__ nch, int nprobe, int filtering,
                                                 uint32_t flo, uint32_t fhi, PerQueryBufs b) {
    __shared__ __align__(16) uint8_t s_lut[16 * 16 * 16];  // npos <= 256 positions x 16 entries
    __shared__ uint32_t s_part[kBS / 32][32][4];
    const int r = blockIdx.x, q = blockIdx.y;
    if (r >= (int)nch[q]) return;
    const uint32_t* so = b.seg_off + (size_t)q * (nprobe + 1);
    if (so[r + 1] > (uint32_t)b.ent_cap) return;  // reported by the fold
    const uint32_t c = chosen[(size_t)q * nprobe + r];
    const uint32_t moff = ix.cell_moff[c];
    const int nc = (int)(ix.cell_moff[c + 1] - moff);
    const int ng = (nc + 7) >> 3;
    const uint32_t* codes = ix.cell_codes + ix.cell_woff[c];
    const uint32_t* crank = b.crank + (size_t)q * ix.M;
    uint64_t* out = b.ent + (size_t)q * b.ent_cap + so[r];
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, nwarps = kBS / 32;
    const int npos = ix.npos;
    {
        const uint4* src = reinterpret_cast<const uint4*>(e.lut + (size_t)q * npos * 16);
        for (int i = threadIdx.x; i < npos; i += kBS) reinterpret_cast<uint4*>(s_lut)[i] = src[i];
    }
    __syncthreads();
    // this warp's slice of the positions
    const int p0 = (int)((long long)npos * warp / nwarps), p1 = (int)((long long)npos * (warp + 1) / nwarps);
    for (int g0 = 0; g0 < ng; g0 += 32) {
        const int g = g0 + lane;
        const bool act = g < ng;
        uint32_t acc[4];
        group_sums_range(codes, ng, g, act, s_lut, p0, p1, acc);
#pragma unroll
        for (int i = 0; i < 4; ++i) s_part[warp][lane][i] = acc[i];
        __syncthreads();
        // thread t: member 8 * (g0 + t / 8) + t % 8 of this chunk
        {
            const int gl = threadIdx.x >> 3, bb = threadIdx.x & 7;
            const int pos = 8 * (g0 + gl) + bb;
            if (pos < nc) {
                uint32_t tot = 0;
#pragma unroll
                for (int w = 0; w < nwarps; ++w) tot += s_part[w][gl][bb >> 1];
                const uint32_t sum = (tot >> (16 * (bb & 1))) & 0xFFFFu;
                const uint32_t d = ix.maxk - sum;
                const uint32_t slot = __ldg(ix.cell_slots + moff + pos);
                bool ok = true;
                if (filtering) {
                    const uint32_t tg = __ldg(ix.tags + slot);
                    ok = tg >= flo && tg <= fhi;
                }
                if (ok && ix.ma > 1) {
                    const uint32_t* hs = ix.slot_cells + (size_t)slot * ix.ma;
                    for (int j = 0; j < ix.ma; ++j) {
                        const uint32_t h = __ldg(hs + j);
                        if (h != kNoCell && h != c) {
                            const uint32_t rh = __ldg(crank + h);
                            if (rh != kNoCell && rh < (uint32_t)r) {
                                ok = false;
                                break;
                            }
                        }
                    }
                }
                out[pos] = ok ? (((uint64_t)d << 32) | slot) : kInvalidEntry;
            }
        }
        __syncthreads();  // s_part is rewritten by the next chunk
    }
}

// The sequential part of the per-query scan: cells in probe order feed a bucket queue on d >> 6
// with a falling cut-off tau, and the scan stops once no later cell can reach the current
// want0-th best (index.rs:1630-1679). tau after any prefix of cells is the target-th smallest
// bucket among that prefix's surviving entries, so whole cells are folded at once.
__global__ void __launch_bounds__(kBS) k_pq_fold(IndexView ix, QueryEnc e, const uint32_t* __restrict__ chosen,
                                                 const float* __restrict__ cscore, const uint32_t* __restrict__ nch,
                                                 int nprobe, int target, int adaptive, float at_margin,
                                                 PerQueryBufs b) {
    extern __shared__ uint32_t sh[];
    const int nb = (int)(ix.maxk >> 6) + 1;
    uint32_t* hist = sh;              // nb buckets
    float* suffix = reinterpret_cast<float*>(sh + nb);  // nprobe + 1
    __shared__ uint32_t s_add, s_tau, s_stop, s_cnt;
    __shared__ unsigned long long s_kept;
    __shared__ uint32_t hist256[256];
    const int q = blockIdx.x;
    const int n = (int)nch[q];
    const uint32_t* so = b.seg_off + (size_t)q * (nprobe + 1);
    const uint64_t* ent = b.ent + (size_t)q * b.ent_cap;
    if (so[n] > (uint32_t)b.ent_cap) {
        if (threadIdx.x == 0) {
            atomicAdd(b.overflow, 1u);
            b.cand_n[q] = 0;
        }
        return;
    }
    for (int i = threadIdx.x; i < nb; i += kBS) hist[i] = 0;
    if (adaptive) {
        // suffix[i] = max bound over cells i..n-1 (index.rs:1467-1490)
        for (int i = threadIdx.x; i < n; i += kBS)
            suffix[i] = cell_bound(cscore[(size_t)q * nprobe + i], ix.r_bound[chosen[(size_t)q * nprobe + i]]);
        if (threadIdx.x == 0) suffix[n] = -INFINITY;
        __syncthreads();
        if (threadIdx.x == 0)
            for (int i = n - 1; i >= 0; --i) suffix[i] = fmaxf(suffix[i], suffix[i + 1]);
    }
    if (threadIdx.x == 0) {
        s_tau = ix.maxk >> 6;
        s_kept = 0;
        s_add = 0;
        s_stop = (uint32_t)n;
    }
    __syncthreads();
    const float norm = fs_norm(ix.dim_pad);
    const float delta = e.fs_delta[q], bias = e.fs_bias[q];
    for (int r = 0; r < n; ++r) {
        const uint32_t tau = s_tau;
        for (uint32_t i = so[r] + threadIdx.x; i < so[r + 1]; i += kBS) {
            uint64_t k = ent[i];
            if (k == kInvalidEntry) continue;
            uint32_t hc = (uint32_t)(k >> 32) >> 6;
            if (hc <= tau) {
                atomicAdd(&hist[hc], 1u);
                atomicAdd(&s_add, 1u);
            }
        }
        __syncthreads();
        // the falling cut-off: the smallest bucket t (not above the current one) whose prefix count
        // still reaches target, i.e. the sequential walk down from tau done as one warp scan
        if (threadIdx.x < 32) {
            const unsigned long long kept0 = s_kept + s_add;
            const uint32_t t0 = s_tau;
            uint32_t t = t0;
            unsigned long long kept = kept0;
            if (kept0 >= (unsigned long long)target && t0 > 0) {
                const int cut = warp_hist_cut(hist, (int)t0, (long long)target);
                unsigned long long below = 0;  // prefix(cut), summed by the warp
                for (int i = threadIdx.x; i <= cut; i += 32) below += hist[i];
#pragma unroll
                for (int o = 16; o > 0; o >>= 1) below += __shfl_xor_sync(0xFFFFFFFFu, below, o);
                t = (uint32_t)cut;
                kept = below;
            }
            if (threadIdx.x == 0) {
                s_add = 0;
                s_kept = kept;
                s_tau = t;
            }
        }
        __syncthreads();
        if (threadIdx.x == 0) {
            const unsigned long long kept = s_kept;
            const uint32_t t = s_tau;
            if (adaptive && kept >= (unsigned long long)target) {
                uint32_t wsub = ((t + 1) << 6) - 1;
                uint32_t worst = ix.maxk > wsub ? ix.maxk - wsub : 0u;
                float thr = clampf(__fdiv_rn(fs_estimate(delta, bias, worst), norm), -1.0f, 1.0f);
                if (suffix[r + 1] < __fsub_rn(thr, at_margin)) s_stop = (uint32_t)(r + 1);
            }
        }
        __syncthreads();
        if (s_stop != (uint32_t)n) break;
    }
    // candidates: entries of the scanned cells with bucket <= tau (index.rs:1680-1685)
    const uint32_t tau = s_tau, end = so[s_stop];
    uint64_t* keys = b.ent + (size_t)q * b.ent_cap;  // compacted in place (order-free)
    using BS = cub::BlockScan<uint32_t, kBS>;
    __shared__ typename BS::TempStorage scan;
    if (threadIdx.x == 0) s_cnt = 0;
    __syncthreads();
    for (uint32_t base = 0; base < end; base += kBS) {
        uint32_t i = base + threadIdx.x;
        uint64_t k = i < end ? ent[i] : kInvalidEntry;
        uint32_t f = (k != kInvalidEntry && ((uint32_t)(k >> 32) >> 6) <= tau) ? 1u : 0u;
        uint32_t pos, agg;
        BS(scan).ExclusiveSum(f, pos, agg);
        __syncthreads();
        uint32_t off = s_cnt;
        if (f) keys[off + pos] = k;
        __syncthreads();
        if (threadIdx.x == 0) s_cnt = off + agg;
        __syncthreads();
    }
    const int cnt = (int)s_cnt;
    // top want0 (= target) by d; ties at the cut broken by ascending slot (index.rs:1689-1691)
    uint64_t K = ~0ull;
    if (cnt > target) K = block_select_kth(keys, cnt, nullptr, 0, target, 5, 0, hist256);
    if (threadIdx.x == 0) s_cnt = 0;
    __syncthreads();
    uint32_t* out = b.cand + (size_t)q * b.cand_cap;
    for (int base = 0; base < cnt; base += kBS) {
        int i = base + threadIdx.x;
        uint64_t k = i < cnt ? keys[i] : ~0ull;
        uint32_t f = (i < cnt && k <= K) ? 1u : 0u;
        uint32_t pos, agg;
        BS(scan).ExclusiveSum(f, pos, agg);
        uint32_t off = s_cnt;
        if (f && off + pos < (uint32_t)b.cand_cap) out[off + pos] = (uint32_t)k;
        __syncthreads();
        if (threadIdx.x == 0) s_cnt = off + agg;
        __syncthreads();
    }
    if (threadIdx.x == 0) b.cand_n[q] = min(s_cnt, (uint32_t)b.cand_cap);
}

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

__device__ __forceinline__ void bulk_row_copy(void* smem_dst, const void* gsrc, uint32_t bytes, uint64_t* bar) {
    asm volatile(
        "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];\n" ::"r"(
            umma::smem_addr(smem_dst)),
        "l"(gsrc), "r"(bytes), "r"(umma::smem_addr(bar))
        : "memory");
}
__device__ __forceinline__ void bar_arrive_expect(uint64_t* bar, uint32_t bytes) {
    uint64_t state;
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 %0, [%1], %2;\n"
                 : "=l"(state)
                 : "r"(umma::smem_addr(bar)), "r"(bytes)
                 : "memory");
    (void)state;
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

namespace {
thread_local KernelClock* t_clock = nullptr;
thread_local cudaError_t t_launch_err = cudaSuccess;
thread_local int t_launch_err_kernel = -1;
std::atomic<unsigned long long> g_launches{0};

// Brackets one kernel launch: counts it, records the first launch error of the calling thread,
// and, with a clock installed, records its events.
struct Tick {
    cudaStream_t st;
    int id;
    bool timed;
    Tick(int i, cudaStream_t s) : st(s), id(i), timed(t_clock && t_clock->wants(i)) {
        g_launches.fetch_add(1, std::memory_order_relaxed);
        if (timed) t_clock->begin(id, st);
    }
    ~Tick() {
        cudaError_t e = cudaGetLastError();
        if (e != cudaSuccess && t_launch_err == cudaSuccess) {
            t_launch_err = e;
            t_launch_err_kernel = id;
        }
        if (timed) t_clock->end(st);
    }
};
}  // namespace

cudaError_t take_launch_error(int* kernel) {
    cudaError_t e = t_launch_err;
    if (kernel) *kernel = t_launch_err_kernel;
    t_launch_err = cudaSuccess;
    t_launch_err_kernel = -1;
    return e;
}

const char* kernel_name(int id) {
    static const char* names[kNumKernels] = {"k_encode", "k_route_flat", "k_route_tree", "k_rescore_select",
                                             "k_seed",   "k_inv_count",  "k_inv_scan",   "k_inv_scatter",
                                             "k_scan_cm", "k_final_cm",  "k_pq_prep",    "k_pq_scan",
                                             "k_pq_fold", "k_rerank",    "k_topk",       "k_rerank_items",
                                             "k_seed_finish", "k_local_list", "k_merge_topk", "k_scan_mma",
                                             "k_seed_scan", "nccl_all_gather"};
    return id >= 0 && id < kNumKernels ? names[id] : "?";
}

KernelClock::~KernelClock() {
    for (auto& m : pending) {
        cudaEventDestroy(m.a);
        cudaEventDestroy(m.b);
    }
    for (auto e : pool) cudaEventDestroy(e);
}

cudaEvent_t KernelClock::take() {
    if (!pool.empty()) {
        cudaEvent_t e = pool.back();
        pool.pop_back();
        return e;
    }
    cudaEvent_t e = nullptr;
    cudaEventCreate(&e);
    return e;
}

void KernelClock::begin(int id, cudaStream_t st) {
    Mark m{id, take(), take()};
    cudaEventRecord(m.a, st);
    pending.push_back(m);
    launches[id] += 1;
}

void KernelClock::end(cudaStream_t st) {
    if (!pending.empty()) cudaEventRecord(pending.back().b, st);
}

void KernelClock::collect() {
    for (auto& m : pending) {
        float t = 0.0f;
        if (cudaEventSynchronize(m.b) == cudaSuccess && cudaEventElapsedTime(&t, m.a, m.b) == cudaSuccess)
            ms[m.id] += t;
        pool.push_back(m.a);
        pool.push_back(m.b);
    }
    pending.clear();
}

void set_thread_clock(KernelClock* c) { t_clock = c; }
void clock_begin(int id, cudaStream_t st) {
    if (t_clock && t_clock->wants(id)) t_clock->begin(id, st);
}
void clock_end(int id, cudaStream_t st) {
    if (t_clock && t_clock->wants(id)) t_clock->end(st);
}
unsigned long long total_launches() { return g_launches.load(); }

// The 48 KiB default covers static plus dynamic shared memory, so any dynamic request opts in to
// its exact size; a refused opt-in surfaces as the launch error recorded by Tick.
static void set_smem(const void* f, size_t bytes) {
    if (bytes > 0) cudaFuncSetAttribute(f, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)bytes);
}

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

void launch_route_all(const IndexView& ix, int nq, uint32_t* sl, uint32_t* sl_n, int sl_cap, cudaStream_t st) {
    if (nq <= 0) return;
    QueryEnc e{};
    Tick tk(kKRouteFlat, st);
    k_route_flat<0><<<(nq + kRouteQB - 1) / kRouteQB, kBS, 0, st>>>(ix, e, nq, 0, 1, 0, nullptr, sl, sl_n, sl_cap);
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
                           uint32_t* rs_items, int expect_n, cudaStream_t st) {
    if (nq <= 0) return;
    const int mode = use_sq8 ? 1 : 0;
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
    if (rs_scores && rs_items && row_bytes % 16 == 0) {
        // scores of every (query, shortlist cell) pair by the flattened register gather, then a
        // per-query selection
        const void* fn = mode == 1 ? (const void*)k_rescore_dots<1> : (const void*)k_rescore_dots<0>;
        const size_t smem = (size_t)8 * ((ix.dim + 3) & ~3) * sizeof(float);
        set_smem(fn, smem);
        int dev = 0, sms = 148, per_sm = 1;
        cudaGetDevice(&dev);
        cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
        if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, fn, 256, smem) != cudaSuccess || per_sm < 1)
            per_sm = 1;
        const RowSrc src{ix.dim, use_sq8 ? e.cqs : Q, e.cqbase, ix.cent_f32, ix.cent_sq8};
        {
            Tick tk(kKRescore, st);
            k_rerank_items<<<1, 1024, 0, st>>>(sl_n, nq, gather_rows(mode), rs_items);
            if (mode == 1)
                k_rescore_dots<1><<<sms * per_sm, 256, smem, st>>>(src, sl, sl_n, rs_items, nq, sl_cap, rs_scores);
            else
                k_rescore_dots<0><<<sms * per_sm, 256, smem, st>>>(src, sl, sl_n, rs_items, nq, sl_cap, rs_scores);
        }
        const int small = std::max(next_pow2(std::max(nprobe, 1)), 1024);
        if (small <= kSortCap) {
            const size_t psm = (size_t)small * sizeof(uint64_t);
            set_smem((const void*)k_probe_select, psm);
            Tick tk(kKRescore, st);
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

void launch_seed(const IndexView& ix, const QueryEnc& e, int nq, const uint32_t* chosen, const float* cscore,
                 const uint32_t* nch, int nprobe, int target, bool adaptive, float at_margin, const CellMajorBufs& b,
                 uint16_t* xlist, uint32_t* xcnt, int xl, cudaStream_t st) {
    if (nq <= 0) return;
    {
        Tick tk(kKSeedScan, st);
        k_seed_scan<<<dim3(nq, std::max(ix.seed_parts, 1)), kSeedScanThreads, (size_t)ix.npos * 16, st>>>(
            ix, e, chosen, nch, nprobe, b);
    }
    // a shard keeps its seed keys in the global buffer: k_seed_finish filters them after the exchange
    const int smem_keys = xlist ? 0 : std::min(b.seed_cap, kSeedSmemKeys);
    const int smem_bits = ix.ma > 1 && b.mwords <= kSeedSmemBitmapWords ? 1 : 0;
    const size_t smem = ((size_t)smem_keys + (smem_bits ? (size_t)b.mwords : 0)) * sizeof(uint64_t);
    set_smem((const void*)k_seed, smem);
    Tick tk(kKSeed, st);
    const int final_cand = !xlist && nprobe <= kSeedCells ? 1 : 0;
    k_seed<<<nq, kBS, smem, st>>>(ix, e, chosen, cscore, nch, nprobe, target, adaptive ? 1 : 0, at_margin, b,
                                  smem_keys, smem_bits, final_cand, xlist, xcnt, xl);
}

void launch_seed_finish(const IndexView& ix, const QueryEnc& e, int nq, const uint32_t* chosen, const float* cscore,
                        const uint32_t* nch, int nprobe, int target, bool adaptive, float at_margin,
                        const CellMajorBufs& b, const uint8_t* xall, size_t rank_bytes, int W, int xl,
                        cudaStream_t st) {
    if (nq <= 0) return;
    Tick tk(kKSeedFinish, st);
    k_seed_finish<<<nq, kBS, 0, st>>>(ix, e, chosen, cscore, nch, nprobe, target, adaptive ? 1 : 0, at_margin, b,
                                      xall, rank_bytes, W, nq, xl);
}

void launch_rest_scan(const IndexView& ix, const QueryEnc& e, int nq, const uint32_t* chosen, const uint32_t* nch,
                      int nprobe, const CellMajorBufs& b, cudaStream_t st) {
    if (nq <= 0 || nprobe <= kSeedCells) return;
    // every probe beyond the seed cells goes through the inverted cell -> queries scan
    cudaMemsetAsync(b.cell_cnt, 0, sizeof(uint32_t) * (ix.M + 1), st);
    cudaMemsetAsync(b.cell_fill, 0, sizeof(uint32_t) * ix.M, st);
    int wb = (nq + 7) / 8;
    { Tick tk(kKInvCount, st);
    k_inv_count<<<wb, kBS, 0, st>>>(chosen, nch, b.rest_hi, nq, nprobe, b.cell_cnt); }
    { Tick tk(kKInvScan, st);
    k_inv_scan<<<1, 1024, 0, st>>>(b.cell_cnt, ix.M); }
    { Tick tk(kKInvScatter, st);
    k_inv_scatter<<<wb, kBS, 0, st>>>(chosen, nch, b.rest_hi, nq, nprobe, b.cell_cnt, b.cell_fill, b.qof); }
    { Tick tk(kKScanCm, st);
    k_scan_cm<<<ix.M, kBS, 0, st>>>(ix, e, b.cell_cnt, b.qof, b, kMmaMinQueries); }
    set_smem((const void*)k_scan_mma, kMmaSmem);
    { Tick tk(kKScanMma, st);
    k_scan_mma<<<ix.M, 256, kMmaSmem, st>>>(ix, e, b.cell_cnt, b.qof, b, kMmaMinQueries, b.overflow + 2); }
}

void launch_local_list(const CellMajorBufs& b, int nq, uint16_t* xlist, uint32_t* xcnt, int xl, cudaStream_t st) {
    if (nq <= 0) return;
    Tick tk(kKLocalList, st);
    k_local_list<<<nq, kBS, 0, st>>>(b, xlist, xcnt, xl);
}

void launch_final(const CellMajorBufs& b, int nq, int target, const uint8_t* xall, size_t rank_bytes, int W, int xl,
                  cudaStream_t st) {
    if (nq <= 0) return;
    Tick tk(kKFinalCm, st);
    k_final_cm<<<nq, kBS, 0, st>>>(b, target, xall, rank_bytes, W, nq, xl);
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

size_t shard_list_block_bytes(int nq, int xl) { return shard_list_bytes(nq, xl); }
size_t shard_topk_block_bytes(int nq, int k) { return shard_topk_bytes(nq, k); }

void launch_cellmajor(const IndexView& ix, const QueryEnc& e, int nq, const uint32_t* chosen, const float* cscore,
                      const uint32_t* nch, int nprobe, int target, bool adaptive, float at_margin,
                      const CellMajorBufs& b, cudaStream_t st) {
    if (nq <= 0) return;
    launch_seed(ix, e, nq, chosen, cscore, nch, nprobe, target, adaptive, at_margin, b, nullptr, nullptr, 0, st);
    if (nprobe <= kSeedCells) return;  // k_seed wrote the candidates: no probes beyond the seed cells
    launch_rest_scan(ix, e, nq, chosen, nch, nprobe, b, st);
    launch_final(b, nq, target, nullptr, 0, 0, 0, st);
}

void launch_perquery(const IndexView& ix, const QueryEnc& e, int nq, const uint32_t* chosen, const float* cscore,
                     const uint32_t* nch, int nprobe, int want0, bool adaptive, float at_margin, bool filtering,
                     uint32_t flo, uint32_t fhi, const PerQueryBufs& b, cudaStream_t st) {
    if (nq <= 0) return;
    { Tick tk(kKPqPrep, st);
    k_pq_prep<<<nq, kBS, 0, st>>>(ix, chosen, nch, nprobe, b); }
    { Tick tk(kKPqScan, st);
    k_pq_scan<<<dim3(nprobe, nq), kBS, 0, st>>>(ix, e, chosen, nch, nprobe, filtering ? 1 : 0, flo, fhi, b); }
    int nb = (int)(ix.maxk >> 6) + 1;
    size_t smem = (size_t)nb * sizeof(uint32_t) + (size_t)(nprobe + 1) * sizeof(float);
    set_smem((const void*)k_pq_fold, smem);
    int target = std::max(want0, 1);
    { Tick tk(kKPqFold, st);
    k_pq_fold<<<nq, kBS, smem, st>>>(ix, e, chosen, cscore, nch, nprobe, target, adaptive ? 1 : 0, at_margin, b); }
}

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
        int dev = 0, sms = 148, per_sm = 1;
        cudaGetDevice(&dev);
        cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
        if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, fn, 256, smem) != cudaSuccess || per_sm < 1)
            per_sm = 1;
        const int grid = sms * per_sm;
        const RowSrc src{ix.dim, ix.rerank_mode == 1 ? e.rqs : Q, e.rbase, ix.vecs_f32, ix.rr_u8};
        // f32 rows of 384 or 768 dimensions: the streamed kernel (the query chain in registers)
        const int rstride = ix.dim + ((8 - ix.dim % 32) + 32) % 32;  // rows of a warp on distinct banks
        const size_t stage_bytes = (size_t)kStreamRows * rstride * sizeof(float);
        const void* sf = nullptr;
        int stages = 0;
        if (ix.rerank_mode == 0 && ix.dim == 384) {
            sf = (const void*)k_rerank_stream<4, 48>;
            stages = 4;
        } else if (ix.rerank_mode == 0 && ix.dim == 768) {
            sf = (const void*)k_rerank_stream<2, 96>;
            stages = 2;
        }
        // the item numbering goes into the stream kernel's shared memory when it fits beside the stages
        const size_t items_bytes = ((size_t)nq + 1) * sizeof(uint32_t);
        const bool local_items = sf && (size_t)stages * stage_bytes + items_bytes <= kStreamSmemMax;
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
                k_rerank_stream<4, 48><<<sms, 256, ssm, st>>>(src, cand, cand_n, io, nq, cand_cap, rstride,
                                                              score_scratch, err);
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
