// Device helpers and launch bookkeeping shared by the kernel files of the query path: FastScan
// table sums, the exactly-once rule, block-wide selections, the falling cut-off's rungs, and the
// per-launch clock / error record (clock.cu).
//
// Integer work (codes, table sums, distances, cut-offs) is exact by construction. Floating-point
// work follows the reference's evaluation order (see common.cuh), so scores are bit-identical to
// the reference's CPU path on the same inputs.
#pragma once

#include <cub/block/block_reduce.cuh>
#include <cub/block/block_scan.cuh>

#include "common.cuh"
#include "kernels.cuh"

namespace maivs {
namespace dev {

// ---- launch bookkeeping (clock.cu) ---------------------------------------------------------------
// Counts a launch and, with a clock installed on the calling thread, opens its timing.
bool tick_begin(int id, cudaStream_t st);
// Records the first launch error of the calling thread and closes the timing.
void tick_end(int id, cudaStream_t st, bool timed);
// Brackets one kernel launch (RAII).
struct Tick {
    cudaStream_t st;
    int id;
    bool timed;
    Tick(int i, cudaStream_t s) : st(s), id(i), timed(tick_begin(i, s)) {}
    ~Tick() { tick_end(id, st, timed); }
};
// The 48 KiB default covers static plus dynamic shared memory, so any dynamic request opts in to
// its exact size; a refused opt-in surfaces as the launch error recorded by Tick.
void set_smem(const void* f, size_t bytes);
// Resident CTAs per SM of kernel f (cudaOccupancyMaxActiveBlocksPerMultiprocessor, at least 1) and
// the current device's SM count, both remembered per device.
int blocks_per_sm(const void* f, int threads, size_t smem);
int sm_count();

// ---- launchers of kernels that another stage's launcher starts -----------------------------------
// k_scan_mma (k_scan_mma.cu) over every cell the batch's rest probes hit kMmaMinQueries times or more.
void launch_scan_mma(const IndexView& ix, const QueryEnc& e, const CellMajorBufs& b, cudaStream_t st);
// Centroid re-order scores of every (query, shortlist cell) pair by the flattened register gather
// (k_rerank.cu): item numbering, then k_rescore_dots.
// Centroid re-order scores of every (query, live cell) pair when every shortlist is the live-cell
// list (k_rerank.cu, tiled); false when the rows do not suit it (then nothing was launched).
bool launch_rescore_all(const IndexView& ix, const QueryEnc& e, const float* Q, int nq, bool use_sq8, int cap,
                        float* rs_scores, cudaStream_t st);
void launch_rescore_dots(const IndexView& ix, const QueryEnc& e, const float* Q, int nq, const uint32_t* sl,
                         const uint32_t* sl_n, int sl_cap, bool use_sq8, float* rs_scores, uint32_t* rs_items,
                         cudaStream_t st);

constexpr uint32_t kMmaMinQueries = 16;  // cells probed by at least this many queries of the batch

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


// warp_hist_cut over the composite histogram run[i] + layers[0][i] + ... + layers[nl - 1][i]
// (layer l at layers + l * stride): the smallest t with prefix(t) >= want, bits when never
// reached; *total receives the composite sum over every bucket. Every lane returns the same.
__device__ int warp_cut_layers(const uint32_t* run, const uint32_t* layers, int stride, int nl, int bits,
                               long long want, long long* total) {
    const int lane = threadIdx.x & 31;
    const int nb = bits + 1;
    const int per = (nb + 31) / 32;
    const int b0 = lane * per, b1 = min(b0 + per, nb);
    auto val = [&](int i) -> uint32_t {
        uint32_t v = run[i];
        for (int l = 0; l < nl; ++l) v += layers[l * stride + i];
        return v;
    };
    long long s = 0;
    for (int i = b0; i < b1; ++i) s += val(i);
    long long inc = s;
    for (int o = 1; o < 32; o <<= 1) {
        long long v = __shfl_up_sync(0xFFFFFFFFu, inc, o);
        if (lane >= o) inc += v;
    }
    *total = __shfl_sync(0xFFFFFFFFu, inc, 31);
    const long long excl = inc - s;
    const int found = (excl < want && inc >= want) ? 1 : 0;
    const unsigned bal = __ballot_sync(0xFFFFFFFFu, found);
    int res = bits;
    if (bal) {
        const int src = __ffs(bal) - 1;
        int t = bits;
        if (lane == src) {
            long long c = excl;
            for (int i = b0; i < b1; ++i) {
                c += val(i);
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

}  // namespace

}  // namespace dev
}  // namespace maivs
