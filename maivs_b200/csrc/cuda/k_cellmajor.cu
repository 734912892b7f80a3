// The cell-major join (index.rs:1999-2311): the seed step with the adaptive prune and the falling
// cut-off's rungs, the cell -> queries inversion, the FastScan scan of low-batch cells, the exact
// candidate cut, and the distance lists cell-range shards exchange.
#include "dev_common.cuh"

namespace maivs {
namespace dev {

namespace {

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

}  // namespace

// ---- launchers ----------------------------------------------------------------------------------------

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
    launch_scan_mma(ix, e, b, st);
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

size_t shard_list_block_bytes(int nq, int xl) { return shard_list_bytes(nq, xl); }
void launch_cellmajor(const IndexView& ix, const QueryEnc& e, int nq, const uint32_t* chosen, const float* cscore,
                      const uint32_t* nch, int nprobe, int target, bool adaptive, float at_margin,
                      const CellMajorBufs& b, cudaStream_t st) {
    if (nq <= 0) return;
    launch_seed(ix, e, nq, chosen, cscore, nch, nprobe, target, adaptive, at_margin, b, nullptr, nullptr, 0, st);
    if (nprobe <= kSeedCells) return;  // k_seed wrote the candidates: no probes beyond the seed cells
    launch_rest_scan(ix, e, nq, chosen, nch, nprobe, b, st);
    launch_final(b, nq, target, nullptr, 0, 0, 0, st);
}

}  // namespace dev
}  // namespace maivs
