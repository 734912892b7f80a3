// The per-query path (index.rs search_one :1381-1864): probe ranks, the scan of every probed cell
// (FastScan table sums, or Hamming distances over the flat codes of an index without FastScan
// blocks), and the sequential bucket queue with the adaptive stop.
#include "dev_common.cuh"

namespace maivs {
namespace dev {

namespace {

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

// Tag filter (index.rs:1430-1439) and the per-query exactly-once rule (:1443-1460): false when
// `slot` is filtered out or has another home ranked before probe r of cell c.
__device__ __forceinline__ bool pq_member_ok(const IndexView& ix, uint32_t slot, uint32_t c, int r,
                                             const uint32_t* crank, int filtering, uint32_t flo, uint32_t fhi) {
    if (filtering) {
        const uint32_t tg = __ldg(ix.tags + slot);
        if (tg < flo || tg > fhi) return false;
    }
    if (ix.ma > 1) {
        const uint32_t* hs = ix.slot_cells + (size_t)slot * ix.ma;
        for (int j = 0; j < ix.ma; ++j) {
            const uint32_t h = __ldg(hs + j);
            if (h != kNoCell && h != c) {
                const uint32_t rh = __ldg(crank + h);
                if (rh != kNoCell && rh < (uint32_t)r) return false;
            }
        }
    }
    return true;
}

// Every member of every chosen cell: (d << 32 | slot) when canonical under the first-ranked-home
// rule (index.rs:1443-1460) and inside the tag filter (index.rs:1430-1439), else kInvalidEntry.
// One CTA per (probe, query). The query's FastScan table sits in shared memory; for each chunk of
// 32 member groups (256 members) the 8 warps sum disjoint slices of the nibble positions and
// combine their packed 16-bit partials in shared memory (exact: a member's total is at most
// 255 x npos), then every thread resolves one member (slot, tag filter, the per-query exactly-once
// rule against the probe ranks), so the members' dependent loads run side by side. Under a filter
// the groups whose eight members all fail it are written out as invalid entries up front and only
// the others are summed (the reference sums every block and drops the members afterwards; the
// entries are the same).
constexpr int kPqMaxG = 512;  // member groups of a cell that the filtered scan compacts (4,096 members)

__global__ void __launch_bounds__(kBS) k_pq_scan(IndexView ix, QueryEnc e, const uint32_t* __restrict__ chosen,
                                                 const uint32_t* __restrict__ nch, int nprobe, int filtering,
                                                 uint32_t flo, uint32_t fhi, PerQueryBufs b) {
    __shared__ __align__(16) uint8_t s_lut[16 * 16 * 16];  // npos <= 256 positions x 16 entries
    __shared__ uint32_t s_part[kBS / 32][32][4];
    __shared__ uint16_t s_gl[kPqMaxG];
    __shared__ int s_nact;
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
    const bool compact = filtering && ng <= kPqMaxG;
    if (threadIdx.x == 0) s_nact = 0;
    {
        const uint4* src = reinterpret_cast<const uint4*>(e.lut + (size_t)q * npos * 16);
        for (int i = threadIdx.x; i < npos; i += kBS) reinterpret_cast<uint4*>(s_lut)[i] = src[i];
    }
    __syncthreads();
    if (compact) {
        for (int g = threadIdx.x; g < ng; g += kBS) {
            bool any = false;
            for (int bb = 0; bb < 8; ++bb) {
                const int pos = 8 * g + bb;
                if (pos < nc) {
                    const uint32_t tg = __ldg(ix.tags + __ldg(ix.cell_slots + moff + pos));
                    any |= tg >= flo && tg <= fhi;
                }
            }
            if (any) {
                s_gl[atomicAdd(&s_nact, 1)] = (uint16_t)g;
            } else {
                for (int bb = 0; bb < 8 && 8 * g + bb < nc; ++bb) out[8 * g + bb] = kInvalidEntry;
            }
        }
        __syncthreads();
    }
    const int nact = compact ? s_nact : ng;
    // this warp's slice of the positions
    const int p0 = (int)((long long)npos * warp / nwarps), p1 = (int)((long long)npos * (warp + 1) / nwarps);
    for (int a0 = 0; a0 < nact; a0 += 32) {
        const int ai = a0 + lane;
        const bool act = ai < nact;
        const int g = act ? (compact ? (int)s_gl[ai] : ai) : 0;
        uint32_t acc[4];
        group_sums_range(codes, ng, g, act, s_lut, p0, p1, acc);
#pragma unroll
        for (int i = 0; i < 4; ++i) s_part[warp][lane][i] = acc[i];
        __syncthreads();
        // thread t: member 8 * group(a0 + t / 8) + t % 8 of this chunk
        {
            const int gl = threadIdx.x >> 3, bb = threadIdx.x & 7;
            const int a = a0 + gl;
            const int pos = a < nact ? 8 * (compact ? (int)s_gl[a] : a) + bb : nc;
            if (pos < nc) {
                uint32_t tot = 0;
#pragma unroll
                for (int w = 0; w < nwarps; ++w) tot += s_part[w][gl][bb >> 1];
                const uint32_t sum = (tot >> (16 * (bb & 1))) & 0xFFFFu;
                const uint32_t d = ix.maxk - sum;
                const uint32_t slot = __ldg(ix.cell_slots + moff + pos);
                const bool ok = pq_member_ok(ix, slot, c, r, crank, filtering, flo, fhi);
                out[pos] = ok ? (((uint64_t)d << 32) | slot) : kInvalidEntry;
            }
        }
        __syncthreads();  // s_part is rewritten by the next chunk
    }
}

// The Hamming scan of an index without compacted FastScan blocks (index.rs:1693-1790): every
// member of every chosen cell as (h << 32 | slot), h = popcount(query code ^ member code) over the
// flat codes (quantize.rs:183-201), under the same filter and exactly-once rules. One CTA per
// (probe, query); a thread scores one member at a time, the query's code in shared memory. The
// members of a compacted cell are consecutive slots, so a warp's code reads are one contiguous run.
__global__ void __launch_bounds__(kBS) k_pq_scan_ham(IndexView ix, QueryEnc e, const uint32_t* __restrict__ chosen,
                                                     const uint32_t* __restrict__ nch, int nprobe, int filtering,
                                                     uint32_t flo, uint32_t fhi, PerQueryBufs b) {
    __shared__ uint64_t s_q[16];  // nw <= 16 words
    const int r = blockIdx.x, q = blockIdx.y;
    if (r >= (int)nch[q]) return;
    const uint32_t* so = b.seg_off + (size_t)q * (nprobe + 1);
    if (so[r + 1] > (uint32_t)b.ent_cap) return;  // reported by the fold
    const uint32_t c = chosen[(size_t)q * nprobe + r];
    const uint32_t moff = ix.cell_moff[c];
    const int nc = (int)(ix.cell_moff[c + 1] - moff);
    const int nw = ix.nw;
    if (threadIdx.x < nw) s_q[threadIdx.x] = e.qbits[(size_t)q * nw + threadIdx.x];
    __syncthreads();
    const uint32_t* crank = b.crank + (size_t)q * ix.M;
    uint64_t* out = b.ent + (size_t)q * b.ent_cap + so[r];
    for (int pos = threadIdx.x; pos < nc; pos += kBS) {
        const uint32_t slot = __ldg(ix.cell_slots + moff + pos);
        uint64_t entry = kInvalidEntry;
        if (pq_member_ok(ix, slot, c, r, crank, filtering, flo, fhi)) {  // the code is read only when kept
            const uint64_t* code = ix.bits + (size_t)slot * nw;
            uint32_t h = 0;
            for (int w = 0; w < nw; ++w) h += (uint32_t)__popcll(s_q[w] ^ __ldg(code + w));
            entry = ((uint64_t)h << 32) | slot;
        }
        out[pos] = entry;
    }
}

// score_to_cos(hamming_score(tau, dp)) of the binary scan (index.rs:1139-1164, quantize.rs:206-208):
// s = dp - 2 tau, h = (dp - s) / 2, cos(pi h / dp), each step rounded to f32 as the reference does;
// the cosine is rounded once from double precision (as cell_bound's).
__device__ __forceinline__ float ham_tau_cos(uint32_t tau, uint32_t dp) {
    const float dpf = (float)dp;
    const float s = __fsub_rn(dpf, __fmul_rn(2.0f, (float)tau));
    const float h = __fmul_rn(__fsub_rn(dpf, s), 0.5f);
    const float x = __fdiv_rn(__fmul_rn(3.14159274101257324f, h), dpf);
    return (float)cos((double)x);
}

// The sequential part of the per-query scan: cells in probe order feed a bucket queue with a
// falling cut-off tau, and the scan stops once no later cell can reach the current want0-th best.
// FastScan (kHam = false, index.rs:1630-1692): buckets d >> 6, the stop threshold from the table
// estimate of the bucket's worst distance, then the top want0 by exact d. Hamming (kHam = true,
// :1693-1848): buckets are the distances themselves, the threshold is score_to_cos of tau, and
// every entry at or below the final tau is a candidate (ties kept).
// tau after cells 0..r is the target-th smallest bucket over those cells' surviving entries (the
// sequential walk's falling cut-off depends only on that multiset), and "kept >= target" is "at
// least target entries so far", so the stop rule is decided for kFoldG cells at once: each cell of
// the round gets its own histogram layer, the layers are made cumulative in place (layer w = the
// running histogram plus cells 0..w of the round), warp w takes the cut-off of layer w, and the
// first cell whose stop rule holds ends the scan. Without adaptive probing every probe is scanned
// and the cut-off is computed once. Entries are read kFoldU per thread with independent loads.
constexpr int kFoldG = kBS / 32;
constexpr int kFoldU = 8;
constexpr int kFoldEqMax = 1024;  // entries of the cut-off bucket ranked directly

// Histogram of the entries [i0, i1) by bucket: into hist[b], or, with s_so (the round's cell
// offsets, ng cells), into the layer of the entry's cell, hist + layer * hs.
template <int kShift>
__device__ __forceinline__ void fold_count(const uint64_t* __restrict__ ent, uint32_t i0, uint32_t i1, uint32_t* hist,
                                           const uint32_t* s_so, int hs) {
    for (uint32_t base = i0 + threadIdx.x; base < i1; base += kBS * kFoldU) {
        uint64_t kk[kFoldU];
#pragma unroll
        for (int u = 0; u < kFoldU; ++u) {
            const uint32_t i = base + (uint32_t)u * kBS;
            kk[u] = i < i1 ? ent[i] : kInvalidEntry;
        }
#pragma unroll
        for (int u = 0; u < kFoldU; ++u) {
            if (kk[u] == kInvalidEntry) continue;
            const uint32_t i = base + (uint32_t)u * kBS;
            int l = 0;
            if (s_so)
                while (i >= s_so[l + 1]) ++l;
            atomicAdd(&hist[l * hs + ((uint32_t)(kk[u] >> 32) >> kShift)], 1u);
        }
    }
}

template <bool kHam>
__global__ void __launch_bounds__(kBS) k_pq_fold(IndexView ix, QueryEnc e, const uint32_t* __restrict__ chosen,
                                                 const float* __restrict__ cscore, const uint32_t* __restrict__ nch,
                                                 int nprobe, int target, int adaptive, float at_margin,
                                                 PerQueryBufs b) {
    extern __shared__ uint32_t sh[];
    constexpr int kShift = kHam ? 0 : 6;
    const uint32_t top = kHam ? (uint32_t)ix.nw * 64u : ix.maxk >> 6;  // the largest bucket
    const int nb = (int)top + 1;
    const int hs = (nb + 3) & ~3;
    uint32_t* run = sh;                                                      // nb buckets: cells before the round
    uint32_t* layers = sh + hs;                                              // kFoldG x hs: the round's cells
    float* suffix = reinterpret_cast<float*>(sh + (size_t)(kFoldG + 1) * hs);  // nprobe + 1
    __shared__ uint32_t s_tau, s_stop, s_cnt;
    __shared__ uint32_t s_cut[kFoldG], s_flag[kFoldG], s_so[kFoldG + 1];
    __shared__ uint32_t hist256[256];
    const int q = blockIdx.x;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
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
    for (int i = threadIdx.x; i < nb; i += kBS) run[i] = 0;
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
        s_tau = top;
        s_stop = (uint32_t)n;
    }
    __syncthreads();
    if (!adaptive) {
        fold_count<kShift>(ent, 0, so[n], run, nullptr, 0);
        __syncthreads();
        if (warp == 0) {
            long long tot;
            const int cut = warp_cut_layers(run, nullptr, 0, 0, (int)top, (long long)target, &tot);
            if (lane == 0) s_tau = (uint32_t)cut;
        }
        __syncthreads();
    } else {
        const float norm = kHam ? 0.0f : fs_norm(ix.dim_pad);
        const float delta = kHam ? 0.0f : e.fs_delta[q], bias = kHam ? 0.0f : e.fs_bias[q];
        for (int g0 = 0; g0 < n; g0 += kFoldG) {
            const int ng = min(kFoldG, n - g0);
            for (int i = threadIdx.x; i < ng * hs; i += kBS) layers[i] = 0;
            if (threadIdx.x <= ng) s_so[threadIdx.x] = so[g0 + threadIdx.x];
            __syncthreads();
            fold_count<kShift>(ent, s_so[0], s_so[ng], layers, s_so, hs);
            __syncthreads();
            // cumulative in place: layer l = run + cells 0..l of the round
            for (int i = threadIdx.x; i < nb; i += kBS) {
                uint32_t v = run[i];
                for (int l = 0; l < ng; ++l) {
                    v += layers[l * hs + i];
                    layers[l * hs + i] = v;
                }
            }
            __syncthreads();
            if (warp < ng) {
                long long tot;
                const int cut =
                    warp_cut_layers(layers + warp * hs, nullptr, 0, 0, (int)top, (long long)target, &tot);
                if (lane == 0) {
                    uint32_t stop = 0;
                    if (tot >= (long long)target) {
                        const uint32_t t = (uint32_t)cut;
                        float thr;
                        if (kHam) {
                            thr = ham_tau_cos(t, top);
                        } else {
                            const uint32_t wsub = ((t + 1) << 6) - 1;
                            const uint32_t worst = ix.maxk > wsub ? ix.maxk - wsub : 0u;
                            thr = clampf(__fdiv_rn(fs_estimate(delta, bias, worst), norm), -1.0f, 1.0f);
                        }
                        stop = suffix[g0 + warp + 1] < __fsub_rn(thr, at_margin) ? 1u : 0u;
                    }
                    s_cut[warp] = (uint32_t)cut;
                    s_flag[warp] = stop;
                }
            }
            __syncthreads();
            if (threadIdx.x == 0) {
                int w = 0;
                while (w < ng && !s_flag[w]) ++w;
                if (w < ng) {
                    s_stop = (uint32_t)(g0 + w + 1);
                    s_tau = s_cut[w];
                } else {
                    s_tau = s_cut[ng - 1];
                }
            }
            __syncthreads();
            if (s_stop != (uint32_t)n) break;
            for (int i = threadIdx.x; i < nb; i += kBS) run[i] = layers[(ng - 1) * hs + i];
            __syncthreads();
        }
    }
    // candidates: entries of the scanned cells with bucket <= tau (index.rs:1680-1685, :1809-1814)
    const uint32_t tau = s_tau, end = so[s_stop];
    using BS = cub::BlockScan<uint32_t, kBS>;
    __shared__ typename BS::TempStorage scan;
    if (kHam) {
        // every one of them goes to the rerank; more than cand_cap is an overflow (the host
        // enlarges the buffers and searches again)
        uint32_t* out = b.cand + (size_t)q * b.cand_cap;
        if (threadIdx.x == 0) s_cnt = 0;
        __syncthreads();
        for (uint32_t base = 0; base < end; base += kBS) {
            uint32_t i = base + threadIdx.x;
            uint64_t k = i < end ? ent[i] : kInvalidEntry;
            uint32_t f = (k != kInvalidEntry && (uint32_t)(k >> 32) <= tau) ? 1u : 0u;
            uint32_t pos, agg;
            BS(scan).ExclusiveSum(f, pos, agg);
            uint32_t off = s_cnt;
            if (f && off + pos < (uint32_t)b.cand_cap) out[off + pos] = (uint32_t)k;
            __syncthreads();
            if (threadIdx.x == 0) s_cnt = off + agg;
            __syncthreads();
        }
        if (threadIdx.x == 0) {
            if (s_cnt > (uint32_t)b.cand_cap) atomicAdd(b.overflow, 1u);
            b.cand_n[q] = min(s_cnt, (uint32_t)b.cand_cap);
        }
        return;
    }
    uint64_t* keys = b.ent + (size_t)q * b.ent_cap;  // compacted in place (order-free)
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
    // top want0 (= target) by d; ties at the cut broken by ascending slot (index.rs:1689-1691).
    // Every entry of a bucket below tau is in (fewer than target of them); the rest are the
    // smallest keys of bucket tau, ranked directly when that bucket is small.
    uint64_t K = ~0ull;
    if (cnt > target) {
        __shared__ uint64_t s_eq[kFoldEqMax];
        __shared__ uint32_t s_neq;
        __shared__ uint64_t s_k;
        if (threadIdx.x == 0) {
            s_neq = 0;
            s_k = ~0ull;
        }
        __syncthreads();
        for (int i = threadIdx.x; i < cnt; i += kBS) {
            const uint64_t k = keys[i];
            if (((uint32_t)(k >> 32) >> 6) == tau) {
                const uint32_t at = atomicAdd(&s_neq, 1u);
                if (at < (uint32_t)kFoldEqMax) s_eq[at] = k;
            }
        }
        __syncthreads();
        const int neq = (int)s_neq;
        if (neq <= kFoldEqMax) {
            const int need = target - (cnt - neq);  // >= 1: the entries below bucket tau are fewer than target
            for (int i = threadIdx.x; i < neq; i += kBS) {
                const uint64_t k = s_eq[i];
                int r = 0;
                for (int j = 0; j < neq; ++j) r += s_eq[j] < k ? 1 : 0;
                if (r == need - 1) s_k = k;
            }
            __syncthreads();
            K = s_k;
        } else {
            K = block_select_kth(keys, cnt, nullptr, 0, target, 5, 0, hist256);
        }
    }
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

}  // namespace

// ---- launchers ----------------------------------------------------------------------------------------

void launch_perquery(const IndexView& ix, const QueryEnc& e, int nq, const uint32_t* chosen, const float* cscore,
                     const uint32_t* nch, int nprobe, int want0, bool adaptive, float at_margin, bool filtering,
                     uint32_t flo, uint32_t fhi, const PerQueryBufs& b, cudaStream_t st) {
    if (nq <= 0) return;
    { Tick tk(kKPqPrep, st);
    k_pq_prep<<<nq, kBS, 0, st>>>(ix, chosen, nch, nprobe, b); }
    { Tick tk(kKPqScan, st);
    if (ix.ham)
        k_pq_scan_ham<<<dim3(nprobe, nq), kBS, 0, st>>>(ix, e, chosen, nch, nprobe, filtering ? 1 : 0, flo, fhi, b);
    else
        k_pq_scan<<<dim3(nprobe, nq), kBS, 0, st>>>(ix, e, chosen, nch, nprobe, filtering ? 1 : 0, flo, fhi, b); }
    const int nb = ix.ham ? ix.nw * 64 + 1 : (int)(ix.maxk >> 6) + 1;
    const size_t smem = (size_t)(kFoldG + 1) * ((nb + 3) & ~3) * sizeof(uint32_t) + (size_t)(nprobe + 1) * sizeof(float);
    const void* fold = ix.ham ? (const void*)k_pq_fold<true> : (const void*)k_pq_fold<false>;
    set_smem(fold, smem);
    int target = std::max(want0, 1);
    { Tick tk(kKPqFold, st);
    if (ix.ham)
        k_pq_fold<true><<<nq, kBS, smem, st>>>(ix, e, chosen, cscore, nch, nprobe, target, adaptive ? 1 : 0,
                                               at_margin, b);
    else
        k_pq_fold<false><<<nq, kBS, smem, st>>>(ix, e, chosen, cscore, nch, nprobe, target, adaptive ? 1 : 0,
                                                at_margin, b); }
}

}  // namespace dev
}  // namespace maivs
