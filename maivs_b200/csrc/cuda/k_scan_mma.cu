// The tensor-core scan of high-batch cells in the cell-major join (index.rs:2231-2275 with the
// FastScan sums of quantize.rs:323-386 as a u8 x u8 -> s32 tcgen05 GEMM).
#include "dev_common.cuh"
#include "umma.cuh"

namespace maivs {
namespace dev {

namespace {

// ---- cell-major: the scan of high-batch cells on the tensor cores -----------------------------------
// The FastScan sum of a (query, member) pair is sum_j LUT_q[16 j + nib_j(member)], i.e. the dot
// product of the query's u8 table row (K = 16 x npos bytes) with the one-hot expansion of the
// member's nibbles. For a cell that many queries probe this is a dense u8 x u8 -> s32 GEMM:
// M = 128 queries x N = up to 256 members per tile (the tile's members rounded up to 16, so a
// 100-member cell costs 112 columns of MMA, not 256), K in chunks of 128 bytes (8 nibble
// positions), A (tables) and B (one-hot nibbles) written into shared memory in the K-major
// 128-byte swizzled layout, four kind::i8 tcgen05.mma per chunk into a TMEM accumulator (128 lanes
// x 256 columns allocated).
// The epilogue reads the sums with tcgen05.ld and applies k_scan_cm's rule (d = maxk - sum <= the
// query's falling cut-off, canonical home) to append survivors, counting them under the query's
// rungs. Sums are exact integers, so the survivors equal k_scan_cm's.
//
// Kernel organisation: persistent CTAs, two per SM, take cells from a work counter. Eight producer
// warps write each chunk's operands into one of S stages and arrive on the stage's `full` mbarrier;
// a ninth warp only waits for `full`, issues the chunk's MMAs and commits them to the stage's
// `empty` mbarrier, which the producers wait on before writing that stage again. There is no
// CTA-wide barrier inside the K loop: producers run ahead of the MMAs by up to S chunks, with their
// next chunks' operands in flight in registers, and the two CTAs of an SM overlap each other's tile
// set-up and epilogue. Every wait is bounded; a thread whose wait runs out still arrives where
// others wait on it, the CTA stops at the end of that tile, sets *err, lets its MMAs land (bounded)
// and frees its TMEM.
constexpr int kMmaQ = 128, kMmaN = 256, kMmaTmemCols = 256;
constexpr int kHitCap = 256;  // survivors one warp collects before resolving them (>= 32 rows x 8 members)
constexpr size_t kMmaStageBytes = (size_t)kMmaQ * 128 + (size_t)kMmaN * 128;  // A + B per stage

constexpr int kPAhead = 2;  // chunks whose operands a producer holds in registers

__device__ __forceinline__ void bar_arrive(uint64_t* bar) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(umma::smem_addr(bar)) : "memory");
}

// NPW producer warps build the operands; warp NPW issues the MMAs; S stages. The epilogue splits the
// accumulator over the producer warps: TMEM lane quarter (warp % 4) x an equal slice of the tile's
// columns (warp / 4).
template <int NPW, int S>
struct PScan {
    static constexpr int kProd = NPW * 32;
    static constexpr int kT = kProd + 32;
    static constexpr int kBlocks = NPW == 8 ? 2 : 1;  // CTAs per SM
    static constexpr int kAPer = kMmaQ * 8 / kProd;   // 16-byte A pieces per producer and chunk
    static constexpr int kBMem = kMmaN * 8 / kProd;   // one-hot members per producer and chunk
    static constexpr size_t kSmem = (size_t)S * kMmaStageBytes + 1024;
};

template <int NPW, int S>
__global__ void __launch_bounds__(PScan<NPW, S>::kT, PScan<NPW, S>::kBlocks) k_scan_mma(IndexView ix, QueryEnc e, const uint32_t* __restrict__ start,
                                                      const uint32_t* __restrict__ qof, CellMajorBufs b,
                                                      uint32_t min_q, uint32_t* work, uint32_t* err) {
    using P = PScan<NPW, S>;
    constexpr int kPStages = S, kPWarps = NPW, kPT = P::kT;
    extern __shared__ uint8_t mraw[];
    __shared__ uint64_t full[kPStages], empty[kPStages], done;
    __shared__ uint32_t s_tmem;
    __shared__ uint32_t s_cell[2];
    __shared__ uint32_t s_q[kMmaQ];
    __shared__ uint32_t s_hit[kPWarps][kHitCap];
    __shared__ uint32_t s_lc[kMmaQ][kLad / 2];
    __shared__ uint8_t s_r0[kMmaQ];
    const uint32_t sbase = umma::smem_addr(mraw);
    uint8_t* tiles = mraw + (((sbase + 1023u) & ~1023u) - sbase);
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int npos = ix.npos, kchunks = npos >> 3;
    const uint32_t maxk = ix.maxk, M = (uint32_t)ix.M;
    if (warp == 0) umma::tmem_alloc(&s_tmem, kMmaTmemCols);
    for (int i = tid; i < kMmaQ * (kLad / 2); i += kPT) (&s_lc[0][0])[i] = 0;
    const bool issuer_warp = warp == kPWarps;
    if (tid == 0) {
        for (int i = 0; i < kPStages; ++i) {
            umma::bar_init(&full[i], kPWarps);
            umma::bar_init(&empty[i], 1);
        }
        umma::bar_init(&done, 1);
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    umma::fence_before_sync();
    __syncthreads();
    umma::fence_after_sync();
    const uint32_t tmem = s_tmem;
    // operand roles: A rows ra + (kProd / 8) u at 16-byte chunk ch; B members 8 g + kBMem hh + u at
    // position ch
    const int ch = tid & 7, ra = tid >> 3, g = (tid >> 3) / (8 / P::kBMem), hh = (tid >> 3) % (8 / P::kBMem);
    uint32_t it = 0;     // chunks this CTA has produced (stage it % kPStages)
    uint32_t ntile = 0;  // tiles finished (parity of `done`)
    bool bad = false;
    int par = 0;
    for (;;) {
        if (tid == 0) s_cell[par] = atomicAdd(work, 1u);
        __syncthreads();
        const uint32_t c = s_cell[par];
        par ^= 1;
        if (c >= M) break;
        const uint32_t s0 = start[c], s1 = start[c + 1];
        const uint32_t nqc = s1 - s0;
        const uint32_t moff = ix.cell_moff[c];
        const int nc = (int)(ix.cell_moff[c + 1] - moff);
        if (nqc < min_q || nqc == 0 || nc == 0) continue;
        const int ng = (nc + 7) >> 3;
        const uint32_t* codes = ix.cell_codes + ix.cell_woff[c];
        for (uint32_t qt = 0; qt < nqc && !bad; qt += kMmaQ) {
            const int nq_t = (int)min((uint32_t)kMmaQ, nqc - qt);
            for (int mt = 0; mt < nc && !bad; mt += kMmaN) {
                // the MMAs cover only this tile's members, rounded up to the M = 128 step of N (16)
                const int n_tile = (min(kMmaN, nc - mt) + 15) & ~15;
                const uint32_t idesc = umma::idesc_u8_s32(kMmaQ, n_tile);
                __syncthreads();  // the previous tile's epilogue is done with s_q, s_r0 and the accumulator
                if (tid < nq_t) {
                    const uint32_t q = qof[s0 + qt + tid];
                    s_q[tid] = q;
                    // rungs at or above the query's cut-off are proven already: the epilogue skips them
                    const uint32_t t0 = *reinterpret_cast<volatile const uint32_t*>(b.gtau + q);
                    const uint32_t* eq = b.lad + (size_t)q * kLadStride;
                    int r0 = 0;
#pragma unroll
                    for (int l = 0; l < kLad; ++l) r0 += __ldg(eq + l) >= t0 ? 1 : 0;
                    s_r0[tid] = (uint8_t)r0;
                }
                __syncthreads();
                if (issuer_warp) {
                    // the MMA issuer: wait for a chunk's operands, issue its four MMAs, free the stage
                    for (int kc = 0; kc < kchunks; ++kc) {
                        const uint32_t ic = it + (uint32_t)kc;
                        const int st = (int)(ic % kPStages);
                        if (lane == 0) {
                            const bool ok = !bad && umma::bar_wait(&full[st], (ic / kPStages) & 1);
                            if (ok) {
                                umma::fence_after_sync();
                                const uint8_t* sA = tiles + (size_t)st * kMmaStageBytes;
                                const uint32_t ad = umma::smem_addr(sA), bd = umma::smem_addr(sA + (size_t)kMmaQ * 128);
#pragma unroll
                                for (int k = 0; k < 4; ++k)
                                    umma::mma_i8(tmem, umma::desc_k_sw128(ad + 32 * k),
                                                 umma::desc_k_sw128(bd + 32 * k), idesc, (kc > 0 || k > 0) ? 1u : 0u);
                            } else {
                                bad = true;
                            }
                            umma::mma_commit(&empty[st]);  // arrives when the MMAs issued so far are done
                            if (kc + 1 == kchunks) umma::mma_commit(&done);
                        }
                    }
                    bad = __shfl_sync(0xFFFFFFFFu, bad ? 1 : 0, 0) != 0;
                } else {
                    const uint8_t* ap[P::kAPer];
#pragma unroll
                    for (int u = 0; u < P::kAPer; ++u) {
                        const int r = ra + (P::kProd / 8) * u;
                        ap[u] = r < nq_t ? e.lut + (size_t)s_q[r] * npos * 16 + ch * 16 : nullptr;
                    }
                    const int gg = (mt >> 3) + g;
                    const uint32_t* bword = 8 * gg < nc ? codes + (size_t)ch * ng + gg : nullptr;
                    // operands of the next kPAhead chunks, in flight while earlier chunks are written
                    uint4 qa[kPAhead][P::kAPer];
                    uint32_t qb[kPAhead];
                    auto load = [&](int kc, uint4 (&x)[P::kAPer], uint32_t& w) {
#pragma unroll
                        for (int u = 0; u < P::kAPer; ++u)
                            if (ap[u]) x[u] = __ldg(reinterpret_cast<const uint4*>(ap[u] + (size_t)kc * 128));
                        if (bword) w = __ldg(bword + (size_t)kc * 8 * ng);
                    };
#pragma unroll
                    for (int j = 0; j < kPAhead; ++j) {
                        qb[j] = 0;
                        if (j < kchunks) load(j, qa[j], qb[j]);
                    }
                    for (int kc0 = 0; kc0 < kchunks; kc0 += kPAhead) {
#pragma unroll
                        for (int j = 0; j < kPAhead; ++j) {
                            const int kc = kc0 + j;
                            if (kc >= kchunks) break;
                            const uint32_t ic = it + (uint32_t)kc;
                            const int st = (int)(ic % kPStages);
                            if (ic >= (uint32_t)kPStages) {  // the MMAs that last read this stage are done
                                bool ok = true;
                                if (lane == 0) ok = umma::bar_wait(&empty[st], ((ic / kPStages) - 1) & 1);
                                if (!__shfl_sync(0xFFFFFFFFu, ok ? 1 : 0, 0)) bad = true;
                            }
                            uint8_t* sA = tiles + (size_t)st * kMmaStageBytes;
                            uint8_t* sB = sA + (size_t)kMmaQ * 128;
                            if (!bad) {
#pragma unroll
                                for (int u = 0; u < P::kAPer; ++u)
                                    if (ap[u])
                                        *reinterpret_cast<uint4*>(sA + umma::sw128_offset(ra + (P::kProd / 8) * u, ch)) =
                                            qa[j][u];
                                if (bword) {
#pragma unroll
                                    for (int u = 0; u < P::kBMem; ++u) {
                                        const int bb = P::kBMem * hh + u;
                                        const uint32_t nb = (qb[j] >> (4 * bb)) & 15u;
                                        const unsigned long long one = 1ull << (8 * (nb & 7u));
                                        ulonglong2 v;
                                        v.x = nb < 8 ? one : 0ull;
                                        v.y = nb < 8 ? 0ull : one;
                                        *reinterpret_cast<ulonglong2*>(sB + umma::sw128_offset(8 * g + bb, ch)) = v;
                                    }
                                }
                                umma::fence_smem_to_async();
                            }
                            __syncwarp();
                            if (lane == 0) bar_arrive(&full[st]);
                            if (kc + kPAhead < kchunks) load(kc + kPAhead, qa[j], qb[j]);
                        }
                    }
                }
                it += (uint32_t)kchunks;
                // epilogue: every warp reads 32 rows (its TMEM lane quarter) x 64 columns
                {
                    bool ok = true;
                    if (lane == 0) ok = umma::bar_wait(&done, ntile & 1);
                    if (!__shfl_sync(0xFFFFFFFFu, ok ? 1 : 0, 0)) bad = true;
                }
                ++ntile;
                umma::fence_after_sync();
                if (!issuer_warp) {
                const int lq = warp & 3, cq = warp >> 2;
                // the tile's n_tile columns split evenly over the column groups, 16 columns a load
                constexpr int kGroups = NPW / 4;
                const int cw = ((n_tile + 16 * kGroups - 1) / (16 * kGroups)) * 16, c0 = cw * cq;
                const int r = 32 * lq + lane;
                const bool vq = !bad && r < nq_t;
                const uint32_t t = vq ? *reinterpret_cast<volatile const uint32_t*>(b.gtau + s_q[r]) : 0u;
                uint32_t* hb = s_hit[warp];
                uint32_t cur = 0;
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
                            if (p < (uint32_t)b.rest_cap)
                                b.rest_buf[(size_t)qq * b.rest_cap + p] = ((uint64_t)d << 32) | slot;
                            const uint32_t* eq = b.lad + (size_t)qq * kLadStride;
                            for (int l = s_r0[rr]; l < kLad && d <= __ldg(eq + l); ++l)
                                atomicAdd(&s_lc[rr][l >> 1], 1u << (16 * (l & 1)));
                        }
                    }
                    __syncwarp();
                };
                for (int cb = 0; cb < cw && c0 + cb < n_tile; cb += 16) {
                    uint32_t v[16];
                    umma::tmem_ld16(tmem + ((uint32_t)(32 * lq) << 16) + (uint32_t)(c0 + cb), v);
                    umma::tmem_wait_ld();
                    const int m0 = mt + c0 + cb;
#pragma unroll
                    for (int h2 = 0; h2 < 2; ++h2) {
                        uint32_t hit = 0;
#pragma unroll
                        for (int j = 0; j < 8; ++j)
                            if (vq && m0 + 8 * h2 + j < nc && maxk - v[8 * h2 + j] <= t) hit |= 1u << j;
                        const uint32_t nh = (uint32_t)__popc(hit);
                        const uint32_t tot = __reduce_add_sync(0xFFFFFFFFu, nh);
                        if (tot == 0) continue;
                        if (cur + tot > (uint32_t)kHitCap) {
                            resolve(cur);
                            cur = 0;
                        }
                        uint32_t pre = nh;
#pragma unroll
                        for (int o = 1; o < 32; o <<= 1) {
                            const uint32_t y = __shfl_up_sync(0xFFFFFFFFu, pre, o);
                            if (lane >= o) pre += y;
                        }
                        uint32_t pos = cur + pre - nh;
                        const uint32_t mbase = (uint32_t)(c0 + cb + 8 * h2);
#pragma unroll
                        for (int j = 0; j < 8; ++j) {
                            if (!((hit >> j) & 1u)) continue;
                            hb[pos++] = ((uint32_t)r << 24) | ((mbase + j) << 16) | (maxk - v[8 * h2 + j]);
                        }
                        cur += tot;
                    }
                }
                resolve(cur);
                }
                umma::fence_before_sync();
                bad = __syncthreads_or(bad ? 1 : 0) != 0;
                if (tid < nq_t) ladder_flush(b, s_q[tid], s_lc[tid]);
            }
        }
        if (bad) break;
    }
    if (bad) {
        if (tid == 0) {
            atomicAdd(err, 1u);
            if (it > 0) umma::bar_wait(&done, (ntile - 1) & 1);  // bounded: let issued MMAs land
        }
    }
    umma::fence_before_sync();
    __syncthreads();
    if (warp == 0) umma::tmem_free(tmem, kMmaTmemCols);
}

}  // namespace

// ---- launchers ----------------------------------------------------------------------------------------

void launch_scan_mma(const IndexView& ix, const QueryEnc& e, const CellMajorBufs& b, cudaStream_t st) {
    using P = PScan<8, 2>;
    const int sms = sm_count();
    cudaMemsetAsync(b.work, 0, sizeof(uint32_t), st);
    set_smem((const void*)k_scan_mma<8, 2>, P::kSmem);
    Tick tk(kKScanMma, st);
    k_scan_mma<8, 2><<<P::kBlocks * sms, P::kT, P::kSmem, st>>>(ix, e, b.cell_cnt, b.qof, b, kMmaMinQueries, b.work,
                                                               b.overflow + 2);
}

}  // namespace dev
}  // namespace maivs
