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
// M = 128 queries x N = 256 members per tile, K in chunks of 128 bytes (8 nibble positions). A
// (tables) is copied and B (one-hot nibbles) is built in shared memory in the K-major 128-byte
// swizzled layout, one elected thread issues four kind::i8 tcgen05.mma per chunk into a TMEM
// accumulator (128 lanes x 256 columns), two stages overlap building chunk k + 1 with the MMAs of
// chunk k, and the epilogue reads the sums with tcgen05.ld and applies k_scan_cm's rule
// (d = maxk - sum <= tau, canonical home) to append survivors. Sums are exact integers, so the
// survivors equal k_scan_cm's. Every mbarrier wait is bounded; a timeout sets *err and the CTA
// stops issuing MMAs.
constexpr int kMmaQ = 128, kMmaN = 256, kMmaTmemCols = 256;
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

}  // namespace

// ---- launchers ----------------------------------------------------------------------------------------

void launch_scan_mma(const IndexView& ix, const QueryEnc& e, const CellMajorBufs& b, cudaStream_t st) {
    set_smem((const void*)k_scan_mma, kMmaSmem);
    Tick tk(kKScanMma, st);
    k_scan_mma<<<ix.M, 256, kMmaSmem, st>>>(ix, e, b.cell_cnt, b.qof, b, kMmaMinQueries, b.overflow + 2);
}

}  // namespace dev
}  // namespace maivs
