// The merge of a multi-segment search (ConcurrentIndex::finish, concurrent.rs:83-110): tombstone
// filter, one entry per external id, best k. One CTA per query; the lists of a query are short
// (segments x want entries), so every test is a pass over them through L1.
#include "dev_common.cuh"

namespace maivs {
namespace dev {

namespace {

constexpr int kMergeBS = 128;

__device__ __forceinline__ bool in_sorted(const uint64_t* __restrict__ a, int n, uint64_t x) {
    int lo = 0, hi = n;
    while (lo < hi) {
        int mid = (lo + hi) >> 1;
        uint64_t v = __ldg(a + mid);
        if (v < x)
            lo = mid + 1;
        else
            hi = mid;
    }
    return lo < n && __ldg(a + lo) == x;
}

// (score desc, id asc): the order of the final top k; a total order on entries with distinct ids
__device__ __forceinline__ bool merge_better(float sa, uint64_t ia, float sb, uint64_t ib) {
    return sa > sb || (sa == sb && ia < ib);
}

__global__ void __launch_bounds__(kMergeBS) k_segment_merge(const uint64_t* __restrict__ ids,
                                                            const float* __restrict__ scores,
                                                            const uint32_t* __restrict__ nout, int L, int nq, int want,
                                                            const uint64_t* __restrict__ tomb, int ntomb, int k,
                                                            char* __restrict__ scratch, uint64_t* __restrict__ out_ids,
                                                            float* __restrict__ out_scores) {
    extern __shared__ uint32_t s_off[];  // L + 1 list offsets
    __shared__ uint32_t s_n;
    const int q = blockIdx.x;
    const size_t cap = (size_t)L * want;
    uint64_t* eid = reinterpret_cast<uint64_t*>(scratch) + (size_t)q * cap;
    float* esc = reinterpret_cast<float*>(scratch + (size_t)nq * cap * 8) + (size_t)q * cap;
    uint32_t* ok = reinterpret_cast<uint32_t*>(scratch + (size_t)nq * cap * 12) + (size_t)q * cap;
    // 1. the query's entries, list after list (the head is the last list)
    if (threadIdx.x == 0) {
        uint32_t o = 0;
        for (int l = 0; l < L; ++l) {
            s_off[l] = o;
            o += min(nout[(size_t)l * nq + q], (uint32_t)want);
        }
        s_off[L] = o;
        s_n = o;
    }
    __syncthreads();
    const int n = (int)s_n;
    for (int l = 0; l < L; ++l) {
        const int m = (int)(s_off[l + 1] - s_off[l]);
        const size_t src = ((size_t)l * nq + q) * want;
        for (int i = threadIdx.x; i < m; i += kMergeBS) {
            eid[s_off[l] + i] = ids[src + i];
            esc[s_off[l] + i] = scores[src + i];
        }
    }
    __syncthreads();
    // 2. survivors: not tombstoned, and the best copy of their id (equal scores: the first copy)
    for (int i = threadIdx.x; i < n; i += kMergeBS) {
        const uint64_t id = eid[i];
        const float sc = esc[i];
        bool keep = !(ntomb > 0 && in_sorted(tomb, ntomb, id));
        for (int j = 0; keep && j < n; ++j)
            if (j != i && eid[j] == id && (esc[j] > sc || (esc[j] == sc && j < i))) keep = false;
        ok[i] = keep ? 1u : 0u;
    }
    __syncthreads();
    // 3. rank of every survivor among the survivors; the first k go out, best first
    uint64_t* oi = out_ids + (size_t)q * k;
    float* os = out_scores + (size_t)q * k;
    for (int r = threadIdx.x; r < k; r += kMergeBS) {
        oi[r] = ~0ull;
        os[r] = -INFINITY;
    }
    __syncthreads();
    for (int i = threadIdx.x; i < n; i += kMergeBS) {
        if (!ok[i]) continue;
        const uint64_t id = eid[i];
        const float sc = esc[i];
        int rank = 0;
        for (int j = 0; j < n && rank < k; ++j)
            if (ok[j] && merge_better(esc[j], eid[j], sc, id)) ++rank;
        if (rank < k) {
            oi[rank] = id;
            os[rank] = sc;
        }
    }
}

}  // namespace

void launch_segment_merge(const uint64_t* ids, const float* scores, const uint32_t* nout, int L, int nq, int want,
                          const uint64_t* tomb, int ntomb, int k, void* scratch, uint64_t* out_ids, float* out_scores,
                          cudaStream_t st) {
    if (nq <= 0) return;
    const size_t smem = ((size_t)L + 1) * sizeof(uint32_t);
    set_smem((const void*)k_segment_merge, smem);
    Tick tk(kKSegMerge, st);
    k_segment_merge<<<nq, kMergeBS, smem, st>>>(ids, scores, nout, L, nq, want, tomb, ntomb, k,
                                                static_cast<char*>(scratch), out_ids, out_scores);
}

}  // namespace dev
}  // namespace maivs
