// Index build on the GPU: spherical k-means (train_centroids and the centroid tree) and vector
// placement (add_batch), with results identical to the host build.
//
// The reference's build decides placement with exact float dot products (dot_f32: eight FMA
// chains over lanes l, l + 8, ..., closed by the hsum_ps tree, src/index.rs:58-65, :136-152) and
// first-maximum argmax loops (src/tree.rs:201-215). A tensor-core GEMM would round differently and
// move points between cells, so every dot here runs on the CUDA cores in that exact order; the
// integer parts (tree descent, counting cut-offs) reuse the search kernels. What stays on the host
// is cheap and order-sensitive: the per-cluster CSR order, the empty-cluster reseed (xorshift64),
// the sequential normalisations and the bookkeeping of cells and slots.
#include <algorithm>
#include <cmath>
#include <memory>
#include <string>
#include <vector>

#include "../host/hostmath.h"
#include "../host/index_host.h"
#include "dev_common.cuh"

namespace maivs {

namespace {

// ---- exact-order dot products -------------------------------------------------------------------

// ((a0 + a4) + (a2 + a6)) + ((a1 + a5) + (a3 + a7)) over the 8 chains.
__device__ __forceinline__ float close_chains(const float a[8]) {
    return __fadd_rn(__fadd_rn(__fadd_rn(a[0], a[4]), __fadd_rn(a[2], a[6])),
                     __fadd_rn(__fadd_rn(a[1], a[5]), __fadd_rn(a[3], a[7])));
}

// ---- k-means: assignment (tree.rs:201-215) ------------------------------------------------------
// A CTA of 256 threads takes kKmP points (kept in shared memory) and walks the centroids in tiles of
// `tc` rows; thread (p = tid / 8, lane l = tid % 8) scores point p against centroids l, l + 8, ...
// of each tile. Every score is dot_f32 in the reference's order; each thread keeps its first
// maximum, and the eight threads of a point combine theirs by (score desc, index asc), which is the
// first maximum of the sequential loop.
constexpr int kKmP = 32;
constexpr int kKmThreads = 256;
constexpr int kKmMaxPerThread = 8;  // centroids per thread and tile

__global__ void __launch_bounds__(kKmThreads) k_km_assign(const float* __restrict__ x, int n, int dim,
                                                          const float* __restrict__ cents, int k, int tc, int stride,
                                                          uint32_t* __restrict__ assign) {
    extern __shared__ __align__(16) float kms[];
    float* xs = kms;                               // kKmP x stride
    float* cs = kms + (size_t)kKmP * stride;       // tc x stride
    const int tid = threadIdx.x, p = tid >> 3, l = tid & 7;
    const int p0 = blockIdx.x * kKmP;
    for (int i = tid; i < kKmP * dim; i += kKmThreads) {
        const int r = i / dim, c = i - r * dim;
        xs[(size_t)r * stride + c] = p0 + r < n ? x[(size_t)(p0 + r) * dim + c] : 0.0f;
    }
    const int d8 = dim & ~7;
    float best = -INFINITY;
    int best_i = 0x7FFFFFFF;
    for (int c0 = 0; c0 < k; c0 += tc) {
        const int nt = min(tc, k - c0);
        __syncthreads();  // the previous tile is done (and, first time, the points are in)
        for (int i = tid; i < nt * dim; i += kKmThreads) {
            const int r = i / dim, c = i - r * dim;
            cs[(size_t)r * stride + c] = cents[(size_t)(c0 + r) * dim + c];
        }
        __syncthreads();
        const float* xp = xs + (size_t)p * stride;
        for (int jj = 0; jj < kKmMaxPerThread; ++jj) {
            const int cl = l + 8 * jj;
            if (cl >= nt) break;
            const float* cp = cs + (size_t)cl * stride;
            float acc[8] = {0.0f, 0.0f, 0.0f, 0.0f, 0.0f, 0.0f, 0.0f, 0.0f};
            for (int i = 0; i < d8; i += 8) {
                const float4 xa = *reinterpret_cast<const float4*>(xp + i);
                const float4 xb = *reinterpret_cast<const float4*>(xp + i + 4);
                const float4 ca = *reinterpret_cast<const float4*>(cp + i);
                const float4 cb = *reinterpret_cast<const float4*>(cp + i + 4);
                acc[0] = __fmaf_rn(xa.x, ca.x, acc[0]);
                acc[1] = __fmaf_rn(xa.y, ca.y, acc[1]);
                acc[2] = __fmaf_rn(xa.z, ca.z, acc[2]);
                acc[3] = __fmaf_rn(xa.w, ca.w, acc[3]);
                acc[4] = __fmaf_rn(xb.x, cb.x, acc[4]);
                acc[5] = __fmaf_rn(xb.y, cb.y, acc[5]);
                acc[6] = __fmaf_rn(xb.z, cb.z, acc[6]);
                acc[7] = __fmaf_rn(xb.w, cb.w, acc[7]);
            }
            float s = close_chains(acc);
            for (int i = d8; i < dim; ++i) s = __fadd_rn(s, __fmul_rn(xp[i], cp[i]));
            if (s > best) {
                best = s;
                best_i = c0 + cl;
            }
        }
    }
    // combine the 8 threads of a point: larger score, then smaller index
#pragma unroll
    for (int o = 4; o > 0; o >>= 1) {
        const float ob = __shfl_xor_sync(0xFFFFFFFFu, best, o);
        const int oi = __shfl_xor_sync(0xFFFFFFFFu, best_i, o);
        if (ob > best || (ob == best && oi < best_i)) {
            best = ob;
            best_i = oi;
        }
    }
    if (l == 0 && p0 + p < n) assign[p0 + p] = best_i == 0x7FFFFFFF ? 0u : (uint32_t)best_i;
}

// ---- k-means: per-cluster sums in point order (tree.rs:218-229) -----------------------------------
// Thread (cluster blockIdx.x, dimension t) adds the cluster's points in ascending index order,
// starting from 0, exactly as the reference's sequential loop does.
__global__ void k_km_sums(const float* __restrict__ x, int dim, const uint32_t* __restrict__ order,
                          const uint32_t* __restrict__ start, float* __restrict__ sums) {
    const int j = blockIdx.x;
    const int t = blockIdx.y * blockDim.x + threadIdx.x;
    if (t >= dim) return;
    float s = 0.0f;
    for (uint32_t r = start[j]; r < start[j + 1]; ++r) s = __fadd_rn(s, x[(size_t)order[r] * dim + t]);
    sums[(size_t)j * dim + t] = s;
}

// ---- placement (index.rs:2442-2560) ---------------------------------------------------------------
// One warp per vector: exact dots of the vector with its tree shortlist (eight lanes per dot, one
// chain each, closed by shuffles in the hsum_ps order), then the homes: the first maximum in
// shortlist order (one home), the orthogonal-polysemy greedy over the 16 best by (score desc, id asc)
// (pick_orthogonal), or the best max_assign within spill_margin of the first (margin replication).
constexpr int kPlaceWarps = 8;
constexpr int kPlaceCap = 128;  // shortlist entries a warp keeps in shared memory

// Dot of a (in shared or global memory) with b (global), eight lanes of a group summing chain l.
__device__ __forceinline__ float group_dot(const float* a, const float* b, int dim, int l) {
    const int d8 = dim & ~7;
    float acc = 0.0f;
    for (int i = l; i < d8; i += 8) acc = __fmaf_rn(a[i], __ldg(b + i), acc);
    // ((a0 + a4) + (a2 + a6)) + ((a1 + a5) + (a3 + a7)) across the 8 lanes
    float s1 = __fadd_rn(acc, __shfl_xor_sync(0xFFFFFFFFu, acc, 4));
    float s2 = __fadd_rn(s1, __shfl_xor_sync(0xFFFFFFFFu, s1, 2));
    float s3 = __fadd_rn(s2, __shfl_xor_sync(0xFFFFFFFFu, s2, 1));
    for (int i = d8; i < dim; ++i) s3 = __fadd_rn(s3, __fmul_rn(a[i], __ldg(b + i)));
    return s3;
}

__global__ void __launch_bounds__(32 * kPlaceWarps) k_place(const float* __restrict__ v, int nv, int dim,
                                                            const float* __restrict__ cents,
                                                            const uint32_t* __restrict__ sl,
                                                            const uint32_t* __restrict__ sl_n, int sl_cap, int ma,
                                                            float lambda, float margin, uint32_t* __restrict__ homes) {
    extern __shared__ __align__(16) float pls[];
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int q = blockIdx.x * kPlaceWarps + warp;
    const int vstride = (dim + 3) & ~3;
    float* vs = pls + (size_t)warp * vstride;
    __shared__ float sc[kPlaceWarps][kPlaceCap];
    __shared__ uint32_t sid[kPlaceWarps][kPlaceCap];
    __shared__ uint8_t taken[kPlaceWarps][kPlaceCap];
    __shared__ float pps[kPlaceWarps][16];           // the pool: scores and cells, best first
    __shared__ uint32_t ppid[kPlaceWarps][16];
    __shared__ float gds[kPlaceWarps][16][16];       // centroid dots of home t with pool entry j
    if (q >= nv) return;  // whole warps leave together
    for (int i = lane; i < dim; i += 32) vs[i] = v[(size_t)q * dim + i];
    const int n = min((int)sl_n[q], sl_cap);
    const uint32_t* cand = sl + (size_t)q * sl_cap;
    uint32_t* out = homes + (size_t)q * ma;
    for (int i = lane; i < ma; i += 32) out[i] = 0xFFFFFFFFu;
    __syncwarp();
    if (n == 0 || n > kPlaceCap) return;  // the host places these
    const int grp = lane >> 3, l = lane & 7;
    for (int c0 = 0; c0 < n; c0 += 4) {
        const int ci = c0 + grp;
        const uint32_t cell = ci < n ? cand[ci] : cand[0];
        const float s = group_dot(vs, cents + (size_t)cell * dim, dim, l);
        if (l == 0 && ci < n) {
            sc[warp][ci] = s;
            sid[warp][ci] = cell;
        }
    }
    __syncwarp();
    if (ma <= 1) {  // first maximum in shortlist order
        float best = -INFINITY;
        int bi = 0x7FFFFFFF;
        for (int i = lane; i < n; i += 32)
            if (sc[warp][i] > best || (sc[warp][i] == best && i < bi)) {
                best = sc[warp][i];
                bi = i;
            }
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) {
            const float ob = __shfl_xor_sync(0xFFFFFFFFu, best, o);
            const int oi = __shfl_xor_sync(0xFFFFFFFFu, bi, o);
            if (ob > best || (ob == best && oi < bi)) {
                best = ob;
                bi = oi;
            }
        }
        if (lane == 0) out[0] = sid[warp][bi == 0x7FFFFFFF ? 0 : bi];
        return;
    }
    // the best `pool` entries by (score desc, cell asc), in that order, by repeated warp argmax
    const int pool = lambda > 0.0f ? min(16, n) : min(ma, n);
    for (int i = lane; i < n; i += 32) taken[warp][i] = 0;
    __syncwarp();
    float* ps = pps[warp];
    uint32_t* pid = ppid[warp];
    for (int r = 0; r < pool; ++r) {
        float best = -INFINITY;
        uint32_t bid = 0xFFFFFFFFu;
        int bi = -1;
        for (int i = lane; i < n; i += 32) {
            if (taken[warp][i]) continue;
            const float s = sc[warp][i];
            const uint32_t c = sid[warp][i];
            if (bi < 0 || s > best || (s == best && c < bid)) {
                best = s;
                bid = c;
                bi = i;
            }
        }
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) {
            const float ob = __shfl_xor_sync(0xFFFFFFFFu, best, o);
            const uint32_t oc = __shfl_xor_sync(0xFFFFFFFFu, bid, o);
            const int oi = __shfl_xor_sync(0xFFFFFFFFu, bi, o);
            if (oi >= 0 && (bi < 0 || ob > best || (ob == best && oc < bid))) {
                best = ob;
                bid = oc;
                bi = oi;
            }
        }
        if (lane == 0) {
            ps[r] = best;
            pid[r] = bid;
            taken[warp][bi] = 1;
        }
        __syncwarp();
    }
    if (lambda <= 0.0f) {  // margin replication: the best ma within spill_margin of the first
        const float cutoff = __fsub_rn(ps[0], margin);
        int w = 0;
        for (int r = 0; r < pool; ++r)
            if (ps[r] >= cutoff) {
                if (lane == 0) out[w] = pid[r];
                ++w;
            }
        return;
    }
    // pick_orthogonal: home 0 is the best; each further home minimises
    // (2 - 2 s_j) + lambda * sum_h ((1 - s_h - s_j + c_h . c_j) / sqrt(max(2 - 2 s_h, 1e-12)))^2
    const int r_homes = min(ma, pool);
    int hidx[16];
    int nh = 1;
    hidx[0] = 0;
    uint32_t used = 1u;  // pool entries taken as homes
    while (nh < r_homes) {
        const int h = hidx[nh - 1];
        // dots of the newest home with every pool entry, four at a time
        for (int j0 = 0; j0 < pool; j0 += 4) {
            const int j = j0 + grp;
            const uint32_t cj = j < pool ? pid[j] : pid[0];
            const float gd = group_dot(cents + (size_t)pid[h] * dim, cents + (size_t)cj * dim, dim, l);
            if (l == 0 && j < pool) gds[warp][nh - 1][j] = gd;
        }
        __syncwarp();
        int best_j = -1;
        float best_l = INFINITY;
        for (int j = 0; j < pool; ++j) {
            if ((used >> j) & 1u) continue;
            const float sj = ps[j];
            float loss = __fsub_rn(2.0f, __fmul_rn(2.0f, sj));
            for (int t = 0; t < nh; ++t) {
                const float sh = ps[hidx[t]];
                const float rn = __fsqrt_rn(fmaxf(__fsub_rn(2.0f, __fmul_rn(2.0f, sh)), 1e-12f));
                const float p = __fdiv_rn(__fadd_rn(__fsub_rn(__fsub_rn(1.0f, sh), sj), gds[warp][t][j]), rn);
                loss = __fadd_rn(loss, __fmul_rn(__fmul_rn(lambda, p), p));
            }
            if (loss < best_l) {
                best_l = loss;
                best_j = j;
            }
        }
        if (best_j < 0) break;
        used |= 1u << best_j;
        hidx[nh++] = best_j;
    }
    if (lane == 0)
        for (int t = 0; t < nh; ++t) out[t] = pid[hidx[t]];
}

// ---- device memory of one build step ----------------------------------------------------------------

struct DevBuf {
    void* p = nullptr;
    ~DevBuf() {
        if (p) cudaFree(p);
    }
    template <typename T>
    T* get() const {
        return static_cast<T*>(p);
    }
};

struct Stream {
    cudaStream_t s = nullptr;
    ~Stream() {
        if (s) cudaStreamDestroy(s);
    }
};

std::string cuda_err(const char* what, cudaError_t e) { return std::string(what) + ": " + cudaGetErrorString(e); }

#define BTRY(call, what)                              \
    do {                                              \
        cudaError_t e_ = (call);                      \
        if (e_ != cudaSuccess) return cuda_err(what, e_); \
    } while (0)

template <typename T>
std::string dev_alloc(DevBuf& b, size_t n) {
    BTRY(cudaMalloc(&b.p, std::max<size_t>(n, 1) * sizeof(T)), "device allocation of the build");
    return "";
}

}  // namespace

// kmeans_spherical (tree.rs:179-248) with the assignment and the sums on `device`.
std::string gpu_kmeans_spherical(int device, const float* x, size_t n, size_t dim, size_t k_in, size_t iters,
                                 uint64_t seed, std::vector<uint32_t>& assign, std::vector<float>& cents) {
    size_t k = std::min(std::max<size_t>(k_in, 1), n);
    cents.assign(k * dim, 0.0f);
    size_t stride = std::max<size_t>(n / k, 1);
    for (size_t j = 0; j < k; ++j) {
        size_t src = std::min(j * stride, n - 1);
        std::copy(x + src * dim, x + (src + 1) * dim, cents.begin() + j * dim);
    }
    assign.assign(n, 0);
    uint64_t state = seed | 1;
    auto next_u = [&state]() {
        state ^= state << 13;
        state ^= state >> 7;
        state ^= state << 17;
        return state;
    };
    BTRY(cudaSetDevice(device), "cudaSetDevice");
    Stream st;
    BTRY(cudaStreamCreateWithFlags(&st.s, cudaStreamNonBlocking), "stream of the build");
    DevBuf dx, dc, da, dorder, dstart, dsums;
    std::string err;
    if (!(err = dev_alloc<float>(dx, n * dim)).empty() || !(err = dev_alloc<float>(dc, k * dim)).empty() ||
        !(err = dev_alloc<uint32_t>(da, n)).empty() || !(err = dev_alloc<uint32_t>(dorder, n)).empty() ||
        !(err = dev_alloc<uint32_t>(dstart, k + 1)).empty() || !(err = dev_alloc<float>(dsums, k * dim)).empty())
        return err;
    BTRY(cudaMemcpyAsync(dx.p, x, n * dim * sizeof(float), cudaMemcpyHostToDevice, st.s), "copy of the points");
    const int sstride = (int)(((dim + 3) & ~(size_t)3) + 4);  // padded rows: 8 centroids of a warp on distinct banks
    int tc = 64;
    while (tc > 8 && ((size_t)kKmP + tc) * sstride * sizeof(float) > 200 * 1024) tc -= 8;
    const size_t smem = ((size_t)kKmP + tc) * sstride * sizeof(float);
    if (smem > 220 * 1024) return "dimension too large for the GPU k-means";
    BTRY(cudaFuncSetAttribute((const void*)k_km_assign, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem),
         "k-means shared memory");
    std::vector<uint32_t> start(k + 1), order(n);
    std::vector<float> sums(k * dim);
    for (size_t it = 0; it < iters; ++it) {
        BTRY(cudaMemcpyAsync(dc.p, cents.data(), k * dim * sizeof(float), cudaMemcpyHostToDevice, st.s),
             "copy of the centroids");
        k_km_assign<<<(unsigned)((n + kKmP - 1) / kKmP), kKmThreads, smem, st.s>>>(
            dx.get<float>(), (int)n, (int)dim, dc.get<float>(), (int)k, tc, sstride, da.get<uint32_t>());
        BTRY(cudaGetLastError(), "launch of k_km_assign");
        BTRY(cudaMemcpyAsync(assign.data(), da.p, n * sizeof(uint32_t), cudaMemcpyDeviceToHost, st.s),
             "copy of the assignment");
        BTRY(cudaStreamSynchronize(st.s), "k-means assignment");
        // clusters in point order (CSR), as the reference's sequential accumulation visits them
        std::fill(start.begin(), start.end(), 0u);
        for (size_t i = 0; i < n; ++i) start[assign[i] + 1] += 1;
        for (size_t j = 0; j < k; ++j) start[j + 1] += start[j];
        {
            std::vector<uint32_t> pos(start.begin(), start.end() - 1);
            for (size_t i = 0; i < n; ++i) order[pos[assign[i]]++] = (uint32_t)i;
        }
        BTRY(cudaMemcpyAsync(dorder.p, order.data(), n * sizeof(uint32_t), cudaMemcpyHostToDevice, st.s),
             "copy of the order");
        BTRY(cudaMemcpyAsync(dstart.p, start.data(), (k + 1) * sizeof(uint32_t), cudaMemcpyHostToDevice, st.s),
             "copy of the offsets");
        dim3 grid((unsigned)k, (unsigned)((dim + 127) / 128));
        k_km_sums<<<grid, 128, 0, st.s>>>(dx.get<float>(), (int)dim, dorder.get<uint32_t>(), dstart.get<uint32_t>(),
                                          dsums.get<float>());
        BTRY(cudaGetLastError(), "launch of k_km_sums");
        BTRY(cudaMemcpyAsync(sums.data(), dsums.p, k * dim * sizeof(float), cudaMemcpyDeviceToHost, st.s),
             "copy of the sums");
        BTRY(cudaStreamSynchronize(st.s), "k-means sums");
        for (size_t j = 0; j < k; ++j) {
            float* c = cents.data() + j * dim;
            if (start[j + 1] == start[j]) {
                size_t src = (size_t)(next_u() % (uint64_t)n);
                std::copy(x + src * dim, x + (src + 1) * dim, c);
                continue;
            }
            std::copy(sums.begin() + j * dim, sums.begin() + (j + 1) * dim, c);
            normalize(c, dim);
        }
    }
    return "";
}

// Placement of n vectors (assign_cells_routed, index.rs:2442-2560) through the centroid tree on
// `device`, in chunks: codes (rotate + pack, also returned in codes_out, n x nw), tree shortlist of
// max(64, 8 max_assign) cells, exact re-score and home choice. A vector whose shortlist is empty or
// longer than the kernel keeps (never with the reference's shortlist length) gets no homes; the
// caller places it on the host.
std::string gpu_place(int device, const HostIndex& h, const float* data, size_t n,
                      std::vector<std::vector<uint32_t>>& asg, uint64_t* codes_out) {
    if (!h.tree) return "placement on the GPU needs the centroid tree";
    const CentroidTree& t = *h.tree;
    if (t.levels.size() > (size_t)dev::kMaxTreeLevels) return "centroid tree deeper than 8 levels";
    const size_t dim = h.dim, nw = h.nw, npos = nw * 16, M = h.cells.size(), ma = std::max<size_t>(h.max_assign, 1);
    const size_t want = std::max(kAssignCandidates, h.max_assign * 8);
    if (want > (size_t)kPlaceCap) return "shortlist longer than the GPU placement keeps";
    BTRY(cudaSetDevice(device), "cudaSetDevice");
    Stream st;
    BTRY(cudaStreamCreateWithFlags(&st.s, cudaStreamNonBlocking), "stream of the build");
    std::string err;
    std::vector<std::unique_ptr<DevBuf>> keep;
    auto upload = [&](const void* src, size_t bytes) -> void* {
        keep.push_back(std::make_unique<DevBuf>());
        if (cudaMalloc(&keep.back()->p, std::max<size_t>(bytes, 1)) != cudaSuccess) return nullptr;
        if (bytes && cudaMemcpyAsync(keep.back()->p, src, bytes, cudaMemcpyHostToDevice, st.s) != cudaSuccess)
            return nullptr;
        return keep.back()->p;
    };
    // the view the encoder and the tree descent read
    dev::IndexView v{};
    v.dim = (int)dim;
    v.dim_pad = (int)h.dim_pad;
    v.nw = (int)nw;
    v.npos = (int)npos;
    v.M = (int)M;
    v.ma = (int)ma;
    v.maxk = 255u * (uint32_t)npos;
    v.signs = static_cast<const float*>(upload(h.signs.data(), h.signs.size() * sizeof(float)));
    std::vector<uint8_t> live(M, 1);  // tree.search has no live filter (index.rs:2448-2452)
    v.live = static_cast<const uint8_t*>(upload(live.data(), M));
    std::vector<float> cents(M * dim);
    for (size_t c = 0; c < M; ++c) std::copy(h.cells[c].centroid.begin(), h.cells[c].centroid.end(), cents.begin() + c * dim);
    const float* dcent = static_cast<const float*>(upload(cents.data(), cents.size() * sizeof(float)));
    v.tree_depth = (int)t.levels.size();
    size_t cap = t.levels.empty() ? 0 : t.levels[0].n;
    std::vector<size_t> beams = t.beams(want);
    int bms[dev::kMaxTreeLevels] = {0};
    for (size_t i = 0; i < t.levels.size(); ++i) {
        const TreeLevel& L = t.levels[i];
        v.tree_codes[i] = static_cast<const uint64_t*>(upload(L.codes.data(), L.codes.size() * 8));
        v.tree_child_start[i] = static_cast<const uint32_t*>(upload(L.child_start.data(), L.child_start.size() * 4));
        v.tree_child_len[i] = static_cast<const uint32_t*>(upload(L.child_len.data(), L.child_len.size() * 4));
        v.tree_n[i] = (int)L.n;
        bms[i] = (int)beams[i];
        // frontier bound: the kept nodes' children at the next level (the first level is whole)
        uint32_t maxlen = 0;
        for (uint32_t x : L.child_len) maxlen = std::max(maxlen, x);
        cap = std::max(cap, std::min<size_t>(L.n, beams[i]) * maxlen);
    }
    v.leaf_codes = static_cast<const uint64_t*>(upload(t.leaf_codes.data(), t.leaf_codes.size() * 8));
    v.leaf_ids = static_cast<const uint32_t*>(upload(t.leaf_ids.data(), t.leaf_ids.size() * 4));
    v.n_leaf = (int)t.n_leaf;
    cap = std::max(cap, (size_t)1);
    for (auto& b : keep)
        if (!b->p) return "device allocation of the build";
    // chunk buffers
    const size_t chunk = std::max<size_t>(1, std::min<size_t>(n, std::max<size_t>(1024, (size_t)(256u << 20) / (cap * 12 + 1))));
    DevBuf dv, dq, dlut, dfd, dfb, dscr, dsl, dsln, dhomes;
    if (!(err = dev_alloc<float>(dv, chunk * dim)).empty() || !(err = dev_alloc<uint64_t>(dq, chunk * nw)).empty() ||
        !(err = dev_alloc<uint8_t>(dlut, chunk * npos * 16)).empty() || !(err = dev_alloc<float>(dfd, chunk)).empty() ||
        !(err = dev_alloc<float>(dfb, chunk)).empty() || !(err = dev_alloc<uint32_t>(dscr, chunk * 3 * cap)).empty() ||
        !(err = dev_alloc<uint32_t>(dsl, chunk * want)).empty() || !(err = dev_alloc<uint32_t>(dsln, chunk)).empty() ||
        !(err = dev_alloc<uint32_t>(dhomes, chunk * ma)).empty())
        return err;
    dev::QueryEnc e{};
    e.qbits = dq.get<uint64_t>();
    e.lut = dlut.get<uint8_t>();
    e.fs_delta = dfd.get<float>();
    e.fs_bias = dfb.get<float>();
    const size_t psmem = (size_t)kPlaceWarps * ((dim + 3) & ~(size_t)3) * sizeof(float);
    BTRY(cudaFuncSetAttribute((const void*)k_place, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)psmem),
         "placement shared memory");
    std::vector<uint32_t> hh(chunk * ma);
    asg.assign(n, {});
    for (size_t c0 = 0; c0 < n; c0 += chunk) {
        const size_t cn = std::min(chunk, n - c0);
        BTRY(cudaMemcpyAsync(dv.p, data + c0 * dim, cn * dim * sizeof(float), cudaMemcpyHostToDevice, st.s),
             "copy of the vectors");
        dev::launch_encode(v, dv.get<float>(), (int)cn, e, false, false, st.s);
        dev::launch_route_tree(v, e, (int)cn, bms, (int)want, dscr.get<uint32_t>(), (int)cap, dsl.get<uint32_t>(),
                               dsln.get<uint32_t>(), (int)want, st.s);
        k_place<<<(unsigned)((cn + kPlaceWarps - 1) / kPlaceWarps), 32 * kPlaceWarps, psmem, st.s>>>(
            dv.get<float>(), (int)cn, (int)dim, dcent, dsl.get<uint32_t>(), dsln.get<uint32_t>(), (int)want, (int)ma,
            h.spill_lambda, h.spill_margin, dhomes.get<uint32_t>());
        BTRY(cudaGetLastError(), "launch of the placement");
        BTRY(cudaMemcpyAsync(hh.data(), dhomes.p, cn * ma * sizeof(uint32_t), cudaMemcpyDeviceToHost, st.s),
             "copy of the homes");
        if (codes_out)
            BTRY(cudaMemcpyAsync(codes_out + c0 * nw, dq.p, cn * nw * sizeof(uint64_t), cudaMemcpyDeviceToHost, st.s),
                 "copy of the codes");
        BTRY(cudaStreamSynchronize(st.s), "placement");
        for (size_t i = 0; i < cn; ++i) {
            auto& a = asg[c0 + i];
            for (size_t j = 0; j < ma; ++j)
                if (hh[i * ma + j] != 0xFFFFFFFFu) a.push_back(hh[i * ma + j]);
        }
    }
    return "";
}

}  // namespace maivs
