// Device image upload and the two search pipelines (cell-major join, per-query scan).
#include <omp.h>

#include <algorithm>
#include <cmath>
#include <cstring>

#include "../host/hostmath.h"
#include "engine.h"

namespace maivs {

namespace {

// Queries per pass of the per-query pipeline: the whole batch when its scratch (probe ranks,
// shortlists, entries and candidates of every query) fits in kPerQueryScratch, else the largest
// power-of-two share of it that does, but never fewer than kPerQueryMinChunk.
constexpr size_t kPerQueryScratch = size_t(4) << 30;
// Batches of this many queries or more may be searched as two halves on two streams.
constexpr int kSplitQueries = 512;
constexpr int kPerQueryMinChunk = 64;
constexpr uint32_t kNoCellHost = 0xFFFFFFFFu;  // an unused home in slot_cells

struct Bump {
    char* base;
    size_t off = 0, cap;
    template <typename T>
    T* take(size_t n) {
        size_t a = (off + 255) & ~size_t(255);
        off = a + n * sizeof(T);
        return base ? reinterpret_cast<T*>(base + a) : nullptr;
    }
};

#define CUDA_TRY(expr)                                             \
    do {                                                           \
        cudaError_t e_ = (expr);                                   \
        if (e_ != cudaSuccess) {                                   \
            err = std::string(#expr) + ": " + cudaGetErrorString(e_); \
            return e_ == cudaErrorMemoryAllocation ? kOom : kCudaError; \
        }                                                          \
    } while (0)

}  // namespace

DeviceIndex::~DeviceIndex() {
    if (device_ >= 0) cudaSetDevice(device_);
    if (stream_) cudaStreamSynchronize(stream_);
    for (void* p : allocs_) cudaFree(p);
    if (stream2_) cudaStreamSynchronize(stream2_);
    for (void* w : ws_)
        if (w) cudaFree(w);
    if (io_) cudaFree(io_);
    if (pin_) cudaFreeHost(pin_);
    for (auto& e : ev_)
        if (e) cudaEventDestroy(e);
    for (auto& e : split_ev_)
        if (e) cudaEventDestroy(e);
    for (auto& e : ws_ev_)
        if (e) cudaEventDestroy(e);
    if (stream2_) cudaStreamDestroy(stream2_);
    if (stream_) cudaStreamDestroy(stream_);
}

void* DeviceIndex::alloc(size_t bytes) {
    void* p = nullptr;
    if (bytes == 0) bytes = 16;
    if (cudaMalloc(&p, bytes) != cudaSuccess) return nullptr;
    allocs_.push_back(p);
    bytes_ += bytes;
    return p;
}

template <typename T>
T* DeviceIndex::upload_vec(const std::vector<T>& v) {
    T* p = static_cast<T*>(alloc(v.size() * sizeof(T)));
    if (p && !v.empty()) cudaMemcpy(p, v.data(), v.size() * sizeof(T), cudaMemcpyHostToDevice);
    return p;
}

std::string DeviceIndex::upload(const HostIndex& h, int device, uint32_t c_lo, uint32_t c_hi) {
    // A compacted FastScan index is scanned by table sums (per-query path and cell-major join);
    // any other index by Hamming distance over its flat codes, per query (index.rs:1624-1626: the
    // FastScan branch needs fastscan && compacted).
    const bool fs = h.compacted && h.fastscan && !h.fs_off.empty();
    if (h.nw > 16) return "codes longer than 1024 bits are not supported";
    if (!fs && h.bits.size() < h.ext_ids.size() * h.nw) return "the index has no flat codes to scan";
    int ndev = 0;
    if (cudaGetDeviceCount(&ndev) != cudaSuccess || ndev == 0) return "no CUDA device is visible";
    if (device < 0 || device >= ndev) return "device ordinal out of range";
    device_ = device;
    cudaSetDevice(device_);
    if (!stream_) cudaStreamCreateWithFlags(&stream_, cudaStreamNonBlocking);
    for (auto& e : ev_)
        if (!e) cudaEventCreate(&e);
    for (void* p : allocs_) cudaFree(p);
    allocs_.clear();
    bytes_ = 0;

    const size_t M = h.cells.size(), dim = h.dim, nw = h.nw, npos = nw * 16, ma = h.max_assign;
    dev::IndexView v{};
    v.dim = (int)dim;
    v.dim_pad = (int)h.dim_pad;
    v.nw = (int)nw;
    v.npos = (int)npos;
    v.M = (int)M;
    v.ma = (int)ma;
    v.maxk = 255u * (uint32_t)npos;
    v.ham = fs ? 0 : 1;

    // ---- scan layout: per cell, its members' codes as position-major 8-member nibble words ----
    // (Hamming scan: the member lists only, beside the flat codes)
    std::vector<uint32_t> moff(M + 1, 0), woff(M + 1, 0);
    max_members_ = 0;
    for (size_t c = 0; c < M; ++c) {
        size_t n = (c >= c_lo && c < c_hi) ? h.cells[c].members.size() : 0;
        max_members_ = std::max(max_members_, n);
        moff[c + 1] = moff[c] + (uint32_t)n;
        woff[c + 1] = woff[c] + (fs ? (uint32_t)(npos * ((n + 7) / 8)) : 0u);
    }
    {
        // seed scan blocks per query: the seed cells' groups of an average live cell, 128 a block,
        // with room for larger cells
        size_t live = 0;
        for (size_t c = 0; c < M; ++c) live += moff[c + 1] > moff[c] ? 1 : 0;
        const double groups = live ? (double)woff[M] / (double)std::max<size_t>(npos, 1) / (double)live : 1.0;
        v.seed_parts = (int)std::min(16.0, std::max(1.0, std::ceil(1.15 * dev::kSeedCells * groups / 128.0)));
    }
    std::vector<uint32_t> slots(moff[M]), codes(woff[M], 0);
#pragma omp parallel for schedule(dynamic, 16)
    for (long long c = 0; c < (long long)M; ++c) {
        const auto& mem = h.cells[c].members;
        size_t n = moff[c + 1] - moff[c], ng = (n + 7) / 8;
        std::copy(mem.begin(), mem.begin() + n, slots.begin() + moff[c]);
        uint32_t* cw = codes.data() + woff[c];
        if (!fs) continue;
        for (size_t g = 0; g < ng; ++g)
            for (size_t b = 0; b < 8 && 8 * g + b < n; ++b) {
                const uint64_t* code = &h.bits[(size_t)mem[8 * g + b] * nw];
                for (size_t j = 0; j < npos; ++j) cw[j * ng + g] |= (uint32_t)nib(code, j) << (4 * b);
            }
    }
    if (ma == 2) {
        std::vector<uint32_t> lower(moff[M], kNoCellHost);
#pragma omp parallel for schedule(dynamic, 64)
        for (long long c = 0; c < (long long)M; ++c)
            for (uint32_t i = moff[c]; i < moff[c + 1]; ++i) {
                const uint32_t* hm = &h.slot_cells[(size_t)slots[i] * 2];
                for (int j = 0; j < 2; ++j)
                    if (hm[j] != kNoCellHost && hm[j] < (uint32_t)c) lower[i] = hm[j];
            }
        v.cell_lower = upload_vec(lower);
    }
    v.cell_moff = upload_vec(moff);
    moff_ = moff;
    v.cell_woff = upload_vec(woff);
    v.cell_slots = upload_vec(slots);
    v.cell_codes = fs ? upload_vec(codes) : nullptr;
    v.bits = fs ? nullptr : upload_vec(h.bits);
    v.slot_cells = upload_vec(h.slot_cells);
    v.ext_ids = upload_vec(h.ext_ids);
    v.tags = h.tags.empty() ? nullptr : upload_vec(h.tags);

    // ---- rerank store (index.rs:1309-1371) ----
    if (h.per_dim_sq) {
        v.rerank_mode = 1;
    } else if (h.i8_rerank) {
        v.rerank_mode = 2;
    } else {
        v.rerank_mode = 0;
    }
    if (v.rerank_mode == 0) {
        v.vecs_f32 = upload_vec(h.vecs_f32);
    } else {
        std::vector<uint8_t> u(h.scan_i8.size());
        std::memcpy(u.data(), h.scan_i8.data(), u.size());
        v.rr_u8 = upload_vec(u);
    }
    if (h.per_dim_sq) {
        v.sq_min = upload_vec(h.sq_min);
        v.sq_step = upload_vec(h.sq_step);
    }

    // ---- routing tables ----
    std::vector<uint8_t> live(M);
    std::vector<float> rb(M), cf(M * dim);
    n_live_ = 0;
    for (size_t c = 0; c < M; ++c) {
        live[c] = h.cells[c].members.empty() ? 0 : 1;
        n_live_ += live[c];
        rb[c] = h.cells[c].r_bound;
        std::copy(h.cells[c].centroid.begin(), h.cells[c].centroid.end(), cf.begin() + c * dim);
    }
    v.live = upload_vec(live);
    {
        std::vector<uint32_t> ll;
        for (size_t c = 0; c < M; ++c)
            if (live[c]) ll.push_back((uint32_t)c);
        v.live_list = upload_vec(ll);
        v.n_live_cells = (int)ll.size();
    }
    v.r_bound = upload_vec(rb);
    v.cent_f32 = upload_vec(cf);
    v.signs = upload_vec(h.signs);
    std::vector<uint64_t> cb = h.cent_bits;
    if (cb.size() != M * nw) {
        // route_batch needs the codes even when only the tree was built (index.rs:1873-1876 reads
        // cent_bits only with two_stage; the codes are cheap, so they always exist here).
        cb.assign(M * nw, 0);
        std::vector<float> rot(h.dim_pad);
        for (size_t c = 0; c < M; ++c) {
            rotate(h.cells[c].centroid.data(), dim, h.signs.data(), h.dim_pad, rot.data());
            pack_signs_trunc(rot.data(), h.dim_pad, &cb[c * nw], nw);
        }
    }
    v.cent_bits = upload_vec(cb);
    use_sq8_ = h.centroid_sq8 && !h.cent_sq8.empty();
    if (use_sq8_) {
        v.cent_sq8 = upload_vec(h.cent_sq8);
        v.csq_min = upload_vec(h.csq_min);
        v.csq_step = upload_vec(h.csq_step);
    }
    // ---- centroid tree ----
    v.tree_depth = 0;
    n_leaf_ = 0;
    tree_cap_ = 0;
    if (h.tree) {
        const CentroidTree& t = *h.tree;
        if (t.levels.size() > (size_t)dev::kMaxTreeLevels) return "centroid tree deeper than 8 levels";
        v.tree_depth = (int)t.levels.size();
        for (size_t i = 0; i < t.levels.size(); ++i) {
            v.tree_codes[i] = upload_vec(t.levels[i].codes);
            v.tree_child_start[i] = upload_vec(t.levels[i].child_start);
            v.tree_child_len[i] = upload_vec(t.levels[i].child_len);
            v.tree_n[i] = (int)t.levels[i].n;
            tree_cap_ = std::max(tree_cap_, t.levels[i].n);
        }
        v.leaf_codes = upload_vec(t.leaf_codes);
        v.leaf_ids = upload_vec(t.leaf_ids);
        v.n_leaf = (int)t.n_leaf;
        n_leaf_ = t.n_leaf;
        tree_cap_ = std::max(tree_cap_, t.n_leaf);
    }
    d_flags_ = static_cast<uint32_t*>(alloc(4 * sizeof(uint32_t)));
    for (void* p : allocs_)
        if (!p) return "device allocation failed";
    cudaError_t e = cudaDeviceSynchronize();
    if (e != cudaSuccess) return std::string("upload: ") + cudaGetErrorString(e);
    if (!d_flags_) return "device allocation failed";
    cudaMemset(d_flags_, 0, 4 * sizeof(uint32_t));
    view_ = v;
    version_ = h.version;
    return "";
}

int DeviceIndex::ensure_ws(size_t bytes, std::string& err) {
    void*& w = ws_[ws_sel_];
    size_t& wb = ws_bytes_[ws_sel_];
    if (bytes <= wb) return kOk;
    if (w) {
        cudaDeviceSynchronize();  // searches in flight on any stream may still use it
        cudaFree(w);
        w = nullptr;
        wb = 0;
    }
    size_t want = bytes + bytes / 4;
    CUDA_TRY(cudaMalloc(&w, want));
    wb = want;
    return kOk;
}

uint32_t DeviceIndex::read_flags(cudaStream_t st) {
    uint32_t f[4] = {0, 0, 0, 0};
    global_flags(st, f);
    return f[0] + f[1] + f[2];
}

int DeviceIndex::global_flags(cudaStream_t st, uint32_t out[4]) {
    out[0] = out[1] = out[2] = out[3] = 0;
    if (!exch_) {
        cudaMemcpyAsync(out, d_flags_, 4 * sizeof(uint32_t), cudaMemcpyDeviceToHost, st);
        return cudaStreamSynchronize(st) == cudaSuccess ? kOk : kCudaError;
    }
    // a sharded search's retry decision must be the same on every rank: gather all ranks' flags
    if (!d_flags_all_) d_flags_all_ = static_cast<uint32_t*>(alloc((size_t)shard_world_ * 4 * sizeof(uint32_t)));
    if (!d_flags_all_) return kOom;
    std::string err;
    int rc = exch_->all_gather(d_flags_, d_flags_all_, 4 * sizeof(uint32_t), st, err);
    if (rc != kOk) return rc;
    std::vector<uint32_t> all((size_t)shard_world_ * 4);
    cudaMemcpyAsync(all.data(), d_flags_all_, all.size() * sizeof(uint32_t), cudaMemcpyDeviceToHost, st);
    if (cudaStreamSynchronize(st) != cudaSuccess) return kCudaError;
    for (int r = 0; r < shard_world_; ++r)
        for (int i = 0; i < 4; ++i) out[i] += all[(size_t)r * 4 + i];
    return kOk;
}

bool DeviceIndex::use_cell_major(const HostIndex& h, const SearchArgs& a) const {
    // cm_ok (index.rs:3343-3348); a part of a split batch keeps the whole batch's choice
    if (a.path >= 0) return a.path == 1;
    return a.cell_major && h.compacted && (h.max_assign == 1 || !h.rep_off.empty()) && !h.has_filter &&
           (size_t)a.nq >= h.cm_min_batch;
}

int DeviceIndex::route(const HostIndex& h, const dev::QueryEnc& e, const float* dQ, int nq, int nprobe, float tc,
                       float beta, bool batch_router, uint16_t* hs, uint32_t* sl, uint32_t* sl_n,
                       uint32_t* tree_scratch, float* rs_scores, uint32_t* rs_items,
                       uint32_t* chosen, float* cscore, uint32_t* nch, cudaStream_t st, std::string& err) {
    const int M = view_.M;
    const size_t mult2 = std::max<size_t>(h.shortlist_mult, 2);
    int expect = (int)std::min<size_t>(n_live_, 1u << 30);  // typical shortlist length
    bool have_codes = h.two_stage && !h.cent_bits.empty();
    bool all_live = false;
    if (batch_router && have_codes) {
        // route_batch (index.rs:1873-1980): exact flat Hamming shortlist for every query
        int want_c = (int)std::min<size_t>((size_t)nprobe * mult2, n_live_);
        dev::launch_route_flat(view_, e, nq, want_c, hs, sl, sl_n, M, st);
        expect = want_c;
    } else if (h.tree) {
        // route_query tree branch (index.rs:1188-1211)
        int want_c = (int)std::min<size_t>((size_t)nprobe * mult2, n_leaf_);
        std::vector<size_t> b = h.tree->beams((size_t)want_c);
        int beams[dev::kMaxTreeLevels] = {0};
        for (size_t i = 0; i < b.size(); ++i) beams[i] = (int)b[i];
        dev::launch_route_tree(view_, e, nq, beams, want_c, tree_scratch, (int)tree_cap_, sl, sl_n, M, st);
        expect = want_c;
    } else if (h.graph_route && n_live_ >= h.graph_min_cells) {
        err = "centroid-graph routing is not supported by the GPU search; call set_graph_route(False)";
        return kUnsupported;
    } else if (have_codes) {
        // route_query two-stage branch (index.rs:1241-1259): note the multiplier is not floored at 2
        int want_c = (int)std::min<size_t>((size_t)nprobe * h.shortlist_mult, n_live_);
        dev::launch_route_flat(view_, e, nq, want_c, hs, sl, sl_n, M, st);
        expect = want_c;
    } else {
        dev::launch_route_all(view_, nq, sl, sl_n, M, st);
        all_live = true;
    }
    dev::launch_rescore_select(view_, e, dQ, nq, sl, sl_n, M, nprobe, tc, beta, use_sq8_, chosen, cscore, nch,
                               d_flags_ + 1, rs_scores, rs_items, expect, all_live, st);
    return kOk;
}

namespace {
template <typename T>
std::vector<T> fetch(const T* d, size_t n, cudaStream_t st) {
    std::vector<T> v(n);
    if (n) cudaMemcpyAsync(v.data(), d, n * sizeof(T), cudaMemcpyDeviceToHost, st);
    return v;
}
}  // namespace

int DeviceIndex::run_cellmajor(const HostIndex& h, const float* dQ, const SearchArgs& a, uint64_t* d_ids,
                               float* d_scores, uint32_t* d_nout, cudaStream_t st, std::string& err) {
    const int nq = a.nq, M = view_.M, dim = view_.dim, nw = view_.nw, npos = view_.npos;
    const int nprobe = std::max(1, std::min(a.nprobe, M));
    const int target = (int)std::max<size_t>((size_t)a.k * h.rerank_factor, 1);
    const int mwords = (M + 63) / 64;
    const int seed_cap = (int)std::max<size_t>(dev::kSeedCells * max_members_, 1);
    const int rest_cap = std::max(32 * target, 16384) * grow_factor;
    const int cand_cap = seed_cap + rest_cap;
    const bool tree_router = !(h.two_stage && !h.cent_bits.empty()) && h.tree;

    float* rsc = nullptr;       // rerank scores (nq x cand_cap) of the flattened gather
    float* rss = nullptr;       // centroid re-order scores of the shortlists (nq x M)
    uint32_t* rsi = nullptr;    // their item numbering (nq + 1)
    uint32_t* ritem = nullptr;  // its item numbering (nq + 1)
    auto carve = [&](Bump& bp, dev::QueryEnc& e, uint32_t*& sl, uint32_t*& sl_n, uint16_t*& hs, uint32_t*& tsc,
                     uint32_t*& chosen, float*& cscore, uint32_t*& nch, dev::CellMajorBufs& b) {
        e.qbits = bp.take<uint64_t>((size_t)nq * nw);
        e.lut = bp.take<uint8_t>((size_t)nq * npos * 16);
        e.fs_delta = bp.take<float>(nq);
        e.fs_bias = bp.take<float>(nq);
        e.cqs = bp.take<float>((size_t)nq * dim);
        e.cqbase = bp.take<float>(nq);
        e.rqs = bp.take<float>((size_t)nq * dim);
        e.rbase = bp.take<float>(nq);
        sl = bp.take<uint32_t>((size_t)nq * M);
        sl_n = bp.take<uint32_t>(nq);
        hs = bp.take<uint16_t>((size_t)nq * M);
        tsc = tree_router ? bp.take<uint32_t>((size_t)nq * 3 * tree_cap_) : nullptr;
        rss = bp.take<float>((size_t)nq * M);
        rsi = bp.take<uint32_t>((size_t)nq + 1);
        chosen = bp.take<uint32_t>((size_t)nq * nprobe);
        cscore = bp.take<float>((size_t)nq * nprobe);
        nch = bp.take<uint32_t>(nq);
        b.mwords = mwords;
        b.probed = h.max_assign > 1 ? bp.take<uint64_t>((size_t)nq * mwords) : nullptr;
        b.seed_cap = seed_cap;
        b.seed_buf = bp.take<uint64_t>((size_t)nq * seed_cap);
        b.seed_dcap = (int)(dev::kSeedCells * 8 * ((max_members_ + 7) / 8));
        b.seed_d = bp.take<uint16_t>((size_t)nq * b.seed_dcap);
        b.seed_n = bp.take<uint32_t>(nq);
        b.tau = bp.take<uint32_t>(nq);
        b.rest_hi = bp.take<uint32_t>(nq);
        b.cell_cnt = bp.take<uint32_t>((size_t)M + 1);
        b.cell_fill = bp.take<uint32_t>(M);
        b.qof = bp.take<uint32_t>((size_t)nq * nprobe);
        b.rest_cap = rest_cap;
        b.rest_buf = bp.take<uint64_t>((size_t)nq * rest_cap);
        b.rest_n = bp.take<uint32_t>(nq);
        b.cand_cap = cand_cap;
        b.cand = bp.take<uint32_t>((size_t)nq * cand_cap);
        b.cand_n = bp.take<uint32_t>(nq);
        b.overflow = d_flags_;
        b.gtau = bp.take<uint32_t>(nq);
        b.lad = bp.take<uint32_t>((size_t)nq * dev::kLadStride);
        b.work = bp.take<uint32_t>(1);
        rsc = bp.take<float>((size_t)nq * cand_cap);
        ritem = bp.take<uint32_t>((size_t)nq + 1);
    };
    dev::QueryEnc e{};
    uint32_t *sl, *sl_n, *tsc, *chosen, *nch;
    uint16_t* hs;
    float* cscore;
    dev::CellMajorBufs b{};
    Bump sizing{nullptr, 0, 0};
    carve(sizing, e, sl, sl_n, hs, tsc, chosen, cscore, nch, b);
    int rc = ensure_ws(sizing.off + 256, err);
    if (rc != kOk) return rc;
    Bump bp{static_cast<char*>(ws()), 0, ws_bytes()};
    carve(bp, e, sl, sl_n, hs, tsc, chosen, cscore, nch, b);

    last_ = LastCall{};
    last_.valid = true;
    last_.cell_major = true;
    last_.nq = nq;
    last_.nprobe = nprobe;
    last_.target = target;
    last_.nch = nch;
    last_.chosen = chosen;
    last_.sl_n = sl_n;
    last_.cell_cnt = b.cell_cnt;
    last_.cand_n = b.cand_n;
    last_.seed_n = b.seed_n;
    last_.rest_n = b.rest_n;
    last_.rest_hi = b.rest_hi;
    last_.st = st;
    dev::set_thread_clock(clock_.get());
    struct Unset {
        ~Unset() { dev::set_thread_clock(nullptr); }
    } unset;
    if (timing_) cudaEventRecord(ev_[0], st);
    dev::launch_encode(view_, dQ, nq, e, use_sq8_, view_.rerank_mode == 1, st);
    if (dbg && dbg->stage == 0) return debug_encode(e, nq, st);
    if (timing_) cudaEventRecord(ev_[1], st);
    rc = route(h, e, dQ, nq, nprobe, a.tc, a.beta, true, hs, sl, sl_n, tsc, rss, rsi, chosen, cscore, nch, st, err);
    if (rc != kOk) return rc;
    if (dbg && dbg->stage == 1) return debug_route(chosen, cscore, nch, nq, nprobe, st);
    if (timing_) cudaEventRecord(ev_[2], st);
    dev::launch_cellmajor(view_, e, nq, chosen, cscore, nch, nprobe, target, h.adaptive, h.at_margin, b, st);
    if (dbg && dbg->stage == 2) {
        dbg->seed_n = fetch(b.seed_n, nq, st);
        dbg->tau = fetch(b.tau, nq, st);
        dbg->rest_hi = fetch(b.rest_hi, nq, st);
        dbg->rest_n = fetch(b.rest_n, nq, st);
        return debug_cands(b.cand, b.cand_n, nq, cand_cap, st);
    }
    if (timing_) cudaEventRecord(ev_[3], st);
    dev::launch_rerank(view_, dQ, e, nq, b.cand, b.cand_n, cand_cap, a.k, d_ids, d_scores, d_nout, rsc, ritem,
                       d_flags_ + 2, st);
    if (timing_) cudaEventRecord(ev_[4], st);
    CUDA_TRY(cudaGetLastError());
    return kOk;
}

int DeviceIndex::run_perquery(const HostIndex& h, const float* dQ, const SearchArgs& a, uint64_t* d_ids,
                              float* d_scores, uint32_t* d_nout, cudaStream_t st, std::string& err) {
    const int M = view_.M, dim = view_.dim, nw = view_.nw, npos = view_.npos;
    const int nprobe = std::max(1, std::min(a.nprobe, M));
    const int want0 = (int)((size_t)a.k * h.rerank_factor);
    const int ent_cap = (int)std::min<size_t>((size_t)nprobe * max_members_ + 1, (size_t)1 << 30);
    // FastScan keeps exactly want0 candidates; the Hamming scan keeps every tie at its cut-off, so
    // its buffer has room to spare and grows after an overflow
    const int cand_cap = view_.ham ? (int)std::min<size_t>((size_t)(2 * std::max(want0, 1) + 256) * grow_factor,
                                                           (size_t)ent_cap)
                                   : std::max(want0, 1);
    const bool filtering = h.has_filter && !h.tags.empty();
    const bool tree_router = h.tree != nullptr;
    int chunk = a.nq;

    float* rsc = nullptr;       // rerank scores (chunk x cand_cap) of the flattened gather
    float* rss = nullptr;       // centroid re-order scores of the shortlists (chunk x M)
    uint32_t* rsi = nullptr;    // their item numbering (chunk + 1)
    uint32_t* ritem = nullptr;  // its item numbering (chunk + 1)
    auto carve = [&](Bump& bp, dev::QueryEnc& e, uint32_t*& sl, uint32_t*& sl_n, uint16_t*& hs, uint32_t*& tsc,
                     uint32_t*& chosen, float*& cscore, uint32_t*& nch, dev::PerQueryBufs& b) {
        int nq = chunk;
        e.qbits = bp.take<uint64_t>((size_t)nq * nw);
        e.lut = bp.take<uint8_t>((size_t)nq * npos * 16);
        e.fs_delta = bp.take<float>(nq);
        e.fs_bias = bp.take<float>(nq);
        e.cqs = bp.take<float>((size_t)nq * dim);
        e.cqbase = bp.take<float>(nq);
        e.rqs = bp.take<float>((size_t)nq * dim);
        e.rbase = bp.take<float>(nq);
        sl = bp.take<uint32_t>((size_t)nq * M);
        sl_n = bp.take<uint32_t>(nq);
        hs = bp.take<uint16_t>((size_t)nq * M);
        tsc = tree_router ? bp.take<uint32_t>((size_t)nq * 3 * tree_cap_) : nullptr;
        rss = bp.take<float>((size_t)nq * M);
        rsi = bp.take<uint32_t>((size_t)nq + 1);
        chosen = bp.take<uint32_t>((size_t)nq * nprobe);
        cscore = bp.take<float>((size_t)nq * nprobe);
        nch = bp.take<uint32_t>(nq);
        b.crank = bp.take<uint32_t>((size_t)nq * M);
        b.seg_off = bp.take<uint32_t>((size_t)nq * (nprobe + 1));
        b.ent_cap = ent_cap;
        b.ent = bp.take<uint64_t>((size_t)nq * ent_cap);
        b.cand_cap = cand_cap;
        b.cand = bp.take<uint32_t>((size_t)nq * cand_cap);
        b.cand_n = bp.take<uint32_t>(nq);
        b.overflow = d_flags_;
        rsc = bp.take<float>((size_t)nq * cand_cap);
        ritem = bp.take<uint32_t>((size_t)nq + 1);
    };
    dev::QueryEnc e{};
    uint32_t *sl, *sl_n, *tsc, *chosen, *nch;
    uint16_t* hs;
    float* cscore;
    dev::PerQueryBufs b{};
    Bump sizing{nullptr, 0, 0};
    carve(sizing, e, sl, sl_n, hs, tsc, chosen, cscore, nch, b);
    while (sizing.off > kPerQueryScratch && chunk > kPerQueryMinChunk) {
        chunk = std::max(kPerQueryMinChunk, (chunk + 1) / 2);
        sizing = Bump{nullptr, 0, 0};
        carve(sizing, e, sl, sl_n, hs, tsc, chosen, cscore, nch, b);
    }
    int rc = ensure_ws(sizing.off + 256, err);
    if (rc != kOk) return rc;
    Bump bp{static_cast<char*>(ws()), 0, ws_bytes()};
    carve(bp, e, sl, sl_n, hs, tsc, chosen, cscore, nch, b);

    last_ = LastCall{};
    last_.valid = a.nq <= chunk;
    last_.nq = a.nq;
    last_.nprobe = nprobe;
    last_.target = std::max(want0, 1);
    last_.nch = nch;
    last_.chosen = chosen;
    last_.sl_n = sl_n;
    last_.cand_n = b.cand_n;
    last_.st = st;
    dev::set_thread_clock(clock_.get());
    struct Unset {
        ~Unset() { dev::set_thread_clock(nullptr); }
    } unset;
    if (timing_) cudaEventRecord(ev_[0], st);
    for (int q0 = 0; q0 < a.nq; q0 += chunk) {
        int nq = std::min(chunk, a.nq - q0);
        const float* Qc = dQ + (size_t)q0 * dim;
        dev::launch_encode(view_, Qc, nq, e, use_sq8_, view_.rerank_mode == 1, st);
        if (dbg && dbg->stage == 0) return debug_encode(e, nq, st);
        if (timing_ && q0 == 0) cudaEventRecord(ev_[1], st);
        rc = route(h, e, Qc, nq, nprobe, a.tc, a.beta, false, hs, sl, sl_n, tsc, rss, rsi, chosen, cscore, nch, st, err);
        if (rc != kOk) return rc;
        if (dbg && dbg->stage == 1) return debug_route(chosen, cscore, nch, nq, nprobe, st);
        if (timing_ && q0 == 0) cudaEventRecord(ev_[2], st);
        dev::launch_perquery(view_, e, nq, chosen, cscore, nch, nprobe, want0, h.adaptive, h.at_margin, filtering,
                             h.filter_lo, h.filter_hi, b, st);
        if (dbg && dbg->stage == 2) return debug_cands(b.cand, b.cand_n, nq, cand_cap, st);
        if (timing_ && q0 == 0) cudaEventRecord(ev_[3], st);
        dev::launch_rerank(view_, Qc, e, nq, b.cand, b.cand_n, cand_cap, a.k, d_ids + (size_t)q0 * a.k,
                           d_scores + (size_t)q0 * a.k, d_nout + q0, rsc, ritem, d_flags_ + 2, st);
    }
    if (timing_) cudaEventRecord(ev_[4], st);
    CUDA_TRY(cudaGetLastError());
    return kOk;
}

int DeviceIndex::search_device(const HostIndex& h, const float* dQ, const SearchArgs& a, uint64_t* d_ids,
                               float* d_scores, uint32_t* d_nout, cudaStream_t st, std::string& err,
                               bool clear_flags) {
    if (h.version != version_) {
        err = "the index changed since it was uploaded";
        return kBadState;
    }
    if (a.k <= 0) {
        err = "k must be positive";
        return kBadArg;
    }
    if (a.k > 4096) {
        err = "k above 4096 is not supported";
        return kUnsupported;
    }
    if (a.nq <= 0) return kOk;
    cudaSetDevice(device_);
    if (!st) st = stream_;
    if (view_.ham && (exch_ || use_cell_major(h, a))) {
        err = exch_ ? "a sharded search needs FastScan blocks: call set_fastscan(True) and compact() first"
                    : "the GPU cell-major join needs FastScan blocks: call set_fastscan(True) (then compact()), "
                      "or search with cell_major=False";
        return kUnsupported;
    }
    if (clear_flags && split_halves(h, a)) return search_halves(h, dQ, nullptr, a, d_ids, d_scores, d_nout, st, err);
    if (a.path < 0) last_split_ = false;
    dev::take_launch_error(nullptr);
    // the previous search with this workspace may have been enqueued on another stream
    const int w = ws_sel_;
    if (ws_ev_live_[w]) cudaStreamWaitEvent(st, ws_ev_[w], 0);
    if (clear_flags) cudaMemsetAsync(d_flags_, 0, 4 * sizeof(uint32_t), st);
    int rc = exch_                  ? search_sharded(h, dQ, a, d_ids, d_scores, d_nout, st, err)
             : use_cell_major(h, a) ? run_cellmajor(h, dQ, a, d_ids, d_scores, d_nout, st, err)
                                    : run_perquery(h, dQ, a, d_ids, d_scores, d_nout, st, err);
    if (!ws_ev_[w]) cudaEventCreateWithFlags(&ws_ev_[w], cudaEventDisableTiming);
    ws_ev_live_[w] = ws_ev_[w] && cudaEventRecord(ws_ev_[w], st) == cudaSuccess;
    int kid = -1;
    cudaError_t le = dev::take_launch_error(&kid);
    if (le != cudaSuccess) {
        err = std::string("launch of ") + dev::kernel_name(kid) + " failed: " + cudaGetErrorString(le);
        return le == cudaErrorMemoryAllocation ? kOom : kCudaError;
    }
    return rc;
}

bool DeviceIndex::split_halves(const HostIndex& h, const SearchArgs& a) const {
    // beyond the seed cells the join scans each probed cell once for all the queries that probe
    // it, and halves would scan it twice (measured: 4.58 -> 6.16 ms for 5,000 queries at nprobe 256)
    if (exch_ || dbg || timing_ || a.path >= 0 || a.nq < kSplitQueries) return false;
    return use_cell_major(h, a) && std::min(a.nprobe, view_.M) <= dev::kSeedCells;
}

int DeviceIndex::search_halves(const HostIndex& h, const float* dQ, const float* hQ, const SearchArgs& a,
                               uint64_t* d_ids, float* d_scores, uint32_t* d_nout, cudaStream_t st,
                               std::string& err) {
    if (!stream2_) {
        CUDA_TRY(cudaStreamCreateWithFlags(&stream2_, cudaStreamNonBlocking));
        for (auto& e : split_ev_) CUDA_TRY(cudaEventCreateWithFlags(&e, cudaEventDisableTiming));
    }
    const size_t nq = a.nq, dim = view_.dim, k = a.k;
    const size_t half = (nq / 2) & ~size_t(63);  // keeps the second half 256-byte aligned
    const size_t q0[2] = {0, half}, n[2] = {half, nq - half};
    cudaStream_t ps[2] = {st, stream2_};
    SearchArgs part = a;
    part.path = use_cell_major(h, a) ? 1 : 0;
    // the counters are cleared once, before either half can raise one
    CUDA_TRY(cudaMemsetAsync(d_flags_, 0, 4 * sizeof(uint32_t), st));
    CUDA_TRY(cudaEventRecord(split_ev_[0], st));
    CUDA_TRY(cudaStreamWaitEvent(stream2_, split_ev_[0], 0));
    // both halves' copies before either search, so that the second crosses PCIe during the first
    // search (a copy enqueued after the first half's launches measured slower)
    if (hQ)
        for (int p = 0; p < 2; ++p)
            CUDA_TRY(cudaMemcpyAsync(const_cast<float*>(dQ) + q0[p] * dim, hQ + q0[p] * dim,
                                     n[p] * dim * sizeof(float), cudaMemcpyHostToDevice, ps[p]));
    int rc = kOk;
    for (int p = 0; p < 2 && rc == kOk; ++p) {
        part.nq = (int)n[p];
        ws_sel_ = p;
        rc = search_device(h, dQ + q0[p] * dim, part, d_ids + q0[p] * k, d_scores + q0[p] * k,
                           d_nout ? d_nout + q0[p] : nullptr, ps[p], err, false);
        ws_sel_ = 0;
        last_half_[p] = last_;
    }
    last_split_ = rc == kOk;
    // the caller's stream goes on after both halves
    CUDA_TRY(cudaEventRecord(split_ev_[1], stream2_));
    CUDA_TRY(cudaStreamWaitEvent(st, split_ev_[1], 0));
    return rc;
}

int DeviceIndex::search_host(const HostIndex& h, const float* Q, const SearchArgs& a, uint64_t* ids, float* scores,
                             uint32_t* nout, std::string& err) {
    if (a.nq <= 0) return kOk;
    cudaSetDevice(device_);
    const size_t nq = a.nq, k = a.k, dim = view_.dim;
    auto al = [](size_t b) { return (b + 255) & ~size_t(255); };
    const size_t qb = nq * dim * sizeof(float), ib = nq * k * sizeof(uint64_t), sb = nq * k * sizeof(float),
                 nb = nq * sizeof(uint32_t), fb = 4 * sizeof(uint32_t);
    const size_t need = al(qb) + al(ib) + al(sb) + al(nb) + al(fb);
    // pinned staging and device I/O buffers persist across calls (grown on demand), so a call
    // allocates nothing in the common case and synchronises once
    if (need > pin_bytes_) {
        if (pin_) cudaFreeHost(pin_);
        pin_ = nullptr;
        pin_bytes_ = 0;
        CUDA_TRY(cudaMallocHost(&pin_, need));
        pin_bytes_ = need;
    }
    if (need > io_bytes_) {
        if (io_) {
            cudaStreamSynchronize(stream_);
            cudaFree(io_);
        }
        io_ = nullptr;
        io_bytes_ = 0;
        CUDA_TRY(cudaMalloc(&io_, need));
        io_bytes_ = need;
    }
    char* hp = static_cast<char*>(pin_);
    char* dp = static_cast<char*>(io_);
    float* hQ_stage = reinterpret_cast<float*>(hp);
    uint64_t* hI = reinterpret_cast<uint64_t*>(hp + al(qb));
    float* hS = reinterpret_cast<float*>(hp + al(qb) + al(ib));
    uint32_t* hN = reinterpret_cast<uint32_t*>(hp + al(qb) + al(ib) + al(sb));
    uint32_t* hF = reinterpret_cast<uint32_t*>(hp + al(qb) + al(ib) + al(sb) + al(nb));
    float* dQ = reinterpret_cast<float*>(dp);
    uint64_t* dI = reinterpret_cast<uint64_t*>(dp + al(qb));
    float* dS = reinterpret_cast<float*>(dp + al(qb) + al(ib));
    uint32_t* dN = reinterpret_cast<uint32_t*>(dp + al(qb) + al(ib) + al(sb));
    // queries already in page-locked memory (cudaMallocHost / cudaHostRegister, e.g. a pinned torch
    // tensor) are copied to the device from where they are; any other buffer goes through the
    // pinned staging copy first
    cudaPointerAttributes pa{};
    const cudaError_t pe = cudaPointerGetAttributes(&pa, Q);
    if (pe != cudaSuccess) cudaGetLastError();  // clears the (non-sticky) error of an unknown pointer
    const bool q_pinned = pe == cudaSuccess && pa.type == cudaMemoryTypeHost;
    const float* hQ = q_pinned ? Q : hQ_stage;
    // staging copy into pinned memory: large batches are copied by several host threads (one
    // thread's memcpy is slower than the PCIe transfer that follows)
    if (!q_pinned) {
        constexpr size_t kPart = size_t(256) << 10;
        const long long parts = (long long)((qb + kPart - 1) / kPart);
        const int thr = (int)std::min<long long>(std::min(parts, 8LL), (long long)omp_get_max_threads());
        if (thr > 1) {
#pragma omp parallel for num_threads(thr) schedule(static)
            for (long long i = 0; i < parts; ++i) {
                const size_t o = (size_t)i * kPart;
                std::memcpy(reinterpret_cast<char*>(hQ_stage) + o, reinterpret_cast<const char*>(Q) + o,
                            std::min(kPart, qb - o));
            }
        } else {
            std::memcpy(hQ_stage, Q, qb);
        }
    }
    // ids, scores and counts are laid out alike in the device and pinned buffers: one copy back
    const size_t out_off = al(qb), out_len = al(ib) + al(sb) + nb;
    const bool split = split_halves(h, a);
    int rc = kOk;
    for (int attempt = 0; attempt < 4; ++attempt) {
        if (!split) {
            CUDA_TRY(cudaMemcpyAsync(dQ, hQ, qb, cudaMemcpyHostToDevice, stream_));
            rc = search_device(h, dQ, a, dI, dS, dN, stream_, err);
        } else {
            rc = search_halves(h, dQ, hQ, a, dI, dS, dN, stream_, err);
        }
        if (rc != kOk) return rc;
        CUDA_TRY(cudaMemcpyAsync(hp + out_off, dp + out_off, out_len, cudaMemcpyDeviceToHost, stream_));
        CUDA_TRY(cudaMemcpyAsync(hF, d_flags_, fb, cudaMemcpyDeviceToHost, stream_));
        CUDA_TRY(cudaStreamSynchronize(stream_));
        if (exch_) {
            rc = global_flags(stream_, hF);
            if (rc != kOk) {
                err = "gathering the shards' overflow flags failed";
                return rc;
            }
        }
        if (hF[1] != 0) {
            err = "a routing shortlist exceeded 16384 cells; lower nprobe or the shortlist multiplier";
            return kUnsupported;
        }
        if (hF[2] != 0) {
            err = "a bounded wait for the GPU's copy or tensor-core engines ran out; the results are not valid";
            return kCudaError;
        }
        if (hF[0] == 0) break;
        if (attempt == 3) {
            err = "candidate buffers overflowed after enlarging them";
            return kOverflow;
        }
        grow_factor *= 4;
    }
    std::memcpy(ids, hI, ib);
    std::memcpy(scores, hS, sb);
    if (nout) std::memcpy(nout, hN, nb);
    return kOk;
}

void DeviceIndex::enable_kernel_clock(bool on) {
    if (on && !clock_) clock_ = std::make_unique<dev::KernelClock>();
    if (!on) clock_.reset();
}

std::vector<std::pair<std::string, double>> DeviceIndex::last_stats() {
    std::vector<std::pair<std::string, double>> out;
    // a split batch: its two halves' per-query arrays, one after the other (only the seed-only join
    // splits, so there is no per-cell query count to combine)
    std::vector<const LastCall*> parts;
    if (last_split_)
        parts = {&last_half_[0], &last_half_[1]};
    else
        parts = {&last_};
    for (const LastCall* p : parts)
        if (!p->valid) return out;
    cudaSetDevice(device_);
    int nq = 0;
    for (const LastCall* p : parts) {
        cudaStreamSynchronize(p->st);
        nq += p->nq;
    }
    const int np = last_.nprobe, M = view_.M;
    auto get = [&](const uint32_t* d, size_t n) {
        std::vector<uint32_t> v(n, 0);
        if (d && n) cudaMemcpy(v.data(), d, n * sizeof(uint32_t), cudaMemcpyDeviceToHost);
        return v;
    };
    // the per-query array `field` of every part, concatenated (`per` entries a query)
    auto gather = [&](const uint32_t* LastCall::*field, size_t per) {
        std::vector<uint32_t> v;
        for (const LastCall* p : parts) {
            std::vector<uint32_t> x = get(p->*field, (size_t)p->nq * per);
            v.insert(v.end(), x.begin(), x.end());
        }
        return v;
    };
    std::vector<uint32_t> nch = gather(&LastCall::nch, 1), chosen = gather(&LastCall::chosen, np),
                          sl_n = gather(&LastCall::sl_n, 1), cand_n = gather(&LastCall::cand_n, 1);
    const double code_bytes = (double)view_.nw * 8.0;
    double probes = 0, shortlist = 0, cands = 0;
    for (int q = 0; q < nq; ++q) {
        probes += nch[q];
        shortlist += sl_n[q];
        cands += cand_n[q];
    }
    out.push_back({"nq", (double)nq});
    out.push_back({"probes", probes});
    out.push_back({"shortlist", shortlist});
    out.push_back({"candidates", cands});
    double row_bytes = view_.rerank_mode == 0 ? 4.0 * view_.dim : (double)view_.dim;
    out.push_back({"rerank_row_bytes", row_bytes});
    out.push_back({"rerank_bytes", cands * row_bytes});
    out.push_back({"route_code_bytes", (double)M * code_bytes});
    if (last_.cell_major) {
        std::vector<uint32_t> start = np > dev::kSeedCells && !last_split_ ? get(last_.cell_cnt, (size_t)M + 1)
                                                                           : std::vector<uint32_t>((size_t)M + 1, 0),
                              seed_n = gather(&LastCall::seed_n, 1),
                              rest_n = gather(&LastCall::rest_n, 1), rest_hi = gather(&LastCall::rest_hi, 1);
        double cells = 0, bytes = 0, pairs = 0, seed_pairs = 0, seed_kept = 0, rest_kept = 0, rest_probes = 0;
        std::vector<uint8_t> seen(M, 0);
        double seed_bytes = 0, seed_union_bytes = 0;
        std::vector<uint8_t> seed_seen(M, 0);
        for (int c = 0; c < M; ++c) {
            uint32_t nqc = start[c + 1] - start[c];
            double nc = (double)(moff_[c + 1] - moff_[c]);
            if (nqc) {
                cells += 1;
                bytes += nc * code_bytes;
                pairs += nqc * nc;
                seen[c] = 1;
            }
        }
        for (int q = 0; q < nq; ++q) {
            int ns = std::min<int>(dev::kSeedCells, (int)nch[q]);
            for (int r = 0; r < ns; ++r) {
                uint32_t c = chosen[(size_t)q * np + r];
                double nc = (double)(moff_[c + 1] - moff_[c]);
                seed_pairs += nc;
                if (!seed_seen[c]) {
                    seed_seen[c] = 1;
                    seed_union_bytes += nc * code_bytes;
                }
                if (!seen[c]) {
                    seen[c] = 2;
                    seed_bytes += nc * code_bytes;
                }
            }
            seed_kept += seed_n[q];
            rest_kept += rest_n[q];
            rest_probes += (double)rest_hi[q] - ns;
        }
        out.push_back({"scan_cells", cells});
        out.push_back({"scan_code_bytes", bytes});
        out.push_back({"scan_pairs", pairs});
        out.push_back({"seed_pairs", seed_pairs});
        out.push_back({"seed_extra_code_bytes", seed_bytes});
        out.push_back({"seed_code_bytes", seed_union_bytes});
        out.push_back({"seed_kept", seed_kept});
        out.push_back({"rest_kept", rest_kept});
        out.push_back({"rest_probes", rest_probes});
    }
    return out;
}

int DeviceIndex::debug_encode(const dev::QueryEnc& e, int nq, cudaStream_t st) {
    dbg->qbits = fetch(e.qbits, (size_t)nq * view_.nw, st);
    dbg->lut = fetch(e.lut, (size_t)nq * view_.npos * 16, st);
    dbg->delta = fetch(e.fs_delta, nq, st);
    dbg->bias = fetch(e.fs_bias, nq, st);
    cudaStreamSynchronize(st);
    return kOk;
}

int DeviceIndex::debug_route(const uint32_t* chosen, const float* cscore, const uint32_t* nch, int nq, int nprobe,
                             cudaStream_t st) {
    dbg->nprobe = nprobe;
    dbg->chosen = fetch(chosen, (size_t)nq * nprobe, st);
    dbg->cscore = fetch(cscore, (size_t)nq * nprobe, st);
    dbg->nch = fetch(nch, nq, st);
    cudaStreamSynchronize(st);
    return kOk;
}

int DeviceIndex::debug_cands(const uint32_t* cand, const uint32_t* cand_n, int nq, int cap, cudaStream_t st) {
    dbg->cand_cap = cap;
    dbg->cand = fetch(cand, (size_t)nq * cap, st);
    dbg->cand_n = fetch(cand_n, nq, st);
    cudaStreamSynchronize(st);
    return kOk;
}

PhaseTimes DeviceIndex::collect_phases() {
    PhaseTimes p;
    if (!timing_ || !ev_[4]) return p;
    if (cudaEventSynchronize(ev_[4]) != cudaSuccess) return p;
    cudaEventElapsedTime(&p.encode, ev_[0], ev_[1]);
    cudaEventElapsedTime(&p.route, ev_[1], ev_[2]);
    cudaEventElapsedTime(&p.scan, ev_[2], ev_[3]);
    cudaEventElapsedTime(&p.rerank, ev_[3], ev_[4]);
    return p;
}

}  // namespace maivs
