// Cell-range sharded search: each rank scans only its cells, three all-gathers keep the result
// identical to the unsharded cell-major join (index.rs:1999-2311).
//
// Every rank encodes the whole batch and routes its block of ceil(nq / world) queries; the probe
// lists are all-gathered (the routing tables are replicated, so every rank then holds the probe
// lists and the exactly-once rule of the unsharded join). Then each rank:
//   1. scans the seed probes that fall in its cells and publishes, per query, its entry count and
//      its smallest `target` distances; all-gather -> every rank derives the global seed cut-off
//      tau, its own seed survivors and the adaptive end of the rest probes;
//   2. (nprobe > 8) scans the rest probes in its cells with tau and publishes its survivors'
//      smallest `target` distances; all-gather -> the global candidate cut (target-th smallest,
//      ties kept, index.rs:2277-2306); with no rest scan every seed survivor is already inside it;
//   3. reranks its candidates to its best k; all-gather -> the best-k lists are merged on the
//      device by (score desc, external id asc).
// The exchanged lists are a few bytes per candidate (u16 distances, then k ids and scores per
// query), not the candidates themselves.
#include <dlfcn.h>
#include <nccl.h>

#include <algorithm>
#include <chrono>
#include <cstring>
#include <thread>

#include "engine.h"

namespace maivs {

namespace {

struct Bump {
    char* base;
    size_t off = 0;
    template <typename T>
    T* take(size_t n) {
        size_t a = (off + 255) & ~size_t(255);
        off = a + n * sizeof(T);
        return base ? reinterpret_cast<T*>(base + a) : nullptr;
    }
};

// ---- NCCL, loaded at first use so that single-GPU users need no libnccl ----
struct NcclApi {
    bool ok = false;
    std::string why;
    ncclResult_t (*GetUniqueId)(ncclUniqueId*) = nullptr;
    ncclResult_t (*CommInitRankConfig)(ncclComm_t*, int, ncclUniqueId, int, ncclConfig_t*) = nullptr;
    ncclResult_t (*CommGetAsyncError)(ncclComm_t, ncclResult_t*) = nullptr;
    ncclResult_t (*AllGather)(const void*, void*, size_t, ncclDataType_t, ncclComm_t, cudaStream_t) = nullptr;
    ncclResult_t (*CommDestroy)(ncclComm_t) = nullptr;
    ncclResult_t (*CommAbort)(ncclComm_t) = nullptr;
    const char* (*GetErrorString)(ncclResult_t) = nullptr;
};

const NcclApi& nccl() {
    static NcclApi api = [] {
        NcclApi a;
        void* h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_GLOBAL);
        if (!h) {
            a.why = std::string("libnccl.so.2 could not be loaded: ") + dlerror();
            return a;
        }
        auto sym = [&](const char* n) { return dlsym(h, n); };
        a.GetUniqueId = reinterpret_cast<decltype(a.GetUniqueId)>(sym("ncclGetUniqueId"));
        a.CommInitRankConfig = reinterpret_cast<decltype(a.CommInitRankConfig)>(sym("ncclCommInitRankConfig"));
        a.CommGetAsyncError = reinterpret_cast<decltype(a.CommGetAsyncError)>(sym("ncclCommGetAsyncError"));
        a.AllGather = reinterpret_cast<decltype(a.AllGather)>(sym("ncclAllGather"));
        a.CommDestroy = reinterpret_cast<decltype(a.CommDestroy)>(sym("ncclCommDestroy"));
        a.CommAbort = reinterpret_cast<decltype(a.CommAbort)>(sym("ncclCommAbort"));
        a.GetErrorString = reinterpret_cast<decltype(a.GetErrorString)>(sym("ncclGetErrorString"));
        a.ok = a.GetUniqueId && a.CommInitRankConfig && a.CommGetAsyncError && a.AllGather && a.CommDestroy &&
               a.CommAbort && a.GetErrorString;
        if (!a.ok) a.why = "libnccl.so.2 lacks a required entry point";
        return a;
    }();
    return api;
}

constexpr double kNcclWaitSeconds = 120.0;  // communicator set-up and each collective's enqueue

// Waits for a non-blocking communicator to leave ncclInProgress; aborts it on error or timeout.
// A collective's enqueue normally settles within microseconds, and the search stream gets no
// further launches until it has, so the first 2 ms poll with yields; longer waits (communicator
// set-up) sleep 50 us between polls.
ncclResult_t nccl_settle(ncclComm_t comm) {
    const NcclApi& n = nccl();
    auto t0 = std::chrono::steady_clock::now();
    ncclResult_t st = ncclInProgress;
    for (;;) {
        if (n.CommGetAsyncError(comm, &st) != ncclSuccess) return ncclSystemError;
        if (st != ncclInProgress) return st;
        double s = std::chrono::duration<double>(std::chrono::steady_clock::now() - t0).count();
        if (s > kNcclWaitSeconds) return ncclInProgress;
        if (s < 2e-3)
            std::this_thread::yield();
        else
            std::this_thread::sleep_for(std::chrono::microseconds(50));
    }
}

class NcclExchange final : public Exchange {
   public:
    explicit NcclExchange(ncclComm_t c) : comm_(c) {}
    ~NcclExchange() override {
        if (comm_) nccl().CommDestroy(comm_);
    }
    int all_gather(const void* send, void* recv, size_t bytes, cudaStream_t st, std::string& err) override {
        const NcclApi& n = nccl();
        ncclResult_t r = n.AllGather(send, recv, bytes, ncclUint8, comm_, st);
        if (r == ncclInProgress) r = nccl_settle(comm_);
        if (r != ncclSuccess) {
            err = std::string("ncclAllGather: ") + (r == ncclInProgress ? "timed out" : n.GetErrorString(r));
            n.CommAbort(comm_);
            comm_ = nullptr;
            return kCudaError;
        }
        return kOk;
    }

   private:
    ncclComm_t comm_;
};

}  // namespace

int nccl_unique_id(uint8_t* id, std::string& err) {
    const NcclApi& n = nccl();
    if (!n.ok) {
        err = n.why;
        return kUnsupported;
    }
    ncclUniqueId u;
    ncclResult_t r = n.GetUniqueId(&u);
    if (r != ncclSuccess) {
        err = std::string("ncclGetUniqueId: ") + n.GetErrorString(r);
        return kCudaError;
    }
    std::memcpy(id, u.internal, NCCL_UNIQUE_ID_BYTES);
    return kOk;
}

std::unique_ptr<Exchange> nccl_exchange(const uint8_t* id, int rank, int world, int device, std::string& err) {
    const NcclApi& n = nccl();
    if (!n.ok) {
        err = n.why;
        return nullptr;
    }
    cudaSetDevice(device);
    ncclUniqueId u;
    std::memcpy(u.internal, id, NCCL_UNIQUE_ID_BYTES);
    ncclConfig_t cfg = NCCL_CONFIG_INITIALIZER;
    cfg.blocking = 0;  // bounded set-up: a rank that never joins ends in an error, not a hang
    ncclComm_t comm = nullptr;
    ncclResult_t r = n.CommInitRankConfig(&comm, world, u, rank, &cfg);
    if (r == ncclInProgress) r = nccl_settle(comm);
    if (r != ncclSuccess) {
        err = std::string("ncclCommInitRankConfig: ") + (r == ncclInProgress ? "timed out" : n.GetErrorString(r));
        if (comm) n.CommAbort(comm);
        return nullptr;
    }
    return std::make_unique<NcclExchange>(comm);
}

void shard_range(const HostIndex& h, int rank, int world, uint32_t* lo, uint32_t* hi) {
    const size_t M = h.cells.size();
    unsigned long long total = 0;
    for (const auto& c : h.cells) total += c.members.size();
    auto bound = [&](int r) -> uint32_t {
        if (r <= 0) return 0;
        if (r >= world) return (uint32_t)M;
        // first cell whose preceding entries reach r / world of the total
        unsigned long long run = 0;
        for (size_t c = 0; c < M; ++c) {
            if (run * (unsigned long long)world >= (unsigned long long)r * total) return (uint32_t)c;
            run += h.cells[c].members.size();
        }
        return (uint32_t)M;
    };
    *lo = bound(rank);
    *hi = bound(rank + 1);
}

int DeviceIndex::shard_begin(const HostIndex& h, const float* dQ, const SearchArgs& a, int W, int rank,
                             cudaStream_t st, ShardRun& r, std::string& err) {
    const int nq = a.nq, M = view_.M, dim = view_.dim, nw = view_.nw, npos = view_.npos;
    r = ShardRun{};
    r.nq = nq;
    r.k = a.k;
    r.W = W;
    r.rank = rank;
    r.qb = (nq + W - 1) / W;
    r.dQ = dQ;
    r.st = st;
    r.nprobe = std::max(1, std::min(a.nprobe, M));
    r.target = (int)std::max<size_t>((size_t)a.k * h.rerank_factor, 1);
    r.xl = r.target;
    r.rest = r.nprobe > dev::kSeedCells;
    if ((size_t)W * a.k > 8192) {
        err = "the sharded search merges at most 8192 results per query (world x k)";
        return kUnsupported;
    }
    if (r.target > 65535) {
        err = "k x rerank_factor above 65535 is not supported by the sharded search";
        return kUnsupported;
    }
    r.lb = dev::shard_list_block_bytes(nq, r.xl);
    r.tb = dev::shard_topk_block_bytes(nq, a.k);
    const int nprobe = r.nprobe, target = r.target;
    const int mwords = (M + 63) / 64;
    const int seed_cap = (int)std::max<size_t>(dev::kSeedCells * max_members_, 1);
    const int rest_cap = std::max(32 * target, 16384) * grow_factor;
    const int cand_cap = seed_cap + rest_cap;
    const bool tree_router = !(h.two_stage && !h.cent_bits.empty()) && h.tree;
    uint32_t *sl, *sl_n, *tsc, *rsi;
    float* rss;
    uint16_t* hs;
    auto carve = [&](Bump& bp) {
        dev::QueryEnc& e = r.e;
        dev::CellMajorBufs& b = r.b;
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
        rss = bp.take<float>((size_t)r.qb * M);
        rsi = bp.take<uint32_t>((size_t)r.qb + 1);
        r.chosen = bp.take<uint32_t>((size_t)W * r.qb * nprobe);
        r.cscore = bp.take<float>((size_t)W * r.qb * nprobe);
        r.nch = bp.take<uint32_t>((size_t)W * r.qb);
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
        r.rsc = bp.take<float>((size_t)nq * cand_cap);
        r.ritem = bp.take<uint32_t>((size_t)nq + 1);
        r.xsend = bp.take<uint8_t>(r.lb);
        r.xrecv = bp.take<uint8_t>(r.lb * W);
        r.tsend = bp.take<uint8_t>(r.tb);
        r.trecv = bp.take<uint8_t>(r.tb * W);
    };
    Bump sizing{nullptr};
    carve(sizing);
    int rc = ensure_ws(sizing.off + 256, err);
    if (rc != kOk) return rc;
    Bump bp{static_cast<char*>(ws())};
    carve(bp);

    last_ = LastCall{};
    last_.valid = true;
    last_.cell_major = true;
    last_.nq = nq;
    last_.nprobe = nprobe;
    last_.target = target;
    last_.nch = r.nch;
    last_.chosen = r.chosen;
    last_.sl_n = sl_n;
    last_.cell_cnt = r.b.cell_cnt;
    last_.cand_n = r.b.cand_n;
    last_.seed_n = r.b.seed_n;
    last_.rest_n = r.b.rest_n;
    last_.rest_hi = r.b.rest_hi;
    last_.st = st;

    dev::launch_encode(view_, dQ, nq, r.e, use_sq8_, view_.rerank_mode == 1, st);
    // route_batch is per query: this rank routes its block, the probe lists are then all-gathered
    const int q0 = rank * r.qb, qn = std::max(0, std::min(r.qb, nq - q0));
    if (qn > 0) {
        dev::QueryEnc eb = r.e;
        eb.qbits += (size_t)q0 * nw;
        eb.lut += (size_t)q0 * npos * 16;
        eb.fs_delta += q0;
        eb.fs_bias += q0;
        eb.cqs += (size_t)q0 * dim;
        eb.cqbase += q0;
        eb.rqs += (size_t)q0 * dim;
        eb.rbase += q0;
        rc = route(h, eb, dQ + (size_t)q0 * dim, qn, nprobe, a.tc, a.beta, true, hs, sl, sl_n, tsc, rss, rsi,
                   r.chosen + (size_t)q0 * nprobe, r.cscore + (size_t)q0 * nprobe, r.nch + q0, st, err);
        if (rc != kOk) return rc;
    }
    if (!r.rest) cudaMemsetAsync(r.b.cell_cnt, 0, sizeof(uint32_t) * ((size_t)M + 1), st);  // read by stats
    return kOk;
}

void DeviceIndex::shard_seed(const HostIndex& h, ShardRun& r) {
    dev::launch_seed(view_, r.e, r.nq, r.chosen, r.cscore, r.nch, r.nprobe, r.target, h.adaptive, h.at_margin, r.b,
                     reinterpret_cast<uint16_t*>(r.xsend + (size_t)r.nq * 4), reinterpret_cast<uint32_t*>(r.xsend),
                     r.xl, r.st);
}

void DeviceIndex::shard_after_seed(const HostIndex& h, ShardRun& r) {
    dev::launch_seed_finish(view_, r.e, r.nq, r.chosen, r.cscore, r.nch, r.nprobe, r.target, h.adaptive,
                            h.at_margin, r.b, r.xrecv, r.lb, r.W, r.xl, r.st);
    if (!r.rest) return;
    dev::launch_rest_scan(view_, r.e, r.nq, r.chosen, r.nch, r.nprobe, r.b, r.st);
    dev::launch_local_list(r.b, r.nq, reinterpret_cast<uint16_t*>(r.xsend + (size_t)r.nq * 4),
                           reinterpret_cast<uint32_t*>(r.xsend), r.xl, r.st);
}

void DeviceIndex::shard_after_cut(const HostIndex&, ShardRun& r) {
    dev::launch_final(r.b, r.nq, r.target, r.rest ? r.xrecv : nullptr, r.lb, r.W, r.xl, r.st);
    const size_t nk = (size_t)r.nq * r.k;
    dev::launch_rerank(view_, r.dQ, r.e, r.nq, r.b.cand, r.b.cand_n, r.b.cand_cap, r.k,
                       reinterpret_cast<uint64_t*>(r.tsend), reinterpret_cast<float*>(r.tsend + nk * 8),
                       reinterpret_cast<uint32_t*>(r.tsend + nk * 12), r.rsc, r.ritem, r.b.overflow + 2, r.st);
}

void DeviceIndex::shard_merge(ShardRun& r, uint64_t* d_ids, float* d_scores, uint32_t* d_nout) {
    dev::launch_merge_topk(r.trecv, r.tb, r.W, r.nq, r.k, d_ids, d_scores, d_nout, r.st);
}

int DeviceIndex::search_sharded(const HostIndex& h, const float* dQ, const SearchArgs& a, uint64_t* d_ids,
                                float* d_scores, uint32_t* d_nout, cudaStream_t st, std::string& err) {
    dev::set_thread_clock(clock_.get());
    struct Unset {
        ~Unset() { dev::set_thread_clock(nullptr); }
    } unset;
    ShardRun r;
    int rc = shard_begin(h, dQ, a, shard_world_, shard_rank_, st, r, err);
    if (rc != kOk) return rc;
    // every exchange is an NCCL all-gather on the search stream, timed as one step on the clock
    auto gather = [&](const void* src, void* dst, size_t bytes) {
        dev::clock_begin(dev::kKAllGather, st);
        int g = exch_->all_gather(src, dst, bytes, st, err);
        dev::clock_end(dev::kKAllGather, st);
        return g;
    };
    // probe lists: in-place all-gathers of each rank's block of rows
    const size_t rows = (size_t)r.qb * r.nprobe;
    rc = gather(r.chosen + (size_t)r.rank * rows, r.chosen, rows * 4);
    if (rc == kOk) rc = gather(r.cscore + (size_t)r.rank * rows, r.cscore, rows * 4);
    if (rc == kOk) rc = gather(r.nch + (size_t)r.rank * r.qb, r.nch, (size_t)r.qb * 4);
    if (rc != kOk) return rc;
    shard_seed(h, r);
    rc = gather(r.xsend, r.xrecv, r.lb);
    if (rc != kOk) return rc;
    shard_after_seed(h, r);
    if (r.rest) {
        rc = gather(r.xsend, r.xrecv, r.lb);
        if (rc != kOk) return rc;
    }
    shard_after_cut(h, r);
    rc = gather(r.tsend, r.trecv, r.tb);
    if (rc != kOk) return rc;
    shard_merge(r, d_ids, d_scores, d_nout);
    return kOk;
}

int search_emulated_shards(const HostIndex& h, std::vector<std::unique_ptr<DeviceIndex>>& shards, const float* dQ,
                           const SearchArgs& a, uint64_t* d_ids, float* d_scores, uint32_t* d_nout, cudaStream_t st,
                           std::string& err) {
    const int W = (int)shards.size();
    for (auto& sh : shards)
        if (sh->hamming()) {
            err = "a sharded search needs FastScan blocks: call set_fastscan(True) and compact() first";
            return kUnsupported;
        }
    std::vector<DeviceIndex::ShardRun> runs(W);
    auto gather = [&](bool topk) -> int {
        for (int s = 0; s < W; ++s)
            for (int r = 0; r < W; ++r) {
                const size_t n = topk ? runs[r].tb : runs[r].lb;
                uint8_t* dst = (topk ? runs[s].trecv : runs[s].xrecv) + (size_t)r * n;
                const uint8_t* src = topk ? runs[r].tsend : runs[r].xsend;
                if (cudaMemcpyAsync(dst, src, n, cudaMemcpyDeviceToDevice, st) != cudaSuccess) {
                    err = "device copy between emulated shards failed";
                    return kCudaError;
                }
            }
        return kOk;
    };
    dev::take_launch_error(nullptr);
    for (int s = 0; s < W; ++s) {
        int rc = shards[s]->shard_begin(h, dQ, a, W, s, st, runs[s], err);
        if (rc != kOk) return rc;
    }
    // probe lists: shard r's block of rows to every shard
    for (int s = 0; s < W; ++s)
        for (int r = 0; r < W; ++r) {
            if (r == s) continue;
            const size_t rows = (size_t)runs[r].qb * runs[r].nprobe, o = (size_t)r * rows;
            cudaMemcpyAsync(runs[s].chosen + o, runs[r].chosen + o, rows * 4, cudaMemcpyDeviceToDevice, st);
            cudaMemcpyAsync(runs[s].cscore + o, runs[r].cscore + o, rows * 4, cudaMemcpyDeviceToDevice, st);
            cudaMemcpyAsync(runs[s].nch + (size_t)r * runs[r].qb, runs[r].nch + (size_t)r * runs[r].qb,
                            (size_t)runs[r].qb * 4, cudaMemcpyDeviceToDevice, st);
        }
    for (int s = 0; s < W; ++s) shards[s]->shard_seed(h, runs[s]);
    int rc = gather(false);
    if (rc != kOk) return rc;
    for (int s = 0; s < W; ++s) shards[s]->shard_after_seed(h, runs[s]);
    if (runs[0].rest && (rc = gather(false)) != kOk) return rc;
    for (int s = 0; s < W; ++s) shards[s]->shard_after_cut(h, runs[s]);
    if ((rc = gather(true)) != kOk) return rc;
    shards[0]->shard_merge(runs[0], d_ids, d_scores, d_nout);
    int kid = -1;
    cudaError_t le = dev::take_launch_error(&kid);
    if (le != cudaSuccess) {
        err = std::string("launch of ") + dev::kernel_name(kid) + " failed: " + cudaGetErrorString(le);
        return kCudaError;
    }
    return kOk;
}

}  // namespace maivs
