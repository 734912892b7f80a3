// Device image of a host index plus the search pipelines that run on it.
#pragma once

#include <cuda_runtime.h>

#include <cstdint>
#include <memory>
#include <mutex>
#include <string>
#include <vector>

#include "../host/index_host.h"
#include "kernels.cuh"

namespace maivs {

// Status codes of the C ABI (mirrored in include/maivs_b200.h).
enum Status : int {
    kOk = 0,
    kBadShape = 1,
    kBadArg = 2,
    kBadState = 3,
    kOom = 4,
    kCudaError = 5,
    kOverflow = 6,
    kUnsupported = 7,
    kNotFound = 8,
    kNoDevice = 9,
};

struct SearchArgs {
    int nq = 0;
    int k = 0;
    int nprobe = 16;
    float tc = 0.95f;
    float beta = 8.0f;
    bool cell_major = true;
    // -1: the batch chooses the cell-major join or the per-query path (index.rs:3343-3348); 0 / 1:
    // a part of a larger batch keeps that batch's choice (per-query / cell-major)
    int path = -1;
};

// Per-phase device times of the last search, in milliseconds (the reference's profile phases
// q.route / q.scan / q.rerank, src/prof.rs:35-42).
struct PhaseTimes {
    float encode = 0, route = 0, scan = 0, rerank = 0;
};

// Intermediate buffers of a search stopped after one stage (parity tests and diagnostics):
// stage 0 = query codes and FastScan tables, 1 = probe lists, 2 = candidate slots sent to rerank.
struct DebugOut {
    int stage = 0;
    int nprobe = 0, cand_cap = 0;
    std::vector<uint64_t> qbits;
    std::vector<uint8_t> lut;
    std::vector<float> delta, bias, cscore;
    std::vector<uint32_t> chosen, nch, cand, cand_n;
    std::vector<uint32_t> seed_n, tau, rest_hi, rest_n;  // cell-major only (stage 2)
};

// All-gather used by the cell-range sharded search: `bytes` from every rank's `send` land in
// `recv`, rank r's block at recv + r * bytes, ordered on stream `st`.
class Exchange {
   public:
    virtual ~Exchange() = default;
    virtual int all_gather(const void* send, void* recv, size_t bytes, cudaStream_t st, std::string& err) = 0;
};

// NCCL over NVLink / NVSwitch (libnccl.so.2 is loaded on first use). `id` is the 128-byte
// ncclUniqueId that rank 0 made with nccl_unique_id and the host shared with every rank.
int nccl_unique_id(uint8_t* id, std::string& err);
std::unique_ptr<Exchange> nccl_exchange(const uint8_t* id, int rank, int world, int device, std::string& err);

// Cells [lo, hi) of rank `rank` of `world`: contiguous ranges balanced by member entries.
void shard_range(const HostIndex& h, int rank, int world, uint32_t* lo, uint32_t* hi);

class DeviceIndex;
// The sharded protocol with every shard in this process on one device, exchanging through device
// copies: results equal the NCCL path's, which equal the unsharded cell-major join's.
int search_emulated_shards(const HostIndex& h, std::vector<std::unique_ptr<DeviceIndex>>& shards, const float* dQ,
                           const SearchArgs& a, uint64_t* d_ids, float* d_scores, uint32_t* d_nout, cudaStream_t st,
                           std::string& err);

class DeviceIndex {
   public:
    // When set, the next search stops after dbg->stage and fills *dbg (synchronous).
    DebugOut* dbg = nullptr;

    ~DeviceIndex();
    // Builds the device image of a host index; returns an error message. A compacted FastScan index
    // gets the FastScan layout (both search paths); any other index its flat codes (per-query).
    // With a cell range, only cells [c_lo, c_hi) keep their members (a cell-range shard); the
    // routing tables and the rerank rows are always whole.
    std::string upload(const HostIndex& h, int device, uint32_t c_lo = 0, uint32_t c_hi = 0xFFFFFFFFu);
    // Makes this image rank `rank` of a sharded search over `x` (not owned; null: unsharded).
    void set_shard(Exchange* x, int rank, int world) {
        exch_ = x;
        shard_rank_ = rank;
        shard_world_ = x ? world : 1;
    }
    bool sharded() const { return exch_ != nullptr; }
    // scanned by Hamming distance over flat codes (no compacted FastScan blocks): per-query only
    bool hamming() const { return view_.ham != 0; }
    uint64_t version() const { return version_; }
    int device() const { return device_; }
    cudaStream_t stream() const { return stream_; }

    // Search with device-resident queries and outputs, enqueued on `st`. Chooses the cell-major
    // join or the per-query path like the reference's search_batch (index.rs:3343-3348).
    // Returns a Status; `err` receives a message on failure.
    // With clear_flags false the overflow/error counters are left as they are (the caller cleared
    // them for several searches in flight together).
    int search_device(const HostIndex& h, const float* dQ, const SearchArgs& a, uint64_t* d_ids, float* d_scores,
                      uint32_t* d_nout, cudaStream_t st, std::string& err, bool clear_flags = true);
    // Per-query search of at most 64 device-resident queries whose scratch is a fixed 32 MiB
    // device array defined in static_search.cu (allocates nothing; calls share the array, so
    // overlapping calls race). Returns kBadArg when the search needs more scratch than that.
    int search_static(const HostIndex& h, const float* dQ, const SearchArgs& a, uint64_t* d_ids, float* d_scores,
                      cudaStream_t st, std::string& err);
    // Host buffers: copies in, searches, copies out, synchronises, and retries with larger
    // candidate buffers if any query overflowed them.
    int search_host(const HostIndex& h, const float* Q, const SearchArgs& a, uint64_t* ids, float* scores,
                    uint32_t* nout, std::string& err);

    // Overflow/error counters of the last device search (synchronises `st`). On a sharded image
    // this is collective: the counters are summed over all ranks, so every rank decides alike.
    uint32_t read_flags(cudaStream_t st);
    int global_flags(cudaStream_t st, uint32_t out[4]);
    bool use_cell_major(const HostIndex& h, const SearchArgs& a) const;
    void set_timing(bool on) { timing_ = on; }
    // Synchronises on the last timed search and returns its phase times.
    PhaseTimes collect_phases();
    size_t device_bytes() const { return bytes_; }

    int grow_factor = 1;  // multiplies the candidate-buffer capacities after an overflow

    // Per-kernel device times (only while enabled) and the work counters of the last search,
    // read from its workspace after synchronising: name -> value.
    void enable_kernel_clock(bool on);
    dev::KernelClock* kernel_clock() { return clock_.get(); }
    std::vector<std::pair<std::string, double>> last_stats();

    // Phases of the cell-range sharded join (one shard's side); search_sharded and
    // search_emulated_shards put the all-gathers between them.
    struct ShardRun {
        int nq = 0, k = 0, nprobe = 0, target = 0, xl = 0, W = 0, rank = 0, qb = 0;  // qb: queries routed per rank
        bool rest = false;
        size_t lb = 0, tb = 0;
        const float* dQ = nullptr;
        cudaStream_t st = nullptr;
        dev::QueryEnc e{};
        dev::CellMajorBufs b{};
        uint32_t *chosen = nullptr, *nch = nullptr, *ritem = nullptr;
        float *cscore = nullptr, *rsc = nullptr;
        uint8_t *xsend = nullptr, *xrecv = nullptr, *tsend = nullptr, *trecv = nullptr;
    };
    // encode every query, route this rank's block of qb queries (rows rank*qb.. of chosen/cscore/nch)
    int shard_begin(const HostIndex& h, const float* dQ, const SearchArgs& a, int W, int rank, cudaStream_t st,
                    ShardRun& r, std::string& err);
    // after the probe lists are all-gathered: scan this shard's seed probes, publish its distances
    void shard_seed(const HostIndex& h, ShardRun& r);
    void shard_after_seed(const HostIndex& h, ShardRun& r);
    void shard_after_cut(const HostIndex& h, ShardRun& r);
    void shard_merge(ShardRun& r, uint64_t* d_ids, float* d_scores, uint32_t* d_nout);

   private:
    int search_sharded(const HostIndex& h, const float* dQ, const SearchArgs& a, uint64_t* d_ids, float* d_scores,
                       uint32_t* d_nout, cudaStream_t st, std::string& err);
    // A batch of kSplitQueries or more whose queries' work is independent of one another (the
    // cell-major join probing only the seed cells) is searched as two halves, one on `st` and one
    // on stream2_, with a workspace each: the halves' short dependent kernels overlap each other.
    // Not for a sharded image (its ranks take the same collective steps), a debug stop or phase
    // timing (both describe one search); the kernel clock times each half's launches.
    // Every query's result depends only on that query and on the path the whole batch chose, which
    // both halves keep, so the results are those of one search over the batch.
    bool split_halves(const HostIndex& h, const SearchArgs& a) const;
    // With hQ (pinned host queries), each half is first copied into dQ on its own stream, so the
    // second half's copy overlaps the first half's search.
    int search_halves(const HostIndex& h, const float* dQ, const float* hQ, const SearchArgs& a, uint64_t* d_ids,
                      float* d_scores, uint32_t* d_nout, cudaStream_t st, std::string& err);
    Exchange* exch_ = nullptr;
    uint32_t* d_flags_all_ = nullptr;  // world x 4 counters gathered by global_flags
    int shard_rank_ = 0, shard_world_ = 1;
    void* alloc(size_t bytes);
    template <typename T>
    T* upload_vec(const std::vector<T>& v);
    int ensure_ws(size_t bytes, std::string& err);
    int run_cellmajor(const HostIndex& h, const float* dQ, const SearchArgs& a, uint64_t* d_ids, float* d_scores,
                      uint32_t* d_nout, cudaStream_t st, std::string& err);
    int debug_encode(const dev::QueryEnc& e, int nq, cudaStream_t st);
    int debug_route(const uint32_t* chosen, const float* cscore, const uint32_t* nch, int nq, int nprobe,
                    cudaStream_t st);
    int debug_cands(const uint32_t* cand, const uint32_t* cand_n, int nq, int cap, cudaStream_t st);
    int run_perquery(const HostIndex& h, const float* dQ, const SearchArgs& a, uint64_t* d_ids, float* d_scores,
                     uint32_t* d_nout, cudaStream_t st, std::string& err);
    int route(const HostIndex& h, const dev::QueryEnc& e, const float* dQ, int nq, int nprobe, float tc, float beta,
              bool batch_router, uint16_t* hs, uint32_t* sl, uint32_t* sl_n, uint32_t* tree_scratch,
              float* rs_scores, uint32_t* rs_items, uint32_t* chosen,
              float* cscore, uint32_t* nch, cudaStream_t st, std::string& err);

    int device_ = -1;
    cudaStream_t stream_ = nullptr;
    uint64_t version_ = 0;
    std::vector<void*> allocs_;
    size_t bytes_ = 0;
    dev::IndexView view_{};
    size_t n_live_ = 0, n_leaf_ = 0, max_members_ = 0, tree_cap_ = 0;
    bool use_sq8_ = false;
    uint32_t* d_flags_ = nullptr;  // [0] overflow, [1] routing errors
    // search workspaces: ws_[ws_sel_] serves the search being enqueued (two for a split batch)
    void* ws_[2] = {nullptr, nullptr};
    size_t ws_bytes_[2] = {0, 0};
    int ws_sel_ = 0;
    void* ws() const { return ws_[ws_sel_]; }
    size_t ws_bytes() const { return ws_bytes_[ws_sel_]; }
    // recorded after each search that used ws_[i]; a later search on another stream waits on it,
    // so searches sharing a workspace never overlap on the device
    cudaEvent_t ws_ev_[2] = {nullptr, nullptr};
    bool ws_ev_live_[2] = {false, false};
    cudaStream_t stream2_ = nullptr;  // the second half of a split batch
    cudaEvent_t split_ev_[2] = {nullptr, nullptr};
    // pinned staging for the host-buffer API
    void* pin_ = nullptr;
    size_t pin_bytes_ = 0;
    void* io_ = nullptr;  // device queries and results of the host-buffer API
    size_t io_bytes_ = 0;
    bool timing_ = false;
    std::unique_ptr<dev::KernelClock> clock_;
    std::vector<uint32_t> moff_;  // host copy of the member offsets
    struct LastCall {
        bool valid = false, cell_major = false;
        int nq = 0, nprobe = 0, target = 0;
        const uint32_t *nch = nullptr, *chosen = nullptr, *sl_n = nullptr, *cell_cnt = nullptr,
                       *cand_n = nullptr, *seed_n = nullptr, *rest_n = nullptr, *rest_hi = nullptr;
        cudaStream_t st = nullptr;
    } last_;
    // a split batch's halves (last_split_): last_stats describes both together
    LastCall last_half_[2];
    bool last_split_ = false;
    PhaseTimes phases_;
    cudaEvent_t ev_[5] = {nullptr, nullptr, nullptr, nullptr, nullptr};
};

}  // namespace maivs
