// Kernel declarations and the device image of a MAIVS index.
#pragma once

#include <cstdint>
#include <cuda_runtime.h>

#include <vector>

namespace maivs {
namespace dev {

// Read-only view of the device image, passed to kernels by value.
struct IndexView {
    int dim, dim_pad, nw, npos, M, ma;
    uint32_t maxk;  // 255 * npos, the largest FastScan table sum
    int seed_parts;  // blocks per query of the seed scan (about the seed cells' groups / 128)
    // routing tables
    const uint64_t* cent_bits;  // M x nw
    const uint8_t* cent_sq8;    // M x dim (null when the SQ8 re-order is off)
    const float* cent_f32;      // M x dim
    const float* csq_min;       // dim
    const float* csq_step;      // dim
    const uint8_t* live;        // M: cell has members
    const uint32_t* live_list;  // the live cells, ascending
    int n_live_cells;
    const float* r_bound;       // M
    const float* signs;         // 2 x dim_pad
    // scan layout: cell c's members are cell_slots[cell_moff[c] ..], its codes are the words
    // cell_codes[cell_woff[c] + j * ng + g] = nibble j of members 8g..8g+7 (nibble b = member 8g+b)
    const uint32_t* cell_moff;  // M + 1
    const uint32_t* cell_woff;  // M + 1
    const uint32_t* cell_codes;
    const uint32_t* cell_slots;
    const uint32_t* slot_cells;  // n_slots x ma
    // per member entry of a cell c: its other home when that home's id is below c, else kNoCell
    // (two homes at most; null otherwise). The exactly-once rule then needs one probed-bit test.
    const uint32_t* cell_lower;
    const uint32_t* tags;        // n_slots or null
    // Hamming scan (an index without compacted FastScan blocks): the members' flat sign codes,
    // nw words per slot, scanned by Hamming distance (index.rs:1693-1808); cell_codes is null
    int ham;
    const uint64_t* bits;
    // rerank store
    int rerank_mode;  // 0 f32, 1 per-dimension SQ8, 2 global int8
    const float* vecs_f32;
    const uint8_t* rr_u8;
    const float* sq_min;
    const float* sq_step;
    const uint64_t* ext_ids;
    // centroid tree (leaf level and up to kMaxTreeLevels levels, coarsest first)
    int tree_depth;
    const uint64_t* tree_codes[8];
    const uint32_t* tree_child_start[8];
    const uint32_t* tree_child_len[8];
    int tree_n[8];
    const uint64_t* leaf_codes;
    const uint32_t* leaf_ids;
    int n_leaf;
};

// Per-kernel device clock. When a clock is installed on the calling thread, every launcher
// brackets its kernels with CUDA events on the launch stream; the owner reads the elapsed times
// after synchronising. Every launch is counted whether or not a clock is installed.
enum KernelId : int {
    kKEncode = 0, kKRouteFlat, kKRouteTree, kKRescore, kKSeed, kKInvCount, kKInvScan, kKInvScatter,
    kKScanCm, kKFinalCm, kKPqPrep, kKPqScan, kKPqFold, kKRerank, kKTopk, kKRerankItems, kKSeedFinish, kKLocalList, kKMergeTopk,
    kKScanMma, kKSeedScan, kKAllGather, kKSegMerge, kKRescoreDots, kKProbeSelect, kNumKernels
};
const char* kernel_name(int id);
// Brackets a step that is not one of this library's kernels (an NCCL collective) on the thread's
// clock, when one is installed; it is timed but not counted as a launch.
void clock_begin(int id, cudaStream_t st);
void clock_end(int id, cudaStream_t st);
struct KernelClock {
    struct Mark {
        int id;
        cudaEvent_t a, b;
    };
    std::vector<Mark> pending;
    std::vector<cudaEvent_t> pool;
    double ms[kNumKernels] = {0};
    // time during which at least one launch of the kernel ran (launches on several streams may
    // overlap; ms counts overlapping time once per launch, busy once)
    double busy[kNumKernels] = {0};
    unsigned long long launches[kNumKernels] = {0};
    int only = -1;  // >= 0: time only this kernel
    bool wants(int id) const { return only < 0 || only == id; }
    ~KernelClock();
    cudaEvent_t take();
    void begin(int id, cudaStream_t st);
    void end(cudaStream_t st);
    // Accumulates the elapsed times of every pending mark (their events must have completed).
    void collect();
};
void set_thread_clock(KernelClock* c);
// First kernel-launch error on this thread since the last call (and the kernel it came from).
cudaError_t take_launch_error(int* kernel);
unsigned long long total_launches();

constexpr int kMaxTreeLevels = 8;
constexpr int kSeedCells = 8;  // index.rs:2019 SEED_CELLS
constexpr int kSortCap = 16384;  // largest shortlist sorted in shared memory
constexpr uint64_t kInvalidEntry = ~0ull;

// Per-query encodings (src/quantize.rs rotate/pack/FsQuery, index.rs:1177-1187, :1320-1327).
struct QueryEnc {
    uint64_t* qbits;  // nq x nw
    uint8_t* lut;     // nq x npos*16
    float* fs_delta;  // nq
    float* fs_bias;   // nq
    float* cqs;       // nq x dim  (centroid SQ8 pre-scale)
    float* cqbase;    // nq
    float* rqs;       // nq x dim  (rerank SQ8 pre-scale)
    float* rbase;     // nq
};

void launch_encode(const IndexView& ix, const float* Q, int nq, const QueryEnc& e, bool want_cqs, bool want_rqs,
                   cudaStream_t st);
// Flat two-stage shortlist: live cells with Hamming <= the want_c-th smallest, ties kept, in cell
// order (index.rs:1903-1927 route_batch, :1241-1259 route_query).
// `hs` is nq x M scratch for the Hamming distances.
void launch_route_flat(const IndexView& ix, const QueryEnc& e, int nq, int want_c, uint16_t* hs, uint32_t* sl,
                       uint32_t* sl_n, int sl_cap, cudaStream_t st);
// Every live cell, in cell order (index.rs:1274-1282).
void launch_route_all(const IndexView& ix, int nq, uint32_t* sl, uint32_t* sl_n, int sl_cap, cudaStream_t st);
// Centroid-tree beam descent (tree.rs:574-628); `beams` per level, `want` leaves.
void launch_route_tree(const IndexView& ix, const QueryEnc& e, int nq, const int* beams, int want, uint32_t* scratch,
                       int scratch_cap, uint32_t* sl, uint32_t* sl_n, int sl_cap, cudaStream_t st);
// SQ8 (or f32) re-order of the shortlist, top-nprobe by score desc (ties: lower cell id first),
// nucleus cut (index.rs:1931-1977, :1283-1301).
// all_live: every query's shortlist is the live-cell list (scored by a tiled product).
void launch_rescore_select(const IndexView& ix, const QueryEnc& e, const float* Q, int nq, const uint32_t* sl,
                           const uint32_t* sl_n, int sl_cap, int nprobe, float tc, float beta, bool use_sq8,
                           uint32_t* chosen, float* cscore, uint32_t* nch, uint32_t* err, float* rs_scores,
                           uint32_t* rs_items, int expect_n, bool all_live, cudaStream_t st);

// Cell-major batch (index.rs:1999-2311).
struct CellMajorBufs {
    uint64_t* probed;     // nq x mwords (polysemy only)
    int mwords;
    uint64_t* seed_buf;   // nq x seed_cap
    int seed_cap;
    uint16_t* seed_d;     // nq x seed_dcap: FastScan distances of the seed cells' member groups
    int seed_dcap;        // a multiple of 8, >= 8 x the seed cells' groups
    uint32_t* seed_n;     // nq
    uint32_t* tau;        // nq
    uint32_t* rest_hi;    // nq (rest range is [min(8, nch), rest_hi))
    uint32_t* cell_cnt;   // M + 1 (counts, then start offsets)
    uint32_t* cell_fill;  // M
    uint32_t* qof;        // nq x nprobe
    uint64_t* rest_buf;   // nq x rest_cap
    int rest_cap;
    uint32_t* rest_n;     // nq
    uint32_t* cand;       // nq x cand_cap slots
    int cand_cap;
    uint32_t* cand_n;     // nq
    uint32_t* overflow;   // 1: queries whose buffers overflowed
    uint32_t* gtau;       // nq: the rest scan's falling cut-off (starts at tau)
    uint32_t* lad;        // nq x kLadStride: rungs below tau, seed shortfalls, rest counts
    uint32_t* work;       // 1: the persistent tensor-core scan's cell counter
};
// Rungs of the falling cut-off per query (see k_seed): 8 rungs at about (3/4)^(l+1) of the seed
// survivors' rank, then as many "needed" counts and as many running counters.
constexpr int kLad = 8;
constexpr int kLadStride = 3 * kLad;
void launch_cellmajor(const IndexView& ix, const QueryEnc& e, int nq, const uint32_t* chosen, const float* cscore,
                      const uint32_t* nch, int nprobe, int target, bool adaptive, float at_margin,
                      const CellMajorBufs& b, cudaStream_t st);

// Cell-range shards run the cell-major join in pieces with all-gathers between them:
// launch_seed (xlist set: publish the shard's seed distances) -> all-gather -> launch_seed_finish
// -> launch_rest_scan -> launch_local_list -> all-gather -> launch_final (W > 0) -> rerank ->
// all-gather of the best-k lists -> launch_merge_topk. Block sizes of one rank's share of the
// gathered buffers: shard_list_block_bytes (nq counts + nq x xl distances) and
// shard_topk_block_bytes (nq x k ids, nq x k scores, nq counts).
void launch_seed(const IndexView& ix, const QueryEnc& e, int nq, const uint32_t* chosen, const float* cscore,
                 const uint32_t* nch, int nprobe, int target, bool adaptive, float at_margin, const CellMajorBufs& b,
                 uint16_t* xlist, uint32_t* xcnt, int xl, cudaStream_t st);
void launch_seed_finish(const IndexView& ix, const QueryEnc& e, int nq, const uint32_t* chosen, const float* cscore,
                        const uint32_t* nch, int nprobe, int target, bool adaptive, float at_margin,
                        const CellMajorBufs& b, const uint8_t* xall, size_t rank_bytes, int W, int xl,
                        cudaStream_t st);
void launch_rest_scan(const IndexView& ix, const QueryEnc& e, int nq, const uint32_t* chosen, const uint32_t* nch,
                      int nprobe, const CellMajorBufs& b, cudaStream_t st);
void launch_local_list(const CellMajorBufs& b, int nq, uint16_t* xlist, uint32_t* xcnt, int xl, cudaStream_t st);
void launch_final(const CellMajorBufs& b, int nq, int target, const uint8_t* xall, size_t rank_bytes, int W, int xl,
                  cudaStream_t st);
void launch_merge_topk(const uint8_t* tall, size_t rank_bytes, int W, int nq, int k, uint64_t* ids, float* scores,
                       uint32_t* out_n, cudaStream_t st);
size_t shard_list_block_bytes(int nq, int xl);
size_t shard_topk_block_bytes(int nq, int k);

// Per-query path (index.rs:1381-1864, FastScan branch).
struct PerQueryBufs {
    uint32_t* crank;     // nq x M probe rank or kNoCell
    uint32_t* seg_off;   // nq x (nprobe + 1)
    uint64_t* ent;       // nq x ent_cap entries (d << 32 | slot) or kInvalidEntry
    int ent_cap;
    uint32_t* cand;      // nq x cand_cap
    int cand_cap;
    uint32_t* cand_n;    // nq
    uint32_t* overflow;
};
void launch_perquery(const IndexView& ix, const QueryEnc& e, int nq, const uint32_t* chosen, const float* cscore,
                     const uint32_t* nch, int nprobe, int want0, bool adaptive, float at_margin, bool filtering,
                     uint32_t flo, uint32_t fhi, const PerQueryBufs& b, cudaStream_t st);

// Exact rerank + top-k (index.rs:1309-1378); writes k ids/scores per query, padded.
// `score_scratch` (nq x cand_cap floats) and `item_scratch` (nq + 1 words) enable the flattened
// register gather + separate top-k, used whenever rows are 16-byte multiples; other rows take a
// one-CTA-per-query kernel.
void launch_rerank(const IndexView& ix, const float* Q, const QueryEnc& e, int nq, const uint32_t* cand,
                   const uint32_t* cand_n, int cand_cap, int k, uint64_t* ids, float* scores, uint32_t* out_n,
                   float* score_scratch, uint32_t* item_scratch, uint32_t* err, cudaStream_t st);

// ConcurrentIndex::finish (concurrent.rs:83-110) of every query over L per-segment result lists:
// list l of query q is ids/scores[(l * nq + q) * want ..] with nout[l * nq + q] entries. Drops the
// ids found in `tomb` (ascending, ntomb entries), keeps one entry per id (its best score), and
// writes the best k by score (exact ties by ascending id) to out_ids/out_scores (nq x k, padded
// with UINT64_MAX / -inf). `scratch` holds L * want * 16 bytes per query.
void launch_segment_merge(const uint64_t* ids, const float* scores, const uint32_t* nout, int L, int nq, int want,
                          const uint64_t* tomb, int ntomb, int k, void* scratch, uint64_t* out_ids, float* out_scores,
                          cudaStream_t st);

}  // namespace dev
}  // namespace maivs
