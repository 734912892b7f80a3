// Host-resident MAIVS index: configuration, arena, cells and the derived routing state.
//
// Mirrors the fields of the reference's FlatCellIndex (src/index.rs:430-566) that the query hot
// path reads. The build (train_centroids, add_batch, compact) runs on the host cores; the search
// runs on the GPU from a device image of this state (see device_index.h).
#pragma once

#include <cstddef>
#include <cstdint>
#include <memory>
#include <string>
#include <unordered_map>
#include <vector>

namespace maivs {

// One cell: member slots plus a running exact centroid (index.rs:361-395).
struct Cell {
    std::vector<uint32_t> members;
    std::vector<float> sum;
    std::vector<float> centroid;
    float r_bound = 0.0f;  // p99 member angle (index.rs:817-861)
    float r_max = 0.0f;
};

// One level of the centroid tree (tree.rs:74-83).
struct TreeLevel {
    size_t n = 0;
    std::vector<float> cents;
    std::vector<uint64_t> codes;
    std::vector<uint32_t> child_start, child_len, child_idx;
};

// Dynamic-depth tree over live cell centroids (tree.rs:85-97).
struct CentroidTree {
    size_t dim = 0, nw = 0, fanout = 0;
    float beam_frac = 0.5f;
    std::vector<TreeLevel> levels;     // coarsest first
    std::vector<uint64_t> leaf_codes;  // by leaf position
    std::vector<uint32_t> leaf_ids;    // leaf position -> cell id
    size_t n_leaf = 0;

    std::vector<size_t> beams(size_t want) const;
    // Beam descent; returns up to `want` cell ids, best first by Hamming, ties in encounter
    // order (tree.rs:574-628).
    void search(const uint64_t* q_bits, size_t want, std::vector<uint32_t>& out) const;
};

constexpr size_t kTreeTopMax = 256;        // tree.rs:41
constexpr size_t kTreeMinBeam = 32;        // tree.rs:45
constexpr float kTreeDefaultBeamFrac = 0.5f;  // tree.rs:66
constexpr size_t kTreeMinCells = 2048;     // tree.rs:70
constexpr size_t kTreeDefaultFanout = 64;  // tree.rs:37
constexpr size_t kAssignCandidates = 64;   // index.rs:401
constexpr size_t kGraphMinCells = 65536;   // graph.rs:33

std::unique_ptr<CentroidTree> build_centroid_tree(const float* cell_cents, const uint32_t* cell_ids, size_t m,
                                                  size_t dim, const float* signs, size_t dim_pad, size_t nw,
                                                  size_t fanout, float beam_frac, int device = -1,
                                                  size_t* gpu_failures = nullptr);

// Spherical Lloyd k-means (tree.rs:179-248); returns (assign, centroids). With device >= 0 the
// assignment and the sums run on that GPU (csrc/cuda/build.cu, same results); a GPU failure is
// counted in *gpu_failures (when given) and the host computes the step instead.
void kmeans_spherical(const float* x, size_t n, size_t dim, size_t k, size_t iters, uint64_t seed,
                      std::vector<uint32_t>& assign, std::vector<float>& cents, int device = -1,
                      size_t* gpu_failures = nullptr);
// Two-level k-means (tree.rs:257-348).
std::vector<float> hierarchical_kmeans(const float* x, size_t n, size_t dim, size_t k, uint64_t seed,
                                       int device = -1, size_t* gpu_failures = nullptr);

// Keep the `keep` smallest (h, id) pairs, ties at the cut-off in encounter order (tree.rs:120-159).
void keep_smallest(std::vector<std::pair<uint32_t, uint32_t>>& v, size_t keep, size_t bits);

struct HostIndex {
    // ---- configuration (index.rs:2672-2755 defaults) ----
    size_t dim = 0, dim_pad = 0, nw = 0;
    uint64_t seed = 0x5EED;
    size_t rerank_factor = 4;
    std::vector<float> signs;  // kRounds x dim_pad

    bool two_stage = false;
    size_t shortlist_mult = 4;
    bool centroid_sq8 = true;
    bool tree_route = true;
    size_t tree_min_cells = kTreeMinCells;
    size_t tree_fanout = kTreeDefaultFanout;
    float tree_beam_frac = kTreeDefaultBeamFrac;
    bool graph_route = true;
    size_t graph_min_cells = kGraphMinCells;
    size_t max_assign = 1;
    float spill_margin = 0.0f;
    float spill_lambda = 0.0f;
    bool fastscan = false;
    bool per_dim_sq = false;
    bool i8_rerank = false;
    bool keep_f32 = true;
    bool adaptive = false;
    float at_margin = 0.02f;
    float quant_scale = 0.0f;
    // Cell-major batches need at least this many queries (the reference uses 2 x its rayon pool,
    // index.rs:3343-3348; 32 = 2 x the 16 threads of its published runs).
    size_t cm_min_batch = 32;

    // ---- arena (slot-indexed) ----
    std::vector<uint64_t> bits;     // nw words per slot
    std::vector<int8_t> scan_i8;    // dim bytes per slot (SQ8 codes or global int8)
    std::vector<float> vecs_f32;    // dim floats per slot
    std::vector<uint64_t> ext_ids;
    std::vector<uint32_t> slot_cell;   // primary cell
    std::vector<uint32_t> slot_cells;  // max_assign homes per slot, UINT32_MAX = unused
    std::vector<uint32_t> free_slots;
    std::unordered_map<uint64_t, uint32_t> id_to_slot;
    std::vector<float> sq_min, sq_step;
    std::vector<uint32_t> tags;
    bool has_filter = false;
    uint32_t filter_lo = 0, filter_hi = 0xFFFFFFFFu;
    size_t n_live = 0;

    // ---- cells and derived routing state ----
    std::vector<Cell> cells;
    std::vector<uint64_t> cent_bits;
    std::vector<uint8_t> cent_sq8;
    std::vector<float> csq_min, csq_step;
    std::unique_ptr<CentroidTree> tree;
    size_t tree_cells = 0;

    // ---- compacted layout (index.rs:929-1112) ----
    bool compacted = false;
    std::vector<uint32_t> prim_len, rep_off;
    std::vector<uint8_t> fs_codes;
    std::vector<uint32_t> fs_off;

    // Bumped on every mutation; the device image remembers the version it was built from.
    uint64_t version = 0;

    // GPU that runs the heavy parts of the build (k-means, placement), or -1 for the host cores.
    // The results are the same either way; build steps the GPU could not run are counted here and
    // were computed on the host.
    int build_device = -1;
    size_t build_gpu_failures = 0;
    std::string build_gpu_error;

    // ---- API mirrored from the reference's #[pymethods] ----
    // Returns an empty string on success, otherwise the error message.
    std::string init(size_t dim, const std::string& scan_mode, size_t rerank_factor, uint64_t seed, size_t code_bits);
    std::string train_centroids(const float* data, size_t n, size_t n_cells, size_t sample, uint64_t seed);
    std::string set_centroids(const float* cents, size_t m);
    std::string add_batch(const uint64_t* ids, const float* data, size_t n);
    bool remove(uint64_t id);
    void compact();
    void set_tree_route(bool on, size_t min_cells, size_t fanout, float beam_frac);
    void set_two_stage(bool on, size_t mult);
    void set_centroid_sq8(bool on);
    void set_per_dim_sq(bool on);
    void set_i8_rerank(bool on);
    void set_orthogonal_polysemy(size_t homes, float lam);
    void set_replication(size_t max_assign, float spill_margin);
    void set_fastscan(bool on);
    std::string set_tags(const uint64_t* ids, const uint32_t* tags, size_t n);
    // fork_empty (index.rs:2330-2400): `f` becomes an empty index with this one's configuration,
    // rotation, quantisation parameters and centroids; FastScan off, not compacted, no tags.
    void fork_empty(HostIndex& f) const;

    size_t live_cell_count() const;
    void refresh_derived();
    void rebuild_centroid_tree();
    void maybe_rebuild_centroid_tree();
    void rebuild_centroid_codes();
    void rebuild_centroid_sq8();
    void recompute_radii();

   private:
    std::vector<uint32_t> assign_cells(const float* v) const;
    std::vector<uint32_t> assign_cells_routed(const float* v, std::vector<float>& rot, std::vector<uint64_t>& qb,
                                              std::vector<uint32_t>& out) const;
    std::vector<uint32_t> pick_orthogonal(std::vector<std::pair<uint32_t, float>>& scored) const;
    void append_parallel(const uint64_t* ids, const float* data, size_t n, const std::vector<std::vector<uint32_t>>& asg,
                         const uint64_t* codes = nullptr);
    void encode_i8(const float* v, int8_t* out) const;
};

// GPU build steps (csrc/cuda/build.cu); each returns an empty string on success.
std::string gpu_kmeans_spherical(int device, const float* x, size_t n, size_t dim, size_t k, size_t iters,
                                 uint64_t seed, std::vector<uint32_t>& assign, std::vector<float>& cents);
// Homes of n vectors through the centroid tree (assign_cells_routed), and their codes (n x nw).
// Vectors left without homes (none with the reference's shortlist) are for the caller to place.
std::string gpu_place(int device, const HostIndex& h, const float* data, size_t n,
                      std::vector<std::vector<uint32_t>>& asg, uint64_t* codes_out);

// Reference on-disk format "MAIVS2\0\1" (src/persist.rs); empty string on success.
std::string save_index(const HostIndex& h, const std::string& path);
std::string load_index(const std::string& path, HostIndex& h);

}  // namespace maivs
