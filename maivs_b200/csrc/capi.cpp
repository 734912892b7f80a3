// C ABI of the B200 MAIVS engine (declared in include/maivs_b200.h).
#include <cuda_runtime.h>
#include <omp.h>

#include <algorithm>
#include <atomic>
#include <cmath>
#include <cstring>
#include <map>
#include <memory>
#include <mutex>
#include <string>
#include <vector>

#include "../../include/maivs_b200.h"
#include "cuda/engine.h"
#include "host/index_host.h"

using maivs::DeviceIndex;
using maivs::HostIndex;

#include "handle.h"

namespace {

std::atomic<bool> g_prof_on{false};
std::mutex g_prof_mu;
// Phase names of the reference profiler (src/prof.rs:35-42); the GPU engine fills the query
// phases it has: q.r_rotate (query encoding), q.route, q.scan, q.rerank and q.count.
const char* kPhaseNames[] = {"q.r_rotate", "q.r_tree", "q.r_rescore", "q.route",     "q.select",
                             "q.bounds",   "q.scan",   "q.topk",      "q.rerank",    "q.count",
                             "b.train",    "b.sqfit",  "b.assign",    "b.encode_place", "b.centroids",
                             "b.radii",    "b.codes",  "b.graph_tree", "b.compact"};
constexpr size_t kNumPhases = sizeof(kPhaseNames) / sizeof(kPhaseNames[0]);
double g_prof[kNumPhases] = {0};

int fail(maivs_index* ix, int status, const std::string& msg) {
    if (ix) ix->err = msg;
    return status;
}

int check(maivs_index* ix, const std::string& msg, int status = MAIVS_BAD_ARG) {
    if (msg.empty()) return MAIVS_OK;
    return fail(ix, status, msg);
}

// Make the device image current; returns a status.
int ensure_device(maivs_index* ix) {
    int n = 0;
    if (cudaGetDeviceCount(&n) != cudaSuccess || n == 0)
        return fail(ix, MAIVS_NO_DEVICE, "no CUDA device is visible; the MAIVS GPU search has no CPU fallback");
    if (ix->d && ix->d->version() == ix->h.version && ix->d->device() == ix->device) return MAIVS_OK;
    auto d = std::make_unique<DeviceIndex>();
    if (ix->d) d->grow_factor = ix->d->grow_factor;  // candidate buffers stay as large as they grew
    uint32_t lo = 0, hi = 0xFFFFFFFFu;
    if (ix->exch) maivs::shard_range(ix->h, ix->shard_rank, ix->shard_world, &lo, &hi);
    std::string e = d->upload(ix->h, ix->device, lo, hi);
    if (!e.empty()) return fail(ix, MAIVS_BAD_STATE, e);
    d->set_shard(ix->exch.get(), ix->shard_rank, ix->shard_world);
    d->set_timing(g_prof_on.load());
    ix->d = std::move(d);
    return MAIVS_OK;
}

void record_phases(maivs_index* ix, int nq) {
    if (!g_prof_on.load() || !ix->d) return;
    maivs::PhaseTimes p = ix->d->collect_phases();
    std::lock_guard<std::mutex> lk(g_prof_mu);
    g_prof[0] += p.encode;  // q.r_rotate: rotation, codes, FastScan tables
    g_prof[3] += p.route;   // q.route
    g_prof[6] += p.scan;    // q.scan (seed, prune, inversion, scan, exact cut)
    g_prof[8] += p.rerank;  // q.rerank
    g_prof[9] += nq;        // q.count
}

template <typename T>
void put(maivs_index* ix, const std::string& name, const T* p, size_t n) {
    auto& v = ix->arrays[name];
    v.resize(n * sizeof(T));
    if (n) std::memcpy(v.data(), p, n * sizeof(T));
}

// Query-time switches (rerank factor, adaptive margin, filter, ...) change no index version, so
// the configuration array is rebuilt on every request.
void put_config(maivs_index* ix) {
    HostIndex& h = ix->h;
    double cfg[] = {(double)h.dim,          (double)h.dim_pad,       (double)h.nw,
                    (double)h.rerank_factor, (double)h.two_stage,     (double)h.shortlist_mult,
                    (double)h.centroid_sq8,  (double)(h.tree != nullptr), (double)h.max_assign,
                    (double)h.fastscan,      (double)h.per_dim_sq,    (double)h.i8_rerank,
                    (double)h.keep_f32,      (double)h.adaptive,      (double)h.at_margin,
                    (double)h.quant_scale,   (double)h.compacted,     (double)h.n_live,
                    (double)h.cm_min_batch,  (double)h.has_filter,    (double)h.filter_lo,
                    (double)h.filter_hi,     (double)(h.tree ? h.tree->beam_frac : 0.0f),
                    (double)(h.tree ? h.tree->n_leaf : 0), (double)h.graph_route, (double)h.graph_min_cells};
    put(ix, "config", cfg, sizeof(cfg) / sizeof(double));
}

void build_arrays(maivs_index* ix) {
    put_config(ix);
    if (ix->arrays_version == ix->h.version) return;
    ix->arrays.clear();
    put_config(ix);
    HostIndex& h = ix->h;
    put(ix, "vecs_f32", h.vecs_f32.data(), h.vecs_f32.size());
    put(ix, "scan_i8", h.scan_i8.data(), h.scan_i8.size());
    put(ix, "bits", h.bits.data(), h.bits.size());
    put(ix, "ext_ids", h.ext_ids.data(), h.ext_ids.size());
    put(ix, "slot_cell", h.slot_cell.data(), h.slot_cell.size());
    put(ix, "slot_cells", h.slot_cells.data(), h.slot_cells.size());
    std::vector<uint32_t> mem, moff{0};
    std::vector<float> cents, rb;
    for (auto& c : h.cells) {
        mem.insert(mem.end(), c.members.begin(), c.members.end());
        moff.push_back((uint32_t)mem.size());
        cents.insert(cents.end(), c.centroid.begin(), c.centroid.end());
        rb.push_back(c.r_bound);
    }
    put(ix, "cell_members", mem.data(), mem.size());
    put(ix, "cell_member_off", moff.data(), moff.size());
    put(ix, "centroids", cents.data(), cents.size());
    put(ix, "r_bound", rb.data(), rb.size());
    put(ix, "prim_len", h.prim_len.data(), h.prim_len.size());
    put(ix, "rep_off", h.rep_off.data(), h.rep_off.size());
    put(ix, "fs_codes", h.fs_codes.data(), h.fs_codes.size());
    put(ix, "fs_off", h.fs_off.data(), h.fs_off.size());
    put(ix, "cent_bits", h.cent_bits.data(), h.cent_bits.size());
    put(ix, "cent_sq8", h.cent_sq8.data(), h.cent_sq8.size());
    put(ix, "csq_min", h.csq_min.data(), h.csq_min.size());
    put(ix, "csq_step", h.csq_step.data(), h.csq_step.size());
    put(ix, "sq_min", h.sq_min.data(), h.sq_min.size());
    put(ix, "sq_step", h.sq_step.data(), h.sq_step.size());
    put(ix, "signs", h.signs.data(), h.signs.size());
    put(ix, "tags", h.tags.data(), h.tags.size());
    std::vector<uint64_t> lvn, tcodes, tcoff{0}, tcs, tcl, tchoff{0}, lcodes;
    std::vector<uint32_t> lids;
    if (h.tree) {
        for (auto& l : h.tree->levels) {
            lvn.push_back(l.n);
            tcodes.insert(tcodes.end(), l.codes.begin(), l.codes.end());
            tcoff.push_back(tcodes.size());
            tcs.insert(tcs.end(), l.child_start.begin(), l.child_start.end());
            tcl.insert(tcl.end(), l.child_len.begin(), l.child_len.end());
            tchoff.push_back(tcs.size());
        }
        lcodes = h.tree->leaf_codes;
        lids = h.tree->leaf_ids;
    }
    put(ix, "tree_level_n", lvn.data(), lvn.size());
    put(ix, "tree_codes", tcodes.data(), tcodes.size());
    put(ix, "tree_code_off", tcoff.data(), tcoff.size());
    put(ix, "tree_child_start", tcs.data(), tcs.size());
    put(ix, "tree_child_len", tcl.data(), tcl.size());
    put(ix, "tree_child_off", tchoff.data(), tchoff.size());
    put(ix, "tree_leaf_codes", lcodes.data(), lcodes.size());
    put(ix, "tree_leaf_ids", lids.data(), lids.size());
    ix->arrays_version = h.version;
}

}  // namespace

namespace maivs_capi {
int device_image(maivs_index* ix) { return ensure_device(ix); }
void host_arrays(maivs_index* ix) { build_arrays(ix); }
}  // namespace maivs_capi

extern "C" {

int maivs_index_new(size_t dim, const char* scan_mode, size_t rerank_factor, uint64_t seed, size_t code_bits,
                    maivs_index** out) {
    if (!out) return MAIVS_BAD_ARG;
    *out = nullptr;
    auto ix = new (std::nothrow) maivs_index();
    if (!ix) return MAIVS_OOM;
    std::string e = ix->h.init(dim, scan_mode ? scan_mode : "", rerank_factor, seed, code_bits);
    if (!e.empty()) {
        // keep the handle so the caller can read the message, then let it free it
        ix->err = e;
        *out = ix;
        return MAIVS_BAD_ARG;
    }
    *out = ix;
    return MAIVS_OK;
}

void maivs_index_free(maivs_index* ix) { delete ix; }

const char* maivs_last_error(const maivs_index* ix) { return ix ? ix->err.c_str() : "null handle"; }

const char* maivs_status_string(int s) {
    switch (s) {
        case MAIVS_OK: return "ok";
        case MAIVS_BAD_SHAPE: return "bad shape";
        case MAIVS_BAD_ARG: return "bad argument";
        case MAIVS_BAD_STATE: return "bad state";
        case MAIVS_OOM: return "out of memory";
        case MAIVS_CUDA_ERROR: return "CUDA error";
        case MAIVS_OVERFLOW: return "candidate buffer overflow";
        case MAIVS_UNSUPPORTED: return "unsupported";
        case MAIVS_NOT_FOUND: return "not found";
        case MAIVS_NO_DEVICE: return "no CUDA device";
        default: return "unknown status";
    }
}

#define LOCK(ix)                    \
    if (!(ix)) return MAIVS_BAD_ARG; \
    std::lock_guard<std::mutex> lk_((ix)->mu)

int maivs_train_centroids(maivs_index* ix, const float* v, size_t n, size_t n_cells, size_t sample, uint64_t seed) {
    LOCK(ix);
    return check(ix, ix->h.train_centroids(v, n, n_cells, sample, seed));
}

int maivs_set_centroids(maivs_index* ix, const float* c, size_t m) {
    LOCK(ix);
    return check(ix, ix->h.set_centroids(c, m));
}

int maivs_add_batch(maivs_index* ix, const uint64_t* ids, const float* v, size_t n) {
    LOCK(ix);
    return check(ix, ix->h.add_batch(ids, v, n), MAIVS_BAD_STATE);
}

int maivs_remove(maivs_index* ix, uint64_t id, int* removed) {
    LOCK(ix);
    bool r = ix->h.remove(id);
    if (removed) *removed = r ? 1 : 0;
    return MAIVS_OK;
}

int maivs_save(maivs_index* ix, const char* path) {
    LOCK(ix);
    if (!path) return fail(ix, MAIVS_BAD_ARG, "path is null");
    return check(ix, maivs::save_index(ix->h, path), MAIVS_BAD_STATE);
}

int maivs_load(const char* path, maivs_index** out) {
    if (!out) return MAIVS_BAD_ARG;
    *out = nullptr;
    auto ix = std::make_unique<maivs_index>();
    if (!path) return MAIVS_BAD_ARG;
    std::string e = maivs::load_index(path, ix->h);
    if (!e.empty()) {
        ix->err = e;
        *out = ix.release();  // the caller reads the message, then frees the handle
        return MAIVS_BAD_ARG;
    }
    *out = ix.release();
    return MAIVS_OK;
}

int maivs_compact(maivs_index* ix) {
    LOCK(ix);
    ix->h.compact();
    return MAIVS_OK;
}

int maivs_set_rerank_factor(maivs_index* ix, size_t rf) {
    LOCK(ix);
    ix->h.rerank_factor = std::max<size_t>(rf, 1);
    return MAIVS_OK;
}
int maivs_set_two_stage(maivs_index* ix, int on, size_t mult) {
    LOCK(ix);
    ix->h.set_two_stage(on != 0, mult);
    return MAIVS_OK;
}
int maivs_set_tree_route(maivs_index* ix, int on, size_t min_cells, size_t fanout, float beam_frac) {
    LOCK(ix);
    ix->h.set_tree_route(on != 0, min_cells, fanout, beam_frac);
    return MAIVS_OK;
}
int maivs_set_graph_route(maivs_index* ix, int on, size_t min_cells) {
    LOCK(ix);
    ix->h.graph_route = on != 0;
    if (min_cells > 0) ix->h.graph_min_cells = min_cells;
    ++ix->h.version;
    return MAIVS_OK;
}
int maivs_set_adaptive(maivs_index* ix, int on, float margin) {
    LOCK(ix);
    ix->h.adaptive = on != 0;
    ix->h.at_margin = margin;
    return MAIVS_OK;
}
int maivs_set_fastscan(maivs_index* ix, int on) {
    LOCK(ix);
    ix->h.set_fastscan(on != 0);
    return MAIVS_OK;
}
int maivs_set_orthogonal_polysemy(maivs_index* ix, size_t homes, float lam) {
    LOCK(ix);
    ix->h.set_orthogonal_polysemy(homes, lam);
    return MAIVS_OK;
}
int maivs_set_replication(maivs_index* ix, size_t ma, float margin) {
    LOCK(ix);
    ix->h.set_replication(ma, margin);
    return MAIVS_OK;
}
int maivs_set_per_dim_sq(maivs_index* ix, int on) {
    LOCK(ix);
    ix->h.set_per_dim_sq(on != 0);
    return MAIVS_OK;
}
int maivs_set_i8_rerank(maivs_index* ix, int on) {
    LOCK(ix);
    ix->h.set_i8_rerank(on != 0);
    return MAIVS_OK;
}
int maivs_set_centroid_sq8(maivs_index* ix, int on) {
    LOCK(ix);
    ix->h.set_centroid_sq8(on != 0);
    return MAIVS_OK;
}
int maivs_set_tags(maivs_index* ix, const uint64_t* ids, const uint32_t* tags, size_t n) {
    LOCK(ix);
    return check(ix, ix->h.set_tags(ids, tags, n));
}
int maivs_set_filter(maivs_index* ix, int has, uint32_t lo, uint32_t hi) {
    LOCK(ix);
    ix->h.has_filter = has != 0;
    ix->h.filter_lo = lo;
    ix->h.filter_hi = hi;
    return MAIVS_OK;
}
int maivs_set_cell_major_min_batch(maivs_index* ix, size_t n) {
    LOCK(ix);
    ix->h.cm_min_batch = n;
    return MAIVS_OK;
}

int maivs_set_build_device(maivs_index* ix, int device) {
    LOCK(ix);
    if (device >= 0) {
        int n = 0;
        if (cudaGetDeviceCount(&n) != cudaSuccess || device >= n)
            return fail(ix, MAIVS_NO_DEVICE, "no CUDA device " + std::to_string(device) + " for the index build");
    }
    ix->h.build_device = device < 0 ? -1 : device;
    return MAIVS_OK;
}

int maivs_len(const maivs_index* ix, size_t* n) {
    if (!ix || !n) return MAIVS_BAD_ARG;
    *n = ix->h.n_live;
    return MAIVS_OK;
}

int maivs_stat(maivs_index* ix, const char* name, double* value) {
    LOCK(ix);
    if (!name || !value) return MAIVS_BAD_ARG;
    const HostIndex& h = ix->h;
    std::string s(name);
    size_t live = 0, smin = SIZE_MAX, smax = 0, entries = 0;
    for (auto& c : h.cells) {
        live += !c.members.empty();
        smin = std::min(smin, c.members.size());
        smax = std::max(smax, c.members.size());
        entries += c.members.size();
    }
    double n = (double)std::max<size_t>(h.n_live, 1);
    if (s == "n_live") *value = (double)h.n_live;
    else if (s == "n_cells") *value = (double)h.cells.size();
    else if (s == "live_cells") *value = (double)live;
    else if (s == "free_slots") *value = (double)h.free_slots.size();
    else if (s == "quant_scale") *value = h.quant_scale;
    else if (s == "scan_bytes_per_vec") *value = (double)(h.nw * 8);
    else if (s == "cell_size_mean") *value = h.cells.empty() ? 0.0 : (double)entries / (double)h.cells.size();
    else if (s == "cell_size_max") *value = (double)smax;
    else if (s == "cell_size_min") *value = h.cells.empty() ? 0.0 : (double)smin;
    else if (s == "max_assign") *value = (double)h.max_assign;
    else if (s == "tree_depth") *value = h.tree ? (double)h.tree->levels.size() : 0.0;
    else if (s == "tree_top_width") *value = h.tree && !h.tree->levels.empty() ? (double)h.tree->levels[0].n : 0.0;
    else if (s == "tree_fanout") *value = (double)h.tree_fanout;
    else if (s == "tree_beam_frac") *value = h.tree_beam_frac;
    else if (s == "replication_factor") *value = (double)entries / n;
    else if (s == "member_entries") *value = (double)entries;
    else if (s == "centroid_graph_nodes") *value = 0.0;
    else if (s == "device_bytes") *value = ix->d ? (double)ix->d->device_bytes() : 0.0;
    else if (s == "build_device") *value = (double)h.build_device;
    else if (s == "build_gpu_failures") *value = (double)h.build_gpu_failures;
    else if (s == "total_bytes") {
        size_t b = h.vecs_f32.size() * 4 + h.scan_i8.size() + h.bits.size() * 8 + h.ext_ids.size() * 8 +
                   h.slot_cell.size() * 4 + h.slot_cells.size() * 4 + h.tags.size() * 4 + entries * 4 +
                   h.cells.size() * h.dim * 8 + h.cent_bits.size() * 8 + h.cent_sq8.size() + h.fs_codes.size() +
                   h.fs_off.size() * 4 + h.prim_len.size() * 4 + h.rep_off.size() * 4;
        *value = (double)b;
    } else
        return fail(ix, MAIVS_NOT_FOUND, "unknown stat '" + s + "'");
    return MAIVS_OK;
}

int maivs_to_device(maivs_index* ix, int device) {
    LOCK(ix);
    ix->device = device;
    ix->d.reset();
    return ensure_device(ix);
}

int maivs_search_batch(maivs_index* ix, const float* Q, size_t nq, size_t k, size_t nprobe, float tc, float beta,
                       int cell_major, uint64_t* ids, float* scores) {
    LOCK(ix);
    if (nq == 0) return MAIVS_OK;
    if (k == 0) return fail(ix, MAIVS_BAD_ARG, "k must be positive");
    if (ix->h.cells.empty() || ix->h.n_live == 0) {
        // empty index: all padding (index.rs:3337-3339)
        for (size_t i = 0; i < nq * k; ++i) {
            ids[i] = UINT64_MAX;
            scores[i] = -INFINITY;
        }
        return MAIVS_OK;
    }
    int rc = ensure_device(ix);
    if (rc != MAIVS_OK) return rc;
    ix->d->set_timing(g_prof_on.load());
    maivs::SearchArgs a;
    a.nq = (int)nq;
    a.k = (int)k;
    a.nprobe = (int)std::min<size_t>(nprobe, 1u << 30);
    a.tc = tc;
    a.beta = beta;
    a.cell_major = cell_major != 0;
    std::string err;
    rc = ix->d->search_host(ix->h, Q, a, ids, scores, nullptr, err);
    if (rc != MAIVS_OK) return fail(ix, rc, err);
    record_phases(ix, (int)nq);
    return MAIVS_OK;
}

int maivs_search(maivs_index* ix, const float* q, size_t k, size_t nprobe, float tc, float beta, uint64_t* ids,
                 float* scores, size_t* n_out) {
    LOCK(ix);
    if (n_out) *n_out = 0;
    if (ix->h.cells.empty() || ix->h.n_live == 0) return MAIVS_OK;  // (index.rs:3294-3296)
    if (k == 0) return fail(ix, MAIVS_BAD_ARG, "k must be positive");
    int rc = ensure_device(ix);
    if (rc != MAIVS_OK) return rc;
    ix->d->set_timing(g_prof_on.load());
    maivs::SearchArgs a;
    a.nq = 1;
    a.k = (int)k;
    a.nprobe = (int)std::min<size_t>(nprobe, 1u << 30);
    a.tc = tc;
    a.beta = beta;
    a.cell_major = false;
    std::string err;
    uint32_t nout = 0;
    rc = ix->d->search_host(ix->h, q, a, ids, scores, &nout, err);
    if (rc != MAIVS_OK) return fail(ix, rc, err);
    if (n_out) *n_out = nout;
    record_phases(ix, 1);
    return MAIVS_OK;
}

int maivs_search_batch_device(maivs_index* ix, const float* dQ, size_t nq, size_t k, size_t nprobe, float tc,
                              float beta, int cell_major, uint64_t* d_ids, float* d_scores, void* stream) {
    LOCK(ix);
    if (nq == 0) return MAIVS_OK;
    if (k == 0) return fail(ix, MAIVS_BAD_ARG, "k must be positive");
    if (ix->h.cells.empty() || ix->h.n_live == 0) return fail(ix, MAIVS_BAD_STATE, "the index is empty");
    int rc = ensure_device(ix);
    if (rc != MAIVS_OK) return rc;
    maivs::SearchArgs a;
    a.nq = (int)nq;
    a.k = (int)k;
    a.nprobe = (int)std::min<size_t>(nprobe, 1u << 30);
    a.tc = tc;
    a.beta = beta;
    a.cell_major = cell_major != 0;
    std::string err;
    // the per-query counts go to a small device buffer owned by the workspace-free path
    static thread_local uint32_t* d_nout = nullptr;
    static thread_local size_t d_nout_cap = 0;
    if (d_nout_cap < nq) {
        if (d_nout) cudaFree(d_nout);
        d_nout = nullptr;
        if (cudaMalloc(&d_nout, nq * sizeof(uint32_t)) != cudaSuccess) return fail(ix, MAIVS_OOM, "cudaMalloc failed");
        d_nout_cap = nq;
    }
    rc = ix->d->search_device(ix->h, dQ, a, d_ids, d_scores, d_nout, (cudaStream_t)stream, err);
    if (rc != MAIVS_OK) return fail(ix, rc, err);
    return MAIVS_OK;
}

int maivs_search_batch_device_noalloc(maivs_index* ix, const float* dQ, size_t nq, size_t k, size_t nprobe,
                                      float tc, float beta, uint64_t* d_ids, float* d_scores, void* stream) {
    LOCK(ix);
    if (nq == 0) return MAIVS_OK;
    if (k == 0) return fail(ix, MAIVS_BAD_ARG, "k must be positive");
    if (k > 4096) return fail(ix, MAIVS_UNSUPPORTED, "k above 4096 is not supported");
    if (nq > 64) return fail(ix, MAIVS_BAD_ARG, "the allocation-free search takes at most 64 queries per call");
    if (ix->exch) return fail(ix, MAIVS_UNSUPPORTED, "the allocation-free search does not run on a sharded index");
    // uploading the index allocates, so the device image must already be current
    if (!ix->d || ix->d->version() != ix->h.version || ix->d->device() != ix->device)
        return fail(ix, MAIVS_BAD_STATE, "no current device image; call maivs_to_device() before this search");
    maivs::SearchArgs a;
    a.nq = (int)nq;
    a.k = (int)k;
    a.nprobe = (int)std::min<size_t>(nprobe, 1u << 30);
    a.tc = tc;
    a.beta = beta;
    a.cell_major = false;
    std::string err;
    int rc = ix->d->search_static(ix->h, dQ, a, d_ids, d_scores, (cudaStream_t)stream, err);
    if (rc != MAIVS_OK) return fail(ix, rc, err);
    return MAIVS_OK;
}

int maivs_nccl_unique_id(uint8_t* id, size_t cap) {
    if (!id || cap < 128) return MAIVS_BAD_ARG;
    std::string err;
    return maivs::nccl_unique_id(id, err);
}

int maivs_shard(maivs_index* ix, int rank, int world, const uint8_t* nccl_id, size_t id_len) {
    LOCK(ix);
    if (world < 1 || rank < 0 || rank >= world) return fail(ix, MAIVS_BAD_ARG, "need 0 <= rank < world");
    int n = 0;
    if (cudaGetDeviceCount(&n) != cudaSuccess || n == 0)
        return fail(ix, MAIVS_NO_DEVICE, "no CUDA device is visible; the MAIVS GPU search has no CPU fallback");
    ix->d.reset();
    ix->exch.reset();
    ix->shard_rank = 0;
    ix->shard_world = 1;
    if (world == 1) return MAIVS_OK;
    if (!nccl_id || id_len != 128) return fail(ix, MAIVS_BAD_ARG, "the NCCL unique id is 128 bytes");
    std::string err;
    auto x = maivs::nccl_exchange(nccl_id, rank, world, ix->device, err);
    if (!x) return fail(ix, MAIVS_CUDA_ERROR, err);
    ix->exch = std::move(x);
    ix->shard_rank = rank;
    ix->shard_world = world;
    return MAIVS_OK;
}

int maivs_shard_range(maivs_index* ix, int rank, int world, uint32_t* lo, uint32_t* hi) {
    LOCK(ix);
    if (world < 1 || rank < 0 || rank >= world) return fail(ix, MAIVS_BAD_ARG, "need 0 <= rank < world");
    maivs::shard_range(ix->h, rank, world, lo, hi);
    return MAIVS_OK;
}

int maivs_search_batch_sharded_emulated(maivs_index* ix, int world, const float* dQ, size_t nq, size_t k,
                                        size_t nprobe, float tc, float beta, uint64_t* d_ids, float* d_scores,
                                        void* stream) {
    LOCK(ix);
    if (nq == 0) return MAIVS_OK;
    if (k == 0) return fail(ix, MAIVS_BAD_ARG, "k must be positive");
    if (world < 1 || world > 64) return fail(ix, MAIVS_BAD_ARG, "world must be in 1..64");
    if (ix->h.cells.empty() || ix->h.n_live == 0) return fail(ix, MAIVS_BAD_STATE, "the index is empty");
    int n = 0;
    if (cudaGetDeviceCount(&n) != cudaSuccess || n == 0)
        return fail(ix, MAIVS_NO_DEVICE, "no CUDA device is visible; the MAIVS GPU search has no CPU fallback");
    if (ix->emu_version != ix->h.version || ix->emu_world != world || ix->emu_device != ix->device) {
        ix->emu.clear();
        ix->emu_version = ~0ull;
        for (int r = 0; r < world; ++r) {
            uint32_t lo, hi;
            maivs::shard_range(ix->h, r, world, &lo, &hi);
            auto d = std::make_unique<DeviceIndex>();
            std::string e = d->upload(ix->h, ix->device, lo, hi);
            if (!e.empty()) {
                ix->emu.clear();
                return fail(ix, MAIVS_BAD_STATE, e);
            }
            ix->emu.push_back(std::move(d));
        }
        ix->emu_version = ix->h.version;
        ix->emu_world = world;
        ix->emu_device = ix->device;
    }
    maivs::SearchArgs a;
    a.nq = (int)nq;
    a.k = (int)k;
    a.nprobe = (int)std::min<size_t>(nprobe, 1u << 30);
    a.tc = tc;
    a.beta = beta;
    a.cell_major = true;
    cudaSetDevice(ix->device);
    static thread_local uint32_t* d_nout = nullptr;
    static thread_local size_t d_nout_cap = 0;
    if (d_nout_cap < nq) {
        if (d_nout) cudaFree(d_nout);
        d_nout = nullptr;
        if (cudaMalloc(&d_nout, nq * sizeof(uint32_t)) != cudaSuccess) return fail(ix, MAIVS_OOM, "cudaMalloc failed");
        d_nout_cap = nq;
    }
    std::string err;
    int rc = maivs::search_emulated_shards(ix->h, ix->emu, dQ, a, d_ids, d_scores, d_nout,
                                           stream ? (cudaStream_t)stream : ix->emu[0]->stream(), err);
    if (rc != MAIVS_OK) return fail(ix, rc, err);
    return MAIVS_OK;
}

int maivs_device_flags(maivs_index* ix, void* stream, uint32_t* flags) {
    LOCK(ix);
    if (!ix->d) return fail(ix, MAIVS_BAD_STATE, "no device image");
    uint32_t f = ix->d->read_flags(stream ? (cudaStream_t)stream : ix->d->stream());
    if (f) ix->d->grow_factor *= 4;
    if (flags) *flags = f;
    return MAIVS_OK;
}

int maivs_array(maivs_index* ix, const char* name, const void** data, size_t* count, size_t* elem_bytes) {
    LOCK(ix);
    if (!name || !data || !count) return MAIVS_BAD_ARG;
    build_arrays(ix);
    auto it = ix->arrays.find(name);
    if (it == ix->arrays.end()) return fail(ix, MAIVS_NOT_FOUND, std::string("unknown array '") + name + "'");
    static const std::map<std::string, size_t> eb = {
        {"vecs_f32", 4},        {"scan_i8", 1},         {"bits", 8},          {"ext_ids", 8},
        {"slot_cell", 4},       {"slot_cells", 4},      {"cell_members", 4},  {"cell_member_off", 4},
        {"centroids", 4},       {"r_bound", 4},         {"prim_len", 4},      {"rep_off", 4},
        {"fs_codes", 1},        {"fs_off", 4},          {"cent_bits", 8},     {"cent_sq8", 1},
        {"csq_min", 4},         {"csq_step", 4},        {"sq_min", 4},        {"sq_step", 4},
        {"signs", 4},           {"tags", 4},            {"tree_level_n", 8},  {"tree_codes", 8},
        {"tree_code_off", 8},   {"tree_child_start", 8}, {"tree_child_len", 8}, {"tree_child_off", 8},
        {"tree_leaf_codes", 8}, {"tree_leaf_ids", 4},   {"config", 8}};
    size_t e = eb.at(name);
    *data = it->second.empty() ? nullptr : it->second.data();
    *count = it->second.size() / e;
    if (elem_bytes) *elem_bytes = e;
    return MAIVS_OK;
}

int maivs_kernel_clock(maivs_index* ix, int on) {
    LOCK(ix);
    int rc = ensure_device(ix);
    if (rc != MAIVS_OK) return rc;
    ix->d->enable_kernel_clock(on != 0);
    if (on) ix->d->kernel_clock()->only = -1;
    return MAIVS_OK;
}

int maivs_kernel_clock_only(maivs_index* ix, const char* kernel) {
    LOCK(ix);
    int rc = ensure_device(ix);
    if (rc != MAIVS_OK) return rc;
    int id = -1;
    if (kernel && *kernel) {
        for (int i = 0; i < maivs::dev::kNumKernels; ++i)
            if (std::strcmp(maivs::dev::kernel_name(i), kernel) == 0) id = i;
        if (id < 0) return fail(ix, MAIVS_BAD_ARG, std::string("unknown kernel name: ") + kernel);
    }
    ix->d->enable_kernel_clock(true);
    ix->d->kernel_clock()->only = id;
    return MAIVS_OK;
}

int maivs_kernel_times(maivs_index* ix, int reset, const char** names, double* ms, uint64_t* launches, size_t cap,
                       size_t* n_out) {
    LOCK(ix);
    size_t n = std::min<size_t>(cap, maivs::dev::kNumKernels);
    if (n_out) *n_out = n;
    maivs::dev::KernelClock* c = ix->d ? ix->d->kernel_clock() : nullptr;
    if (c) c->collect();
    for (size_t i = 0; i < n; ++i) {
        if (names) names[i] = maivs::dev::kernel_name((int)i);
        if (ms) ms[i] = c ? c->ms[i] : 0.0;
        if (launches) launches[i] = c ? c->launches[i] : 0;
    }
    if (reset && c)
        for (size_t i = 0; i < maivs::dev::kNumKernels; ++i) {
            c->ms[i] = 0.0;
            c->busy[i] = 0.0;
            c->launches[i] = 0;
        }
    return MAIVS_OK;
}

int maivs_kernel_busy(maivs_index* ix, const char** names, double* busy_ms, size_t cap, size_t* n_out) {
    LOCK(ix);
    size_t n = std::min<size_t>(cap, maivs::dev::kNumKernels);
    if (n_out) *n_out = n;
    maivs::dev::KernelClock* c = ix->d ? ix->d->kernel_clock() : nullptr;
    if (c) c->collect();
    for (size_t i = 0; i < n; ++i) {
        if (names) names[i] = maivs::dev::kernel_name((int)i);
        if (busy_ms) busy_ms[i] = c ? c->busy[i] : 0.0;
    }
    return MAIVS_OK;
}

uint64_t maivs_launch_count(void) { return maivs::dev::total_launches(); }

int maivs_set_num_threads(int n) {
    if (n < 1) return MAIVS_BAD_ARG;
    omp_set_num_threads(n);
    return MAIVS_OK;
}

int maivs_last_search_stats(maivs_index* ix, char* names, size_t names_cap, double* values, size_t cap,
                            size_t* n_out) {
    LOCK(ix);
    if (!ix->d) return fail(ix, MAIVS_BAD_STATE, "no search has run");
    auto st = ix->d->last_stats();
    size_t n = std::min(cap, st.size());
    std::string joined;
    for (size_t i = 0; i < n; ++i) {
        values[i] = st[i].second;
        joined += st[i].first;
        joined += '\n';
    }
    if (names && names_cap) {
        size_t m = std::min(names_cap - 1, joined.size());
        std::memcpy(names, joined.data(), m);
        names[m] = 0;
    }
    if (n_out) *n_out = n;
    return MAIVS_OK;
}

int maivs_debug_stage(maivs_index* ix, int stage, const float* Q, size_t nq, size_t k, size_t nprobe, float tc,
                      float beta, int cell_major, uint64_t* qbits, uint8_t* lut, float* delta, float* bias,
                      uint32_t* chosen, float* cscore, uint32_t* nch, uint32_t* cand, size_t cand_cap,
                      uint32_t* cand_n) {
    LOCK(ix);
    if (nq == 0 || k == 0) return fail(ix, MAIVS_BAD_ARG, "nq and k must be positive");
    if (!cell_major && nq > 64) return fail(ix, MAIVS_BAD_ARG, "the per-query debug path takes at most 64 queries");
    int rc = ensure_device(ix);
    if (rc != MAIVS_OK) return rc;
    maivs::SearchArgs a;
    a.nq = (int)nq;
    a.k = (int)k;
    a.nprobe = (int)std::min<size_t>(nprobe, 1u << 30);
    a.tc = tc;
    a.beta = beta;
    a.cell_major = cell_major != 0;
    maivs::DebugOut out;
    out.stage = stage;
    float* dQ = nullptr;
    uint64_t* dI = nullptr;
    float* dS = nullptr;
    cudaMalloc(&dQ, nq * ix->h.dim * sizeof(float));
    cudaMalloc(&dI, nq * k * sizeof(uint64_t));
    cudaMalloc(&dS, nq * k * sizeof(float) + nq * sizeof(uint32_t));
    cudaMemcpy(dQ, Q, nq * ix->h.dim * sizeof(float), cudaMemcpyHostToDevice);
    ix->d->dbg = &out;
    std::string err;
    rc = ix->d->search_device(ix->h, dQ, a, dI, dS, reinterpret_cast<uint32_t*>(dS + nq * k), ix->d->stream(), err);
    ix->d->dbg = nullptr;
    cudaStreamSynchronize(ix->d->stream());
    cudaFree(dQ);
    cudaFree(dI);
    cudaFree(dS);
    if (rc != MAIVS_OK) return fail(ix, rc, err);
    const size_t nw = ix->h.nw, npos = nw * 16;
    if (stage == 0) {
        if (qbits) std::memcpy(qbits, out.qbits.data(), nq * nw * 8);
        if (lut) std::memcpy(lut, out.lut.data(), nq * npos * 16);
        if (delta) std::memcpy(delta, out.delta.data(), nq * 4);
        if (bias) std::memcpy(bias, out.bias.data(), nq * 4);
    } else if (stage == 1) {
        const size_t np = (size_t)out.nprobe;
        for (size_t q = 0; q < nq; ++q) {
            if (nch) nch[q] = out.nch[q];
            for (size_t i = 0; i < nprobe; ++i) {
                bool v = i < np && i < out.nch[q];
                if (chosen) chosen[q * nprobe + i] = v ? out.chosen[q * np + i] : UINT32_MAX;
                if (cscore) cscore[q * nprobe + i] = v ? out.cscore[q * np + i] : -INFINITY;
            }
        }
    } else if (stage == 2) {
        const size_t cc = (size_t)out.cand_cap;
        for (size_t q = 0; q < nq; ++q) {
            uint32_t n = out.cand_n[q];
            if (cand_n) cand_n[q] = n;
            if (cand) {
                std::vector<uint32_t> v(out.cand.begin() + q * cc, out.cand.begin() + q * cc + n);
                std::sort(v.begin(), v.end());
                for (size_t i = 0; i < cand_cap; ++i) cand[q * cand_cap + i] = i < v.size() ? v[i] : UINT32_MAX;
            }
        }
    }
    return MAIVS_OK;
}

int maivs_debug_cellmajor(maivs_index* ix, const float* Q, size_t nq, size_t k, size_t nprobe, float tc, float beta,
                          uint32_t* seed_n, uint32_t* tau, uint32_t* rest_hi, uint32_t* rest_n, char* info,
                          size_t info_cap) {
    LOCK(ix);
    if (nq == 0 || k == 0) return fail(ix, MAIVS_BAD_ARG, "nq and k must be positive");
    int rc = ensure_device(ix);
    if (rc != MAIVS_OK) return rc;
    maivs::SearchArgs a;
    a.nq = (int)nq;
    a.k = (int)k;
    a.nprobe = (int)nprobe;
    a.tc = tc;
    a.beta = beta;
    a.cell_major = true;
    if (!ix->d->use_cell_major(ix->h, a)) return fail(ix, MAIVS_BAD_STATE, "this batch does not take the cell-major join");
    maivs::DebugOut out;
    out.stage = 2;
    float* dQ = nullptr;
    void* dO = nullptr;
    cudaMalloc(&dQ, nq * ix->h.dim * sizeof(float));
    cudaMalloc(&dO, nq * k * 16 + nq * 4);
    cudaMemcpy(dQ, Q, nq * ix->h.dim * sizeof(float), cudaMemcpyHostToDevice);
    ix->d->dbg = &out;
    std::string err;
    cudaGetLastError();
    rc = ix->d->search_device(ix->h, dQ, a, (uint64_t*)dO, (float*)((char*)dO + nq * k * 8),
                              (uint32_t*)((char*)dO + nq * k * 12), ix->d->stream(), err);
    ix->d->dbg = nullptr;
    cudaError_t ce = cudaStreamSynchronize(ix->d->stream());
    cudaError_t le = cudaGetLastError();
    cudaFree(dQ);
    cudaFree(dO);
    if (rc != MAIVS_OK) return fail(ix, rc, err);
    for (size_t q = 0; q < nq; ++q) {
        if (seed_n) seed_n[q] = out.seed_n[q];
        if (tau) tau[q] = out.tau[q];
        if (rest_hi) rest_hi[q] = out.rest_hi[q];
        if (rest_n) rest_n[q] = out.rest_n[q];
    }
    if (info && info_cap) {
        std::string s = std::string("sync=") + cudaGetErrorString(ce) + " last=" + cudaGetErrorString(le);
        std::strncpy(info, s.c_str(), info_cap - 1);
        info[info_cap - 1] = 0;
    }
    return MAIVS_OK;
}

int maivs_profile(int on) {
    g_prof_on.store(on != 0);
    return MAIVS_OK;
}

int maivs_profile_read(int reset, const char** names, double* values, size_t cap, size_t* n_out) {
    std::lock_guard<std::mutex> lk(g_prof_mu);
    size_t n = std::min(cap, kNumPhases);
    for (size_t i = 0; i < n; ++i) {
        if (names) names[i] = kPhaseNames[i];
        if (values) values[i] = g_prof[i];
    }
    if (n_out) *n_out = n;
    if (reset)
        for (double& v : g_prof) v = 0.0;
    return MAIVS_OK;
}

}  // extern "C"
