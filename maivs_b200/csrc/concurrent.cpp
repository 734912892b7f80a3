// ConcurrentIndex (src/concurrent.rs): reads over immutable sealed segments plus one mutable head,
// deletes as tombstones by external id. The host side keeps the reference's structure and its lock
// order (head -> sealed -> dead; concurrent.rs:138-141, :266-267, :306); the searches run on the
// GPU: every segment and the head by the per-query path (concurrent.rs:113-131 calls search_one on
// each), into one device buffer of per-segment lists, and the merge (finish, :83-110) is one kernel
// (k_merge.cu). Device work of one handle is serialised by gpu_mu; a search holds the head's
// shared lock only while it enqueues the head's part.
#include <cuda_runtime.h>

#include <algorithm>
#include <cmath>
#include <cstring>
#include <memory>
#include <mutex>
#include <shared_mutex>
#include <string>
#include <unordered_set>
#include <vector>

#include "../../include/maivs_b200.h"
#include "handle.h"

using SegList = std::vector<std::shared_ptr<maivs_index>>;

struct maivs_concurrent {
    // the one mutable segment
    std::shared_mutex head_mu;
    std::unique_ptr<maivs_index> head;
    // sealed segments: a reader copies the pointer and scans them with no lock held
    std::shared_mutex sealed_mu;
    std::shared_ptr<const SegList> sealed = std::make_shared<const SegList>();
    size_t sealed_live = 0;
    // tombstones by external id
    std::shared_mutex dead_mu;
    std::unordered_set<uint64_t> dead;
    uint64_t dead_version = 0;
    size_t seal_at = 1000000;
    bool par_scan = false;

    // device search state (gpu_mu)
    std::mutex gpu_mu;
    int device = 0;
    cudaStream_t st = nullptr;
    void* dbuf = nullptr;
    size_t dbuf_bytes = 0;
    void* pin = nullptr;
    size_t pin_bytes = 0;
    uint64_t* dtomb = nullptr;
    size_t dtomb_cap = 0;
    uint64_t tomb_version = ~0ull;
    int ntomb = 0;
    // per-kernel device times (instrumentation): the merge's here, the searches' in each image
    bool clock_on = false;
    std::unique_ptr<maivs::dev::KernelClock> clock;

    std::mutex err_mu;
    std::string err;

    ~maivs_concurrent() {
        if (st) {
            cudaStreamSynchronize(st);
            cudaStreamDestroy(st);
        }
        if (dbuf) cudaFree(dbuf);
        if (dtomb) cudaFree(dtomb);
        if (pin) cudaFreeHost(pin);
    }
};

namespace {

// Over-fetch factor on k per segment once tombstones exist (concurrent.rs:50-52).
constexpr size_t kOverfetch = 2;
// Queries per device pass of a batch (bounds the per-segment list buffers).
constexpr size_t kQueryChunk = 8192;

int cfail(maivs_concurrent* cx, int status, const std::string& msg) {
    if (cx) {
        std::lock_guard<std::mutex> lk(cx->err_mu);
        cx->err = msg;
    }
    return status;
}

// Freeze the head into a sealed segment (concurrent.rs:134-152). Caller holds head_mu exclusively.
void seal_locked(maivs_concurrent* cx) {
    maivs_index* h = cx->head.get();
    if (h->h.n_live == 0) return;
    h->h.compact();
    auto fresh = std::make_unique<maivs_index>();
    h->h.fork_empty(fresh->h);
    fresh->device = cx->device;
    std::shared_ptr<maivs_index> frozen(cx->head.release());
    cx->head = std::move(fresh);
    const size_t n = frozen->h.n_live;
    std::unique_lock<std::shared_mutex> sl(cx->sealed_mu);
    auto list = std::make_shared<SegList>(*cx->sealed);
    list->push_back(std::move(frozen));
    cx->sealed = std::move(list);
    cx->sealed_live += n;
}

std::shared_ptr<const SegList> snapshot(maivs_concurrent* cx) {
    std::shared_lock<std::shared_mutex> sl(cx->sealed_mu);
    return cx->sealed;
}

template <typename F>
int with_head_write(maivs_concurrent* cx, F&& f) {
    if (!cx) return MAIVS_BAD_ARG;
    std::unique_lock<std::shared_mutex> hl(cx->head_mu);
    f(cx->head->h);
    return MAIVS_OK;
}

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

// One device pass over queries Q[0, nq): every segment's search into its list, the head's, the
// merge. Returns a status; on success ids/scores (nq x k) are filled.
int search_pass(maivs_concurrent* cx, const SegList& segs, const float* Q, size_t nq, size_t dim, size_t k,
                size_t want, size_t nprobe, float tc, float beta, uint64_t* ids, float* scores) {
    const size_t L = segs.size() + 1;
    auto carve = [&](Bump& b, float*& dQ, uint64_t*& lid, float*& lsc, uint32_t*& lnout, uint64_t*& oid,
                     float*& osc, void*& scratch) {
        dQ = b.take<float>(nq * dim);
        lid = b.take<uint64_t>(L * nq * want);
        lsc = b.take<float>(L * nq * want);
        lnout = b.take<uint32_t>(L * nq);
        oid = b.take<uint64_t>(nq * k);
        osc = b.take<float>(nq * k);
        scratch = b.take<char>(nq * L * want * 16);
    };
    float *dQ, *lsc, *osc;
    uint64_t *lid, *oid;
    uint32_t* lnout;
    void* scratch;
    Bump sizing{nullptr};
    carve(sizing, dQ, lid, lsc, lnout, oid, osc, scratch);
    if (sizing.off > cx->dbuf_bytes) {
        if (cx->dbuf) {
            cudaStreamSynchronize(cx->st);
            cudaFree(cx->dbuf);
        }
        cx->dbuf = nullptr;
        cx->dbuf_bytes = 0;
        size_t want_b = sizing.off + sizing.off / 4;
        if (cudaMalloc(&cx->dbuf, want_b) != cudaSuccess) return cfail(cx, MAIVS_OOM, "device allocation failed");
        cx->dbuf_bytes = want_b;
    }
    Bump bp{static_cast<char*>(cx->dbuf)};
    carve(bp, dQ, lid, lsc, lnout, oid, osc, scratch);
    const size_t qb = nq * dim * sizeof(float), ob = nq * k * (sizeof(uint64_t) + sizeof(float));
    if (qb + ob > cx->pin_bytes) {
        if (cx->pin) cudaFreeHost(cx->pin);
        cx->pin = nullptr;
        cx->pin_bytes = 0;
        if (cudaMallocHost(&cx->pin, qb + ob) != cudaSuccess) return cfail(cx, MAIVS_OOM, "pinned allocation failed");
        cx->pin_bytes = qb + ob;
    }
    char* hp = static_cast<char*>(cx->pin);
    std::memcpy(hp, Q, qb);
    maivs::SearchArgs a;
    a.nq = (int)nq;
    a.k = (int)want;
    a.nprobe = (int)std::min<size_t>(nprobe, 1u << 30);
    a.tc = tc;
    a.beta = beta;
    a.cell_major = false;  // query_all runs search_one on every segment (concurrent.rs:120-129)

    for (int attempt = 0; attempt < 4; ++attempt) {
        if (cudaMemcpyAsync(dQ, hp, qb, cudaMemcpyHostToDevice, cx->st) != cudaSuccess)
            return cfail(cx, MAIVS_CUDA_ERROR, "query upload failed");
        std::vector<maivs_index*> searched;
        auto run = [&](maivs_index* seg, size_t l) -> int {
            uint64_t* li = lid + l * nq * want;
            float* ls = lsc + l * nq * want;
            uint32_t* ln = lnout + l * nq;
            if (seg->h.cells.empty() || seg->h.n_live == 0) {  // search_rust on an empty segment
                cudaMemsetAsync(ln, 0, nq * sizeof(uint32_t), cx->st);
                return MAIVS_OK;
            }
            seg->device = cx->device;
            int rc = maivs_capi::device_image(seg);
            if (rc != MAIVS_OK) return cfail(cx, rc, seg->err);
            if (cx->clock_on) seg->d->enable_kernel_clock(true);
            std::string e;
            rc = seg->d->search_device(seg->h, dQ, a, li, ls, ln, cx->st, e);
            if (rc != MAIVS_OK) return cfail(cx, rc, e);
            searched.push_back(seg);
            return MAIVS_OK;
        };
        for (size_t l = 0; l + 1 < L; ++l) {
            int rc = run(segs[l].get(), l);
            if (rc != MAIVS_OK) return rc;
        }
        {
            // the head last (concurrent.rs:125-129); its host state is read only while enqueueing
            std::shared_lock<std::shared_mutex> hl(cx->head_mu);
            int rc = run(cx->head.get(), L - 1);
            if (rc != MAIVS_OK) return rc;
        }
        {
            std::shared_lock<std::shared_mutex> dl(cx->dead_mu);
            if (cx->dead_version != cx->tomb_version) {
                std::vector<uint64_t> t(cx->dead.begin(), cx->dead.end());
                std::sort(t.begin(), t.end());
                cudaStreamSynchronize(cx->st);
                if (t.size() > cx->dtomb_cap) {
                    if (cx->dtomb) cudaFree(cx->dtomb);
                    cx->dtomb = nullptr;
                    cx->dtomb_cap = 0;
                    size_t cap = std::max<size_t>(t.size() * 2, 1024);
                    if (cudaMalloc(&cx->dtomb, cap * sizeof(uint64_t)) != cudaSuccess)
                        return cfail(cx, MAIVS_OOM, "device allocation failed");
                    cx->dtomb_cap = cap;
                }
                if (!t.empty() &&
                    cudaMemcpy(cx->dtomb, t.data(), t.size() * sizeof(uint64_t), cudaMemcpyHostToDevice) != cudaSuccess)
                    return cfail(cx, MAIVS_CUDA_ERROR, "tombstone upload failed");
                cx->ntomb = (int)t.size();
                cx->tomb_version = cx->dead_version;
            }
        }
        maivs::dev::take_launch_error(nullptr);
        maivs::dev::set_thread_clock(cx->clock_on ? cx->clock.get() : nullptr);
        maivs::dev::launch_segment_merge(lid, lsc, lnout, (int)L, (int)nq, (int)want, cx->dtomb, cx->ntomb, (int)k,
                                         scratch, oid, osc, cx->st);
        maivs::dev::set_thread_clock(nullptr);
        int kid = -1;
        cudaError_t le = maivs::dev::take_launch_error(&kid);
        if (le != cudaSuccess)
            return cfail(cx, MAIVS_CUDA_ERROR,
                         std::string("launch of ") + maivs::dev::kernel_name(kid) + " failed: " + cudaGetErrorString(le));
        // ids, then scores (separate device carves)
        if (cudaMemcpyAsync(hp + qb, oid, nq * k * sizeof(uint64_t), cudaMemcpyDeviceToHost, cx->st) != cudaSuccess ||
            cudaMemcpyAsync(hp + qb + nq * k * sizeof(uint64_t), osc, nq * k * sizeof(float), cudaMemcpyDeviceToHost,
                            cx->st) != cudaSuccess ||
            cudaStreamSynchronize(cx->st) != cudaSuccess)
            return cfail(cx, MAIVS_CUDA_ERROR, std::string("search failed: ") + cudaGetErrorString(cudaGetLastError()));
        // candidate-buffer overflows of any segment: enlarge that segment's buffers, search again
        bool again = false;
        for (maivs_index* seg : searched) {
            uint32_t f[4];
            if (seg->d->global_flags(cx->st, f) != 0)
                return cfail(cx, MAIVS_CUDA_ERROR, "reading the search flags failed");
            if (f[1] != 0)
                return cfail(cx, MAIVS_UNSUPPORTED,
                             "a routing shortlist exceeded 16384 cells; lower nprobe or the shortlist multiplier");
            if (f[2] != 0)
                return cfail(cx, MAIVS_CUDA_ERROR,
                             "a bounded wait for the GPU's copy or tensor-core engines ran out; the results are not valid");
            if (f[0] != 0) {
                seg->d->grow_factor *= 4;
                again = true;
            }
        }
        if (!again) {
            std::memcpy(ids, hp + qb, nq * k * sizeof(uint64_t));
            std::memcpy(scores, hp + qb + nq * k * sizeof(uint64_t), nq * k * sizeof(float));
            return MAIVS_OK;
        }
    }
    return cfail(cx, MAIVS_OVERFLOW, "candidate buffers overflowed after enlarging them");
}

}  // namespace

extern "C" {

int maivs_concurrent_new(size_t dim, const char* scan_mode, size_t rerank_factor, uint64_t seed, size_t code_bits,
                         size_t seal_at, maivs_concurrent** out) {
    if (!out) return MAIVS_BAD_ARG;
    *out = nullptr;
    auto cx = new (std::nothrow) maivs_concurrent();
    if (!cx) return MAIVS_OOM;
    cx->head = std::make_unique<maivs_index>();
    cx->seal_at = std::max<size_t>(seal_at, 1);
    *out = cx;
    std::string e = cx->head->h.init(dim, scan_mode ? scan_mode : "", rerank_factor, seed, code_bits);
    if (!e.empty()) return cfail(cx, MAIVS_BAD_ARG, e);  // the caller reads the message, then frees
    return MAIVS_OK;
}

void maivs_concurrent_free(maivs_concurrent* cx) { delete cx; }

const char* maivs_concurrent_last_error(maivs_concurrent* cx) {
    if (!cx) return "null handle";
    std::lock_guard<std::mutex> lk(cx->err_mu);
    return cx->err.c_str();
}

int maivs_concurrent_train_centroids(maivs_concurrent* cx, const float* v, size_t n, size_t n_cells, size_t sample,
                                     uint64_t seed) {
    if (!cx) return MAIVS_BAD_ARG;
    std::unique_lock<std::shared_mutex> hl(cx->head_mu);
    std::string e = cx->head->h.train_centroids(v, n, n_cells, sample, seed);
    return e.empty() ? MAIVS_OK : cfail(cx, MAIVS_BAD_ARG, e);
}

int maivs_concurrent_add_batch(maivs_concurrent* cx, const uint64_t* ids, const float* v, size_t n) {
    if (!cx) return MAIVS_BAD_ARG;
    {
        std::unique_lock<std::shared_mutex> hl(cx->head_mu);
        std::string e = cx->head->h.add_batch(ids, v, n);
        if (!e.empty()) return cfail(cx, MAIVS_BAD_STATE, e);
    }
    // seal outside the insert so the exclusive window stays one operation (concurrent.rs:252-259)
    bool need = false;
    {
        std::shared_lock<std::shared_mutex> hl(cx->head_mu);
        need = cx->head->h.n_live >= cx->seal_at;
    }
    if (need) {
        std::unique_lock<std::shared_mutex> hl(cx->head_mu);
        if (cx->head->h.n_live >= cx->seal_at) seal_locked(cx);
    }
    return MAIVS_OK;
}

int maivs_concurrent_remove(maivs_concurrent* cx, uint64_t id, int* removed) {
    if (!cx) return MAIVS_BAD_ARG;
    bool known = false;
    {
        std::shared_lock<std::shared_mutex> hl(cx->head_mu);
        known = cx->head->h.id_to_slot.count(id) != 0;
    }
    if (!known) {
        auto segs = snapshot(cx);
        for (auto& s : *segs)
            if (s->h.id_to_slot.count(id)) {
                known = true;
                break;
            }
    }
    bool ins = false;
    if (known) {
        std::unique_lock<std::shared_mutex> dl(cx->dead_mu);
        ins = cx->dead.insert(id).second;
        if (ins) ++cx->dead_version;
    }
    if (removed) *removed = ins ? 1 : 0;
    return MAIVS_OK;
}

int maivs_concurrent_remove_many(maivs_concurrent* cx, const uint64_t* ids, size_t n, size_t* n_removed) {
    if (!cx) return MAIVS_BAD_ARG;
    auto segs = snapshot(cx);
    std::shared_lock<std::shared_mutex> hl(cx->head_mu);
    std::unique_lock<std::shared_mutex> dl(cx->dead_mu);
    size_t cnt = 0;
    for (size_t i = 0; i < n; ++i) {
        uint64_t id = ids[i];
        bool known = cx->head->h.id_to_slot.count(id) != 0;
        for (size_t s = 0; !known && s < segs->size(); ++s) known = (*segs)[s]->h.id_to_slot.count(id) != 0;
        if (known && cx->dead.insert(id).second) ++cnt;
    }
    if (cnt) ++cx->dead_version;
    if (n_removed) *n_removed = cnt;
    return MAIVS_OK;
}

int maivs_concurrent_seal(maivs_concurrent* cx) {
    if (!cx) return MAIVS_BAD_ARG;
    std::unique_lock<std::shared_mutex> hl(cx->head_mu);
    seal_locked(cx);
    return MAIVS_OK;
}

int maivs_concurrent_purge_head(maivs_concurrent* cx, size_t* n_purged) {
    if (!cx) return MAIVS_BAD_ARG;
    std::unique_lock<std::shared_mutex> hl(cx->head_mu);
    std::unique_lock<std::shared_mutex> dl(cx->dead_mu);  // head -> dead, as elsewhere
    std::vector<uint64_t> victims;
    for (uint64_t id : cx->dead)
        if (cx->head->h.id_to_slot.count(id)) victims.push_back(id);
    // ascending id (the reference walks a hash set, whose order is unspecified)
    std::sort(victims.begin(), victims.end());
    for (uint64_t id : victims) {
        cx->head->h.remove(id);
        cx->dead.erase(id);
    }
    if (!victims.empty()) ++cx->dead_version;
    cx->head->h.compact();
    if (n_purged) *n_purged = victims.size();
    return MAIVS_OK;
}

int maivs_concurrent_compact(maivs_concurrent* cx) {
    return with_head_write(cx, [](maivs::HostIndex& h) { h.compact(); });
}
int maivs_concurrent_set_per_dim_sq(maivs_concurrent* cx, int on) {
    return with_head_write(cx, [&](maivs::HostIndex& h) { h.set_per_dim_sq(on != 0); });
}
int maivs_concurrent_set_two_stage(maivs_concurrent* cx, int on, size_t mult) {
    return with_head_write(cx, [&](maivs::HostIndex& h) { h.set_two_stage(on != 0, mult); });
}
int maivs_concurrent_set_adaptive(maivs_concurrent* cx, int on, float margin) {
    return with_head_write(cx, [&](maivs::HostIndex& h) {
        h.adaptive = on != 0;
        h.at_margin = margin;
    });
}
int maivs_concurrent_set_parallel_scan(maivs_concurrent* cx, int on) {
    if (!cx) return MAIVS_BAD_ARG;
    std::unique_lock<std::shared_mutex> hl(cx->head_mu);
    cx->par_scan = on != 0;
    return MAIVS_OK;
}
int maivs_concurrent_set_build_device(maivs_concurrent* cx, int device) {
    // kept by fork_empty, so every later head builds there too
    return with_head_write(cx, [&](maivs::HostIndex& h) { h.build_device = device < 0 ? -1 : device; });
}
int maivs_concurrent_set_graph_route(maivs_concurrent* cx, int on, size_t min_cells) {
    return with_head_write(cx, [&](maivs::HostIndex& h) {
        h.graph_route = on != 0;
        if (min_cells > 0) h.graph_min_cells = min_cells;
        ++h.version;
    });
}
int maivs_concurrent_set_tree_route(maivs_concurrent* cx, int on, size_t min_cells, size_t fanout, float beam_frac) {
    return with_head_write(cx, [&](maivs::HostIndex& h) { h.set_tree_route(on != 0, min_cells, fanout, beam_frac); });
}

int maivs_concurrent_len(maivs_concurrent* cx, size_t* n) {
    if (!cx || !n) return MAIVS_BAD_ARG;
    size_t head = 0, sealed = 0, dead = 0;
    {
        std::shared_lock<std::shared_mutex> hl(cx->head_mu);
        head = cx->head->h.n_live;
    }
    {
        std::shared_lock<std::shared_mutex> sl(cx->sealed_mu);
        sealed = cx->sealed_live;
    }
    {
        std::shared_lock<std::shared_mutex> dl(cx->dead_mu);
        dead = cx->dead.size();
    }
    *n = sealed + head > dead ? sealed + head - dead : 0;
    return MAIVS_OK;
}

int maivs_concurrent_stat(maivs_concurrent* cx, const char* name, double* value) {
    if (!cx || !name || !value) return MAIVS_BAD_ARG;
    std::string s(name);
    size_t head_live = 0, nseg = 0, sealed_live = 0, ndead = 0;
    {
        std::shared_lock<std::shared_mutex> hl(cx->head_mu);
        head_live = cx->head->h.n_live;
        if (s != "segments" && s != "head_live" && s != "sealed_live" && s != "tombstones" && s != "n_live") {
            // every other key is the head's (concurrent.rs:229-232)
            int rc = maivs_stat(cx->head.get(), name, value);
            return rc == MAIVS_OK ? rc : cfail(cx, rc, cx->head->err);
        }
    }
    {
        std::shared_lock<std::shared_mutex> sl(cx->sealed_mu);
        nseg = cx->sealed->size();
        sealed_live = cx->sealed_live;
    }
    {
        std::shared_lock<std::shared_mutex> dl(cx->dead_mu);
        ndead = cx->dead.size();
    }
    if (s == "segments") *value = (double)nseg;
    else if (s == "head_live") *value = (double)head_live;
    else if (s == "sealed_live") *value = (double)sealed_live;
    else if (s == "tombstones") *value = (double)ndead;
    else *value = (double)(sealed_live + head_live > ndead ? sealed_live + head_live - ndead : 0);
    return MAIVS_OK;
}

int maivs_concurrent_to_device(maivs_concurrent* cx, int device) {
    if (!cx) return MAIVS_BAD_ARG;
    int ndev = 0;
    if (cudaGetDeviceCount(&ndev) != cudaSuccess || ndev == 0)
        return cfail(cx, MAIVS_NO_DEVICE, "no CUDA device is visible; the MAIVS GPU search has no CPU fallback");
    if (device < 0 || device >= ndev) return cfail(cx, MAIVS_BAD_ARG, "device ordinal out of range");
    std::lock_guard<std::mutex> gl(cx->gpu_mu);
    if (cx->device != device && cx->st) {
        cudaStreamSynchronize(cx->st);
        cudaStreamDestroy(cx->st);
        cx->st = nullptr;
        if (cx->dbuf) cudaFree(cx->dbuf);
        if (cx->dtomb) cudaFree(cx->dtomb);
        cx->dbuf = nullptr;
        cx->dbuf_bytes = 0;
        cx->dtomb = nullptr;
        cx->dtomb_cap = 0;
        cx->tomb_version = ~0ull;
    }
    cx->device = device;
    cudaSetDevice(device);
    if (!cx->st && cudaStreamCreateWithFlags(&cx->st, cudaStreamNonBlocking) != cudaSuccess)
        return cfail(cx, MAIVS_CUDA_ERROR, "stream creation failed");
    return MAIVS_OK;
}

int maivs_concurrent_search_batch(maivs_concurrent* cx, const float* Q, size_t nq, size_t k, size_t nprobe, float tc,
                                  float beta, uint64_t* ids, float* scores) {
    if (!cx) return MAIVS_BAD_ARG;
    if (nq == 0) return MAIVS_OK;
    if (k == 0) return cfail(cx, MAIVS_BAD_ARG, "k must be positive");
    if (k > 4096) return cfail(cx, MAIVS_UNSUPPORTED, "k above 4096 is not supported");
    if (!Q || !ids || !scores) return cfail(cx, MAIVS_BAD_ARG, "null buffer");
    {
        int ndev = 0;
        if (cudaGetDeviceCount(&ndev) != cudaSuccess || ndev == 0)
            return cfail(cx, MAIVS_NO_DEVICE, "no CUDA device is visible; the MAIVS GPU search has no CPU fallback");
    }
    std::lock_guard<std::mutex> gl(cx->gpu_mu);
    cudaSetDevice(cx->device);
    if (!cx->st && cudaStreamCreateWithFlags(&cx->st, cudaStreamNonBlocking) != cudaSuccess)
        return cfail(cx, MAIVS_CUDA_ERROR, "stream creation failed");
    auto segs = snapshot(cx);
    size_t ndead = 0, dim = 0;
    {
        std::shared_lock<std::shared_mutex> dl(cx->dead_mu);
        ndead = cx->dead.size();
    }
    {
        std::shared_lock<std::shared_mutex> hl(cx->head_mu);
        dim = cx->head->h.dim;
    }
    // over-fetch enough to survive tombstone filtering (concurrent.rs:116-117)
    const size_t want = ndead == 0 ? k : k * kOverfetch;
    for (size_t q0 = 0; q0 < nq; q0 += kQueryChunk) {
        const size_t n = std::min(kQueryChunk, nq - q0);
        int rc = search_pass(cx, *segs, Q + q0 * dim, n, dim, k, want, nprobe, tc, beta, ids + q0 * k,
                             scores + q0 * k);
        if (rc != MAIVS_OK) return rc;
    }
    return MAIVS_OK;
}

int maivs_concurrent_search(maivs_concurrent* cx, const float* query, size_t k, size_t nprobe, float tc, float beta,
                            uint64_t* ids, float* scores, size_t* n_out) {
    int rc = maivs_concurrent_search_batch(cx, query, 1, k, nprobe, tc, beta, ids, scores);
    if (rc != MAIVS_OK) return rc;
    size_t n = 0;
    while (n < k && ids[n] != UINT64_MAX) ++n;
    if (n_out) *n_out = n;
    return MAIVS_OK;
}

int maivs_concurrent_kernel_clock(maivs_concurrent* cx, int on) {
    if (!cx) return MAIVS_BAD_ARG;
    std::lock_guard<std::mutex> gl(cx->gpu_mu);
    cx->clock_on = on != 0;
    if (cx->clock_on && !cx->clock) cx->clock = std::make_unique<maivs::dev::KernelClock>();
    if (!cx->clock_on) {
        cx->clock.reset();
        auto segs = snapshot(cx);
        for (auto& sg : *segs)
            if (sg->d) sg->d->enable_kernel_clock(false);
        std::shared_lock<std::shared_mutex> hl(cx->head_mu);
        if (cx->head->d) cx->head->d->enable_kernel_clock(false);
    }
    return MAIVS_OK;
}

int maivs_concurrent_kernel_times(maivs_concurrent* cx, int reset, const char** names, double* ms,
                                  uint64_t* launches, size_t cap, size_t* n_out) {
    if (!cx) return MAIVS_BAD_ARG;
    std::lock_guard<std::mutex> gl(cx->gpu_mu);
    std::vector<maivs::dev::KernelClock*> clocks;
    if (cx->clock) clocks.push_back(cx->clock.get());
    auto segs = snapshot(cx);
    for (auto& sg : *segs)
        if (sg->d && sg->d->kernel_clock()) clocks.push_back(sg->d->kernel_clock());
    {
        std::shared_lock<std::shared_mutex> hl(cx->head_mu);
        if (cx->head->d && cx->head->d->kernel_clock()) clocks.push_back(cx->head->d->kernel_clock());
    }
    if (cx->st) cudaStreamSynchronize(cx->st);
    for (auto* c : clocks) c->collect();
    const size_t n = std::min<size_t>(cap, maivs::dev::kNumKernels);
    if (n_out) *n_out = n;
    for (size_t i = 0; i < n; ++i) {
        double t = 0.0;
        uint64_t l = 0;
        for (auto* c : clocks) {
            t += c->ms[i];
            l += c->launches[i];
        }
        if (names) names[i] = maivs::dev::kernel_name((int)i);
        if (ms) ms[i] = t;
        if (launches) launches[i] = l;
    }
    if (reset)
        for (auto* c : clocks)
            for (size_t i = 0; i < maivs::dev::kNumKernels; ++i) {
                c->ms[i] = 0.0;
                c->launches[i] = 0;
            }
    return MAIVS_OK;
}

int maivs_concurrent_segments(maivs_concurrent* cx, size_t* n) {
    if (!cx || !n) return MAIVS_BAD_ARG;
    *n = snapshot(cx)->size();
    return MAIVS_OK;
}

int maivs_concurrent_array(maivs_concurrent* cx, long long segment, const char* name, const void** data,
                           size_t* count, size_t* elem_bytes) {
    if (!cx) return MAIVS_BAD_ARG;
    if (segment < 0) {
        std::shared_lock<std::shared_mutex> hl(cx->head_mu);
        int rc = maivs_array(cx->head.get(), name, data, count, elem_bytes);
        return rc == MAIVS_OK ? rc : cfail(cx, rc, cx->head->err);
    }
    auto segs = snapshot(cx);
    if ((size_t)segment >= segs->size()) return cfail(cx, MAIVS_NOT_FOUND, "no such segment");
    maivs_index* s = (*segs)[(size_t)segment].get();
    int rc = maivs_array(s, name, data, count, elem_bytes);
    return rc == MAIVS_OK ? rc : cfail(cx, rc, s->err);
}

}  // extern "C"
