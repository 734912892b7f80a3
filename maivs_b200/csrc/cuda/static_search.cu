// Allocation-free small-batch search.
//
// Some callers cannot allocate device memory while they serve queries: a process whose GPU
// memory has already been reserved by another runtime's pool (frameworks that pre-allocate most
// of the device), or a latency-critical serving loop that must not pay cudaMalloc's implicit
// device-wide synchronisation and unpredictable latency. For them this file runs the per-query
// search pipeline (the same kernels as search_batch with cell_major = false) with all of its
// scratch carved from one file-scope device array of kStaticScratchBytes. A GPU holds that array
// from the first allocation-free call made on it (under CUDA's lazy module loading the module,
// and with it the array, is loaded on that device when the first call looks the address up)
// until the process exits.
//
// The array's address is fetched with cudaGetSymbolAddress once per device, on the first call
// made with that device current (so that first call should come before any stream capture). The
// address is cached per device ordinal, so a device whose context is reset must not serve this
// path again in the same process.
// All calls share the array and it keeps the previous call's contents; no part of it has to
// start at zero (every kernel writes what it later reads), but two calls whose work overlaps on
// the GPU race on it, so a caller must serialise them (one stream, or one call at a time).
#include <mutex>
#include <unordered_map>

#include "engine.h"

namespace maivs {

namespace {

constexpr size_t kStaticScratchBytes = size_t(32) << 20;  // 32 MiB
constexpr int kStaticMaxQueries = 64;

__device__ __align__(256) unsigned char g_static_scratch[kStaticScratchBytes];

std::mutex g_addr_mu;
std::unordered_map<int, void*> g_addr;  // device ordinal -> device address of g_static_scratch

// Device address of the scratch array on the current device (set up once per device).
int static_scratch(int device, void** out, std::string& err) {
    std::lock_guard<std::mutex> lk(g_addr_mu);
    auto it = g_addr.find(device);
    if (it != g_addr.end()) {
        *out = it->second;
        return kOk;
    }
    void* p = nullptr;
    cudaError_t e = cudaGetSymbolAddress(&p, g_static_scratch);
    if (e != cudaSuccess || p == nullptr) {
        err = std::string("cudaGetSymbolAddress of the static scratch failed: ") + cudaGetErrorString(e);
        return kCudaError;
    }
    g_addr[device] = p;
    *out = p;
    return kOk;
}

struct Carve {
    char* base;
    size_t off = 0;
    template <typename T>
    T* take(size_t n) {
        size_t a = (off + 255) & ~size_t(255);
        off = a + n * sizeof(T);
        return base ? reinterpret_cast<T*>(base + a) : nullptr;
    }
};

}  // namespace

int DeviceIndex::search_static(const HostIndex& h, const float* dQ, const SearchArgs& a, uint64_t* d_ids,
                               float* d_scores, cudaStream_t st, std::string& err) {
    if (h.version != version_) {
        err = "the index changed since it was uploaded; call maivs_to_device() first";
        return kBadState;
    }
    if (a.k <= 0 || a.nq <= 0) {
        err = "nq and k must be positive";
        return kBadArg;
    }
    if (a.nq > kStaticMaxQueries) {
        err = "the allocation-free search takes at most 64 queries per call";
        return kBadArg;
    }
    cudaSetDevice(device_);
    if (!st) st = stream_;
    const int nq = a.nq, M = view_.M, dim = view_.dim, nw = view_.nw, npos = view_.npos;
    const int nprobe = std::max(1, std::min(a.nprobe, M));
    const int want0 = (int)((size_t)a.k * h.rerank_factor);
    const size_t ent_need = (size_t)nprobe * max_members_ + 1;
    if (ent_need > (size_t)1 << 30) {
        err = "nprobe x largest cell is too large for the allocation-free search";
        return kBadArg;
    }
    const int ent_cap = (int)ent_need;
    // the Hamming scan keeps every tie at its cut-off: room for every scanned member
    const int cand_cap = view_.ham ? ent_cap : std::max(want0, 1);
    const bool filtering = h.has_filter && !h.tags.empty();
    const bool tree_router = h.tree != nullptr;

    dev::QueryEnc e{};
    dev::PerQueryBufs b{};
    uint32_t *sl, *sl_n, *tsc, *chosen, *nch, *nout, *ritem, *rsi;
    float* rss;
    uint16_t* hs;
    float *cscore, *rsc;
    auto carve = [&](Carve& c) {
        e.qbits = c.take<uint64_t>((size_t)nq * nw);
        e.lut = c.take<uint8_t>((size_t)nq * npos * 16);
        e.fs_delta = c.take<float>(nq);
        e.fs_bias = c.take<float>(nq);
        e.cqs = c.take<float>((size_t)nq * dim);
        e.cqbase = c.take<float>(nq);
        e.rqs = c.take<float>((size_t)nq * dim);
        e.rbase = c.take<float>(nq);
        sl = c.take<uint32_t>((size_t)nq * M);
        sl_n = c.take<uint32_t>(nq);
        hs = c.take<uint16_t>((size_t)nq * M);
        tsc = tree_router ? c.take<uint32_t>((size_t)nq * 3 * tree_cap_) : nullptr;
        rss = c.take<float>((size_t)nq * M);
        rsi = c.take<uint32_t>((size_t)nq + 1);
        chosen = c.take<uint32_t>((size_t)nq * nprobe);
        cscore = c.take<float>((size_t)nq * nprobe);
        nch = c.take<uint32_t>(nq);
        b.crank = c.take<uint32_t>((size_t)nq * M);
        b.seg_off = c.take<uint32_t>((size_t)nq * (nprobe + 1));
        b.ent_cap = ent_cap;
        b.ent = c.take<uint64_t>((size_t)nq * ent_cap);
        b.cand_cap = cand_cap;
        b.cand = c.take<uint32_t>((size_t)nq * cand_cap);
        b.cand_n = c.take<uint32_t>(nq);
        b.overflow = d_flags_;
        rsc = c.take<float>((size_t)nq * cand_cap);
        nout = c.take<uint32_t>(nq);
        ritem = c.take<uint32_t>((size_t)nq + 1);
    };
    Carve sizing{nullptr};
    carve(sizing);
    if (sizing.off > kStaticScratchBytes) {
        err = "this search needs " + std::to_string(sizing.off) + " bytes of scratch; the allocation-free search has " +
              std::to_string(kStaticScratchBytes) + " (lower nq or nprobe)";
        return kBadArg;
    }
    void* base = nullptr;
    int rc = static_scratch(device_, &base, err);
    if (rc != kOk) return rc;
    Carve c{static_cast<char*>(base)};
    carve(c);

    dev::take_launch_error(nullptr);
    cudaMemsetAsync(d_flags_, 0, 4 * sizeof(uint32_t), st);
    dev::launch_encode(view_, dQ, nq, e, use_sq8_, view_.rerank_mode == 1, st);
    rc = route(h, e, dQ, nq, nprobe, a.tc, a.beta, false, hs, sl, sl_n, tsc, rss, rsi, chosen, cscore, nch, st, err);
    if (rc != kOk) return rc;
    dev::launch_perquery(view_, e, nq, chosen, cscore, nch, nprobe, want0, h.adaptive, h.at_margin, filtering,
                         h.filter_lo, h.filter_hi, b, st);
    dev::launch_rerank(view_, dQ, e, nq, b.cand, b.cand_n, cand_cap, a.k, d_ids, d_scores, nout, rsc, ritem,
                       d_flags_ + 2, st);
    int kid = -1;
    cudaError_t le = dev::take_launch_error(&kid);
    if (le != cudaSuccess) {
        err = std::string("launch of ") + dev::kernel_name(kid) + " failed: " + cudaGetErrorString(le);
        return kCudaError;
    }
    return kOk;
}

}  // namespace maivs
