// Per-kernel device clock, launch counter and first-launch-error record of the query kernels.
#include <algorithm>
#include <atomic>
#include <map>
#include <mutex>
#include <tuple>
#include <vector>

#include "dev_common.cuh"

namespace maivs {
namespace dev {

namespace {
thread_local KernelClock* t_clock = nullptr;
thread_local cudaError_t t_launch_err = cudaSuccess;
thread_local int t_launch_err_kernel = -1;
std::atomic<unsigned long long> g_launches{0};

}  // namespace

bool tick_begin(int id, cudaStream_t st) {
    g_launches.fetch_add(1, std::memory_order_relaxed);
    const bool timed = t_clock && t_clock->wants(id);
    if (timed) t_clock->begin(id, st);
    return timed;
}

void tick_end(int id, cudaStream_t st, bool timed) {
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess && t_launch_err == cudaSuccess) {
        t_launch_err = e;
        t_launch_err_kernel = id;
    }
    if (timed) t_clock->end(st);
}

cudaError_t take_launch_error(int* kernel) {
    cudaError_t e = t_launch_err;
    if (kernel) *kernel = t_launch_err_kernel;
    t_launch_err = cudaSuccess;
    t_launch_err_kernel = -1;
    return e;
}

const char* kernel_name(int id) {
    static const char* names[kNumKernels] = {"k_encode", "k_route_flat", "k_route_tree", "k_rescore_select",
                                             "k_seed",   "k_inv_count",  "k_inv_scan",   "k_inv_scatter",
                                             "k_scan_cm", "k_final_cm",  "k_pq_prep",    "k_pq_scan",
                                             "k_pq_fold", "k_rerank",    "k_topk",       "k_rerank_items",
                                             "k_seed_finish", "k_local_list", "k_merge_topk", "k_scan_mma",
                                             "k_seed_scan", "nccl_all_gather", "k_segment_merge", "k_rescore_dots", "k_probe_select"};
    return id >= 0 && id < kNumKernels ? names[id] : "?";
}

KernelClock::~KernelClock() {
    for (auto& m : pending) {
        cudaEventDestroy(m.a);
        cudaEventDestroy(m.b);
    }
    for (auto e : pool) cudaEventDestroy(e);
}

cudaEvent_t KernelClock::take() {
    if (!pool.empty()) {
        cudaEvent_t e = pool.back();
        pool.pop_back();
        return e;
    }
    cudaEvent_t e = nullptr;
    cudaEventCreate(&e);
    return e;
}

void KernelClock::begin(int id, cudaStream_t st) {
    Mark m{id, take(), take()};
    cudaEventRecord(m.a, st);
    pending.push_back(m);
    launches[id] += 1;
}

void KernelClock::end(cudaStream_t st) {
    if (!pending.empty()) cudaEventRecord(pending.back().b, st);
}

void KernelClock::collect() {
    // every mark's interval against one origin event (the first pending mark's start; others may
    // start before it on another stream, giving negative offsets), merged per kernel into busy time
    std::vector<std::vector<std::pair<float, float>>> iv(kNumKernels);
    cudaEvent_t origin = nullptr;
    for (auto& m : pending) {
        float t = 0.0f;
        if (cudaEventSynchronize(m.b) == cudaSuccess && cudaEventElapsedTime(&t, m.a, m.b) == cudaSuccess) {
            ms[m.id] += t;
            if (!origin) origin = m.a;
            float s0 = 0.0f, s1 = 0.0f;
            if (cudaEventElapsedTime(&s0, origin, m.a) == cudaSuccess &&
                cudaEventElapsedTime(&s1, origin, m.b) == cudaSuccess)
                iv[m.id].push_back({s0, s1});
            else
                busy[m.id] += t;
        }
    }
    for (int id = 0; id < kNumKernels; ++id) {
        auto& v = iv[id];
        std::sort(v.begin(), v.end());
        float lo = 0.0f, hi = 0.0f;
        bool open = false;
        for (const auto& x : v) {
            if (open && x.first <= hi) {
                hi = std::max(hi, x.second);
                continue;
            }
            if (open) busy[id] += hi - lo;
            lo = x.first;
            hi = x.second;
            open = true;
        }
        if (open) busy[id] += hi - lo;
    }
    for (auto& m : pending) {
        pool.push_back(m.a);
        pool.push_back(m.b);
    }
    pending.clear();
}

void set_thread_clock(KernelClock* c) { t_clock = c; }
void clock_begin(int id, cudaStream_t st) {
    if (t_clock && t_clock->wants(id)) t_clock->begin(id, st);
}
void clock_end(int id, cudaStream_t st) {
    if (t_clock && t_clock->wants(id)) t_clock->end(st);
}
unsigned long long total_launches() { return g_launches.load(); }

// The attribute and occupancy queries cost host time on every launch of a search; their answers
// only change with the device, so they are remembered per (device, kernel).
namespace {
std::mutex g_attr_mu;
std::map<std::pair<int, const void*>, size_t> g_smem_set;
std::map<std::tuple<int, const void*, int, size_t>, int> g_occ;
int cur_device() {
    int dev = 0;
    cudaGetDevice(&dev);
    return dev;
}
}  // namespace

void set_smem(const void* f, size_t bytes) {
    if (bytes == 0) return;
    const auto key = std::make_pair(cur_device(), f);
    std::lock_guard<std::mutex> lk(g_attr_mu);
    auto it = g_smem_set.find(key);
    if (it != g_smem_set.end() && it->second >= bytes) return;
    if (cudaFuncSetAttribute(f, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)bytes) == cudaSuccess)
        g_smem_set[key] = bytes;
}

int blocks_per_sm(const void* f, int threads, size_t smem) {
    const auto key = std::make_tuple(cur_device(), f, threads, smem);
    {
        std::lock_guard<std::mutex> lk(g_attr_mu);
        auto it = g_occ.find(key);
        if (it != g_occ.end()) return it->second;
    }
    int per_sm = 1;
    if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, f, threads, smem) != cudaSuccess || per_sm < 1)
        per_sm = 1;
    std::lock_guard<std::mutex> lk(g_attr_mu);
    g_occ[key] = per_sm;
    return per_sm;
}

int sm_count() {
    const int dev = cur_device();
    static std::mutex mu;
    static std::map<int, int> cache;
    std::lock_guard<std::mutex> lk(mu);
    auto it = cache.find(dev);
    if (it != cache.end()) return it->second;
    int sms = 148;
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    cache[dev] = sms;
    return sms;
}

}  // namespace dev
}  // namespace maivs
