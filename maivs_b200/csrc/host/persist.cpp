// save / load in the reference's on-disk format "MAIVS2\0\1" (src/persist.rs:28-281), so files
// written by either implementation load in the other: little-endian, a 16-word header, four f32
// settings, length-prefixed raw blocks, then the cells. Derived state (id map, rotation signs,
// centroid codes, SQ8 centroids, tree) is rebuilt on load, and a loaded index is not compacted, as
// in the reference (persist.rs:192-280, index.rs:1116-1124).
#include <cstdio>
#include <cstring>
#include <memory>
#include <string>
#include <unordered_set>

#include "hostmath.h"
#include "index_host.h"

namespace maivs {

namespace {

constexpr char kMagic[8] = {'M', 'A', 'I', 'V', 'S', '2', '\0', '\x01'};

struct File {
    FILE* f = nullptr;
    ~File() {
        if (f) fclose(f);
    }
};

bool put(FILE* f, const void* p, size_t n) { return n == 0 || fwrite(p, 1, n, f) == n; }
bool get(FILE* f, void* p, size_t n) { return n == 0 || fread(p, 1, n, f) == n; }

template <typename T>
bool put_pod(FILE* f, const std::vector<T>& v) {
    const uint64_t n = v.size();
    return put(f, &n, 8) && put(f, v.data(), n * sizeof(T));
}

template <typename T>
bool get_pod(FILE* f, std::vector<T>& v) {
    uint64_t n = 0;
    if (!get(f, &n, 8)) return false;
    if (n > (uint64_t(1) << 40) / sizeof(T)) return false;  // a corrupt length, not an allocation
    v.resize((size_t)n);
    return get(f, v.data(), (size_t)n * sizeof(T));
}

}  // namespace

std::string save_index(const HostIndex& h, const std::string& path) {
    File fh;
    fh.f = fopen(path.c_str(), "wb");
    if (!fh.f) return "cannot open '" + path + "' for writing";
    FILE* f = fh.f;
    const uint64_t hdr[16] = {h.dim,
                              2,  // scan mode: binary (the only one this engine serves)
                              h.rerank_factor,
                              h.dim_pad,
                              h.nw,
                              h.seed,
                              h.n_live,
                              h.max_assign,
                              h.shortlist_mult,
                              h.i8_rerank ? 1u : 0u,
                              h.keep_f32 ? 1u : 0u,
                              h.adaptive ? 1u : 0u,
                              h.two_stage ? 1u : 0u,
                              h.tree_route ? 1u : 0u,
                              h.tree_min_cells,
                              h.tree_fanout};
    const float fl[4] = {h.quant_scale, h.spill_margin, h.at_margin, h.tree_beam_frac};
    const std::vector<uint16_t> no_f16;  // f16 rerank rows are not kept by this engine
    bool ok = put(f, kMagic, 8) && put(f, hdr, sizeof(hdr)) && put(f, fl, sizeof(fl)) && put_pod(f, h.bits) &&
              put_pod(f, h.scan_i8) && put_pod(f, no_f16) && put_pod(f, h.sq_min) && put_pod(f, h.sq_step) &&
              put_pod(f, h.vecs_f32) && put_pod(f, h.ext_ids) && put_pod(f, h.slot_cell) &&
              put_pod(f, h.free_slots) && put_pod(f, h.slot_cells) && put_pod(f, h.tags);
    const uint64_t nc = h.cells.size();
    ok = ok && put(f, &nc, 8);
    for (size_t c = 0; ok && c < h.cells.size(); ++c) {
        const Cell& cell = h.cells[c];
        ok = put_pod(f, cell.members) && put_pod(f, cell.sum) && put_pod(f, cell.centroid) &&
             put(f, &cell.r_bound, 4) && put(f, &cell.r_max, 4);
    }
    if (!ok) return "write to '" + path + "' failed";
    if (fflush(f) != 0) return "write to '" + path + "' failed";
    return "";
}

std::string load_index(const std::string& path, HostIndex& h) {
    File fh;
    fh.f = fopen(path.c_str(), "rb");
    if (!fh.f) return "cannot open '" + path + "'";
    FILE* f = fh.f;
    char magic[8];
    if (!get(f, magic, 8) || std::memcmp(magic, kMagic, 8) != 0)
        return "not a MAIVS v2 index file (bad magic or format version)";
    uint64_t hdr[16];
    float fl[4];
    if (!get(f, hdr, sizeof(hdr)) || !get(f, fl, sizeof(fl))) return "truncated index file";
    if (hdr[1] != 2) return "only scan_mode 'binary' indexes are served by the GPU search";
    HostIndex x;
    x.dim = hdr[0];
    x.rerank_factor = hdr[2];
    x.dim_pad = hdr[3];
    x.nw = hdr[4];
    x.seed = hdr[5];
    x.n_live = hdr[6];
    x.max_assign = hdr[7];
    x.shortlist_mult = hdr[8];
    x.i8_rerank = hdr[9] != 0;
    x.keep_f32 = hdr[10] != 0;
    x.adaptive = hdr[11] != 0;
    x.two_stage = hdr[12] != 0;
    x.tree_route = hdr[13] != 0;
    x.tree_min_cells = hdr[14];
    x.tree_fanout = hdr[15];
    x.quant_scale = fl[0];
    x.spill_margin = fl[1];
    x.at_margin = fl[2];
    x.tree_beam_frac = fl[3];
    if (x.dim == 0 || x.dim_pad < x.dim || x.nw == 0 || x.nw * 64 > x.dim_pad) return "corrupt index header";
    std::vector<uint16_t> f16;
    bool ok = get_pod(f, x.bits) && get_pod(f, x.scan_i8) && get_pod(f, f16) && get_pod(f, x.sq_min) &&
              get_pod(f, x.sq_step) && get_pod(f, x.vecs_f32) && get_pod(f, x.ext_ids) && get_pod(f, x.slot_cell) &&
              get_pod(f, x.free_slots) && get_pod(f, x.slot_cells) && get_pod(f, x.tags);
    if (!ok) return "truncated index file";
    if (!f16.empty()) return "f16 rerank rows are not served by the GPU search";
    uint64_t nc = 0;
    if (!get(f, &nc, 8) || nc > (uint64_t(1) << 32)) return "truncated index file";
    x.cells.resize((size_t)nc);
    for (auto& cell : x.cells) {
        if (!get_pod(f, cell.members) || !get_pod(f, cell.sum) || !get_pod(f, cell.centroid) ||
            !get(f, &cell.r_bound, 4) || !get(f, &cell.r_max, 4))
            return "truncated index file";
    }
    const size_t slots = x.ext_ids.size();
    if (x.bits.size() != slots * x.nw || x.slot_cells.size() != slots * x.max_assign)
        return "corrupt index file (array sizes disagree)";
    for (const auto& cell : x.cells)
        for (uint32_t m : cell.members)
            if (m >= slots) return "corrupt index file (member slot out of range)";
    // state the file does not hold, as the reference's load sets it (persist.rs:210-277)
    x.per_dim_sq = !x.sq_min.empty();
    x.centroid_sq8 = true;
    x.graph_route = true;
    x.spill_lambda = 0.0f;
    x.fastscan = false;
    x.compacted = false;
    x.signs = make_signs(x.dim_pad, x.seed);
    std::unordered_set<uint32_t> free(x.free_slots.begin(), x.free_slots.end());
    for (size_t s = 0; s < slots; ++s)
        if (!free.count((uint32_t)s)) x.id_to_slot[x.ext_ids[s]] = (uint32_t)s;
    if (x.two_stage) x.rebuild_centroid_codes();
    if (x.centroid_sq8) x.rebuild_centroid_sq8();
    x.rebuild_centroid_tree();
    x.version = h.version + 1;
    h = std::move(x);
    return "";
}

}  // namespace maivs
