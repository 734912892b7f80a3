// Host-side index build: train_centroids, add_batch (placement + orthogonal polysemy), compact,
// and the derived routing state the GPU search reads (src/index.rs).
//
// Parallel loops use OpenMP where the reference uses rayon; every parallel result is independent
// of the thread count, exactly as in the reference (per-item work, sums in input order).
//
// Tie order: where the reference sorts (score, id) pairs with an unstable sort
// (select_nth_unstable_by / sort_unstable_by), exactly equal scores are ordered by ascending
// cell id here, so the build is deterministic.
#include <omp.h>

#include <algorithm>
#include <cmath>
#include <numeric>

#include "hostmath.h"
#include "index_host.h"

namespace maivs {

namespace {
// Descending score, ascending id on exact ties.
inline bool score_desc(const std::pair<uint32_t, float>& a, const std::pair<uint32_t, float>& b) {
    if (a.second != b.second) return a.second > b.second;
    return a.first < b.first;
}
inline float clampf(float x, float lo, float hi) { return x < lo ? lo : (x > hi ? hi : x); }
}  // namespace

std::string HostIndex::init(size_t d, const std::string& scan_mode, size_t rf, uint64_t sd, size_t code_bits) {
    // index.rs:2672-2755
    if (scan_mode != "f32" && scan_mode != "i8" && scan_mode != "binary")
        return "scan_mode must be 'f32', 'i8' or 'binary', got '" + scan_mode + "'";
    if (scan_mode != "binary")
        return "scan_mode '" + scan_mode + "' is not served by the GPU search; use 'binary'";
    if (d == 0) return "dim must be positive";
    dim = d;
    rerank_factor = std::max<size_t>(rf, 1);
    dim_pad = pad_dim(d);
    nw = code_words(code_bits, dim_pad);
    seed = sd;
    signs = make_signs(dim_pad, sd);
    return "";
}

size_t HostIndex::live_cell_count() const {
    size_t c = 0;
    for (auto& cell : cells) c += !cell.members.empty();
    return c;
}

std::string HostIndex::train_centroids(const float* data, size_t n_all, size_t n_cells, size_t sample, uint64_t sd) {
    // index.rs:2761-2804
    if (n_all == 0) return "no training vectors";
    std::vector<float> train;
    size_t n_train;
    if (sample > 0 && n_all > sample) {
        size_t stride = n_all / sample;
        train.resize(sample * dim);
        for (size_t i = 0; i < sample; ++i) {
            size_t s = std::min(i * stride, n_all - 1);
            std::copy(data + s * dim, data + (s + 1) * dim, train.begin() + i * dim);
        }
        n_train = sample;
    } else {
        train.assign(data, data + n_all * dim);
        n_train = n_all;
    }
    std::vector<float> cents = hierarchical_kmeans(train.data(), n_train, dim, n_cells, sd, build_device,
                                                   &build_gpu_failures);
    size_t m = cents.size() / dim;
    for (size_t c = 0; c < m; ++c) normalize(cents.data() + c * dim, dim);
    cells.clear();
    cells.resize(m);
    for (size_t c = 0; c < m; ++c) {
        cells[c].sum.assign(dim, 0.0f);
        cells[c].centroid.assign(cents.begin() + c * dim, cents.begin() + (c + 1) * dim);
    }
    ++version;
    refresh_derived();
    return "";
}

std::string HostIndex::set_centroids(const float* cents, size_t m) {
    // index.rs:2806-2821
    cells.clear();
    cells.resize(m);
    for (size_t c = 0; c < m; ++c) {
        cells[c].sum.assign(dim, 0.0f);
        cells[c].centroid.assign(cents + c * dim, cents + (c + 1) * dim);
    }
    ++version;
    refresh_derived();
    return "";
}

void HostIndex::set_tree_route(bool on, size_t min_cells, size_t fanout, float beam_frac) {
    // index.rs:2839-2851
    if (beam_frac > 0.0f) tree_beam_frac = beam_frac;
    tree_route = on;
    if (min_cells > 0) tree_min_cells = min_cells;
    if (fanout > 1) tree_fanout = fanout;
    ++version;
    rebuild_centroid_tree();
}

void HostIndex::set_two_stage(bool on, size_t mult) {
    // index.rs:2882-2888
    two_stage = on;
    shortlist_mult = std::max<size_t>(mult, 1);
    if (on) rebuild_centroid_codes();
    ++version;
}

void HostIndex::set_centroid_sq8(bool on) {
    centroid_sq8 = on;
    if (on)
        rebuild_centroid_sq8();
    else
        cent_sq8.clear();
    ++version;
}

void HostIndex::set_per_dim_sq(bool on) {
    // index.rs:2908-2915
    per_dim_sq = on;
    if (on) {
        i8_rerank = true;
        keep_f32 = false;
    }
    ++version;
}

void HostIndex::set_i8_rerank(bool on) {
    // index.rs:2828-2833
    i8_rerank = on;
    keep_f32 = !on;
    ++version;
}

void HostIndex::set_orthogonal_polysemy(size_t homes, float lam) {
    // index.rs:2979-2984
    max_assign = std::max<size_t>(homes, 1);
    spill_margin = 0.0f;
    spill_lambda = std::max(lam, 1e-6f);
    ++version;
}

void HostIndex::set_replication(size_t ma, float margin) {
    max_assign = std::max<size_t>(ma, 1);
    spill_margin = std::max(margin, 0.0f);
    spill_lambda = 0.0f;
    ++version;
}

void HostIndex::set_fastscan(bool on) {
    // index.rs:2962-2968
    fastscan = on;
    if (!on) {
        fs_codes.clear();
        fs_off.clear();
    }
    ++version;
}

std::string HostIndex::set_tags(const uint64_t* ids, const uint32_t* tg, size_t n) {
    // index.rs:3535-3548
    if (tags.size() < ext_ids.size()) tags.resize(ext_ids.size(), 0);
    for (size_t i = 0; i < n; ++i) {
        auto it = id_to_slot.find(ids[i]);
        if (it != id_to_slot.end()) tags[it->second] = tg[i];
    }
    ++version;
    return "";
}

void HostIndex::rebuild_centroid_codes() {
    // index.rs:704-717
    std::vector<float> rot(dim_pad);
    cent_bits.assign(cells.size() * nw, 0);
    for (size_t c = 0; c < cells.size(); ++c) {
        rotate(cells[c].centroid.data(), dim, signs.data(), dim_pad, rot.data());
        pack_signs_trunc(rot.data(), dim_pad, &cent_bits[c * nw], nw);
    }
}

void HostIndex::rebuild_centroid_sq8() {
    // index.rs:724-775: range fitted over live centroids only
    std::vector<float> lo(dim, INFINITY), hi(dim, -INFINITY);
    bool any = false;
    for (auto& c : cells) {
        if (c.members.empty()) continue;
        any = true;
        for (size_t j = 0; j < dim; ++j) {
            float v = c.centroid[j];
            if (v < lo[j]) lo[j] = v;
            if (v > hi[j]) hi[j] = v;
        }
    }
    if (!any) {
        cent_sq8.clear();
        csq_min.clear();
        csq_step.clear();
        return;
    }
    csq_step.resize(dim);
    for (size_t j = 0; j < dim; ++j) {
        float s = (hi[j] - lo[j]) / 255.0f;
        csq_step[j] = s > 1e-12f ? s : 1e-12f;
    }
    csq_min = lo;
    cent_sq8.assign(cells.size() * dim, 0);
    for (size_t c = 0; c < cells.size(); ++c)
        for (size_t j = 0; j < dim; ++j)
            cent_sq8[c * dim + j] = quant_u8((cells[c].centroid[j] - csq_min[j]) / csq_step[j]);
}

void HostIndex::recompute_radii() {
    // index.rs:817-861 (f16 rerank is not supported, so its branch is absent)
    float inv = quant_scale > 0.0f ? 1.0f / quant_scale : 1.0f;
#pragma omp parallel for schedule(dynamic, 16)
    for (long long ci = 0; ci < (long long)cells.size(); ++ci) {
        Cell& cell = cells[ci];
        if (cell.members.empty()) {
            cell.r_bound = 0.0f;
            cell.r_max = 0.0f;
            continue;
        }
        const float* mu = cell.centroid.data();
        std::vector<float> w;
        float base = 0.0f;
        if (per_dim_sq) {
            w.resize(dim);
            for (size_t j = 0; j < dim; ++j) w[j] = sq_step[j] * mu[j];
            for (size_t j = 0; j < dim; ++j) base += sq_min[j] * mu[j];
        }
        std::vector<float> angs;
        angs.reserve(cell.members.size());
        for (uint32_t slot : cell.members) {
            size_t off = (size_t)slot * dim;
            float dot;
            if (per_dim_sq)
                dot = dot_f32_u8(w.data(), (const uint8_t*)&scan_i8[off], dim) + base;
            else if (keep_f32)
                dot = dot_f32(mu, &vecs_f32[off], dim);
            else
                dot = dot_f32_i8(mu, &scan_i8[off], dim) * inv;
            angs.push_back(std::acos(clampf(dot, -1.0f, 1.0f)));
        }
        size_t len = angs.size();
        size_t p99 = (size_t)std::ceil((float)len * 0.99f);
        p99 = p99 > 0 ? p99 - 1 : 0;
        p99 = std::min(p99, len - 1);
        float r_max = -INFINITY;
        for (float a : angs) r_max = std::fmax(r_max, a);
        std::nth_element(angs.begin(), angs.begin() + p99, angs.end());
        cell.r_bound = angs[p99];
        cell.r_max = r_max;
    }
}

void HostIndex::rebuild_centroid_tree() {
    // index.rs:672-700
    tree_cells = live_cell_count();
    std::vector<uint32_t> live;
    for (size_t i = 0; i < cells.size(); ++i)
        if (!cells[i].members.empty()) live.push_back((uint32_t)i);
    if (live.empty() && !cells.empty())
        for (size_t i = 0; i < cells.size(); ++i) live.push_back((uint32_t)i);
    if (!tree_route || live.size() < tree_min_cells) {
        tree.reset();
        return;
    }
    std::vector<float> flat(live.size() * dim);
    for (size_t i = 0; i < live.size(); ++i)
        std::copy(cells[live[i]].centroid.begin(), cells[live[i]].centroid.end(), flat.begin() + i * dim);
    tree = build_centroid_tree(flat.data(), live.data(), live.size(), dim, signs.data(), dim_pad, nw, tree_fanout,
                               tree_beam_frac, build_device, &build_gpu_failures);
}

void HostIndex::maybe_rebuild_centroid_tree() {
    // index.rs:651-663
    size_t live = live_cell_count();
    if (tree && tree_cells == live) return;
    rebuild_centroid_tree();
}

void HostIndex::refresh_derived() {
    // index.rs:864-878 (the centroid HNSW is never built: graph routing is off in every preset)
    recompute_radii();
    if (two_stage) rebuild_centroid_codes();
    if (centroid_sq8) rebuild_centroid_sq8();
    maybe_rebuild_centroid_tree();
}

std::vector<uint32_t> HostIndex::pick_orthogonal(std::vector<std::pair<uint32_t, float>>& scored) const {
    // index.rs:2523-2560
    const size_t kPool = 16;
    std::sort(scored.begin(), scored.end(), score_desc);
    if (scored.size() > kPool) scored.resize(kPool);
    size_t r = std::min(max_assign, scored.size());
    std::vector<std::pair<uint32_t, float>> homes{scored[0]};
    std::vector<bool> taken(scored.size(), false);
    taken[0] = true;
    while (homes.size() < r) {
        size_t best_j = SIZE_MAX;
        float best_l = INFINITY;
        for (size_t j = 0; j < scored.size(); ++j) {
            if (taken[j]) continue;
            uint32_t cj = scored[j].first;
            float sj = scored[j].second;
            float loss = 2.0f - 2.0f * sj;
            for (auto& h : homes) {
                float sh = h.second;
                float rn = std::sqrt(std::max(2.0f - 2.0f * sh, 1e-12f));
                float g = dot_f32(cells[h.first].centroid.data(), cells[cj].centroid.data(), dim);
                float p = (1.0f - sh - sj + g) / rn;
                loss += spill_lambda * p * p;
            }
            if (loss < best_l) {
                best_l = loss;
                best_j = j;
            }
        }
        if (best_j == SIZE_MAX) break;
        taken[best_j] = true;
        homes.push_back(scored[best_j]);
    }
    std::vector<uint32_t> out;
    for (auto& h : homes) out.push_back(h.first);
    return out;
}

std::vector<uint32_t> HostIndex::assign_cells(const float* v) const {
    // index.rs:2485-2512
    std::vector<std::pair<uint32_t, float>> scored(cells.size());
    for (size_t i = 0; i < cells.size(); ++i) scored[i] = {(uint32_t)i, dot_f32(v, cells[i].centroid.data(), dim)};
    if (max_assign <= 1) {
        std::pair<uint32_t, float> best{0u, -INFINITY};
        for (auto& s : scored)
            if (s.second > best.second) best = s;
        return {best.first};
    }
    if (spill_lambda > 0.0f) return pick_orthogonal(scored);
    std::sort(scored.begin(), scored.end(), score_desc);
    size_t r = std::min(max_assign, scored.size());
    scored.resize(r);
    float cutoff = scored[0].second - spill_margin;
    std::vector<uint32_t> out;
    for (auto& s : scored)
        if (s.second >= cutoff) out.push_back(s.first);
    return out;
}

std::vector<uint32_t> HostIndex::assign_cells_routed(const float* v, std::vector<float>& rot, std::vector<uint64_t>& qb,
                                                     std::vector<uint32_t>& out) const {
    // index.rs:2442-2483
    if (!tree) return assign_cells(v);
    rotate(v, dim, signs.data(), dim_pad, rot.data());
    pack_signs_trunc(rot.data(), dim_pad, qb.data(), nw);
    size_t want = std::max(kAssignCandidates, max_assign * 8);
    tree->search(qb.data(), want, out);
    if (out.empty()) return assign_cells(v);
    std::vector<std::pair<uint32_t, float>> scored;
    scored.reserve(out.size());
    for (uint32_t ci : out) scored.push_back({ci, dot_f32(v, cells[ci].centroid.data(), dim)});
    if (max_assign <= 1) {
        auto best = scored[0];
        for (auto& s : scored)
            if (s.second > best.second) best = s;
        return {best.first};
    }
    if (spill_lambda > 0.0f) return pick_orthogonal(scored);
    std::sort(scored.begin(), scored.end(), score_desc);
    size_t r = std::min(max_assign, scored.size());
    scored.resize(r);
    float cutoff = scored[0].second - spill_margin;
    std::vector<uint32_t> res;
    for (auto& s : scored)
        if (s.second >= cutoff) res.push_back(s.first);
    return res;
}

void HostIndex::encode_i8(const float* v, int8_t* out) const {
    // per-dimension SQ8 (index.rs:2612-2617) or global-scale int8 (index.rs:2619-2621)
    if (per_dim_sq) {
        for (size_t j = 0; j < dim; ++j) out[j] = (int8_t)quant_u8((v[j] - sq_min[j]) / sq_step[j]);
    } else {
        for (size_t j = 0; j < dim; ++j) out[j] = quant_i8(v[j] * quant_scale);
    }
}

void HostIndex::append_parallel(const uint64_t* ids, const float* data, size_t n,
                                const std::vector<std::vector<uint32_t>>& asg, const uint64_t* codes) {
    // index.rs:2566-2667
    size_t base = ext_ids.size();
    bool store_i8 = i8_rerank;
    if (keep_f32) vecs_f32.insert(vecs_f32.end(), data, data + n * dim);
    bits.resize((base + n) * nw, 0);
    if (codes) std::copy(codes, codes + n * nw, bits.begin() + base * nw);  // computed on the build GPU
    if (!codes) {
#pragma omp parallel
        {
            std::vector<float> rot(dim_pad);
#pragma omp for schedule(static)
            for (long long i = 0; i < (long long)n; ++i) {
                rotate(data + (size_t)i * dim, dim, signs.data(), dim_pad, rot.data());
                pack_signs_trunc(rot.data(), dim_pad, &bits[(base + i) * nw], nw);
            }
        }
    }
    if (store_i8) {
        scan_i8.resize((base + n) * dim, 0);
#pragma omp parallel for schedule(static)
        for (long long i = 0; i < (long long)n; ++i) encode_i8(data + (size_t)i * dim, &scan_i8[(base + i) * dim]);
    }
    size_t ma = max_assign;
    ext_ids.insert(ext_ids.end(), ids, ids + n);
    for (size_t i = 0; i < n; ++i) slot_cell.push_back(asg[i][0]);
    for (size_t i = 0; i < n; ++i)
        for (size_t j = 0; j < ma; ++j) slot_cells.push_back(j < asg[i].size() ? asg[i][j] : UINT32_MAX);
    for (size_t i = 0; i < n; ++i) {
        uint32_t slot = (uint32_t)(base + i);
        for (uint32_t ci : asg[i]) cells[ci].members.push_back(slot);
        id_to_slot[ids[i]] = slot;
    }
    n_live += n;
    // primary centroid sums, per cell in input order
    size_t m = cells.size();
    std::vector<size_t> start(m + 1, 0);
    for (size_t i = 0; i < n; ++i) start[asg[i][0] + 1] += 1;
    for (size_t c = 0; c < m; ++c) start[c + 1] += start[c];
    std::vector<size_t> pos(start.begin(), start.end() - 1);
    std::vector<uint32_t> order(n);
    for (size_t i = 0; i < n; ++i) order[pos[asg[i][0]]++] = (uint32_t)i;
#pragma omp parallel for schedule(dynamic, 16)
    for (long long c = 0; c < (long long)m; ++c) {
        float* sv = cells[c].sum.data();
        for (size_t t = start[c]; t < start[c + 1]; ++t) {
            const float* v = data + (size_t)order[t] * dim;
            for (size_t j = 0; j < dim; ++j) sv[j] += v[j];
        }
    }
}

std::string HostIndex::add_batch(const uint64_t* ids, const float* data, size_t n) {
    // index.rs:2987-3212
    if (cells.empty()) return "call set_centroids() before add_batch()";
    compacted = false;
    ++version;
    if (quant_scale == 0.0f) {
        float max_abs = 0.0f;
        for (size_t i = 0; i < n * dim; ++i) {
            float a = std::fabs(data[i]);
            if (a > max_abs) max_abs = a;
        }
        quant_scale = max_abs > 0.0f ? 127.0f / max_abs : 1.0f;
    }
    if (per_dim_sq && sq_min.empty() && n > 0) {
        std::vector<float> lo(dim, INFINITY), hi(dim, -INFINITY);
        for (size_t i = 0; i < n; ++i)
            for (size_t j = 0; j < dim; ++j) {
                float x = data[i * dim + j];
                if (x < lo[j]) lo[j] = x;
                if (x > hi[j]) hi[j] = x;
            }
        sq_step.resize(dim);
        for (size_t j = 0; j < dim; ++j) sq_step[j] = std::max(hi[j] - lo[j], 1e-9f) / 255.0f;
        sq_min = lo;
    }
    std::vector<std::vector<uint32_t>> asg(n);
    // on the build GPU: homes and codes of every vector (the codes are then not recomputed here)
    std::vector<uint64_t> gpu_codes;
    bool gpu_placed = false;
    if (build_device >= 0 && tree && n > 0) {
        gpu_codes.resize(n * nw);
        std::string e = gpu_place(build_device, *this, data, n, asg, gpu_codes.data());
        if (e.empty()) {
            gpu_placed = true;
        } else {
            ++build_gpu_failures;
            build_gpu_error = e;
            gpu_codes.clear();
            asg.assign(n, {});
        }
    }
#pragma omp parallel
    {
        std::vector<float> rot(dim_pad);
        std::vector<uint64_t> qb(nw);
        std::vector<uint32_t> out;
#pragma omp for schedule(dynamic, 64)
        for (long long i = 0; i < (long long)n; ++i)
            if (!gpu_placed || asg[i].empty()) asg[i] = assign_cells_routed(data + (size_t)i * dim, rot, qb, out);
    }
    // Freed slots are refilled first, serially (index.rs:3090-3200).
    size_t n_reuse = std::min(free_slots.size(), n);
    std::vector<float> rot(dim_pad);
    for (size_t i = 0; i < n_reuse; ++i) {
        const float* v = data + i * dim;
        uint32_t s = free_slots.back();
        free_slots.pop_back();
        size_t off = (size_t)s * dim;
        if (keep_f32) std::copy(v, v + dim, vecs_f32.begin() + off);
        rotate(v, dim, signs.data(), dim_pad, rot.data());
        pack_signs_trunc(rot.data(), dim_pad, &bits[(size_t)s * nw], nw);
        if (i8_rerank) encode_i8(v, &scan_i8[off]);
        ext_ids[s] = ids[i];
        slot_cell[s] = asg[i][0];
        for (size_t j = 0; j < max_assign; ++j) slot_cells[(size_t)s * max_assign + j] = j < asg[i].size() ? asg[i][j] : UINT32_MAX;
        for (size_t j = 0; j < asg[i].size(); ++j) {
            Cell& c = cells[asg[i][j]];
            c.members.push_back(s);
            if (j == 0)
                for (size_t t = 0; t < dim; ++t) c.sum[t] += v[t];
        }
        id_to_slot[ids[i]] = s;
        n_live += 1;
    }
    if (n_reuse < n) {
        std::vector<std::vector<uint32_t>> rest(asg.begin() + n_reuse, asg.end());
        append_parallel(ids + n_reuse, data + n_reuse * dim, n - n_reuse, rest,
                        gpu_codes.empty() ? nullptr : gpu_codes.data() + n_reuse * nw);
    }
    for (auto& c : cells) {
        // Cell::recompute_centroid (index.rs:380-393)
        if (c.members.empty()) continue;
        float norm = 0.0f;
        for (float v : c.sum) norm += v * v;
        norm = std::sqrt(norm);
        if (norm > 1e-12f)
            for (size_t j = 0; j < dim; ++j) c.centroid[j] = c.sum[j] / norm;
    }
    refresh_derived();
    return "";
}

void HostIndex::fork_empty(HostIndex& f) const {
    // index.rs:2330-2400
    f.dim = dim;
    f.dim_pad = dim_pad;
    f.nw = nw;
    f.seed = seed;
    f.rerank_factor = rerank_factor;
    f.signs = signs;
    f.two_stage = two_stage;
    f.shortlist_mult = shortlist_mult;
    f.centroid_sq8 = centroid_sq8;
    f.tree_route = tree_route;
    f.tree_min_cells = tree_min_cells;
    f.tree_fanout = tree_fanout;
    f.tree_beam_frac = tree_beam_frac;
    f.graph_route = graph_route;
    f.graph_min_cells = graph_min_cells;
    f.max_assign = max_assign;
    f.spill_margin = spill_margin;
    f.spill_lambda = spill_lambda;
    f.fastscan = false;
    f.per_dim_sq = per_dim_sq;
    f.i8_rerank = i8_rerank;
    f.keep_f32 = keep_f32;
    f.adaptive = adaptive;
    f.at_margin = at_margin;
    f.quant_scale = quant_scale;
    f.cm_min_batch = cm_min_batch;
    f.sq_min = sq_min;
    f.sq_step = sq_step;
    f.build_device = build_device;
    f.bits.clear();
    f.scan_i8.clear();
    f.vecs_f32.clear();
    f.ext_ids.clear();
    f.slot_cell.clear();
    f.slot_cells.clear();
    f.free_slots.clear();
    f.id_to_slot.clear();
    f.tags.clear();
    f.has_filter = false;
    f.filter_lo = 0;
    f.filter_hi = 0xFFFFFFFFu;
    f.n_live = 0;
    f.compacted = false;
    f.prim_len.clear();
    f.rep_off.clear();
    f.fs_codes.clear();
    f.fs_off.clear();
    f.tree.reset();
    f.tree_cells = 0;
    f.cells.assign(cells.size(), Cell{});
    for (size_t c = 0; c < cells.size(); ++c) {
        f.cells[c].centroid = cells[c].centroid;
        f.cells[c].sum.assign(dim, 0.0f);
    }
    f.refresh_derived();
    ++f.version;
}

bool HostIndex::remove(uint64_t id) {
    // index.rs:3223-3276
    auto it = id_to_slot.find(id);
    if (it == id_to_slot.end()) return false;
    uint32_t slot = it->second;
    id_to_slot.erase(it);
    compacted = false;
    ++version;
    size_t primary = slot_cell[slot];
    size_t vs = (size_t)slot * dim;
    Cell& pc = cells[primary];
    if (keep_f32) {
        for (size_t j = 0; j < dim; ++j) pc.sum[j] -= vecs_f32[vs + j];
    } else if (per_dim_sq) {
        for (size_t j = 0; j < dim; ++j) {
            float c = (float)(uint8_t)scan_i8[vs + j];
            pc.sum[j] -= c * sq_step[j] + sq_min[j];
        }
    } else {
        float inv = 1.0f / quant_scale;
        for (size_t j = 0; j < dim; ++j) pc.sum[j] -= (float)scan_i8[vs + j] * inv;
    }
    for (size_t j = 0; j < max_assign; ++j) {
        uint32_t ci = slot_cells[(size_t)slot * max_assign + j];
        if (ci == UINT32_MAX) continue;
        auto& mem = cells[ci].members;
        auto p = std::find(mem.begin(), mem.end(), slot);
        if (p != mem.end()) {
            *p = mem.back();
            mem.pop_back();
        }
        slot_cells[(size_t)slot * max_assign + j] = UINT32_MAX;
    }
    if (!pc.members.empty()) {
        float norm = 0.0f;
        for (float v : pc.sum) norm += v * v;
        norm = std::sqrt(norm);
        if (norm > 1e-12f)
            for (size_t j = 0; j < dim; ++j) pc.centroid[j] = pc.sum[j] / norm;
    }
    free_slots.push_back(slot);
    n_live -= 1;
    return true;
}

void HostIndex::compact() {
    // compact_arena (index.rs:929-1112). The flat code arena is kept (the reference frees it
    // once the FastScan blocks exist); the GPU reads its own layout built from it.
    size_t old_n = ext_ids.size();
    if (old_n == 0) return;
    ++version;
    size_t ma = max_assign;
    std::vector<uint32_t> new_of_old(old_n, UINT32_MAX), old_of_new;
    old_of_new.reserve(n_live);
    for (size_t ci = 0; ci < cells.size(); ++ci)
        for (uint32_t s : cells[ci].members) {
            if (slot_cell[s] != ci) continue;
            if (new_of_old[s] != UINT32_MAX) continue;
            new_of_old[s] = (uint32_t)old_of_new.size();
            old_of_new.push_back(s);
        }
    // Live slots missed above (none in a consistent index), visited in slot order.
    std::vector<uint32_t> live_slots;
    for (auto& kv : id_to_slot) live_slots.push_back(kv.second);
    std::sort(live_slots.begin(), live_slots.end());
    for (uint32_t s : live_slots)
        if (new_of_old[s] == UINT32_MAX) {
            new_of_old[s] = (uint32_t)old_of_new.size();
            old_of_new.push_back(s);
        }
    size_t n_new = old_of_new.size();
    auto permute = [&](auto& arr, size_t stride) {
        using T = typename std::remove_reference<decltype(arr)>::type::value_type;
        if (arr.empty()) return;
        std::vector<T> v(n_new * stride);
        for (size_t ns = 0; ns < n_new; ++ns)
            std::copy(arr.begin() + (size_t)old_of_new[ns] * stride, arr.begin() + ((size_t)old_of_new[ns] + 1) * stride,
                      v.begin() + ns * stride);
        arr.swap(v);
    };
    if (keep_f32) permute(vecs_f32, dim);
    permute(scan_i8, dim);
    permute(bits, nw);
    permute(ext_ids, 1);
    permute(slot_cell, 1);
    permute(slot_cells, ma);
    if (!tags.empty()) permute(tags, 1);
    for (auto& c : cells) {
        std::vector<uint32_t> mem;
        for (uint32_t m : c.members)
            if (new_of_old[m] != UINT32_MAX) mem.push_back(new_of_old[m]);
        std::sort(mem.begin(), mem.end());
        c.members.swap(mem);
    }
    id_to_slot.clear();
    for (size_t ns = 0; ns < ext_ids.size(); ++ns) id_to_slot[ext_ids[ns]] = (uint32_t)ns;
    free_slots.clear();

    // Polysemic runs: [primaries | replicas], each ascending.
    prim_len.clear();
    rep_off.clear();
    if (max_assign > 1 && nw > 0) {
        rep_off.push_back(0);
        for (size_t ci = 0; ci < cells.size(); ++ci) {
            std::vector<uint32_t> prim, repl;
            for (uint32_t m : cells[ci].members) (slot_cell[m] == ci ? prim : repl).push_back(m);
            std::sort(prim.begin(), prim.end());
            std::sort(repl.begin(), repl.end());
            prim_len.push_back((uint32_t)prim.size());
            rep_off.push_back(rep_off.back() + (uint32_t)repl.size());
            prim.insert(prim.end(), repl.begin(), repl.end());
            cells[ci].members.swap(prim);
        }
    }
    // FastScan blocks over each cell's member order.
    fs_codes.clear();
    fs_off.clear();
    if (fastscan && nw > 0) {
        size_t bb = fs_block_bytes(nw);
        fs_off.assign(cells.size() + 1, 0);
        for (size_t ci = 0; ci < cells.size(); ++ci) {
            size_t nb = (cells[ci].members.size() + kFsBlock - 1) / kFsBlock;
            fs_off[ci + 1] = fs_off[ci] + (uint32_t)nb;
        }
        fs_codes.assign((size_t)fs_off.back() * bb, 0);
#pragma omp parallel for schedule(dynamic, 16)
        for (long long ci = 0; ci < (long long)cells.size(); ++ci) {
            const auto& mem = cells[ci].members;
            size_t nb = (mem.size() + kFsBlock - 1) / kFsBlock;
            const uint64_t* lanes[kFsBlock];
            for (size_t b = 0; b < nb; ++b) {
                size_t lo = b * kFsBlock, hi = std::min(lo + kFsBlock, mem.size());
                for (size_t i = lo; i < hi; ++i) lanes[i - lo] = &bits[(size_t)mem[i] * nw];
                fs_pack_block(lanes, hi - lo, nw, &fs_codes[((size_t)fs_off[ci] + b) * bb]);
            }
        }
    }
    compacted = true;
}

}  // namespace maivs
