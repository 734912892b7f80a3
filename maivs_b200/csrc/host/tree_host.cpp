// Centroid tree and spherical k-means for the host-side index build (src/tree.rs).
//
// Results do not depend on the thread count: assignment is per point, centroid sums run in
// input order, and the per-group sub-clusterings write disjoint slices (tree.rs:286-336).
#include <omp.h>

#include <algorithm>
#include <cmath>

#include "hostmath.h"
#include "index_host.h"

namespace maivs {

void kmeans_spherical(const float* x, size_t n, size_t dim, size_t k, size_t iters, uint64_t seed,
                      std::vector<uint32_t>& assign, std::vector<float>& cents, int device, size_t* gpu_failures) {
    // tree.rs:179-248
    if (device >= 0 && n > 0) {
        if (gpu_kmeans_spherical(device, x, n, dim, k, iters, seed, assign, cents).empty()) return;
        if (gpu_failures) {
#pragma omp atomic
            ++*gpu_failures;
        }
    }
    k = std::min(std::max<size_t>(k, 1), n);
    cents.assign(k * dim, 0.0f);
    size_t stride = std::max<size_t>(n / k, 1);
    for (size_t j = 0; j < k; ++j) {
        size_t src = std::min(j * stride, n - 1);
        std::copy(x + src * dim, x + (src + 1) * dim, cents.begin() + j * dim);
    }
    assign.assign(n, 0);
    uint64_t state = seed | 1;
    auto next_u = [&state]() {
        state ^= state << 13;
        state ^= state >> 7;
        state ^= state << 17;
        return state;
    };
    std::vector<float> sums;
    std::vector<uint32_t> counts;
    for (size_t it = 0; it < iters; ++it) {
#pragma omp parallel for schedule(static) if (n * k * dim > (1u << 16))
        for (long long i = 0; i < (long long)n; ++i) {
            const float* v = x + (size_t)i * dim;
            uint32_t best = 0;
            float best_s = -INFINITY;
            for (size_t j = 0; j < k; ++j) {
                float s = dot_f32(v, cents.data() + j * dim, dim);
                if (s > best_s) {
                    best_s = s;
                    best = (uint32_t)j;
                }
            }
            assign[i] = best;
        }
        sums.assign(k * dim, 0.0f);
        counts.assign(k, 0);
        for (size_t i = 0; i < n; ++i) {
            size_t j = assign[i];
            counts[j] += 1;
            const float* v = x + i * dim;
            float* s = sums.data() + j * dim;
            for (size_t t = 0; t < dim; ++t) s[t] += v[t];
        }
        for (size_t j = 0; j < k; ++j) {
            float* c = cents.data() + j * dim;
            if (counts[j] == 0) {
                size_t src = (size_t)(next_u() % (uint64_t)n);
                std::copy(x + src * dim, x + (src + 1) * dim, c);
                continue;
            }
            std::copy(sums.begin() + j * dim, sums.begin() + (j + 1) * dim, c);
            normalize(c, dim);
        }
    }
}

std::vector<float> hierarchical_kmeans(const float* x, size_t n, size_t dim, size_t k, uint64_t seed, int device,
                                       size_t* gpu_failures) {
    // tree.rs:257-348
    k = std::min(std::max<size_t>(k, 1), n);
    std::vector<uint32_t> assign;
    std::vector<float> cents;
    if (k <= 64 || n <= k * 4) {
        kmeans_spherical(x, n, dim, k, 12, seed, assign, cents, device, gpu_failures);
        return cents;
    }
    size_t k1 = (size_t)std::ceil(std::sqrt((double)k));
    kmeans_spherical(x, n, dim, k1, 8, seed, assign, cents, device, gpu_failures);
    std::vector<std::vector<uint32_t>> groups(k1);
    for (size_t i = 0; i < n; ++i) groups[assign[i]].push_back((uint32_t)i);

    std::vector<size_t> subs(groups.size(), 0), offs(groups.size(), 0);
    size_t written = 0, before = 0;
    for (size_t g = 0; g < groups.size(); ++g) {
        size_t glen = groups[g].size();
        size_t prev = before;
        before += glen;
        if (glen == 0 || written >= k) continue;
        size_t remaining_groups = k1 - g;
        double denom = (double)std::max<size_t>(n - prev, 1);
        size_t want = (size_t)std::round((double)(k - written) * (double)glen / denom);
        size_t sub = std::min(std::min(std::max<size_t>(want, 1), k - written), glen);
        if (remaining_groups == 1) sub = std::max<size_t>(std::min(k - written, glen), 1);
        if (sub == 0) continue;
        subs[g] = std::min(sub, k - written);
        offs[g] = written;
        written += subs[g];
    }

    std::vector<float> out(k * dim, 0.0f);
    std::vector<size_t> order;
    for (size_t g = 0; g < groups.size(); ++g)
        if (subs[g] > 0) order.push_back(g);
    // Sub-clusterings are independent; each runs single-threaded inside the parallel loop.
#pragma omp parallel for schedule(dynamic, 1)
    for (long long oi = 0; oi < (long long)order.size(); ++oi) {
        size_t g = order[oi];
        const auto& idx = groups[g];
        std::vector<float> buf(idx.size() * dim);
        for (size_t r = 0; r < idx.size(); ++r)
            std::copy(x + (size_t)idx[r] * dim, x + ((size_t)idx[r] + 1) * dim, buf.begin() + r * dim);
        std::vector<uint32_t> a;
        std::vector<float> cs;
        uint64_t gseed = seed ^ ((uint64_t)(g + 1) * 0x9E3779B9ull);
        kmeans_spherical(buf.data(), idx.size(), dim, subs[g], 12, gseed, a, cs, device, gpu_failures);
        std::copy(cs.begin(), cs.begin() + subs[g] * dim, out.begin() + offs[g] * dim);
    }
    size_t fill = 0;
    while (written < k) {
        size_t src = (fill * 7919) % n;
        std::copy(x + src * dim, x + (src + 1) * dim, out.begin() + written * dim);
        ++written;
        ++fill;
    }
    return out;
}

void keep_smallest(std::vector<std::pair<uint32_t, uint32_t>>& v, size_t keep, size_t bits) {
    // tree.rs:120-159
    if (keep >= v.size()) return;
    std::vector<uint32_t> hist(bits + 1, 0);
    for (auto& e : v) hist[e.first] += 1;
    size_t cum = 0, t = 0;
    while (t < bits) {
        cum += hist[t];
        if (cum >= keep) break;
        ++t;
    }
    if (t == bits) cum += hist[t];
    size_t need_eq = keep - (cum - hist[t]);
    size_t w = 0;
    for (size_t r = 0; r < v.size(); ++r) {
        auto e = v[r];
        size_t h = e.first;
        if (h < t || (h == t && need_eq > 0)) {
            if (h == t) --need_eq;
            v[w++] = e;
        }
    }
    v.resize(w);
}

static void code_of_centroid(const float* c, size_t dim, const float* signs, size_t dim_pad, size_t nw,
                             std::vector<float>& rot, uint64_t* out) {
    rotate(c, dim, signs, dim_pad, rot.data());
    pack_signs_trunc(rot.data(), dim_pad, out, nw);
}

std::unique_ptr<CentroidTree> build_centroid_tree(const float* cell_cents, const uint32_t* cell_ids, size_t m,
                                                  size_t dim, const float* signs, size_t dim_pad, size_t nw,
                                                  size_t fanout, float beam_frac, int device, size_t* gpu_failures) {
    // tree.rs:354-453
    if (m < 2 || nw == 0) return nullptr;
    fanout = std::max<size_t>(fanout, 2);
    std::vector<float> rot(dim_pad);
    auto t = std::make_unique<CentroidTree>();
    t->dim = dim;
    t->nw = nw;
    t->fanout = fanout;
    t->beam_frac = beam_frac > 0.0f ? beam_frac : kTreeDefaultBeamFrac;
    t->leaf_codes.resize(m * nw);
    for (size_t i = 0; i < m; ++i) code_of_centroid(cell_cents + i * dim, dim, signs, dim_pad, nw, rot, &t->leaf_codes[i * nw]);
    t->leaf_ids.assign(cell_ids, cell_ids + m);
    t->n_leaf = m;

    std::vector<TreeLevel> rev;
    std::vector<float> cur(cell_cents, cell_cents + m * dim);
    size_t cur_n = m;
    while (cur_n > kTreeTopMax) {
        size_t k = std::max<size_t>((cur_n + fanout - 1) / fanout, 1);
        if (k >= cur_n) break;
        std::vector<uint32_t> assign;
        std::vector<float> parents;
        kmeans_spherical(cur.data(), cur_n, dim, k, 10, 0x9E3779B97F4A7C15ull, assign, parents, device, gpu_failures);
        TreeLevel lv;
        lv.n = k;
        lv.child_len.assign(k, 0);
        for (uint32_t a : assign) lv.child_len[a] += 1;
        lv.child_start.assign(k, 0);
        uint32_t acc = 0;
        for (size_t j = 0; j < k; ++j) {
            lv.child_start[j] = acc;
            acc += lv.child_len[j];
        }
        std::vector<uint32_t> fill = lv.child_start;
        lv.child_idx.assign(cur_n, 0);
        for (size_t i = 0; i < cur_n; ++i) lv.child_idx[fill[assign[i]]++] = (uint32_t)i;
        lv.codes.resize(k * nw);
        for (size_t j = 0; j < k; ++j) code_of_centroid(parents.data() + j * dim, dim, signs, dim_pad, nw, rot, &lv.codes[j * nw]);
        lv.cents = parents;
        rev.push_back(std::move(lv));
        cur = std::move(parents);
        cur_n = k;
    }
    if (rev.empty()) return nullptr;
    std::reverse(rev.begin(), rev.end());
    t->levels = std::move(rev);

    // compact_layout (tree.rs:462-527): children of every node become one contiguous run.
    size_t d = t->levels.size();
    for (size_t i = 0; i < d; ++i) {
        std::vector<uint32_t> order = t->levels[i].child_idx;
        if (i + 1 < d) {
            TreeLevel& l = t->levels[i + 1];
            size_t n = l.n;
            if (order.size() == n) {
                std::vector<float> cents(n * dim);
                std::vector<uint64_t> codes(n * nw);
                std::vector<uint32_t> ns(n), nl(n), nidx;
                nidx.reserve(l.child_idx.size());
                uint32_t acc = 0;
                for (size_t np = 0; np < n; ++np) {
                    size_t o = order[np];
                    std::copy(l.cents.begin() + o * dim, l.cents.begin() + (o + 1) * dim, cents.begin() + np * dim);
                    std::copy(l.codes.begin() + o * nw, l.codes.begin() + (o + 1) * nw, codes.begin() + np * nw);
                    uint32_t st = l.child_start[o], ln = l.child_len[o];
                    ns[np] = acc;
                    nl[np] = ln;
                    acc += ln;
                    nidx.insert(nidx.end(), l.child_idx.begin() + st, l.child_idx.begin() + st + ln);
                }
                l.cents = std::move(cents);
                l.codes = std::move(codes);
                l.child_start = std::move(ns);
                l.child_len = std::move(nl);
                l.child_idx = std::move(nidx);
            }
        } else {
            size_t n = order.size();
            std::vector<uint64_t> codes(n * nw);
            std::vector<uint32_t> ids(n);
            for (size_t np = 0; np < n; ++np) {
                size_t o = order[np];
                std::copy(t->leaf_codes.begin() + o * nw, t->leaf_codes.begin() + (o + 1) * nw, codes.begin() + np * nw);
                ids[np] = t->leaf_ids[o];
            }
            t->leaf_codes = std::move(codes);
            t->leaf_ids = std::move(ids);
            t->n_leaf = n;
        }
        for (size_t k = 0; k < t->levels[i].child_idx.size(); ++k) t->levels[i].child_idx[k] = (uint32_t)k;
    }
    return t;
}

std::vector<size_t> CentroidTree::beams(size_t want) const {
    // tree.rs:559-570
    size_t d = levels.size();
    std::vector<size_t> b(d, 0);
    size_t need = std::max<size_t>(want, 1);
    for (size_t ii = d; ii-- > 0;) {
        size_t raw = (size_t)std::ceil((float)need * beam_frac);
        size_t v = std::min(std::max(raw, kTreeMinBeam), levels[ii].n);
        b[ii] = v;
        need = v;
    }
    return b;
}

void CentroidTree::search(const uint64_t* q, size_t want, std::vector<uint32_t>& out) const {
    // tree.rs:574-628
    out.clear();
    if (levels.empty()) return;
    size_t bits = nw * 64;
    std::vector<size_t> bm = beams(want);
    std::vector<uint32_t> frontier(levels[0].n), expand;
    for (size_t i = 0; i < levels[0].n; ++i) frontier[i] = (uint32_t)i;
    std::vector<std::pair<uint32_t, uint32_t>> scored;
    for (size_t li = 0; li < levels.size(); ++li) {
        const TreeLevel& lv = levels[li];
        scored.clear();
        for (uint32_t node : frontier) scored.push_back({hamming(q, &lv.codes[(size_t)node * nw], nw), node});
        size_t keep = std::min(bm[li], scored.size());
        if (keep == 0) return;
        keep_smallest(scored, keep, bits);
        expand.clear();
        for (auto& e : scored) {
            uint32_t st = lv.child_start[e.second], ln = lv.child_len[e.second];
            expand.insert(expand.end(), lv.child_idx.begin() + st, lv.child_idx.begin() + st + ln);
        }
        frontier.swap(expand);
    }
    scored.clear();
    for (uint32_t leaf : frontier) scored.push_back({hamming(q, &leaf_codes[(size_t)leaf * nw], nw), leaf});
    size_t keep = std::min(want, scored.size());
    if (keep == 0) return;
    keep_smallest(scored, keep, bits);
    for (auto& e : scored) out.push_back(leaf_ids[e.second]);
}

}  // namespace maivs
