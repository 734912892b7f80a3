// TEST INFRASTRUCTURE ONLY - the parity oracle of the B200 MAIVS engine.
//
// A CPU restatement, in C++17 + AVX2 + OpenMP, of the reference's query hot path
// (V47VANSH/MAIVS, Rust): src/quantize.rs (rotation, codes, FastScan tables and block sums),
// src/tree.rs:120-159 and :559-628 (tree beam search), src/index.rs:41-343 (SIMD dots),
// :1168-1305 (route_query), :1309-1378 (rerank_exact), :1381-1864 (search_one, FastScan and
// Hamming branches), :1873-1980 (route_batch), :1999-2311 (search_batch_cellmajor, FastScan),
// :3316-3391 (search_batch), and the build's mutations (add_batch with freed-slot refill, remove,
// compact_arena, fork_empty). Each function below cites the lines it follows.
//
// Only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline arm load this library; the
// product never links or calls it. It consumes an index's arrays (as exported by the product's
// maivs_array) and recomputes every query result from them with the reference's arithmetic.
//
// Parity pinning: the reference ships no golden vectors for this path and cannot be built here
// (Rust; no toolchain). The oracle is pinned by the reference's own property tests
// (quantize.rs:445-492), its invariant suite (tests/test_index.py [11], [12], [14]), published
// splitmix64 outputs, and cross-checks between its own scalar and AVX2 FastScan kernels.
//
// Where the reference orders exactly equal floats with an unstable sort (probe selection,
// candidate cut of the per-query path, final top-k), this oracle breaks ties by ascending cell id,
// slot, and external id respectively; the GPU engine uses the same rule.
#include <immintrin.h>
#include <omp.h>

#include <algorithm>
#include <atomic>
#include <cmath>
#include <cstdint>
#include <cstring>
#include <map>
#include <unordered_map>
#include <string>
#include <vector>

namespace {

// ---- quantize.rs -------------------------------------------------------------------------------

void make_signs(size_t dim_pad, uint64_t seed, float* out) {  // quantize.rs:132-148
    uint64_t state = seed;
    for (size_t r = 0; r < 2; ++r)
        for (size_t i = 0; i < dim_pad; ++i) {
            state += 0x9E3779B97F4A7C15ull;
            uint64_t z = state;
            z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
            z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
            z ^= z >> 31;
            out[r * dim_pad + i] = (z & 1) == 0 ? 1.0f : -1.0f;
        }
}

void fht_inplace(float* a, size_t n) {  // quantize.rs:71-126 (8-blocks, then contiguous halves)
    size_t h = 1;
    if (n >= 8 && n % 8 == 0) {
        for (size_t blk = 0; blk < n; blk += 8) {
            float x[8];
            for (int t = 0; t < 8; ++t) x[t] = a[blk + t];
            for (size_t hh : {1u, 2u, 4u})
                for (size_t i = 0; i < 8; i += hh << 1)
                    for (size_t j = i; j < i + hh; ++j) {
                        float u = x[j], v = x[j + hh];
                        x[j] = u + v;
                        x[j + hh] = u - v;
                    }
            for (int t = 0; t < 8; ++t) a[blk + t] = x[t];
        }
        h = 8;
        while (h < n) {
            for (size_t blk = 0; blk < n; blk += h << 1)
                for (size_t t = 0; t < h; ++t) {
                    float x = a[blk + t], y = a[blk + h + t];
                    a[blk + t] = x + y;
                    a[blk + h + t] = x - y;
                }
            h <<= 1;
        }
    }
    while (h < n) {
        for (size_t i = 0; i < n; i += h << 1)
            for (size_t j = i; j < i + h; ++j) {
                float x = a[j], y = a[j + h];
                a[j] = x + y;
                a[j + h] = x - y;
            }
        h <<= 1;
    }
    float s = 1.0f / std::sqrt((float)n);
    for (size_t i = 0; i < n; ++i) a[i] *= s;
}

void rotate(const float* v, size_t dim, const float* signs, size_t dim_pad, float* out) {  // quantize.rs:152-163
    for (size_t i = 0; i < dim_pad; ++i) out[i] = i < dim ? v[i] : 0.0f;
    for (size_t r = 0; r < 2; ++r) {
        for (size_t i = 0; i < dim_pad; ++i) out[i] *= signs[r * dim_pad + i];
        fht_inplace(out, dim_pad);
    }
}

void pack_signs_trunc(const float* rot, size_t dim_pad, uint64_t* out, size_t nw) {  // quantize.rs:57-67
    for (size_t w = 0; w < nw; ++w) out[w] = 0;
    size_t bits = std::min(nw * 64, dim_pad);
    for (size_t i = 0; i < bits; ++i)
        if (rot[i] < 0.0f) out[i >> 6] |= 1ull << (i & 63);
}

inline uint32_t hamming(const uint64_t* a, const uint64_t* b, size_t nw) {  // quantize.rs:183-201
    uint32_t s = 0;
    for (size_t i = 0; i < nw; ++i) s += (uint32_t)__builtin_popcountll(a[i] ^ b[i]);
    return s;
}

struct FsQuery {  // quantize.rs:268-319
    std::vector<uint8_t> lut;
    float delta = 0, bias = 0;
    size_t npos = 0;
    uint32_t maxk = 0;
    float estimate(uint32_t sum) const { return delta * (float)sum + bias; }
};

FsQuery fs_query(const float* rq, size_t rq_len, size_t nw) {  // quantize.rs:279-313
    FsQuery f;
    size_t npos = nw * 16;
    std::vector<float> raw(npos * 16), mins(npos);
    float range = 0.0f;
    for (size_t j = 0; j < npos; ++j) {
        float lo = INFINITY, hi = -INFINITY;
        for (size_t e = 0; e < 16; ++e) {
            float v = 0.0f;
            for (size_t t = 0; t < 4; ++t) {
                size_t d = 4 * j + t;
                float x = d < rq_len ? rq[d] : 0.0f;
                v += ((e >> t) & 1) ? -x : x;
            }
            raw[j * 16 + e] = v;
            lo = std::fmin(lo, v);
            hi = std::fmax(hi, v);
        }
        mins[j] = lo;
        range = std::fmax(range, hi - lo);
    }
    float delta = std::fmax(range / 255.0f, 1e-12f);
    f.lut.assign(npos * 16, 0);
    for (size_t p = 0; p < npos / 2; ++p)
        for (size_t half = 0; half < 2; ++half) {
            size_t j = 2 * p + half;
            for (size_t e = 0; e < 16; ++e) {
                float q = std::round((raw[j * 16 + e] - mins[j]) / delta);
                q = q < 0.0f ? 0.0f : (q > 255.0f ? 255.0f : q);
                f.lut[p * 32 + half * 16 + e] = (uint8_t)q;
            }
        }
    float bias = 0.0f;
    for (float m : mins) bias += m;
    f.delta = delta;
    f.bias = bias;
    f.npos = npos;
    f.maxk = 255u * (uint32_t)npos;
    return f;
}

void fs_block_sums_scalar(const uint8_t* block, const uint8_t* lut, size_t npairs, uint16_t* out) {  // :335-349
    for (int i = 0; i < 32; ++i) out[i] = 0;
    for (size_t p = 0; p < npairs; ++p)
        for (size_t half = 0; half < 2; ++half) {
            size_t base = p * 32 + half * 16;
            for (size_t i = 0; i < 16; ++i) {
                uint8_t b = block[base + i];
                out[i] = (uint16_t)(out[i] + lut[base + (b & 0xF)]);
                out[i + 16] = (uint16_t)(out[i + 16] + lut[base + (b >> 4)]);
            }
        }
}

void fs_block_sums_avx2(const uint8_t* block, const uint8_t* lut, size_t npairs, uint16_t* out) {  // :351-386
    const __m256i mask = _mm256_set1_epi8(0x0F);
    __m256i a0l = _mm256_setzero_si256(), a1l = _mm256_setzero_si256();
    __m256i a0h = _mm256_setzero_si256(), a1h = _mm256_setzero_si256();
    for (size_t p = 0; p < npairs; ++p) {
        __m256i c = _mm256_loadu_si256((const __m256i*)(block + p * 32));
        __m256i l = _mm256_loadu_si256((const __m256i*)(lut + p * 32));
        __m256i lo = _mm256_and_si256(c, mask);
        __m256i hi = _mm256_and_si256(_mm256_srli_epi16(c, 4), mask);
        __m256i rl = _mm256_shuffle_epi8(l, lo);
        __m256i rh = _mm256_shuffle_epi8(l, hi);
        a0l = _mm256_add_epi16(a0l, rl);
        a1l = _mm256_add_epi16(a1l, _mm256_srli_epi16(rl, 8));
        a0h = _mm256_add_epi16(a0h, rh);
        a1h = _mm256_add_epi16(a1h, _mm256_srli_epi16(rh, 8));
    }
    auto fold = [](__m256i a0, __m256i a1, uint16_t* dst) {
        __m256i even = _mm256_sub_epi16(a0, _mm256_slli_epi16(a1, 8));
        __m128i e = _mm_add_epi16(_mm256_castsi256_si128(even), _mm256_extracti128_si256(even, 1));
        __m128i o = _mm_add_epi16(_mm256_castsi256_si128(a1), _mm256_extracti128_si256(a1, 1));
        _mm_storeu_si128((__m128i*)dst, _mm_unpacklo_epi16(e, o));
        _mm_storeu_si128((__m128i*)(dst + 8), _mm_unpackhi_epi16(e, o));
    };
    fold(a0l, a1l, out);
    fold(a0h, a1h, out + 16);
}

inline uint8_t nib(const uint64_t* code, size_t j) { return (uint8_t)((code[j >> 4] >> ((j & 15) * 4)) & 0xF); }

void fs_pack_block(const uint64_t* const* codes, size_t ncodes, size_t nw, uint8_t* out) {  // quantize.rs:238-250
    size_t npos = nw * 16;
    for (size_t p = 0; p < npos / 2; ++p)
        for (size_t half = 0; half < 2; ++half) {
            size_t j = 2 * p + half;
            for (size_t i = 0; i < 16; ++i) {
                uint8_t lo = i < ncodes ? nib(codes[i], j) : 0;
                uint8_t hi = i + 16 < ncodes ? nib(codes[i + 16], j) : 0;
                out[p * 32 + half * 16 + i] = (uint8_t)(lo | (hi << 4));
            }
        }
}

// ---- index.rs SIMD dots ------------------------------------------------------------------------

inline float hsum_ps(__m256 v) {  // index.rs:58-65
    __m128 lo = _mm256_castps256_ps128(v);
    __m128 hi = _mm256_extractf128_ps(v, 1);
    __m128 s = _mm_add_ps(lo, hi);
    s = _mm_add_ps(s, _mm_movehl_ps(s, s));
    s = _mm_add_ss(s, _mm_shuffle_ps(s, s, 0x55));
    return _mm_cvtss_f32(s);
}

float dot_f32(const float* a, const float* b, size_t n) {  // index.rs:136-152
    __m256 acc = _mm256_setzero_ps();
    size_t i = 0;
    for (; i + 8 <= n; i += 8) acc = _mm256_fmadd_ps(_mm256_loadu_ps(a + i), _mm256_loadu_ps(b + i), acc);
    float s = hsum_ps(acc);
    for (; i < n; ++i) s += a[i] * b[i];
    return s;
}

float dot_f32_u8(const float* qs, const int8_t* v, size_t n) {  // index.rs:278-294
    __m256 acc = _mm256_setzero_ps();
    size_t i = 0;
    for (; i + 8 <= n; i += 8) {
        __m128i b = _mm_loadl_epi64((const __m128i*)(v + i));
        __m256 vf = _mm256_cvtepi32_ps(_mm256_cvtepu8_epi32(b));
        acc = _mm256_fmadd_ps(_mm256_loadu_ps(qs + i), vf, acc);
    }
    float s = hsum_ps(acc);
    for (; i < n; ++i) s += qs[i] * (float)(uint8_t)v[i];
    return s;
}

float dot_f32_i8(const float* q, const int8_t* v, size_t n) {  // index.rs:161-177
    __m256 acc = _mm256_setzero_ps();
    size_t i = 0;
    for (; i + 8 <= n; i += 8) {
        __m128i b = _mm_loadl_epi64((const __m128i*)(v + i));
        __m256 vf = _mm256_cvtepi32_ps(_mm256_cvtepi8_epi32(b));
        acc = _mm256_fmadd_ps(_mm256_loadu_ps(q + i), vf, acc);
    }
    float s = hsum_ps(acc);
    for (; i < n; ++i) s += q[i] * (float)v[i];
    return s;
}

// index.rs:86-104
size_t hamming_cutoff(const std::vector<uint16_t>& hs, const std::vector<uint8_t>& live, size_t want, size_t bits) {
    if (want == 0) return 0;
    std::vector<uint32_t> hist(bits + 1, 0);
    for (size_t i = 0; i < hs.size(); ++i)
        if (live[i]) hist[hs[i]] += 1;
    size_t cum = 0;
    for (size_t t = 0; t <= bits; ++t) {
        cum += hist[t];
        if (cum >= want) return t;
    }
    return bits;
}

// tree.rs:120-159
void keep_smallest(std::vector<std::pair<uint32_t, uint32_t>>& v, size_t keep, size_t bits) {
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
        if (e.first < t || (e.first == t && need_eq > 0)) {
            if (e.first == t) --need_eq;
            v[w++] = e;
        }
    }
    v.resize(w);
}

// ---- the index as the oracle sees it -----------------------------------------------------------

struct Level {
    size_t n;
    std::vector<uint64_t> codes;
    std::vector<uint32_t> child_start, child_len;
};

struct OIndex {
    size_t dim, dim_pad, nw, M, ma, n_slots;
    std::vector<float> signs, centroids, r_bound;
    std::vector<uint32_t> mem, mem_off;
    std::vector<uint8_t> fs_codes;
    std::vector<uint32_t> fs_off;
    std::vector<uint32_t> slot_cells;
    std::vector<uint64_t> ext_ids;
    std::vector<uint64_t> bits;  // nw words per slot (the Hamming scan of a non-FastScan index)
    std::vector<uint64_t> cent_bits;
    std::vector<uint8_t> cent_sq8;
    std::vector<float> csq_min, csq_step;
    std::vector<float> vecs_f32;
    std::vector<int8_t> scan_i8;
    std::vector<float> sq_min, sq_step;
    std::vector<uint32_t> tags;
    std::vector<Level> levels;
    std::vector<uint64_t> leaf_codes;
    std::vector<uint32_t> leaf_ids;
    size_t n_leaf = 0;
    float beam_frac = 0.5f;
    // configuration
    size_t rerank_factor, shortlist_mult, cm_min_batch, n_live, graph_min_cells;
    bool two_stage, centroid_sq8, has_tree, adaptive, per_dim_sq, i8_rerank, compacted, has_filter, fastscan,
        graph_route;
    float at_margin;
    uint32_t flo, fhi;

    size_t members(size_t c) const { return mem_off[c + 1] - mem_off[c]; }
    // non-empty cells: the centroid graph exists when there are graph_min_cells of them
    // (rebuild_centroid_graph, index.rs:625-636)
    size_t live_cells() const {
        size_t n = 0;
        for (size_t c = 0; c + 1 < mem_off.size(); ++c) n += mem_off[c + 1] > mem_off[c];
        return n;
    }
    size_t n_live_cells = 0;
    const uint32_t* member_ptr(size_t c) const { return mem.data() + mem_off[c]; }
    bool live(size_t c) const { return members(c) > 0; }
};

struct SearchBuf {
    std::vector<float> rot, cqs;
    std::vector<uint64_t> q_bits;
    std::vector<std::pair<uint32_t, float>> cscores;
    std::vector<uint32_t> chosen;
};

inline bool score_desc(const std::pair<uint32_t, float>& a, const std::pair<uint32_t, float>& b) {
    if (a.second != b.second) return a.second > b.second;
    return a.first < b.first;
}

// Stage-2 re-order score of one cell (index.rs:782-800).
inline float cent_score(const OIndex& ix, size_t ci, const float* q, const float* cqs, float base) {
    if (ix.centroid_sq8 && !ix.cent_sq8.empty())
        return dot_f32_u8(cqs, (const int8_t*)&ix.cent_sq8[ci * ix.dim], ix.dim) + base;
    return dot_f32(q, &ix.centroids[ci * ix.dim], ix.dim);
}

// Top-`cap` by score (descending), then the nucleus rule (index.rs:1283-1301, :1955-1974).
void select_and_nucleus(std::vector<std::pair<uint32_t, float>>& cs, size_t nprobe, float tc, float beta,
                        std::vector<uint32_t>& chosen) {
    chosen.clear();
    size_t cap = std::min(nprobe, cs.size());
    if (cap == 0) return;
    std::partial_sort(cs.begin(), cs.begin() + cap, cs.end(), score_desc);
    cs.resize(cap);
    if (tc >= 1.0f) {
        for (auto& c : cs) chosen.push_back(c.first);
        return;
    }
    float max_s = cs[0].second, z = 0.0f;
    for (auto& c : cs) z += std::exp((c.second - max_s) * beta);
    float cum = 0.0f;
    for (auto& c : cs) {
        chosen.push_back(c.first);
        cum += std::exp((c.second - max_s) * beta) / (z + 1e-9f);
        if (cum >= tc) break;
    }
}

std::vector<size_t> tree_beams(const OIndex& ix, size_t want) {  // tree.rs:559-570
    size_t d = ix.levels.size();
    std::vector<size_t> b(d, 0);
    size_t need = std::max<size_t>(want, 1);
    for (size_t ii = d; ii-- > 0;) {
        size_t raw = (size_t)std::ceil((float)need * ix.beam_frac);
        size_t v = std::min(std::max<size_t>(raw, 32), ix.levels[ii].n);
        b[ii] = v;
        need = v;
    }
    return b;
}

void tree_search(const OIndex& ix, const uint64_t* q, size_t want, std::vector<uint32_t>& out) {  // tree.rs:574-628
    out.clear();
    if (ix.levels.empty()) return;
    size_t nw = ix.nw, bits = nw * 64;
    auto beams = tree_beams(ix, want);
    std::vector<uint32_t> frontier(ix.levels[0].n), expand;
    for (size_t i = 0; i < frontier.size(); ++i) frontier[i] = (uint32_t)i;
    std::vector<std::pair<uint32_t, uint32_t>> scored;
    for (size_t li = 0; li < ix.levels.size(); ++li) {
        const Level& lv = ix.levels[li];
        scored.clear();
        for (uint32_t node : frontier) scored.push_back({hamming(q, &lv.codes[(size_t)node * nw], nw), node});
        size_t keep = std::min(beams[li], scored.size());
        if (keep == 0) return;
        keep_smallest(scored, keep, bits);
        expand.clear();
        for (auto& e : scored)
            for (uint32_t r = 0; r < lv.child_len[e.second]; ++r) expand.push_back(lv.child_start[e.second] + r);
        frontier.swap(expand);
    }
    scored.clear();
    for (uint32_t leaf : frontier) scored.push_back({hamming(q, &ix.leaf_codes[(size_t)leaf * nw], nw), leaf});
    size_t keep = std::min(want, scored.size());
    if (keep == 0) return;
    keep_smallest(scored, keep, bits);
    for (auto& e : scored) out.push_back(ix.leaf_ids[e.second]);
}

// route_query (index.rs:1168-1305). Returns -1 when graph routing would be needed.
int route_query(const OIndex& ix, const float* q, size_t nprobe, float tc, float beta, SearchBuf& b) {
    size_t dim = ix.dim, nw = ix.nw;
    b.rot.resize(ix.dim_pad);
    b.q_bits.resize(nw);
    b.cqs.resize(dim);
    float cqbase = 0.0f;
    bool cent_q8 = ix.centroid_sq8 && !ix.cent_sq8.empty();
    if (cent_q8)
        for (size_t j = 0; j < dim; ++j) {
            b.cqs[j] = q[j] * ix.csq_step[j];
            cqbase += q[j] * ix.csq_min[j];
        }
    b.cscores.clear();
    size_t mult2 = std::max<size_t>(ix.shortlist_mult, 2);
    if (ix.has_tree) {
        rotate(q, dim, ix.signs.data(), ix.dim_pad, b.rot.data());
        pack_signs_trunc(b.rot.data(), ix.dim_pad, b.q_bits.data(), nw);
        size_t want_c = std::min(nprobe * mult2, ix.n_leaf);
        std::vector<uint32_t> tout;
        tree_search(ix, b.q_bits.data(), want_c, tout);
        for (uint32_t ci : tout)
            if (ix.live(ci)) b.cscores.push_back({ci, cent_score(ix, ci, q, b.cqs.data(), cqbase)});
    } else if (ix.graph_route && ix.n_live_cells >= ix.graph_min_cells) {
        return -1;
    } else if (ix.two_stage && !ix.cent_bits.empty()) {
        rotate(q, dim, ix.signs.data(), ix.dim_pad, b.rot.data());
        pack_signs_trunc(b.rot.data(), ix.dim_pad, b.q_bits.data(), nw);
        std::vector<uint16_t> hs(ix.M);
        std::vector<uint8_t> live(ix.M);
        size_t n_live = 0;
        for (size_t i = 0; i < ix.M; ++i) {
            hs[i] = (uint16_t)hamming(b.q_bits.data(), &ix.cent_bits[i * nw], nw);
            live[i] = ix.live(i);
            n_live += live[i];
        }
        size_t want_c = std::min(nprobe * ix.shortlist_mult, n_live);
        size_t cut = hamming_cutoff(hs, live, want_c, nw * 64);
        for (size_t i = 0; i < ix.M; ++i)
            if (hs[i] <= cut && live[i]) b.cscores.push_back({(uint32_t)i, cent_score(ix, i, q, b.cqs.data(), cqbase)});
    } else {
        for (size_t i = 0; i < ix.M; ++i)
            if (ix.live(i)) b.cscores.push_back({(uint32_t)i, cent_score(ix, i, q, b.cqs.data(), cqbase)});
    }
    select_and_nucleus(b.cscores, nprobe, tc, beta, b.chosen);
    return 0;
}

// rerank_exact (index.rs:1309-1378): exact score of every candidate, then the top k best first.
std::vector<std::pair<float, uint64_t>> rerank_exact(const OIndex& ix, const float* q,
                                                     const std::vector<uint32_t>& cands, size_t k) {
    std::vector<std::pair<float, uint64_t>> out;
    if (cands.empty()) return out;
    size_t dim = ix.dim;
    std::vector<float> qs;
    float base = 0.0f;
    if (ix.per_dim_sq) {
        qs.resize(dim);
        for (size_t j = 0; j < dim; ++j) {
            qs[j] = q[j] * ix.sq_step[j];
            base += q[j] * ix.sq_min[j];
        }
    }
    for (uint32_t slot : cands) {
        float s;
        if (ix.per_dim_sq)
            s = base + dot_f32_u8(qs.data(), &ix.scan_i8[(size_t)slot * dim], dim);
        else if (ix.i8_rerank)
            s = dot_f32_i8(q, &ix.scan_i8[(size_t)slot * dim], dim);
        else
            s = dot_f32(q, &ix.vecs_f32[(size_t)slot * dim], dim);
        out.push_back({s, ix.ext_ids[slot]});
    }
    size_t kk = std::min(k, out.size());
    auto better = [](const std::pair<float, uint64_t>& a, const std::pair<float, uint64_t>& b) {
        if (a.first != b.first) return a.first > b.first;
        return a.second < b.second;
    };
    std::partial_sort(out.begin(), out.begin() + kk, out.end(), better);
    out.resize(kk);
    return out;
}

// search_one, FastScan branch (index.rs:1381-1692, :1843-1864). Also returns the candidate slots
// that go to the rerank (for parity tests) when `cands_out` is given.
std::vector<std::pair<float, uint64_t>> search_one(const OIndex& ix, const float* q, size_t k, size_t nprobe, float tc,
                                                   float beta, SearchBuf& b, std::vector<uint32_t>* cands_out,
                                                   int* err) {
    if (route_query(ix, q, nprobe, tc, beta, b) < 0) {
        *err = 7;
        return {};
    }
    const auto& chosen = b.chosen;
    if (chosen.empty()) return {};
    const size_t nw = ix.nw, ma = ix.ma;
    const bool dedup = ma > 1;
    std::vector<uint32_t> crank;
    std::vector<uint8_t> visited;
    if (dedup) {
        crank.assign(ix.M, 0);
        visited.assign(ix.M, 0);
        for (size_t r = 0; r < chosen.size(); ++r) {
            visited[chosen[r]] = 1;
            crank[chosen[r]] = (uint32_t)r;
        }
    }
    const bool filtering = ix.has_filter && !ix.tags.empty();
    auto keep = [&](uint32_t slot) {
        if (!filtering) return true;
        uint32_t t = ix.tags[slot];
        return t >= ix.flo && t <= ix.fhi;
    };
    auto seen = [&](uint32_t slot, uint32_t ci) {
        for (size_t j = 0; j < ma; ++j) {
            uint32_t h = ix.slot_cells[(size_t)slot * ma + j];
            if (h != UINT32_MAX && h != ci && visited[h] && crank[h] < crank[ci]) return true;
        }
        return false;
    };
    const size_t want0 = k * ix.rerank_factor;
    std::vector<float> suffix;
    if (ix.adaptive) {
        size_t n = chosen.size();
        suffix.assign(n + 1, -INFINITY);
        std::vector<float> bounds(n);
        for (size_t i = 0; i < n; ++i) {
            float cs = b.cscores[i].second;
            float ang = std::acos(std::fmin(std::fmax(cs, -1.0f), 1.0f));
            bounds[i] = std::cos(std::fmax(ang - ix.r_bound[chosen[i]], 0.0f));
        }
        for (size_t i = n; i-- > 0;) suffix[i] = std::fmax(bounds[i], suffix[i + 1]);
    }
    rotate(q, ix.dim, ix.signs.data(), ix.dim_pad, b.rot.data());
    const size_t target = std::max<size_t>(want0, 1);
    if (!(ix.fastscan && ix.compacted && !ix.fs_off.empty())) {
        // Hamming bucket queue over the flat codes (index.rs:1693-1808, no cascade): tau starts
        // at the code length and falls while the candidates strictly below it fill target; every
        // candidate at or below the final tau goes to the rerank, ties included (:1843-1848).
        const uint32_t dp = (uint32_t)(nw * 64);
        std::vector<uint64_t> qb(nw);
        pack_signs_trunc(b.rot.data(), ix.dim_pad, qb.data(), nw);
        std::vector<uint32_t> hist(dp + 1, 0);
        std::vector<std::pair<uint32_t, uint32_t>> hc;  // (h, slot)
        uint32_t tau = dp;
        size_t kept = 0;
        for (size_t ci_i = 0; ci_i < chosen.size(); ++ci_i) {
            uint32_t ci = chosen[ci_i];
            const uint32_t* mem = ix.member_ptr(ci);
            size_t nmem = ix.members(ci);
            for (size_t i = 0; i < nmem; ++i) {
                uint32_t slot = mem[i];
                if (!keep(slot) || (dedup && seen(slot, ci))) continue;
                uint32_t h = hamming(qb.data(), &ix.bits[(size_t)slot * nw], nw);
                if (h <= tau) {  // offer! (:1704-1717)
                    hc.push_back({h, slot});
                    hist[h] += 1;
                    kept += 1;
                    while (tau > 0 && kept - hist[tau] >= target) {
                        kept -= hist[tau];
                        tau -= 1;
                    }
                }
            }
            if (hc.size() > 4 * target + 1024) {
                uint32_t t = tau;
                hc.erase(std::remove_if(hc.begin(), hc.end(), [t](const std::pair<uint32_t, uint32_t>& x) {
                             return x.first > t;
                         }),
                         hc.end());
            }
            if (ix.adaptive && kept >= target) {
                // score_to_cos(hamming_score(tau, dp)) (index.rs:1139-1164, quantize.rs:206-208)
                float dpf = (float)dp;
                float s = dpf - 2.0f * (float)tau;
                float hh = (dpf - s) * 0.5f;
                float thr = std::cos(3.14159265358979323846f * hh / dpf);
                if (suffix[ci_i + 1] < thr - ix.at_margin) break;
            }
        }
        std::vector<uint32_t> slots;
        for (auto& x : hc)
            if (x.first <= tau) slots.push_back(x.second);
        if (cands_out) *cands_out = slots;
        if (slots.empty()) return {};
        return rerank_exact(ix, q, slots, k);
    }
    // FastScan bucket queue on d >> 6 with a falling tau (index.rs:1630-1692)
    FsQuery fq = fs_query(b.rot.data(), ix.dim_pad, nw);
    const size_t bb = nw * 64 * 32 / 8;
    const uint32_t maxk = fq.maxk;
    const float norm = std::sqrt(2.0f * (float)ix.dim_pad / 3.14159265358979323846f);
    std::vector<uint32_t> hist(nw * 64 + 1, 0);
    struct HC {
        uint32_t h, slot;
        float d;
    };
    std::vector<HC> hcands;
    uint32_t tau = maxk >> 6;
    size_t kept = 0;
    uint16_t sums[32];
    for (size_t ci_i = 0; ci_i < chosen.size(); ++ci_i) {
        uint32_t ci = chosen[ci_i];
        const uint32_t* mem = ix.member_ptr(ci);
        size_t nmem = ix.members(ci);
        size_t b0 = ix.fs_off[ci], b1 = ix.fs_off[ci + 1];
        for (size_t blk = b0; blk < b1; ++blk) {
            fs_block_sums_avx2(&ix.fs_codes[blk * bb], fq.lut.data(), fq.npos / 2, sums);
            size_t base = (blk - b0) * 32;
            size_t nv = std::min<size_t>(32, nmem - base);
            for (size_t i = 0; i < nv; ++i) {
                uint32_t d = maxk - sums[i];
                uint32_t hc = d >> 6;
                if (hc <= tau) {
                    uint32_t slot = mem[base + i];
                    if (!keep(slot) || (dedup && seen(slot, ci))) continue;
                    hcands.push_back({hc, slot, (float)d});
                    hist[hc] += 1;
                    kept += 1;
                    while (tau > 0 && kept - hist[tau] >= target) {
                        kept -= hist[tau];
                        tau -= 1;
                    }
                }
            }
        }
        if (hcands.size() > 4 * target + 1024) {
            uint32_t t = tau;
            hcands.erase(std::remove_if(hcands.begin(), hcands.end(), [t](const HC& x) { return x.h > t; }),
                         hcands.end());
        }
        if (ix.adaptive && kept >= target) {
            uint32_t wsub = ((tau + 1) << 6) - 1;
            uint32_t worst = maxk > wsub ? maxk - wsub : 0;
            float thr = fq.estimate(worst) / norm;
            thr = std::fmin(std::fmax(thr, -1.0f), 1.0f);
            if (suffix[ci_i + 1] < thr - ix.at_margin) break;
        }
    }
    // cands = (-d, slot) for h <= tau; top want0 by -d, ties by slot
    std::vector<std::pair<uint32_t, uint32_t>> cands;  // (d, slot)
    for (auto& x : hcands)
        if (x.h <= tau) cands.push_back({(uint32_t)x.d, x.slot});
    if (want0 > 0 && cands.size() > want0) {
        std::nth_element(cands.begin(), cands.begin() + (want0 - 1), cands.end());
        cands.resize(want0);
    }
    std::vector<uint32_t> slots;
    for (auto& c : cands) slots.push_back(c.second);
    if (cands_out) *cands_out = slots;
    size_t want = std::min(want0, slots.size());
    if (want == 0) return {};
    return rerank_exact(ix, q, slots, k);
}

struct Routed {
    std::vector<uint64_t> bits;
    std::vector<uint32_t> chosen;
    std::vector<float> cscore;
};

// route_batch (index.rs:1873-1980)
bool route_batch(const OIndex& ix, const float* data, size_t nq, size_t nprobe, float tc, float beta,
                 std::vector<Routed>& out) {
    if (!ix.two_stage || ix.cent_bits.empty()) return false;
    const size_t QB = 32, dim = ix.dim, nw = ix.nw, m = ix.M, cl = nw * 64;
    std::vector<uint8_t> live(m);
    size_t n_live = 0;
    for (size_t c = 0; c < m; ++c) {
        live[c] = ix.live(c);
        n_live += live[c];
    }
    size_t want_c = std::min(nprobe * std::max<size_t>(ix.shortlist_mult, 2), n_live);
    out.assign(nq, Routed{});
    if (want_c == 0) {
        for (auto& r : out) r.bits.assign(nw, 0);
        return true;
    }
    std::vector<uint64_t> qbits(nq * nw);
#pragma omp parallel
    {
        std::vector<float> rot(ix.dim_pad);
#pragma omp for schedule(static)
        for (long long qi = 0; qi < (long long)nq; ++qi) {
            rotate(data + qi * dim, dim, ix.signs.data(), ix.dim_pad, rot.data());
            pack_signs_trunc(rot.data(), ix.dim_pad, &qbits[qi * nw], nw);
        }
    }
    std::vector<std::vector<uint32_t>> shortlists(nq);
    size_t ntiles = (nq + QB - 1) / QB;
#pragma omp parallel for schedule(dynamic, 1)
    for (long long t = 0; t < (long long)ntiles; ++t) {
        size_t q0 = t * QB, bsz = std::min(QB, nq - q0);
        std::vector<uint16_t> hs(bsz * m);
        for (size_t c = 0; c < m; ++c)
            for (size_t bi = 0; bi < bsz; ++bi)
                hs[bi * m + c] = (uint16_t)hamming(&qbits[(q0 + bi) * nw], &ix.cent_bits[c * nw], nw);
        for (size_t bi = 0; bi < bsz; ++bi) {
            std::vector<uint16_t> row(hs.begin() + bi * m, hs.begin() + (bi + 1) * m);
            size_t cut = hamming_cutoff(row, live, want_c, cl);
            for (size_t c = 0; c < m; ++c)
                if (live[c] && row[c] <= cut) shortlists[q0 + bi].push_back((uint32_t)c);
        }
    }
    bool cent_q8 = ix.centroid_sq8 && !ix.cent_sq8.empty();
#pragma omp parallel for schedule(dynamic, 8)
    for (long long qi = 0; qi < (long long)nq; ++qi) {
        const float* q = data + qi * dim;
        std::vector<float> cqs(dim);
        float cqbase = 0.0f;
        if (cent_q8)
            for (size_t j = 0; j < dim; ++j) {
                cqs[j] = q[j] * ix.csq_step[j];
                cqbase += q[j] * ix.csq_min[j];
            }
        std::vector<std::pair<uint32_t, float>> cs;
        for (uint32_t ci : shortlists[qi]) cs.push_back({ci, cent_score(ix, ci, q, cqs.data(), cqbase)});
        Routed& r = out[qi];
        select_and_nucleus(cs, nprobe, tc, beta, r.chosen);
        for (size_t i = 0; i < r.chosen.size(); ++i) r.cscore.push_back(cs[i].second);
        r.bits.assign(qbits.begin() + qi * nw, qbits.begin() + (qi + 1) * nw);
    }
    return true;
}

struct Entry {
    uint32_t d, slot;
};

// search_batch_cellmajor, FastScan branch (index.rs:1999-2311). Returns per query the candidate
// slots that reach the rerank (in `cands`) and the final top-k.
int search_cellmajor(const OIndex& ix, const float* data, size_t nq, size_t k, size_t nprobe, float tc, float beta,
                     std::vector<std::vector<uint32_t>>& cands, std::vector<std::vector<std::pair<float, uint64_t>>>& res) {
    const size_t dim = ix.dim, nw = ix.nw, ma = ix.ma, M = ix.M;
    const bool poly = ma > 1;
    const size_t bb = nw * 64 * 32 / 8;
    const uint32_t dp = 255u * (uint32_t)nw * 16;
    const size_t want_final = std::max<size_t>(k * ix.rerank_factor, 1);
    const size_t target = want_final;
    const size_t SEED_CELLS = 8;
    const size_t mwords = (M + 63) / 64;

    std::vector<Routed> probes;
    if (!route_batch(ix, data, nq, nprobe, tc, beta, probes)) {
        probes.assign(nq, Routed{});
        int bad = 0;
#pragma omp parallel
        {
            SearchBuf b;
#pragma omp for schedule(dynamic, 8)
            for (long long qi = 0; qi < (long long)nq; ++qi) {
                if (route_query(ix, data + qi * dim, nprobe, tc, beta, b) < 0) {
#pragma omp atomic write
                    bad = 1;
                    continue;
                }
                probes[qi].chosen = b.chosen;
                for (size_t i = 0; i < b.chosen.size(); ++i) probes[qi].cscore.push_back(b.cscores[i].second);
            }
        }
        if (bad) return 7;
    }

    auto canonical = [&](uint32_t slot, uint32_t ci, const std::vector<uint64_t>& probed) {  // :2036-2045
        for (size_t j = 0; j < ma; ++j) {
            uint32_t h = ix.slot_cells[(size_t)slot * ma + j];
            if (h != UINT32_MAX && h < ci && ((probed[h >> 6] >> (h & 63)) & 1)) return false;
        }
        return true;
    };
    auto scan_cell = [&](size_t c, const FsQuery& fq, const std::vector<uint64_t>& probed, uint32_t t,
                         std::vector<Entry>& out) {  // :2048-2075
        size_t nmem = ix.members(c);
        if (nmem == 0) return;
        const uint32_t* mem = ix.member_ptr(c);
        size_t b0 = ix.fs_off[c], b1 = ix.fs_off[c + 1];
        uint16_t sums[32];
        for (size_t blk = b0; blk < b1; ++blk) {
            fs_block_sums_avx2(&ix.fs_codes[blk * bb], fq.lut.data(), fq.npos / 2, sums);
            size_t base = (blk - b0) * 32;
            size_t nv = std::min<size_t>(32, nmem - base);
            for (size_t i = 0; i < nv; ++i) {
                uint32_t d = fq.maxk - sums[i];
                if (d <= t) {
                    uint32_t slot = mem[base + i];
                    if (!poly || canonical(slot, (uint32_t)c, probed)) out.push_back({d, slot});
                }
            }
        }
    };
    struct R {
        std::vector<uint32_t> rest;
        std::vector<Entry> seed;
        uint32_t tau;
        FsQuery fq;
        std::vector<uint64_t> probed;
    };
    std::vector<R> routed(nq);
    const float norm = std::sqrt(2.0f * (float)ix.dim_pad / 3.14159265358979323846f);
#pragma omp parallel
    {
        std::vector<float> rot(ix.dim_pad);
#pragma omp for schedule(dynamic, 4)
        for (long long qi = 0; qi < (long long)nq; ++qi) {  // :2126-2191
            const auto& chosen = probes[qi].chosen;
            R& r = routed[qi];
            size_t ns = std::min(SEED_CELLS, chosen.size());
            if (poly) {
                r.probed.assign(mwords, 0);
                for (uint32_t c : chosen) r.probed[c >> 6] |= 1ull << (c & 63);
            }
            rotate(data + qi * dim, dim, ix.signs.data(), ix.dim_pad, rot.data());
            r.fq = fs_query(rot.data(), ix.dim_pad, nw);
            for (size_t i = 0; i < ns; ++i) scan_cell(chosen[i], r.fq, r.probed, dp, r.seed);
            uint32_t tau = dp;
            if (r.seed.size() >= target) {
                std::nth_element(r.seed.begin(), r.seed.begin() + (target - 1), r.seed.end(),
                                 [](const Entry& a, const Entry& b) { return a.d < b.d; });
                tau = r.seed[target - 1].d;
                r.seed.erase(std::remove_if(r.seed.begin(), r.seed.end(), [tau](const Entry& e) { return e.d > tau; }),
                             r.seed.end());
            }
            size_t rest_end = chosen.size();
            if (ix.adaptive && r.seed.size() >= target && ns < chosen.size()) {
                float thr = r.fq.estimate(r.fq.maxk - tau) / norm;
                thr = std::fmin(std::fmax(thr, -1.0f), 1.0f);
                size_t m = chosen.size();
                std::vector<float> suffix(m + 1, -INFINITY);
                for (size_t i = m; i-- > ns;) {
                    float ang = std::acos(std::fmin(std::fmax(probes[qi].cscore[i], -1.0f), 1.0f));
                    float bnd = std::cos(std::fmax(ang - ix.r_bound[chosen[i]], 0.0f));
                    suffix[i] = std::fmax(bnd, suffix[i + 1]);
                }
                for (size_t i = ns; i < m; ++i)
                    if (suffix[i] < thr - ix.at_margin) {
                        rest_end = i;
                        break;
                    }
            }
            r.rest.assign(chosen.begin() + ns, chosen.begin() + rest_end);
            r.tau = tau;
        }
    }
    // invert: cell -> queries, ascending (:2193-2213)
    std::vector<size_t> start(M + 1, 0);
    for (auto& r : routed)
        for (uint32_t c : r.rest) start[c + 1] += 1;
    for (size_t c = 0; c < M; ++c) start[c + 1] += start[c];
    std::vector<uint32_t> qof(start[M]);
    {
        std::vector<size_t> pos(start.begin(), start.end() - 1);
        for (size_t qi = 0; qi < nq; ++qi)
            for (uint32_t c : routed[qi].rest) qof[pos[c]++] = (uint32_t)qi;
    }
    // equal-work cell ranges (:2215-2229)
    size_t nthreads = (size_t)std::max(1, omp_get_max_threads());
    size_t ntask = nthreads * 4;
    std::vector<size_t> work(M);
    size_t total = 0;
    for (size_t c = 0; c < M; ++c) {
        work[c] = ix.members(c) * (start[c + 1] - start[c]);
        total += work[c];
    }
    total = std::max<size_t>(total, 1);
    std::vector<std::pair<size_t, size_t>> ranges;
    size_t c0 = 0, acc = 0;
    for (size_t c = 0; c < M; ++c) {
        acc += work[c];
        if (acc * ntask >= total * (ranges.size() + 1) || c + 1 == M) {
            ranges.push_back({c0, c + 1});
            c0 = c + 1;
        }
    }
    // scan with per-worker buffers and a shared per-query cut-off (:2231-2275)
    std::vector<std::atomic<uint32_t>> gtau(nq);
    for (size_t qi = 0; qi < nq; ++qi) gtau[qi].store(routed[qi].tau, std::memory_order_relaxed);
    std::vector<std::vector<std::vector<Entry>>> partials(ranges.size());
#pragma omp parallel for schedule(dynamic, 1)
    for (long long ri = 0; ri < (long long)ranges.size(); ++ri) {
        auto& bufs = partials[ri];
        bufs.assign(nq, {});
        std::vector<uint32_t> ltau(nq, dp);
        for (size_t c = ranges[ri].first; c < ranges[ri].second; ++c) {
            if (start[c] == start[c + 1] || ix.members(c) == 0) continue;
            for (size_t p = start[c]; p < start[c + 1]; ++p) {
                size_t qi = qof[p];
                auto& bq = bufs[qi];
                uint32_t t = std::min(ltau[qi], gtau[qi].load(std::memory_order_relaxed));
                size_t before = bq.size();
                scan_cell(c, routed[qi].fq, routed[qi].probed, t, bq);
                if (bq.size() > before) {
                    if (bq.size() >= 2 * target || (bq.size() >= target && t == dp)) {
                        std::nth_element(bq.begin(), bq.begin() + (target - 1), bq.end(),
                                         [](const Entry& a, const Entry& b) { return a.d < b.d; });
                        t = std::min(t, bq[target - 1].d);
                        uint32_t tt = t;
                        bq.erase(std::remove_if(bq.begin(), bq.end(), [tt](const Entry& e) { return e.d > tt; }),
                                 bq.end());
                    }
                }
                if (bq.size() >= target) {
                    uint32_t cur = gtau[qi].load(std::memory_order_relaxed);
                    while (t < cur && !gtau[qi].compare_exchange_weak(cur, t, std::memory_order_relaxed)) {
                    }
                }
                ltau[qi] = t;
            }
        }
    }
    // merge + exact cut + rerank (:2277-2308)
    cands.assign(nq, {});
    res.assign(nq, {});
#pragma omp parallel for schedule(dynamic, 4)
    for (long long qi = 0; qi < (long long)nq; ++qi) {
        uint32_t t = gtau[qi].load(std::memory_order_relaxed);
        std::vector<Entry> v;
        for (auto& e : routed[qi].seed)
            if (e.d <= t) v.push_back(e);
        for (auto& p : partials)
            for (auto& e : p[qi])
                if (e.d <= t) v.push_back(e);
        if (v.size() > target) {
            std::nth_element(v.begin(), v.begin() + (target - 1), v.end(),
                             [](const Entry& a, const Entry& b) { return a.d < b.d; });
            uint32_t cut = v[target - 1].d;
            v.erase(std::remove_if(v.begin(), v.end(), [cut](const Entry& e) { return e.d > cut; }), v.end());
        }
        std::vector<uint32_t> slots;
        for (auto& e : v) slots.push_back(e.slot);
        std::sort(slots.begin(), slots.end());
        res[qi] = rerank_exact(ix, data + qi * dim, slots, k);
        cands[qi] = std::move(slots);
    }
    return 0;
}

// ---- index build: an independent restatement of the reference's build path --------------------
//
// train_centroids (index.rs:2761-2804) -> hierarchical_kmeans / kmeans_spherical
// (tree.rs:160-348); add_batch (index.rs:2987-3212) with assign_cells_routed / assign_cells /
// pick_orthogonal / append_parallel (index.rs:2442-2667); refresh_derived (index.rs:684-878:
// radii, centroid codes, SQ8 centroids, tree via CentroidTree::build + compact_layout,
// tree.rs:354-540); compact (index.rs:3565-3569 -> compact_arena :929-1112). Written from the
// reference source, not from the product's host build, so that a mistake in either shows up as
// an array mismatch (tests/test_oracle_build.py). Only first-batch builds (no deletes, no reused
// slots) are restated: that is all any benchmark or test here builds.

void normalize_rows(float* v, size_t n) {  // tree.rs:163-172 and the loop in index.rs:2787-2794
    float s = 0.0f;
    for (size_t i = 0; i < n; ++i) s += v[i] * v[i];
    s = std::sqrt(s);
    if (s > 1e-12f)
        for (size_t i = 0; i < n; ++i) v[i] /= s;
}

// kmeans_spherical (tree.rs:179-248): strided seeding, Lloyd iterations with the AVX2 dot, first
// maximum wins; per-cluster sums accumulated in point order (grouped by cluster so clusters sum in
// parallel: every cluster still adds its points in ascending index order, as the serial loop does);
// empty clusters reseeded from a xorshift64 stream seeded with seed | 1.
void kmeans_spherical(const float* x, size_t n, size_t dim, size_t k_in, size_t iters, uint64_t seed,
                      std::vector<uint32_t>& assign, std::vector<float>& cents) {
    size_t k = std::min(std::max<size_t>(k_in, 1), n);
    cents.assign(k * dim, 0.0f);
    size_t stride = std::max<size_t>(n / k, 1);
    for (size_t j = 0; j < k; ++j) {
        size_t src = std::min(j * stride, n - 1);
        std::memcpy(&cents[j * dim], x + src * dim, dim * sizeof(float));
    }
    assign.assign(n, 0);
    uint64_t state = seed | 1;
    auto next_u = [&state]() {
        state ^= state << 13;
        state ^= state >> 7;
        state ^= state << 17;
        return state;
    };
    std::vector<size_t> start(k + 1), order(n);
    std::vector<float> sums(k * dim);
    for (size_t it = 0; it < iters; ++it) {
#pragma omp parallel for schedule(static)
        for (size_t i = 0; i < n; ++i) {
            const float* v = x + i * dim;
            uint32_t best = 0;
            float best_s = -INFINITY;
            for (size_t j = 0; j < k; ++j) {
                float s = dot_f32(v, &cents[j * dim], dim);
                if (s > best_s) {
                    best_s = s;
                    best = (uint32_t)j;
                }
            }
            assign[i] = best;
        }
        std::fill(start.begin(), start.end(), 0);
        for (size_t i = 0; i < n; ++i) ++start[assign[i] + 1];
        for (size_t j = 0; j < k; ++j) start[j + 1] += start[j];
        {
            std::vector<size_t> pos(start.begin(), start.end() - 1);
            for (size_t i = 0; i < n; ++i) order[pos[assign[i]]++] = i;
        }
#pragma omp parallel for schedule(dynamic, 16)
        for (size_t j = 0; j < k; ++j) {
            float* s = &sums[j * dim];
            std::fill(s, s + dim, 0.0f);
            for (size_t r = start[j]; r < start[j + 1]; ++r) {
                const float* v = x + order[r] * dim;
                for (size_t t = 0; t < dim; ++t) s[t] += v[t];
            }
        }
        for (size_t j = 0; j < k; ++j) {
            if (start[j + 1] == start[j]) {
                size_t src = (size_t)(next_u() % (uint64_t)n);
                std::memcpy(&cents[j * dim], x + src * dim, dim * sizeof(float));
                continue;
            }
            std::memcpy(&cents[j * dim], &sums[j * dim], dim * sizeof(float));
            normalize_rows(&cents[j * dim], dim);
        }
    }
}

// hierarchical_kmeans (tree.rs:257-348): sqrt(k) top-level groups (8 iterations), sub-cluster
// counts proportional to group size by the sequential budget rule, 12 iterations per group with
// seed ^ (g + 1) * 0x9E3779B9, shortfall rows filled from the data at (fill * 7919) % n.
std::vector<float> hierarchical_kmeans(const float* x, size_t n, size_t dim, size_t k_in, uint64_t seed) {
    size_t k = std::min(std::max<size_t>(k_in, 1), n);
    std::vector<uint32_t> asg;
    std::vector<float> c;
    if (k <= 64 || n <= k * 4) {
        kmeans_spherical(x, n, dim, k, 12, seed, asg, c);
        return c;
    }
    size_t k1 = (size_t)std::ceil(std::sqrt((double)k));
    kmeans_spherical(x, n, dim, k1, 8, seed, asg, c);
    std::vector<std::vector<uint32_t>> groups(k1);
    for (size_t i = 0; i < n; ++i) groups[asg[i]].push_back((uint32_t)i);
    std::vector<size_t> subs(k1, 0), offs(k1, 0);
    size_t written = 0, before = 0;
    for (size_t g = 0; g < k1; ++g) {
        size_t glen = groups[g].size();
        size_t seen = before;  // points in groups[..g]
        before += glen;
        if (glen == 0 || written >= k) continue;
        size_t remaining_groups = k1 - g;
        double denom = (double)std::max<size_t>(n - seen, 1);
        size_t want = (size_t)std::round((double)(k - written) * (double)glen / denom);
        size_t sub = std::min(std::min(std::max<size_t>(want, 1), k - written), glen);
        if (remaining_groups == 1) sub = std::max<size_t>(std::min(k - written, glen), 1);
        if (sub == 0) continue;
        subs[g] = std::min(sub, k - written);
        offs[g] = written;
        written += subs[g];
    }
    std::vector<float> out(k * dim, 0.0f);
    std::vector<size_t> todo;
    for (size_t g = 0; g < k1; ++g)
        if (subs[g] > 0) todo.push_back(g);
    // Sub-clusterings are independent and write disjoint rows (inner parallel regions run serially).
#pragma omp parallel for schedule(dynamic, 1)
    for (size_t t = 0; t < todo.size(); ++t) {
        size_t g = todo[t];
        const auto& idx = groups[g];
        std::vector<float> buf(idx.size() * dim);
        for (size_t r = 0; r < idx.size(); ++r) std::memcpy(&buf[r * dim], x + (size_t)idx[r] * dim, dim * 4);
        std::vector<uint32_t> a2;
        std::vector<float> cs;
        kmeans_spherical(buf.data(), idx.size(), dim, subs[g], 12, seed ^ ((uint64_t)g + 1) * 0x9E3779B9ull, a2, cs);
        std::memcpy(&out[offs[g] * dim], cs.data(), subs[g] * dim * sizeof(float));
    }
    size_t fill = 0;
    while (written < k) {
        size_t src = (fill * 7919) % n;
        std::memcpy(&out[written * dim], x + src * dim, dim * sizeof(float));
        ++written;
        ++fill;
    }
    return out;
}

struct BLevel {  // tree.rs:74-83
    size_t n = 0;
    std::vector<float> cents;
    std::vector<uint64_t> codes;
    std::vector<uint32_t> child_start, child_len, child_idx;
};

struct BCell {  // index.rs:361-395
    std::vector<uint32_t> members;
    std::vector<float> sum, centroid;
    float r_bound = 0.0f, r_max = 0.0f;
};

// The index under construction, with the reference's defaults (index.rs:2672-2755).
struct OBuild {
    size_t dim = 0, dim_pad = 0, nw = 0, rerank_factor = 4;
    uint64_t seed = 0x5EED;
    std::vector<float> signs;
    bool two_stage = false, centroid_sq8 = true, tree_route = true, graph_route = true, fastscan = false;
    bool per_dim_sq = false, i8_rerank = false, keep_f32 = true, adaptive = false, compacted = false;
    size_t shortlist_mult = 4, tree_min_cells = 2048, tree_fanout = 64, graph_min_cells = 65536;
    size_t max_assign = 1, cm_min_batch = 32, n_live = 0, tree_cells = 0;
    float tree_beam_frac = 0.5f, spill_margin = 0.0f, spill_lambda = 0.0f, at_margin = 0.02f, quant_scale = 0.0f;
    // arena
    std::vector<uint64_t> bits, ext_ids;
    std::vector<int8_t> scan_i8;
    std::vector<float> vecs_f32, sq_min, sq_step;
    std::vector<uint32_t> slot_cell, slot_cells;
    std::vector<uint32_t> free_slots;                 // freed by remove, refilled LIFO by add
    std::unordered_map<uint64_t, uint32_t> id_to_slot;
    // cells and derived state
    std::vector<BCell> cells;
    std::vector<uint64_t> cent_bits;
    std::vector<uint8_t> cent_sq8;
    std::vector<float> csq_min, csq_step;
    bool has_tree = false;
    std::vector<BLevel> levels;  // coarsest first, after compact_layout
    std::vector<uint64_t> leaf_codes;
    std::vector<uint32_t> leaf_ids;
    float tree_bf = 0.5f;
    // compacted layout
    std::vector<uint32_t> prim_len, rep_off;
    std::vector<uint8_t> fs_codes;
    std::vector<uint32_t> fs_off;
    // the tree as tree_search reads it
    OIndex tview;

    void code_of(const float* v, std::vector<float>& rot, uint64_t* out) const {
        rotate(v, dim, signs.data(), dim_pad, rot.data());
        pack_signs_trunc(rot.data(), dim_pad, out, nw);
    }
    size_t live_cells() const {
        size_t c = 0;
        for (auto& cl : cells) c += !cl.members.empty();
        return c;
    }
};

// CentroidTree::build (tree.rs:354-453) and compact_layout / permute_level / permute_leaves
// (tree.rs:455-540).
void tree_build(OBuild& b, const std::vector<uint32_t>& ids) {
    b.has_tree = false;
    b.levels.clear();
    b.leaf_codes.clear();
    b.leaf_ids.clear();
    size_t m = ids.size(), dim = b.dim, nw = b.nw;
    if (m < 2 || nw == 0) return;
    size_t fanout = std::max<size_t>(b.tree_fanout, 2);
    std::vector<float> rot(b.dim_pad), cur((size_t)m * dim);
    for (size_t i = 0; i < m; ++i) std::memcpy(&cur[i * dim], b.cells[ids[i]].centroid.data(), dim * 4);
    std::vector<uint64_t> leaf(m * nw);
    for (size_t i = 0; i < m; ++i) b.code_of(&cur[i * dim], rot, &leaf[i * nw]);
    std::vector<BLevel> rev;
    size_t cur_n = m;
    while (cur_n > 256) {  // TOP_MAX, tree.rs:41
        size_t k = std::max<size_t>((cur_n + fanout - 1) / fanout, 1);
        if (k >= cur_n) break;
        std::vector<uint32_t> asg;
        std::vector<float> parents;
        kmeans_spherical(cur.data(), cur_n, dim, k, 10, 0x9E3779B97F4A7C15ull, asg, parents);
        BLevel L;
        L.n = k;
        L.child_len.assign(k, 0);
        for (uint32_t a : asg) ++L.child_len[a];
        L.child_start.assign(k, 0);
        uint32_t acc = 0;
        for (size_t j = 0; j < k; ++j) {
            L.child_start[j] = acc;
            acc += L.child_len[j];
        }
        std::vector<uint32_t> fillp = L.child_start;
        L.child_idx.assign(cur_n, 0);
        for (size_t i = 0; i < cur_n; ++i) L.child_idx[fillp[asg[i]]++] = (uint32_t)i;
        L.codes.resize(k * nw);
        for (size_t j = 0; j < k; ++j) b.code_of(&parents[j * dim], rot, &L.codes[j * nw]);
        L.cents = parents;
        rev.push_back(std::move(L));
        cur = std::move(parents);
        cur_n = k;
    }
    if (rev.empty()) return;
    std::reverse(rev.begin(), rev.end());
    std::vector<uint32_t> lids = ids;
    for (size_t i = 0; i < rev.size(); ++i) {
        std::vector<uint32_t> order = rev[i].child_idx;
        if (i + 1 < rev.size()) {
            BLevel& l = rev[i + 1];
            if (order.size() == l.n) {
                BLevel p;
                p.n = l.n;
                p.cents.resize(l.n * dim);
                p.codes.resize(l.n * nw);
                p.child_start.resize(l.n);
                p.child_len.resize(l.n);
                uint32_t acc = 0;
                for (size_t np_ = 0; np_ < order.size(); ++np_) {
                    size_t o = order[np_];
                    std::memcpy(&p.cents[np_ * dim], &l.cents[o * dim], dim * 4);
                    std::memcpy(&p.codes[np_ * nw], &l.codes[o * nw], nw * 8);
                    p.child_start[np_] = acc;
                    p.child_len[np_] = l.child_len[o];
                    acc += l.child_len[o];
                    p.child_idx.insert(p.child_idx.end(), l.child_idx.begin() + l.child_start[o],
                                       l.child_idx.begin() + l.child_start[o] + l.child_len[o]);
                }
                l = std::move(p);
            }
        } else {
            std::vector<uint64_t> codes(order.size() * nw);
            std::vector<uint32_t> nids(order.size());
            for (size_t np_ = 0; np_ < order.size(); ++np_) {
                std::memcpy(&codes[np_ * nw], &leaf[(size_t)order[np_] * nw], nw * 8);
                nids[np_] = lids[order[np_]];
            }
            leaf = std::move(codes);
            lids = std::move(nids);
        }
        for (size_t t = 0; t < rev[i].child_idx.size(); ++t) rev[i].child_idx[t] = (uint32_t)t;
    }
    b.levels = std::move(rev);
    b.leaf_codes = std::move(leaf);
    b.leaf_ids = std::move(lids);
    b.tree_bf = b.tree_beam_frac > 0.0f ? b.tree_beam_frac : 0.5f;
    b.has_tree = true;
    // the view tree_search reads (tree.rs:574-628)
    OIndex& t = b.tview;
    t.nw = nw;
    t.beam_frac = b.tree_bf;
    t.levels.clear();
    for (auto& L : b.levels) {
        Level v;
        v.n = L.n;
        v.codes = L.codes;
        v.child_start = L.child_start;
        v.child_len = L.child_len;
        t.levels.push_back(std::move(v));
    }
    t.leaf_codes = b.leaf_codes;
    t.leaf_ids = b.leaf_ids;
    t.n_leaf = b.leaf_ids.size();
}

// rebuild_centroid_tree (index.rs:684-708)
void rebuild_tree(OBuild& b) {
    b.tree_cells = b.live_cells();
    std::vector<uint32_t> live;
    for (size_t i = 0; i < b.cells.size(); ++i)
        if (!b.cells[i].members.empty()) live.push_back((uint32_t)i);
    if (live.empty() && !b.cells.empty())
        for (size_t i = 0; i < b.cells.size(); ++i) live.push_back((uint32_t)i);
    if (!b.tree_route || live.size() < b.tree_min_cells) {
        b.has_tree = false;
        b.levels.clear();
        return;
    }
    tree_build(b, live);
}

// recompute_radii (index.rs:817-861): p99 and max of the member angles acos(clamp(mu . v)).
void recompute_radii(OBuild& b) {
    size_t dim = b.dim;
    float inv = b.quant_scale > 0.0f ? 1.0f / b.quant_scale : 1.0f;
#pragma omp parallel for schedule(dynamic, 8)
    for (size_t ci = 0; ci < b.cells.size(); ++ci) {
        BCell& c = b.cells[ci];
        if (c.members.empty()) {
            c.r_bound = c.r_max = 0.0f;
            continue;
        }
        const float* mu = c.centroid.data();
        std::vector<float> w;
        float base = 0.0f;
        if (b.per_dim_sq) {
            w.resize(dim);
            for (size_t j = 0; j < dim; ++j) w[j] = b.sq_step[j] * mu[j];
            for (size_t j = 0; j < dim; ++j) base += b.sq_min[j] * mu[j];
        }
        std::vector<float> angs;
        angs.reserve(c.members.size());
        for (uint32_t s : c.members) {
            size_t off = (size_t)s * dim;
            float dot;
            if (b.per_dim_sq)
                dot = dot_f32_u8(w.data(), &b.scan_i8[off], dim) + base;
            else if (b.keep_f32)
                dot = dot_f32(mu, &b.vecs_f32[off], dim);
            else
                dot = dot_f32_i8(mu, &b.scan_i8[off], dim) * inv;
            dot = std::min(std::max(dot, -1.0f), 1.0f);
            angs.push_back(std::acos(dot));
        }
        size_t len = angs.size();
        size_t p99 = (size_t)std::ceil((float)len * 0.99f);
        p99 = std::min(p99 == 0 ? 0 : p99 - 1, len - 1);
        float mx = -INFINITY;
        for (float a : angs) mx = std::max(mx, a);
        std::nth_element(angs.begin(), angs.begin() + p99, angs.end());
        c.r_bound = angs[p99];
        c.r_max = mx;
    }
}

// rebuild_centroid_codes (index.rs:711-723)
void rebuild_codes(OBuild& b) {
    std::vector<float> rot(b.dim_pad);
    b.cent_bits.assign(b.cells.size() * b.nw, 0);
    for (size_t ci = 0; ci < b.cells.size(); ++ci) b.code_of(b.cells[ci].centroid.data(), rot, &b.cent_bits[ci * b.nw]);
}

// rebuild_centroid_sq8 (index.rs:730-770): range over live centroids, step floor 1e-12,
// round-half-away codes clamped to [0, 255], one row for every cell.
void rebuild_sq8(OBuild& b) {
    size_t d = b.dim;
    std::vector<float> lo(d, INFINITY), hi(d, -INFINITY);
    bool any = false;
    for (auto& c : b.cells) {
        if (c.members.empty()) continue;
        any = true;
        for (size_t j = 0; j < d; ++j) {
            float v = c.centroid[j];
            if (v < lo[j]) lo[j] = v;
            if (v > hi[j]) hi[j] = v;
        }
    }
    b.cent_sq8.clear();
    b.csq_min.clear();
    b.csq_step.clear();
    if (!any) return;
    b.csq_step.resize(d);
    for (size_t j = 0; j < d; ++j) {
        float s = (hi[j] - lo[j]) / 255.0f;
        b.csq_step[j] = s > 1e-12f ? s : 1e-12f;
    }
    b.csq_min = lo;
    b.cent_sq8.assign(b.cells.size() * d, 0);
    for (size_t ci = 0; ci < b.cells.size(); ++ci)
        for (size_t j = 0; j < d; ++j) {
            float q = std::round((b.cells[ci].centroid[j] - b.csq_min[j]) / b.csq_step[j]);
            b.cent_sq8[ci * d + j] = (uint8_t)std::min(std::max(q, 0.0f), 255.0f);
        }
}

// refresh_derived (index.rs:864-878); the centroid graph is not restated (off in both presets).
void refresh_derived(OBuild& b) {
    recompute_radii(b);
    if (b.two_stage) rebuild_codes(b);
    if (b.centroid_sq8) rebuild_sq8(b);
    if (!(b.has_tree && b.tree_cells == b.live_cells())) rebuild_tree(b);  // maybe_rebuild, :667-677
}

// Descending score; exact ties by ascending cell id (the reference's unstable sorts leave them in
// an unspecified order; the product uses the same rule).
inline bool by_score_then_id(const std::pair<uint32_t, float>& a, const std::pair<uint32_t, float>& b) {
    if (a.second != b.second) return a.second > b.second;
    return a.first < b.first;
}

// pick_orthogonal (index.rs:2523-2560): nearest cell first, then greedily the lowest
// ||r||^2 + lambda * sum_h (r . r_h / ||r_h||)^2 over the 16 best candidates.
std::vector<uint32_t> pick_orthogonal(const OBuild& b, std::vector<std::pair<uint32_t, float>>& scored) {
    size_t pool = std::min<size_t>(16, scored.size());
    std::sort(scored.begin(), scored.end(), by_score_then_id);
    scored.resize(pool);
    size_t r = std::min(b.max_assign, scored.size());
    std::vector<std::pair<uint32_t, float>> homes{scored[0]};
    std::vector<uint8_t> taken(scored.size(), 0);
    taken[0] = 1;
    while (homes.size() < r) {
        size_t bj = SIZE_MAX;
        float bl = INFINITY;
        for (size_t j = 0; j < scored.size(); ++j) {
            if (taken[j]) continue;
            uint32_t cj = scored[j].first;
            float sj = scored[j].second;
            float loss = 2.0f - 2.0f * sj;
            for (auto& h : homes) {
                float sh = h.second;
                float rn = std::sqrt(std::max(2.0f - 2.0f * sh, 1e-12f));
                float g = dot_f32(b.cells[h.first].centroid.data(), b.cells[cj].centroid.data(), b.dim);
                float p = (1.0f - sh - sj + g) / rn;
                loss += b.spill_lambda * p * p;
            }
            if (loss < bl) {
                bl = loss;
                bj = j;
            }
        }
        if (bj == SIZE_MAX) break;
        taken[bj] = 1;
        homes.push_back(scored[bj]);
    }
    std::vector<uint32_t> out;
    for (auto& h : homes) out.push_back(h.first);
    return out;
}

// The home choice shared by assign_cells and assign_cells_routed once candidates are scored
// (index.rs:2466-2477, :2489-2504).
std::vector<uint32_t> choose_homes(const OBuild& b, std::vector<std::pair<uint32_t, float>>& scored) {
    if (b.max_assign <= 1) {
        auto best = scored[0];
        for (auto& s : scored)
            if (s.second > best.second) best = s;
        return {best.first};
    }
    if (b.spill_lambda > 0.0f) return pick_orthogonal(b, scored);
    size_t r = std::min(b.max_assign, scored.size());
    std::sort(scored.begin(), scored.end(), by_score_then_id);
    scored.resize(r);
    float cutoff = scored[0].second - b.spill_margin;
    std::vector<uint32_t> out;
    for (auto& s : scored)
        if (s.second >= cutoff) out.push_back(s.first);
    return out;
}

// assign_cells_routed (index.rs:2442-2478) with its flat fallback assign_cells (:2480-2505).
std::vector<uint32_t> assign_cells(const OBuild& b, const float* v, std::vector<float>& rot,
                                   std::vector<uint64_t>& qb, std::vector<uint32_t>& tout) {
    std::vector<std::pair<uint32_t, float>> scored;
    if (b.has_tree) {
        b.code_of(v, rot, qb.data());
        size_t want = std::max<size_t>(64, b.max_assign * 8);  // ASSIGN_CANDIDATES, index.rs:401
        tree_search(b.tview, qb.data(), want, tout);
        for (uint32_t ci : tout) scored.push_back({ci, dot_f32(v, b.cells[ci].centroid.data(), b.dim)});
    }
    if (scored.empty())
        for (size_t ci = 0; ci < b.cells.size(); ++ci)
            scored.push_back({(uint32_t)ci, dot_f32(v, b.cells[ci].centroid.data(), b.dim)});
    return choose_homes(b, scored);
}

// train_centroids (index.rs:2761-2804)
int build_train(OBuild& b, const float* data, size_t n_all, size_t n_cells, size_t sample, uint64_t sd) {
    if (n_all == 0) return 1;
    size_t dim = b.dim;
    std::vector<float> train;
    size_t n_train = n_all;
    const float* tp = data;
    if (sample > 0 && n_all > sample) {
        size_t stride = n_all / sample;
        train.resize(sample * dim);
        for (size_t i = 0; i < sample; ++i) {
            size_t s = std::min(i * stride, n_all - 1);
            std::memcpy(&train[i * dim], data + s * dim, dim * 4);
        }
        n_train = sample;
        tp = train.data();
    }
    std::vector<float> cents = hierarchical_kmeans(tp, n_train, dim, n_cells, sd);
    size_t m = cents.size() / dim;
    b.cells.assign(m, BCell());
    for (size_t c = 0; c < m; ++c) {
        normalize_rows(&cents[c * dim], dim);
        b.cells[c].sum.assign(dim, 0.0f);
        b.cells[c].centroid.assign(cents.begin() + c * dim, cents.begin() + (c + 1) * dim);
    }
    refresh_derived(b);
    return 0;
}

// Cell::recompute_centroid (index.rs:379-392)
void recompute_centroid(BCell& c, size_t dim) {
    if (c.members.empty()) return;
    float nrm = 0.0f;
    for (float v : c.sum) nrm += v * v;
    nrm = std::sqrt(nrm);
    if (nrm > 1e-12f)
        for (size_t j = 0; j < dim; ++j) c.centroid[j] = c.sum[j] / nrm;
}

// fork_empty (index.rs:2330-2400): a new empty index with this one's configuration, rotation,
// quantisation parameters and centroids (sums zero, no members); FastScan off, not compacted;
// derived state refreshed (so its tree covers every cell until the first insert).
void build_fork(const OBuild& src, OBuild& f) {
    f.dim = src.dim;
    f.dim_pad = src.dim_pad;
    f.nw = src.nw;
    f.rerank_factor = src.rerank_factor;
    f.seed = src.seed;
    f.signs = src.signs;
    f.graph_route = src.graph_route;
    f.graph_min_cells = src.graph_min_cells;
    f.tree_route = src.tree_route;
    f.tree_min_cells = src.tree_min_cells;
    f.tree_fanout = src.tree_fanout;
    f.tree_beam_frac = src.tree_beam_frac;
    f.tree_cells = 0;
    f.two_stage = src.two_stage;
    f.centroid_sq8 = src.centroid_sq8;
    f.shortlist_mult = src.shortlist_mult;
    f.quant_scale = src.quant_scale;
    f.n_live = 0;
    f.max_assign = src.max_assign;
    f.spill_margin = src.spill_margin;
    f.spill_lambda = src.spill_lambda;
    f.compacted = false;
    f.fastscan = false;
    f.i8_rerank = src.i8_rerank;
    f.per_dim_sq = src.per_dim_sq;
    f.sq_min = src.sq_min;
    f.sq_step = src.sq_step;
    f.keep_f32 = src.keep_f32;
    f.adaptive = src.adaptive;
    f.at_margin = src.at_margin;
    f.cm_min_batch = src.cm_min_batch;
    f.cells.resize(src.cells.size());
    for (size_t c = 0; c < src.cells.size(); ++c) {
        f.cells[c].centroid = src.cells[c].centroid;
        f.cells[c].sum.assign(src.dim, 0.0f);
    }
    refresh_derived(f);
}

// add_batch (index.rs:2987-3212): scale and SQ8 fit from the first batch, parallel placement, the
// serial refill of freed slots (LIFO, :3076-3198), append_parallel for the rest (:2566-2667),
// centroid update, derived state.
int build_add(OBuild& b, const uint64_t* ids, const float* data, size_t n) {
    if (b.cells.empty()) return 1;
    size_t dim = b.dim, nw = b.nw, ma = b.max_assign;
    b.compacted = false;
    if (b.quant_scale == 0.0f) {
        float mx = 0.0f;
        for (size_t i = 0; i < n * dim; ++i) mx = std::max(mx, std::fabs(data[i]));
        b.quant_scale = mx > 0.0f ? 127.0f / mx : 1.0f;
    }
    if (b.per_dim_sq && b.sq_min.empty()) {
        std::vector<float> lo(dim, INFINITY), hi(dim, -INFINITY);
        for (size_t i = 0; i < n; ++i)
            for (size_t j = 0; j < dim; ++j) {
                float x = data[i * dim + j];
                lo[j] = std::min(lo[j], x);
                hi[j] = std::max(hi[j], x);
            }
        b.sq_step.resize(dim);
        for (size_t j = 0; j < dim; ++j) b.sq_step[j] = std::max(hi[j] - lo[j], 1e-9f) / 255.0f;
        b.sq_min = lo;
    }
    std::vector<std::vector<uint32_t>> asg(n);
#pragma omp parallel
    {
        std::vector<float> rot(b.dim_pad);
        std::vector<uint64_t> qb(nw);
        std::vector<uint32_t> tout;
#pragma omp for schedule(dynamic, 256)
        for (size_t i = 0; i < n; ++i) asg[i] = assign_cells(b, data + i * dim, rot, qb, tout);
    }
    const bool store_i8 = b.i8_rerank;
    auto encode_i8 = [&](const float* v, int8_t* o) {
        for (size_t j = 0; j < dim; ++j) {
            if (b.per_dim_sq) {
                float q = std::round((v[j] - b.sq_min[j]) / b.sq_step[j]);
                o[j] = (int8_t)(uint8_t)std::min(std::max(q, 0.0f), 255.0f);
            } else {
                float q = std::round(v[j] * b.quant_scale);
                o[j] = (int8_t)std::min(std::max(q, -127.0f), 127.0f);
            }
        }
    };
    // freed slots first, one vector at a time
    const size_t n_reuse = std::min(b.free_slots.size(), n);
    {
        std::vector<float> rot(b.dim_pad);
        for (size_t i = 0; i < n_reuse; ++i) {
            const float* v = data + i * dim;
            uint32_t slot = b.free_slots.back();
            b.free_slots.pop_back();
            size_t off = (size_t)slot * dim;
            if (b.keep_f32) std::copy(v, v + dim, b.vecs_f32.begin() + off);
            b.code_of(v, rot, &b.bits[(size_t)slot * nw]);
            if (store_i8) encode_i8(v, &b.scan_i8[off]);
            b.ext_ids[slot] = ids[i];
            b.slot_cell[slot] = asg[i][0];
            for (size_t j = 0; j < ma; ++j) b.slot_cells[(size_t)slot * ma + j] = j < asg[i].size() ? asg[i][j] : UINT32_MAX;
            for (size_t j = 0; j < asg[i].size(); ++j) {
                BCell& c = b.cells[asg[i][j]];
                c.members.push_back(slot);
                if (j == 0)
                    for (size_t t = 0; t < dim; ++t) c.sum[t] += v[t];
            }
            b.id_to_slot[ids[i]] = slot;
            b.n_live += 1;
        }
    }
    // the rest appended to the arena
    const size_t na = n - n_reuse;
    const float* adata = data + n_reuse * dim;
    const uint64_t* aids = ids + n_reuse;
    const std::vector<uint32_t>* aasg = asg.data() + n_reuse;
    size_t base = b.ext_ids.size();
    if (b.keep_f32) b.vecs_f32.insert(b.vecs_f32.end(), adata, adata + na * dim);
    b.bits.resize((base + na) * nw);
    if (store_i8) b.scan_i8.resize((base + na) * dim);
#pragma omp parallel
    {
        std::vector<float> rot(b.dim_pad);
#pragma omp for schedule(static)
        for (size_t i = 0; i < na; ++i) {
            const float* v = adata + i * dim;
            b.code_of(v, rot, &b.bits[(base + i) * nw]);
            if (store_i8) encode_i8(v, &b.scan_i8[(base + i) * dim]);
        }
    }
    for (size_t i = 0; i < na; ++i) {
        uint32_t slot = (uint32_t)(base + i);
        b.ext_ids.push_back(aids[i]);
        b.slot_cell.push_back(aasg[i][0]);
        for (size_t j = 0; j < ma; ++j) b.slot_cells.push_back(j < aasg[i].size() ? aasg[i][j] : UINT32_MAX);
        for (uint32_t ci : aasg[i]) b.cells[ci].members.push_back(slot);
        b.id_to_slot[aids[i]] = slot;
    }
    b.n_live += na;
    // primary sums: each cell adds its own appended vectors in input order
    size_t m = b.cells.size();
    std::vector<size_t> st(m + 1, 0), ord(na);
    for (size_t i = 0; i < na; ++i) ++st[aasg[i][0] + 1];
    for (size_t c = 0; c < m; ++c) st[c + 1] += st[c];
    {
        std::vector<size_t> pos(st.begin(), st.end() - 1);
        for (size_t i = 0; i < na; ++i) ord[pos[aasg[i][0]]++] = i;
    }
#pragma omp parallel for schedule(dynamic, 16)
    for (size_t c = 0; c < m; ++c) {
        float* s = b.cells[c].sum.data();
        for (size_t r = st[c]; r < st[c + 1]; ++r) {
            const float* v = adata + ord[r] * dim;
            for (size_t j = 0; j < dim; ++j) s[j] += v[j];
        }
    }
    for (auto& c : b.cells) recompute_centroid(c, dim);
    refresh_derived(b);
    return 0;
}

// remove (index.rs:3223-3276): the vector leaves its primary cell's sum (read back from whichever
// store exists), is swap-removed from every home's member list, and its slot is freed. The derived
// routing state is not refreshed.
bool build_remove(OBuild& b, uint64_t id) {
    auto it = b.id_to_slot.find(id);
    if (it == b.id_to_slot.end()) return false;
    uint32_t slot = it->second;
    b.id_to_slot.erase(it);
    b.compacted = false;
    size_t dim = b.dim, ma = b.max_assign, primary = b.slot_cell[slot], vs = (size_t)slot * dim;
    BCell& pc = b.cells[primary];
    if (b.keep_f32) {
        for (size_t j = 0; j < dim; ++j) pc.sum[j] -= b.vecs_f32[vs + j];
    } else if (b.per_dim_sq) {
        for (size_t j = 0; j < dim; ++j) pc.sum[j] -= (float)(uint8_t)b.scan_i8[vs + j] * b.sq_step[j] + b.sq_min[j];
    } else {
        float inv = 1.0f / b.quant_scale;
        for (size_t j = 0; j < dim; ++j) pc.sum[j] -= (float)b.scan_i8[vs + j] * inv;
    }
    for (size_t j = 0; j < ma; ++j) {
        uint32_t ci = b.slot_cells[(size_t)slot * ma + j];
        if (ci == UINT32_MAX) continue;
        auto& mem = b.cells[ci].members;
        for (size_t p = 0; p < mem.size(); ++p)
            if (mem[p] == slot) {
                mem[p] = mem.back();
                mem.pop_back();
                break;
            }
        b.slot_cells[(size_t)slot * ma + j] = UINT32_MAX;
    }
    recompute_centroid(pc, dim);
    b.free_slots.push_back(slot);
    b.n_live -= 1;
    return true;
}

// compact_arena (index.rs:929-1112): cluster-major renumbering by primary cell, member lists
// remapped and sorted, polysemic runs (primaries ascending, then replicas ascending), FastScan
// blocks of 32 members per cell.
void build_compact(OBuild& b) {
    size_t old_n = b.ext_ids.size();
    if (old_n == 0) return;
    size_t dim = b.dim, nw = b.nw, ma = b.max_assign;
    std::vector<uint32_t> new_of_old(old_n, UINT32_MAX), old_of_new;
    old_of_new.reserve(b.n_live);
    for (size_t ci = 0; ci < b.cells.size(); ++ci)
        for (uint32_t s : b.cells[ci].members) {
            if (b.slot_cell[s] != ci || new_of_old[s] != UINT32_MAX) continue;
            new_of_old[s] = (uint32_t)old_of_new.size();
            old_of_new.push_back(s);
        }
    {
        // live slots the loop above missed (none in a consistent index), in slot order; freed
        // slots are dropped
        std::vector<uint8_t> live(old_n, 0);
        for (auto& kv : b.id_to_slot) live[kv.second] = 1;
        for (size_t s = 0; s < old_n; ++s)
            if (live[s] && new_of_old[s] == UINT32_MAX) {
                new_of_old[s] = (uint32_t)old_of_new.size();
                old_of_new.push_back((uint32_t)s);
            }
    }
    size_t nn = old_of_new.size();
    auto permute = [&](auto& arr, size_t w) {
        if (arr.empty()) return;
        std::remove_reference_t<decltype(arr)> v(nn * w);
        for (size_t ns = 0; ns < nn; ++ns)
            std::copy(arr.begin() + (size_t)old_of_new[ns] * w, arr.begin() + ((size_t)old_of_new[ns] + 1) * w,
                      v.begin() + ns * w);
        arr.swap(v);
    };
    if (b.keep_f32) permute(b.vecs_f32, dim);
    permute(b.scan_i8, dim);
    permute(b.bits, nw);
    permute(b.ext_ids, 1);
    permute(b.slot_cell, 1);
    permute(b.slot_cells, ma);
    for (auto& c : b.cells) {
        c.members.erase(std::remove_if(c.members.begin(), c.members.end(),
                                       [&](uint32_t mbr) { return new_of_old[mbr] == UINT32_MAX; }),
                        c.members.end());
        for (auto& mbr : c.members) mbr = new_of_old[mbr];
        std::sort(c.members.begin(), c.members.end());
    }
    b.id_to_slot.clear();
    for (size_t ns = 0; ns < b.ext_ids.size(); ++ns) b.id_to_slot[b.ext_ids[ns]] = (uint32_t)ns;
    b.free_slots.clear();
    b.prim_len.clear();
    b.rep_off.clear();
    if (ma > 1 && nw > 0) {
        b.rep_off.push_back(0);
        for (size_t ci = 0; ci < b.cells.size(); ++ci) {
            std::vector<uint32_t> prim, repl;
            for (uint32_t mbr : b.cells[ci].members) (b.slot_cell[mbr] == ci ? prim : repl).push_back(mbr);
            std::sort(prim.begin(), prim.end());
            std::sort(repl.begin(), repl.end());
            b.prim_len.push_back((uint32_t)prim.size());
            b.rep_off.push_back(b.rep_off.back() + (uint32_t)repl.size());
            prim.insert(prim.end(), repl.begin(), repl.end());
            b.cells[ci].members = std::move(prim);
        }
    }
    b.fs_codes.clear();
    b.fs_off.clear();
    if (b.fastscan && nw > 0) {
        size_t bb = nw * 256;
        b.fs_off.push_back(0);
        for (auto& c : b.cells) {
            size_t nb = (c.members.size() + 31) / 32;
            size_t at = b.fs_codes.size();
            b.fs_codes.resize(at + nb * bb);
            for (size_t blk = 0; blk < nb; ++blk) {
                size_t lo = blk * 32, hi = std::min(lo + 32, c.members.size());
                std::vector<const uint64_t*> lanes;
                for (size_t r = lo; r < hi; ++r) lanes.push_back(&b.bits[(size_t)c.members[r] * nw]);
                fs_pack_block(lanes.data(), lanes.size(), nw, &b.fs_codes[at + blk * bb]);
            }
            b.fs_off.push_back((uint32_t)(b.fs_codes.size() / bb));
        }
    }
    b.compacted = true;
}

// ---- index build API (tests and the reference arm of bench.py) ---------------------------------

struct OBuildHandle {
    OBuild b;
    std::map<std::string, std::vector<uint8_t>> arrays;
    std::map<std::string, size_t> elem;
};

template <typename T>
void bput(OBuildHandle* h, const char* name, const T* p, size_t n) {
    auto& v = h->arrays[name];
    v.resize(n * sizeof(T));
    if (n) std::memcpy(v.data(), p, n * sizeof(T));
    h->elem[name] = sizeof(T);
}

// The arrays under the names and in the layouts FlatCellIndex.array() uses, so one OracleIndex
// constructor serves both sources and the test can compare them name by name.
void bexport(OBuildHandle* h) {
    OBuild& b = h->b;
    h->arrays.clear();
    double cfg[] = {(double)b.dim,          (double)b.dim_pad,       (double)b.nw,
                    (double)b.rerank_factor, (double)b.two_stage,     (double)b.shortlist_mult,
                    (double)b.centroid_sq8,  (double)b.has_tree,      (double)b.max_assign,
                    (double)b.fastscan,      (double)b.per_dim_sq,    (double)b.i8_rerank,
                    (double)b.keep_f32,      (double)b.adaptive,      (double)b.at_margin,
                    (double)b.quant_scale,   (double)b.compacted,     (double)b.n_live,
                    (double)b.cm_min_batch,  0.0,                     0.0,
                    (double)0xFFFFFFFFu,     (double)(b.has_tree ? b.tree_bf : 0.0f),
                    (double)(b.has_tree ? b.leaf_ids.size() : 0), (double)b.graph_route,
                    (double)b.graph_min_cells};
    bput(h, "config", cfg, sizeof(cfg) / sizeof(double));
    bput(h, "vecs_f32", b.vecs_f32.data(), b.vecs_f32.size());
    bput(h, "scan_i8", b.scan_i8.data(), b.scan_i8.size());
    bput(h, "ext_ids", b.ext_ids.data(), b.ext_ids.size());
    bput(h, "bits", b.bits.data(), b.bits.size());
    bput(h, "slot_cell", b.slot_cell.data(), b.slot_cell.size());
    bput(h, "slot_cells", b.slot_cells.data(), b.slot_cells.size());
    std::vector<uint32_t> mem, moff{0};
    std::vector<float> cents, rb;
    for (auto& c : b.cells) {
        mem.insert(mem.end(), c.members.begin(), c.members.end());
        moff.push_back((uint32_t)mem.size());
        cents.insert(cents.end(), c.centroid.begin(), c.centroid.end());
        rb.push_back(c.r_bound);
    }
    bput(h, "cell_members", mem.data(), mem.size());
    bput(h, "cell_member_off", moff.data(), moff.size());
    bput(h, "centroids", cents.data(), cents.size());
    bput(h, "r_bound", rb.data(), rb.size());
    bput(h, "prim_len", b.prim_len.data(), b.prim_len.size());
    bput(h, "rep_off", b.rep_off.data(), b.rep_off.size());
    bput(h, "fs_codes", b.fs_codes.data(), b.fs_codes.size());
    bput(h, "fs_off", b.fs_off.data(), b.fs_off.size());
    bput(h, "cent_bits", b.cent_bits.data(), b.cent_bits.size());
    bput(h, "cent_sq8", b.cent_sq8.data(), b.cent_sq8.size());
    bput(h, "csq_min", b.csq_min.data(), b.csq_min.size());
    bput(h, "csq_step", b.csq_step.data(), b.csq_step.size());
    bput(h, "sq_min", b.sq_min.data(), b.sq_min.size());
    bput(h, "sq_step", b.sq_step.data(), b.sq_step.size());
    bput(h, "signs", b.signs.data(), b.signs.size());
    std::vector<uint32_t> tags;
    bput(h, "tags", tags.data(), 0);
    std::vector<uint64_t> lvn, tcodes, tcoff{0}, tcs, tcl, tchoff{0};
    if (b.has_tree)
        for (auto& l : b.levels) {
            lvn.push_back(l.n);
            tcodes.insert(tcodes.end(), l.codes.begin(), l.codes.end());
            tcoff.push_back(tcodes.size());
            tcs.insert(tcs.end(), l.child_start.begin(), l.child_start.end());
            tcl.insert(tcl.end(), l.child_len.begin(), l.child_len.end());
            tchoff.push_back(tcs.size());
        }
    bput(h, "tree_level_n", lvn.data(), lvn.size());
    bput(h, "tree_codes", tcodes.data(), tcodes.size());
    bput(h, "tree_code_off", tcoff.data(), tcoff.size());
    bput(h, "tree_child_start", tcs.data(), tcs.size());
    bput(h, "tree_child_len", tcl.data(), tcl.size());
    bput(h, "tree_child_off", tchoff.data(), tchoff.size());
    std::vector<uint64_t> lc = b.has_tree ? b.leaf_codes : std::vector<uint64_t>();
    std::vector<uint32_t> li = b.has_tree ? b.leaf_ids : std::vector<uint32_t>();
    bput(h, "tree_leaf_codes", lc.data(), lc.size());
    bput(h, "tree_leaf_ids", li.data(), li.size());
}

// The searchable index of a build: its arrays moved out (take) or copied.
OIndex* make_index(OBuild& b, bool take) {
    auto* ix = new OIndex();
    ix->dim = b.dim;
    ix->dim_pad = b.dim_pad;
    ix->nw = b.nw;
    ix->M = b.cells.size();
    ix->ma = b.max_assign;
    ix->n_slots = b.ext_ids.size();
    ix->signs = b.signs;
    ix->mem_off.push_back(0);
    for (auto& c : b.cells) {
        ix->centroids.insert(ix->centroids.end(), c.centroid.begin(), c.centroid.end());
        ix->r_bound.push_back(c.r_bound);
        ix->mem.insert(ix->mem.end(), c.members.begin(), c.members.end());
        ix->mem_off.push_back((uint32_t)ix->mem.size());
    }
    if (take) ix->fs_codes = std::move(b.fs_codes); else ix->fs_codes = b.fs_codes;
    if (take) ix->fs_off = std::move(b.fs_off); else ix->fs_off = b.fs_off;
    if (take) ix->slot_cells = std::move(b.slot_cells); else ix->slot_cells = b.slot_cells;
    if (take) ix->ext_ids = std::move(b.ext_ids); else ix->ext_ids = b.ext_ids;
    ix->cent_bits = b.cent_bits;
    ix->cent_sq8 = b.cent_sq8;
    if (!b.cent_sq8.empty()) {
        ix->csq_min = b.csq_min;
        ix->csq_step = b.csq_step;
    }
    if (take) ix->vecs_f32 = std::move(b.vecs_f32); else ix->vecs_f32 = b.vecs_f32;
    if (take) ix->scan_i8 = std::move(b.scan_i8); else ix->scan_i8 = b.scan_i8;
    ix->sq_min = b.sq_min;
    ix->sq_step = b.sq_step;
    ix->rerank_factor = b.rerank_factor;
    ix->two_stage = b.two_stage;
    ix->shortlist_mult = b.shortlist_mult;
    ix->centroid_sq8 = b.centroid_sq8;
    ix->has_tree = b.has_tree;
    ix->fastscan = b.fastscan;
    ix->per_dim_sq = b.per_dim_sq;
    ix->i8_rerank = b.i8_rerank;
    ix->adaptive = b.adaptive;
    ix->at_margin = b.at_margin;
    ix->compacted = b.compacted;
    ix->n_live = b.n_live;
    ix->cm_min_batch = b.cm_min_batch;
    ix->has_filter = false;
    ix->flo = 0;
    ix->fhi = 0xFFFFFFFFu;
    ix->beam_frac = b.has_tree ? b.tree_bf : 0.0f;
    ix->n_leaf = b.has_tree ? b.leaf_ids.size() : 0;
    ix->graph_route = b.graph_route;
    ix->graph_min_cells = b.graph_min_cells;
    if (b.has_tree) {
        ix->levels = b.tview.levels;
        ix->leaf_codes = b.leaf_codes;
        ix->leaf_ids = b.leaf_ids;
    }
    if (take) {
        ix->bits = std::move(b.bits);
        b.bits.shrink_to_fit();
    } else {
        ix->bits = b.bits;
    }
    ix->n_live_cells = ix->live_cells();
    return ix;
}

}  // namespace

// ---- C API used by the tests and the CPU-baseline arm of bench.py ------------------------------

extern "C" {

struct oracle_arrays {
    // dimensions
    uint64_t dim, dim_pad, nw, M, ma, n_slots;
    // per-array pointers (may be null when empty) and element counts
    const float* signs;
    const float* centroids;
    const float* r_bound;
    const uint32_t* cell_members;
    const uint32_t* cell_member_off;
    const uint8_t* fs_codes;
    uint64_t n_fs_codes;
    const uint32_t* fs_off;
    const uint32_t* slot_cells;
    const uint64_t* ext_ids;
    const uint64_t* cent_bits;
    uint64_t n_cent_bits;
    const uint8_t* cent_sq8;
    uint64_t n_cent_sq8;
    const float* csq_min;
    const float* csq_step;
    const float* vecs_f32;
    uint64_t n_vecs_f32;
    const int8_t* scan_i8;
    uint64_t n_scan_i8;
    const float* sq_min;
    const float* sq_step;
    const uint32_t* tags;
    uint64_t n_tags;
    // tree: levels concatenated
    uint64_t tree_depth;
    const uint64_t* tree_level_n;
    const uint64_t* tree_codes;
    const uint64_t* tree_code_off;
    const uint64_t* tree_child_start;
    const uint64_t* tree_child_len;
    const uint64_t* tree_child_off;
    const uint64_t* tree_leaf_codes;
    const uint32_t* tree_leaf_ids;
    // configuration, in the product's "config" array order
    const double* config;
    uint64_t n_config;
    // flat codes, nw words per slot (may be null for a FastScan index)
    const uint64_t* bits;
    uint64_t n_bits;
};

void* oracle_index_new(const oracle_arrays* a) {
    auto* ix = new OIndex();
    ix->dim = a->dim;
    ix->dim_pad = a->dim_pad;
    ix->nw = a->nw;
    ix->M = a->M;
    ix->ma = a->ma;
    ix->n_slots = a->n_slots;
    auto cp = [](auto& v, const auto* p, size_t n) {
        if (p && n) v.assign(p, p + n);
    };
    cp(ix->signs, a->signs, 2 * a->dim_pad);
    cp(ix->centroids, a->centroids, a->M * a->dim);
    cp(ix->r_bound, a->r_bound, a->M);
    cp(ix->mem_off, a->cell_member_off, a->M + 1);
    cp(ix->mem, a->cell_members, ix->mem_off.empty() ? 0 : ix->mem_off.back());
    cp(ix->fs_codes, a->fs_codes, a->n_fs_codes);
    cp(ix->fs_off, a->fs_off, a->fs_off ? a->M + 1 : 0);
    cp(ix->slot_cells, a->slot_cells, a->n_slots * a->ma);
    cp(ix->ext_ids, a->ext_ids, a->n_slots);
    cp(ix->cent_bits, a->cent_bits, a->n_cent_bits);
    cp(ix->cent_sq8, a->cent_sq8, a->n_cent_sq8);
    cp(ix->csq_min, a->csq_min, a->n_cent_sq8 ? a->dim : 0);
    cp(ix->csq_step, a->csq_step, a->n_cent_sq8 ? a->dim : 0);
    cp(ix->vecs_f32, a->vecs_f32, a->n_vecs_f32);
    cp(ix->scan_i8, a->scan_i8, a->n_scan_i8);
    cp(ix->sq_min, a->sq_min, a->sq_min ? a->dim : 0);
    cp(ix->sq_step, a->sq_step, a->sq_step ? a->dim : 0);
    cp(ix->tags, a->tags, a->n_tags);
    cp(ix->bits, a->bits, a->n_bits);
    const double* c = a->config;
    ix->rerank_factor = (size_t)c[3];
    ix->two_stage = c[4] != 0;
    ix->shortlist_mult = (size_t)c[5];
    ix->centroid_sq8 = c[6] != 0;
    ix->has_tree = c[7] != 0;
    ix->fastscan = c[9] != 0;
    ix->per_dim_sq = c[10] != 0;
    ix->i8_rerank = c[11] != 0;
    ix->adaptive = c[13] != 0;
    ix->at_margin = (float)c[14];
    ix->compacted = c[16] != 0;
    ix->n_live = (size_t)c[17];
    ix->cm_min_batch = (size_t)c[18];
    ix->has_filter = c[19] != 0;
    ix->flo = (uint32_t)c[20];
    ix->fhi = (uint32_t)c[21];
    ix->beam_frac = (float)c[22];
    ix->n_leaf = (size_t)c[23];
    ix->graph_route = c[24] != 0;
    ix->graph_min_cells = (size_t)c[25];
    if (ix->has_tree) {
        for (size_t l = 0; l < a->tree_depth; ++l) {
            Level lv;
            lv.n = a->tree_level_n[l];
            lv.codes.assign(a->tree_codes + a->tree_code_off[l], a->tree_codes + a->tree_code_off[l + 1]);
            for (size_t i = a->tree_child_off[l]; i < a->tree_child_off[l + 1]; ++i) {
                lv.child_start.push_back((uint32_t)a->tree_child_start[i]);
                lv.child_len.push_back((uint32_t)a->tree_child_len[i]);
            }
            ix->levels.push_back(std::move(lv));
        }
        cp(ix->leaf_codes, a->tree_leaf_codes, ix->n_leaf * a->nw);
        cp(ix->leaf_ids, a->tree_leaf_ids, ix->n_leaf);
    }
    ix->n_live_cells = ix->live_cells();
    return ix;
}

void oracle_index_free(void* p) { delete static_cast<OIndex*>(p); }

void oracle_set_threads(int n) { omp_set_num_threads(n > 0 ? n : 1); }

// set_rerank_factor (index.rs:2949-2951): query-time only, so a sweep needs one index.
void oracle_index_set_rerank_factor(void* p, uint64_t rf) {
    static_cast<OIndex*>(p)->rerank_factor = rf > 0 ? rf : 1;
}

// search_batch (index.rs:3316-3391): ids/scores nq*k padded; cand_out (optional) receives per
// query the candidate slots sent to the rerank, sorted, as nq rows of cand_cap (UINT32_MAX pad)
// with counts in cand_n. Returns 0, 7 for an unsupported routing mode, or 8 for a cell-major
// batch over an index without FastScan blocks.
int oracle_search_batch(void* p, const float* Q, uint64_t nq, uint64_t k, uint64_t nprobe, float tc, float beta,
                        int cell_major, uint64_t* ids, float* scores, uint32_t* cand_out, uint64_t cand_cap,
                        uint32_t* cand_n, int* used_cell_major) {
    const OIndex& ix = *static_cast<OIndex*>(p);
    for (size_t i = 0; i < nq * k; ++i) {
        ids[i] = UINT64_MAX;
        scores[i] = -INFINITY;
    }
    if (ix.M == 0 || ix.n_live == 0) return 0;
    // cm_ok (index.rs:3343-3348); a compacted multi-home index always has its polysemic runs
    bool cm = cell_major && ix.compacted && !ix.has_filter && nq >= ix.cm_min_batch;
    if (used_cell_major) *used_cell_major = cm ? 1 : 0;
    // the cell-major join is restated for FastScan codes only
    if (cm && !(ix.fastscan && !ix.fs_off.empty())) return 8;
    std::vector<std::vector<uint32_t>> cands(nq);
    std::vector<std::vector<std::pair<float, uint64_t>>> res(nq);
    if (cm) {
        int rc = search_cellmajor(ix, Q, nq, k, nprobe, tc, beta, cands, res);
        if (rc) return rc;
    } else {
        int bad = 0;
#pragma omp parallel
        {
            SearchBuf b;
#pragma omp for schedule(dynamic, 1)
            for (long long qi = 0; qi < (long long)nq; ++qi) {
                int err = 0;
                res[qi] = search_one(ix, Q + qi * ix.dim, k, nprobe, tc, beta, b, &cands[qi], &err);
                if (err) {
#pragma omp atomic write
                    bad = err;
                }
                std::sort(cands[qi].begin(), cands[qi].end());
            }
        }
        if (bad) return bad;
    }
    for (size_t qi = 0; qi < nq; ++qi) {
        for (size_t i = 0; i < res[qi].size(); ++i) {
            ids[qi * k + i] = res[qi][i].second;
            scores[qi * k + i] = res[qi][i].first;
        }
        if (cand_out) {
            size_t n = std::min<size_t>(cands[qi].size(), cand_cap);
            for (size_t i = 0; i < cand_cap; ++i) cand_out[qi * cand_cap + i] = i < n ? cands[qi][i] : UINT32_MAX;
            if (cand_n) cand_n[qi] = (uint32_t)cands[qi].size();
        }
    }
    return 0;
}

// Routing only: probe lists (chosen) and their re-order scores, nq rows of nprobe.
int oracle_route(void* p, const float* Q, uint64_t nq, uint64_t nprobe, float tc, float beta, int batch_router,
                 uint32_t* chosen, float* cscore, uint32_t* nch) {
    const OIndex& ix = *static_cast<OIndex*>(p);
    std::vector<Routed> r;
    if (!(batch_router && route_batch(ix, Q, nq, nprobe, tc, beta, r))) {
        r.assign(nq, Routed{});
        SearchBuf b;
        for (size_t qi = 0; qi < nq; ++qi) {
            if (route_query(ix, Q + qi * ix.dim, nprobe, tc, beta, b) < 0) return 7;
            r[qi].chosen = b.chosen;
            for (size_t i = 0; i < b.chosen.size(); ++i) r[qi].cscore.push_back(b.cscores[i].second);
        }
    }
    for (size_t qi = 0; qi < nq; ++qi) {
        nch[qi] = (uint32_t)r[qi].chosen.size();
        for (size_t i = 0; i < nprobe; ++i) {
            chosen[qi * nprobe + i] = i < r[qi].chosen.size() ? r[qi].chosen[i] : UINT32_MAX;
            cscore[qi * nprobe + i] = i < r[qi].chosen.size() ? r[qi].cscore[i] : -INFINITY;
        }
    }
    return 0;
}

// ---- component functions (golden checks) ----
void oracle_make_signs(uint64_t dim_pad, uint64_t seed, float* out) { make_signs(dim_pad, seed, out); }
void oracle_splitmix64(uint64_t seed, uint64_t n, uint64_t* out) {
    uint64_t state = seed;
    for (size_t i = 0; i < n; ++i) {
        state += 0x9E3779B97F4A7C15ull;
        uint64_t z = state;
        z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
        z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
        out[i] = z ^ (z >> 31);
    }
}
void oracle_fht(float* a, uint64_t n) { fht_inplace(a, n); }
void oracle_rotate(const float* v, uint64_t dim, const float* signs, uint64_t dim_pad, float* out) {
    rotate(v, dim, signs, dim_pad, out);
}
void oracle_pack_signs_trunc(const float* rot, uint64_t dim_pad, uint64_t* out, uint64_t nw) {
    pack_signs_trunc(rot, dim_pad, out, nw);
}
void oracle_encode(const float* v, uint64_t n, uint64_t dim, const float* signs, uint64_t dim_pad, uint64_t nw,
                   uint64_t* out) {
#pragma omp parallel
    {
        std::vector<float> rot(dim_pad);
#pragma omp for
        for (long long i = 0; i < (long long)n; ++i) {
            rotate(v + i * dim, dim, signs, dim_pad, rot.data());
            pack_signs_trunc(rot.data(), dim_pad, out + i * nw, nw);
        }
    }
}
void oracle_fsquery(const float* rot, uint64_t rot_len, uint64_t nw, uint8_t* lut, float* delta, float* bias) {
    FsQuery f = fs_query(rot, rot_len, nw);
    std::memcpy(lut, f.lut.data(), f.lut.size());
    *delta = f.delta;
    *bias = f.bias;
}
void oracle_fs_block_sums(const uint8_t* block, const uint8_t* lut, uint64_t nw, int avx2, uint16_t* out) {
    if (avx2)
        fs_block_sums_avx2(block, lut, nw * 8, out);
    else
        fs_block_sums_scalar(block, lut, nw * 8, out);
}
void oracle_fs_pack_block(const uint64_t* codes, uint64_t ncodes, uint64_t nw, uint8_t* out) {
    std::vector<const uint64_t*> ptrs;
    for (size_t i = 0; i < ncodes; ++i) ptrs.push_back(codes + i * nw);
    fs_pack_block(ptrs.data(), ncodes, nw, out);
}
float oracle_dot_f32(const float* a, const float* b, uint64_t n) { return dot_f32(a, b, n); }
float oracle_dot_f32_u8(const float* a, const uint8_t* b, uint64_t n) { return dot_f32_u8(a, (const int8_t*)b, n); }
// Hamming cut-off of index.rs:86-104 (all cells live).
uint64_t oracle_hamming_cutoff(const uint16_t* hs, uint64_t n, uint64_t want, uint64_t bits) {
    std::vector<uint16_t> v(hs, hs + n);
    std::vector<uint8_t> live(n, 1);
    return hamming_cutoff(v, live, want, bits);
}
// keep_smallest of tree.rs:120-159 on (h, id) pairs; returns the kept count, ids in out.
uint64_t oracle_keep_smallest(const uint32_t* h, const uint32_t* id, uint64_t n, uint64_t keep, uint64_t bits,
                              uint32_t* out) {
    std::vector<std::pair<uint32_t, uint32_t>> v(n);
    for (size_t i = 0; i < n; ++i) v[i] = {h[i], id[i]};
    keep_smallest(v, keep, bits);
    for (size_t i = 0; i < v.size(); ++i) out[i] = v[i].second;
    return v.size();
}

// FlatCellIndex(dim, "binary", rerank_factor, seed, code_bits) (index.rs:2674-2755).
void* oracle_build_new(uint64_t dim, uint64_t code_bits, uint64_t seed, uint64_t rerank_factor) {
    if (dim == 0) return nullptr;
    auto* h = new OBuildHandle();
    OBuild& b = h->b;
    b.dim = dim;
    size_t p = 1;
    while (p < dim) p <<= 1;
    b.dim_pad = std::max<size_t>(p, 64);  // pad_dim, quantize.rs:38-40
    size_t bits = code_bits == 0 ? b.dim_pad : std::min<size_t>(code_bits, b.dim_pad);
    b.nw = std::max<size_t>(bits / 64, 1);  // code_words, quantize.rs:50-53
    b.seed = seed;
    b.rerank_factor = std::max<uint64_t>(rerank_factor, 1);
    b.signs.resize(2 * b.dim_pad);
    make_signs(b.dim_pad, seed, b.signs.data());
    return h;
}

void oracle_build_free(void* p) { delete static_cast<OBuildHandle*>(p); }

// The setters the presets call (index.rs:2823-2984); returns 0, or 1 for an unknown key.
int oracle_build_set(void* p, const char* key, double a, double b2, double c, double d) {
    OBuild& b = static_cast<OBuildHandle*>(p)->b;
    std::string k(key);
    if (k == "two_stage") {  // :2882-2888
        b.two_stage = a != 0;
        b.shortlist_mult = std::max<size_t>((size_t)b2, 1);
        if (b.two_stage) rebuild_codes(b);
    } else if (k == "tree_route") {  // :2839-2852
        if (d > 0.0) b.tree_beam_frac = (float)d;
        b.tree_route = a != 0;
        if (b2 > 0) b.tree_min_cells = (size_t)b2;
        if (c > 1) b.tree_fanout = (size_t)c;
        rebuild_tree(b);
    } else if (k == "graph_route") {  // :2859-2865
        b.graph_route = a != 0;
        if (b2 > 0) b.graph_min_cells = (size_t)b2;
    } else if (k == "orthogonal_polysemy") {  // :2979-2984
        b.max_assign = std::max<size_t>((size_t)a, 1);
        b.spill_margin = 0.0f;
        b.spill_lambda = std::max((float)b2, 1e-6f);
    } else if (k == "replication") {  // :2966-2970
        b.max_assign = std::max<size_t>((size_t)a, 1);
        b.spill_margin = std::max((float)b2, 0.0f);
        b.spill_lambda = 0.0f;
    } else if (k == "fastscan") {  // :2962-2968
        b.fastscan = a != 0;
        if (!b.fastscan) {
            b.fs_codes.clear();
            b.fs_off.clear();
        }
    } else if (k == "per_dim_sq") {  // :2908-2915
        b.per_dim_sq = a != 0;
        if (b.per_dim_sq) {
            b.i8_rerank = true;
            b.keep_f32 = false;
        }
    } else if (k == "i8_rerank") {  // :2825-2831
        b.i8_rerank = a != 0;
        b.keep_f32 = !b.i8_rerank;
    } else if (k == "adaptive") {  // :2899-2902
        b.adaptive = a != 0;
        b.at_margin = (float)b2;
    } else if (k == "centroid_sq8") {  // :2872-2879
        b.centroid_sq8 = a != 0;
        if (b.centroid_sq8)
            rebuild_sq8(b);
        else
            b.cent_sq8.clear();
    } else if (k == "rerank_factor") {  // :2949-2951
        b.rerank_factor = std::max<size_t>((size_t)a, 1);
    } else if (k == "cm_min_batch") {
        b.cm_min_batch = std::max<size_t>((size_t)a, 1);
    } else {
        return 1;
    }
    return 0;
}

int oracle_build_train(void* p, const float* data, uint64_t n, uint64_t n_cells, uint64_t sample, uint64_t seed) {
    return build_train(static_cast<OBuildHandle*>(p)->b, data, n, n_cells, sample, seed);
}

int oracle_build_add(void* p, const uint64_t* ids, const float* data, uint64_t n) {
    return build_add(static_cast<OBuildHandle*>(p)->b, ids, data, n);
}

void oracle_build_compact(void* p) { build_compact(static_cast<OBuildHandle*>(p)->b); }

int oracle_build_remove(void* p, uint64_t id) { return build_remove(static_cast<OBuildHandle*>(p)->b, id) ? 1 : 0; }

int oracle_build_has_id(void* p, uint64_t id) { return static_cast<OBuildHandle*>(p)->b.id_to_slot.count(id) ? 1 : 0; }

uint64_t oracle_build_n_live(void* p) { return static_cast<OBuildHandle*>(p)->b.n_live; }

// A new build handle: fork_empty of this one.
void* oracle_build_fork(void* p) {
    auto* h = new OBuildHandle();
    build_fork(static_cast<OBuildHandle*>(p)->b, h->b);
    return h;
}

// The searchable index straight from a finished build, moving the large arrays instead of copying
// them (the build handle keeps its configuration but no longer its arena). Same contents as
// oracle_index_new over the exported arrays.
void* oracle_build_take_index(void* p) { return make_index(static_cast<OBuildHandle*>(p)->b, true); }

// A searchable copy of the build as it stands; the build stays usable (a mutable segment).
void* oracle_build_snapshot(void* p) { return make_index(static_cast<OBuildHandle*>(p)->b, false); }

// Snapshot of every array (call after the build steps), then one array by name.
void oracle_build_export(void* p) { bexport(static_cast<OBuildHandle*>(p)); }

int oracle_build_array(void* p, const char* name, const void** data, uint64_t* count, uint64_t* elem_bytes) {
    auto* h = static_cast<OBuildHandle*>(p);
    auto it = h->arrays.find(name);
    if (it == h->arrays.end()) return 1;
    size_t e = h->elem[name];
    *data = it->second.empty() ? nullptr : it->second.data();
    *count = it->second.size() / e;
    *elem_bytes = e;
    return 0;
}

}  // extern "C"
