// TEST INFRASTRUCTURE ONLY - the parity oracle of the B200 MAIVS engine.
//
// A CPU restatement, in C++17 + AVX2 + OpenMP, of the reference's query hot path
// (V47VANSH/MAIVS, Rust): src/quantize.rs (rotation, codes, FastScan tables and block sums),
// src/tree.rs:120-159 and :559-628 (tree beam search), src/index.rs:41-343 (SIMD dots),
// :1168-1305 (route_query), :1309-1378 (rerank_exact), :1381-1864 (search_one, FastScan
// branch), :1873-1980 (route_batch), :1999-2311 (search_batch_cellmajor), :3316-3391
// (search_batch). Each function below cites the lines it follows.
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
    } else if (ix.graph_route && ix.n_live >= ix.graph_min_cells) {
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
    // FastScan bucket queue on d >> 6 with a falling tau (index.rs:1630-1692)
    rotate(q, ix.dim, ix.signs.data(), ix.dim_pad, b.rot.data());
    FsQuery fq = fs_query(b.rot.data(), ix.dim_pad, nw);
    const size_t bb = nw * 64 * 32 / 8;
    const uint32_t maxk = fq.maxk;
    const float norm = std::sqrt(2.0f * (float)ix.dim_pad / 3.14159265358979323846f);
    const size_t target = std::max<size_t>(want0, 1);
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
    return ix;
}

void oracle_index_free(void* p) { delete static_cast<OIndex*>(p); }

void oracle_set_threads(int n) { omp_set_num_threads(n > 0 ? n : 1); }

// search_batch (index.rs:3316-3391): ids/scores nq*k padded; cand_out (optional) receives per
// query the candidate slots sent to the rerank, sorted, as nq rows of cand_cap (UINT32_MAX pad)
// with counts in cand_n. Returns 0, or 7 for an unsupported routing mode.
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

}  // extern "C"
