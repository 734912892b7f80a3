"""GPU search == the reference's CPU path (the oracle), bit for bit, on seeded indexes.

Each case builds an index with the product's host build, runs the same queries through the GPU
engine (C ABI via the FlatCellIndex drop-in) and through the oracle's restatement of the
reference query path, and requires identical ids and identical f32 scores. Ties in the reference's
unstable sorts are broken the same way on both sides (cell id, slot, external id).
"""
from __future__ import annotations

import numpy as np
import pytest

from datagen import build_index, exact_topk, mixture, recall, shifted

pytestmark = pytest.mark.gpu

K = 10


@pytest.fixture(scope="module")
def data():
    rng = np.random.default_rng(7)
    X, centers = mixture(rng, 50_000, 384, 400)
    Q, _ = mixture(rng, 300, 384, 400, centers=centers)
    Qs = shifted(rng, Q[:100])
    return X, np.ascontiguousarray(np.vstack([Q, Qs]))


def _oracle(ix):
    import oracle

    return oracle.OracleIndex.from_index(ix)


def _compare(ix, Q, k, nprobe, tc=1.0, cell_major=True):
    got_ids, got_sc = ix.search_batch_arrays(Q, k, nprobe, tc, 8.0, cell_major)
    o = _oracle(ix)
    ref_ids, ref_sc, _, _, used = o.search_batch(Q, k, nprobe, tc, 8.0, cell_major)
    bad = np.nonzero((got_ids != ref_ids) | ~((got_sc == ref_sc) | (np.isinf(got_sc) & np.isinf(ref_sc))))[0]
    assert bad.size == 0, (
        f"{bad.size} mismatches (first query {bad[0] // k}): gpu {got_ids[bad[:5]]} {got_sc[bad[:5]]} "
        f"oracle {ref_ids[bad[:5]]} {ref_sc[bad[:5]]}")
    return got_ids, used


@pytest.fixture(scope="module")
def quality(data):
    X, _ = data
    return build_index(X, "quality", rf=8, tree_min_cells=64)


@pytest.fixture(scope="module")
def memory(data):
    X, _ = data
    return build_index(X, "memory", rf=16, tree_min_cells=64)


@pytest.mark.parametrize("nprobe", [1, 8, 32, 128, 512])
def test_cellmajor_quality_bit_exact(data, quality, nprobe):
    X, Q = data
    ids, used = _compare(quality, Q, K, nprobe, cell_major=True)
    assert used


@pytest.mark.parametrize("nprobe", [1, 8, 32, 128])
def test_perquery_quality_bit_exact(data, quality, nprobe):
    X, Q = data
    _compare(quality, Q[:64], K, nprobe, cell_major=False)


@pytest.mark.parametrize("nprobe", [4, 64, 256])
def test_memory_preset_both_paths(data, memory, nprobe):
    X, Q = data
    _compare(memory, Q, K, nprobe, cell_major=True)
    _compare(memory, Q[:48], K, nprobe, cell_major=False)


def test_recall_matches_oracle_and_brute_force(data, quality):
    X, Q = data
    truth = exact_topk(X, Q[:300])
    ids, _ = quality.search_batch_arrays(Q[:300], K, 256, 1.0, 8.0, True)
    r = recall(ids, truth)
    o = _oracle(quality)
    ref_ids, *_ = o.search_batch(Q[:300], K, 256, 1.0, 8.0, True)
    assert r == recall(ref_ids, truth)
    assert r > 0.9


@pytest.mark.parametrize("homes,adaptive,two_stage", [(1, False, True), (1, True, False), (3, True, True)])
def test_variants(data, homes, adaptive, two_stage):
    X, Q = data
    ix = build_index(X[:20_000], "quality", rf=4, homes=homes, adaptive=adaptive, two_stage=two_stage,
                     tree_min_cells=10**9)
    for nprobe in (3, 40):
        _compare(ix, Q, K, nprobe, cell_major=True)
        _compare(ix, Q[:40], K, nprobe, cell_major=False)


def test_truncated_codes_and_i8_rerank(data):
    X, Q = data
    import maivs_b200 as M

    ix = M.FlatCellIndex(384, "binary", 8, 0x5EED, 256)
    ix.set_i8_rerank(True)
    ix.set_orthogonal_polysemy(2, 1.0)
    ix.set_fastscan(True)
    ix.set_two_stage(True, 2)
    ix.set_adaptive(True, 0.02)
    ix.train_centroids(X[:20_000], 100)
    ix.add_batch(list(range(20_000)), X[:20_000])
    ix.compact()
    _compare(ix, Q, K, 24, cell_major=True)
    _compare(ix, Q[:40], K, 24, cell_major=False)


def test_d768_codes(data):
    rng = np.random.default_rng(11)
    X, c = mixture(rng, 12_000, 768, 100, sigma=0.3)
    Q, _ = mixture(rng, 64, 768, 100, sigma=0.3, centers=c)
    ix = build_index(X, "memory", rf=8)
    _compare(ix, Q, K, 16, cell_major=True)
    _compare(ix, Q[:16], K, 16, cell_major=False)


def test_filter_per_query_path(data, quality):
    X, Q = data
    n = X.shape[0]
    tags = (np.arange(n) * 2654435761 % 1000).astype(np.uint32)
    quality.set_tags(np.arange(n, dtype=np.uint64), tags)
    try:
        quality.set_filter(0, 99)
        ids, used = _compare(quality, Q[:64], K, 64, cell_major=True)
        assert not used  # a filter disables the cell-major join (index.rs:3347)
        live = ids[ids != np.iinfo(np.uint64).max].astype(np.int64)
        assert np.all(tags[live] <= 99)
    finally:
        quality.set_filter()


def test_nucleus_close_to_oracle(data, quality):
    X, Q = data
    got, _ = quality.search_batch_arrays(Q, K, 64, 0.9, 8.0, True)
    ref, *_ = _oracle(quality).search_batch(Q, K, 64, 0.9, 8.0, True)
    # exp() may round differently by one ulp on the two sides; the probe sets still agree
    assert np.mean(got == ref) > 0.999


def test_single_search_matches_batch(data, quality):
    X, Q = data
    ids, sc = quality.search(Q[0], K, 32, 1.0, 8.0)
    bi, bs = quality.search_batch_arrays(Q[:1], K, 32, 1.0, 8.0, False)
    assert ids == [int(x) for x in bi] and np.array_equal(np.asarray(sc, np.float32), bs)


@pytest.mark.parametrize("dim,preset", [(60, "quality"), (100, "quality"), (100, "memory"), (200, "memory")])
def test_odd_dims(dim, preset):
    # dim_pad 64 uses the block encoder; 100-byte SQ8 rows take the per-thread rerank; f32 rows
    # of 240 / 400 bytes take the staged rerank with a scalar tail (dim % 8 != 0)
    rng = np.random.default_rng(dim)
    X, c = mixture(rng, 6000, dim, 60)
    Q, _ = mixture(rng, 48, dim, 60, centers=c)
    ix = build_index(X, preset, rf=8)
    _compare(ix, Q, K, 12, cell_major=True)
    _compare(ix, Q[:12], K, 12, cell_major=False)


@pytest.mark.parametrize("homes", [1, 2])
def test_large_cells(data, homes):
    """About 1,000 vectors a cell (2,000 member entries with two homes): the seed cells of a query
    then hold more members than the seed step keeps in shared memory, so its entries go through
    the global seed buffer; ragged last groups in every cell."""
    X, Q = data
    ix = build_index(X[:30_000], "quality", rf=8, n_cells=30, tree_min_cells=10**9, homes=homes)
    for nprobe in (8, 12):
        _compare(ix, Q[:120], K, nprobe)


def test_kernel_clock_only_times_one_kernel(data, quality):
    """The bench times only its dominant kernel inside the timed steps: no other kernel gets events."""
    _, Q = data
    quality.kernel_clock(True, only="k_rerank")
    quality.kernel_times(reset=True)
    quality.search_batch_arrays(Q[:64], K, 8, 1.0, 8.0, True)
    kt = quality.kernel_times(reset=True)
    quality.kernel_clock(True)
    quality.search_batch_arrays(Q[:64], K, 8, 1.0, 8.0, True)
    every = quality.kernel_times(reset=True)
    quality.kernel_clock(False)
    assert {k for k, v in kt.items() if v[0] > 0} == {"k_rerank"}
    assert {"k_seed_scan", "k_seed", "k_rerank"} <= {k for k, v in every.items() if v[0] > 0}
    with pytest.raises(ValueError, match="unknown kernel"):
        quality.kernel_clock(True, only="k_nothing")


def test_d768_quality_rerank():
    """f32 rows of 768 dimensions: the streamed rerank's second instantiation."""
    rng = np.random.default_rng(12)
    X, c = mixture(rng, 12_000, 768, 100, sigma=0.3)
    Q, _ = mixture(rng, 64, 768, 100, sigma=0.3, centers=c)
    ix = build_index(X, "quality", rf=8)
    _compare(ix, Q, K, 16, cell_major=True)
    _compare(ix, Q[:16], K, 16, cell_major=False)


@pytest.mark.parametrize("k,rf", [(1, 1), (7, 3), (33, 5)])
def test_ragged_candidate_counts(data, k, rf):
    """Candidate lists that are not whole 16-row items (k x rf = 1, 21, 165) through the streamed
    f32 rerank, with k above the warp top-k's 32 in the last case; batch at the cell-major floor."""
    X, Q = data
    ix = build_index(X[:20_000], "quality", rf=rf, tree_min_cells=64)
    _compare(ix, Q[:32], k, 8)
    _compare(ix, Q[:40], k, 24)


def test_batch_above_the_stream_item_table():
    """7,000 queries: the streamed rerank's item numbering (4 bytes a query) no longer fits beside
    its 4 x 49 KB stages, so it comes from k_rerank_items; each query's result equals its row in
    two 3,500-query batches, which number their items inside the rerank kernel."""
    rng = np.random.default_rng(21)
    X, c = mixture(rng, 20_000, 384, 200)
    Q, _ = mixture(rng, 7_000, 384, 200, centers=c)
    ix = build_index(X, "quality", rf=8, tree_min_cells=64)
    ids, sc = ix.search_batch_arrays(Q, K, 8, 1.0, 8.0, True)
    ids_a, sc_a = ix.search_batch_arrays(Q[:3500], K, 8, 1.0, 8.0, True)
    ids_b, sc_b = ix.search_batch_arrays(Q[3500:], K, 8, 1.0, 8.0, True)
    assert np.array_equal(ids, np.concatenate([ids_a, ids_b]))
    assert np.array_equal(sc.view(np.uint32), np.concatenate([sc_a, sc_b]).view(np.uint32))
