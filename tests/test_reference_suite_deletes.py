"""The reference's delete and polysemy checks (tests/test_index.py [3], [4], [8c], [10]) on this
repository's host build, searched on the CPU by the oracle (the GPU searches of removed and
reloaded indexes are in test_gpu_hamming.py and test_gpu_persist.py).

The fixture is the reference's clustered one (DIM=256, N=4000, 32 cells) with its faiss centroids
replaced by train_centroids (faiss is absent here). Searches probe every cell, as the reference's
`search_all` does. An index with removed ids is searched as the reference searches it: per query,
by Hamming distance over the flat codes (index.rs:1624-1626)."""
from __future__ import annotations

import numpy as np
import pytest

import maivs_b200 as M
import oracle
from datagen import clustered, exact_topk, recall

DIM, N, NCELLS, K = 256, 4000, 32, 10
PAD = np.iinfo(np.uint64).max


@pytest.fixture(scope="module")
def fixture():
    rng = np.random.default_rng(3)
    base, centers = clustered(rng, N, DIM, n_clusters=200, spread=0.7)
    q, _ = clustered(rng, 100, DIM, spread=0.7, skew=False, centers=centers)
    return base, np.ascontiguousarray(q), exact_topk(base, q)


def build(base, homes=1, storage="i8"):
    ix = M.FlatCellIndex(DIM, "binary", 8, 0x5EED, 0)
    if storage == "i8":
        ix.set_i8_rerank(True)
    elif storage == "sq8":
        ix.set_per_dim_sq(True)
    if homes > 1:
        ix.set_orthogonal_polysemy(homes, 1.0)
    ix.train_centroids(base, NCELLS)
    ix.add_batch(list(range(N)), base)
    return ix


def search_all(ix, q, nprobe=NCELLS):
    ids, *_ = oracle.OracleIndex.from_index(ix).search_batch(q, K, nprobe, 1.0, 8.0, False)
    return ids.reshape(len(q), K)


def test_delete_removes_exactly_the_requested_ids(fixture):  # [3]
    base, q, truth = fixture
    ix = build(base)
    victims = [int(v) for v in np.random.default_rng(4).choice(N, 500, replace=False)]
    assert all(ix.remove(v) for v in victims)
    assert len(ix) == N - 500
    got = search_all(ix, q)
    assert not np.isin(got, victims).any()
    assert ix.remove(victims[0]) is False  # re-deleting an id returns False
    # the survivors are still found: recall against the exact top k of the live vectors
    live = np.setdiff1d(np.arange(N), victims)
    truth_live = live[exact_topk(base[live], q)]
    assert recall(got, truth_live) > 0.97


def test_deleted_ids_stay_deleted_across_save_load(fixture, tmp_path):  # [4]
    base, q, _ = fixture
    ix = build(base)
    victims = list(range(0, 1000, 2))
    for v in victims:
        ix.remove(v)
    path = str(tmp_path / "idx.maivs")
    ix.save(path)
    ld = M.FlatCellIndex.load(path)
    assert len(ld) == N - len(victims)
    got = search_all(ld, q)
    assert not np.isin(got, victims).any()
    # the reloaded index answers as the saved one does
    assert np.array_equal(got, search_all(ix, q))


@pytest.mark.parametrize("storage", ["i8", "f32", "sq8"])
def test_delete_works_under_every_storage_mode(fixture, storage):  # [8c]
    base, q, _ = fixture
    ix = build(base, storage=storage)
    for v in range(50):
        assert ix.remove(v)
    assert len(ix) == N - 50
    assert not np.isin(search_all(ix, q), np.arange(50)).any()


@pytest.mark.parametrize("homes", [2, 3])
def test_orthogonal_polysemy_engaged_exact_no_duplicates(fixture, homes):  # [10]
    base, q, truth = fixture
    ix = build(base, homes=homes)
    assert int(ix.stats()["max_assign"]) == homes
    o = oracle.OracleIndex.from_index(ix)
    for npb in (1, 2, 4, 8, NCELLS):
        ids, *_ = o.search_batch(q, K, npb, 1.0, 8.0, False)
        for row in ids.reshape(len(q), K):
            live = row[row != PAD]
            assert len(live) == len(set(live.tolist())), npb
    assert recall(search_all(ix, q), truth) > 0.97
    # deletes unlink every home: no cell lists a removed vector's slot any more
    victims = list(range(0, 400, 2))
    for v in victims:
        ix.remove(v)
    assert len(ix) == N - len(victims)
    assert not np.isin(search_all(ix, q), victims).any()
