"""The reference's invariant suite (tests/test_index.py [1b], [6], [7], [11], [12], [14]) run on
the oracle, on the reference's own clustered fixture (DIM=256, N=4000, 32 cells) with the
faiss centroids replaced by the in-process train_centroids (faiss is absent here)."""
from __future__ import annotations

import numpy as np
import pytest

import oracle
from datagen import clustered, exact_topk, recall

DIM, N, NCELLS, K = 256, 4000, 32, 10


@pytest.fixture(scope="module")
def fixture():
    rng = np.random.default_rng(0)
    base, centers = clustered(rng, N, DIM, n_clusters=200, spread=0.7)
    q, _ = clustered(rng, 100, DIM, spread=0.7, skew=False, centers=centers)
    qq = np.ascontiguousarray(np.repeat(q, 1, axis=0))
    return base, qq, exact_topk(base, qq)


def make(base, homes=1, two_stage=False, adaptive=False, rf=8):
    import maivs_b200 as M

    ix = M.FlatCellIndex(DIM, "binary", rf, 0x5EED, 0)
    ix.set_i8_rerank(True)
    if homes > 1:
        ix.set_orthogonal_polysemy(homes, 1.0)
    if two_stage:
        ix.set_two_stage(True, 2)
    if adaptive:
        ix.set_adaptive(True, 0.02)
    ix.set_fastscan(True)
    ix.train_centroids(base, NCELLS)
    ix.add_batch(list(range(N)), base)
    ix.compact()
    return oracle.OracleIndex.from_index(ix)


def ids_of(o, q, nprobe, cm):
    ids, *_ = o.search_batch(q, K, nprobe, 1.0, 8.0, cm)
    return ids.reshape(len(q), K)


def overlap(a, b):
    return float(np.mean([len(set(x.tolist()) & set(y.tolist())) / K for x, y in zip(a, b)]))


def test_binary_recall_every_cell_probed(fixture):  # [1b]
    base, q, truth = fixture
    assert recall(ids_of(make(base), q, NCELLS, True), truth) > 0.97


@pytest.mark.parametrize("two_stage", [False, True])
def test_cell_major_equals_per_query(fixture, two_stage):  # [11]
    base, q, truth = fixture
    o = make(base, two_stage=two_stage)
    for npb in (1, 4, NCELLS):
        assert overlap(ids_of(o, q, npb, False), ids_of(o, q, npb, True)) > 0.995


@pytest.mark.parametrize("homes", [2, 3])
def test_polysemic_runs_no_duplicates(fixture, homes):  # [12]
    base, q, truth = fixture
    o = make(base, homes=homes, two_stage=True)
    for npb in (1, 4, NCELLS):
        a, b = ids_of(o, q, npb, False), ids_of(o, q, npb, True)
        assert overlap(a, b) > 0.995
        for r in np.vstack([a, b]):
            live = r[r != np.iinfo(np.uint64).max]
            assert len(live) == len(set(live.tolist()))


def test_adaptive_close_to_exhaustive(fixture):  # [6]
    base, q, truth = fixture
    full = ids_of(make(base), q, NCELLS, True)
    ada = ids_of(make(base, adaptive=True), q, NCELLS, True)
    assert overlap(full, ada) > 0.97


def test_two_stage_close_to_single_stage(fixture):  # [7]
    base, q, truth = fixture
    assert overlap(ids_of(make(base), q, NCELLS, True), ids_of(make(base, two_stage=True), q, NCELLS, True)) > 0.98
