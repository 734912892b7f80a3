"""GPU search == the reference's CPU path at the shape of BASELINE configs[4]: d = 768, the
`memory` preset with 768-bit codes (96 B) and per-dimension SQ8 rows, k = 100, and a per-vector
tag filter at 1% and 10% selectivity (uniform tags in [0, 1000), filter tag < t, as the
reference's bench/fair/filtered.py draws them).

A filter turns the cell-major join off (index.rs:3343-3348), so the filtered searches take the
per-query path, with the tag checked in the scan (index.rs:1430-1439). The unfiltered searches
run the cell-major join with k = 100 (the bitonic top-k above the warp top-k's 32). The index is
the product's build; the oracle searches its arrays (and its own independent build is compared
with the product's, array for array, in tests/test_oracle_build.py). Ids must be identical and
scores bit-identical.
"""
from __future__ import annotations

import numpy as np
import pytest

from datagen import build_index, mixture

pytestmark = pytest.mark.gpu

K = 100


@pytest.fixture(scope="module")
def shape4():
    rng = np.random.default_rng(404)
    X, c = mixture(rng, 60_000, 768, 60, sigma=0.3)
    Q, _ = mixture(rng, 96, 768, 60, sigma=0.3, centers=c)
    ix = build_index(X, "memory", rf=4, code_bits=768, tree_min_cells=64)
    tags = np.random.default_rng(2).integers(0, 1000, X.shape[0]).astype(np.uint32)
    ix.set_tags(np.arange(X.shape[0], dtype=np.uint64), tags)
    return X, Q, ix, tags


def _compare(ix, Q, nprobe, cell_major):
    import oracle

    got_ids, got_sc = ix.search_batch_arrays(Q, K, nprobe, 1.0, 8.0, cell_major)
    o = oracle.OracleIndex.from_index(ix)
    ref_ids, ref_sc, _, _, used = o.search_batch(Q, K, nprobe, 1.0, 8.0, cell_major)
    bad = np.nonzero((got_ids != ref_ids) | ~((got_sc == ref_sc) | (np.isinf(got_sc) & np.isinf(ref_sc))))[0]
    assert bad.size == 0, (
        f"{bad.size} mismatches (first query {bad[0] // K}): gpu {got_ids[bad[:5]]} {got_sc[bad[:5]]} "
        f"oracle {ref_ids[bad[:5]]} {ref_sc[bad[:5]]}")
    return got_ids, used


@pytest.mark.parametrize("t", [10, 100])
@pytest.mark.parametrize("nprobe", [32, 256])
def test_filtered_k100(shape4, t, nprobe):
    X, Q, ix, tags = shape4
    ix.set_filter(0, t - 1)
    try:
        ids, used = _compare(ix, Q, nprobe, True)
        assert not used
        live = ids[ids != np.iinfo(np.uint64).max].astype(np.int64)
        assert live.size > 0 and np.all(tags[live] < t)
    finally:
        ix.set_filter()


@pytest.mark.parametrize("nprobe", [16, 128])
def test_unfiltered_k100_both_paths(shape4, nprobe):
    X, Q, ix, _ = shape4
    _, used = _compare(ix, Q, nprobe, True)
    assert used
    _compare(ix, Q[:48], nprobe, False)


def test_filtered_recall_against_exact(shape4):
    """The filtered search is a working search: R@100 against the exact top 100 among the vectors
    that pass the 10% filter, probing a quarter of the cells."""
    X, Q, ix, tags = shape4
    ix.set_filter(0, 99)
    try:
        cells = int(ix.stats()["n_cells"])
        ids, _ = ix.search_batch_arrays(Q, K, cells // 4, 1.0, 8.0, True)
    finally:
        ix.set_filter()
    sub = np.nonzero(tags < 100)[0]
    truth = sub[np.argsort(-(Q @ X[sub].T), axis=1)[:, :K]]
    got = ids.reshape(-1, K).astype(np.int64)
    rec = np.mean([len(set(a) & set(b)) / K for a, b in zip(got.tolist(), truth.tolist())])
    assert rec >= 0.8
