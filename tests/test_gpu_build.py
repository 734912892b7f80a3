"""The index build on the GPU (k-means and vector placement, csrc/cuda/build.cu) against the host
build: every array the search reads must be identical, bit for bit, with no step left to the host.

The host build is in turn checked against the oracle's independent restatement of the reference
build (tests/test_oracle_build.py); one case here closes the loop against the oracle directly."""
from __future__ import annotations

import numpy as np
import pytest

import oracle
from datagen import build_index, mixture, oracle_build_index

pytestmark = pytest.mark.gpu

ARRAYS = oracle.OracleIndex.NAMES + ("prim_len", "rep_off", "slot_cell", "bits")


def gpu_build(X, **kw):
    import maivs_b200 as M

    orig = M.FlatCellIndex.train_centroids

    def train_on_gpu(self, *a, **k):
        self.set_build_device(0)
        return orig(self, *a, **k)

    M.FlatCellIndex.train_centroids = train_on_gpu
    try:
        ix = build_index(X, **kw)
    finally:
        M.FlatCellIndex.train_centroids = orig
    return ix


def assert_same(a_ix, b_ix):
    for name in ARRAYS:
        a, b = a_ix.array(name), b_ix.array(name)
        assert a.dtype == b.dtype and a.shape == b.shape, name
        assert np.array_equal(a.view(np.uint8), b.view(np.uint8)), f"{name}: {(a != b).sum()} entries differ"


CASES = {
    "quality_tree": dict(n=40_000, d=384, comps=300, kw=dict(preset="quality", tree_min_cells=64)),
    "memory_tree": dict(n=40_000, d=384, comps=300, kw=dict(preset="memory", tree_min_cells=64)),
    "two_level_tree": dict(n=300_000, d=384, comps=1000, kw=dict(tree_min_cells=64, fanout=4)),
    "one_home": dict(n=30_000, d=384, comps=200, kw=dict(homes=1, tree_min_cells=64)),
    "replication3": dict(n=30_000, d=384, comps=200, kw=dict(replication=(3, 0.05), tree_min_cells=64)),
    "three_homes": dict(n=30_000, d=384, comps=200, kw=dict(homes=3, tree_min_cells=64)),
    "d100_codes128": dict(n=40_000, d=100, comps=200, kw=dict(code_bits=128, tree_min_cells=64)),
    "d768_codes768": dict(n=40_000, d=768, comps=200, kw=dict(code_bits=768, preset="memory", tree_min_cells=64)),
    "flat_placement": dict(n=60_000, d=384, comps=400, kw=dict()),  # 468 cells: no tree, k-means on the GPU
}


@pytest.mark.parametrize("case", sorted(CASES))
def test_gpu_build_equals_host_build(case):
    c = CASES[case]
    X, _ = mixture(np.random.default_rng(300 + sorted(CASES).index(case)), c["n"], c["d"], c["comps"])
    host = build_index(X, rf=8, **c["kw"])
    gpu = gpu_build(X, rf=8, **c["kw"])
    st = gpu.stats()
    assert st["build_device"] == 0 and st["build_gpu_failures"] == 0
    assert_same(host, gpu)


def test_gpu_build_equals_oracle_build_and_searches_the_same():
    X, cen = mixture(np.random.default_rng(77), 50_000, 384, 400)
    Q, _ = mixture(np.random.default_rng(78), 200, 384, 400, centers=cen)
    gpu = gpu_build(X, rf=16, tree_min_cells=64)
    b = oracle_build_index(X, rf=16, tree_min_cells=64)
    for name in oracle.OracleIndex.NAMES:
        if name == "config":
            continue
        a, c = gpu.array(name), b.array(name)
        assert a.shape == c.shape and np.array_equal(a.view(np.uint8), c.view(np.uint8)), name
    gpu.to_device(0)
    ids, sc = gpu.search_batch_arrays(Q, 10, 32, 1.0, 8.0, True)
    rid, rsc, *_ = b.index().search_batch(Q, 10, 32, 1.0, 8.0, True)
    assert np.array_equal(ids, rid) and np.array_equal(sc.view(np.uint32), rsc.view(np.uint32))
