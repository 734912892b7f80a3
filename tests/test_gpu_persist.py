"""GPU search of an index loaded from the reference's MAIVS2 format (persist.rs:192-281).

The product builds an index, saves it, loads it back (derived state rebuilt, as the reference does),
compacts it with FastScan and uploads it; its GPU search must equal the oracle's own build and
search of the original vectors, ids and f32 scores bit for bit, on both paths.
"""
from __future__ import annotations

import numpy as np
import pytest

import maivs_b200 as M
from datagen import build_index, mixture, oracle_build_index, shifted

pytestmark = pytest.mark.gpu

K = 10


@pytest.fixture(scope="module")
def loaded(tmp_path_factory):
    rng = np.random.default_rng(41)
    X, c = mixture(rng, 40_000, 384, 300)
    Q, _ = mixture(rng, 200, 384, 300, centers=c)
    Q = np.ascontiguousarray(np.vstack([Q, shifted(rng, Q[:100])]))
    ix = build_index(X, "quality", rf=16, tree_min_cells=64)
    path = str(tmp_path_factory.mktemp("persist_gpu") / "ix.maivs")
    ix.save(path)
    del ix
    ld = M.FlatCellIndex.load(path)
    ld.set_fastscan(True)
    ld.compact()
    ld.to_device(0)
    o = oracle_build_index(X, "quality", rf=16, tree_min_cells=64).index()
    return ld, o, Q


@pytest.mark.parametrize("cell_major,nprobe", [(True, 8), (True, 64), (False, 16), (False, 64)])
def test_loaded_index_gpu_search_equals_oracle(loaded, cell_major, nprobe):
    ld, o, Q = loaded
    ids, sc = ld.search_batch_arrays(Q, K, nprobe, 1.0, 8.0, cell_major)
    rid, rsc, *_ = o.search_batch(Q, K, nprobe, 1.0, 8.0, cell_major)
    assert np.array_equal(ids, rid)
    assert np.array_equal(sc.view(np.uint32), rsc.view(np.uint32))
