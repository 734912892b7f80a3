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


@pytest.mark.parametrize("nprobe", [8, 48])
def test_loaded_index_searched_as_loaded(tmp_path, nprobe):
    """A loaded index is not compacted and has FastScan off, exactly as the reference loads it; the
    GPU searches it that way, per query by Hamming distance over the loaded codes, with no host
    rebuild, and equals the oracle's search of the same loaded arrays. As in the reference, a
    cell-major request on an uncompacted index runs the per-query path (index.rs:3343-3348)."""
    import oracle

    rng = np.random.default_rng(43)
    X, c = mixture(rng, 30_000, 384, 250)
    Q, _ = mixture(rng, 128, 384, 250, centers=c)
    ix = build_index(X, "quality", rf=8, tree_min_cells=64)
    path = str(tmp_path / "ix.maivs")
    ix.save(path)
    del ix
    ld = M.FlatCellIndex.load(path)
    cfg = ld.array("config")
    assert cfg[M.CONFIG_FIELDS.index("compacted")] == 0 and cfg[M.CONFIG_FIELDS.index("fastscan")] == 0
    got_ids, got_sc = ld.search_batch_arrays(Q, K, nprobe, 1.0, 8.0, False)
    o = oracle.OracleIndex.from_index(ld)
    ref_ids, ref_sc, _, _, used = o.search_batch(Q, K, nprobe, 1.0, 8.0, False)
    assert not used
    assert np.array_equal(got_ids, ref_ids)
    assert np.array_equal(got_sc.view(np.uint32), ref_sc.view(np.uint32))
    cm_ids, cm_sc = ld.search_batch_arrays(Q, K, nprobe, 1.0, 8.0, True)
    assert np.array_equal(cm_ids, got_ids) and np.array_equal(cm_sc.view(np.uint32), got_sc.view(np.uint32))
    truth = np.argsort(-(Q @ X.T), axis=1)[:, :K]
    rec = np.mean([len(set(a) & set(b)) / K for a, b in zip(got_ids.reshape(-1, K).tolist(), truth.tolist())])
    assert rec >= 0.85
