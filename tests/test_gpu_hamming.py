"""The GPU's per-query Hamming scan == the reference's search_one without FastScan blocks.

An index that is not a compacted FastScan index (fresh inserts before compact(), any remove()
since, FastScan switched off, a loaded file, every ConcurrentIndex segment) takes the Hamming
branch of search_one (index.rs:1693-1848): Hamming distances over the flat sign codes, a bucket
queue whose cut-off falls to the target-th smallest distance, every tie at it kept, the adaptive
stop on score_to_cos of the cut-off, then the exact rerank. The product runs it on the GPU
(k_pq_scan_ham, k_pq_fold<true>); the oracle side builds its own index from the same vectors with
the same operations and searches it on the CPU. Ids must be identical and scores bit-identical.
"""
from __future__ import annotations

import ctypes as C

import numpy as np
import pytest

import maivs_b200 as M
import oracle
from datagen import build_index, mixture, oracle_build_index

pytestmark = pytest.mark.gpu

K = 10


def _compare(ix, o, Q, nprobe, tc=1.0):
    got_ids, got_sc = ix.search_batch_arrays(Q, K, nprobe, tc, 8.0, False)
    ref_ids, ref_sc, _, _, used = o.search_batch(Q, K, nprobe, tc, 8.0, False)
    assert not used
    bad = np.nonzero((got_ids != ref_ids) | (got_sc.view(np.uint32) != ref_sc.view(np.uint32)))[0]
    assert bad.size == 0, (
        f"{bad.size} of {got_ids.size} entries differ (first query {bad[0] // K}): gpu {got_ids[bad[:4]]} "
        f"{got_sc[bad[:4]]} oracle {ref_ids[bad[:4]]} {ref_sc[bad[:4]]}")
    return got_ids


def _data(seed, n=24_000, nq=300):
    rng = np.random.default_rng(seed)
    X, centers = mixture(rng, n, 384, 180)
    Q, _ = mixture(rng, nq, 384, 180, centers=centers)
    return X, Q


@pytest.mark.parametrize("homes", [1, 2])
def test_after_remove_and_refill(homes):
    """A compacted quality index after deletes and inserts is no longer compacted: the reference
    searches it by Hamming distance, multi-home dedup by probe rank included."""
    X, Q = _data(31 + homes)
    base, extra = X[:20_000], X[20_000:]
    kw = dict(homes=homes, tree_min_cells=32)
    ix = build_index(base, rf=8, **kw)
    b = oracle_build_index(base, rf=8, **kw)
    for i in range(5, 20_000, 9):
        ix.remove(i)
        b.remove(i)
    new_ids = np.arange(90_000, 90_000 + extra.shape[0], dtype=np.uint64)
    ix.add_batch(new_ids, extra)
    b.add_batch(new_ids, extra)
    o = b.index()
    for nprobe in (8, 32):
        ids = _compare(ix, o, Q, nprobe)
        assert not np.isin(ids, np.arange(5, 20_000, 9, dtype=np.uint64)).any()


@pytest.mark.parametrize("adaptive", [False, True])
def test_fastscan_off_compacted(adaptive):
    """FastScan switched off on a compacted index: Hamming scan per query; the cell-major join on
    such an index is refused (the GPU join reads FastScan blocks)."""
    X, Q = _data(7)
    ix = build_index(X, rf=8, homes=1, tree_min_cells=10**9, adaptive=adaptive)
    b = oracle_build_index(X, rf=8, homes=1, tree_min_cells=10**9, adaptive=adaptive)
    ix.set_fastscan(False)
    b.set_fastscan(False)
    o = b.index()
    for nprobe in (4, 16, 64):
        _compare(ix, o, Q, nprobe)
    with pytest.raises(M.MaivsError, match="FastScan"):
        ix.search_batch_arrays(Q, K, 16, 1.0, 8.0, True)


def test_fresh_inserts_without_compact():
    """train_centroids + add_batch, never compacted: members are scattered slots."""
    X, Q = _data(12)
    ix = M.FlatCellIndex(384, "binary", 8, 0x5EED, 0)
    b = oracle.OracleBuild(384, "binary", 8, 0x5EED, 0)
    for h in (ix, b):
        h.set_graph_route(False, 10**9)
        h.set_adaptive(True, 0.02)
        h.train_centroids(X, 180)
    order = np.random.default_rng(4).permutation(X.shape[0])
    for part in np.array_split(order, 3):
        ids = part.astype(np.uint64)
        ix.add_batch(ids, np.ascontiguousarray(X[part]))
        b.add_batch(ids, np.ascontiguousarray(X[part]))
    o = b.index()
    for nprobe, tc in ((8, 1.0), (48, 1.0), (48, 0.9)):
        _compare(ix, o, Q, nprobe, tc)


def test_recall_of_the_hamming_scan():
    """The Hamming path is a working search: R@10 against brute force at a generous probe count."""
    X, Q = _data(3)
    ix = build_index(X, rf=16, homes=1, tree_min_cells=10**9, adaptive=False)
    ix.set_fastscan(False)
    ids, _ = ix.search_batch_arrays(Q, K, 48, 1.0, 8.0, False)
    truth = np.argsort(-(Q @ X.T), axis=1)[:, :K]
    got = ids.reshape(-1, K).astype(np.int64)
    rec = np.mean([len(set(a) & set(b)) / K for a, b in zip(got.tolist(), truth.tolist())])
    assert rec >= 0.9


def test_noalloc_entry_on_a_hamming_index():
    """The allocation-free entry point serves the Hamming scan too, with the same results."""
    import torch

    from maivs_b200 import _lib

    X, Q = _data(9, nq=48)
    ix = build_index(X, rf=8, homes=2, tree_min_cells=32)
    ix.remove(17)
    ix.to_device(0)
    dq = torch.from_numpy(Q).cuda()
    want_ids, want_sc = ix.search_batch_arrays(Q, K, 16, 1.0, 8.0, False)
    for _ in range(2):
        d_ids = torch.zeros(Q.shape[0] * K, dtype=torch.int64, device="cuda")
        d_sc = torch.zeros(Q.shape[0] * K, dtype=torch.float32, device="cuda")
        torch.cuda.synchronize()
        rc = _lib.lib().maivs_search_batch_device_noalloc(ix._h, C.c_void_p(dq.data_ptr()), Q.shape[0], K, 16, 1.0,
                                                           8.0, C.c_void_p(d_ids.data_ptr()),
                                                           C.c_void_p(d_sc.data_ptr()), None)
        assert rc == _lib.OK, _lib.lib().maivs_last_error(ix._h).decode()
        torch.cuda.synchronize()
        assert np.array_equal(d_ids.cpu().numpy().view(np.uint64), want_ids)
        assert np.array_equal(d_sc.cpu().numpy().view(np.uint32), want_sc.view(np.uint32))
