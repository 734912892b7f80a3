"""ConcurrentIndex search on the GPU == the reference's query_all + finish (concurrent.rs:83-131).

The product runs every sealed segment and the head through the per-query Hamming scan on the GPU
and merges the lists in one kernel; the oracle restates the same calls on the CPU over its own
builds (OracleConcurrentIndex). After every step of the shared call sequence the two must return
identical ids and bit-identical scores. A second test lets reader threads search while a writer
inserts, deletes and seals, then checks the final state against the oracle.
"""
from __future__ import annotations

import threading

import numpy as np
import pytest

import maivs_b200 as M
import oracle
from concurrent_scenario import DIM, SEAL_AT, checkpoints, data

pytestmark = pytest.mark.gpu

K = 10


def _compare(cx, ox, Q, nprobe, tc, what):
    got_ids, got_sc = cx.search_batch_arrays(Q, K, nprobe, tc, 8.0)
    ref_ids, ref_sc = ox.search_batch(Q, K, nprobe, tc, 8.0)
    bad = np.nonzero((got_ids != ref_ids) | (got_sc.view(np.uint32) != ref_sc.view(np.uint32)))[0]
    assert bad.size == 0, (
        f"{what}: {bad.size} of {got_ids.size} entries differ (first query {bad[0] // K}): gpu {got_ids[bad[:4]]} "
        f"{got_sc[bad[:4]]} oracle {ref_ids[bad[:4]]} {ref_sc[bad[:4]]}")
    return got_ids


@pytest.mark.parametrize("adaptive", [True, False])
def test_search_equals_oracle_at_every_step(adaptive):
    X, extra, Q = data()
    cx = M.ConcurrentIndex(DIM, "binary", 8, 0x5EED, 0, SEAL_AT)
    ox = oracle.OracleConcurrentIndex(DIM, "binary", 8, 0x5EED, 0, SEAL_AT)
    for step_p, step_o in zip(checkpoints(cx, X, extra, adaptive), checkpoints(ox, X, extra, adaptive)):
        assert step_p == step_o
        for nprobe, tc in ((8, 1.0), (24, 1.0), (24, 0.95)):
            ids = _compare(cx, ox, Q, nprobe, tc, f"{step_p} nprobe={nprobe} tc={tc}")
            assert not np.isin(ids, np.fromiter(ox.dead, np.uint64, len(ox.dead))).any()
            rows = ids.reshape(-1, K)
            for r in rows:
                live = r[r != np.iinfo(np.uint64).max]
                assert np.unique(live).size == live.size  # one entry per id


def test_single_query_search_matches_batch():
    X, extra, Q = data(5)
    cx = M.ConcurrentIndex(DIM, "binary", 8, 0x5EED, 0, SEAL_AT)
    for _ in checkpoints(cx, X, extra):
        pass
    ids, sc = cx.search_batch_arrays(Q[:20], K, 16, 1.0, 8.0)
    for qi in range(20):
        i1, s1 = cx.search(Q[qi], K, 16, 1.0, 8.0)
        row = ids[qi * K:(qi + 1) * K]
        n = int((row != np.iinfo(np.uint64).max).sum())
        assert i1 == row[:n].tolist()
        assert np.array_equal(np.asarray(s1, np.float32), sc[qi * K:qi * K + n])


def test_readers_during_writes():
    """Searches from two threads while a third inserts, deletes and seals: no call fails, every
    answer holds distinct, known ids, and the final index searches like the oracle's after the
    same writes."""
    X, extra, Q = data(8)
    cx = M.ConcurrentIndex(DIM, "binary", 8, 0x5EED, 0, 2500)
    cx.set_graph_route(False, 10**9)
    cx.train_centroids(X[:8000], 48, seed=11)
    cx.add_batch(np.arange(0, 1000, dtype=np.uint64), np.ascontiguousarray(X[:1000]))
    errors: list[BaseException] = []
    stop = threading.Event()

    def writer():
        try:
            for lo in range(1000, 9000, 500):
                cx.add_batch(np.arange(lo, lo + 500, dtype=np.uint64), np.ascontiguousarray(X[lo:lo + 500]))
                cx.remove_many(np.arange(lo, lo + 500, 37, dtype=np.uint64))
            cx.purge_head()
        except BaseException as e:  # noqa: BLE001
            errors.append(e)
        finally:
            stop.set()

    def reader(seed):
        rng = np.random.default_rng(seed)
        try:
            while not stop.is_set():
                sel = rng.integers(0, Q.shape[0], 32)
                ids, _ = cx.search_batch_arrays(np.ascontiguousarray(Q[sel]), K, 16, 1.0, 8.0)
                for r in ids.reshape(-1, K):
                    live = r[r != np.iinfo(np.uint64).max]
                    assert np.unique(live).size == live.size
                    assert (live < 9000).all()
        except BaseException as e:  # noqa: BLE001
            errors.append(e)

    threads = [threading.Thread(target=writer)] + [threading.Thread(target=reader, args=(s,)) for s in (1, 2)]
    for t in threads:
        t.start()
    for t in threads:
        t.join(timeout=600)
    assert not errors, errors[0]
    assert cx.n_segments() >= 2

    ox = oracle.OracleConcurrentIndex(DIM, "binary", 8, 0x5EED, 0, 2500)
    ox.set_graph_route(False, 10**9)
    ox.train_centroids(X[:8000], 48, seed=11)
    ox.add_batch(np.arange(0, 1000, dtype=np.uint64), np.ascontiguousarray(X[:1000]))
    for lo in range(1000, 9000, 500):
        ox.add_batch(np.arange(lo, lo + 500, dtype=np.uint64), np.ascontiguousarray(X[lo:lo + 500]))
        ox.remove_many(np.arange(lo, lo + 500, 37, dtype=np.uint64))
    ox.purge_head()
    assert len(cx) == len(ox)
    _compare(cx, ox, Q, 16, 1.0, "after concurrent writes")
