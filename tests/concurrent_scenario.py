"""One sequence of ConcurrentIndex calls (src/concurrent.rs), run the same way on the product and on
the oracle's restatement: inserts across the seal threshold, tombstones in sealed segments and in
the head, ids re-inserted into the head while an older copy sits in a segment, purge_head, an
explicit seal. `checkpoints` yields after each step so a test can compare state or search results.
"""
from __future__ import annotations

import numpy as np

from datagen import mixture

DIM = 384
SEAL_AT = 4000


def data(seed: int = 404):
    rng = np.random.default_rng(seed)
    X, centers = mixture(rng, 9_000, DIM, 60)
    extra, _ = mixture(rng, 40, DIM, 60, centers=centers)
    Q, _ = mixture(rng, 200, DIM, 60, centers=centers)
    return X, extra, np.ascontiguousarray(Q)


def checkpoints(cx, X, extra, adaptive=True):
    """Drive `cx` (product ConcurrentIndex or oracle OracleConcurrentIndex); yields step names."""
    cx.set_graph_route(False, 10**9)
    if adaptive:
        cx.set_adaptive(True, 0.02)
    cx.train_centroids(X[:8000], 48, seed=11)

    def add(lo, hi):
        cx.add_batch(np.arange(lo, hi, dtype=np.uint64), np.ascontiguousarray(X[lo:hi]))

    add(0, 3000)
    yield "head_only"
    add(3000, 5000)  # crosses seal_at: the whole head becomes segment 0
    yield "sealed_one"
    add(5000, 7000)
    yield "segment_and_head"
    for i in list(range(10, 400, 10)) + list(range(5001, 5400, 7)):
        assert cx.remove(i)
    assert not cx.remove(10) and not cx.remove(123_456)
    # re-inserted ids: 10 is tombstoned (both copies stay hidden), 35 is live in segment 0 (the
    # better-scoring copy wins per query)
    cx.add_batch(np.array([10, 35], dtype=np.uint64), np.ascontiguousarray(extra[:2]))
    yield "tombstones"
    assert cx.remove_many(np.arange(6000, 6050, dtype=np.uint64)) == 50
    n = cx.purge_head()
    assert n > 0
    yield "purged"
    add(7000, 9000)
    yield "head_grown"
    cx.add_batch(np.arange(20_000, 20_038, dtype=np.uint64), np.ascontiguousarray(extra[2:]))
    cx.seal()
    yield "sealed_all"
