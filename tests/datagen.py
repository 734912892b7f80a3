"""Seeded synthetic data for the tests, standing in for the reference's corpora.

`mixture` follows BASELINE.json's configs (centres N(0, I) normalised, per-coordinate noise
sigma / sqrt(d) as the reference's own generator scales it, tests/test_index.py:82-90, then
renormalised); `clustered` restates the reference test fixture (tests/test_index.py:51-95).
"""
from __future__ import annotations

import numpy as np


def unit(rng, n, d):
    x = rng.standard_normal((n, d)).astype(np.float32)
    x /= np.linalg.norm(x, axis=1, keepdims=True)
    return np.ascontiguousarray(x)


def mixture(rng, n, d, n_comp, sigma=0.35, centers=None):
    if centers is None:
        centers = unit(rng, n_comp, d)
    lab = rng.integers(0, len(centers), n)
    x = centers[lab] + (sigma / np.sqrt(d)) * rng.standard_normal((n, d)).astype(np.float32)
    x /= np.linalg.norm(x, axis=1, keepdims=True)
    return np.ascontiguousarray(x.astype(np.float32)), centers


def shifted(rng, q, weight=0.5):
    """OOD stand-in: sample + weight * random unit direction, renormalised."""
    u = unit(rng, q.shape[0], q.shape[1])
    x = q + weight * u
    x /= np.linalg.norm(x, axis=1, keepdims=True)
    return np.ascontiguousarray(x.astype(np.float32))


def clustered(rng, n, d, n_clusters=200, spread=0.7, skew=True, centers=None):
    if centers is None:
        centers = unit(rng, n_clusters, d)
    n_clusters = len(centers)
    w = np.geomspace(1.0, 0.05, n_clusters) if skew else np.ones(n_clusters)
    w = w / w.sum()
    counts = np.floor(w * n).astype(int)
    rem = n - counts.sum()
    if rem > 0:
        counts[np.argsort(-(w * n - counts))[:rem]] += 1
    sigma = spread / np.sqrt(d)
    parts = []
    for c, m in zip(centers, counts):
        if m <= 0:
            continue
        p = c[None, :] + sigma * rng.standard_normal((m, d)).astype(np.float32)
        p /= np.linalg.norm(p, axis=1, keepdims=True)
        parts.append(p)
    x = np.concatenate(parts).astype(np.float32)
    rng.shuffle(x)
    return np.ascontiguousarray(x), centers


def exact_topk(base, queries, k=10):
    sims = queries @ base.T
    return np.argsort(-sims, axis=1, kind="stable")[:, :k]


def recall(ids, truth, k=10):
    ids = np.asarray(ids).reshape(len(truth), -1)[:, :k].astype(np.int64)
    return float(np.mean([len(set(a.tolist()) & set(b.tolist())) / k for a, b in zip(ids, truth)]))


def build_index(X, preset="quality", rf=16, n_cells=None, tree_min_cells=2048, ids=None, code_bits=0,
                fanout=16, homes=2, adaptive=True, two_stage=True, replication=None):
    """The reference's benchmark presets (bench/fair/fairbench.py:98-119)."""
    import maivs_b200 as M

    n, d = X.shape
    ix = M.FlatCellIndex(d, "binary", rf, 0x5EED, code_bits)
    if preset == "memory":
        ix.set_per_dim_sq(True)
    if replication is not None:
        ix.set_replication(*replication)
    elif homes > 1:
        ix.set_orthogonal_polysemy(homes, 1.0)
    ix.set_fastscan(True)
    if two_stage:
        ix.set_two_stage(True, 2)
    ix.set_graph_route(False, 10**9)
    ix.set_tree_route(True, tree_min_cells, fanout)
    if adaptive:
        ix.set_adaptive(True, 0.02)
    ix.train_centroids(X, n_cells or max(16, n // 128))
    ix.add_batch(list(range(n)) if ids is None else ids, X)
    ix.compact()
    return ix


def oracle_build_index(X, preset="quality", rf=16, n_cells=None, tree_min_cells=2048, ids=None, code_bits=0,
                       fanout=16, homes=2, adaptive=True, two_stage=True, replication=None):
    """The same presets built by the oracle's own restatement of the reference build (test
    infrastructure; shares no code with the product's host build)."""
    import oracle

    n, d = X.shape
    b = oracle.OracleBuild(d, "binary", rf, 0x5EED, code_bits)
    if preset == "memory":
        b.set_per_dim_sq(True)
    if replication is not None:
        b.set_replication(*replication)
    elif homes > 1:
        b.set_orthogonal_polysemy(homes, 1.0)
    b.set_fastscan(True)
    if two_stage:
        b.set_two_stage(True, 2)
    b.set_graph_route(False, 10**9)
    b.set_tree_route(True, tree_min_cells, fanout)
    if adaptive:
        b.set_adaptive(True, 0.02)
    b.train_centroids(X, n_cells or max(16, n // 128))
    b.add_batch(np.arange(n, dtype=np.uint64) if ids is None else np.asarray(ids, np.uint64), X)
    b.compact()
    return b
