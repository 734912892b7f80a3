"""ConcurrentIndex's host side (src/concurrent.rs) against the oracle's restatement, on the CPU:
after every step of one call sequence, every sealed segment and the head must hold the same arrays
(seal = compact + fork_empty, tombstones, purge_head's removals and compaction), and the counts
(len, stats) must agree. The searches are compared on the GPU (test_gpu_concurrent.py); here the
oracle's own merge is checked against brute force."""
from __future__ import annotations

import numpy as np
import pytest

import maivs_b200 as M
import oracle
from concurrent_scenario import DIM, SEAL_AT, checkpoints, data

ARRAYS = oracle.OracleIndex.NAMES + ("prim_len", "rep_off", "slot_cell")


def _same(a: np.ndarray, c: np.ndarray, what: str):
    assert a.dtype == c.dtype and a.shape == c.shape, what
    assert np.array_equal(a.view(np.uint8), c.view(np.uint8)), f"{what}: {(a != c).sum()} entries differ"


def test_host_state_equals_oracle():
    X, extra, _ = data()
    cx = M.ConcurrentIndex(DIM, "binary", 8, 0x5EED, 0, SEAL_AT)
    ox = oracle.OracleConcurrentIndex(DIM, "binary", 8, 0x5EED, 0, SEAL_AT)
    seen = []
    for step_p, step_o in zip(checkpoints(cx, X, extra), checkpoints(ox, X, extra)):
        assert step_p == step_o
        seen.append(step_p)
        assert cx.n_segments() == len(ox.sealed), step_p
        assert len(cx) == len(ox), step_p
        st = cx.stats()
        assert st["segments"] == len(ox.sealed) and st["tombstones"] == len(ox.dead), step_p
        assert st["head_live"] == ox.head.n_live() and st["sealed_live"] == ox.sealed_live, step_p
        for s, (b, _) in enumerate(ox.sealed):
            for name in ARRAYS:
                _same(cx.segment_array(s, name), b.array(name), f"{step_p}: segment {s} {name}")
        for name in ARRAYS:
            _same(cx.segment_array(-1, name), ox.head.array(name), f"{step_p}: head {name}")
    assert seen[-1] == "sealed_all" and cx.n_segments() == 2


def test_seal_keeps_configuration_and_turns_fastscan_off():
    X, extra, _ = data()
    cx = M.ConcurrentIndex(DIM, "binary", 8, 0x5EED, 0, 1000)
    cx.set_adaptive(True, 0.05)
    cx.train_centroids(X[:4000], 32)
    cx.add_batch(np.arange(1500, dtype=np.uint64), np.ascontiguousarray(X[:1500]))
    assert cx.n_segments() == 1 and cx.stats()["head_live"] == 0
    seg, head = cx.segment_array(0, "config"), cx.segment_array(-1, "config")
    f = M.CONFIG_FIELDS
    assert seg[f.index("compacted")] == 1 and seg[f.index("fastscan")] == 0
    assert head[f.index("compacted")] == 0 and head[f.index("fastscan")] == 0
    for name in ("adaptive", "at_margin", "quant_scale", "rerank_factor", "nw"):
        assert seg[f.index(name)] == head[f.index(name)], name
    assert np.array_equal(cx.segment_array(0, "centroids"), cx.segment_array(-1, "centroids"))


def test_errors_mirror_the_reference():
    with pytest.raises(ValueError, match="scan_mode"):
        M.ConcurrentIndex(DIM, "f64")
    cx = M.ConcurrentIndex(DIM, seal_at=10)
    X, _, _ = data()
    with pytest.raises(ValueError, match="centroids"):  # add_batch before centroids (index.rs:2993-2996)
        cx.add_batch(np.arange(5, dtype=np.uint64), np.ascontiguousarray(X[:5]))
    assert not cx.remove(1) and cx.remove_many([1, 2]) == 0 and len(cx) == 0
    assert cx.purge_head() == 0


def test_oracle_merge_against_brute_force():
    """Probing every cell with a rerank factor covering whole cells, the oracle's multi-segment
    search must return the exact top k over live, non-tombstoned vectors, one entry per id."""
    X, extra, Q = data(9)
    Q = Q[:40]
    ox = oracle.OracleConcurrentIndex(DIM, "binary", 400, 0x5EED, 0, SEAL_AT)
    vec = {}
    for step in checkpoints(ox, X, extra, adaptive=False):
        if step in ("head_only", "sealed_one", "segment_and_head"):
            continue
        ids, sc = ox.search_batch(Q, 10, 48, 1.0, 8.0)
        # every copy of every live id, by segment, then the head
        copies = []
        for b, _ in ox.sealed + [(ox.head, None)]:
            mem = b.array("cell_members")
            ext = b.array("ext_ids")
            live = np.unique(mem)
            dim = DIM
            V = b.array("vecs_f32").reshape(-1, dim)
            copies.append((ext[live], V[live]))
        all_ids = np.concatenate([c[0] for c in copies])
        all_v = np.concatenate([c[1] for c in copies])
        keep = ~np.isin(all_ids, np.fromiter(ox.dead, np.uint64, len(ox.dead)))
        all_ids, all_v = all_ids[keep], all_v[keep]
        for qi in range(Q.shape[0]):
            s = all_v @ Q[qi]
            best = {}
            for i, v in zip(all_ids.tolist(), s.tolist()):
                best[i] = max(best.get(i, -np.inf), v)
            want = [i for i, _ in sorted(best.items(), key=lambda t: (-t[1], t[0]))[:10]]
            got = ids[qi * 10:(qi + 1) * 10].tolist()
            assert len(set(got) ^ set(want)) <= 2, (step, qi)  # float sums differ in the last bits
            assert not set(got) & ox.dead
            assert len(set(got)) == len(got)
