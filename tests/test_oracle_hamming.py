"""The oracle's Hamming scan (search_one without FastScan blocks) and the build's mutations
(remove, refill of freed slots, compaction that drops them, fork_empty), on the CPU.

The Hamming branch (index.rs:1693-1848) keeps every candidate at or below the target-th smallest
Hamming distance over the probed cells, ties included, and reranks them exactly. Here the candidate
sets the oracle sends to its rerank are recomputed in numpy from the index's own codes and probe
lists, and compared slot for slot."""
from __future__ import annotations

import numpy as np
import pytest

import oracle

DIM = 64
K = 10
RF = 8


def _data(n, seed):
    rng = np.random.default_rng(seed)
    c = rng.standard_normal((24, DIM)).astype(np.float32)
    x = c[rng.integers(0, 24, n)] + 0.4 * rng.standard_normal((n, DIM)).astype(np.float32)
    x /= np.linalg.norm(x, axis=1, keepdims=True)
    return np.ascontiguousarray(x, dtype=np.float32)


def _build(n=3000, seed=1, compact=False):
    X = _data(n, seed)
    b = oracle.OracleBuild(DIM, "binary", RF, 0x5EED, 0)
    b.train_centroids(X, 24, seed=7)
    b.add_batch(np.arange(n, dtype=np.uint64), X)
    if compact:
        b.compact()
    return X, b


def _popcount(a: np.ndarray) -> np.ndarray:
    return np.unpackbits(a.view(np.uint8), axis=-1).sum(axis=-1)


def _expected_cands(b: oracle.OracleBuild, Q: np.ndarray, nprobe: int):
    """Candidate slots of the non-adaptive Hamming branch, from the arrays and the probe lists."""
    ix = b.index()
    chosen, _, nch = ix.route(Q, nprobe, 1.0, 8.0, batch_router=False)
    cfg = b.array("config")
    dim_pad, nw = int(cfg[1]), int(cfg[2])
    signs = b.array("signs")
    qbits = oracle.encode(Q, signs, dim_pad, nw)
    bits = b.array("bits").reshape(-1, nw)
    mem, moff = b.array("cell_members"), b.array("cell_member_off")
    target = K * RF
    out = []
    for qi in range(Q.shape[0]):
        slots = np.concatenate([mem[moff[c]:moff[c + 1]] for c in chosen[qi, :nch[qi]]])
        h = _popcount(bits[slots] ^ qbits[qi][None, :])
        tau = np.sort(h)[target - 1] if h.size >= target else nw * 64
        out.append(np.sort(slots[h <= tau]))
    return ix, out


@pytest.mark.parametrize("compact", [False, True])
def test_hamming_candidates_match_numpy(compact):
    X, b = _build(compact=compact)
    Q = _data(40, 99)
    ix, want = _expected_cands(b, Q, 6)
    _, _, cands, cand_n, used = ix.search_batch(Q, K, 6, 1.0, 8.0, cell_major=False, cand_cap=4096)
    assert not used
    for qi in range(Q.shape[0]):
        got = cands[qi, :cand_n[qi]]
        assert np.array_equal(got, want[qi]), qi


def test_hamming_results_are_exact_rerank_of_candidates():
    X, b = _build()
    Q = _data(30, 5)
    ix, want = _expected_cands(b, Q, 8)
    ids, sc, _, _, _ = ix.search_batch(Q, K, 8, 1.0, 8.0, cell_major=False)
    ext = b.array("ext_ids")
    for qi in range(Q.shape[0]):
        cand_ids = ext[want[qi]]
        exact = X[cand_ids.astype(np.int64)] @ Q[qi]
        best = cand_ids[np.lexsort((cand_ids, -exact))][:K]
        got = ids[qi * K:(qi + 1) * K]
        # float sums differ from numpy's in the last bits: compare as sets with the scores close
        assert len(set(got.tolist()) ^ set(best.tolist())) <= 2
        np.testing.assert_allclose(np.sort(sc[qi * K:(qi + 1) * K]), np.sort(exact)[::-1][:K][::-1], rtol=1e-5,
                                   atol=1e-6)


def test_adaptive_stop_scans_a_prefix_of_the_probes():
    """With adaptive probing the candidates are exactly the Hamming branch's over some prefix of
    the probe list (the scan stops after a whole cell)."""
    X, b = _build()
    b.set_adaptive(True, 0.02)
    Q = _data(30, 11)
    ix = b.index()
    nprobe = 12
    chosen, _, nch = ix.route(Q, nprobe, 1.0, 8.0, batch_router=False)
    cfg = b.array("config")
    dim_pad, nw = int(cfg[1]), int(cfg[2])
    qbits = oracle.encode(Q, b.array("signs"), dim_pad, nw)
    bits = b.array("bits").reshape(-1, nw)
    mem, moff = b.array("cell_members"), b.array("cell_member_off")
    _, _, cands, cand_n, _ = ix.search_batch(Q, K, nprobe, 1.0, 8.0, cell_major=False, cand_cap=4096)
    stopped = 0
    for qi in range(Q.shape[0]):
        got = np.sort(cands[qi, :cand_n[qi]])
        match = None
        for p in range(1, int(nch[qi]) + 1):
            slots = np.concatenate([mem[moff[c]:moff[c + 1]] for c in chosen[qi, :p]])
            h = _popcount(bits[slots] ^ qbits[qi][None, :])
            tau = np.sort(h)[K * RF - 1] if h.size >= K * RF else nw * 64
            if np.array_equal(np.sort(slots[h <= tau]), got):
                match = p
                break
        assert match is not None, qi
        stopped += match < nch[qi]
    assert stopped > 0  # the stop rule fired somewhere


def test_remove_refill_and_compact():
    X, b = _build(n=2000)
    n0 = b.n_live()
    gone = list(range(0, 2000, 7))
    for i in gone:
        assert b.remove(i)
    assert not b.remove(0)
    assert not b.has_id(0) and b.has_id(1)
    assert b.n_live() == n0 - len(gone)
    # refill: the freed slots are reused (LIFO) before the arena grows
    Y = _data(100, 3)
    new_ids = np.arange(5000, 5100, dtype=np.uint64)
    slots_before = b.array("ext_ids").size
    b.add_batch(new_ids, Y)
    assert b.array("ext_ids").size == slots_before
    assert b.n_live() == n0 - len(gone) + 100
    mem = b.array("cell_members")
    ext = b.array("ext_ids")
    live = set(range(2000)) - set(gone) | set(new_ids.tolist())
    assert set(ext[mem].tolist()) == live
    b.compact()
    ext = b.array("ext_ids")
    assert ext.size == len(live) and set(ext.tolist()) == live
    mem, moff = b.array("cell_members"), b.array("cell_member_off")
    assert np.array_equal(np.sort(mem), np.arange(len(live)))
    for c in range(moff.size - 1):
        run = mem[moff[c]:moff[c + 1]]
        assert np.all(np.diff(run.astype(np.int64)) == 1)


def test_fork_empty_keeps_configuration_and_centroids():
    X, b = _build(n=2000)
    b.set_adaptive(True, 0.03)
    f = b.fork_empty()
    assert f.n_live() == 0
    assert np.array_equal(f.array("centroids"), b.array("centroids"))
    assert np.array_equal(f.array("signs"), b.array("signs"))
    cf, cb = f.array("config"), b.array("config")
    assert cf[9] == 0 and cf[16] == 0  # FastScan off, not compacted
    assert cf[13] == cb[13] and cf[14] == cb[14] and cf[15] == cb[15]  # adaptive, margin, quant_scale
    f.add_batch(np.arange(10_000, 10_500, dtype=np.uint64), _data(500, 8))
    assert f.n_live() == 500 and b.n_live() == 2000
