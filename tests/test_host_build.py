"""The host-side index build: layouts the GPU reads, checked against the oracle's own encoders,
plus the reference's structural invariants and thread-count independence."""
from __future__ import annotations

import os
import subprocess
import sys

import numpy as np
import pytest

import oracle
from datagen import build_index, mixture

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


@pytest.fixture(scope="module")
def built():
    rng = np.random.default_rng(21)
    X, _ = mixture(rng, 30_000, 384, 300)
    ix = build_index(X, "quality", rf=8, tree_min_cells=64)
    return X, ix


def test_codes_are_the_reference_encoding(built):
    X, ix = built
    signs = ix.array("signs")
    assert np.array_equal(signs, oracle.make_signs(512, 0x5EED))
    ext = ix.array("ext_ids").astype(np.int64)
    bits = ix.array("bits").reshape(-1, 8)
    assert np.array_equal(bits, oracle.encode(X[ext], signs, 512, 8))


def test_fastscan_blocks_are_the_reference_layout(built):
    X, ix = built
    bits = ix.array("bits").reshape(-1, 8)
    mem, moff = ix.array("cell_members"), ix.array("cell_member_off")
    fs, fo = ix.array("fs_codes"), ix.array("fs_off")
    bb = 2048
    for c in range(0, len(moff) - 1, 7):
        m = mem[moff[c]:moff[c + 1]]
        nb = (len(m) + 31) // 32
        assert fo[c + 1] - fo[c] == nb
        for b in range(nb):
            want = oracle.fs_pack_block(bits[m[b * 32:(b + 1) * 32]], 8)
            assert np.array_equal(fs[(fo[c] + b) * bb:(fo[c] + b + 1) * bb], want)


def test_centroid_codes_and_sq8(built):
    X, ix = built
    cents = ix.array("centroids").reshape(-1, 384)
    assert np.array_equal(ix.array("cent_bits").reshape(-1, 8), oracle.encode(cents, ix.array("signs"), 512, 8))
    moff = ix.array("cell_member_off")
    live = np.diff(moff) > 0
    lo, hi = cents[live].min(0), cents[live].max(0)
    step = ((hi - lo) / np.float32(255.0)).astype(np.float32)
    step = np.where(step > np.float32(1e-12), step, np.float32(1e-12)).astype(np.float32)
    assert np.array_equal(ix.array("csq_min"), lo) and np.array_equal(ix.array("csq_step"), step)
    q = np.round(((cents - lo) / step).astype(np.float32))  # numpy rounds half to even; check off-ties only
    sq = ix.array("cent_sq8").reshape(-1, 384).astype(np.float32)
    frac = np.abs(((cents - lo) / step).astype(np.float32) % 1 - 0.5)
    ok = frac > 1e-3
    assert np.array_equal(np.clip(q, 0, 255)[ok], sq[ok])


def test_polysemy_and_compaction_invariants(built):
    X, ix = built
    n = X.shape[0]
    mem, moff = ix.array("cell_members"), ix.array("cell_member_off")
    sc = ix.array("slot_cells").reshape(-1, 2)
    prim = ix.array("slot_cell")
    plen, roff = ix.array("prim_len"), ix.array("rep_off")
    assert len(ix) == n and mem.size == 2 * n  # two homes per vector (index.rs:2523-2560)
    assert np.all(sc[:, 0] == prim) and np.all(sc[:, 0] != sc[:, 1])
    seen = np.zeros(n, np.int64)
    for c in range(len(moff) - 1):
        m = mem[moff[c]:moff[c + 1]]
        p = plen[c]
        # primaries: one contiguous ascending run; replicas ascending (index.rs:1045-1070)
        assert np.all(np.diff(m[:p].astype(np.int64)) == 1)
        assert np.all(np.diff(m[p:].astype(np.int64)) > 0)
        assert roff[c + 1] - roff[c] == len(m) - p
        assert np.all(prim[m[:p]] == c) and np.all(prim[m[p:]] != c)
        assert np.all((sc[m, 0] == c) | (sc[m, 1] == c))
        seen[m] += 1
    assert np.all(seen == 2)
    # compaction puts every cell's primaries in cell order (index.rs:940-956)
    assert np.all(np.diff(prim.astype(np.int64)) >= 0)


def test_recall_of_the_build_matches_brute_force(built):
    X, ix = built
    o = oracle.OracleIndex.from_index(ix)
    Q = X[:64] + np.float32(0.02) * np.random.default_rng(2).standard_normal((64, 384)).astype(np.float32)
    Q = np.ascontiguousarray((Q / np.linalg.norm(Q, axis=1, keepdims=True)).astype(np.float32))
    ids, *_ = o.search_batch(Q, 10, 64, 1.0, 8.0, True)
    truth = np.argsort(-(Q @ X.T), axis=1)[:, :10]
    r = np.mean([len(set(ids[i * 10:(i + 1) * 10].tolist()) & set(truth[i].tolist())) / 10 for i in range(64)])
    assert r > 0.95


_DET_SCRIPT = r"""
import sys, hashlib, numpy as np
sys.path.insert(0, %r); sys.path.insert(0, %r)
from datagen import build_index, mixture
X, _ = mixture(np.random.default_rng(5), 12000, 256, 120)
ix = build_index(X, "memory", rf=4, tree_min_cells=32)
h = hashlib.sha256()
for n in ("bits", "centroids", "cell_members", "slot_cells", "fs_codes", "r_bound", "scan_i8", "tree_codes"):
    h.update(ix.array(n).tobytes())
print(h.hexdigest())
"""


def test_build_is_independent_of_thread_count():
    outs = []
    for t in ("1", "7"):
        env = dict(os.environ, OMP_NUM_THREADS=t)
        r = subprocess.run([sys.executable, "-c", _DET_SCRIPT % (ROOT, os.path.join(ROOT, "tests"))],
                           capture_output=True, text=True, env=env, timeout=600)
        assert r.returncode == 0, r.stderr
        outs.append(r.stdout.strip())
    assert outs[0] == outs[1]


def test_tree_shape(built):
    X, ix = built
    st = ix.stats()
    assert st["tree_depth"] == 0 or st["tree_top_width"] <= 256  # tree.rs:392 TOP_MAX


def test_errors_mirror_the_reference():
    import maivs_b200 as M

    with pytest.raises(ValueError, match="scan_mode must be"):
        M.FlatCellIndex(64, "bogus")
    ix = M.FlatCellIndex(64, "binary", 4, 0x5EED, 0)
    with pytest.raises(ValueError, match="set_centroids"):
        ix.add_batch([1], np.zeros((1, 64), np.float32))
    with pytest.raises(ValueError):
        ix.train_centroids(np.zeros((10, 32), np.float32), 2)
    ix.set_centroids(np.eye(64, dtype=np.float32)[:4])
    with pytest.raises(ValueError, match="shape mismatch"):
        ix.add_batch([1, 2], np.zeros((1, 64), np.float32))
    with pytest.raises(ValueError, match="C-contiguous"):
        ix.add_batch([1, 2], np.zeros((64, 2), np.float32).T)


def test_remove_and_readd():
    import maivs_b200 as M

    rng = np.random.default_rng(9)
    X, _ = mixture(rng, 3000, 128, 30)
    ix = build_index(X, "quality", rf=4)
    assert ix.remove(5) and not ix.remove(5) and len(ix) == 2999
    mem = ix.array("cell_members")
    # slot of id 5 no longer referenced by any cell; re-adding reuses the freed slot
    ix.add_batch([10_000], X[5:6])
    assert len(ix) == 3000
    ix.compact()
    ext = ix.array("ext_ids")
    assert 10_000 in ext.tolist() and 5 not in ext.tolist()
    assert mem.size == 2 * 2999
