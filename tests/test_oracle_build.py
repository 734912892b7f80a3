"""The product's host index build against the oracle's independent restatement of the
reference build (train_centroids, add_batch with placement and polysemy, compact, derived
routing state): every array the search reads must be identical, bit for bit.

The two builds share no code: the product's is maivs_b200/csrc/host/*.cpp, the oracle's is the
build section of oracle/maivs_oracle.cpp, each restated from src/index.rs and src/tree.rs of the
reference. A mistake in k-means, placement, polysemy, compaction or the derived state on either
side shows up here as a mismatch, and the GPU parity tests search the oracle-built index."""
from __future__ import annotations

import numpy as np
import pytest

import oracle
from datagen import build_index, mixture, oracle_build_index

ARRAYS = oracle.OracleIndex.NAMES + ("prim_len", "rep_off", "slot_cell")


def assert_same_index(ix, b):
    for name in ARRAYS:
        a, c = ix.array(name), b.array(name)
        assert a.dtype == c.dtype and a.shape == c.shape, name
        assert np.array_equal(a.view(np.uint8), c.view(np.uint8)), f"{name}: {(a != c).sum()} entries differ"


CASES = {
    # 312 cells with a tree from 64 cells: tree placement (tree.rs:574-628) and one tree level
    "quality_tree": dict(n=40_000, d=384, comps=300, kw=dict(preset="quality", tree_min_cells=64)),
    "memory_tree": dict(n=40_000, d=384, comps=300, kw=dict(preset="memory", tree_min_cells=64)),
    # flat placement (no tree), one home
    "one_home_flat": dict(n=12_000, d=384, comps=100, kw=dict(homes=1)),
    # margin replication: up to three homes within 0.05 of the best (index.rs:2494-2504)
    "replication3": dict(n=12_000, d=384, comps=100, kw=dict(replication=(3, 0.05), tree_min_cells=32)),
    # three orthogonal homes
    "three_homes": dict(n=12_000, d=384, comps=100, kw=dict(homes=3)),
    # odd dimension, truncated 128-bit codes (dim_pad 128, 2 words)
    "d100_codes128": dict(n=8_000, d=100, comps=60, kw=dict(code_bits=128)),
    # d = 768: 1024-bit padding, 12 words at 768 code bits (BASELINE configs[4] layout)
    "d768_codes768": dict(n=6_000, d=768, comps=40, kw=dict(code_bits=768, preset="memory")),
}


@pytest.mark.parametrize("case", sorted(CASES))
def test_product_build_equals_oracle_build(case):
    c = CASES[case]
    X, _ = mixture(np.random.default_rng(100 + sorted(CASES).index(case)), c["n"], c["d"], c["comps"])
    ix = build_index(X, rf=8, **c["kw"])
    b = oracle_build_index(X, rf=8, **c["kw"])
    assert_same_index(ix, b)


def test_config1_index_equals_oracle_build():
    """100k x 384 from the 1,000-component mixture, quality preset (781 cells,
    flat two-stage routing)."""
    from bench import mixture as bench_mixture

    X, _, _ = bench_mixture(2024, 100_000, 10, 384, 1000, 0.35)
    ix = build_index(X, rf=48)
    b = oracle_build_index(X, rf=48)
    assert_same_index(ix, b)


def test_oracle_build_is_thread_count_independent():
    X, _ = mixture(np.random.default_rng(5), 20_000, 384, 150)
    oracle.lib().oracle_set_threads(1)
    b1 = oracle_build_index(X, tree_min_cells=64)
    oracle.lib().oracle_set_threads(8)
    b8 = oracle_build_index(X, tree_min_cells=64)
    for name in ARRAYS:
        assert np.array_equal(b1.array(name).view(np.uint8), b8.array(name).view(np.uint8)), name


@pytest.mark.parametrize("homes", [1, 2])
def test_mutations_equal_oracle(homes):
    """remove (index.rs:3223-3276), the refill of freed slots by add_batch (:3076-3198) and a
    compaction that drops them (:929-1112), in the same order on both sides: the uncompacted and
    the compacted index must match array for array (the uncompacted one is what the GPU's Hamming
    scan reads)."""
    X, _ = mixture(np.random.default_rng(77 + homes), 14_000, 384, 120)
    base, extra = X[:12_000], X[12_000:]
    kw = dict(homes=homes, tree_min_cells=32)
    ix = build_index(base, rf=8, **kw)
    b = oracle_build_index(base, rf=8, **kw)
    gone = list(range(3, 12_000, 11))
    for i in gone:
        assert ix.remove(i) and b.remove(i)
    assert not ix.remove(3) and not b.remove(3)
    assert_same_index(ix, b)
    new_ids = np.arange(50_000, 50_000 + extra.shape[0], dtype=np.uint64)
    ix.add_batch(new_ids, extra)
    b.add_batch(new_ids, extra)
    assert_same_index(ix, b)
    ix.compact()
    b.compact()
    assert_same_index(ix, b)
