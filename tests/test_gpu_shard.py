"""Cell-range sharded search on one GPU: the protocol with its all-gathers done by device copies.

Each emulated shard scans only its cell range, exchanges its smallest distances twice (seed
cut-off, candidate cut-off) and its best-k list once; the merged result must equal the unsharded
cell-major join (index.rs:1999-2311) bit for bit, ids and f32 scores, and hence the oracle's.
"""
from __future__ import annotations

import numpy as np
import pytest

import oracle
from datagen import build_index, mixture

pytestmark = pytest.mark.gpu

K = 10


def _device_search(ix, Q, k, nprobe, world=None):
    import torch

    st = torch.cuda.Stream()
    with torch.cuda.stream(st):
        dq = torch.from_numpy(np.ascontiguousarray(Q)).cuda()
        ids = torch.empty(Q.shape[0] * k, dtype=torch.int64, device="cuda")
        sc = torch.empty(Q.shape[0] * k, dtype=torch.float32, device="cuda")
        if world is None:
            ix.search_batch_device(dq.data_ptr(), Q.shape[0], k, ids.data_ptr(), sc.data_ptr(), nprobe, 1.0, 8.0,
                                   True, st.cuda_stream)
        else:
            ix.search_batch_sharded_emulated(world, dq.data_ptr(), Q.shape[0], k, ids.data_ptr(), sc.data_ptr(),
                                             nprobe, 1.0, 8.0, st.cuda_stream)
    st.synchronize()
    assert ix.device_flags(st.cuda_stream) == 0
    return ids.cpu().numpy().view(np.uint64), sc.cpu().numpy()


@pytest.fixture(scope="module", params=["quality", "memory"])
def built(request):
    rng = np.random.default_rng(77)
    X, c = mixture(rng, 40_000, 384, 300)
    Q, _ = mixture(rng, 96, 384, 300, centers=c)
    ix = build_index(X, request.param, rf=8, tree_min_cells=2048)
    return ix, Q


@pytest.mark.parametrize("world", [2, 3, 5])
@pytest.mark.parametrize("nprobe", [4, 8, 24, 96])
def test_emulated_shards_equal_unsharded(built, world, nprobe):
    ix, Q = built
    ref_ids, ref_sc = _device_search(ix, Q, K, nprobe)
    ids, sc = _device_search(ix, Q, K, nprobe, world=world)
    assert np.array_equal(ids, ref_ids)
    assert np.array_equal(sc.view(np.uint32), ref_sc.view(np.uint32))


def test_emulated_shards_equal_oracle(built):
    ix, Q = built
    ids, sc = _device_search(ix, Q, K, 24, world=4)
    rid, rsc, *_ = oracle.OracleIndex.from_index(ix).search_batch(Q, K, 24, 1.0, 8.0, True)
    assert np.array_equal(ids, rid)
    assert np.array_equal(sc, rsc)


def test_single_shard_and_many_shards(built):
    """world = 1 is the whole index; more shards than needed leave some ranges tiny."""
    ix, Q = built
    ref_ids, ref_sc = _device_search(ix, Q, K, 16)
    for world in (1, 16):
        ids, sc = _device_search(ix, Q, K, 16, world=world)
        assert np.array_equal(ids, ref_ids), world
        assert np.array_equal(sc.view(np.uint32), ref_sc.view(np.uint32)), world


def test_small_batch_and_large_k(built):
    """Below the cell-major batch floor the sharded path still runs the cell-major join, whose
    per-query result does not depend on the rest of the batch: five queries at k = 50 equal their
    rows of the unsharded 96-query batch."""
    ix, Q = built
    ref_ids, ref_sc = _device_search(ix, Q, 50, 24)
    ids, sc = _device_search(ix, Q[:5], 50, 24, world=3)
    assert np.array_equal(ids, ref_ids[:250])
    assert np.array_equal(sc.view(np.uint32), ref_sc[:250].view(np.uint32))
