"""A batch of 512 queries or more whose queries' work is independent (the cell-major join probing
only the seed cells, nprobe <= 8) is searched as two halves on two streams, through both the
device-buffer and the host-buffer API (the host API copies the second half in while the first is
searched). Every query's result depends only on that query and on the path the whole batch chose
(the cell-major join or the per-query path, index.rs:3343-3348), so the split search must return
exactly what the oracle returns for the whole batch: ids identical, scores bit-identical.
"""
from __future__ import annotations

import numpy as np
import pytest

from datagen import build_index, mixture

pytestmark = pytest.mark.gpu

K = 10


def _device_search(ix, Q, k, nprobe, cell_major):
    import torch

    st = torch.cuda.Stream()
    with torch.cuda.stream(st):
        dq = torch.from_numpy(np.ascontiguousarray(Q)).cuda()
        ids = torch.empty(Q.shape[0] * k, dtype=torch.int64, device="cuda")
        sc = torch.empty(Q.shape[0] * k, dtype=torch.float32, device="cuda")
        ix.search_batch_device(dq.data_ptr(), Q.shape[0], k, ids.data_ptr(), sc.data_ptr(), nprobe, 1.0, 8.0,
                               cell_major, st.cuda_stream)
    st.synchronize()
    assert ix.device_flags(st.cuda_stream) == 0
    return ids.cpu().numpy().view(np.uint64), sc.cpu().numpy()


def _oracle(ix, Q, nprobe, cell_major):
    import oracle

    o = oracle.OracleIndex.from_index(ix)
    ids, sc, _, _, used = o.search_batch(Q, K, nprobe, 1.0, 8.0, cell_major)
    return (ids, sc), used


def _same(got, ref):
    assert np.array_equal(np.asarray(got[0]).view(np.uint64), ref[0])
    assert np.array_equal(np.asarray(got[1]).view(np.uint32), ref[1].view(np.uint32))


@pytest.fixture(scope="module", params=["quality", "memory"])
def built(request):
    rng = np.random.default_rng(515)
    X, c = mixture(rng, 50_000, 384, 300)
    Q, _ = mixture(rng, 1_100, 384, 300, centers=c)
    ix = build_index(X, request.param, rf=8, tree_min_cells=2048)
    return ix, Q


@pytest.mark.parametrize("cell_major", [True, False])
@pytest.mark.parametrize("nprobe", [4, 8])
def test_split_batch_equals_oracle(built, cell_major, nprobe):
    ix, Q = built
    ref, used = _oracle(ix, Q, nprobe, cell_major)
    assert used == cell_major
    _same(ix.search_batch_arrays(Q, K, nprobe, 1.0, 8.0, cell_major), ref)
    _same(_device_search(ix, Q, K, nprobe, cell_major), ref)


def test_split_runs_two_halves(built):
    """The seed-only join of 1,100 queries launches every kernel of the search twice."""
    import maivs_b200 as M

    ix, Q = built
    _device_search(ix, Q[:300], K, 8, True)
    n0 = M.launch_count()
    _device_search(ix, Q[:300], K, 8, True)
    one = M.launch_count() - n0
    n0 = M.launch_count()
    _device_search(ix, Q, K, 8, True)
    two = M.launch_count() - n0
    assert two >= 2 * one - 2, (one, two)


def test_split_keeps_the_whole_batch_path(built):
    """With the cell-major threshold between a half and the whole batch, both halves must still
    run the cell-major join the 1,100-query batch chose (a half alone would go per query)."""
    import maivs_b200 as M

    ix, Q = built
    old = int(ix.array("config")[M.CONFIG_FIELDS.index("cm_min_batch")])
    ix.set_cell_major_min_batch(800)
    try:
        ref, used = _oracle(ix, Q, 8, True)
        assert used
        _same(ix.search_batch_arrays(Q, K, 8, 1.0, 8.0, True), ref)
        _same(_device_search(ix, Q, K, 8, True), ref)
        # a batch below the threshold goes per query through both APIs alike
        small = Q[:300]
        ref_s, used_s = _oracle(ix, small, 8, True)
        assert not used_s
        _same(ix.search_batch_arrays(small, K, 8, 1.0, 8.0, True), ref_s)
        _same(_device_search(ix, small, K, 8, True), ref_s)
    finally:
        ix.set_cell_major_min_batch(old)


@pytest.mark.parametrize("nq", [300, 1_100])
def test_pinned_queries_copied_without_staging(built, nq):
    """Queries in page-locked host memory (here a pinned torch tensor) are copied to the device from
    where they are, without the host API's staging copy: the results are the oracle's, for a batch
    that splits into two halves and for one that does not."""
    import torch

    ix, Q = built
    ref, _ = _oracle(ix, Q[:nq], 8, True)
    pinned = torch.from_numpy(np.ascontiguousarray(Q[:nq])).pin_memory()
    assert pinned.is_pinned()
    _same(ix.search_batch_arrays(pinned.numpy(), K, 8, 1.0, 8.0, True), ref)
    # the same buffer again, then a pageable copy: nothing of the previous call is reused
    _same(ix.search_batch_arrays(pinned.numpy(), K, 8, 1.0, 8.0, True), ref)
    _same(ix.search_batch_arrays(np.array(Q[:nq]), K, 8, 1.0, 8.0, True), ref)
