"""The host-buffer API searches a batch of 512 queries or more as two halves on two streams (the
second half's queries are copied in while the first half is searched). Every query's result
depends only on that query and on the path the whole batch chose (the cell-major join or the
per-query path, index.rs:3343-3348), so the split call must return exactly what one device call
over the whole batch returns: ids identical, scores bit-identical.
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


def _same(a, b):
    ids_a, sc_a = a
    ids_b, sc_b = b
    assert np.array_equal(ids_a, ids_b)
    assert np.array_equal(sc_a.view(np.uint32), sc_b.view(np.uint32))


@pytest.fixture(scope="module", params=["quality", "memory"])
def built(request):
    rng = np.random.default_rng(515)
    X, c = mixture(rng, 50_000, 384, 300)
    Q, _ = mixture(rng, 1_100, 384, 300, centers=c)
    ix = build_index(X, request.param, rf=8, tree_min_cells=2048)
    return ix, Q


@pytest.mark.parametrize("cell_major", [True, False])
@pytest.mark.parametrize("nprobe", [8, 48])
def test_split_host_batch_equals_one_device_call(built, cell_major, nprobe):
    ix, Q = built
    host = ix.search_batch_arrays(Q, K, nprobe, 1.0, 8.0, cell_major)
    dev = _device_search(ix, Q, K, nprobe, cell_major)
    _same((np.asarray(host[0]).view(np.uint64), np.asarray(host[1])), dev)


def test_split_keeps_the_whole_batch_path(built):
    """With the cell-major threshold between a half and the whole batch, both halves must still
    run the cell-major join the 1,100-query batch chose (a half alone would go per query)."""
    import maivs_b200 as M

    ix, Q = built
    old = int(ix.array("config")[M.CONFIG_FIELDS.index("cm_min_batch")])
    ix.set_cell_major_min_batch(800)
    try:
        host = ix.search_batch_arrays(Q, K, 24, 1.0, 8.0, True)
        dev = _device_search(ix, Q, K, 24, True)
        _same((np.asarray(host[0]).view(np.uint64), np.asarray(host[1])), dev)
        # and a small batch below the threshold goes per query through both APIs alike
        small = Q[:300]
        host_s = ix.search_batch_arrays(small, K, 24, 1.0, 8.0, True)
        dev_s = _device_search(ix, small, K, 24, True)
        _same((np.asarray(host_s[0]).view(np.uint64), np.asarray(host_s[1])), dev_s)
    finally:
        ix.set_cell_major_min_batch(old)
