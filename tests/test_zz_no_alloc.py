"""The allocation-free search entry point against the ordinary device search.

maivs_search_batch_device_noalloc runs the per-query path with its scratch in a fixed device
array instead of allocated workspace; its results must equal maivs_search_batch_device with
cell_major = 0 bit for bit, on consecutive calls that reuse the same array. The file is named so
that pytest collects it last, which also checks that the array works after the rest of the suite
has used the device.
"""
from __future__ import annotations

import ctypes as C

import numpy as np
import pytest

from maivs_b200 import _lib
from datagen import build_index, mixture

K = 10


def _noalloc(ix, dq, nq, k, nprobe, d_ids, d_sc, stream):
    return _lib.lib().maivs_search_batch_device_noalloc(
        ix._h, C.c_void_p(dq), int(nq), int(k), int(nprobe), 1.0, 8.0, C.c_void_p(d_ids), C.c_void_p(d_sc),
        C.c_void_p(stream))


def _reference(ix, dq, nq, k, nprobe, d_ids, d_sc, stream):
    return _lib.lib().maivs_search_batch_device(
        ix._h, C.c_void_p(dq), int(nq), int(k), int(nprobe), 1.0, 8.0, 0, C.c_void_p(d_ids), C.c_void_p(d_sc),
        C.c_void_p(stream))


def _error(ix) -> str:
    return _lib.lib().maivs_last_error(ix._h).decode()


@pytest.fixture(scope="module", params=["flat_router", "tree_router"])
def built(request):
    rng = np.random.default_rng(20_000)
    X, centers = mixture(rng, 20_000, 384, 200)
    Q, _ = mixture(rng, 128, 384, 200, centers=centers)
    tree = 10**9 if request.param == "flat_router" else 64
    ix = build_index(X, "quality", rf=8, tree_min_cells=tree)
    return ix, Q


def test_requires_current_device_image():
    """Uploading allocates, so the entry point refuses an index without a current device image."""
    rng = np.random.default_rng(3)
    X, _ = mixture(rng, 3_000, 64, 20)
    ix = build_index(X, "quality", rf=4)
    rc = _noalloc(ix, 0, 4, K, 8, 0, 0, 0)
    assert rc == _lib.BAD_STATE
    assert "maivs_to_device" in _error(ix)


@pytest.mark.gpu
@pytest.mark.parametrize("nprobe", [8, 24])
def test_matches_device_search_on_consecutive_calls(built, nprobe):
    import torch

    ix, Q = built
    ix.to_device(0)
    stream = torch.cuda.Stream()
    sp = stream.cuda_stream
    batches = [Q[:40], Q[40:104], Q[104:105], Q[:40]]  # the last repeats the first after other calls
    got, ref = [], []
    with torch.cuda.stream(stream):
        dqs = [torch.from_numpy(np.ascontiguousarray(b)).cuda() for b in batches]
        for dq in dqs:
            n = dq.shape[0]
            ids = torch.empty(n * K, dtype=torch.int64, device="cuda")
            sc = torch.empty(n * K, dtype=torch.float32, device="cuda")
            rc = _noalloc(ix, dq.data_ptr(), n, K, nprobe, ids.data_ptr(), sc.data_ptr(), sp)
            assert rc == _lib.OK, _error(ix)
            got.append((ids, sc))
        for dq in dqs:
            n = dq.shape[0]
            ids = torch.empty(n * K, dtype=torch.int64, device="cuda")
            sc = torch.empty(n * K, dtype=torch.float32, device="cuda")
            rc = _reference(ix, dq.data_ptr(), n, K, nprobe, ids.data_ptr(), sc.data_ptr(), sp)
            assert rc == _lib.OK, _error(ix)
            ref.append((ids, sc))
    stream.synchronize()
    assert ix.device_flags(sp) == 0
    for i, ((gi, gs), (ri, rs)) in enumerate(zip(got, ref)):
        gi, gs, ri, rs = (t.cpu().numpy() for t in (gi, gs, ri, rs))
        assert np.array_equal(gi, ri), f"batch {i}: ids differ"
        assert np.array_equal(gs.view(np.uint32), rs.view(np.uint32)), f"batch {i}: scores differ"
    assert np.array_equal(got[0][0].cpu().numpy(), got[3][0].cpu().numpy())


@pytest.mark.gpu
def test_rejects_requests_beyond_the_scratch():
    import torch

    rng = np.random.default_rng(5)
    X, _ = mixture(rng, 70_000, 32, 300)
    ix = build_index(X, "quality", rf=4, tree_min_cells=10**9)
    ix.to_device(0)
    Q, _ = mixture(rng, 65, 32, 300)
    dq = torch.from_numpy(Q).cuda()
    ids = torch.empty(65 * K, dtype=torch.int64, device="cuda")
    sc = torch.empty(65 * K, dtype=torch.float32, device="cuda")
    rc = _noalloc(ix, dq.data_ptr(), 65, K, 8, ids.data_ptr(), sc.data_ptr(), 0)
    assert rc == _lib.BAD_ARG and "at most 64 queries" in _error(ix)
    # 546 cells holding up to 726 entries each: 64 queries x 540 probed cells of 8-byte entries
    # need well above 32 MiB
    rc = _noalloc(ix, dq.data_ptr(), 64, K, 540, ids.data_ptr(), sc.data_ptr(), 0)
    assert rc == _lib.BAD_ARG and "bytes of scratch" in _error(ix), _error(ix)
    # a request that fits still runs after the rejections
    rc = _noalloc(ix, dq.data_ptr(), 4, K, 8, ids.data_ptr(), sc.data_ptr(), 0)
    assert rc == _lib.OK, _error(ix)
    torch.cuda.synchronize()


@pytest.mark.gpu
def test_allocates_nothing_across_calls(built):
    """Free device memory is the same before and after repeated calls once the first call has set
    the array up (the ordinary device search would have grown its workspace here)."""
    import torch

    ix, Q = built
    ix.to_device(0)
    dq = torch.from_numpy(np.ascontiguousarray(Q[:64])).cuda()
    ids = torch.empty(64 * K, dtype=torch.int64, device="cuda")
    sc = torch.empty(64 * K, dtype=torch.float32, device="cuda")
    assert _noalloc(ix, dq.data_ptr(), 64, K, 16, ids.data_ptr(), sc.data_ptr(), 0) == _lib.OK, _error(ix)
    torch.cuda.synchronize()
    free0 = torch.cuda.mem_get_info()[0]
    for nprobe in (8, 16, 32, 8):
        assert _noalloc(ix, dq.data_ptr(), 64, K, nprobe, ids.data_ptr(), sc.data_ptr(), 0) == _lib.OK, _error(ix)
    torch.cuda.synchronize()
    assert torch.cuda.mem_get_info()[0] == free0
    assert ix.device_flags(0) == 0


@pytest.mark.gpu
def test_flags_report_a_shortlist_beyond_the_sort_limit():
    """A routing shortlist longer than 16,384 cells cannot be ordered; the call still returns OK
    (the work is only enqueued) and the caller learns it from the device flags."""
    import maivs_b200 as M
    import torch

    rng = np.random.default_rng(11)
    d = 64
    cents = rng.standard_normal((20_000, d)).astype(np.float32)
    cents /= np.linalg.norm(cents, axis=1, keepdims=True)
    X = cents[rng.integers(0, len(cents), 40_000)] + 0.02 * rng.standard_normal((40_000, d)).astype(np.float32)
    X = np.ascontiguousarray((X / np.linalg.norm(X, axis=1, keepdims=True)).astype(np.float32))
    ix = M.FlatCellIndex(d, "binary", 4, 0x5EED, 0)
    ix.set_fastscan(True)
    ix.set_graph_route(False, 10**9)
    ix.set_centroids(cents)
    ix.add_batch(list(range(len(X))), X)
    ix.compact()
    ix.to_device(0)
    dq = torch.from_numpy(X[:1].copy()).cuda()
    ids = torch.empty(K, dtype=torch.int64, device="cuda")
    sc = torch.empty(K, dtype=torch.float32, device="cuda")
    nprobe = 16_500  # the tree shortlist asks for 2 x nprobe cells: all live cells, above 16,384
    assert _noalloc(ix, dq.data_ptr(), 1, K, nprobe, ids.data_ptr(), sc.data_ptr(), 0) == _lib.OK, _error(ix)
    torch.cuda.synchronize()
    assert ix.device_flags(0) != 0
    # a request within the limits on the same handle comes back clean
    assert _noalloc(ix, dq.data_ptr(), 1, K, 64, ids.data_ptr(), sc.data_ptr(), 0) == _lib.OK, _error(ix)
    torch.cuda.synchronize()
    assert ix.device_flags(0) == 0
