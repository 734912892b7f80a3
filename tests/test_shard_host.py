"""Host side of the cell-range sharded search, on CPU with world_size-2 gloo process groups.

- every rank computes the same contiguous, entry-balanced cell ranges;
- the distance-list exchange the kernels use is exact: after each shard publishes its count and
  its smallest L distances, the kth smallest of the union equals the kth smallest of all shards'
  entries for every kth <= L (the seed cut-off and the candidate cut-off, index.rs:2150-2160,
  :2277-2306);
- shard_over_torch hands every rank rank 0's NCCL id.
"""
from __future__ import annotations

import os
import socket
import sys

import numpy as np
import pytest
import torch.distributed as dist
import torch.multiprocessing as mp

HERE = os.path.dirname(os.path.abspath(__file__))


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _init(rank: int, world: int, port: int):
    sys.path.insert(0, HERE)
    sys.path.insert(0, os.path.dirname(HERE))
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    import datetime

    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60))


def _small_index():
    from datagen import build_index, mixture

    rng = np.random.default_rng(5)
    X, _ = mixture(rng, 6_000, 64, 40)
    return build_index(X, "quality", rf=4)


def _ranges_worker(rank: int, world: int, port: int, out):
    _init(rank, world, port)
    try:
        ix = _small_index()
        mine = ix.shard_range(rank, world)
        got = [None] * world
        dist.all_gather_object(got, mine)
        off = ix.array("cell_member_off").astype(np.int64)
        if rank == 0:
            out.put((got, off.tolist()))
    finally:
        dist.destroy_process_group()


def test_shard_ranges_agree_and_tile_the_cells():
    port = _free_port()
    q = mp.get_context("spawn").SimpleQueue()
    mp.start_processes(_ranges_worker, args=(2, port, q), nprocs=2, start_method="spawn", join=True)
    ranges, off = q.get()
    M = len(off) - 1
    assert ranges[0][0] == 0 and ranges[-1][1] == M
    assert ranges[0][1] == ranges[1][0]
    sizes = np.diff(np.asarray(off))
    total = int(sizes.sum())
    for lo, hi in ranges:
        assert int(sizes[lo:hi].sum()) <= total / 2 + sizes.max()


def test_shard_ranges_many_worlds():
    ix = _small_index()
    sizes = np.diff(ix.array("cell_member_off").astype(np.int64))
    M, total = len(sizes), int(sizes.sum())
    for world in (1, 3, 7, M + 3):
        rs = [ix.shard_range(r, world) for r in range(world)]
        assert rs[0][0] == 0 and rs[-1][1] == M
        for (a, b), (c, d) in zip(rs, rs[1:]):
            assert b == c and a <= b
        for lo, hi in rs:
            assert int(sizes[lo:hi].sum()) <= total / world + sizes.max()


def _publish(d: np.ndarray, L: int):
    """What a shard publishes: its entry count and its smallest min(count, L) distances."""
    return len(d), np.sort(d)[:L]


def _kth_from_lists(lists, kth: int) -> int:
    return int(np.sort(np.concatenate([l for _, l in lists]))[kth - 1])


def _lists_worker(rank: int, world: int, port: int, out):
    _init(rank, world, port)
    try:
        rng = np.random.default_rng(100 + rank)
        trials = []
        for t in range(60):
            L = int(rng.integers(1, 40))
            # skewed shards: sometimes one shard holds most of the small distances, with ties
            n = int(rng.integers(0, 120))
            hi = int(rng.integers(2, 300))
            d = rng.integers(0, hi, n) + (0 if (t + rank) % 3 else 50)
            trials.append((L, d.astype(np.int64)))
        got = [None] * world
        dist.all_gather_object(got, trials)
        if rank == 0:
            out.put(got)
    finally:
        dist.destroy_process_group()


def test_list_exchange_select_is_exact():
    port = _free_port()
    q = mp.get_context("spawn").SimpleQueue()
    mp.start_processes(_lists_worker, args=(2, port, q), nprocs=2, start_method="spawn", join=True)
    per_rank = q.get()
    for t in range(len(per_rank[0])):
        L = per_rank[0][t][0]
        shards = [per_rank[r][t][1] for r in range(2)]
        union = np.sort(np.concatenate(shards))
        lists = [_publish(d, L) for d in shards]
        total = sum(c for c, _ in lists)
        assert total == len(union)
        for kth in range(1, min(L, total) + 1):
            assert _kth_from_lists(lists, kth) == union[kth - 1]


def _id_worker(rank: int, world: int, port: int, out):
    _init(rank, world, port)
    try:
        import maivs_b200 as M

        calls = []

        class Fake:
            def shard(self, r, w, nid):
                calls.append((r, w, nid))

        M.shard_over_torch(Fake())
        got = [None] * world
        dist.all_gather_object(got, calls[0])
        if rank == 0:
            out.put(got)
    finally:
        dist.destroy_process_group()


def test_shard_over_torch_shares_rank0_id():
    port = _free_port()
    q = mp.get_context("spawn").SimpleQueue()
    mp.start_processes(_id_worker, args=(2, port, q), nprocs=2, start_method="spawn", join=True)
    calls = q.get()
    assert [c[0] for c in calls] == [0, 1] and all(c[1] == 2 for c in calls)
    assert len(calls[0][2]) == 128 and calls[0][2] == calls[1][2]
