"""Cell-range sharded search over NCCL, one process per GPU (needs two or more GPUs).

Each rank computes the unsharded cell-major result on its own GPU first, then shards the same
index over the ranks (rank r scans its cell range, the engine's NCCL communicator all-gathers the
distance lists and best-k lists) and searches again: ids and f32 scores must be identical on every
rank, for a batch with and without the rest scan, through the host and the device entry points.
"""
from __future__ import annotations

import os
import socket
import sys

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

HERE = os.path.dirname(os.path.abspath(__file__))


def _gpus() -> int:
    import torch

    return torch.cuda.device_count() if torch.cuda.is_available() else 0


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank: int, world: int, port: int, out):
    sys.path.insert(0, HERE)
    sys.path.insert(0, os.path.dirname(HERE))
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    import datetime

    import torch
    import torch.distributed as dist

    import maivs_b200 as M
    from datagen import build_index, mixture

    torch.cuda.set_device(rank)
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=120))
    try:
        rng = np.random.default_rng(2024)
        X, c = mixture(rng, 60_000, 384, 400)
        Q, _ = mixture(rng, 200, 384, 400, centers=c)
        ix = build_index(X, "quality", rf=8, tree_min_cells=2048)
        ix.to_device(rank)
        cases = [(10, 8), (10, 40), (20, 24)]
        ref = {case: ix.search_batch_arrays(Q, case[0], case[1], 1.0, 8.0, True) for case in cases}
        M.shard_over_torch(ix)
        bad = []
        for k, nprobe in cases:
            ids, sc = ix.search_batch_arrays(Q, k, nprobe, 1.0, 8.0, True)
            rid, rsc = ref[(k, nprobe)]
            if not (np.array_equal(ids, rid) and np.array_equal(sc.view(np.uint32), rsc.view(np.uint32))):
                bad.append(("host", k, nprobe, int(np.sum(ids != rid))))
        # device entry point on a torch stream
        st = torch.cuda.Stream()
        with torch.cuda.stream(st):
            dq = torch.from_numpy(Q).cuda()
            di = torch.empty(Q.shape[0] * 10, dtype=torch.int64, device="cuda")
            ds = torch.empty(Q.shape[0] * 10, dtype=torch.float32, device="cuda")
            ix.search_batch_device(dq.data_ptr(), Q.shape[0], 10, di.data_ptr(), ds.data_ptr(), 40, 1.0, 8.0, True,
                                   st.cuda_stream)
        st.synchronize()
        rid, rsc = ref[(10, 40)]
        if not np.array_equal(di.cpu().numpy().view(np.uint64), rid):
            bad.append(("device", 10, 40))
        lo, hi = ix.shard_range(rank, world)
        out.put((rank, bad, lo, hi))
        ix.shard(0, 1)  # release the communicator before the process group
    finally:
        dist.destroy_process_group()


@pytest.mark.skipif(_gpus() < 2, reason="needs two GPUs")
def test_nccl_shards_equal_unsharded():
    import torch.multiprocessing as mp

    world = min(_gpus(), 4)
    q = mp.get_context("spawn").SimpleQueue()
    mp.start_processes(_worker, args=(world, _free_port(), q), nprocs=world, start_method="spawn", join=True)
    res = sorted(q.get() for _ in range(world))
    assert all(not r[1] for r in res), res
    assert res[0][2] == 0 and all(res[i][3] == res[i + 1][2] for i in range(world - 1))
