#!/usr/bin/env python3
"""Headline benchmark: batch QPS at R@10 = 0.99 on 500k x 384.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl maivs|reference]

One step = one cell-major search_batch of 1,000 queries (k = 10) through the MAIVS `quality`
preset (bench/fair/fairbench.py:98-119 of the reference) on a seeded synthetic Gaussian mixture
standing in for HotpotQA/MiniLM (absent here). The operating point is the smallest (rerank_factor,
nprobe) on a fixed grid whose R@10 against exact brute force is >= 0.99; it depends only on recall,
so both arms measure the same configuration. Prints one JSON line on rank 0.

`--impl maivs` (default) times the GPU engine: queries and outputs resident in HBM, L2 flushed
between steps (outside each step's CUDA-event interval), max over ranks. Under torchrun each rank
serves its own 1,000-query batches against a full replica (weak scaling). `--impl reference` times
the reference's CPU path (the oracle port, test infrastructure) on the host cores.
"""
from __future__ import annotations

import argparse
import json
import os
import subprocess
import sys
import threading
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

METRIC = "batch QPS at R@10=0.99 (d=384) at 1/2/4/8 B200; scan HBM GB/s vs peak"
K = 10
TARGET_RECALL = 0.99
RF_GRID = (16, 24, 32, 48, 64, 96, 128)
NP_GRID = (8, 12, 16, 24, 32, 48, 64, 96, 128, 192, 256, 384, 512)


# ---- data ---------------------------------------------------------------------------------------

def mixture(seed: int, n: int, nq: int, d: int, comps: int, sigma: float):
    """centres N(0, I) normalised; points = centre + sigma/sqrt(d) noise,
    renormalised (the reference's own generator scales noise by 1/sqrt(d), tests/test_index.py:82-90).
    Returns base vectors, in-distribution queries and shifted (OOD stand-in) queries."""
    rng = np.random.default_rng(seed)
    c = rng.standard_normal((comps, d), dtype=np.float32)
    c /= np.linalg.norm(c, axis=1, keepdims=True)

    def draw(m):
        x = c[rng.integers(0, comps, m)]
        x += np.float32(sigma / np.sqrt(d)) * rng.standard_normal((m, d), dtype=np.float32)
        x /= np.linalg.norm(x, axis=1, keepdims=True)
        return np.ascontiguousarray(x)

    X = draw(n)
    Q = draw(nq)
    u = rng.standard_normal((nq, d), dtype=np.float32)
    u /= np.linalg.norm(u, axis=1, keepdims=True)
    S = Q + np.float32(0.5) * u
    S /= np.linalg.norm(S, axis=1, keepdims=True)
    return X, Q, np.ascontiguousarray(S.astype(np.float32))


def brute_force_topk(X: np.ndarray, Q: np.ndarray, k: int, device: str) -> np.ndarray:
    import torch

    xt = torch.from_numpy(X).to(device)
    out = []
    for i in range(0, Q.shape[0], 256):
        q = torch.from_numpy(Q[i:i + 256]).to(device)
        out.append(torch.topk(q @ xt.T, k, dim=1).indices.cpu().numpy())
    return np.concatenate(out)


def recall(ids: np.ndarray, truth: np.ndarray) -> float:
    ids = np.asarray(ids).reshape(len(truth), -1)[:, :K].astype(np.int64)
    return float(np.mean([len(set(a.tolist()) & set(b.tolist())) / K for a, b in zip(ids, truth)]))


def build_quality(X: np.ndarray, threads: int, build_device: int | None = None):
    """The `quality` preset (bench/fair/fairbench.py:98-119); build_device runs the build's k-means
    and placement on that GPU (the same index as the host build)."""
    import maivs_b200 as M

    M.set_num_threads(threads)  # torchrun exports OMP_NUM_THREADS=1

    n, d = X.shape
    ix = M.FlatCellIndex(d, "binary", 16, 0x5EED, 0)
    ix.set_build_device(build_device)
    ix.set_orthogonal_polysemy(2, 1.0)
    ix.set_fastscan(True)
    ix.set_two_stage(True, 2)
    ix.set_graph_route(False, 10**9)
    ix.set_tree_route(True, 2048, 16)
    ix.set_adaptive(True, 0.02)
    ix.train_centroids(X, max(16, n // 128))
    ix.add_batch(np.arange(n, dtype=np.uint64), X)
    ix.compact()
    return ix


def build_memory(X: np.ndarray, threads: int, build_device: int | None = None):
    """The reference's `memory` preset (bench/fair/fairbench.py:98-106): quality + per-dimension SQ8 rerank."""
    import maivs_b200 as M

    M.set_num_threads(threads)

    n, d = X.shape
    ix = M.FlatCellIndex(d, "binary", 16, 0x5EED, 0)
    ix.set_build_device(build_device)
    ix.set_per_dim_sq(True)
    ix.set_orthogonal_polysemy(2, 1.0)
    ix.set_fastscan(True)
    ix.set_two_stage(True, 2)
    ix.set_graph_route(False, 10**9)
    ix.set_tree_route(True, 2048, 16)
    ix.set_adaptive(True, 0.02)
    ix.train_centroids(X, max(16, n // 128))
    ix.add_batch(np.arange(n, dtype=np.uint64), X)
    ix.compact()
    return ix


def operating_point(search, truth, target: float = TARGET_RECALL) -> tuple[int, int, float]:
    """Smallest rerank factor (then smallest nprobe) on the grid with R@10 >= target."""
    best = None
    for rf in RF_GRID:
        if recall(search(rf, NP_GRID[-1]), truth) < target:
            continue
        lo, hi = 0, len(NP_GRID) - 1
        while lo < hi:
            mid = (lo + hi) // 2
            if recall(search(rf, NP_GRID[mid]), truth) >= target:
                hi = mid
            else:
                lo = mid + 1
        best = (rf, NP_GRID[lo], recall(search(rf, NP_GRID[lo]), truth))
        break
    if best is None:
        rf, np_ = RF_GRID[-1], NP_GRID[-1]
        best = (rf, np_, recall(search(rf, np_), truth))
    return best


# ---- clocks -------------------------------------------------------------------------------------

class ClockSampler:
    """nvidia-smi samples of SM clock and throttle reasons during the timed region."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu: int):
        self.gpu = gpu
        self.proc = None
        self.lines: list[str] = []

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(["nvidia-smi", "-i", str(self.gpu), f"--query-gpu={self.FIELDS}",
                                          "--format=csv,noheader,nounits", "-lms", "50"],
                                         stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            threading.Thread(target=self._read, daemon=True).start()
        except Exception:
            self.proc = None
        return self

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def wait_first(self, timeout: float = 5.0) -> None:
        """Block until nvidia-smi produced its first sample, then mark the timed region's start."""
        t = time.time()
        while self.proc and not self.lines and time.time() - t < timeout:
            time.sleep(0.01)
        self.mark = len(self.lines)

    def stop_mark(self) -> None:
        self.end = len(self.lines) + 1

    def __exit__(self, *a):
        if self.proc:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except Exception:
                self.proc.kill()

    def summary(self) -> dict:
        sm, mx, reasons = [], 0.0, set()
        names = ("hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap")
        lines = self.lines[getattr(self, "mark", 0):getattr(self, "end", len(self.lines))] or self.lines[-1:]
        for ln in lines:
            p = [x.strip() for x in ln.split(",")]
            if len(p) < 9:
                continue
            try:
                sm.append(float(p[1]))
                mx = max(mx, float(p[2]))
            except ValueError:
                continue
            for name, v in zip(names, p[5:9]):
                if v.lower() == "active":
                    reasons.add(name)
        return {"sm_mhz": float(np.median(sm)) if sm else None, "sm_max_mhz": mx or None,
                "reasons": sorted(reasons), "samples": len(sm)}


def measured_peaks() -> dict:
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            p = json.load(f)
        return {"hbm_gbs": float(p["hbm_gbs"]), "src": "measured"}
    except Exception:
        return {"hbm_gbs": 6650.0, "src": "fallback"}


# ---- arms ---------------------------------------------------------------------------------------

def pinned_queries(Q: np.ndarray):
    """A copy of the queries in page-locked host memory, and the tensor that owns it: the
    end-to-end legs read their inputs from pinned host memory, which the host-buffer API copies to
    the device without its staging copy."""
    import torch

    t = torch.from_numpy(np.ascontiguousarray(Q, dtype=np.float32)).pin_memory()
    return t, t.numpy()


def ncu_traffic(kernel: str, stats: dict):
    """DRAM bytes per launch of `kernel` from the committed ncu capture, scaled to this run's work."""
    path = os.path.join(os.path.dirname(os.path.abspath(__file__)), "profiles", "dram_traffic.json")
    try:
        with open(path) as f:
            ent = json.load(f).get(kernel)
    except (OSError, ValueError):
        return None
    if not ent:
        return None
    now = stats.get(ent["scale_counter"], 0.0)
    return round(ent["dram_bytes_per_launch"] * now / ent["counter_at_capture"]) if now else None


def kernel_profile(ix, step, n, flush, dev):
    """Every kernel's share of the device time over n extra steps with all kernels timed, and the
    kernel with the most time. Run outside the timed region: the clock's events between every pair
    of kernels would lengthen the steps."""
    import torch

    ix.kernel_clock(True)
    ix.kernel_times(reset=True)
    for _ in range(n):
        flush.zero_()
        step()
    torch.cuda.synchronize(dev)
    kt = ix.kernel_times(reset=True)
    ix.kernel_clock(False)
    tot = max(sum(v[0] for v in kt.values()), 1e-9)
    shares = {k: round(v[0] / tot, 4) for k, v in kt.items() if v[1]}
    dom = max(kt.items(), key=lambda kv: kv[1][0])[0]
    per_step = {k: v[0] / max(n, 1) for k, v in kt.items() if v[1]}
    return shares, dom, round(tot / max(n, 1), 4), per_step


def dist_env():
    ws = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    return ws, rank, local


def oracle_index(X: np.ndarray, rf: int, threads: int):
    """The oracle's own build of the `quality` preset (its restatement of the reference build,
    independent of the product's host build) and its query path over it."""
    import oracle

    b = oracle.build_preset(X, "quality", rf, threads=threads)
    return b.index()


def time_cpu_batches(o, Q, rf, np_, threads, budget_s=None, steps=None, warmup=1):
    """Full cell-major batches through the oracle on `threads` host threads: (mean s, best s, calls)."""
    o.set_rerank_factor(rf)
    for _ in range(max(warmup, 1)):
        o.search_batch(Q, K, np_, 1.0, 8.0, True, threads=threads)
    ts, t0 = [], time.perf_counter()
    while (steps is not None and len(ts) < steps) or (steps is None and (time.perf_counter() - t0 < budget_s or not ts)):
        t = time.perf_counter()
        o.search_batch(Q, K, np_, 1.0, 8.0, True, threads=threads)
        ts.append(time.perf_counter() - t)
    return float(np.mean(ts)), float(np.min(ts)), len(ts)


def cpu_baseline(o, Q, rf, np_, budget_s=12.0) -> dict:
    """The reference's CPU path (the oracle port) on every host core, over the same full batch."""
    threads = os.cpu_count() or 1
    mean_s, best_s, calls = time_cpu_batches(o, Q, rf, np_, threads, budget_s=budget_s)
    return {"value": round(Q.shape[0] / mean_s, 1), "unit": "queries/s", "cores": threads, "kind": "port",
            "best_of_calls": round(Q.shape[0] / best_s, 1),
            "sample": f"the full batch of {Q.shape[0]} IND queries per call, cell-major, the oracle's own build of "
                      f"the same vectors, (rf={rf}, nprobe={np_}); mean of {calls} calls (~{budget_s:.0f} s)"}


# ---- matched-recall frontier (bench/fair/summarise.py:26-45 of the reference) -------------------

TARGETS = (0.95, 0.98, 0.99, 0.995)
SWEEP_RF = (16, 32, 48, 64, 96)
SWEEP_NP = (8, 16, 32, 64, 128, 256, 512)


def frontier(pts):
    """Points not dominated in (recall up, qps up), ascending recall."""
    s = sorted(pts, key=lambda p: (-p["recall"], -p["qps"]))
    out, best = [], None
    for p in s:
        if best is None or p["qps"] > best:
            out.append(p)
            best = p["qps"]
    return sorted(out, key=lambda p: p["recall"])


def interp(front, t):
    """QPS at recall t, log-interpolated along the frontier, never extrapolated (None if unreached)."""
    import math

    for a, b in zip(front, front[1:]):
        if a["recall"] <= t <= b["recall"]:
            f = (t - a["recall"]) / max(b["recall"] - a["recall"], 1e-12)
            return round(math.exp(math.log(a["qps"]) + f * (math.log(b["qps"]) - math.log(a["qps"]))), 1)
    if front and abs(front[-1]["recall"] - t) < 1e-9:
        return front[-1]["qps"]
    return None


def matched(points):
    f = frontier(points)
    return {str(t): interp(f, t) for t in TARGETS}


def run_maivs(args):
    import torch

    ws, rank, local = dist_env()
    dist = None
    if ws > 1:
        import torch.distributed as dist_mod

        dist = dist_mod
        torch.cuda.set_device(local)
        dist.init_process_group("nccl", timeout=__import__("datetime").timedelta(seconds=600))
    dev = torch.device("cuda", local)
    torch.cuda.set_device(dev)
    torch.backends.cuda.matmul.allow_tf32 = False

    X, Q, Qs = mixture(args.seed, args.n, args.nq, 384, 1000, 0.35)
    threads = max(1, (os.cpu_count() or 1) // max(1, int(os.environ.get("LOCAL_WORLD_SIZE", ws))))
    t0 = time.perf_counter()
    ix = build_quality(X, threads, build_device=local)
    build_s = time.perf_counter() - t0
    ix.to_device(local)
    truth = brute_force_topk(X, Q, K, str(dev))
    truth_s = brute_force_topk(X, Qs, K, str(dev))

    def search(rf, np_, q=Q):
        ix.set_rerank_factor(rf)
        ids, _ = ix.search_batch_arrays(q, K, np_, 1.0, 8.0, True)
        return ids

    rf, np_, rec = operating_point(search, truth)
    rec_ood = recall(search(rf, np_, Qs), truth_s)
    ix.set_rerank_factor(rf)

    # ---- device-resident timing ----
    # a dedicated stream: torch's default (legacy) stream has handle 0, which the engine reads as
    # "the handle's own stream", so events on it would not bracket the search
    stream = torch.cuda.Stream(dev)
    torch.cuda.set_stream(stream)
    dq = torch.from_numpy(Q).to(dev)
    d_ids = torch.empty(args.nq * K, dtype=torch.int64, device=dev)
    d_sc = torch.empty(args.nq * K, dtype=torch.float32, device=dev)
    flush = torch.empty(256 << 20, dtype=torch.uint8, device=dev)

    def step():
        ix.search_batch_device(dq.data_ptr(), args.nq, K, d_ids.data_ptr(), d_sc.data_ptr(), np_, 1.0, 8.0, True,
                               stream.cuda_stream)

    for _ in range(max(args.warmup, 3)):
        flush.zero_()
        step()
    torch.cuda.synchronize(dev)
    if ix.device_flags(stream.cuda_stream):
        for _ in range(2):
            step()
        torch.cuda.synchronize(dev)
        ix.device_flags(stream.cuda_stream)
    # results of the device path equal the host path's
    host_ids, _ = ix.search_batch_arrays(Q, K, np_, 1.0, 8.0, True)
    assert np.array_equal(d_ids.cpu().numpy().view(np.uint64), host_ids)

    from maivs_b200 import launch_count

    # kernel shares from a separate pass; inside the timed region only the dominant kernel carries
    # CUDA events (its live duration is the roofline's denominator)
    shares, dom_kernel, kernel_ms_per_step, kms_step = kernel_profile(ix, step, min(args.steps, 100), flush, dev)
    ix.kernel_clock(True, only=dom_kernel)
    ix.kernel_times(reset=True)
    evs = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(args.steps)]
    if dist:
        dist.barrier()
    torch.cuda.synchronize(dev)
    launches0 = launch_count()
    with ClockSampler(local) as clk:
        clk.wait_first()
        # a profiler started with --profile-from-start off sees only the timed steps
        torch.cuda.profiler.start()
        for s in range(args.steps):
            flush.zero_()
            evs[s][0].record(stream)
            step()
            evs[s][1].record(stream)
        torch.cuda.synchronize(dev)
        torch.cuda.profiler.stop()
        clk.stop_mark()
    launches = launch_count() - launches0
    if dist:
        dist.barrier()
    step_ms = [a.elapsed_time(b) for a, b in evs]
    total_ms = float(sum(step_ms))
    overflow = ix.device_flags(stream.cuda_stream)
    kbusy = ix.kernel_busy()
    ktimes = ix.kernel_times(reset=True)
    ix.kernel_clock(False)
    stats = ix.last_search_stats()

    # ---- end to end through the public host-buffer API, queries in pinned host memory ----
    q_pin_owner, q_pin = pinned_queries(Q)
    e2e_s = []
    for s in range(args.steps):
        flush.zero_()
        torch.cuda.synchronize(dev)
        t = time.perf_counter()
        ix.search_batch_arrays(q_pin, K, np_, 1.0, 8.0, True)
        e2e_s.append(time.perf_counter() - t)
    e2e_total = float(sum(e2e_s))

    if dist:
        t = torch.tensor([total_ms, e2e_total], dtype=torch.float64, device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        total_ms, e2e_total = float(t[0]), float(t[1])

    queries = args.nq * args.steps * ws
    qps = queries / (total_ms / 1e3)
    e2e_qps = queries / e2e_total
    got_ids = d_ids.cpu().numpy().view(np.uint64).copy()
    got_sc = d_sc.cpu().numpy().copy()

    # the union of candidate rows the batch reranks (each row is needed once per batch), from the
    # GPU path's own candidate lists
    cand = ix.debug_stage(2, Q, K, np_, 1.0, 8.0, True, cand_cap=4096)
    rows = np.concatenate([cand["cand"][i, :cand["cand_n"][i]] for i in range(args.nq)])
    union_rows = int(np.unique(rows).size)

    # recall sweep over (rf, nprobe) for in-distribution and shifted queries, device-resident
    sweep = {"IND": [], "OOD": []}
    if not args.no_sweep:
        dqs = torch.from_numpy(Qs).to(dev)
        for tag, qh, qd, tr in (("IND", Q, dq, truth), ("OOD", Qs, dqs, truth_s)):
            for srf in SWEEP_RF:
                for snp in SWEEP_NP:
                    ix.set_rerank_factor(srf)
                    rec_p = recall(ix.search_batch_arrays(qh, K, snp, 1.0, 8.0, True)[0], tr)
                    ev = [torch.cuda.Event(enable_timing=True) for _ in range(2)]
                    ms = []
                    for it in range(8):
                        flush.zero_()
                        ev[0].record(stream)
                        ix.search_batch_device(qd.data_ptr(), args.nq, K, d_ids.data_ptr(), d_sc.data_ptr(), snp,
                                               1.0, 8.0, True, stream.cuda_stream)
                        ev[1].record(stream)
                        ev[1].synchronize()
                        if it >= 2:
                            ms.append(ev[0].elapsed_time(ev[1]))
                    ix.device_flags(stream.cuda_stream)
                    sweep[tag].append({"rf": srf, "nprobe": snp, "recall": round(rec_p, 4),
                                       "qps": round(args.nq / (float(np.mean(ms)) / 1e3), 1)})
        ix.set_rerank_factor(rf)

    # roofline of the dominant kernel
    peaks = measured_peaks()
    name = dom_kernel
    kms, kl = ktimes.get(name, (0.0, 0))
    per_launch_ms = kms / max(kl, 1)
    # launches of the kernel per step: 2 when the library searches the batch as two halves
    lps = kl / max(args.steps, 1)
    row_bytes = stats.get("rerank_row_bytes", 1536.0)
    if name == "k_rerank":
        alg = union_rows * row_bytes
        what = (f"union of the batch's candidate rows x {row_bytes:.0f} B (each row once per batch); "
                f"{union_rows} distinct of {int(stats.get('candidates', 0))} (query, candidate) pairs")
    elif name == "k_seed":
        alg = (stats.get("seed_code_bytes", 0.0) + stats.get("nq", 0.0) * (16 * 128 + 64)
               + stats.get("seed_kept", 0.0) * 8)
        what = "1-bit codes of the union of seed cells, each read once, + query LUTs and codes + kept entries"
    elif name == "k_scan_cm":
        alg = stats.get("scan_code_bytes", 0.0)
        what = "1-bit codes of every scanned cell, each read once (members x 64 B)"
    elif name == "k_route_flat":
        alg = stats.get("route_code_bytes", 0.0)
        what = "centroid codes (cells x 64 B)"
    else:
        alg = stats.get("scan_code_bytes", 0.0) + stats.get("rerank_bytes", 0.0)
        what = "scan codes + rerank rows"
    # the batch's algorithmic bytes over the time per step during which the kernel ran: the two
    # halves' launches of a split batch overlap, so their summed durations would count that twice
    busy_ms = kbusy.get(name, 0.0) / max(args.steps, 1)
    alg_launch = alg / max(lps, 1.0)
    achieved = alg / (busy_ms / 1e3) / 1e9 if busy_ms > 0 else 0.0
    traffic = ncu_traffic(name, stats)
    if traffic:
        traffic = round(traffic / max(lps, 1.0))

    # the scan: algorithmic code bytes (union of scanned cells, each once per batch) over the scan
    # kernels' device time from the all-kernel pass
    scan_k = [k for k in ("k_seed_scan", "k_scan_cm", "k_scan_mma") if k in kms_step]
    scan_ms = sum(kms_step[k] for k in scan_k)
    scan_bytes = stats.get("seed_code_bytes", 0.0) + stats.get("scan_code_bytes", 0.0)
    scan_gbs = scan_bytes / (scan_ms / 1e3) / 1e9 if scan_ms > 0 else 0.0

    # parity: the timed batch's ids and scores against the oracle's own build + search of the
    # same vectors and queries
    threads_cpu = os.cpu_count() or 1
    o = oracle_index(X, rf, threads_cpu)
    ref_ids, ref_sc, *_ = o.search_batch(Q, K, np_, 1.0, 8.0, True, threads=threads_cpu)
    parity = bool(np.array_equal(got_ids, ref_ids) and np.array_equal(got_sc.view(np.uint32), ref_sc.view(np.uint32)))

    out = {
        "metric": METRIC,
        "value": round(qps, 1),
        "unit": "queries/s",
        "n_gpus": ws,
        "steps": args.steps,
        "warmup": args.warmup,
        "ms_per_step": round(total_ms / args.steps, 4),
        "higher_is_better": True,
        "scaling": "weak",
        "vs_baseline": None,
        "dtype": "u8",
        "data": "synthetic",
        "config": {
            "workload": "BASELINE configs[1]: 500k x 384 Gaussian mixture (1000 comps, sigma 0.35), quality preset, "
                        "cell-major batches of 1000 queries, k=10",
            "n": args.n, "dim": 384, "nq_per_step": args.nq, "k": K, "rerank_factor": rf, "nprobe": np_,
            "recall_at_10": round(rec, 4), "recall_at_10_shifted": round(rec_ood, 4),
            "cells": int(ix.stats()["n_cells"]), "l2_flush": "256 MiB write before each step, outside its timing",
            "parallelism": f"replicas x{ws}" if ws > 1 else "1 GPU", "build_s": round(build_s, 1),
            "build": "k-means and placement on the GPU (maivs_set_build_device)",
            "step_ms_min_max": [round(min(step_ms), 4), round(max(step_ms), 4)], "overflow_flags": overflow,
        },
        "e2e": {"value": round(e2e_qps, 1), "unit": "queries/s", "h2d_bytes_per_step": args.nq * 384 * 4,
                "d2h_bytes_per_step": args.nq * K * 12},
        "gpu_launches": int(launches),
        "roofline": {"bound": "hbm", "kernel": name, "achieved": round(achieved, 1), "peak": peaks["hbm_gbs"],
                     "unit": "GB/s", "frac": round(achieved / peaks["hbm_gbs"], 4), "traffic": traffic,
                     "algorithmic_bytes_per_launch": round(alg_launch), "avg_launch_ms": round(per_launch_ms, 5),
                     "launches_per_step": round(lps, 2), "algorithmic_bytes_per_step": round(alg),
                     "busy_ms_per_step": round(busy_ms, 5),
                     "what": what + "; achieved = bytes per step / busy_ms_per_step (the time per step during "
                                    "which at least one launch of the kernel ran)", "peak_src": peaks["src"]},
        "scan": {"kernels": scan_k, "bytes_per_step": round(scan_bytes), "ms_per_step": round(scan_ms, 5),
                 "achieved": round(scan_gbs, 1), "peak": peaks["hbm_gbs"], "unit": "GB/s",
                 "frac": round(scan_gbs / peaks["hbm_gbs"], 4),
                 "what": "1-bit codes of the union of the batch's scanned cells, 64 B per member entry, each cell "
                         "once per batch, over the scan kernels' device time (all-kernel pass)"},
        "parity": parity,
        "parity_src": f"ids and f32 scores of the timed batch ({args.nq} queries) bit-identical to the oracle's "
                      "own build and search of the same vectors",
        "sweep": sweep,
        "qps_at_recall": {t: matched(p) for t, p in sweep.items() if p},
        "sweep_src": "device-resident batch QPS per (rf, nprobe), mean of 6 timed batches, L2 flushed; QPS at "
                     "R@10 targets log-interpolated on the Pareto frontier (reference bench/fair/summarise.py)",
        "kernel_share": shares,
        "kernel_share_src": f"separate pass of {min(args.steps, 100)} steps with every kernel timed: "
                            f"{kernel_ms_per_step} ms of kernel time per step",
        "work": {**{k: round(v, 1) for k, v in stats.items()}, "rerank_union_rows": union_rows},
        "clocks": clk.summary(),
    }
    if rank == 0 and ws == 1:
        out["cpu_baseline"] = cpu_baseline(o, Q, rf, np_)
    if rank == 0:
        print(json.dumps(out), flush=True)
    if dist:
        dist.barrier()
        dist.destroy_process_group()


def mixture_torch(seed: int, n: int, nq: int, d: int, comps: int, sigma: float, device):
    """The same mixture recipe drawn on the GPU (the sharded config is 5.2M vectors): centres
    N(0, I) normalised, points = centre + sigma/sqrt(d) noise, renormalised."""
    import torch

    g = torch.Generator(device=device)
    g.manual_seed(seed)
    c = torch.randn(comps, d, generator=g, device=device)
    c /= c.norm(dim=1, keepdim=True)

    def draw(m):
        out = np.empty((m, d), np.float32)
        for i in range(0, m, 1 << 20):
            j = min(m, i + (1 << 20))
            x = c[torch.randint(0, comps, (j - i,), generator=g, device=device)]
            x += (sigma / d ** 0.5) * torch.randn(j - i, d, generator=g, device=device)
            x /= x.norm(dim=1, keepdim=True)
            out[i:j] = x.cpu().numpy()
        return out

    return draw(n), draw(nq)


def _scratch_dir(need_bytes: int) -> str:
    for d in ("/dev/shm", "/tmp"):
        try:
            st = os.statvfs(d)
            if st.f_bavail * st.f_frsize > 1.2 * need_bytes:
                return d
        except OSError:
            pass
    return "/tmp"


def sharded_paths(args):
    """Scratch files of the sharded workload, shared by the runs of one box: the MAIVS2 index, the
    queries and their exact top-k."""
    tag = f"maivs_cfg4_{args.n}_{args.nq}_{args.seed}"
    d0 = _scratch_dir(args.n * 384 * 6)
    path, qpath, tpath = (os.path.join(d0, tag + ext) for ext in (".maivs", ".q.npy", ".truth.npy"))
    return path, qpath, tpath, d0, tag


def sharded_queries(args, X, Q, dev):
    """The batch and its exact top-k (brute force on the GPU), computed once and cached."""
    _, qpath, tpath, _, _ = sharded_paths(args)
    if not (os.path.exists(qpath) and os.path.exists(tpath)):
        if X is None:
            X, Q = mixture_torch(args.seed, args.n, args.nq, 384, 10_000, 0.35, dev)
        truth = brute_force_topk(X, Q, K, str(dev))
        np.save(qpath + ".part.npy", Q)
        np.save(tpath + ".part.npy", truth)
        os.replace(qpath + ".part.npy", qpath)
        os.replace(tpath + ".part.npy", tpath)
    return np.load(qpath), np.load(tpath)


def sharded_oracle_answers(args, rf, np_, sample, dev):
    """The oracle's answers (its own build of the same vectors, cell-major search) for the first
    `sample` queries of the sharded batch; cached, since an oracle build of 5.2M vectors takes
    minutes on the host cores. Cell-major results do not depend on the other queries of a batch."""
    import oracle

    _, qpath, _, d0, tag = sharded_paths(args)
    cache = os.path.join(d0, f"{tag}.oracle_{rf}_{np_}_{sample}.npz")
    if not os.path.exists(cache):
        X, _ = mixture_torch(args.seed, args.n, args.nq, 384, 10_000, 0.35, dev)
        o = oracle.build_preset(X, "quality", rf, threads=os.cpu_count() or 1).take_index()
        del X
        Q = np.load(qpath)[:sample]
        ids, sc, *_ = o.search_batch(Q, K, np_, 1.0, 8.0, True, threads=os.cpu_count() or 1)
        np.savez(cache + ".part.npz", ids=ids, sc=sc)
        os.replace(cache + ".part.npz", cache)
    z = np.load(cache)
    return z["ids"], z["sc"]


def run_sharded(args):
    """5.2M x 384 (10,000-component mixture), quality preset, 10,000-query
    batches, cells sharded by range over the ranks (one per GPU), NCCL all-gathers + device merge.
    Strong scaling: the index and the batch are the same at every N. Rank 0 builds the index once
    on the host cores and writes it in the MAIVS2 format; every rank loads that file."""
    import datetime

    import torch
    import torch.distributed as tdist

    import maivs_b200 as M

    ws, rank, local = dist_env()
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if ws > 1:
        tdist.init_process_group("gloo", timeout=datetime.timedelta(seconds=1800))
    n, nq = args.n, args.nq
    path, qpath, tpath, d0, tag = sharded_paths(args)
    M.set_num_threads(max(1, (os.cpu_count() or 1) // max(1, int(os.environ.get("LOCAL_WORLD_SIZE", ws)))))
    build_s = 0.0
    if rank == 0 and not os.path.exists(path):
        X, Q = mixture_torch(args.seed, n, nq, 384, 10_000, 0.35, dev)
        t0 = time.perf_counter()
        ix0 = build_quality(X, os.cpu_count() or 1, build_device=local)
        build_s = time.perf_counter() - t0
        ix0.save(path + ".part")
        del ix0
        sharded_queries(args, X, Q, dev)
        del X
        os.replace(path + ".part", path)
    elif rank == 0:
        sharded_queries(args, None, None, dev)
    if ws > 1:
        tdist.barrier()
    Q, truth = sharded_queries(args, None, None, dev)
    ix = M.FlatCellIndex.load(path)
    ix.set_graph_route(False, 10**9)
    ix.set_fastscan(True)
    ix.compact()
    ix.to_device(local)
    if ws > 1:
        M.shard_over_torch(ix)
    lo, hi = ix.shard_range(rank, ws)

    stream = torch.cuda.Stream(dev)
    torch.cuda.set_stream(stream)
    dq = torch.from_numpy(Q).to(dev)
    d_ids = torch.empty(nq * K, dtype=torch.int64, device=dev)
    d_sc = torch.empty(nq * K, dtype=torch.float32, device=dev)
    flush = torch.empty(256 << 20, dtype=torch.uint8, device=dev)

    def run(rf, np_):
        ix.set_rerank_factor(rf)
        ix.search_batch_device(dq.data_ptr(), nq, K, d_ids.data_ptr(), d_sc.data_ptr(), np_, 1.0, 8.0, True,
                               stream.cuda_stream)

    def search(rf, np_, q=None):
        for _ in range(4):
            run(rf, np_)
            # collective on a sharded handle: every rank sees the same sum, so all retry together
            if not ix.device_flags(stream.cuda_stream):
                break
        return d_ids.cpu().numpy().view(np.uint64)

    if args.rf and args.nprobe:
        rf, np_ = args.rf, args.nprobe
        rec = recall(search(rf, np_), truth)
    else:
        rf, np_, rec = operating_point(search, truth)
    search(rf, np_)  # grows the candidate buffers if this point overflows them
    for _ in range(max(args.warmup, 3)):
        flush.zero_()
        run(rf, np_)
    torch.cuda.synchronize(dev)
    evs = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(args.steps)]
    # every rank runs the same number of profiled steps (they hold collectives)
    shares, dom_kernel, kernel_ms_per_step, kms_step = kernel_profile(ix, lambda: run(rf, np_), min(args.steps, 10),
                                                                      flush, dev)
    if dom_kernel == "nccl_all_gather":  # the roofline's kernel is one of this library's
        dom_kernel = max(((k, v) for k, v in kms_step.items() if k != "nccl_all_gather"), key=lambda kv: kv[1])[0]
    ix.kernel_clock(True, only=dom_kernel)
    ix.kernel_times(reset=True)
    if ws > 1:
        tdist.barrier()
    torch.cuda.synchronize(dev)
    with ClockSampler(local) as clk:
        clk.wait_first()
        torch.cuda.profiler.start()  # a profiler started with --profile-from-start off sees the timed steps
        for s in range(args.steps):
            flush.zero_()
            evs[s][0].record(stream)
            run(rf, np_)
            evs[s][1].record(stream)
        torch.cuda.synchronize(dev)
        torch.cuda.profiler.stop()
        clk.stop_mark()
    overflow = ix.device_flags(stream.cuda_stream)
    ktimes = ix.kernel_times(reset=True)
    ix.kernel_clock(False)
    stats = ix.last_search_stats()
    dom_ms = ktimes.get(dom_kernel, (0.0, 0))
    got_ids = d_ids.cpu().numpy().view(np.uint64).copy()
    got_sc = d_sc.cpu().numpy().copy()
    if ws > 1:
        tdist.barrier()
    total_ms = float(sum(a.elapsed_time(b) for a, b in evs))
    q_pin_owner, q_pin = pinned_queries(Q)
    e2e = []
    for _ in range(args.steps):
        flush.zero_()
        torch.cuda.synchronize(dev)
        t = time.perf_counter()
        ix.search_batch_arrays(q_pin, K, np_, 1.0, 8.0, True)
        e2e.append(time.perf_counter() - t)
    e2e_total = float(sum(e2e))
    # every rank's own step time and kernel times (the line's step time is the slowest rank's)
    mine = {"ms_per_step": round(total_ms / args.steps, 4),
            "kernel_ms_per_step": round(sum(kms_step.values()), 4),
            "top": {k: round(v, 4) for k, v in sorted(kms_step.items(), key=lambda kv: -kv[1])[:6]}}
    by_rank = [mine]
    if ws > 1:
        by_rank = [None] * ws
        tdist.all_gather_object(by_rank, mine)
        t = torch.tensor([total_ms, e2e_total], dtype=torch.float64)
        tdist.all_reduce(t, op=tdist.ReduceOp.MAX)
        total_ms, e2e_total = float(t[0]), float(t[1])
    parity = None
    sample = min(args.parity_sample, nq)
    if rank == 0 and sample > 0:
        rid, rsc = sharded_oracle_answers(args, rf, np_, sample, dev)
        parity = bool(np.array_equal(got_ids[:sample * K], rid) and
                      np.array_equal(got_sc[:sample * K].view(np.uint32), rsc.view(np.uint32)))
    if ws > 1:
        tdist.barrier()
    replicated = ("k_encode", "k_seed_finish", "k_local_list", "k_final_cm", "k_merge_topk", "k_topk")
    tot_ms = max(sum(kms_step.values()), 1e-9)
    out = {
        "metric": METRIC, "value": round(nq * args.steps / (total_ms / 1e3), 1), "unit": "queries/s",
        "n_gpus": ws, "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(total_ms / args.steps, 4),
        "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "u8", "data": "synthetic",
        "config": {"workload": "BASELINE configs[3]: 5.2M x 384 Gaussian mixture (10,000 comps, sigma 0.35), "
                               "quality preset, 10,000-query cell-major batches, k=10, cells sharded by range",
                   "n": n, "dim": 384, "nq_per_step": nq, "k": K, "rerank_factor": rf, "nprobe": np_,
                   "recall_at_10": round(rec, 4), "cells": int(ix.stats()["n_cells"]),
                   "rank0_cells": [lo, hi], "parallelism": f"cell-range shards x{ws} (NCCL all-gathers)",
                   "l2_flush": "256 MiB write before each step, outside its timing",
                   "build_s": round(build_s, 1), "overflow_flags": overflow},
        "e2e": {"value": round(nq * args.steps / e2e_total, 1), "unit": "queries/s",
                "h2d_bytes_per_step": nq * 384 * 4, "d2h_bytes_per_step": nq * K * 12},
        "clocks": clk.summary(),
        "kernel_share_rank0": shares,
        "kernel_share_src": f"separate pass of {min(args.steps, 10)} steps with every kernel timed: "
                            f"{kernel_ms_per_step} ms of kernel time per step on rank 0",
        "dominant_kernel_rank0": {"name": dom_kernel, "ms_per_launch": round(dom_ms[0] / max(dom_ms[1], 1), 4),
                                  "launches": dom_ms[1]},
        "ms_per_step_rank0": {k: round(v, 4) for k, v in sorted(kms_step.items(), key=lambda kv: -kv[1])},
        "collective_ms_per_step_rank0": round(kms_step.get("nccl_all_gather", 0.0), 4),
        "replicated_share_rank0": round(sum(kms_step.get(k, 0.0) for k in replicated) / tot_ms, 4),
        "replicated_src": "kernels whose work is per query on every rank (not divided by N): " + ", ".join(replicated),
        "parity": parity,
        "parity_src": f"ids and f32 scores of the first {sample} queries of the timed batch bit-identical to the "
                      "oracle's own build and cell-major search of the same vectors (rank 0)",
        "work_rank0": {k: round(v, 1) for k, v in stats.items()},
        "by_rank": by_rank,
    }
    if rank == 0:
        print(json.dumps(out), flush=True)
    if ws > 1:
        ix.shard(0, 1)
        tdist.barrier()
        tdist.destroy_process_group()


def run_lowbatch(args):
    """500k x 384 `memory` preset, batches of 1 and 16 on the per-query path
    (no cell-major batching), p50/p99 latency and QPS at R@10 >= 0.99 (or the best point)."""
    import torch

    import oracle

    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    X, Q, _ = mixture(args.seed, args.n, args.nq, 384, 1000, 0.35)
    threads = os.cpu_count() or 1
    t0 = time.perf_counter()
    ix = build_memory(X, threads, build_device=0)
    build_s = time.perf_counter() - t0
    ix.to_device(0)
    truth = brute_force_topk(X, Q, K, str(dev))

    def search(rf, np_, q=Q):
        ix.set_rerank_factor(rf)
        ids, _ = ix.search_batch_arrays(q, K, np_, 1.0, 8.0, False)
        return ids

    # the memory preset's SQ8 rerank can top out below 0.99 (it does on the reference's own corpus,
    # docs/RESULTS.md:49); then the point is the cheapest one within 0.002 of the best reachable recall
    best = recall(search(RF_GRID[-1], NP_GRID[-1]), truth)
    target = min(TARGET_RECALL, best - 0.002)
    rf, np_, rec = operating_point(search, truth, target)
    ix.set_rerank_factor(rf)
    stream = torch.cuda.Stream(dev)
    torch.cuda.set_stream(stream)
    out = {"metric": "p50/p99 latency and QPS at R@10=0.99, batch 1 and 16 (memory preset)",
           "unit": "ms", "higher_is_better": False, "n_gpus": 1, "dtype": "u8", "data": "synthetic",
           "config": {"workload": "BASELINE configs[2]: 500k x 384 Gaussian mixture (1000 comps, sigma 0.35), "
                                  "memory preset (per-dimension SQ8 rerank), per-query path", "n": args.n,
                      "rerank_factor": rf, "nprobe": np_, "recall_at_10": round(rec, 4),
                      "best_reachable_recall_at_10": round(best, 4), "recall_target": round(target, 4),
                      "build_s": round(build_s, 1)}}
    calls = max(args.steps, 50)
    for b in (1, 16):
        # end to end through the host API (queries in, ids/scores out, one synchronisation)
        lat = []
        for i in range(args.warmup + calls):
            q = Q[(i * b) % (args.nq - b + 1):][:b]
            t = time.perf_counter()
            ix.search_batch_arrays(q, K, np_, 1.0, 8.0, False)
            if i >= args.warmup:
                lat.append((time.perf_counter() - t) * 1e3)
        # device-resident: CUDA events around each call on the search stream
        dq = torch.from_numpy(Q[:b].copy()).to(dev)
        d_ids = torch.empty(b * K, dtype=torch.int64, device=dev)
        d_sc = torch.empty(b * K, dtype=torch.float32, device=dev)
        dl = []
        for i in range(args.warmup + calls):
            if i == args.warmup:
                torch.cuda.profiler.start()  # a profiler started with --profile-from-start off sees these calls
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record(stream)
            ix.search_batch_device(dq.data_ptr(), b, K, d_ids.data_ptr(), d_sc.data_ptr(), np_, 1.0, 8.0, False,
                                   stream.cuda_stream)
            e1.record(stream)
            e1.synchronize()
            if i >= args.warmup:
                dl.append(e0.elapsed_time(e1))
        torch.cuda.profiler.stop()
        # per-kernel device time in a separate pass (its events would lengthen the calls above)
        ix.kernel_clock(True)
        ix.kernel_times(reset=True)
        for i in range(calls):
            ix.search_batch_device(dq.data_ptr(), b, K, d_ids.data_ptr(), d_sc.data_ptr(), np_, 1.0, 8.0, False,
                                   stream.cuda_stream)
        torch.cuda.synchronize(dev)
        kt = ix.kernel_times(reset=True)
        ix.kernel_clock(False)
        lat, dl = np.asarray(lat), np.asarray(dl)
        out[f"batch{b}"] = {"e2e_p50_ms": round(float(np.percentile(lat, 50)), 4),
                            "e2e_p99_ms": round(float(np.percentile(lat, 99)), 4),
                            "e2e_qps": round(b / (float(lat.mean()) / 1e3), 1),
                            "device_p50_ms": round(float(np.percentile(dl, 50)), 4),
                            "device_p99_ms": round(float(np.percentile(dl, 99)), 4), "calls": calls,
                            "kernel_us_per_call": {k: round(v[0] * 1e3 / calls, 2) for k, v in kt.items() if v[1]}}
    # the reference's single-thread latency (fairbench.py:61-67) on the oracle port, over the
    # oracle's own build of the same vectors
    o = oracle.build_preset(X, "memory", rf, threads=threads).index()
    cl = []
    for i in range(min(calls, 200)):
        t = time.perf_counter()
        o.search_batch(Q[i:i + 1], K, np_, 1.0, 8.0, False, threads=1)
        cl.append((time.perf_counter() - t) * 1e3)
    out["cpu_baseline"] = {"value": round(float(np.percentile(cl, 50)), 4), "unit": "ms (p50, batch 1)", "cores": 1,
                           "kind": "port", "sample": f"{len(cl)} single-query calls, one thread"}
    out["value"] = out["batch1"]["e2e_p50_ms"]
    print(json.dumps(out), flush=True)


def run_concurrent(args):
    """ConcurrentIndex (src/concurrent.rs) on the config-2 vectors: 500k x 384 inserted in batches of
    50k with seal_at 100k (five sealed segments), 1% of them deleted (tombstones), then 20k more
    into the head. One step = one search_batch of 1,000 queries through the public API with host
    buffers (every segment and the head searched on the GPU, merged there): end-to-end QPS, at the
    smallest nprobe on the grid whose R@10 against brute force over the live vectors is >= 0.99."""
    import torch

    import maivs_b200 as M
    import oracle

    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    n_new = 20_000
    X, Q, _ = mixture(args.seed, args.n + n_new, args.nq, 384, 1000, 0.35)
    base, extra = X[:args.n], X[args.n:]
    rf = args.rf or 32
    seal_at = 100_000
    batch = 50_000
    dead = np.arange(0, args.n, 100, dtype=np.uint64)
    ncells = max(16, args.n // 128)

    def drive(cx):
        cx.train_centroids(base, ncells)
        for lo in range(0, args.n, batch):
            cx.add_batch(np.arange(lo, min(lo + batch, args.n), dtype=np.uint64),
                         np.ascontiguousarray(base[lo:lo + batch]))
        cx.remove_many(dead)
        cx.add_batch(np.arange(args.n, args.n + n_new, dtype=np.uint64), np.ascontiguousarray(extra))

    t0 = time.perf_counter()
    cx = M.ConcurrentIndex(384, "binary", rf, 0x5EED, 0, seal_at)
    cx.set_build_device(0)
    drive(cx)
    build_s = time.perf_counter() - t0
    cx.to_device(0)
    live = np.ones(X.shape[0], bool)
    live[dead.astype(np.int64)] = False
    live_ids = np.nonzero(live)[0]
    truth = live_ids[brute_force_topk(X[live_ids], Q, K, str(dev))]

    def search(np_):
        ids, _ = cx.search_batch_arrays(Q, K, np_, 1.0, 8.0)
        return ids

    np_, rec = NP_GRID[-1], 0.0
    for p in NP_GRID:
        r = recall(search(p), truth)
        np_, rec = p, r
        if r >= TARGET_RECALL:
            break
    for _ in range(max(args.warmup, 3)):
        search(np_)
    steps = max(args.steps, 10)
    ts = []
    torch.cuda.profiler.start()  # a profiler started with --profile-from-start off sees the timed steps
    for _ in range(steps):
        t = time.perf_counter()
        search(np_)
        ts.append(time.perf_counter() - t)
    torch.cuda.profiler.stop()
    mean_s = float(np.mean(ts))
    cx.kernel_clock(True)
    cx.kernel_times(reset=True)
    for _ in range(5):
        search(np_)
    kt = cx.kernel_times(reset=True)
    cx.kernel_clock(False)
    tot = max(sum(v[0] for v in kt.values()), 1e-9)
    shares = {k: round(v[0] / tot, 4) for k, v in kt.items() if v[1]}
    # the reference's path restated (the oracle's ConcurrentIndex over its own builds of the same
    # calls), on every host core, over a bounded sample; and parity of that sample
    threads = os.cpu_count() or 1
    oracle.lib().oracle_set_threads(threads)
    ox = oracle.OracleConcurrentIndex(384, "binary", rf, 0x5EED, 0, seal_at)
    drive(ox)
    sample = np.ascontiguousarray(Q[:args.parity_sample or 200])
    ref_ids, ref_sc = ox.search_batch(sample, K, np_, 1.0, 8.0)
    got_ids, got_sc = cx.search_batch_arrays(sample, K, np_, 1.0, 8.0)
    parity = bool(np.array_equal(got_ids, ref_ids) and np.array_equal(got_sc.view(np.uint32), ref_sc.view(np.uint32)))
    ct = []
    t0 = time.perf_counter()
    while time.perf_counter() - t0 < 12.0 or not ct:
        t = time.perf_counter()
        ox.search_batch(sample, K, np_, 1.0, 8.0)
        ct.append(time.perf_counter() - t)
    qps = args.nq / mean_s
    out = {"metric": "ConcurrentIndex batch QPS at R@10=0.99 (d=384), 5 sealed segments + head, 1% tombstones",
           "value": round(qps, 1), "unit": "queries/s", "n_gpus": 1, "steps": steps, "warmup": max(args.warmup, 3),
           "ms_per_step": round(mean_s * 1e3, 4), "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
           "dtype": "u64", "data": "synthetic",
           "e2e": {"value": round(qps, 1), "unit": "queries/s", "h2d_bytes_per_step": int(Q.nbytes),
                   "d2h_bytes_per_step": int(args.nq * K * 12)},
           "config": {"workload": "ConcurrentIndex over BASELINE configs[1]'s vectors (500k x 384 Gaussian mixture, "
                                  "1000 comps, sigma 0.35) + 20k inserted after 1% deletes; reference defaults "
                                  "(tree routing, no adaptive), Hamming scan per query per segment",
                      "n": args.n + n_new, "segments": cx.n_segments(), "head_live": int(cx.stats()["head_live"]),
                      "tombstones": int(dead.size), "rerank_factor": rf, "nprobe": np_,
                      "recall_at_10": round(rec, 4), "build_s": round(build_s, 1), "timing": "host clock around "
                      "each search_batch call (host buffers in and out; the call synchronises)"},
           "kernel_shares": shares, "gpu_launches": int(sum(v[1] for v in kt.values()) / 5),
           "parity": {"sample": int(sample.shape[0]), "ids_and_scores_equal": parity},
           "cpu_baseline": {"value": round(sample.shape[0] / float(np.mean(ct)), 1), "unit": "queries/s",
                            "cores": threads, "kind": "port",
                            "sample": f"{sample.shape[0]} queries per call through the oracle's ConcurrentIndex "
                                      f"(search_one per segment on {threads} threads, then finish); "
                                      f"mean of {len(ct)} calls"}}
    print(json.dumps(out), flush=True)


def run_filtered(args):
    """BASELINE configs[4] scaled to one GPU: d = 768 unit vectors from a seeded mixture (one
    component per 1,000 vectors, sigma 0.3), the `memory` preset with 768-bit codes (96 B) and
    per-dimension SQ8 rows, 10,000-query batches, k = 100, uniform tags in [0, 1000) and a filter
    tag < t at 1% and 10% selectivity (bench/fair/filtered.py of the reference draws them the same
    way). A filter turns the cell-major join off (index.rs:3343-3348), so every search is the
    per-query path with the tag checked in the scan. Per selectivity: the smallest nprobe on the
    grid whose R@100 against the exact top 100 of the vectors that pass is >= 0.9, its
    device-resident and end-to-end batch QPS, and the ids and scores of a sample against the oracle
    over the same index."""
    import torch

    import maivs_b200 as M
    import oracle

    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    n, nq, k, rf = args.n, args.nq, 100, args.rf or 4
    X, Q, _ = mixture(args.seed, n, nq, 768, max(n // 1000, 16), 0.3)
    threads = os.cpu_count() or 1
    t0 = time.perf_counter()
    ix = M.FlatCellIndex(768, "binary", rf, 0x5EED, 768)
    ix.set_per_dim_sq(True)
    ix.set_orthogonal_polysemy(2, 1.0)
    ix.set_fastscan(True)
    ix.set_two_stage(True, 2)
    ix.set_graph_route(False, 10**9)
    ix.set_tree_route(True, 2048, 16)
    ix.set_adaptive(True, 0.02)
    ix.set_build_device(0)
    ix.train_centroids(X, n // 128)
    ix.add_batch(np.arange(n, dtype=np.uint64), X)
    ix.compact()
    build_s = time.perf_counter() - t0
    tags = np.random.default_rng(2).integers(0, 1000, n).astype(np.uint32)
    ix.set_tags(np.arange(n, dtype=np.uint64), tags)
    ix.to_device(0)
    cells = int(ix.stats()["n_cells"])
    stream = torch.cuda.Stream(dev)
    dq = torch.from_numpy(Q).to(dev)
    d_ids = torch.empty(nq * k, dtype=torch.int64, device=dev)
    d_sc = torch.empty(nq * k, dtype=torch.float32, device=dev)
    xt = torch.from_numpy(X).to(dev)
    qt = torch.from_numpy(Q).to(dev)
    out = {"metric": "filtered batch QPS at R@100>=0.9, d=768 memory preset, k=100, 1% and 10% selectivity",
           "unit": "queries/s", "higher_is_better": True, "n_gpus": 1, "steps": args.steps,
           "warmup": max(args.warmup, 3), "scaling": "weak", "vs_baseline": None, "dtype": "u8",
           "data": "synthetic",
           "config": {"workload": f"BASELINE configs[4] scaled to {n:,} x 768 on one GPU (mixture of {max(n // 1000, 16)} "
                                  "components, sigma 0.3), memory preset with 768-bit codes, 10,000-query batches, "
                                  "k=100, uniform tags in [0,1000), filter tag < t; per-query path", "n": n,
                      "nq_per_step": nq, "k": k, "rerank_factor": rf, "cells": cells, "build_s": round(build_s, 1)}}
    per = {}
    for sel, t in (("1%", 10), ("10%", 100)):
        ix.set_filter(0, t - 1)
        sub = np.nonzero(tags < t)[0]
        st = torch.from_numpy(sub.astype(np.int64)).to(dev)
        xs = xt[st]
        truth = []
        for i in range(0, nq, 1024):
            truth.append(st[torch.topk(qt[i:i + 1024] @ xs.T, k, dim=1).indices].cpu().numpy())
        del xs
        truth = np.concatenate(truth)

        def run(np_):
            ix.search_batch_device(dq.data_ptr(), nq, k, d_ids.data_ptr(), d_sc.data_ptr(), np_, 1.0, 8.0, True,
                                   stream.cuda_stream)
            torch.cuda.synchronize(dev)

        def rec100():
            got = d_ids.cpu().numpy().view(np.uint64).reshape(nq, k).astype(np.int64)
            return float(np.mean([len(set(a) & set(b)) / k for a, b in zip(got.tolist(), truth.tolist())]))

        # the smallest nprobe at which a rerank factor on the grid reaches the target, with the
        # smallest such factor (the reference's filtered bench sweeps rf 16 and 32 the same way);
        # else the best point seen
        np_sel, rf_sel, r_sel, sweep = None, rf, -1.0, []
        done = False
        for np_ in (64, 128, 256, 512, 1024, 2048):
            if np_ > cells or done:
                break
            for rf_ in (rf, 16):
                ix.set_rerank_factor(rf_)
                run(np_)
                r = rec100()
                sweep.append({"nprobe": np_, "rf": rf_, "recall_at_100": round(r, 4)})
                if r >= 0.9 or (r > r_sel and not done):
                    np_sel, rf_sel, r_sel = np_, rf_, r
                if r >= 0.9:
                    done = True
                    break
        ix.set_rerank_factor(rf_sel)
        for _ in range(max(args.warmup, 3)):
            run(np_sel)
        ms = []
        torch.cuda.profiler.start()
        for _ in range(args.steps):
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record(stream)
            ix.search_batch_device(dq.data_ptr(), nq, k, d_ids.data_ptr(), d_sc.data_ptr(), np_sel, 1.0, 8.0, True,
                                   stream.cuda_stream)
            e1.record(stream)
            e1.synchronize()
            ms.append(e0.elapsed_time(e1))
        torch.cuda.profiler.stop()
        flags = ix.device_flags(stream.cuda_stream)
        e2e = []
        for _ in range(max(args.steps // 2, 2)):
            t1 = time.perf_counter()
            ids_h, sc_h = ix.search_batch_arrays(Q, k, np_sel, 1.0, 8.0, True)
            e2e.append(time.perf_counter() - t1)
        sample = np.ascontiguousarray(Q[:200])
        o = oracle.OracleIndex.from_index(ix)
        oracle.lib().oracle_set_threads(threads)
        t1 = time.perf_counter()
        ref_ids, ref_sc, *_ = o.search_batch(sample, k, np_sel, 1.0, 8.0, True, threads=threads)
        cpu_s = time.perf_counter() - t1
        del o
        parity = bool(np.array_equal(ids_h[:200 * k], ref_ids)
                      and np.array_equal(sc_h[:200 * k].view(np.uint32), ref_sc.view(np.uint32)))
        per[sel] = {"nprobe": np_sel, "rerank_factor": rf_sel, "recall_at_100": round(r_sel, 4), "sweep": sweep,
                    "value": round(nq / (float(np.mean(ms)) / 1e3), 1), "ms_per_step": round(float(np.mean(ms)), 3),
                    "e2e_qps": round(nq / float(np.mean(e2e)), 1), "overflow_flags": int(flags),
                    "parity": {"sample": 200, "ids_and_scores_equal": parity},
                    "cpu_baseline": {"value": round(200 / cpu_s, 1), "unit": "queries/s", "cores": threads,
                                     "kind": "port", "sample": f"200 queries, one call, nprobe {np_sel}, the oracle "
                                                               "over the same index's arrays"}}
        ix.set_filter()
        ix.set_rerank_factor(rf)
    out["selectivity"] = per
    out["value"] = per["10%"]["value"]
    out["ms_per_step"] = per["10%"]["ms_per_step"]
    out["e2e"] = {"value": per["10%"]["e2e_qps"], "unit": "queries/s", "h2d_bytes_per_step": int(Q.nbytes),
                  "d2h_bytes_per_step": int(nq * k * 12)}
    out["cpu_baseline"] = per["10%"]["cpu_baseline"]
    print(json.dumps(out), flush=True)


def run_reference(args):
    """The reference's CPU path (the oracle: a C++ restatement of the reference's Rust build and
    query path; the reference itself cannot be built here) on every host core. The index is the
    oracle's own build; nothing of the product is loaded. Each step is one full cell-major batch
    of the same queries at the same operating point as the GPU arm."""
    ws, rank, local = dist_env()
    if rank != 0:
        return
    X, Q, Qs = mixture(args.seed, args.n, args.nq, 384, 1000, 0.35)
    threads = os.cpu_count() or 1
    t0 = time.perf_counter()
    o = oracle_index(X, RF_GRID[0], threads)
    build_s = time.perf_counter() - t0
    truth = brute_force_topk(X, Q, K, "cpu")

    def search(rf, np_, q=Q):
        o.set_rerank_factor(rf)
        ids, *_ = o.search_batch(q, K, np_, 1.0, 8.0, True, threads=threads)
        return ids

    rf, np_, rec = operating_point(search, truth)
    mean_s, best_s, steps = time_cpu_batches(o, Q, rf, np_, threads, steps=args.steps, warmup=args.warmup)
    qps = args.nq / mean_s
    desc = (f"the full batch of {args.nq} IND queries per step, cell-major, (rf={rf}, nprobe={np_}), "
            f"mean of {steps} steps")
    print(json.dumps({
        "metric": METRIC, "impl": "reference", "value": round(qps, 1), "unit": "queries/s", "n_gpus": ws,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(mean_s * 1e3, 3),
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "u8", "data": "synthetic",
        "config": {"workload": "BASELINE configs[1]: 500k x 384 Gaussian mixture (1000 comps, sigma 0.35), quality "
                               "preset, cell-major batches of 1000 queries, k=10",
                   "n": args.n, "dim": 384, "nq_per_step": args.nq, "k": K, "rerank_factor": rf, "nprobe": np_,
                   "recall_at_10": round(rec, 4), "build_s": round(build_s, 1),
                   "index": "the oracle's own build (restated reference build), no product code"},
        "best_step_qps": round(args.nq / best_s, 1),
        "cpu_baseline": {"value": round(qps, 1), "unit": "queries/s", "cores": threads, "kind": "port",
                         "sample": desc},
        "e2e": {"value": round(qps, 1), "unit": "queries/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }), flush=True)


def run_reference_sharded(args):
    """The reference's CPU path on the sharded workload's data (5.2M x 384,
    10,000-query batches): the oracle's own build of the same vectors, cell-major search on every
    host core, on rank 0 only (the reference is one process; there is nothing to shard on a CPU).
    The operating point follows the same rule as the GPU arm. A step is the full batch, or a prefix
    of it when K full batches would not end within a few minutes (then the line says so)."""
    ws, rank, local = dist_env()
    if rank != 0:
        return
    import torch

    import oracle

    dev = torch.device("cuda", local)
    torch.cuda.set_device(dev)
    threads = os.cpu_count() or 1
    X, Q = mixture_torch(args.seed, args.n, args.nq, 384, 10_000, 0.35, dev)
    Q, truth = sharded_queries(args, X, Q, dev)
    t0 = time.perf_counter()
    o = oracle.build_preset(X, "quality", RF_GRID[0], threads=threads).take_index()
    build_s = time.perf_counter() - t0
    del X

    def search(rf, np_, q=Q):
        o.set_rerank_factor(rf)
        ids, *_ = o.search_batch(q, K, np_, 1.0, 8.0, True, threads=threads)
        return ids

    if args.rf and args.nprobe:
        rf, np_ = args.rf, args.nprobe
        rec = recall(search(rf, np_), truth)
    else:
        rf, np_, rec = operating_point(search, truth)
    o.set_rerank_factor(rf)
    t = time.perf_counter()
    o.search_batch(Q, K, np_, 1.0, 8.0, True, threads=threads)
    full_s = time.perf_counter() - t
    budget = 150.0
    nq_s = args.nq if full_s * args.steps <= budget else max(1000, int(args.nq * budget / (full_s * args.steps)))
    Qs = np.ascontiguousarray(Q[:nq_s])
    mean_s, best_s, steps = time_cpu_batches(o, Qs, rf, np_, threads, steps=args.steps, warmup=args.warmup)
    qps = nq_s / mean_s
    desc = (f"{nq_s} of the {args.nq} queries per step (cell-major, rf={rf}, nprobe={np_}), mean of {steps} "
            f"steps; the full batch takes {full_s:.2f} s on these cores")
    print(json.dumps({
        "metric": METRIC, "impl": "reference", "value": round(qps, 1), "unit": "queries/s", "n_gpus": ws,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(mean_s * 1e3, 3),
        "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "u8", "data": "synthetic",
        "config": {"workload": "BASELINE configs[3]: 5.2M x 384 Gaussian mixture (10,000 comps, sigma 0.35), quality "
                               "preset, 10,000-query cell-major batches, k=10 (one process on the host cores)",
                   "n": args.n, "dim": 384, "nq_per_step": nq_s, "k": K, "rerank_factor": rf, "nprobe": np_,
                   "recall_at_10": round(rec, 4), "build_s": round(build_s, 1),
                   "index": "the oracle's own build (restated reference build), no product code"},
        "cpu_baseline": {"value": round(qps, 1), "unit": "queries/s", "cores": threads, "kind": "port",
                         "sample": desc},
        "e2e": {"value": round(qps, 1), "unit": "queries/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }), flush=True)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=400)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=("maivs", "reference"), default="maivs")
    ap.add_argument("--vectors", "--n", dest="n", type=int, default=None,
                    help="vectors (500,000; 5,200,000 for --workload sharded)")
    ap.add_argument("--batch", "--nq", dest="nq", type=int, default=None,
                    help="queries per batch (1,000; 10,000 sharded)")
    ap.add_argument("--seed", type=int, default=2024)
    ap.add_argument("--rf", type=int, default=0, help="sharded workload: fixed rerank factor (with --nprobe)")
    ap.add_argument("--nprobe", type=int, default=0, help="sharded workload: fixed nprobe instead of the sweep")
    ap.add_argument("--no-sweep", action="store_true", help="config2: skip the (rf, nprobe) recall sweep")
    ap.add_argument("--workload", choices=("auto", "config2", "sharded", "lowbatch", "concurrent", "filtered"),
                    default="auto",
                    help="auto: sharded under torchrun (WORLD_SIZE set), else config2. config2: the headline 500k "
                         "batch on one GPU (replicas when forced under torchrun); sharded: configs[3], 5.2M vectors "
                         "with cells sharded by range over the N GPUs; lowbatch: configs[2], memory preset at "
                         "batch 1 and 16; concurrent: a ConcurrentIndex (sealed segments + head + tombstones) over "
                         "the config2 vectors; filtered: configs[4] scaled to one GPU (d=768 memory preset, k=100, "
                         "1% and 10% tag filters)")
    ap.add_argument("--parity-sample", type=int, default=1000,
                    help="sharded: queries of the timed batch checked against the oracle (0: none)")
    args = ap.parse_args()
    if args.workload == "auto":
        args.workload = "sharded" if "WORLD_SIZE" in os.environ else "config2"
    sharded = args.workload == "sharded"
    if args.n is None:
        args.n = 5_200_000 if sharded else 1_000_000 if args.workload == "filtered" else 500_000
    if args.nq is None:
        args.nq = 10_000 if sharded or args.workload == "filtered" else 1000
    if args.impl == "reference":
        run_reference_sharded(args) if sharded else run_reference(args)
    elif sharded:
        run_sharded(args)
    elif args.workload == "lowbatch":
        run_lowbatch(args)
    elif args.workload == "concurrent":
        run_concurrent(args)
    elif args.workload == "filtered":
        run_filtered(args)
    else:
        run_maivs(args)


if __name__ == "__main__":
    main()
