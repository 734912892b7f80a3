"""bench.py's measurement helpers on the CPU: the matched-recall frontier and its
log-interpolation (the reference's bench/fair/summarise.py:26-45), and the scaling of a committed
ncu traffic figure to a run's own work counters."""
from __future__ import annotations

import math

import bench


def pts(*rq):
    return [{"recall": r, "qps": q} for r, q in rq]


def test_frontier_drops_dominated_points_and_sorts_by_recall():
    f = bench.frontier(pts((0.90, 100.0), (0.95, 80.0), (0.93, 70.0), (0.99, 50.0), (0.97, 90.0)))
    # (0.93, 70) is beaten by (0.95, 80) and (0.97, 90); (0.95, 80) by (0.97, 90)
    assert [(p["recall"], p["qps"]) for p in f] == [(0.90, 100.0), (0.97, 90.0), (0.99, 50.0)]


def test_interp_is_logarithmic_and_never_extrapolates():
    f = bench.frontier(pts((0.90, 400.0), (0.99, 100.0)))
    mid = bench.interp(f, 0.945)
    assert math.isclose(mid, 200.0, rel_tol=1e-6)  # halfway in recall = geometric mean in QPS
    assert bench.interp(f, 0.90) == 400.0 and bench.interp(f, 0.99) == 100.0
    assert bench.interp(f, 0.995) is None and bench.interp(f, 0.85) is None
    assert bench.interp(bench.frontier(pts((0.99, 100.0))), 0.99) == 100.0


def test_matched_reports_every_target():
    m = bench.matched(pts((0.94, 500.0), (0.985, 300.0), (0.996, 100.0)))
    assert set(m) == {"0.95", "0.98", "0.99", "0.995"}
    assert all(v is not None for v in m.values())
    assert m["0.95"] > m["0.98"] > m["0.99"] > m["0.995"]


def test_ncu_traffic_scales_with_the_work_counter():
    ent = bench.ncu_traffic("k_rerank", {"candidates": 0})
    assert ent is None  # no work, no figure
    a = bench.ncu_traffic("k_rerank", {"candidates": 215_128})
    b = bench.ncu_traffic("k_rerank", {"candidates": 430_256})
    assert a and b == 2 * a
    assert bench.ncu_traffic("no_such_kernel", {"candidates": 1}) is None
