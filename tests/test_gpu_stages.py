"""Stage-by-stage parity of the GPU pipeline with the oracle (bit-exact at every stage).

Stage 0: query sign codes (quantize.rs:57-67 after rotate :152-163) and FastScan tables with their
delta and bias (quantize.rs:279-313). Stage 1: probe lists and re-order scores (route_batch
index.rs:1873-1980 / route_query :1168-1305). Stage 2: the candidate slots sent to the exact
rerank (cell-major exact cut, index.rs:2277-2306; per-query bucket queue, :1630-1692).
"""
from __future__ import annotations

import numpy as np
import pytest

import oracle
from datagen import build_index, mixture

pytestmark = pytest.mark.gpu

CASES = {
    "d384_quality": dict(dim=384, n=30_000, preset="quality", code_bits=0, tree=64),
    "d768_memory": dict(dim=768, n=12_000, preset="memory", code_bits=0, tree=2048),
    "d384_bits256": dict(dim=384, n=20_000, preset="memory", code_bits=256, tree=2048),
    "d100_quality": dict(dim=100, n=8_000, preset="quality", code_bits=0, tree=2048),
}


def _build(case):
    c = CASES[case]
    rng = np.random.default_rng(c["dim"] + c["n"])
    X, centers = mixture(rng, c["n"], c["dim"], max(20, c["n"] // 100))
    Q, _ = mixture(rng, 80, c["dim"], max(20, c["n"] // 100), centers=centers)
    ix = build_index(X, c["preset"], rf=8, tree_min_cells=c["tree"], code_bits=c["code_bits"])
    return ix, Q


@pytest.fixture(scope="module", params=list(CASES))
def built(request):
    return _build(request.param)


def test_stage0_codes_and_tables(built):
    ix, Q = built
    cfg = ix.array("config")
    dim_pad, nw = int(cfg[1]), int(cfg[2])
    got = ix.debug_stage(0, Q, 10, 8, 1.0, 8.0, True)
    signs = ix.array("signs")
    assert np.array_equal(got["qbits"], oracle.encode(Q, signs, dim_pad, nw))
    for i in range(Q.shape[0]):
        rot = oracle.rotate(Q[i], signs, dim_pad)
        lut, delta, bias = oracle.fsquery(rot, nw)
        assert np.array_equal(got["lut"][i], lut), i
        assert np.float32(delta) == got["delta"][i] and np.float32(bias) == got["bias"][i], i


@pytest.mark.parametrize("nprobe", [1, 8, 40])
@pytest.mark.parametrize("cell_major", [True, False])
def test_stage1_probe_lists(built, nprobe, cell_major):
    ix, Q = built
    Qs = Q if cell_major else Q[:40]
    got = ix.debug_stage(1, Qs, 10, nprobe, 1.0, 8.0, cell_major)
    o = oracle.OracleIndex.from_index(ix)
    ch, cs, nch = o.route(Qs, nprobe, 1.0, 8.0, batch_router=cell_major)
    assert np.array_equal(got["nch"], nch)
    assert np.array_equal(got["chosen"], ch)
    assert np.array_equal(got["cscore"], cs)


@pytest.mark.parametrize("nprobe", [4, 8, 24])
@pytest.mark.parametrize("cell_major", [True, False])
def test_stage2_candidate_sets(built, nprobe, cell_major):
    ix, Q = built
    Qs = Q if cell_major else Q[:40]
    cap = 4096
    got = ix.debug_stage(2, Qs, 10, nprobe, 1.0, 8.0, cell_major, cand_cap=cap)
    o = oracle.OracleIndex.from_index(ix)
    _, _, cands, cand_n, used = o.search_batch(Qs, 10, nprobe, 1.0, 8.0, cell_major, cand_cap=cap)
    assert used == (cell_major and Qs.shape[0] >= 32)
    assert np.array_equal(got["cand_n"], cand_n)
    assert np.array_equal(got["cand"], cands)


@pytest.mark.parametrize("cell_major", [True, False])
def test_stage3_final_results(built, cell_major):
    ix, Q = built
    Qs = Q if cell_major else Q[:40]
    ids, sc = ix.search_batch_arrays(Qs, 10, 16, 1.0, 8.0, cell_major)
    o = oracle.OracleIndex.from_index(ix)
    rid, rsc, *_ = o.search_batch(Qs, 10, 16, 1.0, 8.0, cell_major)
    assert np.array_equal(ids, rid)
    assert np.array_equal(sc, rsc)
