"""save / load in the reference's MAIVS2 format (index.rs:3594-3603, src/persist.rs).

The file layout is checked field by field against the format's definition (persist.rs:80-145), and
a loaded index must answer exactly like the one that was saved once it is compacted again (the
reference's own save/load test checks the same rows, tests/test_index.py).
"""
from __future__ import annotations

import struct

import numpy as np
import pytest

import maivs_b200 as M
import oracle
from datagen import build_index, mixture


@pytest.fixture(scope="module")
def saved(tmp_path_factory):
    rng = np.random.default_rng(9)
    X, c = mixture(rng, 8_000, 96, 60)
    Q, _ = mixture(rng, 40, 96, 60, centers=c)
    ix = build_index(X, "memory", rf=6, tree_min_cells=16)
    path = str(tmp_path_factory.mktemp("persist") / "ix.maivs")
    ix.save(path)
    return ix, Q, path


def _read_pod(buf, off, fmt_char, size):
    (n,) = struct.unpack_from("<Q", buf, off)
    off += 8
    arr = np.frombuffer(buf, dtype=np.dtype(fmt_char), count=n, offset=off)
    return arr, off + n * size


def test_file_layout(saved):
    ix, _, path = saved
    buf = open(path, "rb").read()
    assert buf[:8] == b"MAIVS2\x00\x01"
    hdr = struct.unpack_from("<16Q", buf, 8)
    cfg = ix.array("config")
    assert hdr[0] == 96 and hdr[1] == 2 and hdr[2] == 6  # dim, binary, rerank factor
    assert hdr[3] == int(cfg[1]) and hdr[4] == int(cfg[2])  # dim_pad, words
    assert hdr[5] == 0x5EED and hdr[6] == 8_000 and hdr[7] == 2
    quant_scale, spill, at_margin, beam = struct.unpack_from("<4f", buf, 8 + 128)
    assert abs(at_margin - 0.02) < 1e-7 and abs(beam - 0.5) < 1e-7
    off = 8 + 128 + 16
    bits, off = _read_pod(buf, off, "<u8", 8)
    assert np.array_equal(bits, ix.array("bits"))
    sq8, off = _read_pod(buf, off, "i1", 1)
    assert np.array_equal(sq8.view(np.int8), ix.array("scan_i8").view(np.int8))
    f16, off = _read_pod(buf, off, "<u2", 2)
    assert f16.size == 0
    sq_min, off = _read_pod(buf, off, "<f4", 4)
    assert np.array_equal(sq_min, ix.array("sq_min"))
    sq_step, off = _read_pod(buf, off, "<f4", 4)
    vecs, off = _read_pod(buf, off, "<f4", 4)
    assert np.array_equal(vecs, ix.array("vecs_f32"))
    ext, off = _read_pod(buf, off, "<u8", 8)
    assert np.array_equal(ext, ix.array("ext_ids"))
    slot_cell, off = _read_pod(buf, off, "<u4", 4)
    free, off = _read_pod(buf, off, "<u4", 4)
    slot_cells, off = _read_pod(buf, off, "<u4", 4)
    assert np.array_equal(slot_cells, ix.array("slot_cells"))
    tags, off = _read_pod(buf, off, "<u4", 4)
    (ncell,) = struct.unpack_from("<Q", buf, off)
    off += 8
    assert ncell == int(ix.stats()["n_cells"])
    members_total = 0
    for _ in range(ncell):
        mem, off = _read_pod(buf, off, "<u4", 4)
        members_total += mem.size
        _, off = _read_pod(buf, off, "<f4", 4)  # sum
        cen, off = _read_pod(buf, off, "<f4", 4)
        assert cen.size == 96
        off += 8  # r_bound, r_max
    assert off == len(buf)
    assert members_total == ix.array("cell_members").size


def test_loaded_index_answers_the_same(saved):
    ix, Q, path = saved
    ld = M.FlatCellIndex.load(path)
    assert ld.dim == 96 and ld.stats()["n_live"] == 8_000
    ld.set_fastscan(True)
    ld.compact()
    a = oracle.OracleIndex.from_index(ix)
    b = oracle.OracleIndex.from_index(ld)
    for cm in (True, False):
        ia, sa, *_ = a.search_batch(Q, 10, 16, 1.0, 8.0, cm)
        ib, sb, *_ = b.search_batch(Q, 10, 16, 1.0, 8.0, cm)
        assert np.array_equal(ia, ib) and np.array_equal(sa, sb)


def test_load_rejects_bad_files(tmp_path):
    p = tmp_path / "bad"
    p.write_bytes(b"NOTMAIVS" + b"\0" * 64)
    with pytest.raises(ValueError, match="magic"):
        M.FlatCellIndex.load(str(p))
    p.write_bytes(b"MAIVS2\x00\x01" + b"\0" * 10)
    with pytest.raises(ValueError, match="truncated"):
        M.FlatCellIndex.load(str(p))
    with pytest.raises(ValueError):
        M.FlatCellIndex.load(str(tmp_path / "missing"))


def test_loaded_index_has_the_saved_arrays(saved):
    """Load rebuilds the derived state (centroid codes, SQ8 centroids, radii, tree) as the reference
    does (persist.rs:279); after compact() every array the GPU reads equals the saved index's."""
    ix, _, path = saved
    ld = M.FlatCellIndex.load(path)
    ld.set_fastscan(True)
    ld.compact()
    for name in oracle.OracleIndex.NAMES:
        a, b = ix.array(name), ld.array(name)
        if name == "config":
            continue
        assert a.shape == b.shape and np.array_equal(a.view(np.uint8), b.view(np.uint8)), name
