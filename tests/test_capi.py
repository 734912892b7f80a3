"""The C ABI: the shared library loads, exports every function include/maivs_b200.h declares,
and the Python binding declares a signature for each. No compute call needs a GPU here."""
from __future__ import annotations

import ctypes
import os
import re
import subprocess

import numpy as np
import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
HEADER = os.path.join(ROOT, "include", "maivs_b200.h")


def declared() -> list[str]:
    src = open(HEADER).read()
    src = re.sub(r"/\*.*?\*/", "", src, flags=re.S)
    return sorted(set(re.findall(r"\b(maivs_\w+)\s*\(", src)))


def test_header_declares_the_api():
    names = declared()
    for must in ("maivs_index_new", "maivs_search_batch", "maivs_search", "maivs_add_batch", "maivs_compact",
                 "maivs_search_batch_device", "maivs_profile_read"):
        assert must in names


def test_library_exports_every_declared_symbol():
    from maivs_b200 import _lib

    # RTLD_NOW: every undefined reference inside the library must resolve at load time
    L = ctypes.CDLL(_lib.LIB_PATH, mode=os.RTLD_NOW | os.RTLD_LOCAL)
    missing = [n for n in declared() if not hasattr(L, n)]
    assert not missing, missing
    out = subprocess.run(["nm", "-D", "--defined-only", _lib.LIB_PATH], capture_output=True, text=True).stdout
    exported = set(re.findall(r"\s[TW]\s+(maivs_\w+)$", out, flags=re.M))
    assert set(declared()) <= exported


def test_python_binding_covers_the_header():
    from maivs_b200 import _lib

    assert set(declared()) <= set(_lib.exported_symbols())
    _lib.lib()  # every signature resolves


def test_status_strings_and_errors_without_a_gpu():
    from maivs_b200 import _lib

    L = _lib.lib()
    assert L.maivs_status_string(0) == b"ok"
    assert L.maivs_status_string(9) == b"no CUDA device"
    h = ctypes.c_void_p()
    assert L.maivs_index_new(16, b"bogus", 4, 1, 0, ctypes.byref(h)) == _lib.BAD_ARG
    assert b"scan_mode must be" in L.maivs_last_error(h)
    L.maivs_index_free(h)


def test_search_without_device_fails_loudly():
    from conftest import has_gpu

    if has_gpu():
        pytest.skip("a GPU is present")
    import maivs_b200 as M

    rng = np.random.default_rng(0)
    X = rng.standard_normal((600, 64)).astype(np.float32)
    X /= np.linalg.norm(X, axis=1, keepdims=True)
    ix = M.FlatCellIndex(64, "binary", 4, 0x5EED, 0)
    ix.set_fastscan(True)
    ix.train_centroids(X, 4)
    ix.add_batch(list(range(600)), X)
    ix.compact()
    with pytest.raises(M.MaivsError, match="no CUDA device"):
        ix.search_batch(X[:40], 10, 4, 1.0, 8.0)
    # an empty index still answers with padding, as the reference does (index.rs:3337-3339)
    e = M.FlatCellIndex(64, "binary", 4, 0x5EED, 0)
    ids, sc = e.search_batch(X[:2], 3)
    assert ids == [2**64 - 1] * 6 and all(s == float("-inf") for s in sc)
    assert e.search(X[0], 3) == ([], [])


def test_profile_names_match_the_reference():
    import maivs_b200 as M

    names = [n for n, _ in M.profile_read(True)]
    for n in ("q.route", "q.scan", "q.rerank", "q.count", "b.compact"):  # src/prof.rs:35-42
        assert n in names


def test_set_num_threads():
    import maivs_b200 as M

    M.set_num_threads(2)
    with pytest.raises(ValueError):
        M.set_num_threads(0)
    M.set_num_threads(os.cpu_count() or 1)
