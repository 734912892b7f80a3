"""TEST INFRASTRUCTURE ONLY: Python binding of the parity oracle (maivs_oracle.cpp).

The oracle restates the reference's CPU query path (Rust, V47VANSH/MAIVS src/quantize.rs,
src/tree.rs, src/index.rs) in C++ with the reference's AVX2 arithmetic. It reads an index's
arrays through `FlatCellIndex.array()` and recomputes search results from them. Only tests/,
__graft_entry__.smoke() and the CPU-baseline arm of bench.py import this package; the product
(maivs_b200) never does.

Parity pinning: the reference has no golden vectors for this path and cannot be built in this
environment (no Rust toolchain), so value-level parity is unpinned by the reference itself; the
oracle is checked against published splitmix64 outputs, the reference's property tests
(quantize.rs:445-492) and its invariant suite (tests/test_index.py), see tests/test_oracle.py.
"""
from __future__ import annotations

import ctypes as C
import os
import subprocess

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
LIB = os.path.join(HERE, "libmaivs_oracle.so")
SRC = os.path.join(HERE, "maivs_oracle.cpp")

_lib = None


def build(force: bool = False) -> str:
    """Compile the oracle with the committed recipe (oracle/Makefile)."""
    if force or not os.path.exists(LIB) or os.path.getmtime(SRC) > os.path.getmtime(LIB):
        r = subprocess.run(["make", "-C", HERE, "-B" if force else "libmaivs_oracle.so"], capture_output=True,
                           text=True)
        if r.returncode != 0:
            raise RuntimeError(f"oracle build failed:\n{r.stdout}\n{r.stderr}")
    return LIB


class _Arrays(C.Structure):
    _fields_ = [
        ("dim", C.c_uint64), ("dim_pad", C.c_uint64), ("nw", C.c_uint64), ("M", C.c_uint64), ("ma", C.c_uint64),
        ("n_slots", C.c_uint64),
        ("signs", C.c_void_p), ("centroids", C.c_void_p), ("r_bound", C.c_void_p), ("cell_members", C.c_void_p),
        ("cell_member_off", C.c_void_p), ("fs_codes", C.c_void_p), ("n_fs_codes", C.c_uint64),
        ("fs_off", C.c_void_p), ("slot_cells", C.c_void_p), ("ext_ids", C.c_void_p), ("cent_bits", C.c_void_p),
        ("n_cent_bits", C.c_uint64), ("cent_sq8", C.c_void_p), ("n_cent_sq8", C.c_uint64), ("csq_min", C.c_void_p),
        ("csq_step", C.c_void_p), ("vecs_f32", C.c_void_p), ("n_vecs_f32", C.c_uint64), ("scan_i8", C.c_void_p),
        ("n_scan_i8", C.c_uint64), ("sq_min", C.c_void_p), ("sq_step", C.c_void_p), ("tags", C.c_void_p),
        ("n_tags", C.c_uint64),
        ("tree_depth", C.c_uint64), ("tree_level_n", C.c_void_p), ("tree_codes", C.c_void_p),
        ("tree_code_off", C.c_void_p), ("tree_child_start", C.c_void_p), ("tree_child_len", C.c_void_p),
        ("tree_child_off", C.c_void_p), ("tree_leaf_codes", C.c_void_p), ("tree_leaf_ids", C.c_void_p),
        ("config", C.c_void_p), ("n_config", C.c_uint64), ("bits", C.c_void_p), ("n_bits", C.c_uint64),
    ]


def lib() -> C.CDLL:
    global _lib
    if _lib is None:
        build()
        L = C.CDLL(LIB)
        vp, u64, f32 = C.c_void_p, C.c_uint64, C.c_float
        L.oracle_index_new.restype = vp
        L.oracle_index_new.argtypes = [C.POINTER(_Arrays)]
        L.oracle_index_free.argtypes = [vp]
        L.oracle_set_threads.argtypes = [C.c_int]
        L.oracle_index_set_rerank_factor.argtypes = [vp, u64]
        L.oracle_search_batch.restype = C.c_int
        L.oracle_search_batch.argtypes = [vp, vp, u64, u64, u64, f32, f32, C.c_int, vp, vp, vp, u64, vp, vp]
        L.oracle_route.restype = C.c_int
        L.oracle_route.argtypes = [vp, vp, u64, u64, f32, f32, C.c_int, vp, vp, vp]
        L.oracle_make_signs.argtypes = [u64, u64, vp]
        L.oracle_splitmix64.argtypes = [u64, u64, vp]
        L.oracle_fht.argtypes = [vp, u64]
        L.oracle_rotate.argtypes = [vp, u64, vp, u64, vp]
        L.oracle_pack_signs_trunc.argtypes = [vp, u64, vp, u64]
        L.oracle_encode.argtypes = [vp, u64, u64, vp, u64, u64, vp]
        L.oracle_fsquery.argtypes = [vp, u64, u64, vp, vp, vp]
        L.oracle_fs_block_sums.argtypes = [vp, vp, u64, C.c_int, vp]
        L.oracle_fs_pack_block.argtypes = [vp, u64, u64, vp]
        L.oracle_dot_f32.restype = f32
        L.oracle_dot_f32.argtypes = [vp, vp, u64]
        L.oracle_dot_f32_u8.restype = f32
        L.oracle_dot_f32_u8.argtypes = [vp, vp, u64]
        L.oracle_hamming_cutoff.restype = u64
        L.oracle_hamming_cutoff.argtypes = [vp, u64, u64, u64]
        L.oracle_keep_smallest.restype = u64
        L.oracle_keep_smallest.argtypes = [vp, vp, u64, u64, u64, vp]
        L.oracle_build_new.restype = vp
        L.oracle_build_new.argtypes = [u64, u64, u64, u64]
        L.oracle_build_free.argtypes = [vp]
        L.oracle_build_set.restype = C.c_int
        L.oracle_build_set.argtypes = [vp, C.c_char_p, C.c_double, C.c_double, C.c_double, C.c_double]
        L.oracle_build_train.restype = C.c_int
        L.oracle_build_train.argtypes = [vp, vp, u64, u64, u64, u64]
        L.oracle_build_add.restype = C.c_int
        L.oracle_build_add.argtypes = [vp, vp, vp, u64]
        L.oracle_build_compact.argtypes = [vp]
        L.oracle_build_take_index.restype = vp
        L.oracle_build_take_index.argtypes = [vp]
        L.oracle_build_snapshot.restype = vp
        L.oracle_build_snapshot.argtypes = [vp]
        L.oracle_build_remove.restype = C.c_int
        L.oracle_build_remove.argtypes = [vp, u64]
        L.oracle_build_has_id.restype = C.c_int
        L.oracle_build_has_id.argtypes = [vp, u64]
        L.oracle_build_n_live.restype = u64
        L.oracle_build_n_live.argtypes = [vp]
        L.oracle_build_fork.restype = vp
        L.oracle_build_fork.argtypes = [vp]
        L.oracle_build_export.argtypes = [vp]
        L.oracle_build_array.restype = C.c_int
        L.oracle_build_array.argtypes = [vp, C.c_char_p, C.POINTER(vp), C.POINTER(u64), C.POINTER(u64)]
        _lib = L
    return _lib


def _p(a: np.ndarray | None):
    if a is None or a.size == 0:
        return None
    return a.ctypes.data


class OracleIndex:
    """The reference's query path over a snapshot of a FlatCellIndex's arrays."""

    NAMES = ("signs", "centroids", "r_bound", "cell_members", "cell_member_off", "fs_codes", "fs_off", "slot_cells",
             "ext_ids", "cent_bits", "cent_sq8", "csq_min", "csq_step", "vecs_f32", "scan_i8", "sq_min", "sq_step",
             "tags", "tree_level_n", "tree_codes", "tree_code_off", "tree_child_start", "tree_child_len",
             "tree_child_off", "tree_leaf_codes", "tree_leaf_ids", "config", "bits")

    def __init__(self, arrays: dict):
        self.a = {k: np.ascontiguousarray(v) for k, v in arrays.items()}
        a = self.a
        cfg = a["config"]
        self.dim, self.dim_pad, self.nw = int(cfg[0]), int(cfg[1]), int(cfg[2])
        M = a["r_bound"].shape[0]
        ext = a["ext_ids"]
        ma = int(cfg[8])
        s = _Arrays()
        s.dim, s.dim_pad, s.nw, s.M, s.ma, s.n_slots = self.dim, self.dim_pad, self.nw, M, ma, ext.shape[0]
        for name in ("signs", "centroids", "r_bound", "cell_members", "cell_member_off", "fs_codes", "fs_off",
                     "slot_cells", "ext_ids", "cent_bits", "cent_sq8", "csq_min", "csq_step", "vecs_f32",
                     "scan_i8", "sq_min", "sq_step", "tags", "tree_level_n", "tree_codes", "tree_code_off",
                     "tree_child_start", "tree_child_len", "tree_child_off", "tree_leaf_codes", "tree_leaf_ids",
                     "config", "bits"):
            setattr(s, name, _p(a.get(name)))
        s.n_bits = a["bits"].size if "bits" in a else 0
        s.n_fs_codes = a["fs_codes"].size
        s.n_cent_bits = a["cent_bits"].size
        s.n_cent_sq8 = a["cent_sq8"].size
        s.n_vecs_f32 = a["vecs_f32"].size
        s.n_scan_i8 = a["scan_i8"].size
        s.n_tags = a["tags"].size
        s.tree_depth = a["tree_level_n"].size
        s.n_config = cfg.size
        self._s = s
        self.h = lib().oracle_index_new(C.byref(s))

    @classmethod
    def from_index(cls, ix) -> "OracleIndex":
        """Search the arrays of a product-built index (for stage-by-stage checks)."""
        return cls({n: ix.array(n) for n in cls.NAMES})

    @classmethod
    def from_build(cls, b: "OracleBuild") -> "OracleIndex":
        """Search an index the oracle built itself from the raw vectors (independent of the product)."""
        return cls({n: b.array(n) for n in cls.NAMES})

    def __del__(self):
        if getattr(self, "h", None):
            lib().oracle_index_free(self.h)
            self.h = None

    def set_rerank_factor(self, rf: int) -> None:
        lib().oracle_index_set_rerank_factor(self.h, int(rf))

    def search_batch(self, Q: np.ndarray, k: int, nprobe: int = 16, tc: float = 0.95, beta: float = 8.0,
                     cell_major: bool = True, cand_cap: int = 0, threads: int | None = None):
        """Returns (ids[nq*k], scores[nq*k], cands[nq, cand_cap] or None, cand_n or None, used_cm)."""
        Q = np.ascontiguousarray(Q, dtype=np.float32)
        nq = Q.shape[0]
        if threads is not None:
            lib().oracle_set_threads(int(threads))
        ids = np.empty(nq * k, np.uint64)
        sc = np.empty(nq * k, np.float32)
        cands = np.empty((nq, cand_cap), np.uint32) if cand_cap else None
        cand_n = np.empty(nq, np.uint32) if cand_cap else None
        used = C.c_int(0)
        rc = lib().oracle_search_batch(self.h, Q.ctypes.data, nq, k, nprobe, tc, beta, int(cell_major), ids.ctypes.data,
                                       sc.ctypes.data, _p(cands), cand_cap, _p(cand_n), C.byref(used))
        if rc != 0:
            raise RuntimeError(f"oracle_search_batch failed with {rc}")
        return ids, sc, cands, cand_n, bool(used.value)

    def route(self, Q: np.ndarray, nprobe: int, tc: float = 1.0, beta: float = 8.0, batch_router: bool = True):
        Q = np.ascontiguousarray(Q, dtype=np.float32)
        nq = Q.shape[0]
        chosen = np.empty((nq, nprobe), np.uint32)
        cscore = np.empty((nq, nprobe), np.float32)
        nch = np.empty(nq, np.uint32)
        rc = lib().oracle_route(self.h, Q.ctypes.data, nq, nprobe, tc, beta, int(batch_router), chosen.ctypes.data,
                                cscore.ctypes.data, nch.ctypes.data)
        if rc != 0:
            raise RuntimeError(f"oracle_route failed with {rc}")
        return chosen, cscore, nch


# ---- component helpers -------------------------------------------------------------------------

def splitmix64(seed: int, n: int) -> np.ndarray:
    out = np.empty(n, np.uint64)
    lib().oracle_splitmix64(seed, n, out.ctypes.data)
    return out


def make_signs(dim_pad: int, seed: int) -> np.ndarray:
    out = np.empty(2 * dim_pad, np.float32)
    lib().oracle_make_signs(dim_pad, seed, out.ctypes.data)
    return out


def fht(a: np.ndarray) -> np.ndarray:
    a = np.ascontiguousarray(a, dtype=np.float32).copy()
    lib().oracle_fht(a.ctypes.data, a.size)
    return a


def rotate(v: np.ndarray, signs: np.ndarray, dim_pad: int) -> np.ndarray:
    v = np.ascontiguousarray(v, dtype=np.float32)
    out = np.empty(dim_pad, np.float32)
    lib().oracle_rotate(v.ctypes.data, v.size, np.ascontiguousarray(signs).ctypes.data, dim_pad, out.ctypes.data)
    return out


def encode(V: np.ndarray, signs: np.ndarray, dim_pad: int, nw: int) -> np.ndarray:
    V = np.ascontiguousarray(V, dtype=np.float32)
    out = np.empty((V.shape[0], nw), np.uint64)
    lib().oracle_encode(V.ctypes.data, V.shape[0], V.shape[1], np.ascontiguousarray(signs).ctypes.data, dim_pad, nw,
                        out.ctypes.data)
    return out


def fsquery(rot: np.ndarray, nw: int):
    rot = np.ascontiguousarray(rot, dtype=np.float32)
    lut = np.empty(nw * 16 * 16, np.uint8)
    d, b = C.c_float(), C.c_float()
    lib().oracle_fsquery(rot.ctypes.data, rot.size, nw, lut.ctypes.data, C.byref(d), C.byref(b))
    return lut, d.value, b.value


def fs_block_sums(block: np.ndarray, lut: np.ndarray, nw: int, avx2: bool = True) -> np.ndarray:
    out = np.empty(32, np.uint16)
    lib().oracle_fs_block_sums(np.ascontiguousarray(block).ctypes.data, np.ascontiguousarray(lut).ctypes.data, nw,
                               int(avx2), out.ctypes.data)
    return out


def fs_pack_block(codes: np.ndarray, nw: int) -> np.ndarray:
    codes = np.ascontiguousarray(codes, dtype=np.uint64)
    out = np.empty(nw * 64 * 32 // 8, np.uint8)
    lib().oracle_fs_pack_block(codes.ctypes.data if codes.size else None, codes.shape[0], nw, out.ctypes.data)
    return out


def dot_f32(a, b) -> float:
    a = np.ascontiguousarray(a, np.float32)
    b = np.ascontiguousarray(b, np.float32)
    return float(lib().oracle_dot_f32(a.ctypes.data, b.ctypes.data, a.size))


def dot_f32_u8(a, b) -> float:
    a = np.ascontiguousarray(a, np.float32)
    b = np.ascontiguousarray(b, np.uint8)
    return float(lib().oracle_dot_f32_u8(a.ctypes.data, b.ctypes.data, a.size))


def hamming_cutoff(hs: np.ndarray, want: int, bits: int) -> int:
    hs = np.ascontiguousarray(hs, np.uint16)
    return int(lib().oracle_hamming_cutoff(hs.ctypes.data, hs.size, want, bits))


def keep_smallest(h: np.ndarray, ids: np.ndarray, keep: int, bits: int) -> np.ndarray:
    h = np.ascontiguousarray(h, np.uint32)
    ids = np.ascontiguousarray(ids, np.uint32)
    out = np.empty(max(h.size, 1), np.uint32)
    n = lib().oracle_keep_smallest(h.ctypes.data, ids.ctypes.data, h.size, keep, bits, out.ctypes.data)
    return out[:n]


# ---- the reference's index build, restated (independent of the product's host build) -----------

_ARRAY_DTYPES = {
    "vecs_f32": np.float32, "scan_i8": np.int8, "ext_ids": np.uint64, "slot_cell": np.uint32,
    "slot_cells": np.uint32, "cell_members": np.uint32, "cell_member_off": np.uint32, "centroids": np.float32,
    "r_bound": np.float32, "prim_len": np.uint32, "rep_off": np.uint32, "fs_codes": np.uint8, "fs_off": np.uint32,
    "cent_bits": np.uint64, "cent_sq8": np.uint8, "csq_min": np.float32, "csq_step": np.float32,
    "sq_min": np.float32, "sq_step": np.float32, "signs": np.float32, "tags": np.uint32,
    "tree_level_n": np.uint64, "tree_codes": np.uint64, "tree_code_off": np.uint64, "tree_child_start": np.uint64,
    "tree_child_len": np.uint64, "tree_child_off": np.uint64, "tree_leaf_codes": np.uint64,
    "tree_leaf_ids": np.uint32, "config": np.float64, "bits": np.uint64,
}


class OracleBuild:
    """FlatCellIndex's build path (train_centroids, add_batch, compact and the derived routing
    state) restated from the reference (index.rs:684-1112, :2442-2667, :2761-2804, :2987-3212;
    tree.rs:160-540). Method names and arguments follow the reference's pymethods, so a preset
    reads the same on either side. Only the binary scan mode is restated."""

    def __init__(self, dim: int, scan_mode: str = "binary", rerank_factor: int = 4, seed: int = 0x5EED,
                 code_bits: int = 0):
        if scan_mode != "binary":
            raise ValueError("the oracle restates the binary scan mode only")
        self.dim = int(dim)
        self.h = lib().oracle_build_new(self.dim, int(code_bits), int(seed), int(rerank_factor))
        self._exported = False

    def __del__(self):
        if getattr(self, "h", None):
            lib().oracle_build_free(self.h)
            self.h = None

    def _set(self, key: str, a=0.0, b=0.0, c=0.0, d=0.0):
        if lib().oracle_build_set(self.h, key.encode(), float(a), float(b), float(c), float(d)) != 0:
            raise ValueError(key)
        self._exported = False

    def set_two_stage(self, on: bool, mult: int) -> None:
        self._set("two_stage", on, mult)

    def set_tree_route(self, on: bool, min_cells: int = 0, fanout: int = 0, beam_frac: float = 0.0) -> None:
        self._set("tree_route", on, min_cells, fanout, beam_frac)

    def set_graph_route(self, on: bool, min_cells: int = 0) -> None:
        self._set("graph_route", on, min_cells)

    def set_orthogonal_polysemy(self, homes: int = 2, lam: float = 1.0) -> None:
        self._set("orthogonal_polysemy", homes, lam)

    def set_replication(self, max_assign: int, spill_margin: float) -> None:
        self._set("replication", max_assign, spill_margin)

    def set_fastscan(self, on: bool) -> None:
        self._set("fastscan", on)

    def set_per_dim_sq(self, on: bool) -> None:
        self._set("per_dim_sq", on)

    def set_i8_rerank(self, on: bool) -> None:
        self._set("i8_rerank", on)

    def set_adaptive(self, on: bool, margin: float) -> None:
        self._set("adaptive", on, margin)

    def set_centroid_sq8(self, on: bool) -> None:
        self._set("centroid_sq8", on)

    def set_rerank_factor(self, rf: int) -> None:
        self._set("rerank_factor", rf)

    def set_cell_major_min_batch(self, n: int) -> None:
        self._set("cm_min_batch", n)

    def train_centroids(self, vectors: np.ndarray, n_cells: int, sample: int = 262_144, seed: int = 0x5EED) -> None:
        X = np.ascontiguousarray(vectors, dtype=np.float32)
        if X.ndim != 2 or X.shape[1] != self.dim:
            raise ValueError("dim mismatch")
        if lib().oracle_build_train(self.h, X.ctypes.data, X.shape[0], int(n_cells), int(sample), int(seed)) != 0:
            raise ValueError("no training vectors")
        self._exported = False

    def add_batch(self, ids, vectors: np.ndarray) -> None:
        X = np.ascontiguousarray(vectors, dtype=np.float32)
        ids = np.ascontiguousarray(np.asarray(ids, dtype=np.uint64))
        if X.ndim != 2 or X.shape[1] != self.dim or ids.shape[0] != X.shape[0]:
            raise ValueError("shape mismatch")
        if lib().oracle_build_add(self.h, ids.ctypes.data, X.ctypes.data, X.shape[0]) != 0:
            raise ValueError("call train_centroids() before add_batch()")
        self._exported = False

    def compact(self) -> None:
        lib().oracle_build_compact(self.h)
        self._exported = False

    def array(self, name: str) -> np.ndarray:
        """A copy of one index array, under FlatCellIndex.array()'s name and layout."""
        if not self._exported:
            lib().oracle_build_export(self.h)
            self._exported = True
        p, n, e = C.c_void_p(), C.c_uint64(), C.c_uint64()
        if lib().oracle_build_array(self.h, name.encode(), C.byref(p), C.byref(n), C.byref(e)) != 0:
            raise KeyError(name)
        dt = np.dtype(_ARRAY_DTYPES[name])
        if n.value == 0:
            return np.empty(0, dt)
        buf = (C.c_uint8 * (n.value * e.value)).from_address(p.value)
        return np.frombuffer(buf, dtype=dt).copy()

    def index(self) -> "OracleIndex":
        return OracleIndex.from_build(self)

    def remove(self, id: int) -> bool:
        """remove (index.rs:3223-3276)."""
        self._exported = False
        return bool(lib().oracle_build_remove(self.h, int(id)))

    def has_id(self, id: int) -> bool:
        return bool(lib().oracle_build_has_id(self.h, int(id)))

    def n_live(self) -> int:
        return int(lib().oracle_build_n_live(self.h))

    def fork_empty(self) -> "OracleBuild":
        """fork_empty (index.rs:2330-2400): same configuration and centroids, no vectors,
        FastScan off."""
        f = OracleBuild.__new__(OracleBuild)
        f.dim = self.dim
        f.h = lib().oracle_build_fork(self.h)
        f._exported = False
        return f

    def snapshot(self) -> "OracleIndex":
        """A searchable copy of the index as it stands (the build stays usable)."""
        o = OracleIndex.__new__(OracleIndex)
        o.a = {}
        o.h = lib().oracle_build_snapshot(self.h)
        return o

    def take_index(self) -> "OracleIndex":
        """The searchable index, moving the build's large arrays into it (no copies; the build
        cannot export or be searched afterwards). For large builds."""
        o = OracleIndex.__new__(OracleIndex)
        o.a = {}
        o.h = lib().oracle_build_take_index(self.h)
        self._exported = False
        return o


def build_preset(X: np.ndarray, preset: str = "quality", rerank_factor: int = 16, ids=None,
                 threads: int | None = None, n_cells: int | None = None) -> OracleBuild:
    """The reference benchmark presets (bench/fair/fairbench.py:98-119) built by the oracle:
    `quality` = two homes (orthogonal polysemy), FastScan, two-stage routing, tree routing from
    2,048 cells with fanout 16, adaptive probing with margin 0.02, N/128 cells; `memory` adds the
    per-dimension SQ8 rerank store."""
    if threads is not None:
        lib().oracle_set_threads(int(threads))
    n, d = X.shape
    b = OracleBuild(d, "binary", rerank_factor, 0x5EED, 0)
    if preset == "memory":
        b.set_per_dim_sq(True)
    elif preset != "quality":
        raise ValueError(preset)
    b.set_orthogonal_polysemy(2, 1.0)
    b.set_fastscan(True)
    b.set_two_stage(True, 2)
    b.set_graph_route(False, 10**9)
    b.set_tree_route(True, 2048, 16)
    b.set_adaptive(True, 0.02)
    b.train_centroids(X, n_cells if n_cells is not None else max(16, n // 128))
    b.add_batch(np.arange(n, dtype=np.uint64) if ids is None else ids, X)
    b.compact()
    return b


class OracleConcurrentIndex:
    """ConcurrentIndex (src/concurrent.rs) restated over oracle builds: sealed segments, one mutable
    head, tombstones. Every search runs search_one on each segment and on the head (the per-query
    path, :113-131) with k over-fetched twice once tombstones exist (:50-52, :116-117), then
    finish (:83-110): tombstones dropped, the best score per id, the best k (exact ties by ascending
    id, the product's rule for the reference's unstable sort). Single-threaded: the locks of the
    reference order concurrent calls but do not change what one sequence of calls computes."""

    OVERFETCH = 2

    def __init__(self, dim: int, scan_mode: str = "binary", rerank_factor: int = 8, seed: int = 0x5EED,
                 code_bits: int = 0, seal_at: int = 1_000_000):
        self.dim = int(dim)
        self.head = OracleBuild(dim, scan_mode, rerank_factor, seed, code_bits)
        self.sealed: list[tuple[OracleBuild, OracleIndex]] = []
        self.dead: set[int] = set()
        self.sealed_live = 0
        self.seal_at = max(int(seal_at), 1)
        self.par_scan = False

    # seal_locked (:134-152)
    def _seal(self) -> None:
        if self.head.n_live() == 0:
            return
        self.head.compact()
        fresh = self.head.fork_empty()
        frozen, self.head = self.head, fresh
        self.sealed.append((frozen, frozen.snapshot()))
        self.sealed_live += frozen.n_live()

    def add_batch(self, ids, vectors) -> None:  # :247-261
        self.head.add_batch(ids, vectors)
        if self.head.n_live() >= self.seal_at:
            self._seal()

    def _known(self, id: int) -> bool:
        return self.head.has_id(id) or any(b.has_id(id) for b, _ in self.sealed)

    def remove(self, id: int) -> bool:  # :265-277
        id = int(id)
        if not self._known(id) or id in self.dead:
            return False
        self.dead.add(id)
        return True

    def remove_many(self, ids) -> int:  # :280-293
        return sum(self.remove(int(i)) for i in ids)

    def seal(self) -> None:
        self._seal()

    def purge_head(self) -> int:  # :304-314, victims in ascending id
        victims = sorted(i for i in self.dead if self.head.has_id(i))
        for i in victims:
            self.head.remove(i)
            self.dead.discard(i)
        self.head.compact()
        return len(victims)

    def compact(self) -> None:
        self.head.compact()

    def train_centroids(self, vectors, n_cells: int, sample: int = 262_144, seed: int = 0x5EED) -> None:
        self.head.train_centroids(vectors, n_cells, sample, seed)

    def set_per_dim_sq(self, on: bool) -> None:
        self.head.set_per_dim_sq(on)

    def set_two_stage(self, on: bool, mult: int) -> None:
        self.head.set_two_stage(on, mult)

    def set_adaptive(self, on: bool, margin: float) -> None:
        self.head.set_adaptive(on, margin)

    def set_parallel_scan(self, on: bool) -> None:
        self.par_scan = bool(on)

    def set_graph_route(self, on: bool, min_cells: int = 0) -> None:
        self.head.set_graph_route(on, min_cells)

    def set_tree_route(self, on: bool, min_cells: int = 0, fanout: int = 0, beam_frac: float = 0.0) -> None:
        self.head.set_tree_route(on, min_cells, fanout, beam_frac)

    def __len__(self) -> int:
        return max(self.sealed_live + self.head.n_live() - len(self.dead), 0)

    def search_batch(self, Q: np.ndarray, k: int, nprobe: int = 16, tc: float = 0.95, beta: float = 8.0):
        """ids (uint64, nq*k) and scores (float32, nq*k), padded with UINT64_MAX / -inf."""
        Q = np.ascontiguousarray(Q, dtype=np.float32)
        nq = Q.shape[0]
        want = k if not self.dead else k * self.OVERFETCH
        lists = [o.search_batch(Q, want, nprobe, tc, beta, cell_major=False)[:2] for _, o in self.sealed]
        lists.append(self.head.snapshot().search_batch(Q, want, nprobe, tc, beta, cell_major=False)[:2])
        ids = np.full(nq * k, np.iinfo(np.uint64).max, np.uint64)
        sc = np.full(nq * k, -np.inf, np.float32)
        pad = np.iinfo(np.uint64).max
        for qi in range(nq):
            best: dict[int, np.float32] = {}
            for li, ls in lists:
                for i, s in zip(li[qi * want:(qi + 1) * want].tolist(), ls[qi * want:(qi + 1) * want]):
                    if i == pad or i in self.dead:
                        continue
                    if i not in best or s > best[i]:
                        best[i] = s
            top = sorted(best.items(), key=lambda t: (-float(t[1]), t[0]))[:k]
            for r, (i, s) in enumerate(top):
                ids[qi * k + r] = i
                sc[qi * k + r] = s
        return ids, sc
