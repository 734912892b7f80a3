"""B200-native MAIVS query engine: a drop-in for the reference's `maivs` Python module.

`FlatCellIndex` and `ConcurrentIndex` keep the reference's constructors, method names, defaults,
return types and errors (src/index.rs and src/concurrent.rs #[pymethods], src/lib.rs:32-39). The index is built on the host cores;
`search` / `search_batch` run on the GPU through hand-written sm_100a kernels behind the C ABI of
include/maivs_b200.h. There is no CPU search path: without a CUDA device, search raises.
"""
from __future__ import annotations

import ctypes as C
from typing import Optional

import numpy as np

from . import _lib

__all__ = ["FlatCellIndex", "ConcurrentIndex", "profile", "profile_read", "MaivsError", "nccl_unique_id",
           "shard_over_torch"]


class MaivsError(RuntimeError):
    """A failure reported by the engine (CUDA error, overflow, unsupported option)."""


def _ptr(a: np.ndarray) -> C.c_void_p:
    return C.c_void_p(a.ctypes.data)


def _as_f32_matrix(x, name: str, dim: int) -> np.ndarray:
    if not isinstance(x, np.ndarray) or x.dtype != np.float32:
        raise TypeError(f"{name} must be a float32 numpy array")
    if x.ndim != 2:
        raise ValueError(f"{name} must be 2-D")
    if x.shape[1] != dim:
        raise ValueError("query dim mismatch" if name == "queries" else "dim mismatch")
    if not x.flags["C_CONTIGUOUS"]:
        raise ValueError(f"{name} must be C-contiguous (use np.ascontiguousarray)")
    return x


class FlatCellIndex:
    """Partitioned vector index with fixed-size cells, 1-bit FastScan codes, orthogonal polysemy,
    cell-major batch search and exact rerank; queries run on the GPU.

    Only scan_mode="binary" is served (the reference's "f32"/"i8" modes are ablations that no
    preset uses). A compacted FastScan index is searched by FastScan table sums (per query or by
    the cell-major join); any other index (before compact(), after a remove(), FastScan off) by
    Hamming distance per query, as the reference does (the cell-major join then needs
    set_fastscan(True) and compact())."""

    def __init__(self, dim: int, scan_mode: str = "f32", rerank_factor: int = 4, seed: int = 0x5EED,
                 code_bits: int = 0):
        L = _lib.lib()
        h = C.c_void_p()
        rc = L.maivs_index_new(int(dim), scan_mode.encode(), int(rerank_factor), int(seed) & (2**64 - 1),
                               int(code_bits), C.byref(h))
        self._h = h
        self._dim = int(dim)
        if rc != _lib.OK:
            msg = L.maivs_last_error(h).decode() if h else "allocation failed"
            if h:
                L.maivs_index_free(h)
            self._h = None
            raise ValueError(msg)

    def __del__(self):
        h = getattr(self, "_h", None)
        if h:
            _lib.lib().maivs_index_free(h)
            self._h = None

    # ---- plumbing ----
    def _check(self, rc: int) -> None:
        if rc == _lib.OK:
            return
        L = _lib.lib()
        msg = L.maivs_last_error(self._h).decode()
        if rc in (_lib.BAD_SHAPE, _lib.BAD_ARG, _lib.BAD_STATE):
            raise ValueError(msg)
        raise MaivsError(f"{L.maivs_status_string(rc).decode()}: {msg}")

    @property
    def dim(self) -> int:
        return self._dim

    # ---- build (host cores) ----
    def train_centroids(self, vectors: np.ndarray, n_cells: int, sample: int = 262_144, seed: int = 0x5EED) -> None:
        v = _as_f32_matrix(vectors, "vectors", self._dim)
        self._check(_lib.lib().maivs_train_centroids(self._h, _ptr(v), v.shape[0], int(n_cells), int(sample),
                                                     int(seed) & (2**64 - 1)))

    def set_centroids(self, centroids: np.ndarray) -> None:
        c = np.asarray(centroids)
        if c.ndim != 2 or c.shape[1] != self._dim:
            raise ValueError("centroid dim mismatch")
        c = np.ascontiguousarray(c, dtype=np.float32)
        self._check(_lib.lib().maivs_set_centroids(self._h, _ptr(c), c.shape[0]))

    def add_batch(self, ids, vectors: np.ndarray) -> None:
        ids_a = np.ascontiguousarray(np.asarray(list(ids) if not isinstance(ids, np.ndarray) else ids,
                                                dtype=np.uint64))
        v = np.asarray(vectors)
        if v.ndim != 2 or v.shape[0] != ids_a.shape[0] or v.shape[1] != self._dim:
            raise ValueError("shape mismatch")
        if v.dtype != np.float32:
            raise TypeError("vectors must be a float32 numpy array")
        if not v.flags["C_CONTIGUOUS"]:
            raise ValueError("vectors must be C-contiguous (use np.ascontiguousarray)")
        self._check(_lib.lib().maivs_add_batch(self._h, _ptr(ids_a), _ptr(v), ids_a.shape[0]))

    def remove(self, id: int) -> bool:
        r = C.c_int(0)
        self._check(_lib.lib().maivs_remove(self._h, int(id), C.byref(r)))
        return bool(r.value)

    def compact(self) -> None:
        self._check(_lib.lib().maivs_compact(self._h))

    # ---- configuration (index.rs:2823-2984, :3520-3558) ----
    def set_rerank_factor(self, rf: int) -> None:
        self._check(_lib.lib().maivs_set_rerank_factor(self._h, int(rf)))

    def set_two_stage(self, on: bool, mult: int) -> None:
        self._check(_lib.lib().maivs_set_two_stage(self._h, int(bool(on)), int(mult)))

    def set_tree_route(self, on: bool, min_cells: int = 0, fanout: int = 0, beam_frac: float = 0.0) -> None:
        self._check(_lib.lib().maivs_set_tree_route(self._h, int(bool(on)), int(min_cells), int(fanout),
                                                    float(beam_frac)))

    def set_graph_route(self, on: bool, min_cells: int = 0) -> None:
        self._check(_lib.lib().maivs_set_graph_route(self._h, int(bool(on)), int(min_cells)))

    def set_adaptive(self, on: bool, margin: float) -> None:
        self._check(_lib.lib().maivs_set_adaptive(self._h, int(bool(on)), float(margin)))

    def set_fastscan(self, on: bool) -> None:
        self._check(_lib.lib().maivs_set_fastscan(self._h, int(bool(on))))

    def set_orthogonal_polysemy(self, homes: int = 2, lam: float = 1.0) -> None:
        self._check(_lib.lib().maivs_set_orthogonal_polysemy(self._h, int(homes), float(lam)))

    def set_replication(self, max_assign: int, spill_margin: float) -> None:
        self._check(_lib.lib().maivs_set_replication(self._h, int(max_assign), float(spill_margin)))

    def set_per_dim_sq(self, on: bool) -> None:
        self._check(_lib.lib().maivs_set_per_dim_sq(self._h, int(bool(on))))

    def set_i8_rerank(self, on: bool) -> None:
        self._check(_lib.lib().maivs_set_i8_rerank(self._h, int(bool(on))))

    def set_centroid_sq8(self, on: bool) -> None:
        self._check(_lib.lib().maivs_set_centroid_sq8(self._h, int(bool(on))))

    def set_tags(self, ids, tags) -> None:
        ids_a = np.ascontiguousarray(np.asarray(ids, dtype=np.uint64))
        tg = np.ascontiguousarray(np.asarray(tags, dtype=np.uint32))
        if ids_a.shape != tg.shape:
            raise ValueError("ids/tags length mismatch")
        self._check(_lib.lib().maivs_set_tags(self._h, _ptr(ids_a), _ptr(tg), ids_a.shape[0]))

    def set_filter(self, lo: Optional[int] = None, hi: Optional[int] = None) -> None:
        if lo is None and hi is None:
            self._check(_lib.lib().maivs_set_filter(self._h, 0, 0, 0))
        else:
            self._check(_lib.lib().maivs_set_filter(self._h, 1, 0 if lo is None else int(lo),
                                                    0xFFFFFFFF if hi is None else int(hi)))

    def set_cell_major_min_batch(self, n: int) -> None:
        """Smallest batch that takes the cell-major join (reference: 2 x its thread count)."""
        self._check(_lib.lib().maivs_set_cell_major_min_batch(self._h, int(n)))

    def set_build_device(self, device: int | None) -> None:
        """Run the build's k-means and vector placement on CUDA device `device` (None: the host
        cores). The index built is the same either way, array for array."""
        self._check(_lib.lib().maivs_set_build_device(self._h, -1 if device is None else int(device)))

    def to_device(self, device: int = 0) -> None:
        """Build the device image now on CUDA device `device` (search does it on first use)."""
        self._check(_lib.lib().maivs_to_device(self._h, int(device)))

    # ---- search (GPU) ----
    def search(self, query: np.ndarray, k: int, nprobe: int = 16, target_confidence: float = 0.95,
               beta: float = 8.0):
        q = np.ascontiguousarray(np.asarray(query, dtype=np.float32).reshape(-1))
        if q.shape[0] != self._dim:
            raise ValueError("query dim mismatch")
        ids = np.empty(max(int(k), 1), dtype=np.uint64)
        sc = np.empty(max(int(k), 1), dtype=np.float32)
        n = C.c_size_t(0)
        self._check(_lib.lib().maivs_search(self._h, _ptr(q), int(k), int(nprobe), float(target_confidence),
                                            float(beta), _ptr(ids), _ptr(sc), C.byref(n)))
        m = n.value
        return [int(x) for x in ids[:m]], [float(x) for x in sc[:m]]

    def search_batch_arrays(self, queries: np.ndarray, k: int, nprobe: int = 16, target_confidence: float = 0.95,
                            beta: float = 8.0, cell_major: bool = True):
        """search_batch returning numpy arrays (ids uint64 [nq*k], scores float32 [nq*k])."""
        Q = _as_f32_matrix(queries, "queries", self._dim)
        nq = Q.shape[0]
        ids = np.empty(nq * int(k), dtype=np.uint64)
        sc = np.empty(nq * int(k), dtype=np.float32)
        self._check(_lib.lib().maivs_search_batch(self._h, _ptr(Q), nq, int(k), int(nprobe),
                                                  float(target_confidence), float(beta), int(bool(cell_major)),
                                                  _ptr(ids), _ptr(sc)))
        return ids, sc

    def search_batch(self, queries: np.ndarray, k: int, nprobe: int = 16, target_confidence: float = 0.95,
                     beta: float = 8.0, cell_major: bool = True):
        ids, sc = self.search_batch_arrays(queries, k, nprobe, target_confidence, beta, cell_major)
        return ids.tolist(), sc.tolist()

    def search_batch_device(self, d_queries: int, nq: int, k: int, d_ids: int, d_scores: int, nprobe: int = 16,
                            target_confidence: float = 0.95, beta: float = 8.0, cell_major: bool = True,
                            stream: int = 0) -> None:
        """Enqueue a search on device pointers (e.g. torch tensors' data_ptr()) on `stream`."""
        self._check(_lib.lib().maivs_search_batch_device(
            self._h, C.c_void_p(d_queries), int(nq), int(k), int(nprobe), float(target_confidence), float(beta),
            int(bool(cell_major)), C.c_void_p(d_ids), C.c_void_p(d_scores), C.c_void_p(stream or None)))

    # ---- persistence (index.rs:3594-3603) ----
    def save(self, path: str) -> None:
        """Write the index in the reference's on-disk format (MAIVS2, src/persist.rs)."""
        self._check(_lib.lib().maivs_save(self._h, str(path).encode()))

    @staticmethod
    def load(path: str) -> "FlatCellIndex":
        """Load an index written by save() here or by the reference. Like the reference, the loaded
        index is not compacted and has FastScan off, so it is searched per query by Hamming
        distance; set_fastscan(True) and compact() give it the FastScan scan and the cell-major
        join."""
        L = _lib.lib()
        h = C.c_void_p()
        rc = L.maivs_load(str(path).encode(), C.byref(h))
        if rc != _lib.OK:
            msg = L.maivs_last_error(h).decode() if h else "load failed"
            if h:
                L.maivs_index_free(h)
            raise ValueError(msg)
        ix = FlatCellIndex.__new__(FlatCellIndex)
        ix._h = h
        cfg = ix.array("config")
        ix._dim = int(cfg[0])
        return ix

    # ---- cell-range sharding (one rank per GPU; no counterpart in the reference) ----
    def shard(self, rank: int, world: int, nccl_id: bytes = b"") -> None:
        """Make this handle rank `rank` of `world` cell-range shards (collective over the ranks).

        Every later search runs the sharded cell-major join with NCCL all-gathers, so all ranks
        must issue the same searches with the same queries; results equal the unsharded join's.
        `nccl_id` is rank 0's nccl_unique_id(), shared by the host. world=1 unshards."""
        buf = (C.c_uint8 * 128).from_buffer_copy(nccl_id.ljust(128, b"\0")[:128]) if nccl_id else None
        self._check(_lib.lib().maivs_shard(self._h, int(rank), int(world), buf, 128 if nccl_id else 0))

    def shard_range(self, rank: int, world: int) -> tuple[int, int]:
        """Cells [lo, hi) that rank `rank` of `world` scans (balanced by member entries)."""
        lo, hi = C.c_uint32(0), C.c_uint32(0)
        self._check(_lib.lib().maivs_shard_range(self._h, int(rank), int(world), C.byref(lo), C.byref(hi)))
        return int(lo.value), int(hi.value)

    def search_batch_sharded_emulated(self, world: int, d_queries: int, nq: int, k: int, d_ids: int,
                                      d_scores: int, nprobe: int = 16, target_confidence: float = 0.95,
                                      beta: float = 8.0, stream: int = 0) -> None:
        """The sharded protocol with `world` shards in this process on one GPU (device copies
        stand in for NCCL); device pointers in and out, enqueued on `stream`."""
        self._check(_lib.lib().maivs_search_batch_sharded_emulated(
            self._h, int(world), C.c_void_p(d_queries), int(nq), int(k), int(nprobe), float(target_confidence),
            float(beta), C.c_void_p(d_ids), C.c_void_p(d_scores), C.c_void_p(stream or None)))

    def device_flags(self, stream: int = 0) -> int:
        f = C.c_uint32(0)
        self._check(_lib.lib().maivs_device_flags(self._h, C.c_void_p(stream or None), C.byref(f)))
        return int(f.value)

    # ---- instrumentation ----
    def kernel_clock(self, on: bool, only: str | None = None) -> None:
        """Time every kernel of subsequent searches (or only the kernel named `only`) with CUDA
        events on their launch stream."""
        if on and only:
            self._check(_lib.lib().maivs_kernel_clock_only(self._h, only.encode()))
        else:
            self._check(_lib.lib().maivs_kernel_clock(self._h, int(bool(on))))

    def kernel_times(self, reset: bool = False) -> dict:
        """{kernel name: (total ms, launches)} accumulated while the clock was on."""
        n = 32
        names = (C.c_char_p * n)()
        ms = (C.c_double * n)()
        la = (C.c_uint64 * n)()
        got = C.c_size_t(0)
        self._check(_lib.lib().maivs_kernel_times(self._h, int(bool(reset)), names, ms, la, n, C.byref(got)))
        return {names[i].decode(): (float(ms[i]), int(la[i])) for i in range(got.value)}

    def kernel_busy(self) -> dict:
        """{kernel name: ms during which at least one of its launches ran} since the clock's last
        reset (read it before kernel_times(reset=True)); overlapping launches count once."""
        n = 32
        names = (C.c_char_p * n)()
        ms = (C.c_double * n)()
        got = C.c_size_t(0)
        self._check(_lib.lib().maivs_kernel_busy(self._h, names, ms, n, C.byref(got)))
        return {names[i].decode(): float(ms[i]) for i in range(got.value)}

    def last_search_stats(self) -> dict:
        """Work counters of the last search (probes, candidates, bytes scanned and reranked)."""
        cap = 64
        buf = C.create_string_buffer(4096)
        vals = (C.c_double * cap)()
        got = C.c_size_t(0)
        self._check(_lib.lib().maivs_last_search_stats(self._h, buf, 4096, vals, cap, C.byref(got)))
        names = buf.value.decode().split("\n")
        return {names[i]: float(vals[i]) for i in range(got.value)}

    def debug_stage(self, stage: int, queries: np.ndarray, k: int, nprobe: int = 16, target_confidence: float = 0.95,
                    beta: float = 8.0, cell_major: bool = True, cand_cap: int = 4096) -> dict:
        """Run one search only up to `stage` (0 codes/tables, 1 probe lists, 2 rerank candidates)."""
        Q = _as_f32_matrix(queries, "queries", self._dim)
        nq = Q.shape[0]
        cfg = self.array("config")
        nw = int(cfg[2])
        out = {}
        z = C.c_void_p(None)
        if stage == 0:
            out["qbits"] = np.zeros((nq, nw), np.uint64)
            out["lut"] = np.zeros((nq, nw * 256), np.uint8)
            out["delta"] = np.zeros(nq, np.float32)
            out["bias"] = np.zeros(nq, np.float32)
            args = [_ptr(out["qbits"]), _ptr(out["lut"]), _ptr(out["delta"]), _ptr(out["bias"]), z, z, z, z, 0, z]
        elif stage == 1:
            out["chosen"] = np.zeros((nq, nprobe), np.uint32)
            out["cscore"] = np.zeros((nq, nprobe), np.float32)
            out["nch"] = np.zeros(nq, np.uint32)
            args = [z, z, z, z, _ptr(out["chosen"]), _ptr(out["cscore"]), _ptr(out["nch"]), z, 0, z]
        else:
            out["cand"] = np.zeros((nq, cand_cap), np.uint32)
            out["cand_n"] = np.zeros(nq, np.uint32)
            args = [z, z, z, z, z, z, z, _ptr(out["cand"]), cand_cap, _ptr(out["cand_n"])]
        self._check(_lib.lib().maivs_debug_stage(self._h, int(stage), _ptr(Q), nq, int(k), int(nprobe),
                                                 float(target_confidence), float(beta), int(bool(cell_major)), *args))
        return out

    def debug_cellmajor(self, queries: np.ndarray, k: int, nprobe: int, target_confidence: float = 1.0,
                        beta: float = 8.0) -> dict:
        """Per-query internals of the cell-major join (seed survivors, tau, probe range, scan survivors)."""
        Q = _as_f32_matrix(queries, "queries", self._dim)
        nq = Q.shape[0]
        out = {n: np.zeros(nq, np.uint32) for n in ("seed_n", "tau", "rest_hi", "rest_n")}
        info = C.create_string_buffer(256)
        self._check(_lib.lib().maivs_debug_cellmajor(self._h, _ptr(Q), nq, int(k), int(nprobe),
                                                     float(target_confidence), float(beta), _ptr(out["seed_n"]),
                                                     _ptr(out["tau"]), _ptr(out["rest_hi"]), _ptr(out["rest_n"]),
                                                     info, 256))
        out["info"] = info.value.decode()
        return out

    # ---- introspection ----
    def __len__(self) -> int:
        n = C.c_size_t(0)
        self._check(_lib.lib().maivs_len(self._h, C.byref(n)))
        return n.value

    _STATS = ("n_live", "n_cells", "free_slots", "quant_scale", "scan_bytes_per_vec", "cell_size_mean",
              "cell_size_max", "cell_size_min", "max_assign", "centroid_graph_nodes", "tree_depth",
              "tree_top_width", "tree_fanout", "tree_beam_frac", "replication_factor", "member_entries",
              "total_bytes", "live_cells", "device_bytes", "build_device", "build_gpu_failures")

    def stats(self) -> dict:
        out = {}
        v = C.c_double(0.0)
        for name in self._STATS:
            self._check(_lib.lib().maivs_stat(self._h, name.encode(), C.byref(v)))
            out[name] = float(v.value)
        return out

    _DTYPES = {1: np.uint8, 4: None, 8: None}

    def array(self, name: str) -> np.ndarray:
        """Copy of an internal host array (see maivs_array in include/maivs_b200.h)."""
        p = C.c_void_p()
        n = C.c_size_t(0)
        eb = C.c_size_t(0)
        self._check(_lib.lib().maivs_array(self._h, name.encode(), C.byref(p), C.byref(n), C.byref(eb)))
        dt = np.dtype(_ARRAY_DTYPES.get(name))
        if n.value == 0 or not p.value:
            return np.zeros(0, dtype=dt)
        raw = np.ctypeslib.as_array(C.cast(p, C.POINTER(C.c_uint8)), shape=(n.value * eb.value,))
        return raw.view(dt).copy()


_ARRAY_DTYPES = {
    "vecs_f32": np.float32, "scan_i8": np.int8, "bits": np.uint64, "ext_ids": np.uint64, "slot_cell": np.uint32,
    "slot_cells": np.uint32, "cell_members": np.uint32, "cell_member_off": np.uint32, "centroids": np.float32,
    "r_bound": np.float32, "prim_len": np.uint32, "rep_off": np.uint32, "fs_codes": np.uint8, "fs_off": np.uint32,
    "cent_bits": np.uint64, "cent_sq8": np.uint8, "csq_min": np.float32, "csq_step": np.float32,
    "sq_min": np.float32, "sq_step": np.float32, "signs": np.float32, "tags": np.uint32, "tree_level_n": np.uint64,
    "tree_codes": np.uint64, "tree_code_off": np.uint64, "tree_child_start": np.uint64,
    "tree_child_len": np.uint64, "tree_child_off": np.uint64, "tree_leaf_codes": np.uint64,
    "tree_leaf_ids": np.uint32, "config": np.float64,
}

CONFIG_FIELDS = ("dim", "dim_pad", "nw", "rerank_factor", "two_stage", "shortlist_mult", "centroid_sq8", "has_tree",
                 "max_assign", "fastscan", "per_dim_sq", "i8_rerank", "keep_f32", "adaptive", "at_margin",
                 "quant_scale", "compacted", "n_live", "cm_min_batch", "has_filter", "filter_lo", "filter_hi",
                 "tree_beam_frac", "tree_n_leaf", "graph_route", "graph_min_cells")


class ConcurrentIndex:
    """Reads over immutable segments plus one mutable head (src/concurrent.rs): inserts go to the
    head, which is compacted and sealed into a segment at `seal_at` vectors; deletes are tombstones
    by id. Every search runs all segments and the head on the GPU (per query, Hamming scan) and
    merges them there (tombstones dropped, one entry per id, best k). Safe to call from several
    threads; a write blocks readers for one insert batch at most."""

    def __init__(self, dim: int, scan_mode: str = "binary", rerank_factor: int = 8, seed: int = 0x5EED,
                 code_bits: int = 0, seal_at: int = 1_000_000):
        L = _lib.lib()
        h = C.c_void_p()
        rc = L.maivs_concurrent_new(int(dim), scan_mode.encode(), int(rerank_factor), int(seed) & (2**64 - 1),
                                    int(code_bits), int(seal_at), C.byref(h))
        self._h = h
        self._dim = int(dim)
        if rc != _lib.OK:
            msg = L.maivs_concurrent_last_error(h).decode() if h else "allocation failed"
            if h:
                L.maivs_concurrent_free(h)
            self._h = None
            raise ValueError(msg)

    def __del__(self):
        h = getattr(self, "_h", None)
        if h:
            _lib.lib().maivs_concurrent_free(h)
            self._h = None

    def _check(self, rc: int) -> None:
        if rc == _lib.OK:
            return
        L = _lib.lib()
        msg = L.maivs_concurrent_last_error(self._h).decode()
        if rc in (_lib.BAD_SHAPE, _lib.BAD_ARG, _lib.BAD_STATE):
            raise ValueError(msg)
        raise MaivsError(f"{L.maivs_status_string(rc).decode()}: {msg}")

    @property
    def dim(self) -> int:
        return self._dim

    # ---- reads (GPU) ----
    def search(self, query: np.ndarray, k: int, nprobe: int = 16, target_confidence: float = 0.95,
               beta: float = 8.0):
        q = np.ascontiguousarray(np.asarray(query, dtype=np.float32).reshape(-1))
        if q.shape[0] != self._dim:
            raise ValueError("query dim mismatch")
        ids = np.empty(max(int(k), 1), dtype=np.uint64)
        sc = np.empty(max(int(k), 1), dtype=np.float32)
        n = C.c_size_t(0)
        self._check(_lib.lib().maivs_concurrent_search(self._h, _ptr(q), int(k), int(nprobe),
                                                       float(target_confidence), float(beta), _ptr(ids), _ptr(sc),
                                                       C.byref(n)))
        m = n.value
        return [int(x) for x in ids[:m]], [float(x) for x in sc[:m]]

    def search_batch_arrays(self, queries: np.ndarray, k: int, nprobe: int = 16, target_confidence: float = 0.95,
                            beta: float = 8.0):
        """search_batch returning numpy arrays (ids uint64 [nq*k], scores float32 [nq*k])."""
        Q = _as_f32_matrix(queries, "queries", self._dim)
        nq = Q.shape[0]
        ids = np.empty(nq * int(k), dtype=np.uint64)
        sc = np.empty(nq * int(k), dtype=np.float32)
        self._check(_lib.lib().maivs_concurrent_search_batch(self._h, _ptr(Q), nq, int(k), int(nprobe),
                                                             float(target_confidence), float(beta), _ptr(ids),
                                                             _ptr(sc)))
        return ids, sc

    def search_batch(self, queries: np.ndarray, k: int, nprobe: int = 16, target_confidence: float = 0.95,
                     beta: float = 8.0):
        ids, sc = self.search_batch_arrays(queries, k, nprobe, target_confidence, beta)
        return ids.tolist(), sc.tolist()

    def __len__(self) -> int:
        n = C.c_size_t(0)
        self._check(_lib.lib().maivs_concurrent_len(self._h, C.byref(n)))
        return n.value

    def stats(self) -> dict:
        out = {}
        v = C.c_double(0.0)
        for name in FlatCellIndex._STATS + ("segments", "head_live", "sealed_live", "tombstones"):
            self._check(_lib.lib().maivs_concurrent_stat(self._h, name.encode(), C.byref(v)))
            out[name] = float(v.value)
        return out

    # ---- writes (host cores) ----
    def add_batch(self, ids, vectors: np.ndarray) -> None:
        ids_a = np.ascontiguousarray(np.asarray(list(ids) if not isinstance(ids, np.ndarray) else ids,
                                                dtype=np.uint64))
        v = np.asarray(vectors)
        if v.ndim != 2 or v.shape[0] != ids_a.shape[0] or v.shape[1] != self._dim:
            raise ValueError("shape mismatch")
        if v.dtype != np.float32:
            raise TypeError("vectors must be a float32 numpy array")
        if not v.flags["C_CONTIGUOUS"]:
            raise ValueError("vectors must be C-contiguous (use np.ascontiguousarray)")
        self._check(_lib.lib().maivs_concurrent_add_batch(self._h, _ptr(ids_a), _ptr(v), ids_a.shape[0]))

    def remove(self, id: int) -> bool:
        r = C.c_int(0)
        self._check(_lib.lib().maivs_concurrent_remove(self._h, int(id), C.byref(r)))
        return bool(r.value)

    def remove_many(self, ids) -> int:
        a = np.ascontiguousarray(np.asarray(list(ids) if not isinstance(ids, np.ndarray) else ids, dtype=np.uint64))
        n = C.c_size_t(0)
        self._check(_lib.lib().maivs_concurrent_remove_many(self._h, _ptr(a) if a.size else None, a.shape[0],
                                                            C.byref(n)))
        return n.value

    def seal(self) -> None:
        self._check(_lib.lib().maivs_concurrent_seal(self._h))

    def purge_head(self) -> int:
        n = C.c_size_t(0)
        self._check(_lib.lib().maivs_concurrent_purge_head(self._h, C.byref(n)))
        return n.value

    # ---- configuration (the head; concurrent.rs:316-343) ----
    def train_centroids(self, vectors: np.ndarray, n_cells: int, sample: int = 262_144, seed: int = 0x5EED) -> None:
        v = _as_f32_matrix(vectors, "vectors", self._dim)
        self._check(_lib.lib().maivs_concurrent_train_centroids(self._h, _ptr(v), v.shape[0], int(n_cells),
                                                                int(sample), int(seed) & (2**64 - 1)))

    def set_per_dim_sq(self, on: bool) -> None:
        self._check(_lib.lib().maivs_concurrent_set_per_dim_sq(self._h, int(bool(on))))

    def set_two_stage(self, on: bool, mult: int) -> None:
        self._check(_lib.lib().maivs_concurrent_set_two_stage(self._h, int(bool(on)), int(mult)))

    def set_adaptive(self, on: bool, margin: float) -> None:
        self._check(_lib.lib().maivs_concurrent_set_adaptive(self._h, int(bool(on)), float(margin)))

    def set_parallel_scan(self, on: bool) -> None:
        self._check(_lib.lib().maivs_concurrent_set_parallel_scan(self._h, int(bool(on))))

    def set_graph_route(self, on: bool, min_cells: int = 0) -> None:
        self._check(_lib.lib().maivs_concurrent_set_graph_route(self._h, int(bool(on)), int(min_cells)))

    def set_tree_route(self, on: bool, min_cells: int = 0, fanout: int = 0, beam_frac: float = 0.0) -> None:
        self._check(_lib.lib().maivs_concurrent_set_tree_route(self._h, int(bool(on)), int(min_cells), int(fanout),
                                                               float(beam_frac)))

    def compact(self) -> None:
        self._check(_lib.lib().maivs_concurrent_compact(self._h))

    def set_build_device(self, device: int | None) -> None:
        """Run the head's k-means and placement on CUDA device `device` (None: the host cores);
        later heads inherit it. The index built is the same either way."""
        self._check(_lib.lib().maivs_concurrent_set_build_device(self._h, -1 if device is None else int(device)))

    def to_device(self, device: int = 0) -> None:
        """CUDA device of the searches (default 0)."""
        self._check(_lib.lib().maivs_concurrent_to_device(self._h, int(device)))

    # ---- inspection and instrumentation (no counterpart in the reference) ----
    def kernel_clock(self, on: bool) -> None:
        """Time every kernel of subsequent searches (all segments, the head, the merge)."""
        self._check(_lib.lib().maivs_concurrent_kernel_clock(self._h, int(bool(on))))

    def kernel_times(self, reset: bool = False) -> dict:
        """{kernel name: (total ms, launches)} accumulated while the clock was on."""
        n = 32
        names = (C.c_char_p * n)()
        ms = (C.c_double * n)()
        la = (C.c_uint64 * n)()
        got = C.c_size_t(0)
        self._check(_lib.lib().maivs_concurrent_kernel_times(self._h, int(bool(reset)), names, ms, la, n,
                                                             C.byref(got)))
        return {names[i].decode(): (float(ms[i]), int(la[i])) for i in range(got.value)}

    def n_segments(self) -> int:
        n = C.c_size_t(0)
        self._check(_lib.lib().maivs_concurrent_segments(self._h, C.byref(n)))
        return n.value

    def segment_array(self, segment: int, name: str) -> np.ndarray:
        """Copy of one array of sealed segment `segment` (-1: the head), as FlatCellIndex.array."""
        p = C.c_void_p()
        n = C.c_size_t(0)
        eb = C.c_size_t(0)
        self._check(_lib.lib().maivs_concurrent_array(self._h, int(segment), name.encode(), C.byref(p), C.byref(n),
                                                      C.byref(eb)))
        dt = np.dtype(_ARRAY_DTYPES.get(name))
        if n.value == 0 or not p.value:
            return np.zeros(0, dtype=dt)
        raw = np.ctypeslib.as_array(C.cast(p, C.POINTER(C.c_uint8)), shape=(n.value * eb.value,))
        return raw.view(dt).copy()


def nccl_unique_id() -> bytes:
    """A fresh 128-byte NCCL unique id (rank 0 makes it; every rank passes it to shard())."""
    buf = (C.c_uint8 * 128)()
    rc = _lib.lib().maivs_nccl_unique_id(buf, 128)
    if rc != _lib.OK:
        raise MaivsError(f"nccl_unique_id failed: {_lib.lib().maivs_status_string(rc).decode()}")
    return bytes(buf)


def shard_over_torch(ix: "FlatCellIndex", group=None) -> None:
    """Shard `ix` over the ranks of a torch.distributed group (rank r -> cells of rank r).

    Rank 0 makes the NCCL id and the group broadcasts it; torch is only the rendezvous here,
    the searches then run over the engine's own NCCL communicator."""
    import torch.distributed as dist

    rank, world = dist.get_rank(group), dist.get_world_size(group)
    obj = [nccl_unique_id() if rank == 0 else None]
    dist.broadcast_object_list(obj, src=0, group=group)
    ix.shard(rank, world, obj[0])


def set_num_threads(n: int) -> None:
    """Host threads of the index build and of the host search's staging (calling thread)."""
    if _lib.lib().maivs_set_num_threads(int(n)) != _lib.OK:
        raise ValueError("the thread count must be at least 1")


def launch_count() -> int:
    """Kernels this library has launched in this process."""
    return int(_lib.lib().maivs_launch_count())


def profile(on: bool) -> None:
    """Turn phase profiling on or off (process-wide), as the reference's maivs.profile."""
    _lib.lib().maivs_profile(int(bool(on)))


def profile_read(reset: bool = True):
    """Accumulated phase times in milliseconds (q.count is a count), as maivs.profile_read."""
    n = 32
    names = (C.c_char_p * n)()
    vals = (C.c_double * n)()
    got = C.c_size_t(0)
    _lib.lib().maivs_profile_read(int(bool(reset)), names, vals, n, C.byref(got))
    return [(names[i].decode(), float(vals[i])) for i in range(got.value)]
