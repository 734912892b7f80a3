"""ctypes binding of libmaivs_b200.so (the C ABI in include/maivs_b200.h)."""
from __future__ import annotations

import ctypes as C
import os

_HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(_HERE, "libmaivs_b200.so")

OK, BAD_SHAPE, BAD_ARG, BAD_STATE, OOM, CUDA_ERROR, OVERFLOW, UNSUPPORTED, NOT_FOUND, NO_DEVICE = range(10)

_lib = None

_SIGS = {
    "maivs_index_new": (C.c_int, [C.c_size_t, C.c_char_p, C.c_size_t, C.c_uint64, C.c_size_t, C.POINTER(C.c_void_p)]),
    "maivs_index_free": (None, [C.c_void_p]),
    "maivs_last_error": (C.c_char_p, [C.c_void_p]),
    "maivs_status_string": (C.c_char_p, [C.c_int]),
    "maivs_train_centroids": (C.c_int, [C.c_void_p, C.c_void_p, C.c_size_t, C.c_size_t, C.c_size_t, C.c_uint64]),
    "maivs_set_centroids": (C.c_int, [C.c_void_p, C.c_void_p, C.c_size_t]),
    "maivs_add_batch": (C.c_int, [C.c_void_p, C.c_void_p, C.c_void_p, C.c_size_t]),
    "maivs_remove": (C.c_int, [C.c_void_p, C.c_uint64, C.POINTER(C.c_int)]),
    "maivs_compact": (C.c_int, [C.c_void_p]),
    "maivs_set_rerank_factor": (C.c_int, [C.c_void_p, C.c_size_t]),
    "maivs_set_two_stage": (C.c_int, [C.c_void_p, C.c_int, C.c_size_t]),
    "maivs_set_tree_route": (C.c_int, [C.c_void_p, C.c_int, C.c_size_t, C.c_size_t, C.c_float]),
    "maivs_set_graph_route": (C.c_int, [C.c_void_p, C.c_int, C.c_size_t]),
    "maivs_set_adaptive": (C.c_int, [C.c_void_p, C.c_int, C.c_float]),
    "maivs_set_fastscan": (C.c_int, [C.c_void_p, C.c_int]),
    "maivs_set_orthogonal_polysemy": (C.c_int, [C.c_void_p, C.c_size_t, C.c_float]),
    "maivs_set_replication": (C.c_int, [C.c_void_p, C.c_size_t, C.c_float]),
    "maivs_set_per_dim_sq": (C.c_int, [C.c_void_p, C.c_int]),
    "maivs_set_i8_rerank": (C.c_int, [C.c_void_p, C.c_int]),
    "maivs_set_centroid_sq8": (C.c_int, [C.c_void_p, C.c_int]),
    "maivs_set_tags": (C.c_int, [C.c_void_p, C.c_void_p, C.c_void_p, C.c_size_t]),
    "maivs_set_filter": (C.c_int, [C.c_void_p, C.c_int, C.c_uint32, C.c_uint32]),
    "maivs_set_cell_major_min_batch": (C.c_int, [C.c_void_p, C.c_size_t]),
    "maivs_set_build_device": (C.c_int, [C.c_void_p, C.c_int]),
    "maivs_len": (C.c_int, [C.c_void_p, C.POINTER(C.c_size_t)]),
    "maivs_stat": (C.c_int, [C.c_void_p, C.c_char_p, C.POINTER(C.c_double)]),
    "maivs_to_device": (C.c_int, [C.c_void_p, C.c_int]),
    "maivs_search": (C.c_int, [C.c_void_p, C.c_void_p, C.c_size_t, C.c_size_t, C.c_float, C.c_float, C.c_void_p,
                               C.c_void_p, C.POINTER(C.c_size_t)]),
    "maivs_search_batch": (C.c_int, [C.c_void_p, C.c_void_p, C.c_size_t, C.c_size_t, C.c_size_t, C.c_float,
                                     C.c_float, C.c_int, C.c_void_p, C.c_void_p]),
    "maivs_search_batch_device": (C.c_int, [C.c_void_p, C.c_void_p, C.c_size_t, C.c_size_t, C.c_size_t, C.c_float,
                                            C.c_float, C.c_int, C.c_void_p, C.c_void_p, C.c_void_p]),
    "maivs_device_flags": (C.c_int, [C.c_void_p, C.c_void_p, C.POINTER(C.c_uint32)]),
    "maivs_save": (C.c_int, [C.c_void_p, C.c_char_p]),
    "maivs_load": (C.c_int, [C.c_char_p, C.POINTER(C.c_void_p)]),
    "maivs_nccl_unique_id": (C.c_int, [C.c_void_p, C.c_size_t]),
    "maivs_shard": (C.c_int, [C.c_void_p, C.c_int, C.c_int, C.c_void_p, C.c_size_t]),
    "maivs_shard_range": (C.c_int, [C.c_void_p, C.c_int, C.c_int, C.POINTER(C.c_uint32), C.POINTER(C.c_uint32)]),
    "maivs_search_batch_sharded_emulated": (C.c_int, [C.c_void_p, C.c_int, C.c_void_p, C.c_size_t, C.c_size_t,
                                                      C.c_size_t, C.c_float, C.c_float, C.c_void_p, C.c_void_p,
                                                      C.c_void_p]),
    "maivs_search_batch_device_noalloc": (C.c_int, [C.c_void_p, C.c_void_p, C.c_size_t, C.c_size_t, C.c_size_t,
                                                    C.c_float, C.c_float, C.c_void_p, C.c_void_p, C.c_void_p]),
    "maivs_array": (C.c_int, [C.c_void_p, C.c_char_p, C.POINTER(C.c_void_p), C.POINTER(C.c_size_t),
                              C.POINTER(C.c_size_t)]),
    "maivs_kernel_clock": (C.c_int, [C.c_void_p, C.c_int]),
    "maivs_kernel_clock_only": (C.c_int, [C.c_void_p, C.c_char_p]),
    "maivs_kernel_times": (C.c_int, [C.c_void_p, C.c_int, C.POINTER(C.c_char_p), C.POINTER(C.c_double),
                                     C.POINTER(C.c_uint64), C.c_size_t, C.POINTER(C.c_size_t)]),
    "maivs_kernel_busy": (C.c_int, [C.c_void_p, C.POINTER(C.c_char_p), C.POINTER(C.c_double), C.c_size_t,
                                    C.POINTER(C.c_size_t)]),
    "maivs_launch_count": (C.c_uint64, []),
    "maivs_set_num_threads": (C.c_int, [C.c_int]),
    "maivs_last_search_stats": (C.c_int, [C.c_void_p, C.c_char_p, C.c_size_t, C.POINTER(C.c_double), C.c_size_t,
                                          C.POINTER(C.c_size_t)]),
    "maivs_debug_stage": (C.c_int, [C.c_void_p, C.c_int, C.c_void_p, C.c_size_t, C.c_size_t, C.c_size_t, C.c_float,
                                    C.c_float, C.c_int, C.c_void_p, C.c_void_p, C.c_void_p, C.c_void_p, C.c_void_p,
                                    C.c_void_p, C.c_void_p, C.c_void_p, C.c_size_t, C.c_void_p]),
    "maivs_debug_cellmajor": (C.c_int, [C.c_void_p, C.c_void_p, C.c_size_t, C.c_size_t, C.c_size_t, C.c_float,
                                        C.c_float, C.c_void_p, C.c_void_p, C.c_void_p, C.c_void_p, C.c_char_p,
                                        C.c_size_t]),
    "maivs_concurrent_new": (C.c_int, [C.c_size_t, C.c_char_p, C.c_size_t, C.c_uint64, C.c_size_t, C.c_size_t,
                                       C.POINTER(C.c_void_p)]),
    "maivs_concurrent_free": (None, [C.c_void_p]),
    "maivs_concurrent_last_error": (C.c_char_p, [C.c_void_p]),
    "maivs_concurrent_train_centroids": (C.c_int, [C.c_void_p, C.c_void_p, C.c_size_t, C.c_size_t, C.c_size_t,
                                                   C.c_uint64]),
    "maivs_concurrent_add_batch": (C.c_int, [C.c_void_p, C.c_void_p, C.c_void_p, C.c_size_t]),
    "maivs_concurrent_remove": (C.c_int, [C.c_void_p, C.c_uint64, C.POINTER(C.c_int)]),
    "maivs_concurrent_remove_many": (C.c_int, [C.c_void_p, C.c_void_p, C.c_size_t, C.POINTER(C.c_size_t)]),
    "maivs_concurrent_seal": (C.c_int, [C.c_void_p]),
    "maivs_concurrent_purge_head": (C.c_int, [C.c_void_p, C.POINTER(C.c_size_t)]),
    "maivs_concurrent_compact": (C.c_int, [C.c_void_p]),
    "maivs_concurrent_set_per_dim_sq": (C.c_int, [C.c_void_p, C.c_int]),
    "maivs_concurrent_set_two_stage": (C.c_int, [C.c_void_p, C.c_int, C.c_size_t]),
    "maivs_concurrent_set_adaptive": (C.c_int, [C.c_void_p, C.c_int, C.c_float]),
    "maivs_concurrent_set_parallel_scan": (C.c_int, [C.c_void_p, C.c_int]),
    "maivs_concurrent_set_graph_route": (C.c_int, [C.c_void_p, C.c_int, C.c_size_t]),
    "maivs_concurrent_set_tree_route": (C.c_int, [C.c_void_p, C.c_int, C.c_size_t, C.c_size_t, C.c_float]),
    "maivs_concurrent_set_build_device": (C.c_int, [C.c_void_p, C.c_int]),
    "maivs_concurrent_len": (C.c_int, [C.c_void_p, C.POINTER(C.c_size_t)]),
    "maivs_concurrent_stat": (C.c_int, [C.c_void_p, C.c_char_p, C.POINTER(C.c_double)]),
    "maivs_concurrent_to_device": (C.c_int, [C.c_void_p, C.c_int]),
    "maivs_concurrent_search": (C.c_int, [C.c_void_p, C.c_void_p, C.c_size_t, C.c_size_t, C.c_float, C.c_float,
                                          C.c_void_p, C.c_void_p, C.POINTER(C.c_size_t)]),
    "maivs_concurrent_search_batch": (C.c_int, [C.c_void_p, C.c_void_p, C.c_size_t, C.c_size_t, C.c_size_t,
                                                C.c_float, C.c_float, C.c_void_p, C.c_void_p]),
    "maivs_concurrent_segments": (C.c_int, [C.c_void_p, C.POINTER(C.c_size_t)]),
    "maivs_concurrent_kernel_clock": (C.c_int, [C.c_void_p, C.c_int]),
    "maivs_concurrent_kernel_times": (C.c_int, [C.c_void_p, C.c_int, C.POINTER(C.c_char_p), C.POINTER(C.c_double),
                                                C.POINTER(C.c_uint64), C.c_size_t, C.POINTER(C.c_size_t)]),
    "maivs_concurrent_array": (C.c_int, [C.c_void_p, C.c_longlong, C.c_char_p, C.POINTER(C.c_void_p),
                                         C.POINTER(C.c_size_t), C.POINTER(C.c_size_t)]),
    "maivs_profile": (C.c_int, [C.c_int]),
    "maivs_profile_read": (C.c_int, [C.c_int, C.POINTER(C.c_char_p), C.POINTER(C.c_double), C.c_size_t,
                                     C.POINTER(C.c_size_t)]),
}


def lib() -> C.CDLL:
    """Load the shared library; raises if it was not built (there is no fallback)."""
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            raise ImportError(f"{LIB_PATH} is missing: build it with `python -m maivs_b200.build`")
        L = C.CDLL(LIB_PATH, mode=os.RTLD_NOW | os.RTLD_LOCAL)
        for name, (res, args) in _SIGS.items():
            f = getattr(L, name)
            f.restype = res
            f.argtypes = args
        _lib = L
    return _lib


def exported_symbols() -> list[str]:
    return list(_SIGS)
