"""Build libmaivs_b200.so in-tree: hand-written sm_100a kernels plus the host-side index build.

    python -m maivs_b200.build          # incremental
    python -m maivs_b200.build --force  # rebuild everything

Host code and kernels are compiled without floating-point contraction (-ffp-contract=off,
-fmad=false): the reference never fuses a*b+c, and every fused multiply-add the reference does use
is written out explicitly in the sources.
"""
from __future__ import annotations

import os
import subprocess
import sys
from concurrent.futures import ThreadPoolExecutor

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)
CSRC = os.path.join(HERE, "csrc")
OBJ = os.path.join(HERE, "_build")
LIB = os.path.join(HERE, "libmaivs_b200.so")

NVCC = os.environ.get("NVCC", "nvcc")
CXX = os.environ.get("MAIVS_CXX", "g++")
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
HOST_FLAGS = ["-O3", "-std=c++17", "-fPIC", "-fopenmp", "-mavx2", "-mfma", "-ffp-contract=off", "-Wall",
              "-Wno-unused-function"]
CUDA_INC = "/usr/local/cuda/include"

SOURCES = [
    ("host/tree_host.cpp", "cxx"),
    ("host/index_build.cpp", "cxx"),
    ("host/persist.cpp", "cxx"),
    ("capi.cpp", "cxx"),
    ("concurrent.cpp", "cxx"),
    ("cuda/clock.cu", "nvcc"),
    ("cuda/k_route.cu", "nvcc"),
    ("cuda/k_cellmajor.cu", "nvcc"),
    ("cuda/k_scan_mma.cu", "nvcc"),
    ("cuda/k_perquery.cu", "nvcc"),
    ("cuda/k_rerank.cu", "nvcc"),
    ("cuda/engine.cu", "nvcc"),
    ("cuda/static_search.cu", "nvcc"),
    ("cuda/shard.cu", "nvcc"),
    ("cuda/build.cu", "nvcc"),
    ("cuda/k_merge.cu", "nvcc"),
]
HEADERS = ["handle.h", "host/hostmath.h", "host/index_host.h", "cuda/common.cuh", "cuda/kernels.cuh", "cuda/dev_common.cuh",
           "cuda/umma.cuh", "cuda/engine.h"]


def _cmd(src: str, kind: str, obj: str) -> list[str]:
    path = os.path.join(CSRC, src)
    if kind == "cxx":
        return [CXX, *HOST_FLAGS, "-I", CUDA_INC, "-c", path, "-o", obj]
    return [NVCC, *ARCH, "-O3", "-lineinfo", "-std=c++17", "-fmad=false", "--expt-relaxed-constexpr",
            "-Xcompiler", ",".join(["-fPIC", "-fopenmp", "-mavx2", "-mfma", "-ffp-contract=off"]),
            "-c", path, "-o", obj]


def _stale(obj: str, deps: list[str]) -> bool:
    if not os.path.exists(obj):
        return True
    t = os.path.getmtime(obj)
    return any(os.path.getmtime(d) > t for d in deps)


def build(force: bool = False, verbose: bool = False) -> str:
    """Compile every source that changed and link the shared library; returns its path."""
    os.makedirs(OBJ, exist_ok=True)
    hdrs = [os.path.join(CSRC, h) for h in HEADERS] + [os.path.join(ROOT, "include", "maivs_b200.h")]
    jobs = []
    objs = []
    for src, kind in SOURCES:
        obj = os.path.join(OBJ, os.path.basename(src) + ".o")
        objs.append(obj)
        if force or _stale(obj, [os.path.join(CSRC, src), *hdrs]):
            jobs.append(_cmd(src, kind, obj))

    def run(cmd):
        if verbose:
            print(" ".join(cmd), flush=True)
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError(f"compile failed: {' '.join(cmd)}\n{r.stdout}\n{r.stderr}")
        return r.stderr

    with ThreadPoolExecutor(max_workers=max(1, min(len(jobs), os.cpu_count() or 1))) as ex:
        for warn in ex.map(run, jobs):
            if verbose and warn.strip():
                print(warn)
    if force or jobs or _stale(LIB, objs):
        link = [NVCC, *ARCH, "-shared", "-o", LIB, *objs, "-Xcompiler", "-fopenmp", "-lgomp", "-ldl"]
        run(link)
    return LIB


if __name__ == "__main__":
    build(force="--force" in sys.argv, verbose=True)
    print(LIB)
