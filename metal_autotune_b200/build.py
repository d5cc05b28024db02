"""Build libmt.so (the sm_100a region kernels) in-tree with nvcc, and
libmt_graph.so (the host-side graph substitution engine) with g++.

Each translation unit compiles with relocatable device code (the device
status word is shared across them) and the objects are device-linked into
one shared library at metal_autotune_b200/lib/libmt.so. Rebuilds only when a
source or header is newer than the library. Cross-compiles without a GPU.
"""
from __future__ import annotations

import concurrent.futures as cf
import os
import shutil
import subprocess
import sys
from pathlib import Path

PKG = Path(__file__).resolve().parent
CSRC = PKG / "csrc"
LIBDIR = PKG / "lib"
LIB = LIBDIR / "libmt.so"
INCLUDE = PKG.parent / "include"
OBJDIR = PKG / "_build"

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = ["-O3", "-lineinfo", "-std=c++17", "-Xcompiler", "-fPIC", "-rdc=true",
              "--expt-relaxed-constexpr", "-diag-suppress", "177"]


def nvcc() -> str:
    path = shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc"
    if not Path(path).exists():
        raise RuntimeError("nvcc not found; libmt.so cannot be built")
    return path


def sources() -> list[Path]:
    return sorted(CSRC.glob("*.cu"))


def _stale(target: Path, deps: list[Path]) -> bool:
    if not target.exists():
        return True
    t = target.stat().st_mtime
    return any(d.stat().st_mtime > t for d in deps)


def build_library(force: bool = False, verbose: bool = False, jobs: int | None = None) -> Path:
    """Compile every csrc/*.cu for sm_100a and link libmt.so; returns its path."""
    headers = list(CSRC.glob("*.cuh")) + list(CSRC.glob("*.h")) + [INCLUDE / "mt.h"]
    srcs = sources()
    if not force and not _stale(LIB, srcs + headers + [Path(__file__)]):
        return LIB
    OBJDIR.mkdir(exist_ok=True)
    LIBDIR.mkdir(exist_ok=True)
    cc = nvcc()

    def compile_one(src: Path) -> Path:
        obj = OBJDIR / (src.stem + ".o")
        if force or _stale(obj, [src] + headers + [Path(__file__)]):
            cmd = [cc, *ARCH, *NVCC_FLAGS, "-c", str(src), "-o", str(obj)]
            res = subprocess.run(cmd, capture_output=True, text=True)
            if res.returncode != 0:
                raise RuntimeError(f"nvcc failed on {src.name}:\n{res.stdout}\n{res.stderr}")
            if verbose and (res.stdout or res.stderr):
                print(res.stdout, res.stderr, file=sys.stderr)
        return obj

    with cf.ThreadPoolExecutor(max_workers=jobs or min(len(srcs), os.cpu_count() or 4)) as ex:
        objs = list(ex.map(compile_one, srcs))
    tmp = LIB.with_suffix(".so.tmp")
    cmd = [cc, *ARCH, "-shared", "-rdc=true", *map(str, objs), "-o", str(tmp),
           "-lcudart", "-Xcompiler", "-fPIC"]
    res = subprocess.run(cmd, capture_output=True, text=True)
    if res.returncode != 0:
        raise RuntimeError(f"link of libmt.so failed:\n{res.stdout}\n{res.stderr}")
    os.replace(tmp, LIB)
    return LIB


GRAPH_SRC = CSRC / "graph_native.cpp"
GRAPH_LIB = LIBDIR / "libmt_graph.so"


def build_graph_library(force: bool = False) -> Path:
    """Compile csrc/graph_native.cpp (plain C++17, no CUDA) into
    lib/libmt_graph.so; returns its path."""
    deps = [GRAPH_SRC, INCLUDE / "mt_graph.h", Path(__file__)]
    if not force and not _stale(GRAPH_LIB, deps):
        return GRAPH_LIB
    cxx = shutil.which("g++") or shutil.which("c++")
    if cxx is None:
        raise RuntimeError("no C++ compiler; libmt_graph.so cannot be built")
    LIBDIR.mkdir(exist_ok=True)
    tmp = GRAPH_LIB.with_suffix(".so.tmp")
    cmd = [cxx, "-O2", "-std=c++17", "-shared", "-fPIC", "-Wall", "-Wextra", f"-I{INCLUDE}", str(GRAPH_SRC),
           "-o", str(tmp)]
    res = subprocess.run(cmd, capture_output=True, text=True)
    if res.returncode != 0:
        raise RuntimeError(f"g++ failed on {GRAPH_SRC.name}:\n{res.stdout}\n{res.stderr}")
    os.replace(tmp, GRAPH_LIB)
    return GRAPH_LIB


if __name__ == "__main__":
    print(build_library(force="--force" in sys.argv, verbose=True))
    print(build_graph_library(force="--force" in sys.argv))
