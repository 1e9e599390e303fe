"""Build the CUDA library in-tree: ``libirodori_b200.so`` for sm_100a.

nvcc compiles every translation unit under ``csrc/`` with
``-gencode arch=compute_100a,code=sm_100a`` (cross-compiles without a GPU),
objects go to ``_build/`` and are relinked only when a source or header is
newer than the library.
"""

from __future__ import annotations

import os
import shutil
import subprocess
import sys
from concurrent.futures import ThreadPoolExecutor
from pathlib import Path

PKG = Path(__file__).resolve().parent
CSRC = PKG / "csrc"
INCLUDE = PKG.parent / "include"
BUILD = PKG / "_build"
LIB = PKG / "libirodori_b200.so"
# Kernel-level hooks for the GPU unit tests, kept out of the product library.
TEST_LIB = PKG / "libirodori_b200_testhooks.so"
TEST_ONLY = {"testhooks.cpp"}

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
FLAGS = ["-O3", "-std=c++17", "-lineinfo", "-Xcompiler", "-fPIC", "-Xcompiler", "-fvisibility=hidden",
         "--expt-relaxed-constexpr", "-I", str(CSRC), "-I", str(INCLUDE)]


def nvcc() -> str:
    for c in (os.environ.get("NVCC"), "/usr/local/cuda/bin/nvcc", shutil.which("nvcc")):
        if c and Path(c).exists():
            return c
    raise RuntimeError("nvcc not found")


def sources():
    return sorted(list(CSRC.glob("*.cu")) + list(CSRC.glob("*.cpp")))


def _newest_header() -> float:
    hs = list(CSRC.glob("*.hpp")) + list(CSRC.glob("*.cuh")) + list(INCLUDE.glob("*.h"))
    return max((h.stat().st_mtime for h in hs), default=0.0)


def build(verbose: bool = False, force: bool = False) -> Path:
    BUILD.mkdir(exist_ok=True)
    srcs = sources()
    hdr = _newest_header()
    objs = []
    jobs = []
    for s in srcs:
        o = BUILD / (s.name + ".o")
        objs.append(o)
        if force or not o.exists() or o.stat().st_mtime < max(s.stat().st_mtime, hdr):
            extra = ["-x", "cu"] if s.suffix == ".cpp" else []
            jobs.append([nvcc(), *ARCH, *FLAGS, *extra, "-c", str(s), "-o", str(o)])

    def run(cmd):
        if verbose:
            print(" ".join(cmd), flush=True)
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError(f"nvcc failed for {cmd[-3]}:\n{r.stdout}\n{r.stderr}")
        if verbose and r.stderr.strip():
            print(r.stderr, file=sys.stderr)

    with ThreadPoolExecutor(max_workers=min(8, os.cpu_count() or 4)) as ex:
        list(ex.map(run, jobs))
    newest_obj = max(o.stat().st_mtime for o in objs)
    prod = [o for o, s in zip(objs, srcs) if s.name not in TEST_ONLY]
    for lib, members in ((LIB, prod), (TEST_LIB, objs)):
        if force or jobs or not lib.exists() or lib.stat().st_mtime < newest_obj:
            cmd = [nvcc(), *ARCH, "-shared", "-o", str(lib) + ".tmp", *map(str, members), "-lcudart_static", "-ldl",
                   "-lpthread", "-lrt"]
            run(cmd)
            os.replace(str(lib) + ".tmp", lib)
    return LIB


if __name__ == "__main__":
    build(verbose="-v" in sys.argv, force="-f" in sys.argv)
    print(LIB)
