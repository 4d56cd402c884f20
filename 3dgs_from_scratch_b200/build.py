"""Build the native library lib3dgs_b200.so (C ABI, sm_100a) in-tree.

Each csrc/*.cu file is compiled by nvcc for sm_100a (B200) into
_build/*.o in parallel and linked into a shared library next to this file.
The library links the CUDA runtime statically and has no torch dependency;
its entry points are declared in include/gs_b200.h.
"""
from __future__ import annotations

import concurrent.futures as cf
import glob
import os
import shutil
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
CSRC = os.path.join(HERE, "csrc")
BUILD = os.path.join(HERE, "_build")
LIB_NAME = "lib3dgs_b200.so"
LIB_PATH = os.path.join(HERE, LIB_NAME)
INCLUDE = os.path.join(os.path.dirname(HERE), "include")

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = ["-O3", "-lineinfo", "-std=c++17", "--expt-relaxed-constexpr", "-Xcompiler",
              "-fPIC", "-Xcompiler", "-fvisibility=hidden"] + ARCH


def nvcc() -> str:
    path = shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc"
    if not os.path.exists(path):
        raise RuntimeError("nvcc not found; the CUDA toolkit is required to build lib3dgs_b200")
    return path


def _sources():
    return sorted(glob.glob(os.path.join(CSRC, "*.cu")))


def _headers():
    return sorted(glob.glob(os.path.join(CSRC, "*.cuh")) + glob.glob(os.path.join(INCLUDE, "*.h")))


def _stale(target: str, deps) -> bool:
    if not os.path.exists(target):
        return True
    t = os.path.getmtime(target)
    return any(os.path.getmtime(d) > t for d in deps)


def _compile(src: str, verbose: bool, ptxas_info: bool) -> str:
    obj = os.path.join(BUILD, os.path.basename(src)[:-3] + ".o")
    if not _stale(obj, [src] + _headers()):
        return obj
    cmd = [nvcc()] + NVCC_FLAGS + ["-I", INCLUDE, "-c", src, "-o", obj]
    if ptxas_info:
        cmd += ["-Xptxas", "-v"]
    if verbose:
        print(" ".join(cmd), flush=True)
    res = subprocess.run(cmd, capture_output=True, text=True)
    if res.returncode != 0:
        raise RuntimeError(f"nvcc failed for {src}:\n{res.stdout}\n{res.stderr}")
    if ptxas_info and res.stderr:
        print(res.stderr, file=sys.stderr)
    return obj


def build(verbose: bool = False, ptxas_info: bool = False, force: bool = False) -> str:
    """Compile (if stale) and link lib3dgs_b200.so; returns its path."""
    os.makedirs(BUILD, exist_ok=True)
    srcs = _sources()
    if force:
        for o in glob.glob(os.path.join(BUILD, "*.o")):
            os.remove(o)
    with cf.ThreadPoolExecutor(max_workers=min(len(srcs), os.cpu_count() or 4)) as ex:
        objs = list(ex.map(lambda s: _compile(s, verbose, ptxas_info), srcs))
    if _stale(LIB_PATH, objs):
        tmp = LIB_PATH + ".tmp"
        cmd = [nvcc()] + ARCH + ["-shared", "-Xcompiler", "-fPIC", "-o", tmp] + objs
        if verbose:
            print(" ".join(cmd), flush=True)
        res = subprocess.run(cmd, capture_output=True, text=True)
        if res.returncode != 0:
            raise RuntimeError(f"link failed:\n{res.stdout}\n{res.stderr}")
        os.replace(tmp, LIB_PATH)
    return LIB_PATH


if __name__ == "__main__":
    print(build(verbose="-v" in sys.argv, ptxas_info="--ptxas" in sys.argv,
                force="--force" in sys.argv))
