"""Build libmoearc_b200.so in-tree with nvcc for sm_100a.

    python -m moearc_b200.build            # incremental
    python -m moearc_b200.build --clean

Each csrc/*.cu compiles with nvcc, each csrc/*.cpp (host-only code) with the host C++ compiler,
to an object under moearc_b200/_build/ (in parallel, skipped when up to date against its sources
and headers), then both link into moearc_b200/libmoearc_b200.so.
"""
from __future__ import annotations

import concurrent.futures as cf
import glob
import os
import shutil
import subprocess
import sys

PKG = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(PKG)
CSRC = os.path.join(PKG, "csrc")
BUILD = os.path.join(PKG, "_build")
LIB = os.path.join(PKG, "libmoearc_b200.so")
NVCC = os.environ.get("NVCC", "/usr/local/cuda/bin/nvcc")
CXX = os.environ.get("CXX", "g++")

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
FLAGS = ["-O3", "-std=c++17", "-lineinfo", "-Xcompiler", "-fPIC", "--expt-relaxed-constexpr",
         "-Xptxas", "-v"]
# host code: no contraction of a * b + c into an FMA unless the source asks for one
CXXFLAGS = ["-O3", "-std=c++17", "-fPIC", "-pthread", "-ffp-contract=off", "-Wall", "-Wextra"]


def _deps() -> list[str]:
    return (glob.glob(os.path.join(CSRC, "*.cuh")) + glob.glob(os.path.join(CSRC, "*.hpp")) +
            [os.path.join(ROOT, "include", "moearc.h")])


def _stale(obj: str, src: str) -> bool:
    if not os.path.exists(obj):
        return True
    t = os.path.getmtime(obj)
    return any(os.path.getmtime(d) > t for d in [src] + _deps())


def _compile(src: str) -> tuple[str, str]:
    base, ext = os.path.splitext(os.path.basename(src))
    obj = os.path.join(BUILD, base + (".o" if ext == ".cu" else ".host.o"))
    if not _stale(obj, src):
        return obj, ""
    cmd = [NVCC, *ARCH, *FLAGS, "-c", src, "-o", obj] if ext == ".cu" else [CXX, *CXXFLAGS, "-c", src, "-o", obj]
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"nvcc failed on {src}:\n{r.stdout}\n{r.stderr}")
    with open(obj + ".ptxas.txt", "w") as f:
        f.write(r.stderr)
    return obj, r.stderr


def build(verbose: bool = False) -> str:
    os.makedirs(BUILD, exist_ok=True)
    srcs = sorted(glob.glob(os.path.join(CSRC, "*.cu")) + glob.glob(os.path.join(CSRC, "*.cpp")))
    with cf.ThreadPoolExecutor(max_workers=min(8, os.cpu_count() or 4)) as ex:
        results = list(ex.map(_compile, srcs))
    objs = [o for o, _ in results]
    if verbose:
        for _, log in results:
            if log:
                print(log)
    if not os.path.exists(LIB) or any(os.path.getmtime(o) > os.path.getmtime(LIB) for o in objs):
        # the CUDA runtime is linked statically: the library keeps its own runtime state (current
        # device, streams) whatever else the host process has loaded
        cmd = [NVCC, *ARCH, "-shared", "-Xcompiler", "-fPIC", "-cudart", "static", "-o", LIB, *objs, "-lpthread", "-ldl"]
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError(f"link failed:\n{r.stdout}\n{r.stderr}")
    return LIB


def main() -> None:
    if "--clean" in sys.argv:
        shutil.rmtree(BUILD, ignore_errors=True)
        if os.path.exists(LIB):
            os.remove(LIB)
    print(build(verbose="-v" in sys.argv))


if __name__ == "__main__":
    main()
