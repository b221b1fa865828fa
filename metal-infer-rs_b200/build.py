"""Builds the engine's shared library in-tree for sm_100a.

    python metal-infer-rs_b200/build.py [--force] [-j N]

Every csrc/*.cu is compiled by nvcc (-gencode arch=compute_100a,code=sm_100a)
into _build/, then linked into metal_infer/libmetal_infer.so next to the
Python binding. Objects are rebuilt when their source or any header changed.
"""
from __future__ import annotations

import argparse
import concurrent.futures as cf
import glob
import os
import shutil
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)
CSRC = os.path.join(HERE, "csrc")
BUILD = os.path.join(HERE, "_build")
LIB = os.path.join(HERE, "metal_infer", "libmetal_infer.so")

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]


def nvcc() -> str:
    cand = os.path.join(os.environ.get("CUDA_HOME", "/usr/local/cuda"), "bin", "nvcc")
    return cand if os.path.exists(cand) else (shutil.which("nvcc") or "nvcc")


def nccl_dirs():
    """Include and library directories of the NCCL that torch ships with."""
    try:
        import nvidia.nccl  # type: ignore  (a namespace package: no __file__)
        base = list(nvidia.nccl.__path__)[0]
        inc, lib = os.path.join(base, "include"), os.path.join(base, "lib")
        if os.path.exists(os.path.join(inc, "nccl.h")):
            return inc, lib
    except Exception:
        pass
    return None, None


def cflags():
    flags = ARCH + ["-O3", "-std=c++17", "-lineinfo", "-Xcompiler", "-fPIC,-O3",
                    "--expt-relaxed-constexpr", "-I", os.path.join(ROOT, "include"),
                    "-I", CSRC, "-ccbin", "/usr/bin/g++"]
    inc, _ = nccl_dirs()
    if inc:
        flags += ["-I", inc, "-DMI_HAVE_NCCL=1"]
    return flags


def newest_header() -> float:
    hs = glob.glob(os.path.join(CSRC, "*.h")) + glob.glob(os.path.join(CSRC, "*.cuh")) + \
        glob.glob(os.path.join(ROOT, "include", "*.h"))
    return max((os.path.getmtime(h) for h in hs), default=0.0)


def compile_one(src: str, force: bool, extra=()) -> str:
    obj = os.path.join(BUILD, os.path.basename(src) + ".o")
    if (not force and os.path.exists(obj) and os.path.getmtime(obj) >= os.path.getmtime(src)
            and os.path.getmtime(obj) >= newest_header()):
        return obj
    cmd = [nvcc()] + cflags() + list(extra) + ["-c", src, "-o", obj]
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"nvcc failed for {src}:\n{r.stdout}\n{r.stderr}")
    if r.stderr.strip():
        sys.stderr.write(r.stderr)
    return obj


def build(force: bool = False, jobs: int | None = None, verbose_ptxas: bool = False) -> str:
    os.makedirs(BUILD, exist_ok=True)
    srcs = sorted(glob.glob(os.path.join(CSRC, "*.cu")))
    extra = ["-Xptxas", "-v"] if verbose_ptxas else []
    with cf.ThreadPoolExecutor(max_workers=jobs or os.cpu_count() or 4) as ex:
        objs = list(ex.map(lambda s: compile_one(s, force, extra), srcs))
    if (force or not os.path.exists(LIB)
            or os.path.getmtime(LIB) < max(os.path.getmtime(o) for o in objs)):
        _, nccl_lib = nccl_dirs()
        link = [nvcc()] + ARCH + ["-shared", "-cudart", "shared", "-o", LIB] + objs
        if nccl_lib:
            link += ["-L", nccl_lib, "-l:libnccl.so.2", "-Xlinker", "-rpath," + nccl_lib]
        link += ["-lcuda"]
        r = subprocess.run(link, capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError(f"link failed:\n{r.stdout}\n{r.stderr}")
    return LIB


if __name__ == "__main__":
    ap = argparse.ArgumentParser()
    ap.add_argument("--force", action="store_true")
    ap.add_argument("-j", type=int, default=None)
    ap.add_argument("--ptxas-v", action="store_true")
    a = ap.parse_args()
    print(build(a.force, a.j, a.ptxas_v))
