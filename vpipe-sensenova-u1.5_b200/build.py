"""Build libu15c.so in-tree: every csrc/*.cu compiled for sm_100a with nvcc
and linked into vpipe-sensenova-u1.5_b200/lib/libu15c.so (static cudart).

    python vpipe-sensenova-u1.5_b200/build.py [--force]

Incremental: an object is rebuilt when its source or any csrc header or
include/u15c.h is newer than it.
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
LIB = os.path.join(HERE, "lib", "libu15c.so")

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
FLAGS = ARCH + ["-O3", "-lineinfo", "-std=c++17", "-Xcompiler", "-fPIC",
                "-Xcompiler", "-Wall", "--expt-relaxed-constexpr", "-I", CSRC,
                "-I", os.path.join(ROOT, "include")]


def nvcc() -> str:
    for c in (shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if c and os.path.exists(c):
            return c
    raise RuntimeError("nvcc not found: the CUDA toolkit is required to build libu15c")


def _headers():
    return glob.glob(os.path.join(CSRC, "*.h")) + glob.glob(os.path.join(CSRC, "*.cuh")) + [
        os.path.join(ROOT, "include", "u15c.h")]


def _stale(src: str, obj: str, hdr_mtime: float) -> bool:
    if not os.path.exists(obj):
        return True
    m = os.path.getmtime(obj)
    return os.path.getmtime(src) > m or hdr_mtime > m


def build(force: bool = False, verbose: bool = False) -> str:
    os.makedirs(BUILD, exist_ok=True)
    os.makedirs(os.path.dirname(LIB), exist_ok=True)
    cc = nvcc()
    srcs = sorted(glob.glob(os.path.join(CSRC, "*.cu")))
    hdr = max(os.path.getmtime(h) for h in _headers())
    objs = [os.path.join(BUILD, os.path.basename(s)[:-3] + ".o") for s in srcs]
    todo = [(s, o) for s, o in zip(srcs, objs) if force or _stale(s, o, hdr)]

    def one(so):
        s, o = so
        cmd = [cc] + FLAGS + ["-c", s, "-o", o]
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError(f"nvcc failed on {os.path.basename(s)}:\n{r.stderr}")
        return r.stderr if verbose else ""

    if todo:
        with cf.ThreadPoolExecutor(max_workers=min(8, len(todo))) as ex:
            for msg in ex.map(one, todo):
                if msg:
                    print(msg, file=sys.stderr)
    if todo or not os.path.exists(LIB):
        tmp = LIB + ".tmp"
        cmd = [cc] + ARCH + ["-shared", "-o", tmp] + objs
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError(f"link failed:\n{r.stderr}")
        os.replace(tmp, LIB)
    return LIB


if __name__ == "__main__":
    ap = argparse.ArgumentParser()
    ap.add_argument("--force", action="store_true")
    ap.add_argument("-v", "--verbose", action="store_true")
    a = ap.parse_args()
    print(build(a.force, a.verbose))
