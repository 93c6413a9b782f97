"""Builds libinferc_b200.so in-tree with nvcc for sm_100a (B200 only).

    python -m inferc_b200.build [--force]

Objects go to inferc_b200/_build/ and the shared library to
inferc_b200/libinferc_b200.so; both are git-ignored build products.
"""
from __future__ import annotations

import argparse
import concurrent.futures as cf
import glob
import os
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
CSRC = os.path.join(HERE, "csrc")
BUILD = os.path.join(HERE, "_build")
LIB = os.path.join(HERE, "libinferc_b200.so")
INCLUDE = os.path.join(os.path.dirname(HERE), "include")
NVCC = os.environ.get("NVCC", "/usr/local/cuda/bin/nvcc")

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
FLAGS = ["-O3", "-std=c++17", "-lineinfo", "-Xcompiler", "-fPIC", "-Xcompiler", "-Wall",
         "--expt-relaxed-constexpr", f"-I{INCLUDE}"]


def _deps() -> list[str]:
    return (glob.glob(os.path.join(CSRC, "*.cuh")) + glob.glob(os.path.join(CSRC, "*.h")) +
            glob.glob(os.path.join(INCLUDE, "*.h")))


def _stale(target: str, sources: list[str]) -> bool:
    if not os.path.exists(target):
        return True
    t = os.path.getmtime(target)
    return any(os.path.getmtime(s) > t for s in sources)


def _compile(src: str, force: bool, verbose_ptxas: bool) -> str:
    obj = os.path.join(BUILD, os.path.basename(src) + ".o")
    if force or _stale(obj, [src] + _deps()):
        cmd = [NVCC, *ARCH, *FLAGS, "-c", src, "-o", obj]
        if verbose_ptxas:
            cmd.insert(1, "-Xptxas=-v")
        subprocess.run(cmd, check=True)
    return obj


def build(force: bool = False, verbose_ptxas: bool = False) -> str:
    os.makedirs(BUILD, exist_ok=True)
    sources = sorted(glob.glob(os.path.join(CSRC, "*.cu")) + glob.glob(os.path.join(CSRC, "*.cc")))
    with cf.ThreadPoolExecutor(max_workers=min(8, os.cpu_count() or 1)) as ex:
        objs = list(ex.map(lambda s: _compile(s, force, verbose_ptxas), sources))
    if force or _stale(LIB, objs):
        subprocess.run([NVCC, *ARCH, "-shared", "-o", LIB, *objs, "-lcudart"], check=True)
    return LIB


if __name__ == "__main__":
    ap = argparse.ArgumentParser()
    ap.add_argument("--force", action="store_true")
    ap.add_argument("--ptxas-v", action="store_true")
    a = ap.parse_args()
    print(build(a.force, a.ptxas_v), file=sys.stderr)
