"""Build libtosa_b200.so in-tree for sm_100a (nvcc cross-compiles without a GPU).

Usage: python -m tosa_b200.build [--force]

Each translation unit under csrc/ is compiled in parallel into _build/ and the
objects are linked into tosa_b200/libtosa_b200.so (CUDA runtime linked
statically; driver entry points are resolved at run time).
"""

from __future__ import annotations

import glob
import os
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
CSRC = os.path.join(HERE, "csrc")
BUILD = os.path.join(HERE, "_build")
OUT = os.path.join(HERE, "libtosa_b200.so")
NVCC = os.environ.get("NVCC", "/usr/local/cuda/bin/nvcc")

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
CFLAGS = ARCH + ["-O3", "-lineinfo", "-std=c++17", "-Xcompiler", "-fPIC", "-Xcompiler", "-fvisibility=hidden"]


def _sources():
    return sorted(glob.glob(os.path.join(CSRC, "*.cu")))


def _newest_input():
    files = glob.glob(os.path.join(CSRC, "*")) + glob.glob(os.path.join(HERE, "..", "include", "*.h"))
    return max(os.path.getmtime(f) for f in files)


def build(force: bool = False, verbose: bool = False) -> str:
    if not force and os.path.exists(OUT) and os.path.getmtime(OUT) >= _newest_input():
        return OUT
    os.makedirs(BUILD, exist_ok=True)
    newest_header = max(os.path.getmtime(f) for f in glob.glob(os.path.join(CSRC, "*.cuh")) +
                        glob.glob(os.path.join(CSRC, "*.hpp")) + glob.glob(os.path.join(HERE, "..", "include", "*.h")))
    procs, objs = [], []
    for src in _sources():
        obj = os.path.join(BUILD, os.path.basename(src) + ".o")
        objs.append(obj)
        if not force and os.path.exists(obj) and os.path.getmtime(obj) >= max(os.path.getmtime(src), newest_header):
            continue
        cmd = [NVCC, *CFLAGS, "-c", "-o", obj, src]
        if verbose:
            print(" ".join(cmd), flush=True)
        procs.append((src, subprocess.Popen(cmd)))
    failed = [src for src, p in procs if p.wait() != 0]
    if failed:
        raise RuntimeError(f"nvcc failed for {failed}")
    link = [NVCC, *ARCH, "-shared", "-o", OUT + ".tmp", *objs]
    if verbose:
        print(" ".join(link), flush=True)
    subprocess.check_call(link)
    os.replace(OUT + ".tmp", OUT)
    return OUT


if __name__ == "__main__":
    print(build(force="--force" in sys.argv, verbose=True))
