"""Builds libnvfp4_b200.so in-tree from csrc/*.cu for sm_100a.

Each translation unit is compiled with nvcc (-gencode arch=compute_100a,code=sm_100a
-lineinfo -O3) into ``_build/`` and linked into ``libnvfp4_b200.so`` beside this
file, so the library travels with the source tree.  A unit is rebuilt when it,
or any header under ``csrc/`` or ``include/``, is newer than its object.
"""
from __future__ import annotations

import concurrent.futures as cf
import glob
import os
import subprocess
import sys

PKG = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(PKG)
CSRC = os.path.join(PKG, "csrc")
BUILD = os.path.join(PKG, "_build")
LIB = os.path.join(PKG, "libnvfp4_b200.so")

NVCC_FLAGS = [
    "-std=c++17", "-O3", "-lineinfo",
    "-gencode", "arch=compute_100a,code=sm_100a",
    "-Xcompiler", "-fPIC", "-Xcompiler", "-fvisibility=hidden",
    "--expt-relaxed-constexpr",
    f"-I{os.path.join(ROOT, 'include')}",
]


def _headers_mtime() -> float:
    hs = glob.glob(os.path.join(CSRC, "*.cuh")) + glob.glob(os.path.join(CSRC, "*.h")) + \
        glob.glob(os.path.join(ROOT, "include", "*.h"))
    return max((os.path.getmtime(h) for h in hs), default=0.0)


def _compile(src: str, extra: list[str], verbose: bool) -> str:
    obj = os.path.join(BUILD, os.path.basename(src).replace(".cu", ".o"))
    if (os.path.exists(obj) and os.path.getmtime(obj) >= os.path.getmtime(src)
            and os.path.getmtime(obj) >= _headers_mtime()
            and os.path.getmtime(obj) >= os.path.getmtime(__file__)):
        return obj
    cmd = ["nvcc", *NVCC_FLAGS, *extra, "-c", src, "-o", obj]
    if verbose:
        print(" ".join(cmd), flush=True)
    subprocess.run(cmd, check=True)
    return obj


def build(verbose: bool = False, extra: list[str] | None = None) -> str:
    os.makedirs(BUILD, exist_ok=True)
    srcs = sorted(glob.glob(os.path.join(CSRC, "*.cu")))
    with cf.ThreadPoolExecutor(max_workers=min(8, len(srcs))) as ex:
        objs = list(ex.map(lambda s: _compile(s, extra or [], verbose), srcs))
    if (not os.path.exists(LIB)
            or any(os.path.getmtime(o) > os.path.getmtime(LIB) for o in objs)):
        cmd = ["nvcc", "-shared", "-gencode", "arch=compute_100a,code=sm_100a", "-o", LIB, *objs,
               "-lcudart"]
        if verbose:
            print(" ".join(cmd), flush=True)
        subprocess.run(cmd, check=True)
    return LIB


if __name__ == "__main__":
    extra = [a for a in sys.argv[1:] if a.startswith("-")]
    print(build(verbose=True, extra=extra))
