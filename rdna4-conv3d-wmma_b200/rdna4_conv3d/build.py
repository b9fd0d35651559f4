"""Build ``libr4c_conv3d.so`` in-tree for sm_100a (``python -m rdna4_conv3d.build``).

The library is plain nvcc output (no torch extension): the kernels and the
C-ABI in ``csrc/`` compile (one object per source, in parallel) and link to
one shared object next to this file, where ``_native`` loads it. Cross-compiles on a machine without a GPU.
"""
from __future__ import annotations

import os
import shutil
import subprocess
import sys
from concurrent.futures import ThreadPoolExecutor

PKG_DIR = os.path.dirname(os.path.abspath(__file__))
SRC_DIR = os.path.join(os.path.dirname(PKG_DIR), "csrc")
INC_DIR = os.path.join(os.path.dirname(os.path.dirname(PKG_DIR)), "include")
OUT = os.path.join(PKG_DIR, "libr4c_conv3d.so")
OBJ_DIR = os.path.join(os.path.dirname(PKG_DIR), "_build")  # objects (git-ignored)
SOURCES = ["r4c_api.cu", "r4c_generic.cu", "r4c_tc.cu", "r4c_tc_dw.cu", "r4c_tc_stem.cu", "r4c_tc_stem_dx.cu", "r4c_tc_tconv.cu", "r4c_noalloc.cu", "r4c_general.cu", "r4c_bn.cu", "r4c_watchdog.cu", "r4c_ce.cu"]
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]


def nvcc() -> str:
    for cand in (shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if cand and os.path.exists(cand):
            return cand
    raise RuntimeError("nvcc not found")


def _newest(paths):
    return max(os.path.getmtime(p) for p in paths)


def _compile(src: str, obj: str, verbose: bool) -> None:
    cmd = [nvcc(), *ARCH, "-O3", "-lineinfo", "-std=c++17", "-Xcompiler", "-fPIC", "-c", "-diag-suppress", "177",
           "-I", INC_DIR, "-o", obj + ".tmp", src]
    if verbose:
        print(" ".join(cmd), flush=True)
    subprocess.run(cmd, check=True)
    os.replace(obj + ".tmp", obj)


def build(force: bool = False, verbose: bool = False) -> str:
    """Compile every source to an object (in parallel, only the stale ones) and link the library."""
    srcs = [os.path.join(SRC_DIR, s) for s in SOURCES]
    headers = [os.path.join(SRC_DIR, f) for f in os.listdir(SRC_DIR) if f.endswith((".h", ".cuh"))]
    headers.append(os.path.join(INC_DIR, "r4c_conv3d.h"))
    if not force and os.path.exists(OUT) and os.path.getmtime(OUT) >= _newest(srcs + headers):
        return OUT
    os.makedirs(OBJ_DIR, exist_ok=True)
    newest_header = _newest(headers)
    jobs = []
    objs = []
    for s in srcs:
        o = os.path.join(OBJ_DIR, os.path.basename(s) + ".o")
        objs.append(o)
        if force or not os.path.exists(o) or os.path.getmtime(o) < max(os.path.getmtime(s), newest_header):
            jobs.append((s, o))
    with ThreadPoolExecutor(max_workers=max(1, min(len(jobs), os.cpu_count() or 1))) as ex:
        for f in [ex.submit(_compile, s, o, verbose) for s, o in jobs]:
            f.result()
    cmd = [nvcc(), *ARCH, "-shared", "-o", OUT + ".tmp", *objs]
    if verbose:
        print(" ".join(cmd), flush=True)
    subprocess.run(cmd, check=True)
    os.replace(OUT + ".tmp", OUT)
    return OUT


if __name__ == "__main__":
    print(build(force="--force" in sys.argv, verbose=True))
