"""Build recipe for libb2q.so (the C-ABI library) -- nvcc for sm_100a only.

Usage: python build.py [--verbose] [--ptxas-info]
Object files go to _build/ (git-ignored); the library to lib/libb2q.so.
"""
from __future__ import annotations

import argparse
import concurrent.futures as cf
import os
import shutil
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
CSRC = os.path.join(HERE, "csrc")
BUILD = os.path.join(HERE, "_build")
LIB = os.path.join(HERE, "lib", "libb2q.so")
NVCC = shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc"

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
COMMON = ["-O3", "-std=c++17", "-lineinfo", "-Xcompiler", "-fPIC", "-Xcompiler", "-fvisibility=hidden",
          "--expt-relaxed-constexpr", "-DB2Q_BUILD"]


def sources():
    out = []
    for name in sorted(os.listdir(CSRC)):
        if name.endswith((".cu", ".cpp")):
            out.append(os.path.join(CSRC, name))
    return out


def _compile(src, verbose, ptxas_info):
    obj = os.path.join(BUILD, os.path.basename(src) + ".o")
    deps = [src] + [os.path.join(CSRC, h) for h in os.listdir(CSRC) if h.endswith((".cuh", ".hpp", ".h"))]
    deps.append(os.path.join(HERE, "..", "include", "b2q.h"))
    if os.path.exists(obj) and not ptxas_info:
        t = os.path.getmtime(obj)
        if all(os.path.getmtime(d) <= t for d in deps if os.path.exists(d)):
            return obj, ""
    cmd = [NVCC, *ARCH, *COMMON, "-c", src, "-o", obj]
    if src.endswith(".cpp"):
        cmd = [NVCC, *COMMON, "-x", "cu", *ARCH, "-c", src, "-o", obj]
    if ptxas_info:
        cmd.insert(1, "-Xptxas=-v")
    if verbose:
        print(" ".join(cmd), flush=True)
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"nvcc failed for {src}:\n{r.stdout}\n{r.stderr}")
    return obj, r.stderr


def build(verbose: bool = False, ptxas_info: bool = False) -> str:
    os.makedirs(BUILD, exist_ok=True)
    os.makedirs(os.path.dirname(LIB), exist_ok=True)
    srcs = sources()
    with cf.ThreadPoolExecutor(max_workers=min(8, len(srcs))) as ex:
        results = list(ex.map(lambda s: _compile(s, verbose, ptxas_info), srcs))
    if ptxas_info:
        for _, log in results:
            if log:
                print(log)
    objs = [o for o, _ in results]
    need_link = not os.path.exists(LIB) or any(os.path.getmtime(o) > os.path.getmtime(LIB) for o in objs)
    if need_link:
        cmd = [NVCC, *ARCH, "-shared", "-o", LIB, *objs, "-lcudart", "-ldl"]
        if verbose:
            print(" ".join(cmd), flush=True)
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError(f"link failed:\n{r.stdout}\n{r.stderr}")
    return LIB


if __name__ == "__main__":
    ap = argparse.ArgumentParser()
    ap.add_argument("--verbose", action="store_true")
    ap.add_argument("--ptxas-info", action="store_true")
    a = ap.parse_args()
    try:
        print(build(a.verbose, a.ptxas_info))
    except RuntimeError as e:
        print(e, file=sys.stderr)
        sys.exit(1)
