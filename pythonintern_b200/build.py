"""Build ``libb2tp.so`` (the sm_100a kernels and their C ABI) in-tree with nvcc.

Usage: ``python -m pythonintern_b200.build [--force] [-j N]``.  Objects go to
``pythonintern_b200/_build/``; the library is written next to this file so that it
travels with the source tree.  nvcc cross-compiles, so no GPU is needed to build.
"""

import argparse
import concurrent.futures as cf
import os
import shutil
import subprocess
import sys

PKG = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(PKG)
CSRC = os.path.join(PKG, "csrc")
INCLUDE = os.path.join(ROOT, "include")
BUILD = os.path.join(PKG, "_build")
LIB = os.path.join(PKG, "libb2tp.so")

SOURCES = ["api.cu", "norm.cu", "rope_kv.cu", "attention.cu", "gemm_simt.cu", "gemm_tc.cu", "gemm.cu", "comm.cu", "prefill_tc.cu"]
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
FLAGS = ["-O3", "-std=c++17", "-lineinfo", "-Xcompiler", "-fPIC", "--expt-relaxed-constexpr",
         "-I", INCLUDE, "-I", CSRC]


def nvcc():
    for cand in (os.environ.get("NVCC"), shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if cand and os.path.exists(cand):
            return cand
    raise RuntimeError("nvcc not found")


def _deps(src):
    headers = [os.path.join(CSRC, h) for h in os.listdir(CSRC) if h.endswith(".cuh")]
    return [src, os.path.join(INCLUDE, "b2tp.h")] + headers


def _stale(target, deps):
    if not os.path.exists(target):
        return True
    t = os.path.getmtime(target)
    return any(os.path.getmtime(d) > t for d in deps)


def _compile(src, obj, extra, verbose):
    cmd = [nvcc(), "-c", src, "-o", obj] + ARCH + FLAGS + extra
    if verbose:
        print(" ".join(cmd), flush=True)
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"nvcc failed for {os.path.basename(src)}:\n{r.stdout}\n{r.stderr}")
    if verbose and (r.stdout or r.stderr):
        print(r.stdout + r.stderr, flush=True)
    return obj


def build(force=False, jobs=None, verbose=False, ptxas_info=False):
    """Compile every CUDA source for sm_100a and link libb2tp.so; returns its path."""
    os.makedirs(BUILD, exist_ok=True)
    extra = ["-Xptxas", "-v"] if ptxas_info else []
    todo = []
    objs = []
    for s in SOURCES:
        src = os.path.join(CSRC, s)
        obj = os.path.join(BUILD, s.replace(".cu", ".o"))
        objs.append(obj)
        if force or ptxas_info or _stale(obj, _deps(src)):
            todo.append((src, obj))
    if todo:
        with cf.ThreadPoolExecutor(max_workers=jobs or min(8, os.cpu_count() or 4)) as ex:
            for f in [ex.submit(_compile, s, o, extra, verbose or ptxas_info) for s, o in todo]:
                f.result()
    if force or todo or _stale(LIB, objs):
        tmp = LIB + ".tmp"
        cmd = [nvcc(), "-shared", "-o", tmp] + objs + ARCH + ["-Xcompiler", "-fPIC"]
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError(f"link failed:\n{r.stdout}\n{r.stderr}")
        os.replace(tmp, LIB)
    return LIB


def main(argv=None):
    ap = argparse.ArgumentParser(description=__doc__)
    ap.add_argument("--force", action="store_true")
    ap.add_argument("-j", "--jobs", type=int, default=None)
    ap.add_argument("-v", "--verbose", action="store_true")
    ap.add_argument("--ptxas-info", action="store_true", help="print registers/spills/smem per kernel")
    a = ap.parse_args(argv)
    print(build(a.force, a.jobs, a.verbose, a.ptxas_info))


if __name__ == "__main__":
    sys.exit(main())
