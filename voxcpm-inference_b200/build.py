"""Builds libvxb.so (CUDA kernels + C ABI + C++ host API) for sm_100a, in-tree.

    python voxcpm-inference_b200/build.py [-v]

Objects go to voxcpm-inference_b200/_build/, the library to
voxcpm-inference_b200/lib/libvxb.so.  Only files whose sources (or shared
headers) changed are recompiled.
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
LIB = os.path.join(PKG, "lib", "libvxb.so")
NVCC = os.environ.get("NVCC", "/usr/local/cuda/bin/nvcc")
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
INC = ["-I" + os.path.join(ROOT, "include"), "-I" + CSRC, "-I" + os.path.join(PKG, "include")]


def _sources():
    cu = sorted(glob.glob(os.path.join(CSRC, "*.cu")))
    cpp = sorted(glob.glob(os.path.join(CSRC, "*.cpp")) + glob.glob(os.path.join(CSRC, "host", "*.cpp")))
    return cu, cpp


def _headers():
    hs = glob.glob(os.path.join(CSRC, "**", "*.cuh"), recursive=True)
    hs += glob.glob(os.path.join(CSRC, "**", "*.h"), recursive=True)
    hs += glob.glob(os.path.join(ROOT, "include", "*.h"))
    hs += glob.glob(os.path.join(PKG, "include", "**", "*.h"), recursive=True)
    return hs


def _stale(obj, src, hdr_mtime):
    return not os.path.exists(obj) or os.path.getmtime(obj) < max(os.path.getmtime(src), hdr_mtime)


def _run(cmd, verbose):
    if verbose:
        print(" ".join(cmd), flush=True)
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"build failed: {' '.join(cmd)}\n{r.stdout}\n{r.stderr}")
    return r.stdout + r.stderr


def build(verbose: bool = False) -> str:
    os.makedirs(BUILD, exist_ok=True)
    os.makedirs(os.path.dirname(LIB), exist_ok=True)
    cu, cpp = _sources()
    hdr_mtime = max([os.path.getmtime(h) for h in _headers()] + [os.path.getmtime(__file__)])
    jobs, objs = [], []
    for s in cu:
        o = os.path.join(BUILD, os.path.basename(s) + ".o")
        objs.append(o)
        if _stale(o, s, hdr_mtime):
            jobs.append([NVCC, *ARCH, "-lineinfo", "-O3", "-std=c++17", "-Xcompiler", "-fPIC,-fvisibility=hidden",
                         *INC, "-c", s, "-o", o])
    for s in cpp:
        o = os.path.join(BUILD, os.path.basename(s) + ".o")
        objs.append(o)
        if _stale(o, s, hdr_mtime):
            jobs.append(["g++", "-O2", "-std=c++17", "-fPIC", "-fvisibility=hidden", "-Wall",
                         "-I/usr/local/cuda/include", *INC, "-c", s, "-o", o])
    with cf.ThreadPoolExecutor(max_workers=os.cpu_count() or 4) as ex:
        for out in ex.map(lambda c: _run(c, verbose), jobs):
            if verbose and out.strip():
                print(out)
    if jobs or not os.path.exists(LIB):
        _run([NVCC, *ARCH, "-shared", "-cudart", "static", "-o", LIB, *objs, "-lpthread", "-ldl", "-lrt"], verbose)
    return LIB


if __name__ == "__main__":
    print(build(verbose="-v" in sys.argv))
