"""Builds libwxx_cuda.so (all CUDA kernels + the C ABI) in-tree for sm_100a.

Usage: python -m wxx_b200.csrc.build [--force] [--jobs N]

Objects go to ``wxx_b200/csrc/_build/`` and the library to
``wxx_b200/lib/libwxx_cuda.so``; sources are recompiled when they (or any
header in this directory or ``include/``) are newer than their object.  The
CUDA runtime is linked statically, so the library loads on a machine without
a GPU (the entry points then report that no device is present).
"""

import argparse
import os
import subprocess
import sys
from concurrent.futures import ThreadPoolExecutor

HERE = os.path.dirname(os.path.abspath(__file__))
PKG = os.path.dirname(HERE)
REPO = os.path.dirname(PKG)
BUILD_DIR = os.path.join(HERE, "_build")
LIB_DIR = os.path.join(PKG, "lib")
LIB_PATH = os.path.join(LIB_DIR, "libwxx_cuda.so")
INCLUDE = os.path.join(REPO, "include")

SOURCES = [
    "runtime.cu",
    "elementwise.cu",
    "reduce.cu",
    "gemm.cu",
    "stem.cu",
    "fft.cu",
    "fft_static.cu",
    "hyena_filter.cu",
    "attention.cu",
    "generate.cu",
    "train.cu",
    "pool.cu",
    "nccl.cu",
]

ARCH_FLAGS = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = ARCH_FLAGS + [
    "-O3",
    "-lineinfo",
    "-std=c++17",
    "-Xcompiler",
    "-fPIC,-fvisibility=hidden",
    "-I" + INCLUDE,
    "-I" + HERE,
]


def _nvcc():
    cand = os.path.join(os.environ.get("CUDA_HOME", "/usr/local/cuda"), "bin", "nvcc")
    return cand if os.path.exists(cand) else "nvcc"


def _headers():
    out = []
    for d in (HERE, INCLUDE):
        for name in os.listdir(d):
            if name.endswith((".cuh", ".h", ".hpp")):
                out.append(os.path.join(d, name))
    return out


def _stale(src, obj, headers):
    if not os.path.exists(obj):
        return True
    t = os.path.getmtime(obj)
    return os.path.getmtime(src) > t or any(os.path.getmtime(h) > t for h in headers)


def build(force=False, jobs=None, verbose=False):
    """Compiles stale sources and relinks the library; returns its path."""
    os.makedirs(BUILD_DIR, exist_ok=True)
    os.makedirs(LIB_DIR, exist_ok=True)
    nvcc = _nvcc()
    headers = _headers()
    todo = []
    objs = []
    for src in SOURCES:
        path = os.path.join(HERE, src)
        obj = os.path.join(BUILD_DIR, src.replace(".cu", ".o"))
        objs.append(obj)
        if force or _stale(path, obj, headers):
            todo.append((path, obj))

    def compile_one(item):
        path, obj = item
        cmd = [nvcc] + NVCC_FLAGS + ["-c", path, "-o", obj]
        if verbose:
            print(" ".join(cmd), flush=True)
        res = subprocess.run(cmd, capture_output=True, text=True)
        if res.returncode != 0:
            raise RuntimeError(f"nvcc failed for {os.path.basename(path)}:\n{res.stderr}")
        return path

    if todo:
        with ThreadPoolExecutor(max_workers=jobs or min(len(todo), os.cpu_count() or 4)) as ex:
            list(ex.map(compile_one, todo))
    if todo or not os.path.exists(LIB_PATH):
        tmp = LIB_PATH + ".tmp"
        cmd = [nvcc] + ARCH_FLAGS + ["-shared", "-o", tmp] + objs + ["-ldl"]
        res = subprocess.run(cmd, capture_output=True, text=True)
        if res.returncode != 0:
            raise RuntimeError(f"link failed:\n{res.stderr}")
        os.replace(tmp, LIB_PATH)
    return LIB_PATH


def main(argv=None):
    ap = argparse.ArgumentParser(description=__doc__)
    ap.add_argument("--force", action="store_true")
    ap.add_argument("--jobs", type=int, default=None)
    ap.add_argument("-v", "--verbose", action="store_true")
    args = ap.parse_args(argv)
    path = build(force=args.force, jobs=args.jobs, verbose=args.verbose)
    print(path)
    return 0


if __name__ == "__main__":
    sys.exit(main())
