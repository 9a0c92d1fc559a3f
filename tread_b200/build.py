"""Build the tread_b200 C-ABI library (`tread_b200/_lib/libtread_b200.so`) for sm_100a.

Every `csrc/*.cu` is compiled with nvcc for `sm_100a` only and linked into one shared
library with the CUDA runtime linked statically, so the `.so` has no dependency beyond the
driver. The library is built in-tree so that it travels with the source tree.

    python -m tread_b200.build [-v] [--force]
"""
import argparse
import os
import shutil
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)
CSRC = os.path.join(HERE, "csrc")
OUT_DIR = os.path.join(HERE, "_lib")
OBJ_DIR = os.path.join(ROOT, "_build", "obj")
LIB = os.path.join(OUT_DIR, "libtread_b200.so")

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = ARCH + [
    "-O3", "-lineinfo", "-std=c++17", "-Xcompiler", "-fPIC", "--expt-relaxed-constexpr",
    "-Xptxas", "-warn-spills", "-I", os.path.join(ROOT, "include"),
]


def nvcc():
    path = shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc"
    if not os.path.exists(path):
        raise RuntimeError("nvcc not found: the tread_b200 CUDA library cannot be built")
    return path


def _deps(src):
    headers = [os.path.join(CSRC, f) for f in os.listdir(CSRC) if f.endswith((".cuh", ".h"))]
    headers.append(os.path.join(ROOT, "include", "tread_b200.h"))
    return [src] + headers


def _stale(target, deps):
    if not os.path.exists(target):
        return True
    t = os.path.getmtime(target)
    return any(os.path.getmtime(d) > t for d in deps if os.path.exists(d))


def build(verbose=False, force=False, ptxas_verbose=False):
    os.makedirs(OUT_DIR, exist_ok=True)
    os.makedirs(OBJ_DIR, exist_ok=True)
    srcs = sorted(f for f in os.listdir(CSRC) if f.endswith(".cu"))
    objs = []
    cc = nvcc()
    for f in srcs:
        src = os.path.join(CSRC, f)
        obj = os.path.join(OBJ_DIR, f[:-3] + ".o")
        objs.append(obj)
        if force or _stale(obj, _deps(src)):
            cmd = [cc] + NVCC_FLAGS + (["-Xptxas", "-v"] if ptxas_verbose else []) + ["-c", src, "-o", obj]
            if verbose:
                print(" ".join(cmd), flush=True)
            subprocess.run(cmd, check=True)
    if force or _stale(LIB, objs):
        cmd = [cc] + ARCH + ["-shared", "-cudart", "static", "-o", LIB] + objs
        if verbose:
            print(" ".join(cmd), flush=True)
        subprocess.run(cmd, check=True)
    return LIB


if __name__ == "__main__":
    ap = argparse.ArgumentParser()
    ap.add_argument("-v", "--verbose", action="store_true")
    ap.add_argument("--force", action="store_true")
    ap.add_argument("--ptxas", action="store_true", help="print -Xptxas -v resource usage")
    a = ap.parse_args()
    print(build(verbose=a.verbose, force=a.force, ptxas_verbose=a.ptxas))
    sys.exit(0)
