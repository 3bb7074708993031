"""Build libkd_attn.so in-tree (kandinsky.cpp_b200/kd_attn/libkd_attn.so).

nvcc compiles every csrc/*.cu for sm_100a only (-gencode arch=compute_100a,
code=sm_100a) and links one shared library with a static CUDA runtime.
Run directly (python kandinsky.cpp_b200/build.py) or through
__graft_entry__.build().
"""
import concurrent.futures as cf
import glob
import os
import shutil
import subprocess
import sys

PKG = os.path.dirname(os.path.abspath(__file__))
CSRC = os.path.join(PKG, "csrc")
INCLUDE = os.path.join(os.path.dirname(PKG), "include")
OUT_DIR = os.path.join(PKG, "kd_attn")
LIB = os.path.join(OUT_DIR, "libkd_attn.so")
OBJ_DIR = os.path.join(PKG, "_build")

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
FLAGS = ["-O3", "-lineinfo", "-std=c++17", "-Xcompiler", "-fPIC", "-Xcompiler", "-Wall",
         "--expt-relaxed-constexpr", "-I", INCLUDE]


def nvcc():
    cand = shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc"
    if not os.path.exists(cand):
        raise RuntimeError("nvcc not found: libkd_attn needs the CUDA toolkit to build")
    return cand


def _deps():
    return sorted(glob.glob(os.path.join(CSRC, "*"))) + [os.path.join(INCLUDE, "kd_attn.h"), __file__]


def stale():
    if not os.path.exists(LIB):
        return True
    t = os.path.getmtime(LIB)
    return any(os.path.getmtime(d) > t for d in _deps())


def _compile(src, verbose):
    obj = os.path.join(OBJ_DIR, os.path.basename(src) + ".o")
    cmd = [nvcc()] + ARCH + FLAGS + ["-c", src, "-o", obj]
    if verbose:
        print(" ".join(cmd), flush=True)
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"nvcc failed on {src}:\n{r.stdout}\n{r.stderr}")
    return obj


def build(force=False, verbose=False):
    if not force and not stale():
        return LIB
    os.makedirs(OBJ_DIR, exist_ok=True)
    srcs = sorted(glob.glob(os.path.join(CSRC, "*.cu")))
    with cf.ThreadPoolExecutor(max_workers=min(8, len(srcs))) as ex:
        objs = list(ex.map(lambda s: _compile(s, verbose), srcs))
    tmp = LIB + ".tmp"
    cmd = [nvcc()] + ARCH + ["-shared", "-o", tmp] + objs + ["-ldl"]
    if verbose:
        print(" ".join(cmd), flush=True)
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"link failed:\n{r.stdout}\n{r.stderr}")
    os.replace(tmp, LIB)
    return LIB


if __name__ == "__main__":
    print(build(force="--force" in sys.argv, verbose=True))
