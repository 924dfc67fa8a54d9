"""Builds libcpab_b200.so (the sm_100a kernels and their C ABI) in-tree.

    python fg-cpab_b200/build.py [--force]

The library is written next to the Python package
(fg-cpab_b200/cpab/libcpab_b200.so) so that it ships with the source tree.
nvcc cross-compiles for sm_100a without a GPU.  The CUDA runtime is linked
statically: the library carries its own runtime and shares the primary
context (and therefore streams and graph capture) with the host process.
"""
import os
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
CSRC = os.path.join(HERE, "csrc")
INCLUDE = os.path.join(os.path.dirname(HERE), "include")
OUT_DIR = os.path.join(HERE, "cpab")
LIB_NAME = "libcpab_b200.so"
LIB_PATH = os.path.join(OUT_DIR, LIB_NAME)
OBJ_DIR = os.path.join(HERE, "_build")

SOURCES = ["integrate.cu", "basis.cu", "resample.cu", "capi.cu", "noalloc.cu"]
HEADERS = ["cpab_device.cuh", "launch.h"]

NVCC_FLAGS = [
    "-gencode", "arch=compute_100a,code=sm_100a",
    "-lineinfo", "-O3", "-std=c++17",
    "-Xcompiler", "-fPIC,-O2",
    "-Xptxas", "-warn-spills",
]


def _nvcc():
    for cand in (os.environ.get("NVCC"), "/usr/local/cuda/bin/nvcc", "nvcc"):
        if cand and (os.path.isabs(cand) and os.path.exists(cand) or not os.path.isabs(cand)):
            return cand
    return "nvcc"


def _mtime(path):
    return os.path.getmtime(path) if os.path.exists(path) else -1.0


def build(force=False, verbose=False, extra_flags=()):
    """Compile (if stale) and link the library; returns its path."""
    os.makedirs(OBJ_DIR, exist_ok=True)
    nvcc = _nvcc()
    deps = [os.path.join(CSRC, h) for h in HEADERS] + [os.path.join(INCLUDE, "cpab_b200.h")]
    dep_time = max(_mtime(p) for p in deps)
    objs = []
    for src in SOURCES:
        src_path = os.path.join(CSRC, src)
        obj = os.path.join(OBJ_DIR, src.replace(".cu", ".o"))
        objs.append(obj)
        if force or _mtime(obj) < max(_mtime(src_path), dep_time):
            cmd = [nvcc, *NVCC_FLAGS, *extra_flags, "-I", INCLUDE, "-c", src_path, "-o", obj]
            if verbose:
                print(" ".join(cmd), flush=True)
            subprocess.run(cmd, check=True)
    if force or _mtime(LIB_PATH) < max(_mtime(o) for o in objs):
        tmp = LIB_PATH + ".tmp"
        cmd = [nvcc, "-shared", "-gencode", "arch=compute_100a,code=sm_100a",
               "-cudart", "static", "-Xcompiler", "-fPIC", *objs, "-o", tmp]
        if verbose:
            print(" ".join(cmd), flush=True)
        subprocess.run(cmd, check=True)
        os.replace(tmp, LIB_PATH)
    return LIB_PATH


if __name__ == "__main__":
    path = build(force="--force" in sys.argv, verbose=True,
                 extra_flags=["-Xptxas", "-v"] if "--ptxas-v" in sys.argv else [])
    print(path)
