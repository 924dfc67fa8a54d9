"""Builds libcpab_b200.so (the sm_100a kernels and their C ABI) in-tree.

    python fg-cpab_b200/build.py [--force] [--ptxas-v] [-DNAME=VALUE ... --out PATH]

-D options set compile-time choices of the kernels (e.g. -DCPAB_MOMENT_FLUSH=1,
see csrc/cpab_device.cuh); such a variant is built into its own object
directory and written to --out (load it with CPAB_B200_LIB=PATH).

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

SOURCES = ["integrate.cu", "warp.cu", "basis.cu", "resample.cu", "capi.cu", "noalloc.cu"]
HEADERS = ["cpab_device.cuh", "integrate_body.cuh", "launch.h", "resample_device.cuh"]

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


def build(force=False, verbose=False, extra_flags=(), out=None):
    """Compile (if stale) and link the library; returns its path.  With
    `out`, objects go to a directory of their own beside it."""
    lib_path = LIB_PATH if out is None else os.path.abspath(out)
    obj_dir = OBJ_DIR if out is None else lib_path + ".objs"
    os.makedirs(obj_dir, exist_ok=True)
    nvcc = _nvcc()
    deps = [os.path.join(CSRC, h) for h in HEADERS] + [os.path.join(INCLUDE, "cpab_b200.h")]
    dep_time = max(_mtime(p) for p in deps)
    objs, cmds = [], []
    for src in SOURCES:
        src_path = os.path.join(CSRC, src)
        obj = os.path.join(obj_dir, src.replace(".cu", ".o"))
        objs.append(obj)
        if force or _mtime(obj) < max(_mtime(src_path), dep_time):
            cmds.append([nvcc, *NVCC_FLAGS, *extra_flags, "-I", INCLUDE, "-c", src_path, "-o", obj])
    # The translation units are independent: compile them side by side (the
    # two integration units take most of the time).
    procs = []
    for cmd in cmds:
        if verbose:
            print(" ".join(cmd), flush=True)
        procs.append((cmd, subprocess.Popen(cmd)))
    failed = [cmd for cmd, p in procs if p.wait() != 0]
    if failed:
        raise subprocess.CalledProcessError(1, failed[0])
    if force or _mtime(lib_path) < max(_mtime(o) for o in objs):
        tmp = lib_path + ".tmp"
        cmd = [nvcc, "-shared", "-gencode", "arch=compute_100a,code=sm_100a",
               "-cudart", "static", "-Xcompiler", "-fPIC", *objs, "-o", tmp]
        if verbose:
            print(" ".join(cmd), flush=True)
        subprocess.run(cmd, check=True)
        os.replace(tmp, lib_path)
    return lib_path


EXT_NAME = "_cpab_ext"
EXT_PATH = os.path.join(OUT_DIR, EXT_NAME + ".so")
EXT_SRC = os.path.join(CSRC, "torch_ext.cpp")


def build_ext(force=False, verbose=False):
    """Compile the C++ autograd node (csrc/torch_ext.cpp, host code only) into
    cpab/_cpab_ext.so against this Python's torch, linked to libcpab_b200.so
    (found next to it at run time).  Returns its path."""
    import sysconfig

    import torch
    from torch.utils import cpp_extension

    lib = build(verbose=verbose)
    if not (force or _mtime(EXT_PATH) < max(_mtime(EXT_SRC), _mtime(lib), _mtime(__file__),
                                           _mtime(os.path.join(INCLUDE, "cpab_b200.h")))):
        return EXT_PATH
    cuda_home = cpp_extension.CUDA_HOME or "/usr/local/cuda"
    incs = cpp_extension.include_paths() + [sysconfig.get_paths()["include"], INCLUDE,
                                            os.path.join(cuda_home, "include")]
    libdirs = cpp_extension.library_paths()
    abi = int(torch._C._GLIBCXX_USE_CXX11_ABI)
    tmp = EXT_PATH + ".tmp"
    cmd = (["g++", "-O2", "-std=c++17", "-fPIC", "-shared", EXT_SRC, "-o", tmp,
            "-D_GLIBCXX_USE_CXX11_ABI=%d" % abi, "-DTORCH_EXTENSION_NAME=" + EXT_NAME,
            "-DTORCH_API_INCLUDE_EXTENSION_H", "-Wno-deprecated-declarations"]
           + ["-I" + i for i in incs] + ["-L" + d for d in libdirs]
           + ["-L" + OUT_DIR, "-lcpab_b200", "-lc10", "-lc10_cuda", "-ltorch", "-ltorch_cpu",
              "-ltorch_cuda", "-ltorch_python", "-Wl,-rpath,$ORIGIN"])
    if verbose:
        print(" ".join(cmd), flush=True)
    subprocess.run(cmd, check=True)
    os.replace(tmp, EXT_PATH)
    return EXT_PATH


if __name__ == "__main__":
    args = sys.argv[1:]
    defines = [a for a in args if a.startswith("-D")]
    out = args[args.index("--out") + 1] if "--out" in args else None
    if defines and out is None:
        sys.exit("a -D variant needs --out PATH (the default library keeps the default choices)")
    flags = (["-Xptxas", "-v"] if "--ptxas-v" in args else []) + defines
    path = build(force="--force" in args, verbose=True, extra_flags=flags, out=out)
    print(path)
    if out is None and "--no-ext" not in args:
        print(build_ext(force="--force" in args, verbose=True))
