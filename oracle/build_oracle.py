"""Build recipe for the oracle (test infrastructure only).

    python oracle/build_oracle.py            # liboracle.so (the C restatement)
    python oracle/build_oracle.py --ref      # also oracle/_ref/libcpab_ref.so

liboracle.so: gcc, -O2 -mfma -ffp-contract=off -fopenmp, so fmaf() is one
fused instruction (like __fmaf_rn) and no other expression is contracted.

oracle/_ref/libcpab_ref.so: the reference's own CUDA kernels
(cpab/core/cpab_ops_{1,2,3}d.cu, compiled where they lie, unmodified) linked
with ref_shim.cu, a C ABI that launches them with the reference's launch
geometry (cpab/pytorch/transformer_cuda.cu).  Built only when the reference
tree is present; the .so then travels with the repository to the GPU box,
where it serves as a second, GPU-side oracle.
"""
import os
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
# The reference checkout: $CPAB_REFERENCE, else a sibling of this repository
# named "reference".
REF_ROOT = os.path.normpath(os.environ.get(
    "CPAB_REFERENCE", os.path.join(os.path.dirname(HERE), os.pardir, "reference")))
REF_CORE = os.environ.get("CPAB_REFERENCE_CORE", os.path.join(REF_ROOT, "cpab", "core"))
REF_DIR = os.path.join(HERE, "_ref")


def _stale(target, deps):
    if not os.path.exists(target):
        return True
    t = os.path.getmtime(target)
    return any(os.path.getmtime(d) > t for d in deps if os.path.exists(d))


def build_oracle(force=False):
    src = os.path.join(HERE, "cpab_oracle.c")
    out = os.path.join(HERE, "liboracle.so")
    if force or _stale(out, [src, __file__]):
        tmp = out + ".tmp"
        subprocess.run(["gcc", "-O2", "-mfma", "-ffp-contract=off", "-fopenmp", "-fPIC",
                        "-shared", src, "-o", tmp, "-lm"], check=True)
        os.replace(tmp, out)
    return out


def build_ref(force=False):
    """Compile the reference kernels + shim; returns the .so path or None."""
    sources = [os.path.join(REF_CORE, f) for f in
               ("cpab_ops_1d.cu", "cpab_ops_2d.cu", "cpab_ops_3d.cu")]
    if not all(os.path.exists(s) for s in sources):
        return None
    shim = os.path.join(HERE, "ref_shim.cu")
    out = os.path.join(REF_DIR, "libcpab_ref.so")
    if not (force or _stale(out, sources + [shim, __file__])):
        return out
    os.makedirs(REF_DIR, exist_ok=True)
    objs = []
    flags = ["-gencode", "arch=compute_100a,code=sm_100a", "-O3", "-Xcompiler", "-fPIC",
             "-I", REF_CORE]
    for s in sources + [shim]:
        o = os.path.join(REF_DIR, os.path.basename(s).replace(".cu", ".o"))
        subprocess.run(["nvcc", *flags, "-c", s, "-o", o], check=True)
        objs.append(o)
    tmp = out + ".tmp"
    subprocess.run(["nvcc", "-shared", "-gencode", "arch=compute_100a,code=sm_100a",
                    "-cudart", "static", *objs, "-o", tmp], check=True)
    os.replace(tmp, out)
    return out


if __name__ == "__main__":
    print(build_oracle(force="--force" in sys.argv))
    if "--ref" in sys.argv:
        print(build_ref(force="--force" in sys.argv))
