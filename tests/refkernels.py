"""ctypes access to oracle/_ref/libcpab_ref.so: the reference's own CUDA
kernels, launched as the reference launches them (test infrastructure).

The kernels run on the legacy default stream, which is torch's default
stream; outputs are allocated with torch.zeros as the reference's launcher
allocates them."""
import ctypes
import os

import torch

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
PATH = os.path.join(ROOT, "oracle", "_ref", "libcpab_ref.so")
_lib = None


def available():
    return os.path.exists(PATH)


def reference_present():
    """True when the reference's kernel sources are on this machine (where
    oracle/build_oracle.py --ref would build oracle/_ref)."""
    import importlib.util
    spec = importlib.util.spec_from_file_location(
        "cpab_oracle_build", os.path.join(ROOT, "oracle", "build_oracle.py"))
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return os.path.exists(os.path.join(mod.REF_CORE, "cpab_ops_2d.cu"))


def require():
    """Skip when the reference kernels cannot exist here (no build, no
    sources: the GPU box without a prebuilt oracle/_ref); fail when the
    sources are present but the build is missing, so that a forgotten build
    does not pass as a silent skip."""
    import pytest
    if available():
        return
    if reference_present():
        pytest.fail("the reference sources are present but oracle/_ref/libcpab_ref.so is not "
                    "built: run python oracle/build_oracle.py --ref")
    pytest.skip("oracle/_ref not built and the reference sources are absent")


def lib():
    global _lib
    if _lib is None:
        L = ctypes.CDLL(PATH)
        i, f, p = ctypes.c_int, ctypes.c_float, ctypes.c_void_p
        L.ref_expm.argtypes = [i, p, i, f, p]
        L.ref_forward.argtypes = [i, i, i, i, p, i, i, p, p, i, i, i, p]
        L.ref_backward.argtypes = [i, i, i, i, i, p, i, i, p, i, p, i, i, p, p]
        _lib = L
    return _lib


def _p(t):
    return ctypes.c_void_p(t.data_ptr() if t is not None else 0)


def _ncxyz(nc):
    nc = list(nc) + [1] * (3 - len(nc))
    return nc[0], nc[1], nc[2]


def expm(As, dT):
    nd = As.shape[-2]
    out = torch.zeros_like(As)
    assert lib().ref_expm(nd, _p(As), As.numel() // (nd * (nd + 1)), dT, _p(out)) == 0
    return out


def forward(nc, points, batched, trels, As, T, adaptive):
    nd = len(nc)
    n_theta = As.shape[0]
    nP = points.shape[-1]
    out = torch.zeros((n_theta, nd, nP), device=As.device)
    nx, ny, nz = _ncxyz(nc)
    assert lib().ref_forward(nd, nx, ny, nz, _p(points), nP, int(batched), _p(trels), _p(As),
                             n_theta, T, int(adaptive), _p(out)) == 0
    return out


def backward(nc, points, batched, As, grad, T, adaptive):
    nd = len(nc)
    n_theta, nC = As.shape[0], As.shape[1]
    nP = points.shape[-1]
    mom = torch.zeros((n_theta, nC, nd * (nd + 1)), device=As.device)
    gp = torch.zeros((n_theta, nd, nP), device=As.device)
    nx, ny, nz = _ncxyz(nc)
    assert lib().ref_backward(nd, nx, ny, nz, nC, _p(points), nP, int(batched), _p(As), n_theta,
                              _p(grad), T, int(adaptive), _p(mom), _p(gp)) == 0
    return mom, gp
