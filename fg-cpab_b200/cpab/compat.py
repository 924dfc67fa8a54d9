"""Stand-in for the reference's JIT-built ``cpab_gpu`` extension module.

The reference's cpab/pytorch/transformer.py:10-21 compiles five native
functions with torch.utils.cpp_extension (bound at
cpab/pytorch/transformer_cuda.cpp:171-178).  ``cpab_gpu`` below offers the
same five functions -- same arguments, shapes, output allocation
(``torch.zeros`` on the current CUDA device) and RuntimeError on bad input --
implemented over libcpab_b200's C ABI, so that the reference's transformer.py
can switch backends by replacing its ``load(...)`` call with an import of
this module.  The module also works when loaded by file path from
another package (it then loads _native.py next to it the same way), so the
reference's own ``cpab`` package can use it without a name clash.
"""
import os

import torch

try:
    from . import _native
except ImportError:  # loaded by file path, outside this package
    import importlib.util as _util
    _spec = _util.spec_from_file_location(
        "cpab_b200_native", os.path.join(os.path.dirname(os.path.abspath(__file__)), "_native.py"))
    _native = _util.module_from_spec(_spec)
    _spec.loader.exec_module(_native)


def _check_input(t, name):
    if not t.is_cuda:
        raise RuntimeError(name + " must be a CUDA tensor")
    if not t.is_contiguous():
        raise RuntimeError(name + " must be contiguous")


def _nc(ndim, ncx, ncy, nC):
    """Cells per axis; ncz is inferred from nC as the reference does
    (cpab/pytorch/transformer_cuda.cu:65-75)."""
    if ndim == 1:
        return [ncx]
    if ndim == 2:
        return [ncx, ncy]
    per_z = 5 * ncx * ncy
    if per_z <= 0:
        raise RuntimeError("Invalid ncx/ncy for 3D: %d x %d" % (ncx, ncy))
    if nC % per_z != 0:
        raise RuntimeError("Could not infer ncz from nC=%d, ncx=%d, ncy=%d" % (nC, ncx, ncy))
    return [ncx, ncy, nC // per_z]


def _layout(points, batch):
    broadcast = points.dim() == 3 and points.size(0) == batch
    ndim = points.size(1) if broadcast else points.size(0)
    nP = points.size(2) if broadcast else points.size(1)
    return broadcast, ndim, nP


class _CpabGpu:
    """forward / forward_1d_closed_form / backward_moments /
    backward_moments_and_points / expm with the reference's signatures."""

    @staticmethod
    def forward(points_in, trels_in, As_in, nstepsolver, ncx, ncy, adaptive_substeps):
        """cpab/pytorch/transformer_cuda.cpp:32-61."""
        for t, n in ((points_in, "points_in"), (trels_in, "trels_in"), (As_in, "As_in")):
            _check_input(t, n)
        if tuple(As_in.shape) != tuple(trels_in.shape):
            raise RuntimeError("As_in shape mismatch")
        if adaptive_substeps not in (0, 1):
            raise RuntimeError("adaptive_substeps must be 0 or 1")
        batch = trels_in.size(0)
        broadcast, ndim, nP = _layout(points_in, batch)
        nc = _nc(ndim, ncx, ncy, trels_in.size(1))
        out = _native.forward(ndim, nc, points_in, broadcast, trels_in, As_in, nstepsolver,
                              adaptive_substeps)
        return out

    @staticmethod
    def forward_1d_closed_form(points_in, As_in, ncx):
        """cpab/pytorch/transformer_cuda.cpp:66-85."""
        _check_input(points_in, "points_in")
        _check_input(As_in, "As_in")
        if As_in.dim() != 4 or As_in.size(2) != 1 or As_in.size(3) != 2:
            raise RuntimeError("As_in must have affine 1D shape [batch, nC, 1, 2]")
        broadcast, ndim, nP = _layout(points_in, As_in.size(0))
        if ndim != 1:
            raise RuntimeError("points_in must be 1D for forward_1d_closed_form")
        return _native.forward(1, [ncx], points_in, broadcast, None, As_in, 1, 0)

    @staticmethod
    def _backward(points_in, As_in, grad_output_in, nstepsolver, ncx, ncy, adaptive_substeps,
                  want_points):
        for t, n in ((points_in, "points_in"), (As_in, "As_in"), (grad_output_in, "grad")):
            _check_input(t, n)
        if adaptive_substeps not in (0, 1):
            raise RuntimeError("adaptive_substeps must be 0 or 1")
        ndim = As_in.size(2)
        if grad_output_in.size(1) != ndim:
            raise RuntimeError("grad_output ndim mismatch")
        broadcast = points_in.dim() == 3 and points_in.size(0) == As_in.size(0)
        nc = _nc(ndim, ncx, ncy, As_in.size(1))
        return _native.backward(ndim, nc, points_in, broadcast, As_in, grad_output_in,
                                nstepsolver, adaptive_substeps, want_points)

    @staticmethod
    def backward_moments(points_in, As_in, grad_output_in, nstepsolver, ncx, ncy,
                         adaptive_substeps):
        """cpab/pytorch/transformer_cuda.cpp:92-116: moments [n_theta, nC, ppc]."""
        return _CpabGpu._backward(points_in, As_in, grad_output_in, nstepsolver, ncx, ncy,
                                  adaptive_substeps, False)[0]

    @staticmethod
    def backward_moments_and_points(points_in, As_in, grad_output_in, nstepsolver, ncx, ncy,
                                    adaptive_substeps):
        """cpab/pytorch/transformer_cuda.cpp:122-153: [moments, grad_points]."""
        m, gp = _CpabGpu._backward(points_in, As_in, grad_output_in, nstepsolver, ncx, ncy,
                                   adaptive_substeps, True)
        return [m, gp]

    @staticmethod
    def expm(As_in, dT):
        """cpab/pytorch/transformer_cuda.cpp:159-170: [n, ndim, ndim+1] -> same."""
        _check_input(As_in, "As_in")
        ndim = As_in.size(1)
        if ndim not in (1, 2, 3) or As_in.size(2) != ndim + 1:
            raise RuntimeError("As_in must be affine with shape [n, ndim, ndim+1]")
        return _native.expm(As_in, dT)


cpab_gpu = _CpabGpu()
