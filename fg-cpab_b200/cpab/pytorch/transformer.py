"""Differentiable CPA transformation of points (cpab/pytorch/transformer.py of
the reference), backed by libcpab_b200.

Forward:  A = B theta (+ Trels = expm(A / nstepsolver), fused), a counting
          sort of the points by initial cell (processing order only), then
          the integration kernel (closed form in 1D, nstepsolver exact
          per-cell steps in 2D/3D).
Backward: the fused adjoint kernel produces per-cell moments (and the point
          gradient lambda(0) when the points need one), then one sparse
          projection dtheta = B^T vec(moments).  Optionally the projected
          gradient is summed over a process group (points sharded over GPUs).
"""
from dataclasses import dataclass

import numpy as np
import torch

from .. import _ext, _native


@dataclass
class DeviceBasis:
    """CSR copies of B (D x d) and B^T (d x D) on one device, fp32 values.
    ``dense``: more than 4 nonzeros per row of B on average (bases without the
    zero-boundary constraint), whose A-build and projection run on
    transposed operands (build_A / project below)."""
    d: int
    D: int
    rowptr: torch.Tensor
    colidx: torch.Tensor
    vals: torch.Tensor
    t_rowptr: torch.Tensor
    t_colidx: torch.Tensor
    t_vals: torch.Tensor
    dense: bool = False

    @property
    def tensors(self):
        return [self.rowptr, self.colidx, self.vals, self.t_rowptr, self.t_colidx, self.t_vals]


def _csr_arrays(M, device):
    M = M.tocsr()
    M.sort_indices()
    return (torch.from_numpy(M.indptr.astype(np.int32)).to(device),
            torch.from_numpy(M.indices.astype(np.int32)).to(device),
            torch.from_numpy(M.data.astype(np.float32)).to(device))


def device_basis(params, device):
    """B and B^T of ``params.basis`` on ``device``, built once per device.

    (The reference caches its sparse basis for cuda:0 only and rebuilds it
    from scipy on every call for other devices, cpab/pytorch/transformer.py:47-66.)
    """
    cache = params.__dict__.setdefault("_device_basis", {})
    key = (device.type, device.index if device.index is not None else torch.cuda.current_device())
    hit = cache.get(key)
    if hit is None:
        B = params.basis
        r, c, v = _csr_arrays(B, device)
        tr, tc, tv = _csr_arrays(B.T, device)
        hit = DeviceBasis(int(B.shape[1]), int(B.shape[0]), r, c, v, tr, tc, tv,
                          dense=int(B.nnz) > 4 * int(B.shape[0]))
        cache[key] = hit
    return hit


def build_A(ndim, nC, basis, theta, dT=None):
    """As (and Trels when dT is given) for theta [n, d].  A general basis
    spreads every row and column over the whole domain, so its products
    gather scattered entries; there theta goes in transposed, which makes the
    entries of all transformations at one basis column one contiguous load."""
    if basis.dense:
        return _native.build_A_tt(ndim, nC, basis, theta.t().contiguous(), theta.shape[0], dT)
    return _native.build_A(ndim, nC, basis, theta, dT)


def project(basis, moments):
    """dtheta [n, d] = B^T vec(moments[n]) (moments transposed for general bases)."""
    if basis.dense:
        n = moments.shape[0]
        return _native.project_tt(basis, moments.reshape(n, -1).t().contiguous(), n)
    return _native.project(basis, moments)


def _get_sparse_basis(params, device, dtype=torch.float32):
    """B as a coalesced torch sparse COO tensor on `device` (the helper of the
    reference's transformer module, cpab/pytorch/transformer.py:47-66, kept for
    code that uses it; the kernels here read the CSR copy of device_basis).
    Like the reference, the cuda:0 float32 copy is kept in
    params.basis_gpu_sparse and its transpose in params.basis_gpu_sparse_t."""
    device = torch.device(device)
    cached = getattr(params, "basis_gpu_sparse", None)
    if cached is not None and cached.device == device and cached.dtype == dtype:
        return cached
    coo = params.basis.tocoo()
    idx = torch.stack((torch.from_numpy(coo.row.astype(np.int64)),
                       torch.from_numpy(coo.col.astype(np.int64)))).to(device)
    with torch.sparse.check_sparse_tensor_invariants(enable=True):  # O(nnz), once per device
        B = torch.sparse_coo_tensor(idx, torch.from_numpy(coo.data).to(device=device, dtype=dtype),
                                    size=params.basis.shape, device=device, dtype=dtype).coalesce()
    if device.type == "cuda" and device.index in (None, 0) and dtype == torch.float32:
        params.basis_gpu_sparse = B
        params.basis_gpu_sparse_t = B.transpose(0, 1).coalesce()
    return B


def CPAB_transformer(points, theta, params, compute_points_grad=False):
    """Transform points through the CPA velocity field given by theta.

    Arguments:
        points: [ndim, n_points] or [n_batch, ndim, n_points] CUDA tensor
        theta: [n_batch, d] CUDA tensor of transformation parameters
        params: parameter object from Cpab
        compute_points_grad: bool, return a gradient for the points in backward

    Returns:
        transformed_points: [n_batch, ndim, n_points]
    """
    assert points.is_cuda and theta.is_cuda, "Only GPU tensors supported"
    assert params.ndim in (1, 2, 3), "GPU transformer supports 1D, 2D, and 3D"
    assert type(compute_points_grad) == bool, "compute_points_grad must be bool"
    return transform(points, theta, params, compute_points_grad, None)


def _allreduce_grad(group):
    def hook(g):
        g = g.contiguous().clone()
        torch.distributed.all_reduce(g, group=group)
        return g
    return hook


def transform(points, theta, params, compute_points_grad=False, group=None):
    """The transform_grid autograd node: the C++ one (_cpab_ext) when it is
    built, else _CPABFunction; both issue the same C ABI calls.  With a
    process group, dtheta is summed over the group once per backward: for the
    C++ node by a gradient hook on an identity view of theta, so that exactly
    this node's contribution is reduced (as _CPABFunction's backward does)."""
    ext = _ext.module()
    if ext is None:
        return _CPABFunction.apply(points, theta, params, compute_points_grad, group)
    batched, _ = _layout(points, theta, params)
    if theta.dtype != torch.float32 or points.dtype != torch.float32:
        raise TypeError("points and theta must be float32")
    basis = device_basis(params, theta.device)
    points_c = points.contiguous()
    if group is not None and theta.requires_grad:
        theta = theta.view_as(theta)
        theta.register_hook(_allreduce_grad(group))
    return _ext.call(ext.transform, points_c, theta, basis.tensors, basis.d, basis.dense,
                     _nc(params), int(params.nstepsolver),
                     bool(getattr(params, "adaptive_substeps", False)),
                     _order(params, points_c, batched), compute_points_grad, batched)


def _layout(points, theta, params):
    """Validate shapes; returns (batched, nP)."""
    nd = params.ndim
    n_theta = theta.shape[0]
    if theta.dim() != 2 or theta.shape[1] != params.d:
        raise ValueError("theta must be [n_batch, %d], got %s" % (params.d, tuple(theta.shape)))
    if points.device != theta.device:
        raise ValueError("points on %s, theta on %s" % (points.device, theta.device))
    if points.dim() == 2:
        if points.shape[0] != nd:
            raise ValueError("points must be [%d, n_points], got %s" % (nd, tuple(points.shape)))
        return False, points.shape[1]
    if points.dim() == 3 and points.shape[0] == n_theta and points.shape[1] == nd:
        return True, points.shape[2]
    raise ValueError("points must be [%d, n_points] or [%d, %d, n_points], got %s"
                     % (nd, n_theta, nd, tuple(points.shape)))


def _nc(params):
    return [int(c) for c in params.nc]


# Below this many points per set the kernels take the points in storage order.
ORDER_MIN_POINTS = 4096


def _order(params, points, batched):
    """Processing order of ``points`` (sorted by initial cell), or None.

    The order depends on the points only, and callers usually transform the
    same points (a fixed meshgrid) under changing theta, so the last order is
    kept per device, keyed on the tensor's storage pointer, version counter
    and shape.  A stale hit (a new tensor at a reused address) is harmless:
    results never depend on the processing order, which is always a
    permutation of the right size.

    Under CUDA graph capture the sort is always recorded into the graph (a
    replay may see new point values in the same buffer) and nothing is
    cached: captured kernels have not run yet, so the order's contents are
    only defined inside the graph's replays.
    """
    nP = points.shape[-1]
    # 1D: few cells, so a sorted warp would funnel all its lanes into the same
    # shared-memory moment counters (compare-and-swap retries); storage order
    # measured 17% faster per step there.
    if nP < ORDER_MIN_POINTS or params.ndim == 1:
        return None
    if torch.cuda.is_current_stream_capturing():
        return _native.order_points(_nc(params), points, batched)
    cache = params.__dict__.setdefault("_order_cache", {})
    key = (points.data_ptr(), points._version, tuple(points.shape), bool(batched),
           tuple(_nc(params)))
    hit = cache.get(points.device)
    if hit is not None and hit[0] == key:
        return hit[1]
    order = _native.order_points(_nc(params), points, batched)
    cache[points.device] = (key, order)
    return order


def clear_order_cache(params):
    """Forget the kept point orders, so that the next call sorts its points again."""
    params.__dict__.pop("_order_cache", None)


class _CPABFunction(torch.autograd.Function):
    """A = B theta -> integrate; backward: fused adjoint moments -> B^T projection."""

    @staticmethod
    def forward(ctx, points, theta, params, compute_points_grad=False, group=None):
        batched, _ = _layout(points, theta, params)
        nd = params.ndim
        basis = device_basis(params, theta.device)
        theta_c = theta.contiguous()
        points_c = points.contiguous()
        T = int(params.nstepsolver)
        adaptive = int(bool(getattr(params, "adaptive_substeps", False)))
        dT = None if nd == 1 else 1.0 / T
        As, trels = build_A(nd, int(params.nC), basis, theta_c, dT)
        order = _order(params, points_c, batched)
        out = _native.forward(nd, _nc(params), points_c, batched, trels, As, T, adaptive, order)
        ctx.params = params
        ctx.batched = batched
        ctx.nstepsolver = T
        ctx.adaptive = adaptive
        ctx.compute_points_grad = compute_points_grad
        ctx.group = group
        ctx.order = order
        ctx.save_for_backward(points_c, As)
        return out

    @staticmethod
    @torch.autograd.function.once_differentiable
    def backward(ctx, grad):
        points, As = ctx.saved_tensors
        params = ctx.params
        want_points = ctx.compute_points_grad and ctx.needs_input_grad[0]
        moments, grad_points = _native.backward(
            params.ndim, _nc(params), points, ctx.batched, As, grad.contiguous(),
            ctx.nstepsolver, ctx.adaptive, want_points, ctx.order)
        if grad_points is not None and points.dim() == 2:
            grad_points = grad_points.sum(dim=0)
        grad_theta = None
        if ctx.needs_input_grad[1]:
            grad_theta = project(device_basis(params, As.device), moments)
            if ctx.group is not None:
                torch.distributed.all_reduce(grad_theta, group=ctx.group)
        return grad_points, grad_theta, None, None, None


def transform_chain(points, theta_stages, params, compute_points_grad=False):
    """Fused transform_grid_chain (2D/3D): theta_stages [n_stages, n_batch, d]
    (already scaled), applied in order to points in one kernel each way."""
    assert params.ndim in (2, 3), "the fused chain supports 2D and 3D"
    return _ChainFunction.apply(points, theta_stages, params, compute_points_grad)


class _ChainFunction(torch.autograd.Function):
    """transform_grid_chain (cpab/cpab.py:269-278): the stages' A/Trels from one
    build_A call, one forward kernel through all stages, one backward kernel
    walking the stages back (lambda handed from stage to stage inside it)."""

    @staticmethod
    def forward(ctx, points, theta_stages, params, compute_points_grad=False):
        K, nb, d = theta_stages.shape
        batched, _ = _layout(points, theta_stages[0], params)
        nd = params.ndim
        basis = device_basis(params, theta_stages.device)
        T = int(params.nstepsolver)
        adaptive = int(bool(getattr(params, "adaptive_substeps", False)))
        points_c = points.contiguous()
        As, trels = build_A(nd, int(params.nC), basis,
                                    theta_stages.reshape(K * nb, d).contiguous(), 1.0 / T)
        order = _order(params, points_c, batched)
        out, sp = _native.forward_chain(nd, _nc(params), points_c, batched, trels, As, K, T,
                                        adaptive, order)
        ctx.params, ctx.batched, ctx.T, ctx.adaptive = params, batched, T, adaptive
        ctx.K, ctx.order, ctx.compute_points_grad = K, order, compute_points_grad
        ctx.save_for_backward(points_c, As, sp)
        return out

    @staticmethod
    @torch.autograd.function.once_differentiable
    def backward(ctx, grad):
        points, As, sp = ctx.saved_tensors
        params = ctx.params
        want_points = ctx.compute_points_grad and ctx.needs_input_grad[0]
        moments, grad_points = _native.backward_chain(
            params.ndim, _nc(params), points, ctx.batched, As, ctx.K, grad.contiguous(), sp,
            ctx.T, ctx.adaptive, want_points, ctx.order)
        if grad_points is not None and points.dim() == 2:
            grad_points = grad_points.sum(dim=0)
        grad_theta = None
        if ctx.needs_input_grad[1]:
            grad_theta = project(device_basis(params, As.device), moments)
            grad_theta = grad_theta.reshape(ctx.K, -1, grad_theta.shape[-1])
        return grad_points, grad_theta, None, None
