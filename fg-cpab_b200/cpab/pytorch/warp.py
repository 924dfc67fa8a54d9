"""The CPAB spatial-transformer warp: the CpabWarp layer of the reference's
stn/stn.py:58-86, with the integration and F.grid_sample fused.

CpabWarp(tess)(x, theta) resamples x [B, C, *spatial] on its own pixel grid
mapped through T_1 o ... o T_K (theta a [B, d] tensor for one transformation,
or a list / [K, B, d] tensor of them, T_K acting first), exactly as the
reference's layer does: the pixel centres sit at linspace(-1, 1, n) per axis
(stn/stn.py:43-46), CPAB coordinate i runs along x.shape[2 + i] on the domain
[0, 1] (stn/stn.py:80-86), and the image is sampled with
F.grid_sample(align_corners=True, padding_mode) (stn/stn.py:48-54).

In 2D and 3D the K integrations and the sampling run in one kernel each way
(cpab_b200_warp / cpab_b200_warp_backward, called from the C++ autograd node
of _cpab_ext when it is built, else from _Warp): the pixel grid, the intermediate
grids and the grid gradient never pass through memory as separate tensors,
and the backward starts the adjoint sweep from the sampling gradient held in
registers.  1D (grid_sample has no 1D mode: the reference samples a
[B, C, 1, W] image) keeps the reference's composition on this package's
transformer.
"""
import torch
import torch.nn as nn
import torch.nn.functional as F

from .. import _ext, _native
from ..cpab import Cpab
from .transformer import CPAB_transformer, _nc, build_A, device_basis, project

PADDING_MODES = {"zeros": 0, "border": 1, "reflection": 2}


def pixel_axes(size, device):
    """The pixel centres of each axis in CPAB coordinates: (linspace(-1, 1, n)
    + 1) / 2, a one-pixel axis at 0.5.  The same torch operations as the
    reference's grid (stn/stn.py:46 and :82), so the values are identical."""
    f32 = dict(device=device, dtype=torch.float32)
    return [((torch.linspace(-1, 1, n, **f32) if n > 1 else torch.zeros(1, **f32)) + 1) / 2
            for n in size]


def _pixel_mesh(params, size, device):
    """(axes, order) of the pixel grid of `size`, cached per params/device.
    order lists the pixels sorted by the cell they start in (as for
    transform_data: a warp's lanes then share cells, table rows and moment
    rows).  A miss under CUDA graph capture is not cached."""
    cache = params.__dict__.setdefault("_warp_mesh", {})
    key = (tuple(int(s) for s in size), str(device))
    hit = cache.get(key)
    if hit is None:
        capturing = torch.cuda.is_current_stream_capturing()
        lin = pixel_axes(size, device)
        axes = torch.cat(lin).contiguous()
        mesh = torch.meshgrid(*lin, indexing="ij")  # output order: last axis fastest
        pts = torch.stack([g.reshape(-1) for g in mesh]).contiguous()
        order = _native.order_points(_nc(params), pts, False)[0].contiguous()
        hit = (axes, order)
        if not capturing:
            cache[key] = hit
    return hit


def warp(x, thetas, params, padding_mode="zeros"):
    """Fused 2D/3D warp: out[b] = grid_sample(x[b], T_1 o ... o T_K(pixel grid),
    align_corners=True, padding_mode) for thetas = [theta_1, ..., theta_K],
    each [B, d] float32; x float32 [B, C, *spatial].  Differentiable in every
    theta and in x.  An x expanded along the batch (stride 0, e.g.
    template.expand(B, ...)) is read as the one image it is."""
    nd = params.ndim
    if nd not in (2, 3):
        raise ValueError("the fused warp supports 2D and 3D")
    if padding_mode not in PADDING_MODES:
        raise ValueError("padding_mode must be one of %s, got %r"
                         % (sorted(PADDING_MODES), padding_mode))
    if x.dim() != nd + 2:
        raise ValueError("expected a %dD input [B, C, *spatial], got %s" % (nd, tuple(x.shape)))
    thetas = list(thetas)
    if not thetas:
        raise ValueError("at least one theta is needed")
    B = thetas[0].shape[0]
    for th in thetas:
        if th.dim() != 2 or th.shape[0] != B or th.shape[1] != params.d:
            raise ValueError("each theta must be [B, %d] with the same B" % params.d)
        if th.device != x.device:
            raise ValueError("theta on %s, x on %s" % (th.device, x.device))
    if x.shape[0] != B:
        raise ValueError("x holds %d images for %d transformations" % (x.shape[0], B))
    data = x[:1] if B > 1 and x.stride(0) == 0 else x
    size = tuple(int(s) for s in x.shape[2:])
    ext = _ext.module()
    if ext is None:
        return _Warp.apply(data, params, size, PADDING_MODES[padding_mode], *thetas)
    basis = device_basis(params, x.device)
    axes, order = _pixel_mesh(params, size, x.device)
    return _ext.call(ext.warp, data, thetas, basis.tensors, basis.d, basis.dense, _nc(params),
                     int(params.nstepsolver), bool(getattr(params, "adaptive_substeps", False)),
                     axes, order, PADDING_MODES[padding_mode])


def warp_composed(x, thetas, params, padding_mode="zeros"):
    """The reference layer's composition, step by step (stn/stn.py:40-54 with
    CpabWarp.transform, :79-86): the pixel grid in [-1, 1], one
    CPAB_transformer call per theta (the last first), then F.grid_sample;
    1D samples a [B, C, 1, W] image at y = 0.  The 1D path of CpabWarp, and
    the unfused baseline of warp() in 2D and 3D."""
    size = x.shape[2:]
    f32 = dict(device=x.device, dtype=torch.float32)
    axes = [torch.linspace(-1, 1, n, **f32) if n > 1 else torch.zeros(1, **f32) for n in size]
    points = torch.stack(torch.meshgrid(*axes, indexing="ij")[::-1]).flatten(1)  # (x, y, z)
    points = (points.flip(-2) + 1) / 2          # CPAB coordinates on [0, 1]
    for theta in reversed(list(thetas)):
        points = CPAB_transformer(points, theta, params, points.requires_grad)
    grid = (points * 2 - 1).flip(-2).transpose(1, 2).reshape(len(points), *size, -1)
    if len(size) == 1:
        out = F.grid_sample(x.unsqueeze(2), F.pad(grid, (0, 1)).unsqueeze(1),
                            align_corners=True, padding_mode=padding_mode)
        return out.squeeze(2)
    return F.grid_sample(x, grid, align_corners=True, padding_mode=padding_mode)


class _Warp(torch.autograd.Function):
    """The chain of K transformations runs stage 0 first, so the stages are
    thetas reversed (the STN's T_K acts first); A/Trels of all K*B rows come
    from one build_A call, stage-major."""

    @staticmethod
    def forward(ctx, data, params, size, padding, *thetas):
        nd, K = params.ndim, len(thetas)
        B, d = thetas[0].shape
        T = int(params.nstepsolver)
        adaptive = int(bool(getattr(params, "adaptive_substeps", False)))
        stages = torch.stack([th.contiguous() for th in reversed(thetas)]).reshape(K * B, d)
        basis = device_basis(params, stages.device)
        As, trels = build_A(nd, int(params.nC), basis, stages.contiguous(), 1.0 / T)
        axes, order = _pixel_mesh(params, size, stages.device)
        data_c = data.contiguous()
        out, grid_t, sp = _native.warp(nd, _nc(params), size, axes, trels, As, K, T, adaptive,
                                       data_c, padding, order)
        ctx.params, ctx.size, ctx.padding, ctx.T, ctx.adaptive = params, size, padding, T, adaptive
        ctx.K, ctx.B, ctx.order = K, B, order
        ctx.save_for_backward(data_c, As, grid_t, sp, axes)
        return out

    @staticmethod
    @torch.autograd.function.once_differentiable
    def backward(ctx, grad):
        data, As, grid_t, sp, axes = ctx.saved_tensors
        K = ctx.K
        want_data = ctx.needs_input_grad[0]
        want_theta = any(ctx.needs_input_grad[4:])
        if not (want_data or want_theta):
            return (None,) * (4 + K)
        params = ctx.params
        moments, gd = _native.warp_backward(
            params.ndim, _nc(params), ctx.size, axes, As, K, ctx.T, ctx.adaptive, data,
            ctx.padding, sp, grid_t, grad.contiguous(), want_data, ctx.order)
        grads = [None] * K
        if want_theta:
            g = project(device_basis(params, As.device), moments).reshape(K, ctx.B, -1)
            grads = [g[K - 1 - i] for i in range(K)]  # theta_i ran as stage K-1-i
        return (gd, None, None, None, *grads)


class CpabWarp(nn.Module):
    """Drop-in for the reference's stn.CpabWarp (stn/stn.py:58-86): same
    constructor (tess_size, zero_boundary=True, nstepsolver=50,
    padding_mode="zeros", **cpab_kwargs for cpab.Cpab), attributes (ndim,
    padding_mode, cpab, theta_dim) and calls (forward(x, theta),
    transform(points, thetas)).  The output has x's shape and dtype; the
    warp is computed in float32 whatever the autocast state, as there."""

    def __init__(self, tess_size, zero_boundary=True, nstepsolver=50, padding_mode="zeros",
                 **cpab_kwargs):
        super().__init__()
        tess_size = [int(t) for t in tess_size]
        assert len(tess_size) in (1, 2, 3), "only 1D, 2D and 3D inputs are supported"
        self.ndim, self.padding_mode = len(tess_size), padding_mode
        self.cpab = Cpab(tess_size, zero_boundary=zero_boundary, **cpab_kwargs)
        self.cpab.set_solver_params(nstepsolver)
        self.theta_dim = self.cpab.get_theta_dim()

    def transform(self, points, thetas):
        """points [ndim, P] in [-1, 1], grid_sample's (x, y, z) order, mapped
        through T_1 o ... o T_K (thetas[-1] first); returns [B, ndim, P]."""
        points = (points.flip(-2) + 1) / 2  # grid (x, y, z) -> CPAB coordinates on [0, 1]
        for theta in reversed(thetas):
            points = CPAB_transformer(points, theta, self.cpab.params, points.requires_grad)
        return (points * 2 - 1).flip(-2)

    def forward(self, x, theta):
        size = x.shape[2:]
        assert len(size) == self.ndim, \
            f"expected a {self.ndim}D input [B, C, *spatial], got {tuple(x.shape)}"
        thetas = [theta] if torch.is_tensor(theta) and theta.dim() == 2 else list(theta)
        with torch.autocast(x.device.type, enabled=False):
            thetas = [th.float() for th in thetas]
            fn = warp if self.ndim > 1 else warp_composed
            out = fn(x.float(), thetas, self.cpab.params, self.padding_mode)
        return out.to(x.dtype)
