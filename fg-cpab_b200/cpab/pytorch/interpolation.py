"""Linear / bilinear / trilinear resampling on a (warped) grid
(cpab/pytorch/interpolation.py of the reference), one fused kernel each way.

data: [n_batch, n_channels, *in_size]; grid: [n_batch, ndim, prod(outsize)]
with coordinate 0 fastest; output: [n_batch, n_channels, *outsize].  Grid
coordinate k is scaled by in_size[k]-1 and indexes data axis 2+k; corners are
clamped to the border.  Differentiable in grid and data.
"""
import torch

from .. import _native


def interpolate(ndim, data, grid, outsize):
    if ndim not in (1, 2, 3):
        raise ValueError("ndim must be 1, 2 or 3")
    return _Interpolate.apply(data, grid, int(ndim), tuple(int(s) for s in outsize))


def interpolate1D(data, grid, outsize):
    return interpolate(1, data, grid, outsize)


def interpolate2D(data, grid, outsize):
    return interpolate(2, data, grid, outsize)


def interpolate3D(data, grid, outsize):
    return interpolate(3, data, grid, outsize)


def _check(data, grid, ndim, outsize):
    if data.dim() != ndim + 2:
        raise ValueError("data must be [n_batch, n_channels, *in_size] with %d spatial axes" % ndim)
    if len(outsize) != ndim:
        raise ValueError("outsize must have %d entries" % ndim)
    P = 1
    for s in outsize:
        P *= s
    if grid.dim() != 3 or grid.shape[0] != data.shape[0] or grid.shape[1] != ndim or grid.shape[2] != P:
        raise ValueError("grid must be [%d, %d, %d], got %s"
                         % (data.shape[0], ndim, P, tuple(grid.shape)))


class _Interpolate(torch.autograd.Function):

    @staticmethod
    def forward(ctx, data, grid, ndim, outsize):
        _check(data, grid, ndim, outsize)
        data_c, grid_c = data.contiguous(), grid.contiguous()
        out = _native.interpolate(ndim, data_c, grid_c, outsize)
        ctx.ndim, ctx.outsize = ndim, outsize
        ctx.save_for_backward(data_c, grid_c)
        return out

    @staticmethod
    @torch.autograd.function.once_differentiable
    def backward(ctx, grad):
        data, grid = ctx.saved_tensors
        want_data, want_grid = ctx.needs_input_grad[0], ctx.needs_input_grad[1]
        if not (want_data or want_grid):
            return None, None, None, None
        gg, gd = _native.interpolate_backward(ctx.ndim, data, grid, ctx.outsize, grad.contiguous(),
                                              want_grid, want_data)
        return gd, gg, None, None
