"""The way spatial-transformer code drives the library (the reference's
stn/stn.py:58-86 CpabWarp): Cpab(...).set_solver_params(T), get_theta_dim(),
then CPAB_transformer(points, theta, params, points.requires_grad) once per
transformation of a composition, the warped points fed to F.grid_sample.
This module restates that usage; it must keep running, differentiably, and
compose exactly like transform_grid_chain."""
import pytest
import torch
import torch.nn.functional as F

from cpab import Cpab
from cpab.pytorch.transformer import CPAB_transformer

pytestmark = [pytest.mark.gpu,
              pytest.mark.skipif(not torch.cuda.is_available(), reason="needs a CUDA GPU")]
DEV = "cuda"


class Warp(torch.nn.Module):
    def __init__(self, tess, nstepsolver=50):
        super().__init__()
        self.cpab = Cpab(list(tess), zero_boundary=True)
        self.cpab.set_solver_params(nstepsolver)
        self.theta_dim = self.cpab.get_theta_dim()

    def transform(self, points, thetas):
        for theta in thetas:
            points = CPAB_transformer(points, theta, self.cpab.params, points.requires_grad)
        return points

    def forward(self, x, thetas):
        B, C, H, W = x.shape
        pts = self.cpab.uniform_meshgrid([H, W], device=x.device)     # [2, H*W], coord 0 on H
        warped = self.transform(pts, thetas)                           # [B, 2, H*W]
        # grid_sample wants (x, y) = (W axis, H axis) in [-1, 1], laid out [B, H, W, 2]
        grid = warped.flip(1) * 2 - 1
        grid = grid.reshape(B, 2, W, H).permute(0, 3, 2, 1)
        return F.grid_sample(x, grid, align_corners=True, padding_mode="zeros")


def test_stn_style_composition_runs_and_matches_the_chain():
    torch.manual_seed(0)
    warp = Warp((4, 4))
    B, K = 3, 2
    thetas = [(0.3 * torch.randn(B, warp.theta_dim, device=DEV)).requires_grad_(True)
              for _ in range(K)]
    x = torch.rand(B, 3, 24, 32, device=DEV, requires_grad=True)
    y = warp(x, thetas)
    assert y.shape == x.shape and torch.isfinite(y).all()
    y.square().mean().backward()
    for th in thetas:
        assert th.grad is not None and torch.isfinite(th.grad).all() and th.grad.abs().sum() > 0
    assert x.grad is not None and torch.isfinite(x.grad).all()

    # the composition equals transform_grid_chain on stacked thetas (no dt scaling)
    pts = warp.cpab.uniform_meshgrid([24, 32], device=DEV)
    th_stack = torch.stack([t.detach() for t in thetas])
    chain = warp.cpab.transform_grid_chain(pts, th_stack)
    assert torch.equal(chain, warp.transform(pts, [t.detach() for t in thetas]))


def test_stn_style_points_gradient_flows_through_every_stage():
    warp = Warp((3, 3))
    th = [0.5 * torch.randn(2, warp.theta_dim, device=DEV) for _ in range(3)]
    pts = warp.cpab.uniform_meshgrid([10, 10], device=DEV).requires_grad_(True)
    out = warp.transform(pts, th)
    out.sum().backward()
    assert pts.grad is not None and pts.grad.shape == pts.shape and torch.isfinite(pts.grad).all()
