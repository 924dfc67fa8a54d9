"""Fused transform_data (one kernel each way, 2D/3D) against the composition
it replaces -- uniform_meshgrid, transform_grid, interpolate
(cpab/cpab.py:306-308) -- through the public API."""
import numpy as np
import pytest
import torch

from cpab.pytorch.transform_data import transform_data as fused
from helpers import cpab, rand_theta, rel_l2

pytestmark = [pytest.mark.gpu,
              pytest.mark.skipif(not torch.cuda.is_available(), reason="needs a CUDA GPU")]
DEV = "cuda"

CASES = [
    # tess, zero_boundary, batch, channels, in_size, outsize, theta scale, adaptive
    ((6, 6), True, 3, 3, (40, 50), (40, 50), 1.0, False),
    ((5, 7), False, 2, 1, (33, 47), (52, 36), 0.5, False),
    ((4, 4), True, 2, 2, (30, 30), (45, 45), 1.0, True),
    ((3, 3, 3), True, 2, 1, (16, 18, 14), (16, 18, 14), 1.0, False),
    ((2, 3, 2), False, 1, 2, (12, 10, 14), (15, 11, 9), 0.5, False),
    ((3, 3, 3), True, 1, 1, (10, 12, 11), (12, 10, 11), 1.0, True),
]
IDS = ["2d", "2d-dense-resize", "2d-adaptive", "3d", "3d-dense-resize", "3d-adaptive"]


def composed(C, data, theta, outsize):
    grid = C.uniform_meshgrid(outsize, device=theta.device)
    grid_t = C.transform_grid(grid, theta)
    return C.interpolate(data, grid_t, outsize), grid_t


@pytest.mark.parametrize("case", CASES, ids=IDS)
def test_fused_transform_data_matches_composition(case):
    tess, zb, B, Ch, in_size, outsize, scale, adaptive = case
    C = cpab(tess, zb)
    C.set_solver_params(50, adaptive)
    try:
        g = torch.Generator().manual_seed(11)
        data = torch.rand(B, Ch, *in_size, generator=g).to(DEV)
        th = torch.from_numpy(rand_theta(B, C.params.d, 12, scale)).to(DEV)
        w = torch.randn(B, Ch, *outsize, generator=g).to(DEV)

        d1, t1 = data.clone().requires_grad_(True), th.clone().requires_grad_(True)
        out_f = fused(d1, t1, C.params, outsize)
        (out_f * w).sum().backward()
        d2, t2 = data.clone().requires_grad_(True), th.clone().requires_grad_(True)
        out_c, grid_t = composed(C, d2, t2, outsize)
        (out_c * w).sum().backward()

        # same arithmetic: the forward is bit-identical
        assert torch.equal(out_f, out_c)
        # gradients differ only by the order of fp32 atomic sums
        assert rel_l2(t1.grad.cpu().numpy(), t2.grad.cpu().numpy()) < 1e-5
        assert rel_l2(d1.grad.cpu().numpy(), d2.grad.cpu().numpy()) < 1e-5
        # the public method takes the fused path in 2D/3D
        out_m = C.transform_data(data, th, outsize)
        assert torch.equal(out_m, out_c.detach())
    finally:
        C.set_solver_params(50, False)


def test_fused_grid_is_the_transformed_meshgrid_in_output_order():
    from cpab import _native
    from cpab.pytorch.transform_data import mesh_axes
    from cpab.pytorch.transformer import _nc, device_basis
    C = cpab((5, 5), True)
    outsize = (24, 31)
    th = torch.from_numpy(rand_theta(2, C.params.d, 3)).to(DEV)
    data = torch.rand(2, 1, 20, 20, device=DEV)
    As, trels = _native.build_A(2, C.params.nC, device_basis(C.params, th.device), th, 1.0 / 50)
    _, grid_t = _native.transform_data(2, _nc(C.params), outsize, mesh_axes(C.params, outsize, th.device),
                                       trels, As, 50, 0, data)
    ref = C.transform_grid(C.uniform_meshgrid(outsize, device=th.device), th)
    # grid order (coordinate 0 fastest) -> output order (last axis fastest)
    ref_o = ref.reshape(2, 2, outsize[1], outsize[0]).transpose(2, 3).reshape(2, 2, -1)
    assert torch.equal(grid_t, ref_o)


def test_fused_theta_only_and_no_grad():
    C = cpab((4, 4), True)
    th = torch.from_numpy(rand_theta(2, C.params.d, 5)).to(DEV).requires_grad_(True)
    data = torch.rand(2, 3, 16, 16, device=DEV)
    out = C.transform_data(data, th, (16, 16))
    out.square().mean().backward()
    assert th.grad is not None and torch.isfinite(th.grad).all()
    with torch.no_grad():
        out2 = C.transform_data(data, th, (16, 16))
    assert torch.equal(out.detach(), out2)


def test_fused_rejects_mismatched_batch():
    C = cpab((4, 4), True)
    th = torch.from_numpy(rand_theta(2, C.params.d, 5)).to(DEV)
    with pytest.raises(ValueError):
        fused(torch.rand(3, 1, 8, 8, device=DEV), th, C.params, (8, 8))
