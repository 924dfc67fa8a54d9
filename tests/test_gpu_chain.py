"""Fused transform_grid_chain (one kernel through all stages each way)
against the per-stage composition it replaces (cpab/cpab.py:269-278)."""
import numpy as np
import pytest
import torch

from cpab.pytorch.transformer import CPAB_transformer, transform_chain
from helpers import cpab, rand_points, rand_theta, rel_l2

pytestmark = [pytest.mark.gpu,
              pytest.mark.skipif(not torch.cuda.is_available(), reason="needs a CUDA GPU")]
DEV = "cuda"

CASES = [
    # tess, zero_boundary, stages, batch, points, batched input, adaptive
    ((6, 6), True, 4, 3, 20000, False, False),
    ((5, 4), False, 3, 2, 9000, True, False),
    ((4, 4), True, 2, 2, 6000, False, True),
    ((3, 3, 3), True, 4, 2, 12000, False, False),
    ((2, 3, 2), False, 3, 1, 5000, True, False),
]
IDS = ["2d", "2d-dense-batched", "2d-adaptive", "3d", "3d-dense-batched"]


@pytest.mark.parametrize("case", CASES, ids=IDS)
def test_fused_chain_matches_per_stage_composition(case):
    tess, zb, K, B, nP, batched, adaptive = case
    C = cpab(tess, zb)
    nd = len(tess)
    C.set_solver_params(50, adaptive)
    try:
        th = torch.from_numpy(rand_theta(K * B, C.params.d, 41, 0.5)).reshape(K, B, -1).to(DEV)
        pts = torch.from_numpy(rand_points(nd, nP, 42)).to(DEV)
        if batched:
            pts = pts[None].repeat(B, 1, 1) + 0.01 * torch.rand(B, nd, nP, device=DEV)
        w = torch.randn(B, nd, nP, device=DEV)

        p1, t1 = pts.clone().requires_grad_(True), th.clone().requires_grad_(True)
        out_f = transform_chain(p1, t1, C.params, compute_points_grad=True)
        (out_f * w).sum().backward()

        p2, t2 = pts.clone().requires_grad_(True), th.clone().requires_grad_(True)
        out_c = p2
        for k in range(K):
            out_c = CPAB_transformer(out_c, t2[k], C.params, compute_points_grad=True)
        (out_c * w).sum().backward()

        assert torch.equal(out_f, out_c)  # same per-stage arithmetic
        assert rel_l2(t1.grad.cpu().numpy(), t2.grad.cpu().numpy()) < 1e-5
        np.testing.assert_allclose(p1.grad.cpu().numpy(), p2.grad.cpu().numpy(),
                                   rtol=1e-4, atol=1e-5)
    finally:
        C.set_solver_params(50, False)


def test_transform_grid_chain_uses_the_fused_path_and_scales():
    C = cpab((5, 5), True)
    K = 3
    thc = torch.from_numpy(rand_theta(K, C.params.d, 7)).to(DEV).requires_grad_(True)
    grid = C.uniform_meshgrid([40, 30], device=DEV)
    out = C.transform_grid_chain(grid, thc, scale_by_dt=True)
    ref = grid
    for k in range(K):
        ref = CPAB_transformer(ref, thc[k:k + 1] / K, C.params, compute_points_grad=True)
    assert torch.equal(out, ref)
    out.sum().backward()
    assert thc.grad.shape == thc.shape and torch.isfinite(thc.grad).all()
