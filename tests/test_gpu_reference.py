"""sm_100a kernels versus the reference's own CUDA kernels (unmodified
cpab/core/cpab_ops_*.cu built into oracle/_ref) on identical inputs."""
import numpy as np
import pytest
import torch

import refkernels as R
from cpab import _native
from cpab.pytorch.transformer import device_basis
from oracle import oracle as O
from helpers import X_ATOL, cpab, near_boundary, rand_points, rand_theta, rel_l2

pytestmark = [pytest.mark.gpu,
              pytest.mark.skipif(not torch.cuda.is_available(), reason="needs a CUDA GPU")]


@pytest.fixture(autouse=True)
def _reference_kernels_built():
    R.require()


DEV = "cuda"

CASES = [((50,), True, 4, 20000, False, False, 50),
         ((20, 20), True, 4, 20000, False, False, 50),
         ((30, 30), False, 2, 20000, False, False, 50),
         ((7, 5), False, 3, 20000, True, True, 40),
         ((10, 10, 10), True, 2, 20000, False, False, 50),
         ((4, 3, 5), False, 2, 20000, True, True, 50),
         ((16, 16, 16), True, 1, 20000, False, False, 50)]


@pytest.mark.parametrize("case", CASES, ids=[str(c[0]) + ("-ad" if c[5] else "") for c in CASES])
def test_kernels_match_reference_kernels(case):
    nc, zb, n_theta, nP, batched, adaptive, T = case
    C = cpab(nc, zb)
    nd = len(nc)
    th = torch.from_numpy(rand_theta(n_theta, C.params.d, 31)).to(DEV)
    lo, hi = (0, 1) if zb else (-0.2, 1.2)
    pts_h = (np.stack([rand_points(nd, nP, 40 + b, lo, hi) for b in range(n_theta)])
             if batched else rand_points(nd, nP, 40, lo, hi))
    pts = torch.from_numpy(pts_h).to(DEV)
    As, trels = _native.build_A(nd, C.params.nC, device_basis(C.params, th.device), th,
                                None if nd == 1 else 1.0 / T)
    if nd > 1:
        tr_ref = R.expm(As, 1.0 / T)
        assert (trels - tr_ref).abs().max().item() <= 1e-6
        trels = tr_ref     # integrate both from the reference's Trels
    out = _native.forward(nd, list(nc), pts, batched, trels, As, T, int(adaptive))
    out_ref = R.forward(nc, pts, batched, trels, As, T, adaptive)
    assert (out - out_ref).abs().max().item() <= X_ATOL
    fo = out.permute(1, 0, 2).reshape(nd, -1).cpu().numpy()
    fr = out_ref.permute(1, 0, 2).reshape(nd, -1).cpu().numpy()
    differ = O.cells(list(nc), fo) != O.cells(list(nc), fr)
    assert not (differ & ~near_boundary(list(nc), fr)).any()
    g = torch.randn(n_theta, nd, nP, device=DEV, generator=torch.Generator(DEV).manual_seed(3))
    mom, gp = _native.backward(nd, list(nc), pts, batched, As, g, T, int(adaptive), True)
    mom_ref, gp_ref = R.backward(nc, pts, batched, As, g, T, adaptive)
    assert rel_l2(mom.cpu().numpy(), mom_ref.cpu().numpy()) < 1e-5
    assert (gp - gp_ref).abs().max().item() <= 1e-4 * max(1.0, gp_ref.abs().max().item())
    basis = device_basis(C.params, th.device)
    d_ours = _native.project(basis, mom)
    d_ref = _native.project(basis, mom_ref)
    assert rel_l2(d_ours.cpu().numpy(), d_ref.cpu().numpy()) < 1e-4
