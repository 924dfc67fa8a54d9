"""The reference-side binding: compat.py loaded by file path (as the
reference's transformer.py would load it) and driven with the reference's
own composition (cpab/pytorch/transformer.py:73-168: torch.sparse.mm A-build,
expm, forward, backward_moments_and_points, sparse projection)."""
import importlib.util
import os

import numpy as np
import pytest
import torch

from helpers import DTHETA_RTOL, X_ATOL, cpab, rand_points, rand_theta, rel_l2

pytestmark = [pytest.mark.gpu,
              pytest.mark.skipif(not torch.cuda.is_available(), reason="needs a CUDA GPU")]

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def load_compat():
    spec = importlib.util.spec_from_file_location(
        "cpab_b200_compat_test", os.path.join(ROOT, "fg-cpab_b200", "cpab", "compat.py"))
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod.cpab_gpu


def reference_composition(cpab_gpu, C, points, theta, grad):
    """cpab/pytorch/transformer.py:73-168, restated over ``cpab_gpu``."""
    p = C.params
    B = C._get_basis_sparse_gpu(device=theta.device)
    Bt = B.transpose(0, 1).coalesce()
    n = theta.shape[0]
    As = torch.sparse.mm(B, theta.t()).t().reshape(n * p.nC, *p.Ashape)
    As_b = As.view(n, p.nC, *p.Ashape)
    ncx = int(p.nc[0])
    ncy = int(p.nc[1]) if p.ndim > 1 else 1
    if p.ndim == 1:
        out = cpab_gpu.forward_1d_closed_form(points.contiguous(), As_b.contiguous(), ncx)
    else:
        Trels = cpab_gpu.expm(As.contiguous(), 1.0 / p.nstepsolver).view(n, p.nC, *p.Ashape)
        out = cpab_gpu.forward(points.contiguous(), Trels.contiguous(), As_b.contiguous(),
                               p.nstepsolver, ncx, ncy, 0)
    mom, gp = cpab_gpu.backward_moments_and_points(points.contiguous(), As_b.contiguous(),
                                                   grad.contiguous(), p.nstepsolver, ncx, ncy, 0)
    if points.dim() == 2:
        gp = gp.sum(dim=0)
    mom_only = cpab_gpu.backward_moments(points.contiguous(), As_b.contiguous(),
                                         grad.contiguous(), p.nstepsolver, ncx, ncy, 0)
    dth = torch.sparse.mm(Bt, mom.reshape(n, -1).t()).t()
    return out, dth, gp, mom, mom_only


@pytest.mark.parametrize("nc", [(12,), (8, 8), (3, 4, 3)])
def test_compat_module_matches_public_api(nc):
    cpab_gpu = load_compat()
    C = cpab(nc)
    nd = len(nc)
    th = torch.from_numpy(rand_theta(3, C.params.d, 1, 0.5)).cuda()
    pts = torch.from_numpy(rand_points(nd, 5000, 2)).cuda()
    g = torch.from_numpy(rand_points(nd, 15000, 3, -1, 1).reshape(nd, 3, 5000)
                         .transpose(1, 0, 2).copy()).cuda()
    out, dth, gp, mom, mom_only = reference_composition(cpab_gpu, C, pts, th, g)
    t = th.clone().requires_grad_(True)
    p = pts.clone().requires_grad_(True)
    ours = C.transform_grid(p, t)
    (ours * g).sum().backward()
    assert (out - ours).abs().max().item() <= X_ATOL
    assert rel_l2(dth.cpu().numpy(), t.grad.cpu().numpy()) < DTHETA_RTOL
    assert rel_l2(gp.cpu().numpy(), p.grad.cpu().numpy()) < 1e-4
    assert rel_l2(mom_only.cpu().numpy(), mom.cpu().numpy()) < 1e-5


def test_compat_errors_like_reference():
    cpab_gpu = load_compat()
    As = torch.zeros(2, 3, 2, 3, device="cuda")
    with pytest.raises(RuntimeError):
        cpab_gpu.forward(torch.zeros(2, 5, device="cuda"), As, As, 50, 4, 4, 2)
    with pytest.raises(RuntimeError):
        cpab_gpu.expm(torch.zeros(3, 2, 4, device="cuda"), 0.1)
    with pytest.raises(RuntimeError):
        cpab_gpu.forward(torch.zeros(2, 5, device="cuda"), As, As, 101 * 3, 4, 4, 0)
