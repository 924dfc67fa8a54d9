"""sm_100a kernels versus the CPU oracle, stage by stage on identical inputs
and end to end through the public API (CUDA path through the C ABI)."""
import numpy as np
import pytest
import torch

from cpab import _native
from cpab.pytorch.transformer import device_basis
from oracle import oracle as O
from helpers import (BOUNDARY_EPS, DTHETA_RTOL, X_ATOL, cpab, near_boundary, rand_points,
                     rand_theta, rel_l2)

pytestmark = [pytest.mark.gpu,
              pytest.mark.skipif(not torch.cuda.is_available(), reason="needs a CUDA GPU")]

DEV = "cuda"

# (nc, zero_boundary, n_theta, nP, batched, adaptive, nstepsolver, theta scale, point range)
CASES = [
    ((8,), True, 3, 3000, False, False, 50, 1.0, (0, 1)),
    ((50,), True, 4, 5000, True, False, 50, 1.0, (0, 1)),
    ((6,), False, 3, 3000, False, False, 50, 1.0, (-0.2, 1.2)),
    ((4, 4), True, 3, 4000, False, False, 50, 1.0, (0, 1)),
    ((12, 12), True, 4, 6000, False, False, 50, 1.0, (0, 1)),
    ((20, 20), True, 2, 6000, True, False, 50, 1.0, (0, 1)),
    ((5, 3), False, 3, 4000, False, False, 37, 0.7, (-0.3, 1.3)),
    ((6, 6), True, 2, 4000, False, True, 50, 1.5, (0, 1)),
    ((4, 5), False, 2, 4000, True, True, 20, 1.0, (-0.2, 1.2)),
    ((30, 30), False, 2, 3000, False, False, 50, 0.5, (0, 1)),
    ((3, 3, 3), True, 3, 4000, False, False, 50, 1.0, (0, 1)),
    ((4, 3, 2), False, 2, 4000, True, False, 30, 0.8, (-0.2, 1.2)),
    ((3, 3, 3), True, 2, 3000, False, True, 50, 1.0, (0, 1)),
    ((10, 10, 10), True, 2, 4000, False, False, 50, 1.0, (0, 1)),
    ((2, 2), True, 2, 2000, False, False, 256, 1.0, (0, 1)),
    ((3, 3), True, 2, 2000, False, False, 1, 1.0, (0, 1)),
]
IDS = ["%dd-%s-zb%d-b%d-n%d-%s-ad%d-T%d" % (len(c[0]), "x".join(map(str, c[0])), c[1], c[2], c[3],
                                            "bat" if c[4] else "shr", c[5], c[6]) for c in CASES]


def setup(case):
    nc, zb, n_theta, nP, batched, adaptive, T, scale, (lo, hi) = case
    C = cpab(nc, zb)
    nd = len(nc)
    seed = abs(hash(case)) % 1000
    th = rand_theta(n_theta, C.params.d, seed, scale)
    pts = rand_points(nd, nP, seed + 1, lo, hi)
    if batched:
        pts = np.stack([rand_points(nd, nP, seed + 2 + b, lo, hi) for b in range(n_theta)])
    return C, list(nc), th, pts, batched, adaptive, T


@pytest.mark.parametrize("case", CASES, ids=IDS)
def test_stages_match_oracle_on_identical_inputs(case):
    C, nc, th, pts, batched, adaptive, T = setup(case)
    nd = len(nc)
    p = C.params
    th_d = torch.from_numpy(th).to(DEV)
    pts_d = torch.from_numpy(pts).to(DEV)
    basis = device_basis(p, th_d.device)
    As, trels = _native.build_A(nd, p.nC, basis, th_d, None if nd == 1 else 1.0 / T)
    As_h = As.cpu().numpy()
    # A = B theta
    np.testing.assert_allclose(As_h, O.build_A(p.basis, th, nd), rtol=1e-5, atol=1e-5)
    # expm (fused into build_A)
    if nd > 1:
        tr_h = trels.cpu().numpy()
        np.testing.assert_allclose(tr_h, O.expm(As_h, 1.0 / T), rtol=1e-6, atol=1e-6)
        ex = _native.expm(As.view(-1, nd, nd + 1), 1.0 / T).view_as(As).cpu().numpy()
        np.testing.assert_array_equal(ex, tr_h)
    else:
        tr_h = None
    # integration, given the same A / Trels
    out = _native.forward(nd, nc, pts_d, batched, trels, As, T, int(adaptive)).cpu().numpy()
    ref = O.integrate(nc, pts, As_h, tr_h, T, adaptive)
    err = np.abs(out - ref).max()
    assert err <= X_ATOL, err
    # final cells bit-exact except within BOUNDARY_EPS of a facet
    flat_o = out.transpose(1, 0, 2).reshape(nd, -1)
    flat_r = ref.transpose(1, 0, 2).reshape(nd, -1)
    gpu_cells = _native.cell_index(nc, torch.from_numpy(np.ascontiguousarray(flat_o)).to(DEV)).cpu().numpy()
    np.testing.assert_array_equal(gpu_cells, O.cells(nc, flat_o))   # lookup is bit-exact
    differ = O.cells(nc, flat_o) != O.cells(nc, flat_r)
    assert not (differ & ~near_boundary(nc, flat_r, BOUNDARY_EPS)).any()
    # adjoint moments and lambda(0), given the same A and upstream gradient
    g = rand_points(nd, pts.shape[-1] * th.shape[0], 99, -1, 1).reshape(
        nd, th.shape[0], -1).transpose(1, 0, 2).copy()
    mom, gp = _native.backward(nd, nc, pts_d, batched, As, torch.from_numpy(g).to(DEV), T,
                               int(adaptive), True)
    mom_r, gp_r = O.adjoint(nc, pts, As_h, g, T, adaptive)
    assert rel_l2(mom.cpu().numpy(), mom_r) < 1e-5
    np.testing.assert_allclose(gp.cpu().numpy(), gp_r, rtol=1e-4, atol=1e-5)
    # projection, given the same moments
    dth = _native.project(basis, mom).cpu().numpy()
    assert rel_l2(dth, O.project(p.basis, mom.cpu().numpy())) < 1e-6


@pytest.mark.parametrize("case", CASES, ids=IDS)
def test_public_api_matches_oracle_end_to_end(case):
    C, nc, th, pts, batched, adaptive, T = setup(case)
    nd = len(nc)
    C.set_solver_params(T, bool(adaptive))
    try:
        th_d = torch.from_numpy(th).to(DEV).requires_grad_(True)
        pts_d = torch.from_numpy(pts).to(DEV).requires_grad_(True)
        out = C.transform_grid(pts_d, th_d)
        w = torch.from_numpy(rand_points(nd, out.numel() // nd, 7, -1, 1)).to(DEV).reshape(
            nd, out.shape[0], -1).permute(1, 0, 2).contiguous()
        (out * w).sum().backward()
        x_r, As_r, _ = O.transform(nc, C.params.basis, pts, th, T, adaptive)
        assert np.abs(out.detach().cpu().numpy() - x_r).max() <= X_ATOL
        dth_r, gp_r = O.gradient(nc, C.params.basis, pts, As_r, w.cpu().numpy(), T, adaptive)
        assert rel_l2(th_d.grad.cpu().numpy(), dth_r) < DTHETA_RTOL
        np.testing.assert_allclose(pts_d.grad.cpu().numpy(), gp_r, rtol=1e-3, atol=1e-4)
    finally:
        C.set_solver_params(50, False)


@pytest.mark.parametrize("nc", [(7,), (5, 4), (3, 2, 4)])
def test_cell_lookup_bit_exact_on_adversarial_points(nc):
    """Facets, vertices, corners, outside the domain, +-0, huge, NaN."""
    nd = len(nc)
    rng = np.random.default_rng(5)
    grids = [np.arange(n + 1) / n for n in nc]
    pts = []
    for _ in range(20000):
        p = []
        for k in range(nd):
            r = rng.random()
            if r < 0.3:
                v = rng.choice(grids[k])
            elif r < 0.4:
                v = rng.choice(grids[k]) + rng.choice([-1, 1]) * rng.random() * 1e-6
            elif r < 0.5:
                v = rng.choice([-0.0, 0.0, 1.0, 1.0 - 1e-7, 0.5])
            elif r < 0.7:
                v = rng.uniform(-1.5, 2.5)
            else:
                v = rng.random()
            p.append(v)
        pts.append(p)
    pts = np.asarray(pts, np.float32).T.copy()
    pts[:, :7] = np.array([[np.nan] * nd, [1e30] * nd, [-1e30] * nd, [-0.0] * nd, [1.0] * nd,
                           [0.0] * nd, [0.5] * nd], np.float32).T
    got = _native.cell_index(list(nc), torch.from_numpy(pts).to(DEV)).cpu().numpy()
    np.testing.assert_array_equal(got, O.cells(list(nc), pts))


def test_zero_theta_is_exact_identity():
    for nc in [(10,), (20, 20), (4, 4, 4)]:
        C = cpab(nc)
        pts = torch.rand(len(nc), 10000, device=DEV)
        out = C.transform_grid(pts, C.identity(3))
        assert torch.equal(out, pts.expand(3, -1, -1))


# (nc, zero_boundary, n_theta): sparse and general bases, fewer and more
# transformations than a warp's 32 lanes.
PRODUCT_CASES = [((30, 30), False, 32), ((30, 30), False, 40), ((5, 3), False, 7),
                 ((20, 20), True, 16), ((6,), False, 33), ((4, 3, 2), False, 3),
                 ((10, 10, 10), True, 4)]


@pytest.mark.parametrize("case", PRODUCT_CASES,
                         ids=["%s-zb%d-t%d" % ("x".join(map(str, c[0])), c[1], c[2])
                              for c in PRODUCT_CASES])
def test_basis_products_match_oracle_bit_for_bit(case):
    """A = B theta and dtheta = B^T m, through both the plain entry points and
    the transposed-operand ones (used for general bases): every entry is one
    sequential fma chain over its row, as the oracle sums it, so all four
    agree with the oracle exactly; both Trels are the same GPU expm of the
    same A (against the oracle's libm-based expm within 1e-6, as above)."""
    nc, zb, n_theta = case
    C = cpab(nc, zb)
    p, nd = C.params, len(nc)
    th = rand_theta(n_theta, p.d, 11, 0.7)
    th_d = torch.from_numpy(th).to(DEV)
    basis = device_basis(p, th_d.device)
    dT = None if nd == 1 else 1.0 / 50
    ref_A = O.build_A(p.basis, th, nd)
    A1, T1 = _native.build_A(nd, p.nC, basis, th_d, dT)
    A2, T2 = _native.build_A_tt(nd, p.nC, basis, th_d.t().contiguous(), n_theta, dT)
    np.testing.assert_array_equal(A1.cpu().numpy(), ref_A)
    np.testing.assert_array_equal(A2.cpu().numpy(), ref_A)
    if dT is not None:
        np.testing.assert_array_equal(T1.cpu().numpy(), T2.cpu().numpy())
        np.testing.assert_allclose(T1.cpu().numpy(), O.expm(ref_A, dT), rtol=1e-6, atol=1e-6)
    mom = np.random.default_rng(12).standard_normal((n_theta, p.nC, nd * (nd + 1))).astype(np.float32)
    mom_d = torch.from_numpy(mom).to(DEV)
    ref_d = O.project(p.basis, mom)
    d1 = _native.project(basis, mom_d)
    d2 = _native.project_tt(basis, mom_d.reshape(n_theta, -1).t().contiguous(), n_theta)
    np.testing.assert_array_equal(d1.cpu().numpy(), ref_d)
    np.testing.assert_array_equal(d2.cpu().numpy(), ref_d)
