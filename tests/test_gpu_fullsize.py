"""Parity at the benchmark configurations' full sizes.

The oracle cannot integrate millions of points in a test, but every point's
trajectory is independent of the others, so full-size runs are checked
through properties that do not depend on the size:
  * the GPU's outputs at a random sample of points equal the oracle's for
    those points alone;
  * a backward whose upstream gradient is zero except on a sample equals the
    oracle's gradient over that sample (points with zero gradient add
    nothing to the moments);
  * dtheta is linear in the upstream gradient.
Inputs are the bench's seeded synthetic inputs."""
import numpy as np
import pytest
import torch

from cpab import _native
from cpab.pytorch.transform_data import mesh_axes
from cpab.pytorch.transformer import device_basis
from oracle import oracle as O
from helpers import (BOUNDARY_EPS, DTHETA_RTOL, X_ATOL, cpab, near_boundary, rel_l2)

pytestmark = [pytest.mark.gpu,
              pytest.mark.skipif(not torch.cuda.is_available(), reason="needs a CUDA GPU")]
DEV = "cuda"
T = 50


def gen(seed):
    return torch.Generator().manual_seed(seed)


def sample(n, k, seed):
    return np.sort(np.random.default_rng(seed).choice(n, size=k, replace=False))


@pytest.mark.parametrize("nc", [[20, 20], [12, 12], [30, 30]], ids=["20x20", "12x12", "30x30"])
def test_bench_2d_config_forward_and_gradient_at_full_size(nc):
    # Cpab([20,20]), batch 16, 125,000 points, theta ~ N(0,1);
    # the same workload is repeated at tessellations 12x12 and 30x30.
    C = cpab(tuple(nc), True)
    B, nP = 16, 125_000
    th = torch.randn(B, C.params.d, generator=gen(0))
    pts = torch.rand(2, nP, generator=gen(1))
    th_d = th.to(DEV).requires_grad_(True)
    pts_d = pts.to(DEV)
    out = C.transform_grid(pts_d, th_d)

    As, trels = _native.build_A(2, C.params.nC, device_basis(C.params, th_d.device),
                                th_d.detach(), 1.0 / T)
    As_h, tr_h = As.cpu().numpy(), trels.cpu().numpy()
    idx = sample(nP, 2000, 5)
    ref = O.integrate(nc, pts[:, idx].numpy(), As_h, tr_h, T)
    got = out.detach()[:, :, idx].cpu().numpy()
    assert np.abs(got - ref).max() <= X_ATOL
    flat_g = got.transpose(1, 0, 2).reshape(2, -1)
    flat_r = ref.transpose(1, 0, 2).reshape(2, -1)
    differ = O.cells(nc, flat_g) != O.cells(nc, flat_r)
    assert not (differ & ~near_boundary(nc, flat_r, BOUNDARY_EPS)).any()

    # upstream gradient on a sample of 500 points only
    sub = sample(nP, 500, 6)
    w = np.zeros((B, 2, nP), np.float32)
    w[:, :, sub] = np.random.default_rng(7).uniform(-1, 1, (B, 2, len(sub)))
    (out * torch.from_numpy(w).to(DEV)).sum().backward()
    dth_ref, _ = O.gradient(nc, C.params.basis, pts[:, sub].numpy(), As_h, w[:, :, sub], T)
    assert rel_l2(th_d.grad.cpu().numpy(), dth_ref) < DTHETA_RTOL


def test_bench_2d_config_gradient_is_linear_in_upstream_gradient():
    C = cpab((20, 20), True)
    B, nP = 16, 125_000
    th = torch.randn(B, C.params.d, generator=gen(0)).to(DEV)
    pts = torch.rand(2, nP, generator=gen(1)).to(DEV)
    g1 = torch.randn(B, 2, nP, generator=gen(2)).to(DEV)
    g2 = torch.randn(B, 2, nP, generator=gen(3)).to(DEV)

    def grad(g):
        t = th.clone().requires_grad_(True)
        (C.transform_grid(pts, t) * g).sum().backward()
        return t.grad.double()

    lhs = grad(g1 + g2)
    rhs = grad(g1) + grad(g2)
    # exact in exact arithmetic; each dtheta sums ~10^8 fp32 moment contributions
    # in atomic order (measured 2e-5), so the bound is the dtheta tolerance
    assert float((lhs - rhs).norm() / rhs.norm()) < DTHETA_RTOL


def test_chain_config_at_full_size():
    # BASELINE 3D chain: Cpab([16,16,16]), 4 stages, scale_by_dt, theta ~ N(0, 0.5^2),
    # 160 x 192 x 160 meshgrid (4,915,200 points).
    C = cpab((16, 16, 16), True)
    nc = [16, 16, 16]
    K = 4
    thc = torch.randn(K, C.params.d, generator=gen(0)) * 0.5
    grid = C.uniform_meshgrid([160, 192, 160], device="cpu")
    nP = grid.shape[1]
    th_d = thc.to(DEV).requires_grad_(True)
    out = C.transform_grid_chain(grid.to(DEV), th_d, scale_by_dt=True)

    idx = sample(nP, 1000, 11)
    x = grid[:, idx].numpy()
    stages = []
    for k in range(K):
        xk, As_k, _ = O.transform(nc, C.params.basis, x, thc[k:k + 1].numpy() / K, T)
        stages.append((x, As_k))
        x = xk
    got = out.detach()[:, :, idx].cpu().numpy()
    # A = B theta is summed in a fixed order on both sides, but the stages compound it
    assert np.abs(got - x).max() <= 2 * X_ATOL

    w = np.zeros((1, 3, nP), np.float32)
    w[:, :, idx] = np.random.default_rng(12).uniform(-1, 1, (1, 3, len(idx)))
    (out * torch.from_numpy(w).to(DEV)).sum().backward()
    lam = w[:, :, idx]
    grads = []
    for k in reversed(range(K)):
        xin, As_k = stages[k]
        mom, gp = O.adjoint(nc, xin, As_k, lam, T)
        grads.append(O.project(C.params.basis, mom)[0] / K)
        lam = gp
    dth_ref = np.stack(grads[::-1])
    assert rel_l2(th_d.grad.cpu().numpy(), dth_ref) < DTHETA_RTOL


def test_dense_2d_transform_data_config_at_full_size():
    # BASELINE dense 2D: Cpab([30,30], zero_boundary=False), 32 x 3 x 512 x 512 images,
    # theta ~ N(0, 0.5^2), transform_data to [512, 512].
    C = cpab((30, 30), False)
    nc = [30, 30]
    B, Ch, n = 32, 3, 512
    th = torch.randn(B, C.params.d, generator=gen(0)) * 0.5
    data = torch.rand(B, Ch, n, n, generator=gen(2))
    th_d = th.to(DEV).requires_grad_(True)
    out = C.transform_data(data.to(DEV), th_d, (n, n))

    As, trels = _native.build_A(2, C.params.nC, device_basis(C.params, th_d.device),
                                th_d.detach(), 1.0 / T)
    As_h, tr_h = As.cpu().numpy(), trels.cpu().numpy()
    axes = mesh_axes(C.params, (n, n), th_d.device).cpu().numpy()  # the meshgrid's values
    pix = sample(n * n, 1500, 13)           # output pixels o = i0 * n + i1
    i0, i1 = pix // n, pix % n
    pts = np.stack([axes[i0], axes[n + i1]]).astype(np.float32)
    x = O.integrate(nc, pts, As_h, tr_h, T)                 # [B, 2, 1500]
    ref = O.interpolate(2, data.numpy(), x, (1, len(pix)))  # [B, C, 1, 1500]
    got = out.detach().reshape(B, Ch, -1)[:, :, pix].cpu().numpy()
    assert np.abs(got - ref[:, :, 0]).max() <= 1e-5

    # upstream gradient on the sampled pixels only
    g = np.zeros((B, Ch, n * n), np.float32)
    gs = np.random.default_rng(14).uniform(-1, 1, (B, Ch, len(pix))).astype(np.float32)
    g[:, :, pix] = gs
    (out * torch.from_numpy(g.reshape(B, Ch, n, n)).to(DEV)).sum().backward()
    dgrid, _ = O.interpolate_backward(2, data.numpy(), x, (1, len(pix)), gs[:, :, None, :])
    dth_ref, _ = O.gradient(nc, C.params.basis, pts, As_h, dgrid, T)
    assert rel_l2(th_d.grad.cpu().numpy(), dth_ref) < DTHETA_RTOL


def test_1d_config_at_full_size():
    # Cpab([50], zero_boundary=True), batch 8, theta ~ N(0,1),
    # 100,000 shared points ~ U[0,1]; loss sum((x_t - x)^2).  The forward is the
    # closed-form integration (cpab/core/cpab_ops_1d.cu:131-205).
    C = cpab((50,), True)
    nc = [50]
    B, nP = 8, 100_000
    th = torch.randn(B, C.params.d, generator=gen(0))
    pts = torch.rand(1, nP, generator=gen(1))
    th_d = th.to(DEV).requires_grad_(True)
    pts_d = pts.to(DEV)
    out = C.transform_grid(pts_d, th_d)

    As, _ = _native.build_A(1, C.params.nC, device_basis(C.params, th_d.device),
                            th_d.detach(), 1.0 / T)
    As_h = As.cpu().numpy()
    idx = sample(nP, 4000, 21)
    ref = O.integrate(nc, pts[:, idx].numpy(), As_h, None, T)
    got = out.detach()[:, :, idx].cpu().numpy()
    assert np.abs(got - ref).max() <= X_ATOL
    flat_g, flat_r = got.reshape(1, -1), ref.reshape(1, -1)
    differ = O.cells(nc, flat_g) != O.cells(nc, flat_r)
    assert not (differ & ~near_boundary(nc, flat_r, BOUNDARY_EPS)).any()

    # the bench's loss, with its upstream gradient 2 (x_t - x) kept on a sample only
    sub = sample(nP, 1000, 22)
    mask = torch.zeros(1, 1, nP)
    mask[:, :, sub] = 1.0
    loss = (((out - pts_d) ** 2) * mask.to(DEV)).sum()
    loss.backward()
    x_sub = O.integrate(nc, pts[:, sub].numpy(), As_h, None, T)
    w = (2.0 * (x_sub - pts[:, sub].numpy()[None])).astype(np.float32)
    dth_ref, _ = O.gradient(nc, C.params.basis, pts[:, sub].numpy(), As_h, w, T)
    assert rel_l2(th_d.grad.cpu().numpy(), dth_ref) < DTHETA_RTOL


def test_3d_transform_data_config_at_full_size():
    # BASELINE 3D: Cpab([10,10,10], zero_boundary=True), batch 4, theta ~ N(0,1),
    # single-channel 128^3 volumes, each a seeded sum of 20 Gaussian blobs;
    # transform_data to [128, 128, 128] (trilinear).  The reference composes
    # uniform_meshgrid, transform_grid and interpolate (cpab/cpab.py:306-308,
    # cpab/pytorch/interpolation.py:97-160); this library runs it fused.
    import bench
    C = cpab((10, 10, 10), True)
    nc = [10, 10, 10]
    B, n = 4, 128
    th = torch.randn(B, C.params.d, generator=gen(0))
    g = gen(2)
    data = torch.stack([bench.blobs([n, n, n], g) for _ in range(B)])[:, None]
    th_d = th.to(DEV).requires_grad_(True)
    out = C.transform_data(data.to(DEV), th_d, (n, n, n))
    assert out.shape == (B, 1, n, n, n)

    As, trels = _native.build_A(3, C.params.nC, device_basis(C.params, th_d.device),
                                th_d.detach(), 1.0 / T)
    As_h, tr_h = As.cpu().numpy(), trels.cpu().numpy()
    axes = mesh_axes(C.params, (n, n, n), th_d.device).cpu().numpy()
    vox = sample(n ** 3, 1500, 31)          # output voxels o = (i0 * n + i1) * n + i2
    i0, i1, i2 = vox // (n * n), (vox // n) % n, vox % n
    pts = np.stack([axes[i0], axes[n + i1], axes[2 * n + i2]]).astype(np.float32)
    x = O.integrate(nc, pts, As_h, tr_h, T)                      # [B, 3, 1500]
    ref = O.interpolate(3, data.numpy(), x, (1, 1, len(vox)))     # [B, 1, 1, 1, 1500]
    got = out.detach().reshape(B, 1, -1)[:, :, vox].cpu().numpy()
    assert np.abs(got - ref[:, :, 0, 0]).max() <= 1e-5

    # upstream gradient on the sampled voxels only
    gr = np.zeros((B, 1, n ** 3), np.float32)
    gs = np.random.default_rng(32).uniform(-1, 1, (B, 1, len(vox))).astype(np.float32)
    gr[:, :, vox] = gs
    (out * torch.from_numpy(gr.reshape(B, 1, n, n, n)).to(DEV)).sum().backward()
    dgrid, _ = O.interpolate_backward(3, data.numpy(), x, (1, 1, len(vox)),
                                      gs[:, :, None, None, :])
    dth_ref, _ = O.gradient(nc, C.params.basis, pts, As_h, dgrid, T)
    assert rel_l2(th_d.grad.cpu().numpy(), dth_ref) < DTHETA_RTOL
