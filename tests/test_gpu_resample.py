"""Resampling kernels versus the reference's interpolate (golden fixtures)
and the oracle; transform_data end to end."""
import os

import numpy as np
import pytest
import torch

from cpab.pytorch.interpolation import interpolate
from oracle import oracle as O
from helpers import cpab, rand_theta, rel_l2

pytestmark = [pytest.mark.gpu,
              pytest.mark.skipif(not torch.cuda.is_available(), reason="needs a CUDA GPU")]
DEV = "cuda"
G = np.load(os.path.join(os.path.dirname(__file__), "golden", "interp_golden.npz"))
KEYS = sorted({k.split("_")[0] for k in G.files})


@pytest.mark.parametrize("key", KEYS)
def test_matches_reference_fixture(key):
    m = G[key + "_meta"].tolist()
    nd = m[0]
    outsz = m[3 + nd:3 + 2 * nd]
    data = torch.from_numpy(G[key + "_data"]).to(DEV).requires_grad_(True)
    grid = torch.from_numpy(G[key + "_grid"]).to(DEV).requires_grad_(True)
    out = interpolate(nd, data, grid, outsz)
    np.testing.assert_array_equal(out.detach().cpu().numpy(), G[key + "_out"])  # bitwise
    (out * torch.from_numpy(G[key + "_w"]).to(DEV)).sum().backward()
    np.testing.assert_allclose(grid.grad.cpu().numpy(), G[key + "_dgrid"], rtol=1e-5, atol=1e-5)
    np.testing.assert_allclose(data.grad.cpu().numpy(), G[key + "_ddata"], rtol=1e-5, atol=1e-6)


@pytest.mark.parametrize("nd,B,C,insz,outsz", [
    (1, 3, 2, [300], [257]), (2, 2, 3, [70, 50], [33, 65]), (2, 1, 1, [512, 512], [100, 300]),
    (3, 2, 2, [20, 17, 15], [19, 33, 14])])
def test_matches_oracle_random(nd, B, C, insz, outsz):
    rng = np.random.default_rng(nd * 100 + B)
    data = rng.random((B, C, *insz), dtype=np.float32)
    P = int(np.prod(outsz))
    grid = rng.uniform(-0.2, 1.2, (B, nd, P)).astype(np.float32)
    w = rng.standard_normal((B, C, *outsz)).astype(np.float32)
    d_t = torch.from_numpy(data).to(DEV).requires_grad_(True)
    g_t = torch.from_numpy(grid).to(DEV).requires_grad_(True)
    out = interpolate(nd, d_t, g_t, outsz)
    np.testing.assert_array_equal(out.detach().cpu().numpy(), O.interpolate(nd, data, grid, outsz))
    (out * torch.from_numpy(w).to(DEV)).sum().backward()
    dg, dd = O.interpolate_backward(nd, data, grid, outsz, w)
    np.testing.assert_allclose(g_t.grad.cpu().numpy(), dg, rtol=1e-4, atol=1e-4)
    # d data: float32 atomics vs the oracle's float64 sum.  Border pixels of a
    # grid that leaves the image collect many large, cancelling contributions
    # (weights like -99 and +100 for points far outside), so only the interior
    # is held to a tight bound.
    gd = d_t.grad.cpu().numpy()
    assert rel_l2(gd, dd) < 1e-3
    inner = (slice(None), slice(None)) + tuple(slice(1, n - 1) for n in insz)
    np.testing.assert_allclose(gd[inner], dd[inner], rtol=1e-4, atol=1e-5)


@pytest.mark.parametrize("nc,zb,insz", [((6,), True, [40]), ((5, 5), False, [40, 30]),
                                         ((3, 3, 3), True, [12, 10, 9])])
def test_transform_data_end_to_end(nc, zb, insz):
    C = cpab(nc, zb)
    nd = len(nc)
    B, ch = 2, 2
    rng = np.random.default_rng(3)
    data = rng.random((B, ch, *insz), dtype=np.float32)
    th = rand_theta(B, C.params.d, 4, 0.5)
    th_t = torch.from_numpy(th).to(DEV).requires_grad_(True)
    out = C.transform_data(torch.from_numpy(data).to(DEV), th_t, insz)
    tgt = rng.random(out.shape, dtype=np.float32)
    loss = ((out - torch.from_numpy(tgt).to(DEV)) ** 2).mean()
    loss.backward()
    grid = C.uniform_meshgrid(insz, device="cpu").numpy()
    x, As, _ = O.transform(list(nc), C.params.basis, grid, th)
    ref = O.interpolate(nd, data, x, insz)
    np.testing.assert_allclose(out.detach().cpu().numpy(), ref, atol=1e-4)
    gout = 2 * (ref - tgt) / ref.size
    dgrid, _ = O.interpolate_backward(nd, data, x, insz, gout)
    dth, _ = O.gradient(list(nc), C.params.basis, grid, As, dgrid)
    assert rel_l2(th_t.grad.cpu().numpy(), dth) < 1e-3
