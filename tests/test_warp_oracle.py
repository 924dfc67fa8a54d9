"""The oracle's restatement of the STN sampling (F.grid_sample with
align_corners=True at CPAB points, stn/stn.py:48-54 and :86 of the
reference), pinned against torch's own F.grid_sample on the CPU, which is
the function the reference calls."""
import numpy as np
import pytest
import torch
import torch.nn.functional as F

from oracle import oracle as O


def _grid(pts, nd):
    """CPAB points [B, nd, P] -> grid_sample's grid [B, *ones, P, nd] in
    (x, y, z) order, as stn/stn.py:86 and :48 build it."""
    g = torch.from_numpy(pts) * 2 - 1
    g = g.flip(1).transpose(1, 2)                         # [B, P, nd], x first
    return g.reshape(g.shape[0], *([1] * (nd - 1)), g.shape[1], nd)


def _case(nd, seed, spread):
    rng = np.random.default_rng(seed)
    in_size = (7, 9) if nd == 2 else (5, 6, 4)
    B, C, P = 3, 2, 257
    data = rng.random((B, C, *in_size)).astype(np.float32)
    # points inside and around the image: every padding rule is exercised
    pts = (rng.random((B, nd, P)) * (1 + 2 * spread) - spread).astype(np.float32)
    return data, pts


@pytest.mark.parametrize("nd", [2, 3])
@pytest.mark.parametrize("padding", ["zeros", "border", "reflection"])
@pytest.mark.parametrize("spread", [0.0, 0.7])
def test_sampling_matches_torch_grid_sample(nd, padding, spread):
    data, pts = _case(nd, 10 * nd + int(10 * spread), spread)
    want = F.grid_sample(torch.from_numpy(data), _grid(pts, nd), mode="bilinear",
                         padding_mode=padding, align_corners=True)
    got = O.grid_sample_points(data, pts, padding)
    np.testing.assert_allclose(got, want.reshape(got.shape).numpy(), rtol=1e-5, atol=1e-6)


@pytest.mark.parametrize("nd", [2, 3])
@pytest.mark.parametrize("padding", ["zeros", "border", "reflection"])
@pytest.mark.parametrize("spread", [0.0, 0.7])
def test_sampling_gradients_match_torch_autograd(nd, padding, spread):
    data, pts = _case(nd, 100 + 10 * nd + int(10 * spread), spread)
    rng = np.random.default_rng(7)
    x = torch.from_numpy(data).requires_grad_(True)
    p = torch.from_numpy(pts).requires_grad_(True)
    g = p * 2 - 1                                      # the STN's points * 2 - 1
    grid = g.flip(1).transpose(1, 2).reshape(pts.shape[0], *([1] * (nd - 1)), pts.shape[2], nd)
    out = F.grid_sample(x, grid, mode="bilinear", padding_mode=padding, align_corners=True)
    w = rng.standard_normal(out.shape).astype(np.float32)
    (out * torch.from_numpy(w)).sum().backward()
    dp, dd = O.grid_sample_points_backward(data, pts, w.reshape(w.shape[0], w.shape[1], -1),
                                           padding)
    np.testing.assert_allclose(dp, p.grad.numpy(), rtol=1e-4, atol=1e-5)
    np.testing.assert_allclose(dd, x.grad.numpy(), rtol=1e-5, atol=1e-6)


def test_shared_image_is_broadcast():
    data, pts = _case(2, 3, 0.3)
    one = data[:1]
    np.testing.assert_array_equal(O.grid_sample_points(one, pts),
                                  O.grid_sample_points(np.repeat(one, 3, axis=0), pts))
    g = np.ones((3, data.shape[1], pts.shape[2]), np.float32)
    _, dd1 = O.grid_sample_points_backward(one, pts, g)
    _, dd3 = O.grid_sample_points_backward(np.repeat(one, 3, axis=0), pts, g)
    np.testing.assert_allclose(dd1[0], dd3.sum(0), rtol=1e-5, atol=1e-5)
