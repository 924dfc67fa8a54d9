"""The CPU oracle: pinned to the reference's golden fixtures and checked
against the mathematics it restates."""
import os

import numpy as np
import pytest

from oracle import oracle as O
from helpers import cpab, rand_points, rand_theta, rel_l2

GOLD = os.path.join(os.path.dirname(__file__), "golden")
INTERP = np.load(os.path.join(GOLD, "interp_golden.npz"))
INTERP_KEYS = sorted({k.split("_")[0] for k in INTERP.files})


def meta(key):
    m = INTERP[key + "_meta"].tolist()
    nd, B, C = m[:3]
    return nd, B, C, m[3:3 + nd], m[3 + nd:3 + 2 * nd]


@pytest.mark.parametrize("key", INTERP_KEYS)
def test_interpolate_matches_reference_bitwise(key):
    nd, B, C, insz, outsz = meta(key)
    out = O.interpolate(nd, INTERP[key + "_data"], INTERP[key + "_grid"], outsz)
    np.testing.assert_array_equal(out, INTERP[key + "_out"])


@pytest.mark.parametrize("key", INTERP_KEYS)
def test_interpolate_gradient_matches_reference(key):
    nd, B, C, insz, outsz = meta(key)
    dg, dd = O.interpolate_backward(nd, INTERP[key + "_data"], INTERP[key + "_grid"], outsz,
                                    INTERP[key + "_w"])
    np.testing.assert_allclose(dg, INTERP[key + "_dgrid"], rtol=1e-5, atol=1e-5)
    np.testing.assert_allclose(dd, INTERP[key + "_ddata"], rtol=1e-5, atol=1e-6)


KERNEL_GOLDEN = os.path.join(GOLD, "kernel_golden.npz")


@pytest.mark.skipif(not os.path.exists(KERNEL_GOLDEN), reason="kernel golden not generated yet")
def test_oracle_matches_reference_kernels():
    """Outputs of the reference's CUDA kernels (run on a B200 through
    oracle/_ref, tests/golden/make_kernel_golden.py) versus the oracle."""
    G = np.load(KERNEL_GOLDEN)
    for key in sorted({k.split("__")[0] for k in G.files}):
        nc = G[key + "__nc"].tolist()
        T, adaptive, batched = G[key + "__cfg"].tolist()
        pts, As = G[key + "__points"], G[key + "__As"]
        nd = len(nc)
        trels = O.expm(As, 1.0 / T) if nd > 1 else None
        if nd > 1:
            np.testing.assert_allclose(trels, G[key + "__trels"], rtol=2e-6, atol=2e-7)
            trels = G[key + "__trels"]          # integrate the reference's Trels
        x = O.integrate(nc, pts, As, trels, T, adaptive)
        np.testing.assert_allclose(x, G[key + "__out"], rtol=0, atol=1e-5, err_msg=key)
        flat = x.transpose(1, 0, 2).reshape(nd, -1)
        ref_flat = G[key + "__out"].transpose(1, 0, 2).reshape(nd, -1)
        from helpers import near_boundary
        differ = O.cells(nc, flat) != O.cells(nc, ref_flat)
        assert not (differ & ~near_boundary(nc, ref_flat)).any(), key
        mom, gp = O.adjoint(nc, pts, As, G[key + "__grad"], T, adaptive)
        assert rel_l2(mom, G[key + "__moments"]) < 1e-5, key
        np.testing.assert_allclose(gp, G[key + "__grad_points"], rtol=1e-4, atol=1e-5, err_msg=key)


@pytest.mark.parametrize("nc", [[6], [3, 3], [2, 2, 2]])
def test_zero_theta_is_identity(nc):
    T = cpab(tuple(nc))
    pts = rand_points(len(nc), 500, 3)
    th = np.zeros((2, T.params.d), np.float32)
    x, As, trels = O.transform(nc, T.params.basis, pts, th)
    np.testing.assert_array_equal(x, np.broadcast_to(pts, x.shape))


@pytest.mark.parametrize("nc,adaptive", [([5], False), ([2, 2], False), ([2, 2], True),
                                          ([2, 2, 2], False), ([2, 2, 2], True)])
def test_adjoint_is_gradient_of_midpoint_replay(nc, adaptive):
    """dtheta from the adjoint equals central finite differences of the
    midpoint-rule trajectory it differentiates (float32, loose tolerance)."""
    T = cpab(tuple(nc))
    nd = len(nc)
    d = T.params.d
    pts = rand_points(nd, 64, 11, 0.05, 0.95)
    th = rand_theta(1, d, 12, 0.5)
    w = rand_points(nd, 64, 13, -1, 1)[None]
    As = O.build_A(T.params.basis, th, nd)
    mom, _ = O.adjoint(nc, pts, As, w, 20, adaptive)
    g = O.project(T.params.basis, mom)[0]
    rng = np.random.default_rng(0)
    for _ in range(3):
        v = rng.standard_normal(d).astype(np.float32)
        eps = 1e-2
        lp = (w * O.midpoint_integrate(nc, pts, O.build_A(T.params.basis, th + eps * v, nd), 20,
                                       adaptive)).sum(dtype=np.float64)
        lm = (w * O.midpoint_integrate(nc, pts, O.build_A(T.params.basis, th - eps * v, nd), 20,
                                       adaptive)).sum(dtype=np.float64)
        fd = (lp - lm) / (2 * eps)
        an = float(np.dot(g.astype(np.float64), v))
        assert abs(fd - an) <= 2e-2 * max(1.0, abs(an)), (fd, an)


def test_expm_against_series():
    rng = np.random.default_rng(1)
    for nd in (1, 2, 3):
        A = rng.standard_normal((40, nd, nd + 1)).astype(np.float32) * 3
        got = O.expm(A, 0.1)
        M = np.zeros((40, nd + 1, nd + 1))
        M[:, :nd] = 0.1 * A
        E = np.stack([_expm(m) for m in M])[:, :nd]
        np.testing.assert_allclose(got, E, rtol=2e-4, atol=2e-5)


def _expm(m):
    import scipy.linalg
    return scipy.linalg.expm(m)


def test_cycle_consistency_2d():
    T = cpab((4, 4))
    pts = rand_points(2, 400, 5, 0.1, 0.9)
    th = rand_theta(1, T.params.d, 6, 0.3)
    x, _, _ = O.transform([4, 4], T.params.basis, pts, th)
    back, _, _ = O.transform([4, 4], T.params.basis, x, -th)
    assert np.abs(back[0] - pts).max() < 5e-3
