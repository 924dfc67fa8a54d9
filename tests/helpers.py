"""Shared test helpers: seeded inputs, cached tessellations, tolerances."""
import functools

import numpy as np
import torch

from oracle import oracle as O

# Tolerances of the hot path's parity bar.
X_ATOL = 1e-5          # warped coordinates, absolute
DTHETA_RTOL = 1e-4     # dtheta, relative L2
BOUNDARY_EPS = 1e-6    # cell indices may differ only this close to a facet


@functools.lru_cache(maxsize=None)
def cpab(nc, zero_boundary=True, volume_perservation=False):
    from cpab import Cpab
    return Cpab(list(nc), zero_boundary=zero_boundary, volume_perservation=volume_perservation)


def rel_l2(a, b):
    a = np.asarray(a, dtype=np.float64)
    b = np.asarray(b, dtype=np.float64)
    return float(np.linalg.norm(a - b) / max(np.linalg.norm(b), 1e-30))


def seeded(seed):
    return torch.Generator().manual_seed(seed)


def rand_theta(n, d, seed, scale=1.0):
    return (torch.randn(n, d, generator=seeded(seed)) * scale).numpy().astype(np.float32)


def rand_points(ndim, n, seed, lo=0.0, hi=1.0):
    g = seeded(seed)
    return (lo + (hi - lo) * torch.rand(ndim, n, generator=g)).numpy().astype(np.float32)


def near_boundary(nc, points, eps=BOUNDARY_EPS):
    """Mask of points [ndim, n] whose cell changes under some perturbation of
    size eps (axis-aligned and diagonal), i.e. within ~eps of a facet."""
    pts = np.asarray(points, dtype=np.float32)
    nd = pts.shape[0]
    base = O.cells(nc, pts)
    mask = np.zeros(pts.shape[1], dtype=bool)
    dirs = []
    for k in range(nd):
        e = np.zeros(nd, np.float32)
        e[k] = 1
        dirs += [e, -e]
    if nd >= 2:
        for s0 in (-1, 1):
            for s1 in (-1, 1):
                e = np.zeros(nd, np.float32)
                e[0], e[1] = s0, s1
                dirs.append(e / np.sqrt(2))
                if nd == 3:
                    for s2 in (-1, 1):
                        e3 = np.array([s0, s1, s2], np.float32) / np.sqrt(3)
                        dirs.append(e3)
    for e in dirs:
        mask |= O.cells(nc, pts + eps * e[:, None]) != base
    return mask
