"""Golden outputs of the reference's CUDA kernels (needs a GPU and
oracle/_ref/libcpab_ref.so, built by oracle/build_oracle.py --ref).

    python tests/golden/make_kernel_golden.py OUT.npz

Small seeded cases in 1D/2D/3D; for each: points, As, the reference's Trels
(its expm kernel), its forward output, an upstream gradient, and its
moments and grad_points.  tests/test_oracle.py checks the CPU oracle against
this file, pinning the oracle to the reference's kernels.
"""
import os
import sys

import numpy as np
import torch

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path[:0] = [os.path.dirname(HERE), os.path.join(os.path.dirname(os.path.dirname(HERE)),
                                                    "fg-cpab_b200"),
                os.path.dirname(os.path.dirname(HERE))]
import refkernels as R  # noqa: E402
from helpers import cpab, rand_points, rand_theta  # noqa: E402
from oracle import oracle as O  # noqa: E402

CASES = [("d1", (10,), True, 3, 300, False, False, 50),
         ("d1b", (6,), False, 2, 300, True, False, 50),
         ("d2", (5, 5), True, 3, 400, False, False, 50),
         ("d2o", (4, 3), False, 2, 400, True, False, 30),
         ("d2a", (4, 4), True, 2, 400, False, True, 50),
         ("d3", (3, 3, 3), True, 2, 300, False, False, 50),
         ("d3o", (2, 3, 2), False, 2, 300, True, True, 40)]


def main(out_path):
    out = {}
    for key, nc, zb, n_theta, nP, batched, adaptive, T in CASES:
        C = cpab(nc, zb)
        nd = len(nc)
        th = rand_theta(n_theta, C.params.d, 50)
        lo, hi = (0, 1) if zb else (-0.2, 1.2)
        pts = (np.stack([rand_points(nd, nP, 60 + b, lo, hi) for b in range(n_theta)])
               if batched else rand_points(nd, nP, 60, lo, hi))
        As = O.build_A(C.params.basis, th, nd)
        As_d = torch.from_numpy(As).cuda()
        pts_d = torch.from_numpy(pts).cuda()
        trels = R.expm(As_d, 1.0 / T) if nd > 1 else None
        x = R.forward(nc, pts_d, batched, trels, As_d, T, adaptive)
        g = rand_points(nd, n_theta * nP, 70, -1, 1).reshape(nd, n_theta, nP).transpose(1, 0, 2).copy()
        mom, gp = R.backward(nc, pts_d, batched, As_d, torch.from_numpy(g).cuda(), T, adaptive)
        out[key + "__nc"] = np.asarray(nc)
        out[key + "__cfg"] = np.asarray([T, int(adaptive), int(batched)])
        out[key + "__points"] = pts
        out[key + "__As"] = As
        if trels is not None:
            out[key + "__trels"] = trels.cpu().numpy()
        out[key + "__out"] = x.cpu().numpy()
        out[key + "__grad"] = g
        out[key + "__moments"] = mom.cpu().numpy()
        out[key + "__grad_points"] = gp.cpu().numpy()
    np.savez_compressed(out_path, **out)
    print("wrote", out_path)


if __name__ == "__main__":
    main(sys.argv[1] if len(sys.argv) > 1 else os.path.join(HERE, "kernel_golden.npz"))
