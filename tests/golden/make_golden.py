"""Generate golden fixtures from the reference implementation's own Python code.

    python tests/golden/make_golden.py [path/to/reference]

Needs the reference source tree: the path argument, else $CPAB_REFERENCE, else
a directory "reference" beside this repository.  It is copied to a
temporary directory first because constructing a reference tessellation writes
a basis cache next to the package.  The reference's cpab/__init__.py
JIT-compiles CUDA, so cpab.core and cpab.pytorch.interpolation are loaded as
plain modules without it (both run on CPU).

Writes:
  basis_golden.npz   the CPA basis B (CSR arrays) of small tessellations in
                     1D/2D/3D with zero_boundary / volume_perservation on and
                     off (cpab/core/tesselation.py)
  interp_golden.npz  interpolate{1,2,3}D outputs on seeded data and grids,
                     plus d(sum(out * w))/d(grid, data) from torch autograd
                     (cpab/pytorch/interpolation.py)
"""
import os
import shutil
import sys
import tempfile
import types

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))

BASIS_CASES = [
    ([5], True, False), ([5], False, False), ([5], False, True), ([7], True, False),
    ([2, 2], True, False), ([3, 3], False, False), ([3, 2], False, True), ([3, 3], True, True),
    ([4, 3], False, False), ([5, 5], True, False), ([1, 1], False, False),
    ([2, 2, 2], True, False), ([2, 2, 2], False, False), ([2, 3, 2], False, False),
    ([3, 2, 2], False, True), ([3, 3, 3], True, False),
]

INTERP_CASES = [
    # (ndim, batch, channels, in_size, out_size, grid spread)
    (1, 2, 3, [17], [23], 0.2),
    (2, 2, 3, [13, 9], [11, 7], 0.2),
    (2, 1, 1, [8, 8], [8, 8], 0.0),
    (3, 2, 2, [7, 6, 5], [5, 4, 6], 0.2),
]


def load_reference(ref_root):
    tmp = tempfile.mkdtemp(prefix="cpab_ref_")
    shutil.copytree(os.path.join(ref_root, "cpab"), os.path.join(tmp, "cpab"))
    pkg = types.ModuleType("cpab")
    pkg.__path__ = [os.path.join(tmp, "cpab")]
    sys.modules["cpab"] = pkg
    sys.path.insert(0, tmp)
    import cpab.core.tesselation as tess  # noqa: E402
    import cpab.pytorch.interpolation as interp  # noqa: E402
    return tmp, tess, interp


def case_key(nc, zb, vp):
    return "d%d_%s_zb%d_vp%d" % (len(nc), "x".join(map(str, nc)), int(zb), int(vp))


def main():
    # The reference checkout: first argument, else $CPAB_REFERENCE, else a
    # sibling of this repository named "reference".
    ref_root = (sys.argv[1] if len(sys.argv) > 1 else
                os.environ.get("CPAB_REFERENCE",
                               os.path.join(HERE, os.pardir, os.pardir, os.pardir, "reference")))
    tmp, tess, interp = load_reference(ref_root)
    import torch

    out = {}
    for nc, zb, vp in BASIS_CASES:
        cls = getattr(tess, "Tesselation%dD" % len(nc))
        t = cls(nc, [0] * len(nc), [1] * len(nc), zb, vp, os.path.join(tmp, "basis_"), True)
        B = t.B.tocsr()
        B.sort_indices()
        k = case_key(nc, zb, vp)
        out[k + "_data"] = B.data
        out[k + "_indices"] = B.indices
        out[k + "_indptr"] = B.indptr
        out[k + "_shape"] = np.asarray(B.shape)
    np.savez_compressed(os.path.join(HERE, "basis_golden.npz"), **out)

    out = {}
    rng = np.random.default_rng(20261201)
    for n, (nd, B, C, insz, outsz, spread) in enumerate(INTERP_CASES):
        data = rng.random((B, C, *insz), dtype=np.float32)
        P = int(np.prod(outsz))
        lin = [np.linspace(0, 1, s, dtype=np.float32) for s in outsz]
        mesh = np.meshgrid(*lin[::-1], indexing="ij")
        base = np.stack([m.reshape(-1) for m in mesh[::-1]])          # coordinate 0 fastest
        grid = base[None] + spread * rng.standard_normal((B, nd, P)).astype(np.float32)
        grid = grid.astype(np.float32)
        w = rng.standard_normal((B, C, *outsz)).astype(np.float32)
        d_t = torch.from_numpy(data).requires_grad_(True)
        g_t = torch.from_numpy(grid).requires_grad_(True)
        y = interp.interpolate(nd, d_t, g_t, outsz)
        (y * torch.from_numpy(w)).sum().backward()
        key = "c%d" % n
        out[key + "_data"] = data
        out[key + "_grid"] = grid
        out[key + "_w"] = w
        out[key + "_out"] = y.detach().numpy()
        out[key + "_dgrid"] = g_t.grad.numpy()
        out[key + "_ddata"] = d_t.grad.numpy()
        out[key + "_meta"] = np.asarray([nd, B, C] + insz + outsz)
    np.savez_compressed(os.path.join(HERE, "interp_golden.npz"), **out)
    shutil.rmtree(tmp, ignore_errors=True)
    print("wrote basis_golden.npz and interp_golden.npz to", HERE)


if __name__ == "__main__":
    main()
