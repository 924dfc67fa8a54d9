"""The CPA basis B equals the reference's, entry for entry (golden fixtures
from the reference's cpab/core/tesselation.py, tests/golden/make_golden.py)."""
import os
import pickle

import numpy as np
import pytest
import scipy.sparse as sp

from cpab.core.tesselation import Tesselation1D, Tesselation2D, Tesselation3D

GOLDEN = np.load(os.path.join(os.path.dirname(__file__), "golden", "basis_golden.npz"))
KEYS = sorted({k.rsplit("_", 1)[0] for k in GOLDEN.files})
CLASSES = {1: Tesselation1D, 2: Tesselation2D, 3: Tesselation3D}


def parse(key):
    d, size, zb, vp = key.split("_")
    nc = [int(s) for s in size.split("x")]
    return nc, zb == "zb1", vp == "vp1"


def golden_B(key):
    return sp.csr_matrix((GOLDEN[key + "_data"], GOLDEN[key + "_indices"], GOLDEN[key + "_indptr"]),
                         shape=tuple(GOLDEN[key + "_shape"]))


@pytest.mark.parametrize("key", KEYS)
def test_basis_equals_reference(key):
    nc, zb, vp = parse(key)
    t = CLASSES[len(nc)](nc, [0] * len(nc), [1] * len(nc), zb, vp, None, True)
    ref = golden_B(key)
    assert t.B.shape == ref.shape
    assert (t.B != ref).nnz == 0, "basis differs from the reference"


@pytest.mark.parametrize("key", [k for k in KEYS if "d3" not in k or "2x2x2" in k])
def test_basis_spans_constraint_null_space(key):
    nc, zb, vp = parse(key)
    t = CLASSES[len(nc)](nc, [0] * len(nc), [1] * len(nc), zb, vp, None, True)
    if t.B.shape[1] == 0:
        return
    resid = abs(t.L @ t.B)
    assert resid.max() < 1e-6 if resid.nnz else True
    norms = np.sqrt(np.asarray(t.B.power(2).sum(axis=0))).ravel()
    np.testing.assert_allclose(norms, 1.0, rtol=1e-12)


def test_cache_roundtrip_and_reference_pickle(tmp_path):
    t1 = Tesselation2D([3, 2], [0, 0], [1, 1], False, False, str(tmp_path), False)
    t2 = Tesselation2D([3, 2], [0, 0], [1, 1], False, False, str(tmp_path), False)
    assert (t1.B != t2.B).nnz == 0
    # A basis cached by the reference (pickled __dict__ with B) is read as is.
    stem = tmp_path / t1._stem()
    os.remove(str(stem) + ".npz")
    fake = sp.random(144, 5, density=0.1, format="csr", random_state=0)
    with open(str(stem) + ".pkl", "wb") as f:
        pickle.dump({"B": fake, "nodal_vertices": np.zeros((0, 3))}, f)
    t3 = Tesselation2D([3, 2], [0, 0], [1, 1], False, False, str(tmp_path), False)
    assert (t3.B != fake).nnz == 0


def test_cell_centers_and_counts():
    t = Tesselation3D([2, 3, 4], [0, 0, 0], [1, 1, 1], True, False, None, True)
    assert t.nC == 5 * 24 and t.verts.shape == (120, 4, 4)
    c = t.get_cell_centers()
    assert c.shape == (120, 3) and c.min() > 0 and c.max() < 1
