"""Host-side logic that needs no GPU: the Cpab API surface, argument
checks, grid layout, sharding."""
import os

import numpy as np
import pytest
import torch

from cpab import Cpab
from cpab.distributed import shard_bounds, shard_points
from cpab.pytorch.transformer import CPAB_transformer
from helpers import cpab


def test_params_fields_match_reference_layout():
    T = cpab((20, 20))
    p = T.params
    assert (p.ndim, p.nC, p.params_pr_cell, p.D, p.d) == (2, 1600, 6, 9600, 1522)
    assert p.Ashape == [2, 3] and p.nstepsolver == 50 and p.adaptive_substeps is False
    assert T.get_theta_dim() == 1522 and T.get_basis() is p.basis
    assert p.zero_boundary and not p.valid_outside
    assert "theta length d" in repr(T)


def test_constraint_matrix_is_lazy():
    T = Cpab([3, 3], zero_boundary=False)
    assert "constrain_mat" not in T.params.__dict__
    L = T.params.constrain_mat
    assert L.shape[1] == T.params.D and "constrain_mat" in T.params.__dict__


@pytest.mark.parametrize("args", [("20x20",), ([20, 0],), ([2.0, 2],), ([1, 2, 3, 4],)])
def test_constructor_checks(args):
    with pytest.raises(AssertionError):
        Cpab(*args)


def test_solver_param_checks():
    T = cpab((4,))
    with pytest.raises(AssertionError):
        T.set_solver_params(0)
    with pytest.raises(AssertionError):
        T.set_solver_params(10.0)
    with pytest.raises(AssertionError):
        T.set_solver_params(10, adaptive_substeps=1)


def test_meshgrid_has_coordinate_zero_fastest():
    T = cpab((2, 2, 2))
    g = T.uniform_meshgrid([3, 4, 5], device="cpu")
    assert g.shape == (3, 60)
    i0, i1, i2 = 2, 1, 3
    p = i0 + 3 * (i1 + 4 * i2)
    np.testing.assert_allclose(g[:, p].numpy(), [i0 / 2, i1 / 3, i2 / 4], rtol=1e-6)


def test_cpu_tensors_are_rejected():
    T = cpab((4, 4))
    with pytest.raises(AssertionError, match="Only GPU"):
        CPAB_transformer(torch.zeros(2, 5), torch.zeros(1, T.params.d), T.params)


@pytest.mark.parametrize("n,w", [(10, 3), (7, 8), (1000001, 8), (0, 2)])
def test_shard_bounds_partition(n, w):
    spans = [shard_bounds(n, r, w) for r in range(w)]
    assert spans[0][0] == 0 and spans[-1][1] == n
    assert all(a[1] == b[0] for a, b in zip(spans, spans[1:]))
    sizes = [hi - lo for lo, hi in spans]
    assert max(sizes) - min(sizes) <= 1


def test_shard_points_slices_last_axis():
    x = torch.arange(30.0).reshape(3, 10)
    parts = [shard_points(x, r, 3) for r in range(3)]
    assert torch.equal(torch.cat(parts, dim=1), x)


def _build_basis_in(direc, out_q):
    try:
        import sys
        sys.path[:0] = [os.path.join(os.path.dirname(os.path.dirname(os.path.abspath(__file__))),
                                     "fg-cpab_b200")]
        from cpab.core.tesselation import Tesselation2D
        T = Tesselation2D([9, 7], [0, 0], [1, 1], direc=direc)
        out_q.put(("ok", T.B.nnz))
    except BaseException as e:  # reported to the parent
        out_q.put(("error", repr(e)))


def test_basis_cache_survives_concurrent_writers(tmp_path):
    """One process per GPU builds the same basis on a fresh machine: all of
    them must succeed and leave one complete cache file."""
    import multiprocessing as mp
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=_build_basis_in, args=(str(tmp_path), q)) for _ in range(4)]
    for p in procs:
        p.start()
    results = [q.get(timeout=120) for _ in procs]
    for p in procs:
        p.join(timeout=60)
    assert all(r[0] == "ok" for r in results), results
    assert len({r[1] for r in results}) == 1
    files = sorted(f.name for f in tmp_path.iterdir())
    assert len(files) == 1 and files[0].endswith(".npz") and ".tmp" not in files[0]


def test_reference_helpers_exist():
    """Helpers of the reference's modules that user code may import."""
    from cpab.core.utility import make_hashable
    from cpab.pytorch.transformer import _get_sparse_basis
    assert make_hashable(np.array([[1, 2], [3, 4]])) == ((1, 2), (3, 4))
    C = Cpab([3, 3], zero_boundary=True)
    B = _get_sparse_basis(C.params, "cpu", torch.float64)
    assert B.is_sparse and tuple(B.shape) == C.params.basis.shape
    np.testing.assert_allclose(B.to_dense().numpy(), C.params.basis.toarray())


@pytest.mark.parametrize("tess,zb", [([5], True), ([3, 3], True), ([3, 2], False), ([2, 2, 2], True)])
def test_prior_covariance_equals_the_dense_construction(tess, zb):
    """sample_transformation_with_prior's covariance B^T K B against K built as
    the reference does: a dense D x D matrix, entry ((i,p),(j,q)) =
    v^2 exp(-M/(2 l^2)), M = |c_i - c_j|^2 when p == q, else 100 max |c_i - c_j|^2."""
    C = Cpab(tess, zero_boundary=zb)
    l, v = 0.15, 1.3
    cov = C._prior_covariance(l, v, device="cpu").double()
    ppc, nC = C.params.params_pr_cell, C.params.nC
    c = torch.tensor(C.tesselation.get_cell_centers(), dtype=torch.float32)
    norm = (c * c).sum(1, keepdim=True)
    dist = norm - 2 * c @ c.t() + norm.t()
    M = torch.full((nC * ppc, nC * ppc), float(100 * dist.max()))
    for k in range(ppc):
        M[k::ppc, k::ppc] = dist
    K = (v ** 2 * torch.exp(-(M / (2 * l ** 2)))).double()
    B = torch.from_numpy(C.params.basis.toarray()).double()
    ref = B.t() @ K @ B
    tol = 1e-5 * float(ref.abs().max())
    assert float((cov - ref).abs().max()) <= tol
    assert torch.allclose(cov, cov.t(), atol=tol)


def test_order_cache_is_bypassed_under_graph_capture(monkeypatch):
    """Inside a CUDA graph capture the point sort is recorded every call and
    nothing is cached (captured buffers hold no data until a replay); outside
    it the order of an unchanged points tensor is kept until cleared."""
    from cpab import _native
    from cpab.pytorch import transformer as tr

    calls = []

    def fake_order(nc, points, batched):
        calls.append(points.data_ptr())
        return torch.arange(points.shape[-1], dtype=torch.int32)[None]

    C = Cpab([4, 4])
    pts = torch.rand(2, 5000)
    monkeypatch.setattr(_native, "order_points", fake_order)
    monkeypatch.setattr(torch.cuda, "is_current_stream_capturing", lambda: True)
    tr.clear_order_cache(C.params)
    tr._order(C.params, pts, False)
    tr._order(C.params, pts, False)
    assert len(calls) == 2 and "_order_cache" not in C.params.__dict__
    monkeypatch.setattr(torch.cuda, "is_current_stream_capturing", lambda: False)
    o1 = tr._order(C.params, pts, False)
    assert tr._order(C.params, pts, False) is o1 and len(calls) == 3
    tr.clear_order_cache(C.params)
    tr._order(C.params, pts, False)
    assert len(calls) == 4
