"""Public API behaviour on the GPU: chains, batching, errors, streams and
devices, CUDA graph capture, and the sharded (multi-rank) gradient."""
import numpy as np
import pytest
import torch

from cpab import _native
from cpab.distributed import shard_points, transform_grid_sharded
from oracle import oracle as O
from helpers import DTHETA_RTOL, X_ATOL, cpab, rand_points, rand_theta, rel_l2

pytestmark = [pytest.mark.gpu,
              pytest.mark.skipif(not torch.cuda.is_available(), reason="needs a CUDA GPU")]
DEV = "cuda"


@pytest.mark.parametrize("nc,scale_by_dt", [((8,), True), ((6, 6), True), ((3, 3, 3), False)])
def test_transform_grid_chain_matches_oracle(nc, scale_by_dt):
    C = cpab(nc)
    nd = len(nc)
    K = 3
    thc = rand_theta(K, C.params.d, 21, 0.5)
    pts = rand_points(nd, 3000, 22)
    th_t = torch.from_numpy(thc).to(DEV).requires_grad_(True)
    out = C.transform_grid_chain(torch.from_numpy(pts).to(DEV), th_t, scale_by_dt=scale_by_dt)
    w = rand_points(nd, 3000, 23, -1, 1)[None]
    (out * torch.from_numpy(w).to(DEV)).sum().backward()
    dt = 1.0 / K if scale_by_dt else 1.0
    x = pts
    stages = []
    for k in range(K):
        xk, As, _ = O.transform(list(nc), C.params.basis, x, thc[k:k + 1] * dt)
        stages.append((x, As))
        x = xk
    assert np.abs(out.detach().cpu().numpy() - x).max() <= 2 * X_ATOL
    g = w
    grads = []
    for k in reversed(range(K)):
        xin, As = stages[k]
        mom, gp = O.adjoint(list(nc), xin, As, g)
        grads.append(O.project(C.params.basis, mom)[0] * dt)
        g = gp if xin.ndim == 3 else gp
    ref = np.stack(grads[::-1])
    assert rel_l2(th_t.grad.cpu().numpy(), ref) < 1e-3


def test_errors_raise():
    C = cpab((4, 4))
    th = C.identity(2)
    with pytest.raises(ValueError):
        C.transform_grid(torch.rand(3, 10, device=DEV), th)
    with pytest.raises(AssertionError):
        C.transform_grid(torch.rand(3, 2, 10, device=DEV), th)
    C.set_solver_params(_native.max_steps() + 1)
    try:
        with pytest.raises(_native.CpabNativeError, match="nstepsolver"):
            C.transform_grid(torch.rand(2, 10, device=DEV), th)
    finally:
        C.set_solver_params(50)
    with pytest.raises(TypeError):
        C.transform_grid(torch.rand(2, 10, device=DEV), th.double())


def test_empty_inputs():
    C = cpab((4, 4))
    out = C.transform_grid(torch.rand(2, 0, device=DEV), C.identity(2))
    assert out.shape == (2, 2, 0)


def test_runs_on_side_stream_and_non_default_device():
    C = cpab((6, 6))
    th = torch.from_numpy(rand_theta(2, C.params.d, 3)).to(DEV)
    pts = torch.rand(2, 5000, device=DEV)
    ref = C.transform_grid(pts, th)
    s = torch.cuda.Stream()
    with torch.cuda.stream(s):
        out = C.transform_grid(pts, th)
    s.synchronize()
    assert torch.equal(out, ref)
    if torch.cuda.device_count() > 1:
        d1 = torch.device("cuda:1")
        out1 = C.transform_grid(pts.to(d1), th.to(d1))
        assert torch.equal(out1.cpu(), ref.cpu())


def test_cuda_graph_capture_of_forward_and_backward():
    C = cpab((8, 8))
    th = torch.from_numpy(rand_theta(4, C.params.d, 5)).to(DEV).requires_grad_(True)
    pts = torch.rand(2, 4000, device=DEV)
    tgt = torch.rand(4, 2, 4000, device=DEV)

    def step():
        th.grad = None
        out = C.transform_grid(pts, th)
        ((out - tgt) ** 2).mean().backward()
        return th.grad

    eager = step().clone()
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        for _ in range(2):
            step()
    torch.cuda.current_stream().wait_stream(s)
    g = torch.cuda.CUDAGraph()
    th.grad = None
    with torch.cuda.graph(g):
        out = C.transform_grid(pts, th)
        loss = ((out - tgt) ** 2).mean()
        grad = torch.autograd.grad(loss, th)[0]
    g.replay()
    torch.cuda.synchronize()
    assert rel_l2(grad.cpu().numpy(), eager.cpu().numpy()) < 1e-5


def test_sharded_gradient_equals_full_single_process():
    """Shards processed one after another in one process, summed, equal the
    unsharded gradient (the multi-rank path adds only the allreduce)."""
    C = cpab((10, 10))
    th = torch.from_numpy(rand_theta(3, C.params.d, 8)).to(DEV)
    pts = torch.rand(2, 9001, device=DEV)
    w = torch.randn(3, 2, 9001, device=DEV)
    t_full = th.clone().requires_grad_(True)
    (C.transform_grid(pts, t_full) * w).sum().backward()
    acc = torch.zeros_like(th)
    for r in range(4):
        t_r = th.clone().requires_grad_(True)
        out = transform_grid_sharded(C, shard_points(pts, r, 4), t_r, group=None)
        (out * shard_points(w, r, 4)).sum().backward()
        acc += t_r.grad
    assert rel_l2(acc.cpu().numpy(), t_full.grad.cpu().numpy()) < 1e-5


def test_order_cache_reuses_and_invalidates():
    """The processing order is cached for the same points tensor, recomputed
    after an in-place change, and never changes results."""
    from cpab.pytorch import transformer as tr
    C = cpab((6, 6))
    pts = torch.from_numpy(rand_points(2, 20000, 31)).to(DEV)
    th = torch.from_numpy(rand_theta(3, C.params.d, 32)).to(DEV)
    C.params.__dict__.pop("_order_cache", None)
    out1 = C.transform_grid(pts, th)
    o1 = C.params._order_cache[pts.device][1]
    out2 = C.transform_grid(pts, th)
    assert C.params._order_cache[pts.device][1] is o1  # reused
    assert torch.equal(out1, out2)
    pts.mul_(0.5)  # in place: version counter moves, order is rebuilt
    out3 = C.transform_grid(pts, th)
    o3 = C.params._order_cache[pts.device][1]
    assert o3 is not o1
    # a stale order only changes which thread integrates which point
    C.params._order_cache[pts.device] = (C.params._order_cache[pts.device][0], o1)
    out4 = C.transform_grid(pts, th)
    assert torch.equal(out3, out4)
    # and an order for the right points is a permutation
    assert torch.equal(torch.sort(o3.flatten())[0], torch.arange(20000, device=DEV, dtype=torch.int32))
    assert tr.ORDER_MIN_POINTS <= 20000


def test_sample_transformation_with_prior_on_gpu():
    """Samples of the smooth prior: right shape, and their empirical covariance
    follows the prior's (checked on the largest-variance directions)."""
    C = cpab((4, 4))
    torch.manual_seed(3)
    th = C.sample_transformation_with_prior(20000, length_scale=0.2, output_variance=1.0)
    assert th.shape == (20000, C.params.d) and th.is_cuda and torch.isfinite(th).all()
    cov = C._prior_covariance(0.2, 1.0).double()
    emp = torch.cov(th.double().t())
    top = torch.argsort(torch.diagonal(cov), descending=True)[:20]
    rel = (torch.diagonal(emp)[top] - torch.diagonal(cov)[top]).abs() / torch.diagonal(cov)[top]
    assert float(rel.max()) < 0.1   # 20000 samples: ~1% standard error per variance
