"""A whole training step (A-build, point sort, forward, loss, backward,
projection) captured in one CUDA graph and replayed: the replays must give
the eager results, also after new inputs are copied into the captured
buffers (the point sort is recorded into the graph, so it follows them).
Nothing the library caches may be built inside a capture."""
import pytest
import torch
import torch.nn.functional as F

from cpab import Cpab
from cpab.pytorch.transformer import clear_order_cache

pytestmark = [pytest.mark.gpu,
              pytest.mark.skipif(not torch.cuda.is_available(), reason="needs a CUDA GPU")]
DEV = torch.device("cuda")
DTHETA_RTOL = 1e-4   # relative L2 of dtheta (fp32 moment sums in a different order)


def _capture(fn, *static):
    """Warm fn up on a side stream, then capture one call; returns (graph, outputs)."""
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        for _ in range(2):
            fn(*static)
    torch.cuda.current_stream().wait_stream(s)
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        out = fn(*static)
    return g, out


def _rel(a, b):
    return float((a - b).norm() / b.norm())


def _grid_step(C):
    def step(theta, pts):
        theta.grad = None
        out = C.transform_grid(pts, theta)
        loss = F.mse_loss(out, pts.expand_as(out))
        loss.backward()
        return out, loss, theta.grad
    return step


def _eager(step, theta, pts):
    t = theta.detach().clone().requires_grad_(True)
    out, loss, grad = step(t, pts)
    return out.detach(), loss.detach(), grad.detach()


@pytest.mark.parametrize("tess,nP", [((20, 20), 20000), ((4, 4, 4), 12000)])
def test_graphed_transform_grid_step_matches_eager(tess, nP):
    C = Cpab(list(tess), zero_boundary=True)
    gen = torch.Generator().manual_seed(5)
    th0 = torch.randn(3, C.params.d, generator=gen).to(DEV)
    p0 = torch.rand(len(tess), nP, generator=gen).to(DEV)
    step = _grid_step(C)

    theta = th0.clone().requires_grad_(True)
    pts = p0.clone()
    clear_order_cache(C.params)
    g, (out, loss, grad) = _capture(step, theta, pts)

    for rep in range(3):
        if rep:  # new inputs in the captured buffers
            with torch.no_grad():
                theta.copy_(torch.randn(3, C.params.d, generator=gen).to(DEV))
            pts.copy_(torch.rand(len(tess), nP, generator=gen).to(DEV))
        g.replay()
        torch.cuda.synchronize()
        e_out, e_loss, e_grad = _eager(step, theta, pts.clone())
        assert torch.equal(out, e_out), rep
        assert abs(float(loss.detach()) - float(e_loss)) <= 1e-6 * abs(float(e_loss)), rep
        assert _rel(grad, e_grad) < DTHETA_RTOL, rep


def test_graphed_capture_leaves_no_cached_order_behind():
    C = Cpab([8, 8], zero_boundary=True)
    theta = torch.randn(2, C.params.d, device=DEV).requires_grad_(True)
    pts = torch.rand(2, 8192, device=DEV)
    clear_order_cache(C.params)
    g, _ = _capture(_grid_step(C), theta, pts)
    # the eager warm-up calls cached their order; the captured call must not
    # have replaced it with the never-run graph's buffer
    entry = C.params.__dict__["_order_cache"][pts.device][1]
    assert sorted(entry[0].tolist()) == list(range(8192))
    del g


def test_graphed_transform_data_and_chain_match_eager():
    gen = torch.Generator().manual_seed(7)
    C3 = Cpab([3, 3, 3], zero_boundary=True)
    data = torch.rand(2, 1, 24, 24, 24, generator=gen).to(DEV)
    th3 = torch.randn(2, C3.params.d, generator=gen).to(DEV)

    def data_step(theta, x):
        theta.grad = None
        out = C3.transform_data(x, theta, outsize=(20, 20, 20))
        loss = out.square().mean()
        loss.backward()
        return out, theta.grad

    C2 = Cpab([6, 6], zero_boundary=True)
    thc = torch.randn(3, 2, C2.params.d, generator=gen).to(DEV)
    grid = C2.uniform_meshgrid([64, 80], device=DEV)

    def chain_step(theta, pts):
        theta.grad = None
        out = C2.transform_grid_chain(pts, theta, scale_by_dt=True)
        loss = (out - pts).square().sum()
        loss.backward()
        return out, theta.grad

    for step, th, x in ((data_step, th3, data), (chain_step, thc, grid)):
        theta = th.clone().requires_grad_(True)
        g, (out, grad) = _capture(step, theta, x)
        g.replay()
        torch.cuda.synchronize()
        t = th.clone().requires_grad_(True)
        e_out, e_grad = step(t, x)
        assert torch.allclose(out, e_out, atol=1e-6, rtol=0)
        assert _rel(grad, e_grad) < DTHETA_RTOL
