"""The fused spatial-transformer warp (cpab.pytorch.warp.CpabWarp: the
reference's stn/stn.py:58-86 layer, integration and F.grid_sample in one
kernel each way) against

  * the reference layer's own composition (stn/stn.py:40-54,79-86: one
    CPAB_transformer call per transformation, then torch's F.grid_sample),
    on this package's transformer and on the reference's own CUDA kernels
    (oracle/_ref);
  * the oracle (its integration, adjoint and grid_sample restatement).

Tolerances: outputs within 2e-5 (images in [0, 1]), dtheta within 1e-4
relative L2, the image gradient within 2e-5 where both sides integrate with
the same kernels (else 1e-4 relative L2)."""
import numpy as np
import pytest
import torch
import torch.nn.functional as F

import refkernels as R
from cpab import _native
from cpab.pytorch.transformer import CPAB_transformer, _get_sparse_basis, device_basis
from cpab.pytorch.warp import CpabWarp, pixel_axes, warp
from helpers import rel_l2
from oracle import oracle as O

pytestmark = [pytest.mark.gpu,
              pytest.mark.skipif(not torch.cuda.is_available(), reason="needs a CUDA GPU")]
DEV = "cuda"
OUT_ATOL = 2e-5
DTHETA_RTOL = 1e-4


def composed(layer, x, thetas, transformer=CPAB_transformer):
    """The reference layer's forward, step by step (stn/stn.py:40-54 with
    CpabWarp.transform, :79-86), with `transformer` in place of
    CPAB_transformer."""
    size = x.shape[2:]
    f32 = dict(device=x.device, dtype=torch.float32)
    axes = [torch.linspace(-1, 1, s, **f32) if s > 1 else torch.zeros(1, **f32) for s in size]
    points = torch.stack(torch.meshgrid(*axes, indexing="ij")[::-1]).flatten(1)
    points = (points.flip(-2) + 1) / 2
    for theta in reversed(thetas):
        points = transformer(points, theta, layer.cpab.params, points.requires_grad)
    points = (points * 2 - 1).flip(-2)
    grid = points.transpose(1, 2).reshape(len(points), *size, -1)
    src = x.float()
    if len(size) == 1:  # a [B, C, 1, W] image sampled at y = 0
        grid = F.pad(grid, (0, 1)).unsqueeze(1)
        src = src.unsqueeze(2)
    out = F.grid_sample(src, grid, align_corners=True, padding_mode=layer.padding_mode)
    return out.squeeze(2) if len(size) == 1 else out


def _inputs(layer, B, C, size, K, seed, scale, shared=False):
    g = torch.Generator(DEV).manual_seed(seed)
    if shared:
        x = torch.rand(1, C, *size, device=DEV, generator=g).expand(B, -1, *([-1] * len(size)))
    else:
        x = torch.rand(B, C, *size, device=DEV, generator=g)
    thetas = [scale * torch.randn(B, layer.theta_dim, device=DEV, generator=g) for _ in range(K)]
    return x, thetas


def _run(fn, x, thetas, w):
    """fn(x, thetas), then d/d(theta_i) and d/dx of sum(out * w)."""
    xs = x.detach().clone().requires_grad_(True) if x.stride(0) != 0 else \
        x[:1].detach().clone().requires_grad_(True)
    xin = xs if x.stride(0) != 0 else xs.expand_as(x)
    ths = [t.detach().clone().requires_grad_(True) for t in thetas]
    out = fn(xin, ths)
    (out * w).sum().backward()
    return out.detach(), [t.grad for t in ths], xs.grad


# (tess, zero_boundary, K, padding, C, size, shared, theta scale)
CASES = [
    ((3, 3), False, 1, "zeros", 3, (32, 40), False, 0.7),
    ((3, 3), False, 2, "border", 3, (48, 48), True, 0.7),       # demo_2d's layer
    ((4, 4), True, 1, "reflection", 1, (29, 33), False, 1.0),
    ((3, 3), False, 3, "reflection", 2, (24, 20), False, 0.5),
    ((3, 3), False, 2, "zeros", 2, (1, 17), False, 0.5),        # a one-pixel axis
    ((30, 30), True, 1, "zeros", 1, (64, 64), False, 1.0),      # table and record in smem
    ((4, 4, 4), True, 2, "zeros", 1, (16, 18, 20), False, 1.0), # demo_3d's layer
    ((2, 3, 2), False, 1, "border", 2, (12, 10, 14), True, 0.5),
    ((2, 2, 2), False, 2, "reflection", 1, (9, 11, 7), False, 0.5),
]
IDS = ["%s-%s-K%d-%s-C%d%s" % ("x".join(map(str, c[0])), "zb" if c[1] else "free", c[2], c[3],
                               c[4], "-shared" if c[6] else "") for c in CASES]


@pytest.mark.parametrize("case", CASES, ids=IDS)
def test_fused_warp_matches_the_reference_composition(case):
    tess, zb, K, padding, C, size, shared, scale = case
    layer = CpabWarp(tess, zero_boundary=zb, padding_mode=padding)
    x, thetas = _inputs(layer, 3, C, size, K, 11, scale, shared)
    w = torch.randn(3, C, *size, device=DEV, generator=torch.Generator(DEV).manual_seed(5))
    out, gth, gx = _run(lambda a, t: layer(a, t), x, thetas, w)
    ref, rth, rx = _run(lambda a, t: composed(layer, a, t), x, thetas, w)
    assert out.shape == ref.shape == x.shape
    assert (out - ref).abs().max().item() <= OUT_ATOL
    for a, b in zip(gth, rth):
        assert rel_l2(a.cpu().numpy(), b.cpu().numpy()) < DTHETA_RTOL
    assert (gx - rx).abs().max().item() <= OUT_ATOL


def test_adaptive_substeps_match_the_composition():
    layer = CpabWarp((5, 4), zero_boundary=False, padding_mode="border")
    layer.cpab.set_solver_params(40, adaptive_substeps=True)
    x, thetas = _inputs(layer, 2, 2, (20, 26), 2, 3, 0.8)
    w = torch.randn(2, 2, 20, 26, device=DEV, generator=torch.Generator(DEV).manual_seed(1))
    out, gth, gx = _run(lambda a, t: layer(a, t), x, thetas, w)
    ref, rth, rx = _run(lambda a, t: composed(layer, a, t), x, thetas, w)
    assert (out - ref).abs().max().item() <= OUT_ATOL
    for a, b in zip(gth, rth):
        assert rel_l2(a.cpu().numpy(), b.cpu().numpy()) < DTHETA_RTOL
    assert (gx - rx).abs().max().item() <= OUT_ATOL


class _RefTransformer(torch.autograd.Function):
    """CPAB_transformer on the reference's own kernels: A = B theta
    (torch.sparse, cpab/pytorch/transformer.py:84-88), expm and forward
    integration, backward_moments_and_points, dtheta = B^T m (:165-166)."""

    @staticmethod
    def forward(ctx, points, theta, params, compute_points_grad):
        nd, T = params.ndim, int(params.nstepsolver)
        B = _get_sparse_basis(params, theta.device)
        As = torch.sparse.mm(B, theta.t()).t().reshape(theta.shape[0], params.nC, nd, nd + 1)
        As = As.contiguous()
        batched = points.dim() == 3
        out = R.forward(params.nc, points.contiguous(), batched, R.expm(As, 1.0 / T), As, T, False)
        ctx.save_for_backward(points.contiguous(), As)
        ctx.params, ctx.batched, ctx.cpg = params, batched, compute_points_grad
        return out

    @staticmethod
    def backward(ctx, grad):
        points, As = ctx.saved_tensors
        p = ctx.params
        mom, gp = R.backward(p.nc, points, ctx.batched, As, grad.contiguous(),
                             int(p.nstepsolver), False)
        Bt = _get_sparse_basis(p, As.device).t()
        dtheta = torch.sparse.mm(Bt, mom.reshape(mom.shape[0], -1).t()).t()
        gpts = gp if (ctx.cpg and ctx.batched) else (gp.sum(0) if ctx.cpg else None)
        return gpts, dtheta, None, None


REF_CASES = [((3, 3), False, 2, "border", 3, (40, 44), True, 0.7),
             ((4, 4), True, 1, "zeros", 1, (33, 31), False, 1.0),
             ((4, 4, 4), True, 2, "zeros", 1, (16, 14, 18), False, 1.0)]


@pytest.mark.parametrize("case", REF_CASES, ids=["2d-K2-border", "2d-K1-zeros", "3d-K2-zeros"])
def test_fused_warp_matches_the_reference_kernels(case):
    R.require()
    tess, zb, K, padding, C, size, shared, scale = case
    layer = CpabWarp(tess, zero_boundary=zb, padding_mode=padding)
    x, thetas = _inputs(layer, 2, C, size, K, 21, scale, shared)
    w = torch.randn(2, C, *size, device=DEV, generator=torch.Generator(DEV).manual_seed(9))
    out, gth, gx = _run(lambda a, t: layer(a, t), x, thetas, w)
    ref, rth, rx = _run(lambda a, t: composed(layer, a, t, _RefTransformer.apply), x, thetas, w)
    assert (out - ref).abs().max().item() <= OUT_ATOL
    for a, b in zip(gth, rth):
        assert rel_l2(a.cpu().numpy(), b.cpu().numpy()) < DTHETA_RTOL
    # The two integrations agree within 1e-5 per point, and a sampling weight
    # moves by (n - 1) times that, so the image gradient is compared relatively.
    assert rel_l2(gx.cpu().numpy(), rx.cpu().numpy()) < DTHETA_RTOL


ORACLE_CASES = [((3, 3), False, 2, "border", 2, (12, 14)),
                ((3, 2), False, 1, "reflection", 1, (9, 16)),
                ((2, 2, 2), False, 1, "zeros", 1, (6, 7, 5))]


@pytest.mark.parametrize("case", ORACLE_CASES, ids=["2d-K2-border", "2d-K1-refl", "3d-K1"])
def test_fused_warp_matches_the_oracle(case):
    tess, zb, K, padding, C, size = case
    layer = CpabWarp(tess, zero_boundary=zb, padding_mode=padding)
    x, thetas = _inputs(layer, 2, C, size, K, 31, 0.5)
    w = torch.randn(2, C, *size, device=DEV, generator=torch.Generator(DEV).manual_seed(2))
    out, gth, gx = _run(lambda a, t: layer(a, t), x, thetas, w)
    axes = [a.cpu().numpy() for a in pixel_axes(size, DEV)]
    basis = layer.cpab.params.basis
    o_out, final, stages = O.warp_forward(list(tess), basis, x.cpu().numpy(),
                                          [t.cpu().numpy() for t in thetas], axes, padding)
    o_gth, o_gx = O.warp_backward(list(tess), basis, x.cpu().numpy(), final, stages,
                                  w.cpu().numpy(), padding)
    np.testing.assert_allclose(out.cpu().numpy(), o_out, atol=OUT_ATOL, rtol=0)
    for a, b in zip(gth, o_gth):
        assert rel_l2(a.cpu().numpy(), b) < DTHETA_RTOL
    np.testing.assert_allclose(gx.cpu().numpy(), o_gx, atol=OUT_ATOL, rtol=0)


def test_warp_follows_the_reference_conventions():
    """theta as one [B, d] tensor, a list, or a [K, B, d] tensor; output in
    x's dtype; theta = 0 is the identity; 1D goes through the composition."""
    layer = CpabWarp((3, 3), zero_boundary=False)
    x = torch.rand(2, 3, 20, 24, device=DEV)
    zero = torch.zeros(2, layer.theta_dim, device=DEV)
    assert (layer(x, zero) - x).abs().max().item() <= 1e-5
    th = [0.4 * torch.randn(2, layer.theta_dim, device=DEV) for _ in range(2)]
    a = layer(x, th)
    assert torch.equal(a, layer(x, torch.stack(th)))
    assert layer(x.half(), th).dtype == torch.float16
    assert torch.equal(layer(x, th[0]), layer(x, [th[0]]))
    l1 = CpabWarp((6,), zero_boundary=False, padding_mode="border")
    x1 = torch.rand(3, 2, 50, device=DEV)
    t1 = [0.5 * torch.randn(3, l1.theta_dim, device=DEV) for _ in range(2)]
    assert torch.equal(l1(x1, t1), composed(l1, x1, t1))


def test_warp_errors():
    layer = CpabWarp((3, 3))
    x = torch.rand(2, 1, 8, 8, device=DEV)
    th = torch.zeros(2, layer.theta_dim, device=DEV)
    with pytest.raises(ValueError):
        warp(x, [th], layer.cpab.params, "nearest")
    with pytest.raises(ValueError):
        warp(x[:1].clone(), [th], layer.cpab.params)
    with pytest.raises(ValueError):
        warp(x, [th[:, :-1]], layer.cpab.params)
    with pytest.raises(ValueError):
        warp(x, [th.cpu()], layer.cpab.params)
    with pytest.raises(AssertionError):
        layer(torch.rand(2, 1, 8, device=DEV), th)


def test_warp_graph_replay_matches_eager():
    layer = CpabWarp((3, 3), zero_boundary=False, padding_mode="border")
    x, thetas = _inputs(layer, 4, 3, (40, 40), 2, 7, 0.6)
    ths = [t.clone().requires_grad_(True) for t in thetas]
    target = torch.rand_like(x)

    def step():
        for t in ths:
            t.grad = None
        loss = F.mse_loss(layer(x, ths), target)
        loss.backward()
        return loss

    eager = step().item()
    eager_g = [t.grad.clone() for t in ths]
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        step()
    torch.cuda.current_stream().wait_stream(s)
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        loss = step()
    g.replay()
    torch.cuda.synchronize()
    assert abs(loss.item() - eager) <= 1e-6 * max(1.0, abs(eager))
    for a, b in zip(ths, eager_g):
        assert rel_l2(a.grad.cpu().numpy(), b.cpu().numpy()) < 1e-5


def test_cpp_node_matches_python_node():
    """The C++ autograd node (_cpab_ext.warp) issues the Python node's C ABI
    calls: identical outputs, gradients equal up to the order of atomics."""
    from cpab import _ext
    if _ext.module() is None:
        pytest.skip("_cpab_ext.so is not built")
    layer = CpabWarp((3, 3), zero_boundary=False, padding_mode="reflection")
    x, thetas = _inputs(layer, 3, 2, (30, 26), 2, 4, 0.6)
    w = torch.randn(3, 2, 30, 26, device=DEV, generator=torch.Generator(DEV).manual_seed(8))
    out, gth, gx = _run(lambda a, t: layer(a, t), x, thetas, w)
    with _ext.python_path():
        ref, rth, rx = _run(lambda a, t: layer(a, t), x, thetas, w)
    assert torch.equal(out, ref)
    for a, b in zip(gth, rth):
        assert rel_l2(a.cpu().numpy(), b.cpu().numpy()) < 1e-5
    assert (gx - rx).abs().max().item() <= 1e-6


# one-pixel axes (grid_sample's size-1 rules: the pixel at 0.5, reflection's
# degenerate fold), a batch of one, every padding mode
EDGE = [((3, 3), size, pad) for size in [(1, 1), (1, 6), (5, 1)]
        for pad in ("zeros", "border", "reflection")] + \
       [((2, 2, 2), size, pad) for size in [(1, 1, 1), (3, 1, 4)]
        for pad in ("zeros", "border", "reflection")]


@pytest.mark.parametrize("case", EDGE, ids=["%s-%s-%s" % ("x".join(map(str, t)), "x".join(map(str, s)), p)
                                            for t, s, p in EDGE])
def test_degenerate_images_match_the_composition(case):
    tess, size, padding = case
    layer = CpabWarp(tess, zero_boundary=False, padding_mode=padding)
    x, thetas = _inputs(layer, 1, 2, size, 2, 17, 0.8)
    w = torch.randn(1, 2, *size, device=DEV, generator=torch.Generator(DEV).manual_seed(4))
    out, gth, gx = _run(lambda a, t: layer(a, t), x, thetas, w)
    ref, rth, rx = _run(lambda a, t: composed(layer, a, t), x, thetas, w)
    assert (out - ref).abs().max().item() <= OUT_ATOL
    for a, b in zip(gth, rth):
        na = float(b.norm())
        assert float((a - b).norm()) <= DTHETA_RTOL * max(na, 1e-6)
    assert (gx - rx).abs().max().item() <= OUT_ATOL
