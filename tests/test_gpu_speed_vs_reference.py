"""Speed of this implementation versus the reference's own CUDA kernels
(oracle/_ref, launched as the reference launches them) on the benchmark
workload: 2D Cpab([20,20]), batch 16, 125,000 points, nstepsolver 50.

Both sides get the same A (this library's A-build); the reference side
uses its expm, forward and backward kernels and torch.sparse.mm for the
projection, as its transformer.py does.  Times are CUDA-event medians.
Set CPAB_SPEED_REPORT=path to write the numbers as JSON.
"""
import json
import os

import numpy as np
import pytest
import torch

import refkernels as R
from cpab import _native
from cpab.pytorch.transformer import device_basis
from helpers import cpab

pytestmark = [pytest.mark.gpu,
              pytest.mark.skipif(not torch.cuda.is_available(), reason="needs a CUDA GPU")]


@pytest.fixture(autouse=True)
def _reference_kernels_built():
    R.require()


def _time(fn, reps=10):
    for _ in range(3):
        fn()
    torch.cuda.synchronize()
    ts = []
    for _ in range(reps):
        s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        s.record()
        fn()
        e.record()
        torch.cuda.synchronize()
        ts.append(s.elapsed_time(e))
    return float(np.median(ts))


def test_faster_than_reference_kernels():
    nc, B, nP, T = [20, 20], 16, 125000, 50
    C = cpab(tuple(nc))
    dev = torch.device("cuda")
    th = torch.randn(B, C.params.d, generator=torch.Generator().manual_seed(0)).to(dev)
    pts = torch.rand(2, nP, generator=torch.Generator().manual_seed(1)).to(dev)
    basis = device_basis(C.params, dev)
    As, trels = _native.build_A(2, C.params.nC, basis, th, 1.0 / T)
    g = torch.randn(B, 2, nP, device=dev)
    Bt = C._get_basis_sparse_gpu(device=dev).transpose(0, 1).coalesce()
    order = _native.order_points(nc, pts, False)

    ours = {
        "forward": _time(lambda: _native.forward(2, nc, pts, False, trels, As, T, 0, order)),
        "backward": _time(lambda: _native.backward(2, nc, pts, False, As, g, T, 0, False, order)),
        "order": _time(lambda: _native.order_points(nc, pts, False)),
    }
    ref = {
        "forward": _time(lambda: R.forward(nc, pts, False, trels, As, T, False)),
        "backward": _time(lambda: R.backward(nc, pts, False, As, g, T, False)),
    }
    mom = _native.backward(2, nc, pts, False, As, g, T, 0, False, order)[0]
    ours["project"] = _time(lambda: _native.project(basis, mom))
    ref["project"] = _time(lambda: torch.sparse.mm(Bt, mom.reshape(B, -1).t()).t().contiguous())
    ours["total"] = ours["forward"] + ours["backward"] + ours["order"] + ours["project"]
    ref["total"] = ref["forward"] + ref["backward"] + ref["project"]
    report = {"workload": "2D 20x20, batch 16, 125000 points, T=50", "unit": "ms",
              "ours": ours, "reference_kernels": ref,
              "speedup": {k: ref[k] / ours[k] for k in ("forward", "backward", "total")}}
    print(json.dumps(report))
    path = os.environ.get("CPAB_SPEED_REPORT")
    if path:
        with open(path, "w") as f:
            json.dump(report, f, indent=1)
    assert ours["total"] < ref["total"]


@pytest.mark.parametrize("case", ["stn2d", "stn3d"])
def test_warp_faster_than_reference_layer(case):
    """The fused spatial-transformer warp against the reference's CpabWarp
    composition (stn/stn.py:40-54,79-86: a CPAB_transformer call per
    transformation on the reference's kernels, then F.grid_sample), fwd+bwd
    of a weighted sum on the demo layers' shapes (stn/demos/demo_2d.py,
    demo_3d.py): 32 images, two composed transformations."""
    import test_gpu_warp as W
    from cpab.pytorch.warp import CpabWarp
    tess, pad, shape, scale = (((3, 3), "border", (3, 128, 128), 0.7) if case == "stn2d"
                               else ((4, 4, 4), "zeros", (1, 32, 32, 32), 1.0))
    layer = CpabWarp(tess, padding_mode=pad)
    g = torch.Generator("cuda").manual_seed(0)
    x = torch.rand(32, *shape, device="cuda", generator=g)
    ths = [(scale * torch.randn(32, layer.theta_dim, device="cuda", generator=g)).requires_grad_(True)
           for _ in range(2)]
    w = torch.randn(32, *shape, device="cuda", generator=g)

    def step(fn):
        def run():
            for t in ths:
                t.grad = None
            (fn() * w).sum().backward()
        return run

    ours = _time(step(lambda: layer(x, ths)))
    composed_ours = _time(step(lambda: W.composed(layer, x, ths)))
    ref = _time(step(lambda: W.composed(layer, x, ths, W._RefTransformer.apply)))
    print(json.dumps({"workload": case, "unit": "ms", "fused_warp": ours,
                      "composition_on_this_library": composed_ours,
                      "composition_on_reference_kernels": ref, "speedup_vs_reference": ref / ours}))
    assert ours < ref
