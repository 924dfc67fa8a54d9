"""The C++ transform_grid node (cpab/_cpab_ext.so, csrc/torch_ext.cpp) against
the Python one (_CPABFunction): both issue the same C ABI calls, so outputs
are identical and gradients agree up to the order of the moments' fp32
reductions in L2."""
import numpy as np
import pytest
import torch

from cpab import _ext
from cpab.pytorch.transformer import transform
from helpers import DTHETA_RTOL, cpab, rand_points, rand_theta, rel_l2

pytestmark = [pytest.mark.gpu,
              pytest.mark.skipif(not torch.cuda.is_available(), reason="needs a CUDA GPU")]

# (nc, zero_boundary, n_theta, nP, batched, adaptive)
CASES = [((50,), True, 4, 5000, False, False), ((20, 20), True, 3, 20000, False, False),
         ((30, 30), False, 2, 6000, False, False), ((6, 6), True, 2, 5000, True, True),
         ((10, 10, 10), True, 2, 8000, False, False), ((4, 3, 2), False, 3, 3000, True, False)]


def run(case, python_path):
    nc, zb, n, nP, batched, adaptive = case
    C = cpab(nc, zb)
    C.params.adaptive_substeps = adaptive
    try:
        th = torch.from_numpy(rand_theta(n, C.params.d, 5, 0.7)).cuda().requires_grad_(True)
        pts = rand_points(len(nc), nP, 6)
        if batched:
            pts = np.stack([rand_points(len(nc), nP, 7 + b) for b in range(n)])
        p = torch.from_numpy(pts).cuda().requires_grad_(True)
        g = torch.randn(n, len(nc), nP, generator=torch.Generator().manual_seed(8)).cuda()
        if python_path:
            with _ext.python_path():
                out = transform(p, th, C.params, True)
                (out * g).sum().backward()
        else:
            out = transform(p, th, C.params, True)
            (out * g).sum().backward()
        torch.cuda.synchronize()
        return out.detach().cpu().numpy(), th.grad.cpu().numpy(), p.grad.cpu().numpy()
    finally:
        C.params.adaptive_substeps = False


@pytest.mark.parametrize("case", CASES, ids=[str(c[0]) + ("-bat" if c[4] else "") +
                                              ("-ad" if c[5] else "") for c in CASES])
def test_cpp_node_matches_python_node(case):
    assert _ext.module() is not None, "the C++ extension is not built"
    o1, t1, p1 = run(case, False)
    o2, t2, p2 = run(case, True)
    np.testing.assert_array_equal(o1, o2)
    assert rel_l2(t1, t2) < DTHETA_RTOL
    np.testing.assert_allclose(p1, p2, rtol=1e-5, atol=1e-6)


def test_cpp_node_rejects_cpu_tensors_and_bad_shapes():
    C = cpab((4, 4), True)
    th = torch.zeros(2, C.params.d, device="cuda")
    with pytest.raises(AssertionError):
        from cpab.pytorch.transformer import CPAB_transformer
        CPAB_transformer(torch.rand(2, 100), th, C.params)
    with pytest.raises(ValueError):
        transform(torch.rand(3, 100, device="cuda"), th, C.params)

