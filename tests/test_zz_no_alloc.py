"""The allocation-free ordering entry point, cpab_b200_order_points_static.

It exists for callers that cannot allocate device memory themselves -- a host
that only passes in the buffers it owns, code that must not call
cudaMalloc/cudaFree because they can synchronize the device, code under a
fixed memory budget -- and keeps its scratch counters in an array built into
the library instead of taking a scratch buffer.  Called here through the C ABI
and compared with cpab_b200_order_points (the entry point that takes caller
scratch) on two calls in a row with different inputs: the built-in array keeps
the previous call's counts, so the second call also checks that the entry
point clears what it uses.  This file is collected last on purpose."""
import ctypes

import numpy as np
import pytest
import torch

from cpab import _native
from oracle import oracle as O

pytestmark = [pytest.mark.gpu,
              pytest.mark.skipif(not torch.cuda.is_available(), reason="needs a CUDA GPU")]


def _static_order(nc, points, n_sets):
    nP = points.shape[-1]
    order = torch.empty((n_sets, nP), device=points.device, dtype=torch.int32)
    ncs = (ctypes.c_int32 * len(nc))(*nc)
    L = _native.lib()
    st = L.cpab_b200_order_points_static(len(nc), ncs, ctypes.c_void_p(points.data_ptr()), nP,
                                         n_sets, ctypes.c_void_p(order.data_ptr()),
                                         ctypes.c_void_p(torch.cuda.current_stream().cuda_stream))
    assert st == 0, L.cpab_b200_last_error().decode()
    return order


def _check_same_ordering(nc, points_2d, a, b):
    """a and b are permutations of the points that visit them in the same
    cell sequence (ties inside a cell may come in any order)."""
    nP = points_2d.shape[1]
    a, b = a.cpu().numpy(), b.cpu().numpy()
    assert np.array_equal(np.sort(a), np.arange(nP)) and np.array_equal(np.sort(b), np.arange(nP))
    cells = O.cells(nc, points_2d)
    np.testing.assert_array_equal(cells[a], cells[b])
    assert np.all(np.diff(cells[a]) >= 0)


@pytest.mark.parametrize("nc,batched", [([20, 20], False), ([4, 5, 3], True)])
def test_static_scratch_matches_caller_scratch_on_two_calls(nc, batched):
    torch.cuda.synchronize()
    nd = len(nc)
    g = torch.Generator().manual_seed(7)
    for call in range(2):  # second call: the built-in counters hold the first call's counts
        n_sets, nP = (3, 20000 + 77 * call) if batched else (1, 30000 + 1000 * call)
        pts = torch.rand((n_sets, nd, nP) if batched else (nd, nP), generator=g).cuda()
        got = _static_order(nc, pts, n_sets)
        ref = _native.order_points(nc, pts, batched)
        torch.cuda.synchronize()
        for s in range(n_sets):
            p2 = (pts[s] if batched else pts).cpu().numpy()
            _check_same_ordering(nc, p2, got[s], ref[s])


def test_static_scratch_rejects_sizes_beyond_its_limit():
    L = _native.lib()
    nc = (ctypes.c_int32 * 3)(128, 128, 128)           # 5 * 128^3 cells > 2^20 counters
    st = L.cpab_b200_order_points_static(3, nc, ctypes.c_void_p(16), 10, 1, ctypes.c_void_p(16),
                                         None)
    assert st == -4
    assert "exceeds the built-in scratch" in L.cpab_b200_last_error().decode()
