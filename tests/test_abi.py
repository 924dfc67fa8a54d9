"""The C ABI: the library loads, exports every entry point the header
declares, and rejects bad arguments on the host (no GPU needed)."""
import ctypes
import os
import re

import pytest

from cpab import _native

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
HEADER = os.path.join(ROOT, "include", "cpab_b200.h")


def declared():
    with open(HEADER) as f:
        text = f.read()
    return sorted(set(re.findall(r"^\s*(?:const\s+)?\w+\s*\*?\s*(cpab_b200_\w+)\s*\(", text, re.M)))


def test_header_declares_entry_points():
    names = declared()
    assert "cpab_b200_forward" in names and "cpab_b200_backward" in names
    assert len(names) >= 12


def test_library_exports_every_declared_symbol():
    L = _native.lib()
    for name in declared():
        assert hasattr(L, name), name
    assert set(declared()) == set(_native.EXPORTS)


def test_version_and_limits():
    L = _native.lib()
    assert L.cpab_b200_version() >= 10000
    assert L.cpab_b200_max_steps() == 256


NC2 = (ctypes.c_int32 * 2)(4, 4)
P = ctypes.c_void_p(16)  # never dereferenced: validation fails first


@pytest.mark.parametrize("args,code,msg", [
    ((4, NC2, P, 10, 0, None, P, P, 1, 50, 0, P, None), -1, "ndim"),
    ((2, NC2, P, 10, 0, None, P, P, 1, 0, 0, P, None), -2, "nstepsolver"),
    ((2, NC2, P, 10, 0, None, P, P, 1, 257, 0, P, None), -2, "nstepsolver"),
    ((2, NC2, P, 10, 0, None, P, P, 1, 50, 2, P, None), -1, "adaptive"),
    ((2, NC2, P, 10, 2, None, P, P, 1, 50, 0, P, None), -1, "points_batched"),
    ((2, NC2, P, 10, 0, None, P, P, 70000, 50, 0, P, None), -4, "n_theta"),
    ((2, NC2, P, -1, 0, None, P, P, 1, 50, 0, P, None), -1, "negative"),
    ((2, NC2, None, 10, 0, None, P, P, 1, 50, 0, P, None), -1, "null"),
    ((2, NC2, P, 10, 0, None, None, P, 1, 50, 0, P, None), -1, "trels"),
])
def test_forward_argument_errors(args, code, msg):
    L = _native.lib()
    assert L.cpab_b200_forward(*args) == code
    assert msg in L.cpab_b200_last_error().decode()


def test_zero_sized_calls_succeed_without_work():
    L = _native.lib()
    assert L.cpab_b200_forward(2, NC2, P, 0, 0, None, P, P, 3, 50, 0, P, None) == 0
    assert L.cpab_b200_forward(2, NC2, P, 10, 0, None, P, P, 0, 50, 0, P, None) == 0
    assert L.cpab_b200_last_error().decode() == ""


def test_other_entry_points_validate():
    L = _native.lib()
    bad = (ctypes.c_int32 * 2)(0, 4)
    assert L.cpab_b200_backward(2, bad, P, 10, 0, None, P, 1, P, 50, 0, P, None, None) == -1
    assert L.cpab_b200_backward(2, NC2, P, 10, 0, None, P, 1, P, 50, 0, None, None, None) == -1
    assert L.cpab_b200_order_points(2, bad, P, 10, 1, P, P, None) == -1
    assert L.cpab_b200_order_points(2, NC2, P, 10, 1, None, P, None) == -1
    assert L.cpab_b200_expm(5, P, 3, 0.1, P, None) == -1
    assert L.cpab_b200_project(-1, 4, 1, P, P, P, P, P, None) == -1
    assert L.cpab_b200_build_A(0, 4, 4, 1, P, P, P, P, 0.1, P, P, None) == -1
    assert L.cpab_b200_cell_index(2, bad, P, 5, P, None) == -1
    sz = (ctypes.c_int64 * 2)(8, 8)
    assert L.cpab_b200_interpolate(4, P, 1, 1, sz, P, sz, P, None) == -1
    zero = (ctypes.c_int64 * 2)(0, 8)
    assert L.cpab_b200_interpolate(2, P, 1, 1, zero, P, sz, P, None) == -1
    assert L.cpab_b200_interpolate_backward(2, P, 1, 1, sz, P, sz, None, P, None, None) == -1
    assert L.cpab_b200_forward_1d_closed_form(P, 10, 0, None, P, 1, 0, P, None) == -1


def test_order_points_rejects_huge_tessellations_before_any_gpu_work():
    """Axes within the per-axis limit can still multiply to more cells than
    the sort indexes (int) or than the built-in scratch holds; both entry
    points must refuse on the host (no CUDA call: these run without a GPU)."""
    L = _native.lib()
    err = lambda: L.cpab_b200_last_error().decode()  # noqa: E731
    nc2 = (ctypes.c_int32 * 2)(1 << 20, 1 << 20)        # 4 * 2^40 cells
    assert L.cpab_b200_order_points(2, nc2, P, 10, 1, P, P, None) == -4
    assert "too many cells" in err()
    nc3 = (ctypes.c_int32 * 3)(1 << 20, 1 << 20, 1 << 20)  # 5 * 2^60 cells
    assert L.cpab_b200_order_points(3, nc3, P, 10, 1, P, P, None) == -4
    # n_sets * nC would overflow int64 if formed; the static variant must
    # still report its scratch limit, not reach the GPU.
    assert L.cpab_b200_order_points_static(3, nc3, P, 10, 2, P, None) == -4
    assert "exceeds the built-in scratch" in err()
    assert L.cpab_b200_order_points_static(3, nc3, P, 10, 65535, P, None) == -4
    over = (ctypes.c_int32 * 2)((1 << 20) + 1, 4)       # one axis beyond 2^20
    assert L.cpab_b200_order_points_static(2, over, P, 10, 1, P, None) == -1
    assert "[1, 2^20]" in err()
    nc = (ctypes.c_int32 * 2)(512, 512)                 # 2^20 cells: fits once, not twice
    assert L.cpab_b200_order_points_static(2, nc, P, 10, 2, P, None) == -4


def test_transform_data_entry_points_validate():
    L = _native.lib()
    sz = (ctypes.c_int64 * 2)(8, 8)
    zero = (ctypes.c_int64 * 2)(0, 8)
    neg = (ctypes.c_int64 * 2)(-1, 8)
    huge = (ctypes.c_int64 * 2)(1 << 16, 1 << 15)
    fwd = L.cpab_b200_transform_data
    bwd = L.cpab_b200_transform_data_backward
    err = lambda: L.cpab_b200_last_error().decode()  # noqa: E731
    assert fwd(1, NC2, sz, P, None, P, P, 1, 50, 0, P, 1, sz, P, P, None) == -1 and "ndim" in err()
    assert fwd(2, NC2, neg, P, None, P, P, 1, 50, 0, P, 1, sz, P, P, None) == -1
    assert fwd(2, NC2, sz, P, None, P, P, 1, 50, 0, P, 1, zero, P, P, None) == -1
    assert fwd(2, NC2, huge, P, None, P, P, 1, 50, 0, P, 1, sz, P, P, None) == -4
    assert fwd(2, NC2, sz, P, None, P, P, 1, 0, 0, P, 1, sz, P, P, None) == -2
    assert fwd(2, NC2, sz, P, None, P, P, 70000, 50, 0, P, 1, sz, P, P, None) == -4
    assert fwd(2, NC2, sz, P, None, None, P, 1, 50, 0, P, 1, sz, P, P, None) == -1 and "trels" in err()
    assert fwd(2, NC2, sz, P, None, P, P, 1, 50, 0, P, 1, sz, None, P, None) == -1
    assert fwd(2, NC2, sz, P, None, P, P, 1, 50, 0, None, 1, sz, P, P, None) == -1
    assert bwd(2, NC2, sz, P, None, P, 1, 50, 0, P, 1, sz, P, P, None, None, None) == -1
    assert "moments" in err()
    nc3 = (ctypes.c_int32 * 3)(2, 2, 2)
    sz3, bad3 = (ctypes.c_int64 * 3)(4, 4, 4), (ctypes.c_int64 * 3)(4, 0, 4)
    assert bwd(3, nc3, sz3, P, None, P, 1, 50, 0, P, 1, bad3, P, P, P, None, None) == -1
    # nothing to do: no transformations
    assert fwd(2, NC2, sz, P, None, P, P, 0, 50, 0, P, 1, sz, P, P, None) == 0


def test_chain_entry_points_validate():
    L = _native.lib()
    f, g = L.cpab_b200_forward_chain, L.cpab_b200_backward_chain
    err = lambda: L.cpab_b200_last_error().decode()  # noqa: E731
    nc1 = (ctypes.c_int32 * 1)(4)
    assert f(1, nc1, P, 10, 0, None, P, P, 2, 1, 50, 0, P, P, None) == -1 and "ndim" in err()
    assert f(2, NC2, P, 10, 0, None, P, P, 0, 1, 50, 0, P, P, None) == -1 and "n_stages" in err()
    assert f(2, NC2, P, 10, 0, None, P, P, 3, 1, 50, 0, None, P, None) == -1
    assert f(2, NC2, P, 10, 0, None, None, P, 3, 1, 50, 0, P, P, None) == -1 and "trels" in err()
    assert f(2, NC2, P, 10, 0, None, P, P, 3, 1, 0, 0, P, P, None) == -2
    assert g(2, NC2, P, 10, 0, None, P, 3, 1, P, P, 50, 0, None, None, None) == -1
    assert "moments" in err()
    assert g(2, NC2, P, 10, 0, None, P, 3, 1, P, None, 50, 0, P, None, None) == -1
    assert f(2, NC2, P, 0, 0, None, P, P, 3, 1, 50, 0, P, P, None) == 0  # no points


def test_warp_entry_points_validate():
    L = _native.lib()
    f, g = L.cpab_b200_warp, L.cpab_b200_warp_backward
    err = lambda: L.cpab_b200_last_error().decode()  # noqa: E731
    sz = (ctypes.c_int64 * 2)(8, 8)
    # ndim, nc, out_size, axes, order, trels, As, n_stages, n_theta, T, adaptive, data,
    # data_batched, C, in_size, padding, stage_points, grid_t, out, stream
    ok = [2, NC2, sz, P, None, P, P, 1, 1, 50, 0, P, 1, 1, sz, 0, None, P, P, None]

    def call(fn, base, **kw):
        a = list(base)
        for i, v in kw.items():
            a[int(i[1:])] = v
        return fn(*a)

    assert call(f, ok, a0=1) == -1 and "ndim" in err()
    assert call(f, ok, a15=3) == -1 and "padding_mode" in err()
    assert call(f, ok, a15=-1) == -1
    assert call(f, ok, a12=2) == -1 and "data_batched" in err()
    assert call(f, ok, a7=0) == -1 and "n_stages" in err()
    assert call(f, ok, a7=5000) == -1
    assert call(f, ok, a7=2) == -1 and "stage_points" in err()
    assert call(f, ok, a5=None) == -1 and "trels" in err()
    assert call(f, ok, a9=0) == -2
    assert call(f, ok, a8=70000) == -4
    assert call(f, ok, a18=None) == -1 and "output" in err()
    assert call(f, ok, a8=0) == 0                        # no transformations: nothing to do
    # backward: ..., padding, stage_points, grid_t, grad_out, moments, grad_data, stream
    okb = [2, NC2, sz, P, None, P, 1, 1, 50, 0, P, 1, 1, sz, 0, None, P, P, P, None, None]
    assert call(g, okb, a18=None) == -1 and "moments" in err()
    assert call(g, okb, a14=7) == -1 and "padding_mode" in err()
    assert call(g, okb, a6=2) == -1 and "stage_points" in err()
    assert call(g, okb, a17=None) == -1 and "grad_out" in err()


def test_errors_are_per_thread():
    import threading
    L = _native.lib()
    L.cpab_b200_expm(5, P, 3, 0.1, P, None)
    seen = []
    t = threading.Thread(target=lambda: seen.append(L.cpab_b200_last_error().decode()))
    t.start()
    t.join()
    assert seen == [""] and "ndim" in L.cpab_b200_last_error().decode()


def test_misaligned_tables_rejected():
    L = _native.lib()
    odd = ctypes.c_void_p(16 + 4)
    assert L.cpab_b200_forward(2, NC2, P, 10, 0, None, P, odd, 1, 50, 0, P, None) == -1
    assert "aligned" in L.cpab_b200_last_error().decode()
    assert L.cpab_b200_forward(2, NC2, P, 10, 0, None, odd, P, 1, 50, 0, P, None) == -1
    big = (ctypes.c_int32 * 2)((1 << 20) + 1, 2)
    assert L.cpab_b200_forward(2, big, P, 10, 0, None, P, P, 1, 50, 0, P, None) == -1


def test_cpp_extension_loads_next_to_the_library():
    """The C++ autograd node is built beside libcpab_b200.so and imports
    without a GPU (it only links the library; no CUDA call at import)."""
    from cpab import _ext
    m = _ext.module()
    assert m is not None and hasattr(m, "transform")
    with _ext.python_path():
        assert _ext.module() is None
    assert _ext.module() is m
