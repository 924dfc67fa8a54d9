"""ctypes binding of libcpab_b200.so (the C ABI in include/cpab_b200.h).

Tensors cross the boundary as raw device pointers plus sizes; every call is
enqueued on torch's current stream of the tensors' device.  There is no CPU
fallback: if the library is missing or the tensors are not CUDA tensors the
call raises.
"""
import contextlib
import ctypes
import functools
import os

import torch

# The library built next to this file; CPAB_B200_LIB names another build of
# the same ABI (e.g. one with other compile-time kernel choices).
LIB_PATH = os.environ.get("CPAB_B200_LIB") or os.path.join(
    os.path.dirname(os.path.abspath(__file__)), "libcpab_b200.so")

_c_int, _c_i64, _c_float, _p = ctypes.c_int, ctypes.c_int64, ctypes.c_float, ctypes.c_void_p

# name -> argtypes (all return int status)
_SIGNATURES = {
    "cpab_b200_expm": [_c_int, _p, _c_i64, _c_float, _p, _p],
    "cpab_b200_build_A": [_c_int, _c_i64, _c_i64, _c_int, _p, _p, _p, _p, _c_float, _p, _p, _p],
    "cpab_b200_forward": [_c_int, _p, _p, _c_i64, _c_int, _p, _p, _p, _c_int, _c_int, _c_int, _p,
                          _p],
    "cpab_b200_forward_1d_closed_form": [_p, _c_i64, _c_int, _p, _p, _c_int, _c_int, _p, _p],
    "cpab_b200_backward": [_c_int, _p, _p, _c_i64, _c_int, _p, _p, _c_int, _p, _c_int, _c_int,
                           _p, _p, _p],
    "cpab_b200_order_points": [_c_int, _p, _p, _c_i64, _c_int, _p, _p, _p],
    "cpab_b200_order_points_static": [_c_int, _p, _p, _c_i64, _c_int, _p, _p],
    "cpab_b200_cell_index": [_c_int, _p, _p, _c_i64, _p, _p],
    "cpab_b200_project": [_c_i64, _c_i64, _c_int, _p, _p, _p, _p, _p, _p],
    "cpab_b200_build_A_tt": [_c_int, _c_i64, _c_i64, _c_int, _p, _p, _p, _p, _c_float, _p, _p, _p],
    "cpab_b200_project_tt": [_c_i64, _c_i64, _c_int, _p, _p, _p, _p, _p, _p],
    "cpab_b200_interpolate": [_c_int, _p, _c_int, _c_int, _p, _p, _p, _p, _p],
    "cpab_b200_interpolate_backward": [_c_int, _p, _c_int, _c_int, _p, _p, _p, _p, _p, _p, _p],
    "cpab_b200_forward_chain": [_c_int, _p, _p, _c_i64, _c_int, _p, _p, _p, _c_int, _c_int,
                                _c_int, _c_int, _p, _p, _p],
    "cpab_b200_backward_chain": [_c_int, _p, _p, _c_i64, _c_int, _p, _p, _c_int, _c_int, _p, _p,
                                 _c_int, _c_int, _p, _p, _p],
    "cpab_b200_transform_data": [_c_int, _p, _p, _p, _p, _p, _p, _c_int, _c_int, _c_int, _p,
                                 _c_int, _p, _p, _p, _p],
    "cpab_b200_transform_data_backward": [_c_int, _p, _p, _p, _p, _p, _c_int, _c_int, _c_int,
                                          _p, _c_int, _p, _p, _p, _p, _p, _p],
    "cpab_b200_warp": [_c_int, _p, _p, _p, _p, _p, _p, _c_int, _c_int, _c_int, _c_int, _p,
                       _c_int, _c_int, _p, _c_int, _p, _p, _p, _p],
    "cpab_b200_warp_backward": [_c_int, _p, _p, _p, _p, _p, _c_int, _c_int, _c_int, _c_int, _p,
                                _c_int, _c_int, _p, _c_int, _p, _p, _p, _p, _p, _p],
}

EXPORTS = tuple(_SIGNATURES) + ("cpab_b200_version", "cpab_b200_max_steps",
                                "cpab_b200_last_error")

_lib = None


class CpabNativeError(RuntimeError):
    """A libcpab_b200 call returned a non-zero status."""


def lib():
    """Load (once) and return the native library."""
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            raise RuntimeError(
                "libcpab_b200.so is not built (expected at %s); run "
                "`python fg-cpab_b200/build.py` first" % LIB_PATH)
        L = ctypes.CDLL(LIB_PATH)
        for name, args in _SIGNATURES.items():
            fn = getattr(L, name)
            fn.argtypes = args
            fn.restype = ctypes.c_int
        L.cpab_b200_version.restype = ctypes.c_int
        L.cpab_b200_max_steps.restype = ctypes.c_int
        L.cpab_b200_last_error.restype = ctypes.c_char_p
        _lib = L
    return _lib


def max_steps():
    return lib().cpab_b200_max_steps()


def _check(status):
    if status != 0:
        msg = lib().cpab_b200_last_error().decode(errors="replace")
        raise CpabNativeError(msg or "libcpab_b200 error %d" % status)


def _ptr(t):
    """Device pointer of t (None = NULL); ctypes converts it for the void* arguments."""
    return t.data_ptr() if t is not None else None


# The raw cudaStream_t of the current stream in one call (torch's own query for
# generated kernels); current_stream() builds a Stream object per call, which
# is a sizeable share of a call's host time.
_raw_stream = getattr(torch._C, "_cuda_getCurrentRawStream", None)


def _stream(device):
    index = device.index if device.index is not None else torch.cuda.current_device()
    if _raw_stream is not None:
        return _raw_stream(index)
    return torch.cuda.current_stream(device).cuda_stream


def _require(t, name, dtype=torch.float32):
    if not t.is_cuda:
        raise RuntimeError("%s must be a CUDA tensor (no CPU path)" % name)
    if t.dtype != dtype:
        raise TypeError("%s must be %s, got %s" % (name, dtype, t.dtype))
    if not t.is_contiguous():
        raise RuntimeError("%s must be contiguous" % name)


@functools.lru_cache(maxsize=256)
def _i32_cached(values):
    return (ctypes.c_int32 * len(values))(*values)


@functools.lru_cache(maxsize=256)
def _i64_cached(values):
    return (ctypes.c_int64 * len(values))(*values)


def _i32_array(values):
    """Read-only int32 array for a call (tessellation sizes): cached per value."""
    return _i32_cached(tuple(int(v) for v in values))


def _i64_array(values):
    """Read-only int64 array for a call (tensor sizes): cached per value."""
    return _i64_cached(tuple(int(v) for v in values))


def _on(device):
    """Context making `device` current; nothing to do when it already is."""
    if device.index is None or device.index == torch.cuda.current_device():
        return contextlib.nullcontext()
    return torch.cuda.device(device)


# ---------------------------------------------------------------------------
# Thin wrappers: shapes in, tensors out (allocated with torch on the device).
# ---------------------------------------------------------------------------

def expm(As, dT):
    """Trels = expm(dT * A) for As [n, ndim, ndim+1]."""
    _require(As, "As")
    n, nd = As.shape[0], As.shape[1]
    out = torch.empty_like(As)
    with _on(As.device):
        _check(lib().cpab_b200_expm(nd, _ptr(As), n, float(dT), _ptr(out), _stream(As.device)))
    return out


def build_A(ndim, nC, basis, theta, dT=None):
    """As = reshape(B theta^T) [n_theta, nC, ndim, ndim+1] and, when dT is given,
    Trels = expm(dT * As).  ``basis`` is a DeviceBasis."""
    _require(theta, "theta")
    n_theta = theta.shape[0]
    As = torch.empty((n_theta, nC, ndim, ndim + 1), device=theta.device, dtype=torch.float32)
    trels = torch.empty_like(As) if dT is not None else None
    with _on(theta.device):
        _check(lib().cpab_b200_build_A(
            ndim, nC, basis.d, n_theta, _ptr(basis.rowptr), _ptr(basis.colidx), _ptr(basis.vals),
            _ptr(theta), float(dT) if dT is not None else 0.0, _ptr(As), _ptr(trels),
            _stream(theta.device)))
    return As, trels


def build_A_tt(ndim, nC, basis, theta_t, n_theta, dT=None):
    """build_A with theta given transposed, theta_t [d, n_theta]."""
    _require(theta_t, "theta_t")
    As = torch.empty((n_theta, nC, ndim, ndim + 1), device=theta_t.device, dtype=torch.float32)
    trels = torch.empty_like(As) if dT is not None else None
    with _on(theta_t.device):
        _check(lib().cpab_b200_build_A_tt(
            ndim, nC, basis.d, n_theta, _ptr(basis.rowptr), _ptr(basis.colidx), _ptr(basis.vals),
            _ptr(theta_t), float(dT) if dT is not None else 0.0, _ptr(As), _ptr(trels),
            _stream(theta_t.device)))
    return As, trels


def order_points(nc, points, batched):
    """Processing order of the points sorted by initial cell: int32
    [n_sets, nP] (n_sets = batch when batched, else 1)."""
    _require(points, "points")
    nd, nP = points.shape[-2], points.shape[-1]
    n_sets = points.shape[0] if batched else 1
    nC = int(np_prod(nc)) * {1: 1, 2: 4, 3: 5}[nd]
    counts = torch.empty((n_sets, nC), device=points.device, dtype=torch.int32)
    order = torch.empty((n_sets, nP), device=points.device, dtype=torch.int32)
    with _on(points.device):
        _check(lib().cpab_b200_order_points(nd, _i32_array(nc), _ptr(points), nP, n_sets,
                                            _ptr(counts), _ptr(order), _stream(points.device)))
    return order


def np_prod(xs):
    r = 1
    for x in xs:
        r *= int(x)
    return r


def forward(ndim, nc, points, batched, trels, As, nstepsolver, adaptive, order=None):
    _require(points, "points")
    _require(As, "As")
    n_theta = As.shape[0]
    nP = points.shape[-1]
    out = torch.empty((n_theta, ndim, nP), device=As.device, dtype=torch.float32)
    with _on(As.device):
        if ndim == 1:
            _check(lib().cpab_b200_forward_1d_closed_form(
                _ptr(points), nP, int(batched), _ptr(order), _ptr(As), n_theta, int(nc[0]),
                _ptr(out), _stream(As.device)))
        else:
            _require(trels, "Trels")
            _check(lib().cpab_b200_forward(
                ndim, _i32_array(nc), _ptr(points), nP, int(batched), _ptr(order), _ptr(trels),
                _ptr(As), n_theta, int(nstepsolver), int(adaptive), _ptr(out),
                _stream(As.device)))
    return out


def backward(ndim, nc, points, batched, As, grad_out, nstepsolver, adaptive, want_points,
             order=None):
    """Returns (moments [n_theta, nC, ppc], grad_points [n_theta, ndim, nP] or None)."""
    _require(points, "points")
    _require(As, "As")
    _require(grad_out, "grad")
    n_theta, nC = As.shape[0], As.shape[1]
    nP = points.shape[-1]
    ppc = ndim * (ndim + 1)
    moments = torch.empty((n_theta, nC, ppc), device=As.device, dtype=torch.float32)
    gp = (torch.empty((n_theta, ndim, nP), device=As.device, dtype=torch.float32)
          if want_points else None)
    with _on(As.device):
        _check(lib().cpab_b200_backward(
            ndim, _i32_array(nc), _ptr(points), nP, int(batched), _ptr(order), _ptr(As), n_theta,
            _ptr(grad_out), int(nstepsolver), int(adaptive), _ptr(moments), _ptr(gp),
            _stream(As.device)))
    return moments, gp


def cell_index(nc, points):
    """Cell of every point, points [ndim, n] -> int32 [n]."""
    _require(points, "points")
    nd, n = points.shape
    out = torch.empty(n, device=points.device, dtype=torch.int32)
    with _on(points.device):
        _check(lib().cpab_b200_cell_index(nd, _i32_array(nc), _ptr(points), n, _ptr(out),
                                          _stream(points.device)))
    return out


def project(basis, moments):
    """dtheta [n_theta, d] = B^T vec(moments)."""
    _require(moments, "moments")
    n_theta = moments.shape[0]
    D = moments[0].numel()
    out = torch.empty((n_theta, basis.d), device=moments.device, dtype=torch.float32)
    with _on(moments.device):
        _check(lib().cpab_b200_project(
            basis.d, D, n_theta, _ptr(basis.t_rowptr), _ptr(basis.t_colidx), _ptr(basis.t_vals),
            _ptr(moments), _ptr(out), _stream(moments.device)))
    return out


def project_tt(basis, moments_t, n_theta):
    """project with the moments given transposed, moments_t [D, n_theta]."""
    _require(moments_t, "moments_t")
    out = torch.empty((n_theta, basis.d), device=moments_t.device, dtype=torch.float32)
    with _on(moments_t.device):
        _check(lib().cpab_b200_project_tt(
            basis.d, moments_t.shape[0], n_theta, _ptr(basis.t_rowptr), _ptr(basis.t_colidx),
            _ptr(basis.t_vals), _ptr(moments_t), _ptr(out), _stream(moments_t.device)))
    return out


def interpolate(ndim, data, grid, outsize):
    _require(data, "data")
    _require(grid, "grid")
    B, C = data.shape[0], data.shape[1]
    out = torch.empty((B, C, *outsize), device=data.device, dtype=torch.float32)
    with _on(data.device):
        _check(lib().cpab_b200_interpolate(
            ndim, _ptr(data), B, C, _i64_array(data.shape[2:]), _ptr(grid), _i64_array(outsize),
            _ptr(out), _stream(data.device)))
    return out


def interpolate_backward(ndim, data, grid, outsize, grad_out, want_grid, want_data):
    _require(data, "data")
    _require(grid, "grid")
    _require(grad_out, "grad")
    B, C = data.shape[0], data.shape[1]
    gg = torch.empty_like(grid) if want_grid else None
    gd = torch.empty_like(data) if want_data else None
    with _on(data.device):
        _check(lib().cpab_b200_interpolate_backward(
            ndim, _ptr(data), B, C, _i64_array(data.shape[2:]), _ptr(grid), _i64_array(outsize),
            _ptr(grad_out), _ptr(gg), _ptr(gd), _stream(data.device)))
    return gg, gd


def transform_data(ndim, nc, outsize, axes, trels, As, nstepsolver, adaptive, data, order=None):
    """Fused transform_data: returns (out [n_theta, C, *outsize], grid_t
    [n_theta, ndim, prod(outsize)] in processing order)."""
    _require(data, "data")
    _require(As, "As")
    _require(trels, "Trels")
    _require(axes, "mesh axes")
    n_theta, C = As.shape[0], data.shape[1]
    P = int(np_prod(outsize))
    out = torch.empty((n_theta, C, *outsize), device=As.device, dtype=torch.float32)
    grid_t = torch.empty((n_theta, ndim, P), device=As.device, dtype=torch.float32)
    with _on(As.device):
        _check(lib().cpab_b200_transform_data(
            ndim, _i32_array(nc), _i64_array(outsize), _ptr(axes), _ptr(order), _ptr(trels),
            _ptr(As), n_theta,
            int(nstepsolver), int(adaptive), _ptr(data), C, _i64_array(data.shape[2:]),
            _ptr(grid_t), _ptr(out), _stream(As.device)))
    return out, grid_t


def transform_data_backward(ndim, nc, outsize, axes, As, nstepsolver, adaptive, data, grid_t,
                            grad_out, want_data, order=None):
    """Returns (moments [n_theta, nC, ppc], grad_data or None)."""
    _require(data, "data")
    _require(As, "As")
    _require(grid_t, "grid_t")
    _require(grad_out, "grad")
    n_theta, nC, C = As.shape[0], As.shape[1], data.shape[1]
    moments = torch.empty((n_theta, nC, ndim * (ndim + 1)), device=As.device, dtype=torch.float32)
    gd = torch.empty_like(data) if want_data else None
    with _on(As.device):
        _check(lib().cpab_b200_transform_data_backward(
            ndim, _i32_array(nc), _i64_array(outsize), _ptr(axes), _ptr(order), _ptr(As), n_theta,
            int(nstepsolver), int(adaptive), _ptr(data), C, _i64_array(data.shape[2:]),
            _ptr(grid_t), _ptr(grad_out), _ptr(moments), _ptr(gd), _stream(As.device)))
    return moments, gd


def _data_batched(data, n_theta):
    """1 when data holds one image per transformation, 0 for one shared image."""
    if data.shape[0] not in (1, n_theta):
        raise ValueError("data must hold 1 or n_theta = %d images, got %d" % (n_theta, data.shape[0]))
    return int(data.shape[0] == n_theta)


def warp(ndim, nc, outsize, axes, trels, As, n_stages, nstepsolver, adaptive, data, padding,
         order=None):
    """Fused spatial-transformer warp of n_theta = As.shape[0] / n_stages
    transformations; data is [n_theta, C, *in_size] or [1, C, *in_size]
    (shared).  Returns (out [n_theta, C, *outsize], grid_t [n_theta, ndim, P],
    stage_points [n_stages-1, n_theta, ndim, P] or None)."""
    _require(data, "data")
    _require(As, "As")
    _require(trels, "Trels")
    _require(axes, "mesh axes")
    n_theta, C = As.shape[0] // n_stages, data.shape[1]
    P = int(np_prod(outsize))
    out = torch.empty((n_theta, C, *outsize), device=As.device, dtype=torch.float32)
    grid_t = torch.empty((n_theta, ndim, P), device=As.device, dtype=torch.float32)
    sp = (torch.empty((n_stages - 1, n_theta, ndim, P), device=As.device, dtype=torch.float32)
          if n_stages > 1 else None)
    batched = _data_batched(data, n_theta)
    with _on(As.device):
        _check(lib().cpab_b200_warp(
            ndim, _i32_array(nc), _i64_array(outsize), _ptr(axes), _ptr(order), _ptr(trels),
            _ptr(As), n_stages, n_theta, int(nstepsolver), int(adaptive), _ptr(data), batched, C,
            _i64_array(data.shape[2:]), int(padding), _ptr(sp), _ptr(grid_t), _ptr(out),
            _stream(As.device)))
    return out, grid_t, sp


def warp_backward(ndim, nc, outsize, axes, As, n_stages, nstepsolver, adaptive, data, padding,
                  stage_points, grid_t, grad_out, want_data, order=None):
    """Returns (moments [n_stages * n_theta, nC, ppc], grad_data shaped like
    data, or None)."""
    _require(data, "data")
    _require(As, "As")
    _require(grid_t, "grid_t")
    _require(grad_out, "grad")
    n_theta, nC, C = As.shape[0] // n_stages, As.shape[1], data.shape[1]
    moments = torch.empty((n_stages * n_theta, nC, ndim * (ndim + 1)), device=As.device,
                          dtype=torch.float32)
    gd = torch.empty_like(data) if want_data else None
    batched = _data_batched(data, n_theta)
    with _on(As.device):
        _check(lib().cpab_b200_warp_backward(
            ndim, _i32_array(nc), _i64_array(outsize), _ptr(axes), _ptr(order), _ptr(As),
            n_stages, n_theta, int(nstepsolver), int(adaptive), _ptr(data), batched, C,
            _i64_array(data.shape[2:]), int(padding), _ptr(stage_points), _ptr(grid_t),
            _ptr(grad_out), _ptr(moments), _ptr(gd), _stream(As.device)))
    return moments, gd


def forward_chain(ndim, nc, points, batched, trels, As, n_stages, nstepsolver, adaptive,
                  order=None):
    """Fused chain; trels/As [n_stages * n_theta, nC, ...] stage-major.  Returns
    (out [n_theta, ndim, nP], stage_points [n_stages-1, n_theta, ndim, nP] or None)."""
    _require(points, "points")
    _require(As, "As")
    _require(trels, "Trels")
    n_theta = As.shape[0] // n_stages
    nP = points.shape[-1]
    out = torch.empty((n_theta, ndim, nP), device=As.device, dtype=torch.float32)
    sp = (torch.empty((n_stages - 1, n_theta, ndim, nP), device=As.device, dtype=torch.float32)
          if n_stages > 1 else None)
    with _on(As.device):
        _check(lib().cpab_b200_forward_chain(
            ndim, _i32_array(nc), _ptr(points), nP, int(batched), _ptr(order), _ptr(trels),
            _ptr(As), n_stages, n_theta, int(nstepsolver), int(adaptive), _ptr(sp), _ptr(out),
            _stream(As.device)))
    return out, sp


def backward_chain(ndim, nc, points, batched, As, n_stages, grad_out, stage_points, nstepsolver,
                   adaptive, want_points, order=None):
    """Returns (moments [n_stages * n_theta, nC, ppc], grad_points or None)."""
    _require(points, "points")
    _require(As, "As")
    _require(grad_out, "grad")
    n_theta, nC = As.shape[0] // n_stages, As.shape[1]
    nP = points.shape[-1]
    moments = torch.empty((n_stages * n_theta, nC, ndim * (ndim + 1)), device=As.device,
                          dtype=torch.float32)
    gp = (torch.empty((n_theta, ndim, nP), device=As.device, dtype=torch.float32)
          if want_points else None)
    with _on(As.device):
        _check(lib().cpab_b200_backward_chain(
            ndim, _i32_array(nc), _ptr(points), nP, int(batched), _ptr(order), _ptr(As), n_stages,
            n_theta, _ptr(grad_out), _ptr(stage_points), int(nstepsolver), int(adaptive),
            _ptr(moments), _ptr(gp), _stream(As.device)))
    return moments, gp
