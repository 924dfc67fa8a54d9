"""CPU parity oracle for the FG-CPAB hot path.

TEST INFRASTRUCTURE ONLY: imported by tests/, __graft_entry__.smoke() and the
CPU-baseline legs of bench.py, as the checker -- never by the product.

  * integration / adjoint / expm / cell lookup: liboracle.so, the C
    restatement in cpab_oracle.c (cpab/core/cpab_ops_{1,2,3}d.cu);
  * A = B theta and dtheta = B^T m: fp32 CSR products summed in the GPU
    kernels' fixed order (one fma chain per row for A; 32-nonzero chunk sums
    added left to right for dtheta), the products torch.sparse.mm computes
    in cpab/pytorch/transformer.py:84-88, :165-166;
  * resampling: numpy float32 restatement of cpab/pytorch/interpolation.py:8-160
    (forward, op for op) and of the gradient its autograd graph produces.

Pinned against the reference by the golden fixtures in tests/golden/ (basis
and interpolation from the reference's Python run on CPU; kernel outputs from
the reference's CUDA kernels built into oracle/_ref and run on a B200).
"""
import ctypes
import os

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "liboracle.so")

_c_int, _c_i64, _c_f, _p = ctypes.c_int, ctypes.c_int64, ctypes.c_float, ctypes.c_void_p
_lib = None


def lib():
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            import importlib.util
            spec = importlib.util.spec_from_file_location(
                "build_oracle", os.path.join(HERE, "build_oracle.py"))
            mod = importlib.util.module_from_spec(spec)
            spec.loader.exec_module(mod)
            mod.build_oracle()
        L = ctypes.CDLL(LIB_PATH)
        L.oracle_cells.argtypes = [_c_int, _p, _p, _c_i64, _p]
        L.oracle_expm.argtypes = [_c_int, _p, _c_i64, _c_f, _p]
        L.oracle_forward.argtypes = [_c_int, _p, _p, _c_i64, _c_int, _p, _p, _c_int, _c_int, _c_int, _p]
        L.oracle_backward.argtypes = [_c_int, _p, _p, _c_i64, _c_int, _p, _c_int, _p, _c_int, _c_int,
                                      _p, _p]
        L.oracle_midpoint_forward.argtypes = [_c_int, _p, _p, _c_i64, _c_int, _p, _c_int, _c_int,
                                              _c_int, _p]
        L.oracle_midpoint_forward.restype = None
        L.oracle_csr_matmul.argtypes = [_c_i64, _p, _p, _p, _c_int, _p, _c_i64, _p, _c_i64, _c_int]
        L.oracle_csr_matmul.restype = None
        L.oracle_num_threads.restype = _c_int
        L.oracle_set_num_threads.argtypes = [_c_int]
        for fn in (L.oracle_cells, L.oracle_expm, L.oracle_forward, L.oracle_backward):
            fn.restype = None
        _lib = L
    return _lib


def _f32(a):
    return np.ascontiguousarray(a, dtype=np.float32)


def _ptr(a):
    return a.ctypes.data_as(ctypes.c_void_p) if a is not None else ctypes.c_void_p(0)


def _nc(nc):
    return np.ascontiguousarray(nc, dtype=np.int32)


def num_threads():
    return lib().oracle_num_threads()


def set_num_threads(n):
    lib().oracle_set_num_threads(int(n))


def n_cells(nc):
    k = int(np.prod(nc))
    return {1: k, 2: 4 * k, 3: 5 * k}[len(nc)]


def cells(nc, points):
    """Cell index of every point, points [ndim, n] -> int32 [n]."""
    pts = _f32(points)
    nd, n = pts.shape
    out = np.empty(n, dtype=np.int32)
    nca = _nc(nc)
    lib().oracle_cells(nd, _ptr(nca), _ptr(pts), n, _ptr(out))
    return out


def expm(As, dT):
    """Trels for As [..., ndim, ndim+1]."""
    A = _f32(As)
    nd = A.shape[-2]
    out = np.empty_like(A)
    lib().oracle_expm(nd, _ptr(A), A.size // (nd * (nd + 1)), float(dT), _ptr(out))
    return out


def _csr32(M):
    M = M.tocsr().astype(np.float32)
    M.sort_indices()
    return (np.ascontiguousarray(M.indptr, np.int32), np.ascontiguousarray(M.indices, np.int32),
            np.ascontiguousarray(M.data, np.float32))


# Nonzeros per chunk of the projection's rows (k_project sums 32-nonzero
# chunks on different warps and adds the chunk sums left to right).
PROJECT_CHUNK = 32


def csr_matmul(M, X, chunk=0):
    """(M @ X^T)^T for a sparse M [rows, cols] and X [n, cols] in fp32, summed
    in the GPU kernels' order: chunk = 0, one fma chain per row; chunk = K, an
    fma chain per K consecutive nonzeros of a row, chunk sums added left to
    right."""
    X = _f32(X)
    rp, ci, v = _csr32(M)
    rows = M.shape[0]
    out = np.empty((X.shape[0], rows), dtype=np.float32)
    lib().oracle_csr_matmul(rows, _ptr(rp), _ptr(ci), _ptr(v), X.shape[0], _ptr(X), X.shape[1],
                            _ptr(out), rows, int(chunk))
    return out


def build_A(basis, theta, ndim):
    """As [n_theta, nC, ndim, ndim+1] = reshape(B theta^T)^T (fp32), every
    entry one fma chain over its row of B (k_build_A's order in both of its
    mappings)."""
    th = _f32(theta)
    nC = basis.shape[0] // (ndim * (ndim + 1))
    return csr_matmul(basis, th, 0).reshape(th.shape[0], nC, ndim, ndim + 1)


def project(basis, moments):
    """dtheta [n_theta, d] = B^T vec(moments) (fp32), every entry summed in
    32-nonzero chunks of its row of B^T (k_project's order)."""
    m = _f32(moments).reshape(moments.shape[0], -1)
    return csr_matmul(basis.T, m, PROJECT_CHUNK)


def integrate(nc, points, As, trels, nstepsolver=50, adaptive=False):
    """Forward integration; points [ndim, nP] or [n_theta, ndim, nP]."""
    pts, A = _f32(points), _f32(As)
    nd = A.shape[2]
    n_theta = A.shape[0]
    batched = int(pts.ndim == 3)
    nP = pts.shape[-1]
    out = np.empty((n_theta, nd, nP), dtype=np.float32)
    tr = _f32(trels) if trels is not None else None
    nca = _nc(nc)
    lib().oracle_forward(nd, _ptr(nca), _ptr(pts), nP, batched, _ptr(tr), _ptr(A), n_theta,
                         int(nstepsolver), int(adaptive), _ptr(out))
    return out


def midpoint_integrate(nc, points, As, nstepsolver=50, adaptive=False):
    """The midpoint-rule trajectory end points that the adjoint differentiates."""
    pts, A = _f32(points), _f32(As)
    nd, n_theta = A.shape[2], A.shape[0]
    batched = int(pts.ndim == 3)
    nP = pts.shape[-1]
    out = np.empty((n_theta, nd, nP), dtype=np.float32)
    nca = _nc(nc)
    lib().oracle_midpoint_forward(nd, _ptr(nca), _ptr(pts), nP, batched, _ptr(A), n_theta,
                                  int(nstepsolver), int(adaptive), _ptr(out))
    return out


def adjoint(nc, points, As, grad_out, nstepsolver=50, adaptive=False, want_points=True):
    """Fused adjoint: (moments [n_theta, nC, ppc], grad_points [n_theta, ndim, nP])."""
    pts, A, g = _f32(points), _f32(As), _f32(grad_out)
    n_theta, nC, nd = A.shape[0], A.shape[1], A.shape[2]
    batched = int(pts.ndim == 3)
    nP = pts.shape[-1]
    mom = np.empty((n_theta, nC, nd * (nd + 1)), dtype=np.float32)
    gp = np.empty((n_theta, nd, nP), dtype=np.float32) if want_points else None
    nca = _nc(nc)
    lib().oracle_backward(nd, _ptr(nca), _ptr(pts), nP, batched, _ptr(A), n_theta, _ptr(g),
                          int(nstepsolver), int(adaptive), _ptr(mom), _ptr(gp))
    return mom, gp


def transform(nc, basis, points, theta, nstepsolver=50, adaptive=False):
    """The reference's forward composition: (x_t, As, Trels)."""
    nd = len(nc)
    As = build_A(basis, theta, nd)
    trels = expm(As, 1.0 / nstepsolver) if nd > 1 else None
    return integrate(nc, points, As, trels, nstepsolver, adaptive), As, trels


def gradient(nc, basis, points, As, grad_out, nstepsolver=50, adaptive=False):
    """The reference's backward composition: (dtheta, grad_points as returned)."""
    mom, gp = adjoint(nc, points, As, grad_out, nstepsolver, adaptive, True)
    if np.asarray(points).ndim == 2:
        gp = gp.sum(axis=0, dtype=np.float32)
    return project(basis, mom), gp


# ---------------------------------------------------------------------------
# Resampling (cpab/pytorch/interpolation.py:8-160), float32, op by op.
# ---------------------------------------------------------------------------

def _axis(g, n):
    x = (g.astype(np.float32) * np.float32(n - 1)).astype(np.float32)
    f = np.floor(x)
    lo = np.clip(f, 0, n - 1)
    hi = np.clip(f + 1, 0, n - 1)
    w = (x - lo).astype(np.float32)
    return lo.astype(np.int64), hi.astype(np.int64), w


def _lerp(a, b, w):
    one = np.float32(1.0)
    return (a * (one - w)).astype(np.float32) + (b * w).astype(np.float32)


def interpolate(ndim, data, grid, outsize):
    """data [B, C, *in], grid [B, ndim, P] -> [B, C, *outsize]."""
    data = _f32(data)
    grid = _f32(grid)
    B, C = data.shape[:2]
    bidx = np.arange(B)[:, None]
    if ndim == 1:
        x0, x1, xw = _axis(grid[:, 0], data.shape[2])
        c0 = data[bidx, :, x0]      # [B, P, C]
        c1 = data[bidx, :, x1]
        out = _lerp(c0, c1, xw[..., None])
        return np.ascontiguousarray(out.transpose(0, 2, 1).reshape(B, C, *outsize))
    if ndim == 2:
        x0, x1, xw = _axis(grid[:, 0], data.shape[2])
        y0, y1, yw = _axis(grid[:, 1], data.shape[3])
        g = lambda xi, yi: data[bidx, :, xi, yi]
        xw, yw = xw[..., None], yw[..., None]
        c0 = _lerp(g(x0, y0), g(x1, y0), xw)
        c1 = _lerp(g(x0, y1), g(x1, y1), xw)
        c = _lerp(c0, c1, yw)       # [B, P, C], P = i0 + n0*i1
        n0, n1 = outsize
        return np.ascontiguousarray(c.reshape(B, n1, n0, C).transpose(0, 3, 2, 1))
    x0, x1, xw = _axis(grid[:, 0], data.shape[2])
    y0, y1, yw = _axis(grid[:, 1], data.shape[3])
    z0, z1, zw = _axis(grid[:, 2], data.shape[4])
    g = lambda xi, yi, zi: data[bidx, :, xi, yi, zi]
    xw, yw, zw = xw[..., None], yw[..., None], zw[..., None]
    c00 = _lerp(g(x0, y0, z0), g(x1, y0, z0), xw)
    c01 = _lerp(g(x0, y0, z1), g(x1, y0, z1), xw)
    c10 = _lerp(g(x0, y1, z0), g(x1, y1, z0), xw)
    c11 = _lerp(g(x0, y1, z1), g(x1, y1, z1), xw)
    c0 = _lerp(c00, c10, yw)
    c1 = _lerp(c01, c11, yw)
    c = _lerp(c0, c1, zw)
    n0, n1, n2 = outsize
    return np.ascontiguousarray(c.reshape(B, n2, n1, n0, C).transpose(0, 4, 3, 2, 1))


def _gdiff(g, hi, lo):
    """sum_ch(g*hi) - sum_ch(g*lo), float32 (autograd's two product edges)."""
    f = np.float32
    return (g * hi).astype(f).sum(-1, dtype=f) - (g * lo).astype(f).sum(-1, dtype=f)


def interpolate_backward(ndim, data, grid, outsize, grad_out):
    """Gradients (d grid [B, ndim, P], d data [B, C, *in]) of interpolate.

    d grid restates, in float32, the autograd graph of the reference's
    expressions (c = c0*(1-w) + c1*w nested per axis): per axis the gradient
    of the weight is sum_ch(g*hi) - sum_ch(g*lo) with g the incoming gradient
    of that lerp, then times (in_size-1).  d data is the scatter-add of
    g * weights, accumulated in float64."""
    f = np.float32
    data = _f32(data)
    grid = _f32(grid)
    B, C = data.shape[:2]
    P = grid.shape[2]
    g = _f32(grad_out)
    # [B, C, *outsize] -> [B, P, C] with P in grid order (coordinate 0 fastest)
    g = g.reshape(B, C, -1).transpose(0, 2, 1) if ndim == 1 else np.moveaxis(g, 1, -1).transpose(
        *([0] + list(range(ndim, 0, -1)) + [ndim + 1])).reshape(B, P, C)
    g = np.ascontiguousarray(g, dtype=f)
    bidx = np.arange(B)[:, None]
    axes = [_axis(grid[:, k], data.shape[2 + k]) for k in range(ndim)]
    one = f(1.0)
    dgrid = np.zeros((B, ndim, P), dtype=f)
    ddata = np.zeros(data.shape, dtype=np.float64)

    def corner(*bits):
        return data[(bidx, slice(None)) + tuple(axes[k][1] if b else axes[k][0]
                                                for k, b in enumerate(bits))]

    def scatter(bits, val):
        idx = tuple(axes[k][1] if b else axes[k][0] for k, b in enumerate(bits))
        for b in range(B):
            np.add.at(ddata[b], (slice(None),) + tuple(i[b] for i in idx), val[b].T)

    w = [a[2][..., None] for a in axes]
    wc = [(one - a[2])[..., None] for a in axes]
    if ndim == 1:
        c0, c1 = corner(0), corner(1)
        dgrid[:, 0] = _gdiff(g, c1, c0)
        scatter((0,), g * wc[0])
        scatter((1,), g * w[0])
    elif ndim == 2:
        c00, c01, c10, c11 = corner(0, 0), corner(0, 1), corner(1, 0), corner(1, 1)
        c0 = _lerp(c00, c10, w[0])
        c1 = _lerp(c01, c11, w[0])
        g0, g1 = (g * wc[1]).astype(f), (g * w[1]).astype(f)
        dgrid[:, 0] = _gdiff(g0, c10, c00) + _gdiff(g1, c11, c01)
        dgrid[:, 1] = _gdiff(g, c1, c0)
        for bits, val in (((0, 0), g0 * wc[0]), ((1, 0), g0 * w[0]), ((0, 1), g1 * wc[0]),
                          ((1, 1), g1 * w[0])):
            scatter(bits, val)
    else:
        c = {bits: corner(*bits) for bits in __import__("itertools").product((0, 1), repeat=3)}
        # lerp along x at each (y, z)
        cx = {(y, z): _lerp(c[(0, y, z)], c[(1, y, z)], w[0]) for y in (0, 1) for z in (0, 1)}
        c0 = _lerp(cx[(0, 0)], cx[(1, 0)], w[1])
        c1 = _lerp(cx[(0, 1)], cx[(1, 1)], w[1])
        gc0, gc1 = (g * wc[2]).astype(f), (g * w[2]).astype(f)
        dgrid[:, 2] = _gdiff(g, c1, c0)
        dgrid[:, 1] = _gdiff(gc0, cx[(1, 0)], cx[(0, 0)]) + _gdiff(gc1, cx[(1, 1)], cx[(0, 1)])
        gy = {(0, 0): (gc0 * wc[1]).astype(f), (1, 0): (gc0 * w[1]).astype(f),
              (0, 1): (gc1 * wc[1]).astype(f), (1, 1): (gc1 * w[1]).astype(f)}
        dgrid[:, 0] = sum(_gdiff(gy[(y, z)], c[(1, y, z)], c[(0, y, z)])
                          for z in (0, 1) for y in (0, 1))
        for (y, z), gv in gy.items():
            scatter((0, y, z), gv * wc[0])
            scatter((1, y, z), gv * w[0])
    for k in range(ndim):
        dgrid[:, k] = dgrid[:, k] * f(data.shape[2 + k] - 1)
    return dgrid, ddata.astype(f)


# ---------------------------------------------------------------------------
# The spatial-transformer sampling (stn/stn.py:48-54 of the reference):
# F.grid_sample(x, grid, align_corners=True, padding_mode) bilinear (2D) /
# trilinear (3D), at CPAB points p whose grid coordinate is g = 2p - 1
# (stn/stn.py:86; CPAB coordinate k along image axis k).  Restates PyTorch
# 2.11's rule (aten/src/ATen/native/GridSampler.h: unnormalisation and
# padding; aten/src/ATen/native/cuda/GridSampler.cu: neighbours, weights and
# gradients).  The source index is evaluated in float32 as there; weights
# and sums in float64 (a checker, compared within tolerances).
# ---------------------------------------------------------------------------

GRID_SAMPLE_PADDING = {"zeros": 0, "border": 1, "reflection": 2}


def _gs_index(p, n, padding):
    """(source index [float32], d index / d g) along an axis of n pixels."""
    f = np.float32
    p = _f32(p)
    g = (p * f(2) - f(1)).astype(f)
    top = f(n - 1)
    x = (((g + f(1)).astype(f) * f(0.5)).astype(f) * top).astype(f)
    mult = np.full(x.shape, float(top) * 0.5)
    if padding == "reflection":
        if n == 1:
            x = np.zeros_like(x)
            mult = np.zeros_like(mult)
        else:
            sgn = np.where(x < 0, -1.0, 1.0)
            a = np.abs(x)
            extra = np.fmod(a, top).astype(f)
            flips = np.floor((a / top).astype(f)).astype(np.int64)
            odd = flips % 2 == 1
            x = np.where(odd, (top - extra).astype(f), extra).astype(f)
            mult = mult * np.where(odd, -sgn, sgn)
    if padding in ("border", "reflection"):
        clamped = (x <= 0) | (x >= top)
        x = np.clip(x, f(0), top).astype(f)
        mult = np.where(clamped, 0.0, mult)
    bad = ~((x <= f(2.0 ** 31)) & (x >= f(-2.0 ** 31)))
    x = np.where(bad, f(-100.0), x).astype(f)
    return x, mult


def _gs_taps(in_size, pts, padding):
    """Per point: per axis (lo, fl, fh, mult) and the corner list."""
    nd = len(in_size)
    axes = []
    for k in range(nd):
        x, mult = _gs_index(pts[k], in_size[k], padding)
        lo = np.floor(x).astype(np.int64)
        xd = x.astype(np.float64)
        axes.append((lo, (lo + 1) - xd, xd - lo, mult))
    corners = []
    for m in range(1 << nd):
        hi = [(m >> (nd - 1 - k)) & 1 for k in range(nd)]
        idx = [axes[k][0] + hi[k] for k in range(nd)]
        inside = np.ones(pts.shape[1], dtype=bool)
        for k in range(nd):
            inside &= (idx[k] >= 0) & (idx[k] < in_size[k])
        fac = [axes[k][2] if hi[k] else axes[k][1] for k in range(nd)]
        corners.append((hi, [np.where(inside, i, 0) for i in idx], inside, fac))
    return axes, corners


def grid_sample_points(data, pts, padding="zeros"):
    """data [B or 1, C, *in], pts [B, ndim, P] (CPAB coordinates) ->
    [B, C, P]: the STN's F.grid_sample of data at the points."""
    data = np.asarray(data, dtype=np.float64)
    pts = _f32(pts)
    B, nd, P = pts.shape
    C = data.shape[1]
    in_size = data.shape[2:]
    out = np.zeros((B, C, P))
    for b in range(B):
        img = data[b if data.shape[0] > 1 else 0]
        _, corners = _gs_taps(in_size, pts[b], padding)
        for hi, idx, inside, fac in corners:
            w = np.prod(fac, axis=0)
            v = img[(slice(None),) + tuple(idx)]                  # [C, P]
            out[b] += np.where(inside, v * w, 0.0)
    return out.astype(np.float32)


def grid_sample_points_backward(data, pts, grad_out, padding="zeros"):
    """Gradients of grid_sample_points: (d pts [B, ndim, P] -- the CPAB
    coordinates, i.e. twice the grid gradient --, d data shaped like data)."""
    data = np.asarray(data, dtype=np.float64)
    pts = _f32(pts)
    g = np.asarray(grad_out, dtype=np.float64)
    B, nd, P = pts.shape
    in_size = data.shape[2:]
    dpts = np.zeros((B, nd, P))
    ddata = np.zeros(data.shape)
    for b in range(B):
        bi = b if data.shape[0] > 1 else 0
        img = data[bi]
        axes, corners = _gs_taps(in_size, pts[b], padding)
        gk = np.zeros((nd, P))
        for hi, idx, inside, fac in corners:
            v = img[(slice(None),) + tuple(idx)]                  # [C, P]
            vg = np.where(inside, (v * g[b]).sum(axis=0), 0.0)   # sum over channels
            w = np.prod(fac, axis=0)
            for k in range(nd):
                other = np.prod([fac[j] for j in range(nd) if j != k], axis=0) if nd > 1 else 1.0
                gk[k] += (1.0 if hi[k] else -1.0) * vg * other
            for c in range(data.shape[1]):
                np.add.at(ddata[bi, c], tuple(i[inside] for i in idx), (w * g[b, c])[inside])
        for k in range(nd):
            dpts[b, k] = 2.0 * axes[k][3] * gk[k]
    return dpts.astype(np.float32), ddata.astype(np.float32)


def warp_forward(nc, basis, data, thetas, axes, padding="zeros", nstepsolver=50):
    """The STN layer's forward (stn/stn.py:40-54,79-86) from the oracle's
    pieces: thetas [theta_1, ..., theta_K] (each [B, d]), theta_K acting
    first on the pixel grid whose CPAB coordinates per axis are `axes`
    ((linspace(-1, 1, n) + 1) / 2 as torch evaluates it).  Returns
    (out [B, C, *out_size], the sampled points, per stage (points in, As))."""
    nd = len(nc)
    axes = [_f32(a) for a in axes]
    out_size = [len(a) for a in axes]
    mesh = np.meshgrid(*axes, indexing="ij")
    pts = np.stack([m.reshape(-1) for m in mesh]).astype(np.float32)
    stages = []
    for theta in reversed(list(thetas)):
        As = build_A(basis, theta, nd)
        trels = expm(As, 1.0 / nstepsolver)
        stages.append((pts, As))
        pts = integrate(nc, pts, As, trels, nstepsolver)
    out = grid_sample_points(data, pts, padding)
    return out.reshape(out.shape[0], out.shape[1], *out_size), pts, stages


def warp_backward(nc, basis, data, final_pts, stages, grad_out, padding="zeros",
                  nstepsolver=50):
    """Gradients of warp_forward: (d thetas in the order of thetas, d data)."""
    g = np.asarray(grad_out, dtype=np.float32).reshape(grad_out.shape[0], grad_out.shape[1], -1)
    lam, ddata = grid_sample_points_backward(data, final_pts, g, padding)
    grads = []
    for pts, As in reversed(stages):  # last stage first
        mom, lam = adjoint(nc, pts, As, lam, nstepsolver, False, True)
        grads.append(project(basis, mom))
    return grads, ddata
