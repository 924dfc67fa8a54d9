"""Tessellations of [0,1]^ndim and their continuous piecewise-affine (CPA) basis.

A CPA velocity field is affine inside every cell (intervals in 1D, four
triangles per square in 2D, five tetrahedra per cube in 3D) and continuous
across cells.  Its cell matrices A_c (ndim x ndim+1) stacked into a vector of
length D = nC * ndim * (ndim+1) are A = B theta, where the columns of the
sparse D x d matrix B span the admissible fields.

B is built the way the reference builds it (cpab/core/tesselation.py:41-307),
because theta is only meaningful relative to that exact basis:

  1. N -- the nodal prolongation: the field is determined by its values at the
     tessellation vertices (interior vertices only when zero_boundary), and
     each cell's affine map is the interpolant of its vertex values.  Such a
     field is continuous and vanishes on the boundary by construction.
  2. Constraints that N does not satisfy by construction -- continuity
     "outside" the domain when zero_boundary is False, and zero trace per cell
     when volume_perservation -- form C = L N, whose null space Z (dense SVD)
     gives B = N Z.  The continuity and zero-boundary rows of the reference's L
     evaluate to rounding noise on N and are dropped by its 1e-6 threshold, so
     they are not assembled here; the surviving rows are built in the same
     order with the same values, which keeps the SVD input -- and therefore
     the null-space basis -- identical.
  3. Columns are scaled to unit L2 norm.

The full constraint matrix L is still available (``Tesselation.L``), built
lazily on first access.
"""
import os
import uuid
import warnings
from itertools import combinations

import numpy as np
import scipy.sparse as sp

from .utility import drop_zero_rows, load_obj, null

_BASIS_VERSION = "nodal_v2"
_EPS = 1e-6


class Tesselation:
    """Base class; subclasses define the cell vertices (``_cell_vertices``)
    and the constraints that make the field continuous outside the domain
    (``_outside_pairs``).

    Attributes mirror the reference's: nc, ndim, nC, n_params, verts
    [nC, ndim+1, ndim+1] (homogeneous vertex coordinates), cells, B, L,
    nodal_vertices.
    """

    ndim = 0
    n_params = 0
    cells_per_box = 1

    def __init__(self, nc, domain_min, domain_max, zero_boundary=True,
                 volume_perservation=False, direc=None, override=False):
        self.nc = list(nc)
        self.domain_min = list(domain_min)
        self.domain_max = list(domain_max)
        self.zero_boundary = zero_boundary
        self.volume_perservation = volume_perservation
        self.nC = int(self.cells_per_box * np.prod(self.nc))
        self.dir = direc
        self._L = None
        self.verts, self.cells = self._cell_vertices()

        loaded = False
        if direc is not None and not override:
            loaded = self._load_cache()
        if not loaded:
            self.B = self._build_basis()
            if direc is not None:
                self._save_cache()

    # ------------------------------------------------------------ caching
    def _stem(self):
        return ("cpab_basis_dim%d_tess%s_vo%d_zb%d_vp%d_%s" % (
            self.ndim, "_".join(str(e) for e in self.nc), int(not self.zero_boundary),
            int(self.zero_boundary), int(self.volume_perservation), _BASIS_VERSION))

    def _load_cache(self):
        stem = os.path.join(self.dir, self._stem())
        if os.path.isfile(stem + ".npz"):
            z = np.load(stem + ".npz")
            self.B = sp.csr_matrix((z["data"], z["indices"], z["indptr"]), shape=tuple(z["shape"]))
            self.nodal_vertices = z["nodal_vertices"]
            return True
        if os.path.isfile(stem + ".pkl"):
            # A basis cached by the reference implementation (pickled __dict__).
            d = load_obj(stem)
            self.B = sp.csr_matrix(d["B"])
            self.nodal_vertices = np.asarray(d.get("nodal_vertices", np.zeros((0, self.ndim + 1))))
            if "L" in d:
                self._L = sp.csr_matrix(d["L"])
            return True
        return False

    def _save_cache(self):
        """Write the basis next to the others.  Several processes (one per
        GPU) may build the same basis at once on a fresh machine: each writes
        its own temporary file and renames it atomically, so readers only ever
        see a complete file, and a failed write only costs the cache."""
        stem = os.path.join(self.dir, self._stem())
        B = self.B.tocsr()
        tmp = "%s.%d.%s.tmp.npz" % (stem, os.getpid(), uuid.uuid4().hex[:8])
        try:
            os.makedirs(self.dir, exist_ok=True)
            np.savez(tmp, data=B.data, indices=B.indices, indptr=B.indptr,
                     shape=np.asarray(B.shape), nodal_vertices=self.nodal_vertices)
            os.replace(tmp, stem + ".npz")
        except OSError as e:
            warnings.warn("could not cache the CPA basis in %s: %s" % (self.dir, e))
            try:
                os.remove(tmp)
            except OSError:
                pass

    # ------------------------------------------------------------ geometry
    def get_cell_centers(self):
        """Centroid of every cell, [nC, ndim]."""
        return np.mean(self.verts[:, :, :self.ndim], axis=1)

    def _cell_vertices(self):
        raise NotImplementedError

    def _outside_pairs(self):
        """[(cell_i, cell_j, aux_vertex)] in constraint order."""
        return []

    def _is_boundary(self, pts):
        """Rows of pts [n, >=ndim] with any coordinate on the domain boundary."""
        on = np.zeros(len(pts), dtype=bool)
        for d in range(self.ndim):
            on |= np.isclose(pts[:, d], self.domain_min[d], atol=1e-12)
            on |= np.isclose(pts[:, d], self.domain_max[d], atol=1e-12)
        return on

    # ------------------------------------------------------------ basis
    def _nodal_prolongation(self):
        nd, P = self.ndim, self.n_params
        nv = nd + 1
        flat = self.verts.reshape(-1, nv)
        # Unique vertices in first-seen order over (cell, local vertex).
        _, first, inverse = np.unique(flat, axis=0, return_index=True, return_inverse=True)
        order = np.argsort(first, kind="stable")
        rank = np.empty_like(order)
        rank[order] = np.arange(len(order))
        vid = rank[inverse.reshape(-1)].reshape(self.nC, nv)   # discovery index per (cell, lv)
        uniq = flat[np.sort(first)]
        active = ~self._is_boundary(uniq) if self.zero_boundary else np.ones(len(uniq), bool)
        dof = np.full(len(uniq), -1, dtype=np.int64)
        dof[active] = np.arange(int(active.sum()))
        self.nodal_vertices = uniq[active]
        n_dofs = nd * int(active.sum())
        D = P * self.nC
        if n_dofs == 0:
            return sp.csr_matrix((D, 0))
        # Row lv of inv(V^T) holds vertex lv's weight in each affine coefficient.
        winv = np.linalg.inv(np.transpose(self.verts, (0, 2, 1)))  # [nC, nv(lv), nv(q)]
        c, lv, k, q = np.meshgrid(np.arange(self.nC), np.arange(nv), np.arange(nd),
                                  np.arange(nv), indexing="ij")
        a = dof[vid[c, lv]]
        val = winv[c, lv, q]
        keep = (a >= 0) & (val != 0.0)
        rows = (P * c + k * nv + q)[keep]
        cols = (nd * a + k)[keep]
        N = sp.coo_matrix((val[keep], (rows, cols)), shape=(D, n_dofs)).tocsr()
        N.eliminate_zeros()
        return N

    def _residual_constraints(self):
        """Rows of L that are not identically satisfied by the nodal basis:
        continuity through auxiliary vertices outside the domain, then zero
        trace per cell.  Same row order and entries as the reference's L."""
        nd, P = self.ndim, self.n_params
        rows, cols, vals = [], [], []
        r = 0
        if not self.zero_boundary:
            for (i, j, v) in self._outside_pairs():
                for k in range(nd):
                    for qq, value in enumerate(v):
                        if value != 0.0:
                            rows += [r, r]
                            cols += [P * i + k * (nd + 1) + qq, P * j + k * (nd + 1) + qq]
                            vals += [value, -value]
                    r += 1
        if self.volume_perservation:
            for cidx in range(self.nC):
                for k in range(nd):
                    rows.append(r)
                    cols.append(P * cidx + k * (nd + 1) + k)
                    vals.append(1.0)
                r += 1
        return sp.coo_matrix((vals, (rows, cols)), shape=(r, P * self.nC)).tocsr()

    def _build_basis(self):
        N = self._nodal_prolongation()
        C = (self._residual_constraints() @ N).tocsr()
        if C.nnz:
            C.data[np.abs(C.data) <= _EPS] = 0.0
            C.eliminate_zeros()
        C = drop_zero_rows(C)
        if C.shape[0] == 0 or C.shape[1] == 0:
            return _unit_columns(N)
        Z = null(C, eps=_EPS, zero_tol=_EPS)
        if Z.shape[1] == 0:
            return sp.csr_matrix((N.shape[0], 0))
        B = (N @ Z).tocsr()
        if B.nnz:
            B.data[np.abs(B.data) <= _EPS] = 0.0
            B.eliminate_zeros()
        return _unit_columns(B)

    # ------------------------------------------------------------ full L
    @property
    def L(self):
        """Full constraint matrix of the reference (continuity on shared
        faces, outside continuity, zero boundary, zero trace), built lazily."""
        if self._L is None:
            self._L = self._full_constraints()
        return self._L

    @L.setter
    def L(self, value):
        self._L = value

    def _shared_faces(self):
        faces = {}
        for i in range(self.nC):
            vi = [tuple(row.tolist()) for row in self.verts[i]]
            for face in combinations(vi, self.ndim):
                faces.setdefault(tuple(sorted(face)), []).append(i)
        out = []
        for face, cells in faces.items():
            for a in range(len(cells)):
                for b in range(a + 1, len(cells)):
                    out.append((cells[a], cells[b], list(face)))
        return out

    def _full_constraints(self):
        nd, P = self.ndim, self.n_params
        pairs = [(i, j, vs) for (i, j, vs) in self._shared_faces()]
        if not self.zero_boundary:
            pairs += [(i, j, [v]) for (i, j, v) in self._outside_pairs()]
        rows, cols, vals = [], [], []
        r = 0
        for (i, j, vs) in pairs:
            for v in vs:
                for k in range(nd):
                    for qq, value in enumerate(v):
                        if value != 0.0:
                            rows += [r, r]
                            cols += [P * i + k * (nd + 1) + qq, P * j + k * (nd + 1) + qq]
                            vals += [value, -value]
                    r += 1
        if self.zero_boundary:
            for cidx in range(self.nC):
                for v in self.verts[cidx]:
                    for d in range(nd):
                        if v[d] == self.domain_min[d] or v[d] == self.domain_max[d]:
                            for qq, value in enumerate(v):
                                if value != 0.0:
                                    rows.append(r)
                                    cols.append(P * cidx + d * (nd + 1) + qq)
                                    vals.append(value)
                            r += 1
        if self.volume_perservation:
            for cidx in range(self.nC):
                for k in range(nd):
                    rows.append(r)
                    cols.append(P * cidx + k * (nd + 1) + k)
                    vals.append(1.0)
                r += 1
        return sp.coo_matrix((vals, (rows, cols)), shape=(r, P * self.nC)).tocsr()


def _unit_columns(B):
    """Scale every column of B to unit L2 norm (zero columns untouched)."""
    if B.shape[1] == 0:
        return B.tocsr()
    Bc = B.tocsc(copy=True)
    norms = np.sqrt(np.asarray(Bc.power(2).sum(axis=0)).ravel())
    norms[norms == 0.0] = 1.0
    counts = np.diff(Bc.indptr)
    Bc.data /= np.repeat(norms, counts)
    Bc.eliminate_zeros()
    return Bc.tocsr()


class Tesselation1D(Tesselation):
    """nc[0] intervals.  cpab/core/tesselation.py:309-346."""
    ndim = 1
    n_params = 2
    cells_per_box = 1

    def _cell_vertices(self):
        x = np.linspace(self.domain_min[0], self.domain_max[0], self.nc[0] + 1)
        verts = np.stack([np.stack([x[:-1], np.ones(self.nc[0])], axis=1),
                          np.stack([x[1:], np.ones(self.nc[0])], axis=1)], axis=1)
        return verts, list(range(self.nc[0]))


class Tesselation2D(Tesselation):
    """Every square split by its diagonals into triangles bottom(0), right(1),
    top(2), left(3); squares row-major with x fastest.
    cpab/core/tesselation.py:349-455."""
    ndim = 2
    n_params = 6
    cells_per_box = 4

    def _cell_vertices(self):
        nx, ny = self.nc
        X = np.linspace(self.domain_min[0], self.domain_max[0], nx + 1)
        Y = np.linspace(self.domain_min[1], self.domain_max[1], ny + 1)
        verts, cells = [], []
        for iy in range(ny):
            for ix in range(nx):
                x0, x1, y0, y1 = X[ix], X[ix + 1], Y[iy], Y[iy + 1]
                ctr = ((x0 + x1) / 2, (y0 + y1) / 2, 1.0)
                a, b, c, d = (x0, y0, 1.0), (x1, y0, 1.0), (x1, y1, 1.0), (x0, y1, 1.0)
                # Triangle = (centre, then the two corners of its outer edge).
                verts += [(ctr, a, b), (ctr, b, c), (ctr, c, d), (ctr, d, a)]
                cells += [(ix, iy, t) for t in range(4)]
        return np.asarray(verts, dtype=np.float64), cells

    def _outside_pairs(self):
        nx, ny = self.nc
        index = {cell: n for n, cell in enumerate(self.cells)}
        out = []
        for i, (ix, iy, tri) in enumerate(self.cells):
            side = None
            if ix == 0 and tri == 3:
                cand, side = [(0, iy + 1, 3), (0, iy - 1, 3)], 0
            if ix == nx - 1 and tri == 1:
                cand, side = [(nx - 1, iy + 1, 1), (nx - 1, iy - 1, 1)], 0
            if iy == 0 and tri == 0:
                cand, side = [(ix + 1, 0, 0), (ix - 1, 0, 0)], 1
            if iy == ny - 1 and tri == 2:
                cand, side = [(ix + 1, ny - 1, 2), (ix - 1, ny - 1, 2)], 1
            if side is None:
                continue
            for other in cand:
                j = index.get(other)
                if j is None or j <= i:
                    continue
                common = set(map(tuple, self.verts[i].tolist())) & set(map(tuple, self.verts[j].tolist()))
                if len(common) != 1:
                    continue
                aux = list(next(iter(common)))
                aux[side] -= 10   # a point off the boundary along the shared edge's normal axis
                out.append((i, j, tuple(aux)))
        return out


class Tesselation3D(Tesselation):
    """Every cube split into a central tetrahedron (0) and four corner ones;
    cubes x fastest, split orientation alternating with cube parity.
    cpab/core/tesselation.py:457-578."""
    ndim = 3
    n_params = 12
    cells_per_box = 5

    def _cell_vertices(self):
        nx, ny, nz = self.nc
        X = np.linspace(self.domain_min[0], self.domain_max[0], nx + 1)
        Y = np.linspace(self.domain_min[1], self.domain_max[1], ny + 1)
        Z = np.linspace(self.domain_min[2], self.domain_max[2], nz + 1)
        verts, cells = [], []
        for iz in range(nz):
            for iy in range(ny):
                for ix in range(nx):
                    # Corners of the bottom (z0) and top (z1) faces, counter-clockwise.
                    lo = [(X[ix], Y[iy], Z[iz], 1.0), (X[ix + 1], Y[iy], Z[iz], 1.0),
                          (X[ix + 1], Y[iy + 1], Z[iz], 1.0), (X[ix], Y[iy + 1], Z[iz], 1.0)]
                    hi = [(X[ix], Y[iy], Z[iz + 1], 1.0), (X[ix + 1], Y[iy], Z[iz + 1], 1.0),
                          (X[ix + 1], Y[iy + 1], Z[iz + 1], 1.0), (X[ix], Y[iy + 1], Z[iz + 1], 1.0)]
                    if (ix + iy + iz) % 2 == 1:   # odd cubes: rotate the split a quarter turn
                        lo = lo[1:] + lo[:1]
                        hi = hi[1:] + hi[:1]
                    a0, b0, c0, d0 = lo
                    a1, b1, c1, d1 = hi
                    verts += [(d1, b1, a0, c0), (a1, b1, d1, a0), (c1, b1, d1, c0),
                              (d0, a0, c0, d1), (b0, a0, c0, b1)]
                    cells += [(ix, iy, iz, t) for t in range(5)]
        return np.asarray(verts, dtype=np.float64), cells

    def _outside_pairs(self):
        out = []
        for cube in range(self.nC // 5):
            for a in range(5):
                for b in range(a + 1, 5):
                    i, j = 5 * cube + a, 5 * cube + b
                    vi, vj = self.verts[i], self.verts[j]
                    for d in range(3):
                        low = (np.sum(vi[:, d] == self.domain_min[d]) == 3 and
                               np.sum(vj[:, d] == self.domain_min[d]) == 3)
                        high = (np.sum(vi[:, d] == self.domain_max[d]) == 3 and
                                np.sum(vj[:, d] == self.domain_max[d]) == 3)
                        if low or high:
                            ctr = [(p + q) / 2.0 for p, q in zip(vi[0].tolist(), vj[0].tolist())]
                            ctr[d] += -1 if low else 1
                            out.append((i, j, tuple(ctr)))
        return out
