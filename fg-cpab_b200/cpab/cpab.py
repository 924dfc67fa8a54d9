"""Public API: the ``Cpab`` class (drop-in for cpab/cpab.py of the reference).

Same constructor, methods, argument meaning, shapes and assertions as the
reference; the compute path underneath is libcpab_b200 (sm_100a kernels).
"""
import numpy as np
import torch

from .core.tesselation import Tesselation1D, Tesselation2D, Tesselation3D
from .core.utility import create_dir, get_dir, params
from .pytorch.interpolation import interpolate
from .pytorch.transformer import CPAB_transformer as transformer
from .pytorch.transformer import _CPABFunction, device_basis, transform_chain
from .pytorch.transform_data import transform_data as fused_transform_data

# GPU device constant (the current CUDA device).
_DEVICE = torch.device("cuda")


class Cpab(object):
    """Continuous piecewise-affine transformations with a B200 (sm_100a) backend.

    The velocity field is affine on each cell of a regular tessellation of
    [0, 1]^ndim (intervals, four triangles per square, or five tetrahedra per
    cube) and continuous across cells; ``theta`` holds its coordinates in the
    basis of that space.

    tess_size -- cells per axis, a list or tuple of 1 to 3 positive ints
    zero_boundary -- pin the velocity to zero on the domain's boundary
    volume_perservation -- restrict the field to divergence-free ones
    override -- recompute the basis even when a cached file exists
    """

    def __init__(self, tess_size, zero_boundary=True, volume_perservation=False, override=False):
        self._check_input(tess_size, zero_boundary, volume_perservation, override)
        p = self.params = params()
        p.nc = tess_size
        p.ndim = len(tess_size)
        p.Ashape = [p.ndim, p.ndim + 1]
        p.valid_outside = not zero_boundary
        p.zero_boundary = zero_boundary
        p.volume_perservation = volume_perservation
        p.domain_max = [1] * p.ndim
        p.domain_min = [0] * p.ndim
        p.inc = [(p.domain_max[i] - p.domain_min[i]) / p.nc[i] for i in range(p.ndim)]
        p.nstepsolver = 50
        p.adaptive_substeps = False

        self._dir = get_dir(__file__) + "/../basis_files/"
        create_dir(self._dir)

        cls, p.nC, p.params_pr_cell = {
            1: (Tesselation1D, int(np.prod(p.nc)), 2),
            2: (Tesselation2D, 4 * int(np.prod(p.nc)), 6),
            3: (Tesselation3D, 5 * int(np.prod(p.nc)), 12),
        }[p.ndim]
        self.tesselation = cls(p.nc, p.domain_min, p.domain_max, p.zero_boundary,
                               p.volume_perservation, self._dir, override)
        tess = self.tesselation
        p._lazy = {"constrain_mat": lambda: tess.L}
        p.basis = self.tesselation.B
        p.D, p.d = p.basis.shape
        p.basis_gpu_sparse = None
        p.basis_gpu_sparse_t = None

    def get_theta_dim(self):
        """Return the dimensionality of the transformation parameters."""
        return self.params.d

    def get_params(self):
        """Return the parameter container for the transformation."""
        return self.params

    def get_basis(self):
        """Return the basis matrix of the transformation."""
        return self.params.basis

    def _get_basis_sparse_gpu(self, dtype=torch.float32, device=_DEVICE):
        """B as a torch sparse COO tensor on ``device`` (compatibility helper)."""
        coo = self.params.basis.tocoo()
        idx = torch.from_numpy(np.vstack((coo.row, coo.col)).astype(np.int64)).to(device)
        val = torch.from_numpy(coo.data).to(device=device, dtype=dtype)
        with torch.sparse.check_sparse_tensor_invariants(enable=True):
            return torch.sparse_coo_tensor(idx, val, size=self.params.basis.shape).coalesce()

    def set_solver_params(self, nstepsolver=50, adaptive_substeps=False):
        """Set parameters controlling the integration algorithm.

        Arguments:
            nstepsolver: int, number of integration steps (at most
                ``cpab._native.max_steps()``, 256; the reference allows 100)
            adaptive_substeps: bool, Heun crossing correction when a step
                leaves its cell
        """
        assert nstepsolver > 0, "nstepsolver must be a positive number"
        assert type(nstepsolver) == int, "nstepsolver must be integer"
        assert type(adaptive_substeps) == bool, "adaptive_substeps must be bool"
        self.params.nstepsolver = nstepsolver
        self.params.adaptive_substeps = adaptive_substeps

    def uniform_meshgrid(self, n_points, device=None):
        """[ndim, prod(n_points)] regular grid over the domain, coordinate 0 fastest."""
        device = _DEVICE if device is None else device
        lin = [torch.linspace(self.params.domain_min[i], self.params.domain_max[i], n_points[i],
                              device=device) for i in range(self.params.ndim)]
        mesh = torch.meshgrid(lin[::-1], indexing="ij")
        return torch.cat([g.reshape(1, -1) for g in mesh[::-1]], dim=0)

    def sample_transformation(self, n_sample=1, mean=None, cov=None):
        """[n_sample, d] samples of N(mean, cov) (default N(0, I))."""
        d = self.params.d
        mean = torch.zeros(d, dtype=torch.float32, device=_DEVICE) if mean is None else mean
        cov = torch.eye(d, dtype=torch.float32, device=_DEVICE) if cov is None else cov
        return torch.distributions.MultivariateNormal(mean, cov).sample((n_sample,))

    def sample_transformation_with_prior(self, n_sample=1, mean=None, length_scale=0.1,
                                         output_variance=1):
        """Smooth samples: a squared-exponential prior over the cell parameters
        (same covariance as the reference, cpab/cpab.py:164-206), pushed to
        theta space as B^T K B without materialising the D x D matrix K.

        K[(i,p),(j,q)] = v^2 exp(-M/(2 l^2)) with M = |c_i - c_j|^2 when p == q
        and M = 100 max|c_i - c_j|^2 otherwise (c = cell centres).
        """
        cov = self._prior_covariance(length_scale, output_variance)
        return self.sample_transformation(n_sample, mean=mean, cov=cov)

    def _prior_covariance(self, length_scale=0.1, output_variance=1, device=None):
        """[d, d] covariance of sample_transformation_with_prior: B^T K B, with
        K split per cell parameter k as E (nC x nC, same parameter) plus a
        constant for all other entries, so that only nC x nC and d x d
        matrices are formed (the reference builds K as a dense D x D matrix in a
        loop over cell pairs)."""
        p = self.params
        device = _DEVICE if device is None else device
        ppc = p.params_pr_cell
        centers = torch.tensor(self.tesselation.get_cell_centers(), dtype=torch.float32,
                               device=device)
        sq = (centers * centers).sum(1, keepdim=True)
        dist = sq - 2 * centers @ centers.t() + sq.t()
        scale = 2 * length_scale ** 2
        var = output_variance ** 2
        E = var * torch.exp(-(dist / scale))                    # same-parameter blocks
        e_off = var * torch.exp(-(100 * dist.max()) / scale)    # cross-parameter entries
        cov = torch.zeros(p.d, p.d, device=device)
        s = torch.zeros(p.d, device=device)
        basis = p.basis.tocsr()
        for k in range(ppc):
            Bk = basis[k::ppc].tocoo()                           # parameter k of every cell, [nC, d]
            idx = torch.from_numpy(np.vstack((Bk.col, Bk.row)).astype(np.int64)).to(device)
            with torch.sparse.check_sparse_tensor_invariants(enable=True):
                BkT = torch.sparse_coo_tensor(idx, torch.from_numpy(Bk.data).float().to(device),
                                              size=(p.d, p.nC)).coalesce()
            EBk = torch.sparse.mm(BkT, E).t()                    # E Bk (E symmetric), [nC, d]
            sk = torch.sparse.sum(BkT, dim=1).to_dense()
            cov += torch.sparse.mm(BkT, EBk) - e_off * torch.outer(sk, sk)
            s += sk
        cov += e_off * torch.outer(s, s)
        return cov

    def identity(self, n_sample=1, epsilon=0):
        """[n_sample, d] identity parameters (zeros), plus epsilon."""
        assert epsilon >= 0, "epsilon need to be larger than 0"
        return torch.zeros(n_sample, self.params.d, dtype=torch.float32, device=_DEVICE) + epsilon

    def transform_grid(self, grid, theta):
        """Move every point of ``grid`` along the flow of each transformation.

        ``grid`` is shared by all transformations as [ndim, n_points], or
        given per transformation as [n_batch, ndim, n_points]; ``theta`` is
        [n_batch, d].  Returns the end points, [n_batch, ndim, n_points],
        differentiable in ``theta`` and in ``grid``.
        """
        if len(grid.shape) == 3:
            assert grid.shape[0] == theta.shape[0], \
                "When passing a batched grid, the first dimension must match theta"
        return transformer(grid, theta, self.params, compute_points_grad=True)

    def transform_grid_chain(self, grid, theta_chain, scale_by_dt=False):
        """Compose several transformations: stage i moves the output of stage i-1.

        ``theta_chain`` is [n_stages, d] (one transformation per stage) or
        [n_stages, n_batch, d]; ``grid`` is laid out as in transform_grid.
        With ``scale_by_dt`` every stage's theta is divided by n_stages, so
        that the chain integrates over unit time in total.  Returns
        [n_batch, ndim, n_points].
        """
        assert type(scale_by_dt) == bool, "scale_by_dt must be bool"
        assert theta_chain.dim() in (2, 3), \
            "theta_chain must have shape [n_transforms, d] or [n_transforms, n_batch, d]"
        if theta_chain.dim() == 2:
            theta_chain = theta_chain[:, None, :]
        n_transforms, n_batch, d = theta_chain.shape
        assert n_transforms > 0, "theta_chain must contain at least one transform"
        assert d == self.params.d, f"theta_chain has d={d}, expected d={self.params.d}"
        if grid.dim() == 3:
            assert grid.shape[0] == n_batch, \
                "When passing a 3D grid, its batch dimension must match theta_chain"
        dt = (1.0 / n_transforms) if scale_by_dt else 1.0
        if self.params.ndim in (2, 3) and n_transforms > 1:
            # One kernel through all stages each way (same per-stage arithmetic).
            return transform_chain(grid, theta_chain * dt, self.params, compute_points_grad=True)
        out = grid
        for i in range(n_transforms):
            out = transformer(out, theta_chain[i] * dt, self.params, compute_points_grad=True)
        return out

    def interpolate(self, data, grid, outsize):
        """Resample data [n_batch, C, *in_size] at grid [n_batch, ndim, prod(outsize)]."""
        return interpolate(self.params.ndim, data, grid, outsize)

    def transform_data(self, data, theta, outsize):
        """transform_grid of a uniform meshgrid followed by interpolate.

        2D and 3D run both in one fused kernel each way (same results as the
        composition); 1D composes transform_grid and interpolate.

        Output: [n_batch, n_channels, *outsize]
        """
        if self.params.ndim in (2, 3):
            return fused_transform_data(data, theta, self.params, outsize)
        grid = self.uniform_meshgrid(outsize, device=theta.device)
        grid_t = self.transform_grid(grid, theta)
        return self.interpolate(data, grid_t, outsize)

    def _check_input(self, tess_size, zero_boundary, volume_perservation, override):
        assert type(tess_size) in [list, tuple], "tess_size must be a list or tuple"
        assert len(tess_size) in [1, 2, 3], "Only 1D, 2D, and 3D tesselations are supported"
        assert all([type(e) == int for e in tess_size]), "All elements must be integers"
        assert all([e > 0 for e in tess_size]), "All elements must be positive"
        assert type(zero_boundary) == bool, "zero_boundary must be True or False"
        assert type(volume_perservation) == bool, "volume_perservation must be True or False"
        assert type(override) == bool, "override must be True or False"

    def __repr__(self):
        p = self.params
        rows = [("dimensions", p.ndim), ("cells per axis", p.nc), ("cells", p.nC),
                ("theta length d", p.d), ("domain", "%s to %s" % (p.domain_min, p.domain_max)),
                ("zero boundary", p.zero_boundary),
                ("volume preserving", p.volume_perservation)]
        return "Cpab (sm_100a backend)\n" + "\n".join("  %-18s %s" % r for r in rows)
