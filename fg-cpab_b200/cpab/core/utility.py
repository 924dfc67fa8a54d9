"""Small helpers shared by the host code (cpab/core/utility.py of the reference)."""
import os
import pickle

import numpy as np
import scipy.linalg as la
import scipy.sparse as sp


class params:
    """Attribute bag holding a transformation's configuration.

    Same role and field names as the reference's ``params`` container
    (cpab/core/utility.py:11-16), so callers that read ``T.params.nc`` etc.
    keep working.
    """

    def __getattr__(self, name):
        # Fields registered in ``_lazy`` (e.g. constrain_mat) are computed on
        # first access and then stored like ordinary attributes.
        lazy = self.__dict__.get("_lazy", {})
        if name in lazy:
            value = lazy.pop(name)()
            setattr(self, name, value)
            return value
        raise AttributeError(name)

    def __repr__(self):
        return str({k: v for k, v in self.__dict__.items() if not k.startswith("_")})


def get_dir(file):
    """Directory containing ``file`` (symlinks resolved)."""
    return os.path.dirname(os.path.realpath(file))


def create_dir(direc):
    """Create ``direc`` (and parents) if it does not exist."""
    os.makedirs(direc, exist_ok=True)


def check_if_file_exist(file):
    return os.path.isfile(file)


def load_obj(name):
    """Load ``name + '.pkl'`` (the reference's basis cache format)."""
    with open(name + ".pkl", "rb") as f:
        return pickle.load(f)


def save_obj(obj, name):
    with open(name + ".pkl", "wb") as f:
        pickle.dump(obj, f, pickle.HIGHEST_PROTOCOL)


def drop_zero_rows(A):
    """Remove the rows of a CSR matrix that hold no stored entries."""
    A = A.tocsr()
    keep = np.flatnonzero(np.diff(A.indptr))
    return A if keep.size == A.shape[0] else A[keep]


def null(A, eps=1e-6, zero_tol=None):
    """Orthonormal null-space basis of A (columns), entries <= tol zeroed, CSR.

    Right-singular vectors of a full SVD whose singular value is <= eps, plus
    those beyond the rank deficit of a wide matrix -- the rule of the
    reference's ``null`` (cpab/core/utility.py:36-56).  The same LAPACK call is
    used so that the basis chosen inside a degenerate null space is the same.
    """
    A = A.toarray() if sp.issparse(A) else np.asarray(A)
    if A.shape[1] == 0:
        return sp.csr_matrix((0, 0))
    _, s, vh = la.svd(A)
    extra = max(0, A.shape[1] - s.shape[0])
    mask = np.concatenate((s <= eps, np.ones(extra, dtype=bool)))
    Z = vh[mask].T.copy()
    Z[np.abs(Z) <= (eps if zero_tol is None else zero_tol)] = 0.0
    Z = sp.csr_matrix(Z)
    Z.eliminate_zeros()
    return Z


def make_hashable(arr):
    """Rows of a 2D array as a tuple of tuples (usable in sets and as keys)."""
    return tuple(tuple(row.tolist()) for row in arr)
