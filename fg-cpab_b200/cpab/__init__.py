"""FG-CPAB on sm_100a: CPA diffeomorphisms in 1D/2D/3D with factorized gradients.

    from cpab import Cpab

Drop-in for the reference package's public API (``Cpab``,
``cpab.pytorch.transformer.CPAB_transformer``, ``cpab.pytorch.interpolation``);
the compute path is libcpab_b200.so (hand-written CUDA for B200).
"""
from .cpab import Cpab

__all__ = ["Cpab"]
