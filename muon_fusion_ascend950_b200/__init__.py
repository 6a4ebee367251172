"""B200-native (sm_100a) Polar Express operator, drop-in for muon_ascend950.

``polar_step(x, a, b, c)`` computes one Polar Express (Newton-Schulz) step of
Muon, ``Y = a*X + (b*A + c*A@A) @ X`` with ``A = X @ X.mT``, on bf16 CUDA
tensors of shape ``[M,N]`` or ``[B,M,N]``.
"""

from ._loader import load_library

load_library()

from .ops import POLAR_EXPRESS_COEFFICIENTS, polar_express, polar_step  # noqa: E402
from .optim import Muon  # noqa: E402

__all__ = ["polar_step", "polar_express", "Muon", "POLAR_EXPRESS_COEFFICIENTS", "load_library"]

__version__ = "0.1.1"
