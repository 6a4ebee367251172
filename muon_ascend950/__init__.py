"""Drop-in alias: ``import muon_ascend950`` resolves to the B200 build.

Code written against the Ascend 950PR package runs unchanged on CUDA
tensors: ``from muon_ascend950 import polar_step``, and the reference's
submodule paths ``muon_ascend950.ops`` (ops.py) and
``muon_ascend950._loader`` (_loader.py) name this build's modules of the same
role, registered here as the same module objects.
"""
import sys as _sys

import muon_fusion_ascend950_b200 as _impl
from muon_fusion_ascend950_b200 import _loader, ops  # noqa: F401
from muon_fusion_ascend950_b200 import __version__, load_library, polar_step  # noqa: F401

_sys.modules[__name__ + ".ops"] = ops
_sys.modules[__name__ + "._loader"] = _loader

__all__ = ["polar_step"]
del _impl
