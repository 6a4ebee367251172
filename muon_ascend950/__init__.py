"""Drop-in alias: ``import muon_ascend950`` resolves to the B200 build.

Code written against the Ascend 950PR package
(``from muon_ascend950 import polar_step``) runs unchanged on CUDA tensors.
"""

from muon_fusion_ascend950_b200 import __version__, load_library, polar_step  # noqa: F401

__all__ = ["polar_step"]
