"""Loads the native operator library and registers its FakeTensor kernel.

Mirrors muon_ascend950/_loader.py of the reference (lines 10-49): the
``MUON_ASCEND950_LIBRARY`` override, otherwise the first ``_C*.so`` next to
this file, loaded with ``torch.ops.load_library``; then
``register_fake("muon_ascend950::polar_step")`` returning
``empty_like(x, memory_format=contiguous)``, tolerating an existing
registration.  The reference imports torch_npu here; this build needs only
torch with CUDA.
"""
from __future__ import annotations

import os
from pathlib import Path

_LOADED = False


def _library_path() -> Path:
    configured = os.environ.get("MUON_ASCEND950_LIBRARY")
    if configured:
        path = Path(configured).expanduser().resolve()
        if not path.is_file():
            raise RuntimeError(f"MUON_ASCEND950_LIBRARY does not exist: {path}")
        return path

    package_dir = Path(__file__).resolve().parent
    candidates = sorted(package_dir.glob("_C*.so"))
    if not candidates:
        raise RuntimeError(
            "muon_ascend950 native library is missing. Build it with "
            "`python -m muon_fusion_ascend950_b200.build` (or "
            "`python -c 'import __graft_entry__ as g; g.build()'`)."
        )
    return candidates[0]


def load_library() -> None:
    global _LOADED
    if _LOADED:
        return

    try:
        import torch
    except ImportError as exc:  # pragma: no cover - torch is a hard requirement
        raise RuntimeError("muon_ascend950 requires torch") from exc

    torch.ops.load_library(str(_library_path()))

    def fake_polar_step(x, a: float, b: float, c: float):
        return torch.empty_like(x, memory_format=torch.contiguous_format)

    def fake_polar_express(x, coefficients, normalize=True):
        return torch.empty_like(x, dtype=torch.bfloat16, memory_format=torch.contiguous_format)

    def fake_muon_update(param, grad, momentum_buffer, lr, momentum, nesterov, weight_decay,
                         scale, coefficients):
        return None

    # Extensions of this build: polar_step_t (the step of x^T in x's layout)
    # has polar_step's output contract; polar_express returns bf16 of x's
    # shape; muon_update_ mutates its arguments and returns nothing.
    fakes = (("muon_ascend950::polar_step", fake_polar_step),
             ("muon_ascend950::polar_step_t", fake_polar_step),
             ("muon_ascend950::polar_express", fake_polar_express),
             ("muon_ascend950::muon_update_", fake_muon_update))
    for name, fn in fakes:
        try:
            torch.library.register_fake(name)(fn)
        except RuntimeError as exc:
            if "already has" not in str(exc):
                raise
    _LOADED = True
