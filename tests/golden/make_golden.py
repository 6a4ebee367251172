"""Generate the golden vectors in tests/golden/polar_golden.npz.

Runs the reference's OWN accuracy oracle -- the ``_reference`` function and
``COEFFICIENTS`` table of tests/test_polar_step.py in
Lucien-Nova/Muon_fusion_Ascend950 -- on seeded inputs and stores inputs and
outputs as bf16 bit patterns.  The two definitions are extracted from the
reference test file with ``ast`` and executed on their own, because the
module as a whole calls ``pytest.importorskip("torch_npu")`` at import time.

Usage (build container only; the reference tree is not present on GPU
boxes, which use the committed .npz):

    python tests/golden/make_golden.py <reference>/tests/test_polar_step.py
"""
from __future__ import annotations

import ast
import json
import sys
from pathlib import Path

import numpy as np
import torch

HERE = Path(__file__).resolve().parent
REPO = HERE.parent.parent
sys.path.insert(0, str(REPO))

from oracle.polar_oracle import make_input  # noqa: E402

# The reference test file: first command-line argument, else the
# MUON_REFERENCE_TEST environment variable (no default path).
SOURCE_ENV = "MUON_REFERENCE_TEST"

# (name, shape, seed, number of Polar Express steps)
CASES = (
    ("cfg2_129x130", (129, 130), 0, 1),
    ("cfg2_2x150x2050", (2, 150, 2050), 0, 1),
    ("cfg2_1x130x129", (1, 130, 129), 0, 1),
    ("five_step_1x129x130", (1, 129, 130), 0, 5),
    ("aligned_1x128x256", (1, 128, 256), 0, 1),
)


def load_reference_oracle(source: Path):
    """Return (_reference, COEFFICIENTS) defined by the reference test file."""
    tree = ast.parse(source.read_text(encoding="utf-8"), filename=str(source))
    keep = []
    for node in tree.body:
        if isinstance(node, ast.FunctionDef) and node.name == "_reference":
            keep.append(node)
        elif isinstance(node, ast.Assign) and any(
            isinstance(t, ast.Name) and t.id == "COEFFICIENTS" for t in node.targets
        ):
            keep.append(node)
    if len(keep) != 2:
        raise RuntimeError(f"_reference / COEFFICIENTS not found in {source}")
    module = ast.Module(body=keep, type_ignores=[])
    namespace = {"torch": torch}
    exec(compile(module, str(source), "exec"), namespace)
    return namespace["_reference"], namespace["COEFFICIENTS"]


def bits(t: torch.Tensor) -> np.ndarray:
    return t.contiguous().view(torch.int16).numpy().copy()


def main() -> None:
    import os

    arg = sys.argv[1] if len(sys.argv) > 1 else os.environ.get(SOURCE_ENV)
    if not arg:
        raise SystemExit(f"usage: make_golden.py <reference tests/test_polar_step.py> "
                         f"(or set {SOURCE_ENV})")
    source = Path(arg)
    reference, coefficients = load_reference_oracle(source)
    arrays = {}
    meta = {"source": "tests/test_polar_step.py:_reference", "torch": torch.__version__,
            "coefficients": [list(c) for c in coefficients], "cases": []}
    for name, shape, seed, steps in CASES:
        x = make_input(shape, seed)
        y = reference(x, coefficients[:steps])
        assert y.dtype == torch.bfloat16 and y.shape == x.shape
        arrays[f"{name}.x"] = bits(x)
        arrays[f"{name}.y"] = bits(y)
        meta["cases"].append({"name": name, "shape": list(shape), "seed": seed, "steps": steps})
    arrays["meta"] = np.frombuffer(json.dumps(meta).encode(), dtype=np.uint8)
    out = HERE / "polar_golden.npz"
    np.savez_compressed(out, **arrays)
    print(f"wrote {out} ({out.stat().st_size} bytes, {len(CASES)} cases)")


if __name__ == "__main__":
    main()
