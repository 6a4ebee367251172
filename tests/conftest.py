"""Shared pytest setup: the `gpu` marker, repo import path and fixtures."""
from __future__ import annotations

import json
import sys
from pathlib import Path

import numpy as np
import pytest

REPO = Path(__file__).resolve().parent.parent
if str(REPO) not in sys.path:
    sys.path.insert(0, str(REPO))

GOLDEN = REPO / "tests" / "golden" / "polar_golden.npz"


def pytest_configure(config):
    config.addinivalue_line(
        "markers", "gpu: needs an sm_100 (B200) GPU; run with -m gpu")


def load_golden():
    """{case name: (meta, x bf16, y bf16)} from the committed fixtures."""
    import torch

    z = np.load(GOLDEN)
    meta = json.loads(bytes(z["meta"]).decode())
    cases = {}
    for case in meta["cases"]:
        x = torch.from_numpy(z[case["name"] + ".x"].copy()).view(torch.bfloat16)
        y = torch.from_numpy(z[case["name"] + ".y"].copy()).view(torch.bfloat16)
        cases[case["name"]] = (case, x, y)
    return meta, cases


@pytest.fixture(scope="session")
def golden():
    return load_golden()


@pytest.fixture(scope="session")
def cuda_device():
    import torch

    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    major, minor = torch.cuda.get_device_capability(0)
    if (major, minor) != (10, 0):
        pytest.skip(f"needs sm_100, found sm_{major}{minor}")
    torch.cuda.set_device(0)
    return torch.device("cuda", 0)
