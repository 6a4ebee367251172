"""In-tree build of the two native libraries of this package.

* ``libmuon_polar_sm100.so`` -- the sm_100a kernels and the C ABI declared in
  ``include/muon_polar_sm100.h`` (nvcc, static CUDA runtime, no torch): the
  Polar Express step (``muon_polar_sm100.cu``) and the Muon update around it
  (``muon_update_sm100.cu``).
* ``_C.so`` -- the PyTorch operator ``muon_ascend950::polar_step`` on the CUDA
  dispatch key, linked against the library above (rpath ``$ORIGIN``).

Both land next to this file so that they travel with the source tree.  The
build is skipped when the outputs are newer than every input.  Run with
``python -m muon_fusion_ascend950_b200.build`` (``--force`` to rebuild).
"""
from __future__ import annotations

import os
import shutil
import subprocess
import sys
from pathlib import Path

PKG = Path(__file__).resolve().parent
REPO = PKG.parent
CSRC = PKG / "csrc"
INCLUDE = REPO / "include"
LIB_NAME = "libmuon_polar_sm100.so"
OP_NAME = "_C.so"

NVCC_ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]


def _cuda_home() -> Path:
    home = os.environ.get("CUDA_HOME") or os.environ.get("CUDA_PATH")
    if home:
        return Path(home)
    nvcc = shutil.which("nvcc")
    if nvcc:
        return Path(nvcc).resolve().parent.parent
    return Path("/usr/local/cuda")


def _newer(target: Path, sources) -> bool:
    if not target.exists():
        return False
    t = target.stat().st_mtime
    return all(Path(s).stat().st_mtime <= t for s in sources)


def _run(cmd) -> None:
    print("+", " ".join(str(c) for c in cmd), flush=True)
    subprocess.run([str(c) for c in cmd], check=True, cwd=REPO)


def build_library(force: bool = False, verbose_ptxas: bool = False) -> Path:
    """nvcc -> libmuon_polar_sm100.so (kernels + C ABI)."""
    out = PKG / LIB_NAME
    cu = [CSRC / "muon_polar_sm100.cu", CSRC / "muon_update_sm100.cu"]
    sources = [*cu, CSRC / "sm100_ptx.cuh", INCLUDE / "muon_polar_sm100.h"]
    if not force and _newer(out, sources):
        return out
    nvcc = _cuda_home() / "bin" / "nvcc"
    cmd = [nvcc, *NVCC_ARCH, "-O3", "-std=c++17", "-lineinfo",
           "-Xcompiler", "-fPIC", "-shared", "-I", INCLUDE, *cu, "-o", out]
    if verbose_ptxas:
        cmd.insert(1, "-Xptxas=-v")
    _run(cmd)
    return out


def build_op(force: bool = False) -> Path:
    """g++ -> _C.so (torch operator), linked to the C ABI library."""
    import torch
    from torch.utils import cpp_extension

    lib = build_library(force=force)
    out = PKG / OP_NAME
    sources = [CSRC / "polar_step_op.cpp", INCLUDE / "muon_polar_sm100.h", lib]
    if not force and _newer(out, sources):
        return out
    cuda_home = _cuda_home()
    abi = int(torch._C._GLIBCXX_USE_CXX11_ABI)
    includes = cpp_extension.include_paths() + [str(cuda_home / "include"), str(INCLUDE)]
    torch_lib = Path(torch.__file__).resolve().parent / "lib"
    # The operator's inline ATen/c10 helpers call the CUDA runtime: bind them
    # to the same libcudart torch itself loads.
    cudart_dir = torch_lib.parent.parent / "nvidia" / "cuda_runtime" / "lib"
    if (cudart_dir / "libcudart.so.12").exists():
        cudart = [f"-L{cudart_dir}", "-l:libcudart.so.12", f"-Wl,-rpath,{cudart_dir}"]
    else:
        cudart = [f"-L{cuda_home / 'lib64'}", "-lcudart"]
    cmd = ["g++", "-O2", "-std=c++17", "-fPIC", "-shared",
           f"-D_GLIBCXX_USE_CXX11_ABI={abi}", "-DTORCH_EXTENSION_NAME=_C",
           *[f"-I{p}" for p in includes],
           CSRC / "polar_step_op.cpp", "-o", out,
           f"-L{torch_lib}", f"-L{PKG}",
           "-lc10", "-ltorch", "-ltorch_cpu", "-lc10_cuda", "-ltorch_cuda",
           "-lmuon_polar_sm100", *cudart,
           "-Wl,-rpath,$ORIGIN", f"-Wl,-rpath,{torch_lib}"]
    _run(cmd)
    return out


def build_all(force: bool = False) -> None:
    build_library(force=force)
    build_op(force=force)


if __name__ == "__main__":
    build_all(force="--force" in sys.argv)
