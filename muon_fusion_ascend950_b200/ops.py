"""Python entry point of the Polar Express step.

Same contract as muon_ascend950/ops.py:6-33 of the reference, with CUDA in
place of the NPU: argument checks with the same exception types and texts,
and 2-D input unsqueezed to a batch of one.  For M > N the reference
transposes around the native operator (two transposed copies); here the
operator ``polar_step_t`` computes the step of X^T directly in X's layout
(the same result, no copies).  ``transpose_copies=True`` restores the
reference's copy policy.
"""
from __future__ import annotations

import torch


def polar_step(x: torch.Tensor, a: float, b: float, c: float, *,
               transpose_copies: bool = False) -> torch.Tensor:
    """Run one Polar Express iteration and return a tensor with the same shape.

    ``x`` must be a BF16 CUDA tensor with shape ``[M,N]`` or ``[B,M,N]``.
    ``M > N`` runs the step of ``x^T`` in ``x``'s own layout (operator
    ``polar_step_t``), or, with ``transpose_copies=True``, by transposing
    around the native operator as the reference does.
    Non-aligned dimensions are handled inside the C++ operator.
    """
    if not isinstance(x, torch.Tensor):
        raise TypeError("x must be a torch.Tensor")
    if x.device.type != "cuda":
        raise ValueError(f"x must be on a CUDA device, got {x.device}")
    if x.dtype != torch.bfloat16:
        raise TypeError(f"x must use torch.bfloat16, got {x.dtype}")
    if x.ndim not in (2, 3):
        raise ValueError(f"x must have shape [M,N] or [B,M,N], got {tuple(x.shape)}")
    if any(size <= 0 for size in x.shape):
        raise ValueError("all input dimensions must be positive")

    squeeze_batch = x.ndim == 2
    work = x.unsqueeze(0) if squeeze_batch else x
    tall = work.size(-2) > work.size(-1)
    if tall and not transpose_copies:
        out = torch.ops.muon_ascend950.polar_step_t(work, float(a), float(b), float(c))
        return out.squeeze(0) if squeeze_batch else out
    if tall:
        work = work.mT.contiguous()

    out = torch.ops.muon_ascend950.polar_step(work, float(a), float(b), float(c))
    if tall:
        out = out.mT.contiguous()
    return out.squeeze(0) if squeeze_batch else out
