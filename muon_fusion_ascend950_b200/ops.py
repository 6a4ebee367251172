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


# The five Polar Express coefficient rows (a, b, c) of the reference's
# example loop (examples/five_steps.py:7-13): the same table, since the
# steps must reproduce the reference's iteration.
POLAR_EXPRESS_COEFFICIENTS = (
    (8.156554524902461, -22.48329292557795, 15.878769915207462),
    (4.042929935166739, -2.808917465908714, 0.5000178451051316),
    (3.8916678022926607, -2.772484153217685, 0.5060648178503393),
    (3.285753657755655, -2.3681294933425376, 0.46449024233003106),
    (2.3465413258596377, -1.7097828382687081, 0.42323551169305323),
)


def _flat_coefficients(coefficients) -> list:
    rows = [tuple(float(v) for v in row) for row in coefficients]
    if not rows or any(len(row) != 3 for row in rows):
        raise ValueError("coefficients must be a non-empty sequence of (a, b, c) rows")
    return [v for row in rows for v in row]


def polar_express(x: torch.Tensor, coefficients=POLAR_EXPRESS_COEFFICIENTS, *,
                  normalize: bool = True) -> torch.Tensor:
    """Several Polar Express steps in one native call: the reference example's
    loop (examples/five_steps.py:18-21) -- ``x / (||x||_F * 1.01 + 1e-6)`` per
    matrix, then ``polar_step`` once per coefficient row -- with the
    normalisation fused into one device pass and no host round trip.

    ``x``: CUDA ``[M,N]`` or ``[B,M,N]``, bf16 (or fp32 when ``normalize``).
    Returns bf16 of the same shape.  Tall ``x`` runs transpose-free.
    """
    if not isinstance(x, torch.Tensor):
        raise TypeError("x must be a torch.Tensor")
    if x.device.type != "cuda":
        raise ValueError(f"x must be on a CUDA device, got {x.device}")
    if x.dtype not in (torch.bfloat16, torch.float32) or (
            x.dtype == torch.float32 and not normalize):
        raise TypeError(f"x must use torch.bfloat16 (or float32 with normalize=True), got {x.dtype}")
    if x.ndim not in (2, 3):
        raise ValueError(f"x must have shape [M,N] or [B,M,N], got {tuple(x.shape)}")
    if any(size <= 0 for size in x.shape):
        raise ValueError("all input dimensions must be positive")
    flat = _flat_coefficients(coefficients)
    squeeze_batch = x.ndim == 2
    work = x.unsqueeze(0) if squeeze_batch else x
    out = torch.ops.muon_ascend950.polar_express(work, flat, bool(normalize))
    return out.squeeze(0) if squeeze_batch else out
