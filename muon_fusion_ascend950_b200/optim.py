"""Muon optimizer on the B200 kernels: the caller side of the reference's
operator, fused on the device.

The reference ships only the orthogonalisation step and leaves "the
five-step loop, input normalisation and the optimizer's momentum, weight
decay and parameter update" to its caller (README.md:5, 130).  ``Muon`` is
that caller: for every matrix parameter one native call
(``torch.ops.muon_ascend950.muon_update_``, C ABI ``muon_polar_update_sm100``)
runs

    buf <- lerp(buf, grad, 1 - momentum)              (momentum buffer)
    v    = nesterov ? lerp(grad, buf, momentum) : buf
    X    = bf16( v / (||v||_F * 1.01 + 1e-6) )         (examples/five_steps.py:18)
    Y    = Polar Express steps of X                     (one polar_step per row)
    p   <- p * (1 - lr * weight_decay) - lr * scale * Y

with ``scale = max(1, rows / cols) ** 0.5`` by default.  Parameters must be
matrices (``[M, N]``) or batches of matrices (``[B, M, N]``) in fp32 or bf16;
vectors and scalars belong to another optimizer (e.g. AdamW), as usual for
Muon.
"""
from __future__ import annotations

from typing import Iterable, Optional

import torch

from .ops import POLAR_EXPRESS_COEFFICIENTS, _flat_coefficients


def default_scale(rows: int, cols: int) -> float:
    return max(1.0, rows / cols) ** 0.5


class Muon(torch.optim.Optimizer):
    """Momentum + Polar Express orthogonalisation + scaled update, one fused
    native call per parameter on its CUDA stream."""

    def __init__(self, params: Iterable, lr: float = 0.02, momentum: float = 0.95,
                 nesterov: bool = True, weight_decay: float = 0.0,
                 coefficients=POLAR_EXPRESS_COEFFICIENTS, scale: Optional[float] = None):
        if lr < 0.0:
            raise ValueError(f"invalid learning rate {lr}")
        if not 0.0 <= momentum < 1.0:
            raise ValueError(f"invalid momentum {momentum}")
        if weight_decay < 0.0:
            raise ValueError(f"invalid weight_decay {weight_decay}")
        defaults = dict(lr=lr, momentum=momentum, nesterov=nesterov, weight_decay=weight_decay,
                        coefficients=tuple(tuple(float(v) for v in row) for row in coefficients),
                        scale=scale)
        _flat_coefficients(defaults["coefficients"])
        super().__init__(params, defaults)

    @torch.no_grad()
    def step(self, closure=None):
        loss = None
        if closure is not None:
            with torch.enable_grad():
                loss = closure()
        for group in self.param_groups:
            flat = _flat_coefficients(group["coefficients"])
            for p in group["params"]:
                if p.grad is None:
                    continue
                if p.ndim not in (2, 3):
                    raise ValueError("Muon updates matrices ([M,N] or [B,M,N]) only; "
                                     f"got a parameter of shape {tuple(p.shape)}")
                if p.device.type != "cuda" or p.dtype not in (torch.float32, torch.bfloat16):
                    raise TypeError("Muon parameters must be fp32 or bf16 CUDA tensors")
                if not p.is_contiguous():
                    raise ValueError("Muon parameters must be contiguous")
                grad = p.grad
                if grad.dtype != p.dtype or not grad.is_contiguous():
                    grad = grad.to(dtype=p.dtype, memory_format=torch.contiguous_format)
                state = self.state[p]
                if "momentum_buffer" not in state:
                    state["momentum_buffer"] = torch.zeros_like(
                        p, memory_format=torch.contiguous_format)
                rows, cols = p.shape[-2], p.shape[-1]
                scale = group["scale"] if group["scale"] is not None else default_scale(rows, cols)
                torch.ops.muon_ascend950.muon_update_(
                    p, grad, state["momentum_buffer"], float(group["lr"]),
                    float(group["momentum"]), bool(group["nesterov"]),
                    float(group["weight_decay"]), float(scale), flat)
        return loss
