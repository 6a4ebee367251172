"""CPU oracle for the Polar Express step -- TEST INFRASTRUCTURE ONLY.

This module is the checker, never the thing measured or shipped.  Only
``tests/``, ``__graft_entry__.smoke()`` and ``bench.py``'s CPU-baseline /
``--impl reference`` arm may import it.  The product path
(``muon_fusion_ascend950_b200``) never imports it and has no CPU fallback.

It restates, on the CPU with PyTorch, two things from the reference
(Lucien-Nova/Muon_fusion_Ascend950; paths relative to that project):

1. ``reference_formula`` -- the reference's own accuracy oracle,
   ``_reference`` at tests/test_polar_step.py:22-28 (also README.md:172-174):
   ``gram = out @ out.mT; P = b*gram + c*(gram @ gram); out = a*out + P @ out``
   evaluated in the dtype of its input (bf16 in the reference test, fp32 for
   an accuracy reference).

2. ``kernel_dataflow`` -- the numerics of the reference's three device
   kernels, as written in csrc/muon_polar_unified_ascend950.asc:
     * padding: rows = align(M,128), cols = max(align(N,16), rows), zero
       fill (csrc/muon_polar_step_binding.cpp:626-640);
     * Cube1: A = RINT_bf16(X.X^T accumulated in fp32) (asc:406-409);
     * Cube2+P: P = RINT_bf16( fl32(b*f32(A)) + fl32(c*A2) ), A2 = A.A^T in
       fp32, separate multiplies and add (asc:929-940), b and c as fp32
       (binding.cpp:348-349);
     * Cube3+Y: Y = bf16( RINT_bf16(T) + bf16(alpha_bf16 * X) ), T = P.X in
       fp32, alpha rounded to bf16 on the host (asc:1454-1476,
       binding.cpp:156-162, 470);
     * crop back to [B, M, N] (binding.cpp:667-672);
   plus the Python wrapper's transpose policy for M > N
   (muon_ascend950/ops.py:24-33).

Pinning: ``reference_formula`` is checked against golden vectors produced by
running the reference's own ``_reference`` function (extracted from
tests/test_polar_step.py by tests/golden/make_golden.py) on seeded inputs in
this repository's build container; the fixtures are tests/golden/*.npz.  The
reference's device kernels need an Ascend NPU and CANN 9.0.0 and cannot run
anywhere here, so ``kernel_dataflow`` is pinned to the reference formula only
within the reference test tolerance (rtol = atol = 6e-2) and the tighter
bounds stated in the tests.
"""
from __future__ import annotations

from typing import Iterable, Sequence, Tuple

import torch

# Polar Express coefficients, in order (tests/test_polar_step.py:12-18,
# examples/five_steps.py:7-13).
COEFFICIENTS: Tuple[Tuple[float, float, float], ...] = (
    (8.156554524902461, -22.48329292557795, 15.878769915207462),
    (4.042929935166739, -2.808917465908714, 0.5000178451051316),
    (3.8916678022926607, -2.772484153217685, 0.5060648178503393),
    (3.285753657755655, -2.3681294933425376, 0.46449024233003106),
    (2.3465413258596377, -1.7097828382687081, 0.42323551169305323),
)

TILE = 128


def align_up(value: int, alignment: int) -> int:
    """AlignUp of csrc/muon_polar_step_binding.cpp:88-91."""
    return (value + alignment - 1) // alignment * alignment


def padded_shape(m: int, n: int) -> Tuple[int, int]:
    """(rows, cols) of the reference's padded work tensor
    (csrc/muon_polar_step_binding.cpp:630-631)."""
    rows = align_up(m, 128)
    cols = max(align_up(n, 16), rows)
    return rows, cols


def upper_tiles(dim: int) -> list:
    """Upper-triangle tile set {(tm, tn): tm <= tn < dim} in the row-major
    order the B200 kernels walk it.  The reference enumerates the same set of
    128x128 tiles (csrc/muon_polar_unified_ascend950.asc:129-146 for the Gram,
    609-630 for Cube2 column jobs); only the visiting order differs."""
    return [(tm, tn) for tm in range(dim) for tn in range(tm, dim)]


def make_input(shape: Sequence[int], seed: int = 0) -> torch.Tensor:
    """Seeded bf16 input normalised per matrix as the reference test does
    (tests/test_polar_step.py:38-39): N(0,1) entries, then
    x / (||x||_F * 1.01 + 1e-6) evaluated in bf16."""
    gen = torch.Generator().manual_seed(seed)
    x = torch.randn(tuple(shape), generator=gen, dtype=torch.float32)
    x = x.to(torch.bfloat16)
    return x / (x.norm(dim=(-2, -1), keepdim=True) * 1.01 + 1e-6)


def reference_formula(x: torch.Tensor, coefficients: Iterable) -> torch.Tensor:
    """tests/test_polar_step.py:22-28, evaluated in x's dtype."""
    out = x
    for a, b, c in coefficients:
        gram = out @ out.mT
        polynomial = b * gram + c * (gram @ gram)
        out = a * out + polynomial @ out
    return out


def _rne_bf16(t: torch.Tensor) -> torch.Tensor:
    """fp32 -> bf16 round-to-nearest-even (RINT), back as fp32 values."""
    return t.to(torch.bfloat16).to(torch.float32)


def kernel_dataflow_3d(x: torch.Tensor, a: float, b: float, c: float) -> torch.Tensor:
    """One step through the reference op for x[B, M, N] with M <= N
    (csrc/muon_polar_step_binding.cpp:613-673), bf16 in, bf16 out."""
    assert x.dim() == 3 and x.shape[1] <= x.shape[2]
    bsz, m, n = x.shape
    rows, cols = padded_shape(m, n)
    xp = torch.zeros((bsz, rows, cols), dtype=torch.float32)
    xp[:, :m, :n] = x.to(torch.float32)
    f32 = torch.float32
    b32 = torch.tensor(b, dtype=f32)
    c32 = torch.tensor(c, dtype=f32)
    alpha = torch.tensor(a, dtype=f32).to(torch.bfloat16).to(f32)
    gram = _rne_bf16(xp @ xp.mT)                          # Cube1, bf16 storage
    a2 = gram @ gram.mT                                   # Cube2 fp32 acc
    poly = _rne_bf16((b32 * gram) + (c32 * a2))           # separate mul/add
    t = poly @ xp                                         # Cube3 fp32 acc
    ax = _rne_bf16(alpha * xp)                            # bf16 Muls
    y = (_rne_bf16(t) + ax).to(torch.bfloat16)            # bf16 Add
    return y[:, :m, :n].contiguous()


def polar_step_oracle(x: torch.Tensor, a: float, b: float, c: float) -> torch.Tensor:
    """Wrapper semantics of muon_ascend950/ops.py:24-33 around
    kernel_dataflow_3d: 2-D input is unsqueezed, M > N is transposed in and
    out."""
    squeeze = x.dim() == 2
    work = x.unsqueeze(0) if squeeze else x
    transposed = work.size(-2) > work.size(-1)
    if transposed:
        work = work.mT.contiguous()
    out = kernel_dataflow_3d(work, a, b, c)
    if transposed:
        out = out.mT.contiguous()
    return out.squeeze(0) if squeeze else out


class CpuKernels:
    """CPU stand-in for the C-ABI kernel entry points (the methods of
    muon_fusion_ascend950_b200.capi.CAPI used by the multi-GPU drivers), for
    the gloo tests of those drivers.  Same buffer shapes and the same
    arithmetic as kernels 1-3 of the reference (fp32 Gram, round-to-nearest
    bf16, separate multiply/add in the polynomial, bf16 add in the apply)."""

    @staticmethod
    def padded_rows(m: int) -> int:
        return align_up(m, 256)

    @staticmethod
    def gram_f32(x, out, n=None, scratch=None, stream=None):
        m = x.shape[1]
        xf = x.to(torch.float32)
        out.zero_()
        out[:, :m, :m] = xf @ xf.mT

    @staticmethod
    def gram_f32_band(x, out, row_begin, row_count, sm_reserve=0, n=None, scratch=None,
                      stream=None):
        """Rows [row_begin, row_begin + row_count) of the upper triangle
        (columns >= row_begin) and their mirror, as the banded kernel 1."""
        m = x.shape[1]
        xf = x.to(torch.float32)
        mp = out.shape[-1]
        r1 = row_begin + row_count
        full = torch.zeros((x.shape[0], mp, mp), dtype=torch.float32)
        full[:, :m, :m] = xf @ xf.mT
        out[:, row_begin:r1, row_begin:] = full[:, row_begin:r1, row_begin:]
        out[:, row_begin:, row_begin:r1] = full[:, row_begin:, row_begin:r1]

    @staticmethod
    def cast_f32_bf16(src, dst, stream=None):
        dst.copy_(src.to(torch.bfloat16))

    @staticmethod
    def poly(gram, poly, b, c, scratch=None, stream=None):
        a32 = gram.to(torch.float32)
        b32 = torch.tensor(b, dtype=torch.float32)
        c32 = torch.tensor(c, dtype=torch.float32)
        poly.copy_(((b32 * a32) + (c32 * (a32 @ a32.mT))).to(torch.bfloat16))

    @staticmethod
    def poly_rows(gram, poly, b, c, row_begin, row_count, stream=None):
        a32 = gram.to(torch.float32)
        rows = slice(row_begin, row_begin + row_count)
        b32 = torch.tensor(b, dtype=torch.float32)
        c32 = torch.tensor(c, dtype=torch.float32)
        poly[:, rows].copy_(((b32 * a32[:, rows]) + (c32 * (a32[:, rows] @ a32.mT)))
                            .to(torch.bfloat16))

    # Packed upper-triangle units ([B, units, 256, 256]), as the packed
    # entry points of the C ABI lay them out.
    @staticmethod
    def packed_units(m: int) -> int:
        d = align_up(m, 256) // 256
        return d * (d + 1) // 2

    @staticmethod
    def unit_grid(mp: int) -> list:
        d = mp // 256
        return [(i, j) for i in range(d) for j in range(i, d)]

    @classmethod
    def gram_f32_packed(cls, x, out, n=None, scratch=None, stream=None):
        m = x.shape[1]
        mp = align_up(m, 256)
        full = torch.zeros((x.shape[0], mp, mp), dtype=torch.float32)
        xf = x.to(torch.float32)
        full[:, :m, :m] = xf @ xf.mT
        for u, (i, j) in enumerate(cls.unit_grid(mp)):
            out[:, u] = full[:, 256 * i:256 * i + 256, 256 * j:256 * j + 256]

    @classmethod
    def poly_packed(cls, gram, out, b, c, unit_begin, unit_count, stream=None):
        a32 = gram.to(torch.float32)
        b32 = torch.tensor(b, dtype=torch.float32)
        c32 = torch.tensor(c, dtype=torch.float32)
        grid = cls.unit_grid(gram.shape[-1])
        for u in range(unit_begin, unit_begin + unit_count):
            i, j = grid[u]
            rows, cols = slice(256 * i, 256 * i + 256), slice(256 * j, 256 * j + 256)
            out[:, u] = ((b32 * a32[:, rows, cols]) + (c32 * (a32[:, rows] @ a32[:, cols].mT))
                         ).to(torch.bfloat16)

    @classmethod
    def unpack_sym(cls, packed, full, stream=None):
        for u, (i, j) in enumerate(cls.unit_grid(full.shape[-1])):
            rows, cols = slice(256 * i, 256 * i + 256), slice(256 * j, 256 * j + 256)
            blk = packed[:, u].clone()
            if i == j:  # the lower-left quarter mirrors the upper-right one
                blk[:, 128:, :128] = blk[:, :128, 128:].mT
                full[:, rows, cols] = blk
            else:
                full[:, rows, cols] = blk
                full[:, cols, rows] = blk.mT

    @staticmethod
    def apply(poly, x, y, a, n=None, stream=None):
        m = x.shape[1]
        t = poly.to(torch.float32)[:, :m, :m] @ x.to(torch.float32)
        alpha = torch.tensor(a, dtype=torch.float32).to(torch.bfloat16).to(torch.float32)
        y.copy_((_rne_bf16(t) + _rne_bf16(alpha * x.to(torch.float32))).to(torch.bfloat16))


def nominal_flops(m: int, n: int) -> int:
    """Nominal FLOPs of one step on one matrix (M <= N): 4 M^2 N + 2 M^3."""
    m, n = min(m, n), max(m, n)
    return 4 * m * m * n + 2 * m ** 3


def error_stats(actual: torch.Tensor, expected: torch.Tensor) -> dict:
    """max / mean absolute error and relative Frobenius error in fp64."""
    a = actual.to(torch.float64)
    e = expected.to(torch.float64)
    d = (a - e).abs()
    denom = float(e.norm())
    return {
        "max_abs": float(d.max()) if d.numel() else 0.0,
        "mean_abs": float(d.mean()) if d.numel() else 0.0,
        "rel_fro": float((a - e).norm()) / denom if denom > 0 else float((a - e).norm()),
        "max_ref": float(e.abs().max()) if e.numel() else 0.0,
    }


def ulp_bf16(t: torch.Tensor) -> torch.Tensor:
    """Spacing of bf16 numbers at |t| (fp64), 2^(floor(log2|t|) - 7); the
    spacing of the smallest normal for zeros."""
    a = t.to(torch.float64).abs().clamp_min(2.0 ** -126)
    return torch.pow(2.0, torch.floor(torch.log2(a)) - 7)


def bf16_bits(t: torch.Tensor) -> torch.Tensor:
    """bf16 tensor -> its int16 bit patterns (for exact comparisons)."""
    return t.contiguous().view(torch.int16)


__all__ = [
    "COEFFICIENTS",
    "TILE",
    "align_up",
    "padded_shape",
    "upper_tiles",
    "make_input",
    "reference_formula",
    "kernel_dataflow_3d",
    "polar_step_oracle",
    "normalize_oracle",
    "polar_express_oracle",
    "muon_update_oracle",
    "nominal_flops",
    "CpuKernels",
    "error_stats",
    "ulp_bf16",
    "bf16_bits",
]


# ------------------------------------------------------------------ caller side
# The reference leaves the loop, the normalisation and the optimizer update to
# its caller (README.md:5, 130).  Its example caller normalises with
# x / (||x||_F * 1.01 + 1e-6) and runs one polar_step per coefficient row
# (examples/five_steps.py:18-21).  These restate that caller, plus the usual
# Muon momentum / weight-decay / scaled update, in fp32 torch on the CPU:
# the checker of muon_polar_express_sm100 and muon_polar_update_sm100.

def normalize_oracle(v: torch.Tensor) -> torch.Tensor:
    """bf16( v / (||v||_F * 1.01 + 1e-6) ) per matrix, fp32 arithmetic."""
    v32 = v.to(torch.float32)
    norm = torch.linalg.vector_norm(v32.to(torch.float64), dim=(-2, -1), keepdim=True)
    s = (norm.to(torch.float32) * 1.01) + 1e-6
    return (v32 / s).to(torch.bfloat16)


def polar_express_oracle(x: torch.Tensor, coefficients, normalize: bool = True) -> torch.Tensor:
    """examples/five_steps.py:18-21: normalise, then one step per row."""
    y = normalize_oracle(x) if normalize else x.to(torch.bfloat16)
    for a, b, c in coefficients:
        y = polar_step_oracle(y, a, b, c)
    return y


def muon_update_oracle(param, grad, buf, lr, momentum, nesterov, weight_decay, scale,
                       coefficients):
    """One Muon update in the tensors' own dtype (torch.lerp semantics), the
    orthogonalisation through polar_express_oracle; returns (param, buf)."""
    buf = buf.clone().lerp_(grad, 1.0 - momentum)
    v = grad.lerp(buf, momentum) if nesterov else buf
    y = polar_express_oracle(v, coefficients, normalize=True).to(torch.float32)
    p = param.to(torch.float32) * (1.0 - lr * weight_decay) - (lr * scale) * y
    return p.to(param.dtype), buf
