"""GPU parity of the transpose-free path for tall X (M > N).

The reference's wrapper runs a tall X as polar_step(X^T) transposed back
(muon_ascend950/ops.py:27-32 of the reference).  The library computes the same
step in X's own layout (muon_polar_{gram,apply,step}_t_sm100): A = X^T.X with
M-contiguous operand tiles, the unchanged polynomial, Y = a.X + X.P.  Each
stage is checked against the CPU oracle fed the same inputs, with the bounds
of the plain stages (tests/test_gpu_parity.py), and the whole step against
the reference's wrapper semantics (oracle.polar_step_oracle) and against the
copy-based path.
"""
from __future__ import annotations

import pytest
import torch

from oracle.polar_oracle import (
    COEFFICIENTS,
    error_stats,
    make_input,
    polar_step_oracle,
    reference_formula,
    ulp_bf16,
)

pytestmark = pytest.mark.gpu

A1, B1, C1 = COEFFICIENTS[0]
MODES = ["single", "single_split", "pair", "pair_split"]
_POLICY = {"single": 2, "pair": 1}


@pytest.fixture(scope="module")
def api(cuda_device):
    from muon_fusion_ascend950_b200.capi import capi

    return capi()


@pytest.fixture
def mode_policy(api):
    def set_mode(mode):
        api.set_kernel_policy(_POLICY[mode.split("_")[0]])
        split = mode.endswith("_split")
        api.set_split_mode(1 if split else 0)
        return split
    yield set_mode
    api.set_kernel_policy(0)
    api.set_split_mode(0)


def _rne(t64):
    return t64.to(torch.float32).to(torch.bfloat16).to(torch.float64)


def _gamma(k):
    return 2.0 * k * 2.0 ** -24


def _padded(x, device):
    """x [B, M, N] on `device` with a row stride that is a multiple of 16
    elements (the TMA stride rule), zero columns beyond N."""
    bsz, m, n = x.shape
    ld = (n + 15) // 16 * 16 if n % 8 else n
    xp = torch.zeros((bsz, m, ld), dtype=torch.bfloat16, device=device)
    xp[:, :, :n] = x.to(device)
    return xp


def _check_watchdog(api):
    assert api.read_device_status(torch.cuda.current_device()) == 0


@pytest.mark.parametrize("mode", MODES)
@pytest.mark.parametrize("shape", [(1, 130, 129), (2, 2050, 152), (8, 2048, 512),
                                   (1, 1000, 300), (3, 72, 64), (1, 8192, 256)])
def test_gram_t_stage(api, cuda_device, shape, mode, mode_policy):
    """A = rne(X^T X): within one ulp plus the fp32 summation slack of the
    exact product, exactly symmetric, zero beyond N; and (nearly always) the
    same bits as the plain Gram of the transposed copy."""
    split = mode_policy(mode)
    bsz, m, n = shape
    x = make_input(shape, seed=21)
    xd = _padded(x, cuda_device)
    npad = api.padded_rows(n)
    scratch = api.new_scratch(bsz, n, m) if split else None
    gram = torch.full((bsz, npad, npad), float("nan"), dtype=torch.bfloat16, device=cuda_device)
    api.gram_t(xd, gram, n=n, scratch=scratch)
    torch.cuda.synchronize()
    _check_watchdog(api)
    if split and scratch.numel() > 1:
        assert int(scratch[:1024].cpu().count_nonzero()) == 0
    g = gram.cpu()
    x64 = torch.zeros((bsz, m, npad), dtype=torch.float64)
    x64[:, :, :n] = x.to(torch.float64)
    exact = x64.mT @ x64
    slack = _gamma(m) * (x64.abs().mT @ x64.abs())
    diff = (g.to(torch.float64) - _rne(exact)).abs()
    bound = ulp_bf16(_rne(exact)) + slack + 1e-30
    assert bool((diff <= bound * (1 + 1e-9)).all()), f"gram_t {shape}: {float(diff.max())}"
    assert float((diff > 0).double().mean()) <= 0.02
    assert torch.equal(g.view(torch.int16), g.mT.contiguous().view(torch.int16))
    assert torch.equal(g[:, n:].float(), torch.zeros_like(g[:, n:].float()))
    # the plain kernel on X^T
    xt = _padded(x.mT.contiguous(), cuda_device)
    plain = torch.empty_like(gram)
    api.gram(xt, plain, n=m, scratch=scratch)
    torch.cuda.synchronize()
    same = (plain.cpu().view(torch.int16) == g.view(torch.int16)).double().mean()
    assert float(same) >= 0.98


@pytest.mark.parametrize("mode", ["single", "pair"])
@pytest.mark.parametrize("shape", [(1, 130, 129), (2, 2064, 150), (8, 2048, 512),
                                   (1, 1000, 200), (2, 520, 384)])
def test_apply_t_stage(api, cuda_device, shape, mode, mode_policy):
    """Y = rne(rne(X.P) + rne(alpha*X)) within the apply stage's bound."""
    mode_policy(mode)
    bsz, m, n = shape
    x = make_input(shape, seed=22)
    xd = _padded(x, cuda_device)
    npad = api.padded_rows(n)
    gram = torch.empty((bsz, npad, npad), dtype=torch.bfloat16, device=cuda_device)
    poly = torch.empty_like(gram)
    scratch = api.new_scratch(bsz, n, m)
    api.gram_t(xd, gram, n=n, scratch=scratch)
    api.poly(gram, poly, B1, C1, scratch=scratch)
    y = torch.full_like(xd, float("nan"))
    api.apply_t(poly, xd, y, A1, n=n)
    torch.cuda.synchronize()
    _check_watchdog(api)
    p64 = poly.cpu().to(torch.float64)[:, :n, :n]
    x64 = x.to(torch.float64)
    t = x64 @ p64
    alpha = torch.tensor(A1, dtype=torch.float32).to(torch.bfloat16).to(torch.float64)
    expected = _rne(_rne(t) + _rne(alpha * x64))
    got = y.cpu().to(torch.float64)[:, :, :n]
    diff = (got - expected).abs()
    bound = ulp_bf16(t) + ulp_bf16(expected) + _gamma(n) * (x64.abs() @ p64.abs())
    assert bool((diff <= bound).all()), f"apply_t {shape}: max diff {float(diff.max())}"
    assert float((diff > 0).double().mean()) <= 0.05
    if y.shape[-1] > n:
        # columns beyond N: untouched, except that the tile stores complete
        # the 16-byte unit holding column N-1 with zeros
        pad = y[:, :, n:].float().cpu()
        assert bool((torch.isnan(pad) | (pad == 0)).all())
        assert bool(torch.isnan(pad[:, :, (8 - n % 8) % 8:]).all())


@pytest.mark.parametrize("shape", [(130, 129), (1, 130, 129), (2, 2050, 150),
                                   (8, 2048, 512), (4, 1000, 300), (1, 4096, 1024)])
def test_step_tall_matches_oracle(cuda_device, shape):
    """polar_step on tall X (transpose-free by default) against the
    reference's wrapper semantics and the fp32 formula, with the reference
    test tolerance, and against the reference's copy policy."""
    import muon_fusion_ascend950_b200 as pkg

    x = make_input(shape, seed=23)
    xd = x.to(cuda_device)
    y = pkg.polar_step(xd, A1, B1, C1)
    y_copy = pkg.polar_step(xd, A1, B1, C1, transpose_copies=True)
    torch.cuda.synchronize()
    y, y_copy = y.cpu(), y_copy.cpu()
    assert y.shape == x.shape and y.dtype == torch.bfloat16
    ref16 = reference_formula(x, COEFFICIENTS[:1])
    torch.testing.assert_close(y.float(), ref16.float(), rtol=6e-2, atol=6e-2)
    y32 = reference_formula(x.float(), COEFFICIENTS[:1])
    e = error_stats(y, y32)
    e_or = error_stats(polar_step_oracle(x, A1, B1, C1), y32)
    assert e["max_abs"] <= 2.0 * e_or["max_abs"] + 1e-6, (e, e_or)
    assert e["rel_fro"] <= 1e-2, e
    d = error_stats(y, y_copy)
    assert d["rel_fro"] <= 2e-3, d


def test_step_tall_five_steps(cuda_device):
    import muon_fusion_ascend950_b200 as pkg

    x = make_input((2, 1536, 384), seed=24)
    y = x.to(cuda_device)
    for a, b, c in COEFFICIENTS:
        y = pkg.polar_step(y, a, b, c)
    y = y.cpu()
    torch.testing.assert_close(y.float(), reference_formula(x, COEFFICIENTS).float(),
                               rtol=6e-2, atol=6e-2)
    assert error_stats(y, reference_formula(x.float(), COEFFICIENTS))["rel_fro"] <= 5e-2


def test_step_t_capi_equals_op(api, cuda_device):
    """The C-ABI step and the torch operator give the same bits."""
    import muon_fusion_ascend950_b200 as pkg

    x = make_input((3, 768, 256), seed=25).to(cuda_device)
    ws = torch.empty(api.workspace_bytes(3, 256), dtype=torch.uint8, device=cuda_device)
    y = torch.empty_like(x)
    api.step_t(x, y, ws, A1, B1, C1, scratch=api.new_scratch(3, 256, 768))
    y_op = pkg.polar_step(x, A1, B1, C1)
    torch.cuda.synchronize()
    _check_watchdog(api)
    assert torch.equal(y.view(torch.int16), y_op.view(torch.int16))
