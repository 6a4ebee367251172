"""GPU tests of the caller side of the step: the multi-step entry
(muon_polar_express_sm100 / polar_express) and the fused Muon update
(muon_polar_update_sm100 / muon_update_ / optim.Muon), against the CPU
oracle's restatement of the reference's example caller
(examples/five_steps.py:18-21) and against compositions of this library's
own verified pieces.
"""
from __future__ import annotations

import pytest
import torch

from oracle.polar_oracle import (
    COEFFICIENTS,
    error_stats,
    make_input,
    muon_update_oracle,
    normalize_oracle,
    polar_express_oracle,
)

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def pkg(cuda_device):
    import muon_fusion_ascend950_b200 as pkg

    return pkg


@pytest.fixture(scope="module")
def api(cuda_device):
    from muon_fusion_ascend950_b200.capi import capi

    return capi()


def _watchdog_clear(api):
    assert api.read_device_status(torch.cuda.current_device()) == 0


@pytest.mark.parametrize("shape", [(8, 512, 2048), (1, 129, 130), (2, 150, 2050), (3, 640, 256)])
def test_polar_express_without_normalisation_equals_step_chain(pkg, api, cuda_device, shape):
    """Five steps in one call give the bits of five polar_step calls."""
    x = make_input(shape, seed=31).to(cuda_device)
    y = pkg.polar_express(x, COEFFICIENTS, normalize=False)
    ref = x
    for a, b, c in COEFFICIENTS:
        ref = pkg.polar_step(ref, a, b, c)
    torch.cuda.synchronize()
    _watchdog_clear(api)
    assert y.shape == x.shape and y.dtype == torch.bfloat16
    assert torch.equal(y.view(torch.int16), ref.view(torch.int16))


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float32])
@pytest.mark.parametrize("shape", [(8, 512, 2048), (2, 150, 2050), (2, 1000, 300), (129, 130)])
def test_polar_express_with_normalisation(pkg, api, cuda_device, shape, dtype):
    """Normalisation + five steps against the oracle of the reference's
    example loop (reference test tolerance), and against this library's
    step chain fed the oracle's normalised input."""
    g = torch.Generator().manual_seed(32)
    x = torch.randn(shape, generator=g).to(dtype)
    y = pkg.polar_express(x.to(cuda_device), COEFFICIENTS, normalize=True).cpu()
    _watchdog_clear(api)
    ref = polar_express_oracle(x, COEFFICIENTS, normalize=True)
    torch.testing.assert_close(y.float(), ref.float(), rtol=6e-2, atol=6e-2)
    x0 = normalize_oracle(x)
    chain = x0.to(cuda_device)
    for a, b, c in COEFFICIENTS:
        chain = pkg.polar_step(chain, a, b, c)
    e = error_stats(y, chain.cpu())
    assert e["rel_fro"] <= 2e-2, e


def test_polar_express_capi_workspace_and_errors(api, cuda_device):
    x = make_input((2, 256, 512), seed=33).to(cuda_device)
    y = torch.empty_like(x)
    ws = torch.empty(api.express_workspace_bytes(2, 256, 512), dtype=torch.uint8,
                     device=cuda_device)
    api.polar_express(x, y, ws, COEFFICIENTS, normalize=False)
    torch.cuda.synchronize()
    from muon_fusion_ascend950_b200.capi import MuonPolarError
    with pytest.raises(MuonPolarError):
        api.polar_express(x, y, ws[:-256], COEFFICIENTS, normalize=False)
    with pytest.raises(MuonPolarError):  # fp32 input without normalisation
        api.polar_express(x.float(), y, ws, COEFFICIENTS, normalize=False)


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
@pytest.mark.parametrize("nesterov", [True, False])
@pytest.mark.parametrize("shape", [(4, 512, 1024), (1, 300, 200), (2, 256, 2056)])
def test_muon_update_matches_oracle(pkg, api, cuda_device, shape, dtype, nesterov):
    g = torch.Generator().manual_seed(34)
    # small weights and a large step keep bf16 rounding of p well below the
    # step itself
    p0 = (torch.randn(shape, generator=g) * 0.01).to(dtype)
    grad = torch.randn(shape, generator=g).to(dtype)
    buf0 = (torch.randn(shape, generator=g) * 0.5).to(dtype)
    lr, mu, wd = 0.1, 0.95, 0.01
    scale = max(1.0, shape[-2] / shape[-1]) ** 0.5
    p = p0.to(cuda_device)
    buf = buf0.to(cuda_device)
    torch.ops.muon_ascend950.muon_update_(p, grad.to(cuda_device), buf, lr, mu, nesterov, wd,
                                          scale, [v for row in COEFFICIENTS for v in row])
    torch.cuda.synchronize()
    _watchdog_clear(api)
    p_ref, buf_ref = muon_update_oracle(p0, grad, buf0, lr, mu, nesterov, wd, scale, COEFFICIENTS)
    # momentum buffer: torch.lerp's formula, one rounding
    tol = 1e-6 if dtype == torch.float32 else 8e-3
    torch.testing.assert_close(buf.cpu().float(), buf_ref.float(), rtol=tol, atol=tol)
    # parameter step: the orthogonalised direction agrees with the oracle's
    d_gpu = (p.cpu().double() - p0.double() * (1 - lr * wd))
    d_ref = (p_ref.double() - p0.double() * (1 - lr * wd))
    rel = float((d_gpu - d_ref).norm() / d_ref.norm())
    assert rel <= (0.1 if dtype == torch.float32 else 0.2), rel


def test_muon_update_equals_its_pieces(pkg, api, cuda_device):
    """With momentum 0 and no Nesterov the update direction is the
    normalised gradient: the fused call equals polar_express + the update
    formula computed with torch on the same device (fp32 parameters)."""
    shape = (2, 384, 1024)
    g = torch.Generator().manual_seed(35)
    p0 = torch.randn(shape, generator=g).to(cuda_device) * 0.05
    grad = torch.randn(shape, generator=g).to(cuda_device)
    lr, wd, scale = 0.05, 0.1, 1.0
    p = p0.clone()
    buf = torch.zeros_like(p)
    torch.ops.muon_ascend950.muon_update_(p, grad, buf, lr, 0.0, False, wd, scale,
                                          [v for row in COEFFICIENTS for v in row])
    y = pkg.polar_express(grad, COEFFICIENTS, normalize=True).float()
    expect = p0 * (1 - lr * wd) - (lr * scale) * y
    torch.cuda.synchronize()
    _watchdog_clear(api)
    assert torch.equal(buf, grad)
    assert float((p - expect).abs().max()) <= 1e-6


def test_muon_optimizer_step_and_descent(pkg, api, cuda_device):
    """Muon.step equals the direct native call, and a few steps reduce a
    least-squares loss."""
    torch.manual_seed(36)
    w = torch.nn.Parameter(torch.randn(256, 512, device=cuda_device) * 0.02)
    w_copy = w.detach().clone()
    buf = torch.zeros_like(w_copy)
    inputs = torch.randn(512, 1024, device=cuda_device)
    target = torch.randn(256, 1024, device=cuda_device) * 0.1
    opt = pkg.Muon([w], lr=0.02, momentum=0.9, nesterov=True, weight_decay=0.0)
    losses = []
    for i in range(6):
        opt.zero_grad()
        loss = ((w @ inputs - target) ** 2).mean()
        loss.backward()
        if i == 0:
            torch.ops.muon_ascend950.muon_update_(w_copy, w.grad.clone(), buf, 0.02, 0.9, True,
                                                  0.0, 1.0,
                                                  [v for row in COEFFICIENTS for v in row])
        opt.step()
        if i == 0:
            assert torch.equal(w.detach(), w_copy)
        losses.append(float(loss.detach()))
    torch.cuda.synchronize()
    _watchdog_clear(api)
    assert losses[-1] < losses[0]


def test_muon_tall_and_batched_parameters(pkg, api, cuda_device):
    """Tall matrices run the transposed step; 3-D parameters are batches."""
    torch.manual_seed(37)
    tall = torch.nn.Parameter(torch.randn(1024, 256, device=cuda_device) * 0.02)
    batched = torch.nn.Parameter(torch.randn(3, 128, 384, device=cuda_device,
                                             dtype=torch.bfloat16) * 0.02)
    opt = pkg.Muon([tall, batched], lr=0.01)
    t0, b0 = tall.detach().clone(), batched.detach().clone()
    tall.grad = torch.randn_like(tall)
    batched.grad = torch.randn_like(batched)
    g_tall = tall.grad.clone()
    opt.step()
    torch.cuda.synchronize()
    _watchdog_clear(api)
    # first step from a zero buffer with Nesterov: v = lerp(g, (1-mu) g, mu)
    mu = 0.95
    v = g_tall.lerp(g_tall * (1 - mu), mu)
    y = polar_express_oracle(v.cpu(), COEFFICIENTS)
    d = (tall.detach() - t0).cpu() / (-0.01 * 2.0)  # scale = sqrt(1024 / 256)
    assert error_stats(d.to(torch.bfloat16), y)["rel_fro"] <= 0.05
    assert not torch.equal(batched.detach(), b0)


def _steps_fused_vs_chain(api, x, coeffs, mode):
    """muon_polar_steps_sm100 in step mode `mode`, split-K off (the fused
    kernel never splits K; a split changes the fp32 summation order) ->
    (y, counters after)."""
    bsz, m, n = x.shape
    ws = torch.empty(api.workspace_bytes(bsz, m), dtype=torch.uint8, device=x.device)
    scratch = torch.zeros(api.scratch_bytes(bsz, m, n), dtype=torch.uint8, device=x.device)
    y = torch.full_like(x, float("nan"))
    bufs = [torch.full_like(x, float("nan")) for _ in range(2)]
    prev = api.lib.muon_polar_set_step_mode(mode)
    prev_split = api.lib.muon_polar_set_split_mode(2)
    try:
        api.steps(x, y, bufs[0], bufs[1], ws, coeffs, scratch=scratch)
        torch.cuda.synchronize()
    finally:
        api.lib.muon_polar_set_step_mode(prev)
        api.lib.muon_polar_set_split_mode(prev_split)
    return y, scratch[:1024].clone()


@pytest.mark.parametrize("steps", [1, 2, 5, 9])
@pytest.mark.parametrize("shape", [(16, 256, 1024), (8, 512, 2048), (32, 384, 1024),
                                   (3, 200, 704), (1, 768, 3072)])
def test_steps_single_launch_matches_three_kernel_chain(api, cuda_device, shape, steps):
    """Up to 8 steps in ONE fused persistent launch (9 steps: a launch of 8
    and one of 1) give the bits of the three-kernel chain, and the launch
    leaves its dependency counters zeroed for the next call."""
    x = make_input(shape, seed=41).to(cuda_device)
    # past the five rows, the last (convergent, p(1) = 1) row repeats, as
    # Polar Express schedules do; cycling back to the first row diverges
    coeffs = [COEFFICIENTS[min(i, len(COEFFICIENTS) - 1)] for i in range(steps)]
    before = api.launch_count()
    y_f, ctr = _steps_fused_vs_chain(api, x, coeffs, 1)
    launches = api.launch_count() - before
    assert launches == (steps + 7) // 8
    y_c, _ = _steps_fused_vs_chain(api, x, coeffs, 2)
    _watchdog_clear(api)
    assert not torch.isnan(y_f.float()).any()
    assert torch.equal(y_f.view(torch.int16), y_c.view(torch.int16))
    assert int(ctr.count_nonzero()) == 0


def test_steps_match_step_calls_and_oracle(pkg, api, cuda_device):
    """The five-step fused launch equals five polar_step calls and the
    oracle's loop of the reference's example at the reference tolerance."""
    x = make_input((16, 256, 1024), seed=42).to(cuda_device)
    y, _ = _steps_fused_vs_chain(api, x, COEFFICIENTS, 1)
    ref = x
    for a, b, c in COEFFICIENTS:
        ref = pkg.polar_step(ref, a, b, c)
    assert torch.equal(y.view(torch.int16), ref.view(torch.int16))
    want = polar_express_oracle(x.cpu(), COEFFICIENTS, normalize=False)
    torch.testing.assert_close(y.cpu().float(), want.float(), rtol=6e-2, atol=6e-2)


def test_steps_in_place_ping_pong(api, cuda_device):
    """x may be buf1 (the caller's iterate is overwritten by step 1) and y
    may be the buffer the last step would write: the Muon update's layout."""
    x = make_input((8, 256, 1024), seed=43).to(cuda_device)
    bsz, m, n = x.shape
    ws = torch.empty(api.workspace_bytes(bsz, m), dtype=torch.uint8, device=cuda_device)
    scratch = torch.zeros(api.scratch_bytes(bsz, m, n), dtype=torch.uint8, device=cuda_device)
    want, _ = _steps_fused_vs_chain(api, x, COEFFICIENTS, 2)
    for mode in (1, 2):
        it0, it1 = x.clone(), torch.empty_like(x)
        prev = api.lib.muon_polar_set_step_mode(mode)
        prev_split = api.lib.muon_polar_set_split_mode(2)
        try:
            # five steps: it0 -> it1 -> it0 -> it1 -> it0 -> y = it1
            api.steps(it0, it1, it1, it0, ws, COEFFICIENTS, scratch=scratch)
            torch.cuda.synchronize()
        finally:
            api.lib.muon_polar_set_step_mode(prev)
            api.lib.muon_polar_set_split_mode(prev_split)
        assert torch.equal(it1.view(torch.int16), want.view(torch.int16)), mode
    _watchdog_clear(api)
