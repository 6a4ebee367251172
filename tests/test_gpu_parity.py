"""GPU parity of the sm_100a kernels against the CPU oracle.

Stage tests drive each kernel through the C ABI (include/muon_polar_sm100.h)
and compare it with the oracle fed the SAME inputs (the previous stage's GPU
output), so each bound isolates one kernel:

* Gram / Poly: the output is one round-to-nearest-even of an fp32
  accumulation of K products, whose error is at most
  gamma_K * sum|products| with gamma_K = K * 2^-24 (deterministic bound for
  recursive fp32 summation; doubled here for the tensor core's blocked
  order).  So |out - rne(exact)| <= 1 ulp_bf16(exact) + 2*gamma_K*sum|.|,
  and only a small fraction of elements may differ at all.
* Apply: Y = rne(rne(T) + rne(alpha*x)); the accumulation error of T plus a
  one-ulp flip of rne(T) moves Y by at most
  ulp(T) + ulp(Y) + 2*gamma_K*sum|P||X|.

End-to-end tests use the reference test standard (fp32 compare,
rtol = atol = 6e-2, tests/test_polar_step.py:42,53 of the reference), plus
max abs error vs an fp32 evaluation of the formula no worse than 2x the
oracle's own error (the emulated reference kernels) and relative Frobenius
error <= 1e-2 per step.
"""
from __future__ import annotations

import pytest
import torch

from oracle.polar_oracle import (
    COEFFICIENTS,
    error_stats,
    kernel_dataflow_3d,
    make_input,
    polar_step_oracle,
    reference_formula,
    ulp_bf16,
)

pytestmark = pytest.mark.gpu

A1, B1, C1 = COEFFICIENTS[0]


@pytest.fixture(scope="module")
def api(cuda_device):
    from muon_fusion_ascend950_b200.capi import capi

    return capi()


@pytest.fixture(scope="module")
def op(cuda_device):
    import muon_fusion_ascend950_b200 as pkg

    return pkg.polar_step


def _rne(t64: torch.Tensor) -> torch.Tensor:
    return t64.to(torch.float32).to(torch.bfloat16).to(torch.float64)


def _gamma(k: int) -> float:
    return 2.0 * k * 2.0 ** -24


def _assert_within_ulps(actual, expected64, ulps, what, abs_slack=0.0, max_frac=0.02):
    a = actual.to(torch.float64)
    diff = (a - expected64).abs()
    bound = ulps * ulp_bf16(expected64) + abs_slack + 1e-30
    bad = diff > bound * (1 + 1e-9)
    assert not bool(bad.any()), (
        f"{what}: {int(bad.sum())} elements beyond {ulps} ulp, max diff {float(diff.max())}")
    frac = float((diff > 0).double().mean())
    assert frac <= max_frac, f"{what}: {frac:.4f} of elements differ (> {max_frac})"
    return frac


# engine (single CTAs / CTA pairs) x split-K: none (no scratch), "split"
# (uniform split forced wherever the device has room), "auto" (scratch
# passed, plan by size as the operator runs it: the exchange split of the
# off-diagonal tiles where it pays, e.g. the config-1 Gram on single CTAs)
MODES = ["single", "single_split", "single_auto", "pair", "pair_split", "pair_auto"]
_POLICY = {"single": 2, "pair": 1}


@pytest.fixture
def mode_policy(api):
    """Sets the kernel policy for one test and restores the default after;
    returns whether the mode passes split-K scratch."""
    def set_mode(mode):
        api.set_kernel_policy(_POLICY[mode.split("_")[0]])
        split = mode.endswith("_split") or mode.endswith("_auto")
        api.set_split_mode(1 if mode.endswith("_split") else 0)
        return split
    yield set_mode
    api.set_kernel_policy(0)
    api.set_split_mode(0)


def _check_watchdog(api):
    assert api.read_device_status(torch.cuda.current_device()) == 0


def _counters_zero(scratch):
    """The split-K arrival counters (first 1024 bytes) are back to zero."""
    if scratch.numel() > 1:
        assert int(scratch[:1024].cpu().count_nonzero()) == 0


# ------------------------------------------------------------------ stages
@pytest.mark.parametrize("mode", MODES)
@pytest.mark.parametrize("shape", [(1, 128, 128), (2, 150, 2064), (8, 512, 2048),
                                   (1, 300, 1000), (3, 64, 72), (1, 640, 640),
                                   (1, 256, 8192)])
def test_gram_stage(api, cuda_device, shape, mode, mode_policy):
    split = mode_policy(mode)
    bsz, m, n = shape
    x = make_input(shape, seed=1)
    mp = api.padded_rows(m)
    xd = x.to(cuda_device)
    scratch = api.new_scratch(bsz, m, n) if split else None
    gram = torch.full((bsz, mp, mp), float("nan"), dtype=torch.bfloat16, device=cuda_device)
    api.gram(xd, gram, scratch=scratch)
    torch.cuda.synchronize()
    _check_watchdog(api)
    if split:
        _counters_zero(scratch)
        again = torch.empty_like(gram)
        api.gram(xd, again, scratch=scratch)
        torch.cuda.synchronize()
        assert torch.equal(again.view(torch.int16), gram.view(torch.int16))
    g = gram.cpu()
    x64 = torch.zeros((bsz, mp, n), dtype=torch.float64)
    x64[:, :m] = x.to(torch.float64)
    exact = x64 @ x64.mT
    slack = _gamma(n) * (x64.abs() @ x64.abs().mT)
    _assert_within_ulps(g, _rne(exact), 1, f"gram {shape}", abs_slack=slack)
    # padded rows/cols are exact zeros; the result is exactly symmetric
    assert torch.equal(g[:, m:, :].float(), torch.zeros_like(g[:, m:, :].float()))
    assert torch.equal(g.view(torch.int16), g.mT.contiguous().view(torch.int16))


@pytest.mark.parametrize("mode", MODES)
@pytest.mark.parametrize("shape", [(1, 128, 128), (2, 256, 2064), (8, 512, 2048)])
def test_gram_f32_stage(api, cuda_device, shape, mode, mode_policy):
    split = mode_policy(mode)
    bsz, m, n = shape
    x = make_input(shape, seed=2)
    mp = api.padded_rows(m)
    scratch = api.new_scratch(bsz, m, n) if split else None
    gram = torch.full((bsz, mp, mp), float("nan"), dtype=torch.float32, device=cuda_device)
    api.gram_f32(x.to(cuda_device), gram, scratch=scratch)
    torch.cuda.synchronize()
    g = gram.cpu().to(torch.float64)
    x64 = x.to(torch.float64)
    exact = x64 @ x64.mT
    scale = (x64 * x64).sum(-1).max()
    assert float((g[:, :m, :m] - exact).abs().max()) <= 1e-5 * float(scale)
    assert torch.equal(g, g.mT)


@pytest.mark.parametrize("mode", MODES)
@pytest.mark.parametrize("shape", [(1, 128, 256), (2, 256, 512), (8, 512, 2048), (1, 1024, 1024)])
def test_poly_stage(api, cuda_device, shape, mode, mode_policy):
    split = mode_policy(mode)
    bsz, m, n = shape
    x = make_input(shape, seed=3)
    mp = api.padded_rows(m)
    xd = x.to(cuda_device)
    scratch = api.new_scratch(bsz, m, n) if split else None
    gram = torch.empty((bsz, mp, mp), dtype=torch.bfloat16, device=cuda_device)
    poly = torch.full_like(gram, float("nan"))
    api.gram(xd, gram, scratch=scratch)
    api.poly(gram, poly, B1, C1, scratch=scratch)
    torch.cuda.synchronize()
    _check_watchdog(api)
    if split:
        _counters_zero(scratch)
    a64 = gram.cpu().to(torch.float64)
    a2 = (a64 @ a64.mT).to(torch.float32)
    slack = abs(C1) * _gamma(mp) * (a64.abs() @ a64.abs().mT)
    b32 = torch.tensor(B1, dtype=torch.float32)
    c32 = torch.tensor(C1, dtype=torch.float32)
    expected = ((b32 * a64.to(torch.float32)) + (c32 * a2)).to(torch.float64)
    p = poly.cpu()
    _assert_within_ulps(p, _rne(expected), 1, f"poly {shape}", abs_slack=slack)
    assert torch.equal(p.view(torch.int16), p.mT.contiguous().view(torch.int16))


@pytest.mark.parametrize("mode", ["single", "pair"])
@pytest.mark.parametrize("shape,slabs", [((2, 512, 1024), ((0, 256), (256, 256))),
                                         ((1, 1024, 512), ((256, 512), (0, 1024)))])
def test_poly_rows_match_full(api, cuda_device, shape, slabs, mode, mode_policy):
    """Row slabs of kernel (2) (muon_polar_poly_rows_sm100, the multi-GPU
    split of the polynomial) equal the full kernel's rows bit for bit and
    leave the other rows untouched."""
    mode_policy(mode)
    bsz, m, n = shape
    x = make_input(shape, seed=10).to(cuda_device)
    mp = api.padded_rows(m)
    gram = torch.empty((bsz, mp, mp), dtype=torch.bfloat16, device=cuda_device)
    full = torch.empty_like(gram)
    api.gram(x, gram)
    api.poly(gram, full, B1, C1)
    for begin, rows in slabs:
        out = torch.full_like(gram, float("nan"))
        api.poly_rows(gram, out, B1, C1, begin, rows)
        torch.cuda.synchronize()
        _check_watchdog(api)
        sl = slice(begin, begin + rows)
        assert torch.equal(out[:, sl].view(torch.int16), full[:, sl].view(torch.int16))
        rest = torch.cat([out[:, :begin], out[:, begin + rows:]], dim=1)
        assert bool(torch.isnan(rest.float()).all())


@pytest.mark.parametrize("mode", ["single", "pair"])
@pytest.mark.parametrize("shape", [(1, 128, 256), (2, 150, 2064), (8, 512, 2048),
                                   (1, 200, 1000), (2, 384, 520)])
def test_apply_stage(api, cuda_device, shape, mode, mode_policy):
    mode_policy(mode)
    bsz, m, n = shape
    x = make_input(shape, seed=4)
    mp = api.padded_rows(m)
    xd = x.to(cuda_device)
    gram = torch.empty((bsz, mp, mp), dtype=torch.bfloat16, device=cuda_device)
    poly = torch.empty_like(gram)
    scratch = api.new_scratch(bsz, m, n)
    api.gram(xd, gram, scratch=scratch)
    api.poly(gram, poly, B1, C1, scratch=scratch)
    y = torch.full_like(xd, float("nan"))
    api.apply(poly, xd, y, A1)
    torch.cuda.synchronize()
    _check_watchdog(api)
    p64 = poly.cpu().to(torch.float64)[:, :, :m]
    x64 = x.to(torch.float64)
    t = p64[:, :m] @ x64
    alpha = torch.tensor(A1, dtype=torch.float32).to(torch.bfloat16).to(torch.float64)
    expected = _rne(_rne(t) + _rne(alpha * x64))
    got = y.cpu().to(torch.float64)
    diff = (got - expected).abs()
    bound = ulp_bf16(t) + ulp_bf16(expected) + _gamma(m) * (p64[:, :m].abs() @ x64.abs())
    assert bool((diff <= bound).all()), f"apply {shape}: max diff {float(diff.max())}"
    assert float((diff > 0).double().mean()) <= 0.05


# ------------------------------------------------------------------ end to end
def _end_to_end_check(y_gpu, x_cpu, steps, y_ref_bf16=None):
    coeffs = COEFFICIENTS[:steps]
    y32 = reference_formula(x_cpu.float(), coeffs)
    df = x_cpu
    for a, b, c in coeffs:
        df = polar_step_oracle(df, a, b, c)
    if y_ref_bf16 is None:
        y_ref_bf16 = reference_formula(x_cpu, coeffs)
    # reference test standard
    torch.testing.assert_close(y_gpu.float(), y_ref_bf16.float(), rtol=6e-2, atol=6e-2)
    e_gpu = error_stats(y_gpu, y32)
    e_df = error_stats(df, y32)
    assert e_gpu["max_abs"] <= 2.0 * e_df["max_abs"] + 1e-6, (e_gpu, e_df)
    assert e_gpu["rel_fro"] <= 1e-2 * steps, e_gpu
    return e_gpu, e_df


@pytest.mark.parametrize("name", ["cfg2_129x130", "cfg2_2x150x2050", "cfg2_1x130x129",
                                  "aligned_1x128x256"])
def test_golden_one_step(op, cuda_device, golden, name):
    _, cases = golden
    case, x, y_ref = cases[name]
    y = op(x.to(cuda_device), A1, B1, C1).cpu()
    assert y.shape == x.shape and y.dtype == torch.bfloat16
    _end_to_end_check(y, x, 1, y_ref)


def test_golden_five_steps(op, cuda_device, golden):
    _, cases = golden
    case, x, y_ref = cases["five_step_1x129x130"]
    y = x.to(cuda_device)
    for a, b, c in COEFFICIENTS:
        y = op(y, a, b, c)
    y = y.cpu()
    torch.testing.assert_close(y.float(), y_ref.float(), rtol=6e-2, atol=6e-2)
    y32 = reference_formula(x.float(), COEFFICIENTS)
    df = x
    for a, b, c in COEFFICIENTS:
        df = polar_step_oracle(df, a, b, c)
    assert error_stats(y, y32)["max_abs"] <= 2.0 * error_stats(df, y32)["max_abs"] + 1e-6


def test_config1_step(op, cuda_device):
    x = make_input((8, 512, 2048), seed=0)
    y = op(x.to(cuda_device), A1, B1, C1).cpu()
    e_gpu, e_df = _end_to_end_check(y, x, 1)
    # the kernels restate the reference dataflow: compare with it directly
    df = kernel_dataflow_3d(x, A1, B1, C1)
    d = (y.to(torch.float64) - df.to(torch.float64)).abs()
    assert float(d.max()) <= 4 * float(ulp_bf16(df.abs().max().reshape(1)))


def test_config3_five_step_loop(op, cuda_device):
    x = make_input((8, 512, 2048), seed=0)
    y = x.to(cuda_device)
    for a, b, c in COEFFICIENTS:
        y = op(y, a, b, c)
    y = y.cpu()
    y_ref = reference_formula(x, COEFFICIENTS)
    torch.testing.assert_close(y.float(), y_ref.float(), rtol=6e-2, atol=6e-2)
    y32 = reference_formula(x.float(), COEFFICIENTS)
    assert error_stats(y, y32)["rel_fro"] <= 5e-2


@pytest.mark.parametrize("shape", [(1, 128, 256), (2, 150, 2064), (8, 512, 2048)])
def test_kernel_paths_agree_bitwise(api, cuda_device, shape, mode_policy):
    """The single-CTA and CTA-pair kernels accumulate each output in the same
    K order and apply the same epilogue arithmetic, so they give identical
    bits.  (Regression guard: a multiply and an add that the reference rounds
    separately must not be contracted into one fused multiply-add.)"""
    bsz, m, n = shape
    x = make_input(shape, seed=6).to(cuda_device)
    mp = api.padded_rows(m)
    outs = {}
    for mode in ("single", "pair"):
        mode_policy(mode)
        gram = torch.empty((bsz, mp, mp), dtype=torch.bfloat16, device=cuda_device)
        poly = torch.empty_like(gram)
        y = torch.empty_like(x)
        api.gram(x, gram)
        api.poly(gram, poly, B1, C1)
        api.apply(poly, x, y, A1)
        torch.cuda.synchronize()
        outs[mode] = (gram.cpu(), poly.cpu(), y.cpu())
    for a, b, what in zip(outs["single"], outs["pair"], ("gram", "poly", "apply")):
        assert torch.equal(a.view(torch.int16), b.view(torch.int16)), what


@pytest.fixture
def step_mode(api):
    """Sets the step mode for one test and restores the default after."""
    def set_mode(mode):
        api.set_step_mode(mode)
    yield set_mode
    api.set_step_mode(0)


@pytest.mark.parametrize("shape", [(8, 512, 2048), (2, 150, 2064), (1, 128, 256),
                                   (3, 640, 1000), (1, 1024, 1024), (16, 256, 1024),
                                   (32, 256, 512), (16, 512, 2048)])
def test_fused_step_matches_three_kernels(api, cuda_device, shape, step_mode):
    """One fused persistent launch gives the bits of the three kernels, and
    repeated launches reuse the scratch counters correctly (they are reset by
    the last CTA of each launch).  The three kernels run without scratch, so
    without split-K: the fused kernel does not split K, and a split changes
    the fp32 summation order of the Gram and the polynomial.  [16|32,256,*]
    run polynomial items first on some pairs and then apply items with fewer
    polynomial K-blocks than stages (a change of stage layout mid-ring)."""
    bsz, m, n = shape
    x = make_input(shape, seed=8).to(cuda_device)
    ws = torch.empty(api.workspace_bytes(bsz, m), dtype=torch.uint8, device=cuda_device)
    scratch = api.new_scratch(bsz, m, n)
    outs = {}
    for mode in (2, 1):
        step_mode(mode)
        ys = []
        for _ in range(3):
            y = torch.full_like(x, float("nan"))
            api.step(x, y, ws, A1, B1, C1, scratch=scratch if mode == 1 else None)
            ys.append(y)
        torch.cuda.synchronize()
        _check_watchdog(api)
        _counters_zero(scratch)
        for y in ys[1:]:
            assert torch.equal(y.view(torch.int16), ys[0].view(torch.int16))
        outs[mode] = ys[0].cpu()
    assert torch.equal(outs[1].view(torch.int16), outs[2].view(torch.int16))
    e = error_stats(outs[1], reference_formula(make_input(shape, seed=8).float(), COEFFICIENTS[:1]))
    assert e["rel_fro"] <= 1e-2, e


@pytest.mark.parametrize("shape,fused", [((16, 512, 2048), True), ((64, 256, 1024), True),
                                         ((8, 512, 2048), False), ((4, 1024, 4096), False),
                                         ((64, 512, 2048), False)])
def test_step_by_size_choice(api, cuda_device, shape, fused, step_mode):
    """The default step mode picks one fused launch for many small matrices
    and three kernels otherwise, with the bits of the forced mode."""
    bsz, m, n = shape
    x = make_input(shape, seed=12).to(cuda_device)
    ws = torch.empty(api.workspace_bytes(bsz, m), dtype=torch.uint8, device=cuda_device)
    scratch = api.new_scratch(bsz, m, n)
    step_mode(0)
    y0 = torch.empty_like(x)
    before = api.launch_count()
    api.step(x, y0, ws, A1, B1, C1, scratch=scratch)
    launches = api.launch_count() - before
    step_mode(1 if fused else 2)
    y1 = torch.empty_like(x)
    api.step(x, y1, ws, A1, B1, C1, scratch=scratch)
    torch.cuda.synchronize()
    _check_watchdog(api)
    _counters_zero(scratch)
    assert launches == (1 if fused else 3)
    assert torch.equal(y0.view(torch.int16), y1.view(torch.int16))


@pytest.mark.parametrize("shape", [(8, 512, 2048), (4, 512, 2048), (1, 256, 1024),
                                   (2, 150, 2064), (3, 640, 1000), (1, 1024, 512),
                                   (9, 512, 2048)])
def test_column_halves_match_whole_tiles(api, cuda_device, shape):
    """The column-halves layout of the single-CTA Gram and polynomial (each
    off-diagonal tile as two 128 x 64 halves, one item per CTA) gives the
    bits of whole tiles: the Gram, the polynomial and a whole step, without
    split-K.  (9, 512, 2048) has more items than CTAs, so the by-size rule
    keeps whole tiles there and both modes agree trivially."""
    bsz, m, n = shape
    x = make_input(shape, seed=31).to(cuda_device)
    mp = api.padded_rows(m)
    prev_policy = api.set_kernel_policy(2)
    outs = {}
    try:
        for mode in (2, 0):
            api.set_halves_mode(mode)
            g = torch.full((bsz, mp, mp), float("nan"), device=cuda_device, dtype=torch.bfloat16)
            api.gram(x, g)
            pm = torch.full_like(g, float("nan"))
            api.poly(g, pm, B1, C1)
            ws = torch.empty(api.workspace_bytes(bsz, m), dtype=torch.uint8, device=cuda_device)
            y = torch.full_like(x, float("nan"))
            api.step(x, y, ws, A1, B1, C1)
            torch.cuda.synchronize()
            _check_watchdog(api)
            outs[mode] = (g, pm, y)
    finally:
        api.set_halves_mode(0)
        api.set_kernel_policy(prev_policy)
    for a, b in zip(outs[2], outs[0]):
        assert torch.equal(a.view(torch.int16), b.view(torch.int16))
    g = outs[0][0].float()
    assert torch.equal(g, g.mT)  # both triangles written, exactly symmetric


@pytest.mark.parametrize("shape", [(8, 512, 2048), (1, 129, 136), (16, 512, 2048)])
def test_tensor_maps_are_memoised(api, cuda_device, shape):
    """A step on the same buffers encodes no tensor map the second time
    (the memo of the C ABI's launch state), and gives the same bits."""
    bsz, m, n = shape
    x = make_input(shape, seed=21).to(cuda_device)
    ws = torch.empty(api.workspace_bytes(bsz, m), dtype=torch.uint8, device=cuda_device)
    scratch = api.new_scratch(bsz, m, n)
    y0 = torch.empty_like(x)
    api.step(x, y0, ws, A1, B1, C1, scratch=scratch)
    torch.cuda.synchronize()
    before = api.tensor_map_encodes()
    y1 = torch.empty_like(x)
    api.step(x, y1, ws, A1, B1, C1, scratch=scratch)
    api.step(x, y1, ws, A1, B1, C1, scratch=scratch)
    torch.cuda.synchronize()
    _check_watchdog(api)
    # y1 is a new output buffer: at most its own maps are new (first call)
    assert api.tensor_map_encodes() - before <= 3
    again = api.tensor_map_encodes()
    api.step(x, y1, ws, A1, B1, C1, scratch=scratch)
    torch.cuda.synchronize()
    assert api.tensor_map_encodes() == again
    assert torch.equal(y0.view(torch.int16), y1.view(torch.int16))


def test_torch_compile_matches_eager(op, cuda_device):
    """torch.compile (aot_eager backend, full graph) traces the operator with
    its FakeTensor kernel and runs it; the result equals eager bit for bit."""
    x = make_input((2, 256, 512), seed=11).to(cuda_device)

    def f(t):
        return torch.ops.muon_ascend950.polar_step(t, A1, B1, C1)

    compiled = torch.compile(f, backend="aot_eager", fullgraph=True)
    y_c = compiled(x)
    y_e = f(x)
    torch.cuda.synchronize()
    assert torch.equal(y_c.view(torch.int16), y_e.view(torch.int16))


@pytest.mark.parametrize("shape,bands", [((1, 1024, 4096), 3), ((2, 768, 2048), 3),
                                         ((1, 2048, 1024), 4)])
@pytest.mark.parametrize("reserve", [0, 16])
def test_gram_f32_bands_assemble_the_gram(api, cuda_device, shape, bands, reserve):
    """Band by band from row 0, each band's rows are complete right after its
    call, and the last band leaves the fp32 Gram of muon_polar_gram_f32_sm100
    (split-K off on both sides: same tiles, same K order, same bits)."""
    from muon_fusion_ascend950_b200.distributed import gram_bands

    bsz, m, n = shape
    x = make_input(shape, seed=51).to(cuda_device)
    mp = api.padded_rows(m)
    full = torch.empty((bsz, mp, mp), dtype=torch.float32, device=cuda_device)
    banded = torch.full_like(full, float("nan"))
    prev = api.lib.muon_polar_set_split_mode(2)
    try:
        api.gram_f32(x, full)
        for begin, count in gram_bands(mp, bands):
            api.gram_f32_band(x, banded, begin, count, reserve)
            torch.cuda.synchronize()
            rows = slice(0, begin + count)
            assert torch.equal(banded[:, rows], full[:, rows]), (begin, count)
    finally:
        api.lib.muon_polar_set_split_mode(prev)
    assert torch.equal(banded, full)


@pytest.mark.parametrize("shape", [(8, 512, 2048), (2, 150, 2064), (4, 512, 1024),
                                   (1, 129, 136), (3, 640, 1000), (9, 512, 2048)])
def test_deep_gram_stages_match(api, cuda_device, shape):
    """The single-CTA bf16 Gram with three-atom stages (K = 192) gives the bits
    of two-atom stages (K = 128): the k-steps run in the same order and the
    last stage's columns past n add zeros.  Checked on the Gram and on a whole
    step, with the column halves and with whole tiles ((9, 512, 2048)), and
    on widths that are and are not multiples of 192."""
    bsz, m, n = shape
    x = make_input(shape, seed=37).to(cuda_device)
    mp = api.padded_rows(m)
    prev_policy = api.set_kernel_policy(2)
    outs = {}
    try:
        for mode in (2, 1):
            api.set_stage_mode(mode)
            g = torch.full((bsz, mp, mp), float("nan"), device=cuda_device, dtype=torch.bfloat16)
            api.gram(x, g)
            ws = torch.empty(api.workspace_bytes(bsz, m), dtype=torch.uint8, device=cuda_device)
            y = torch.full_like(x, float("nan"))
            api.step(x, y, ws, A1, B1, C1)
            torch.cuda.synchronize()
            _check_watchdog(api)
            outs[mode] = (g, y)
    finally:
        api.set_stage_mode(0)
        api.set_kernel_policy(prev_policy)
    for a, b in zip(outs[2], outs[1]):
        assert torch.equal(a.view(torch.int16), b.view(torch.int16))
