"""CPU tests of the oracle: pinned to the reference's own golden vectors.

The fixtures in tests/golden/polar_golden.npz were produced by running the
reference's `_reference` function (tests/test_polar_step.py:22-28 of the
reference) on seeded inputs; see tests/golden/make_golden.py.
"""
from __future__ import annotations

import pytest
import torch

from oracle.polar_oracle import (
    COEFFICIENTS,
    align_up,
    error_stats,
    kernel_dataflow_3d,
    make_input,
    nominal_flops,
    padded_shape,
    polar_step_oracle,
    reference_formula,
    ulp_bf16,
    upper_tiles,
)


def test_golden_meta(golden):
    meta, cases = golden
    assert [tuple(c) for c in meta["coefficients"]] == [tuple(c) for c in COEFFICIENTS]
    assert {"cfg2_129x130", "cfg2_2x150x2050", "cfg2_1x130x129",
            "five_step_1x129x130", "aligned_1x128x256"} <= set(cases)


@pytest.mark.parametrize("name", ["cfg2_129x130", "cfg2_2x150x2050", "cfg2_1x130x129",
                                  "five_step_1x129x130", "aligned_1x128x256"])
def test_formula_matches_reference_golden(golden, name):
    """The restated formula reproduces the reference's own outputs (bf16)."""
    _, cases = golden
    case, x, y_ref = cases[name]
    y = reference_formula(x, COEFFICIENTS[: case["steps"]])
    d = (y.to(torch.float64) - y_ref.to(torch.float64)).abs()
    # bit-exact on the machine that made the fixtures; other CPUs may round a
    # bf16 matmul differently by one ulp
    assert bool((d <= 2 * ulp_bf16(y_ref)).all()), float(d.max())


@pytest.mark.parametrize("name", ["cfg2_129x130", "cfg2_2x150x2050", "cfg2_1x130x129",
                                  "aligned_1x128x256"])
def test_inputs_regenerate_from_seed(golden, name):
    _, cases = golden
    case, x, _ = cases[name]
    assert torch.equal(make_input(tuple(case["shape"]), case["seed"]).view(torch.int16),
                       x.view(torch.int16))


@pytest.mark.parametrize("name", ["cfg2_129x130", "cfg2_2x150x2050", "cfg2_1x130x129",
                                  "aligned_1x128x256"])
def test_kernel_dataflow_within_reference_tolerance(golden, name):
    """The restated kernel numerics meet the reference test standard and are
    at least as accurate as the bf16 formula's own rounding suggests."""
    _, cases = golden
    case, x, y_ref = cases[name]
    a, b, c = COEFFICIENTS[0]
    y = polar_step_oracle(x, a, b, c)
    assert y.shape == x.shape and y.dtype == torch.bfloat16
    torch.testing.assert_close(y.float(), y_ref.float(), rtol=6e-2, atol=6e-2)
    y32 = reference_formula(x.float(), COEFFICIENTS[:1])
    s = error_stats(y, y32)
    assert s["rel_fro"] < 1e-2, s
    # within 4 ulps of the output scale of the fp32 result
    assert s["max_abs"] <= 4 * float(ulp_bf16(y32.abs().max().reshape(1))), s


def test_five_step_loop_oracle(golden):
    _, cases = golden
    case, x, y_ref = cases["five_step_1x129x130"]
    y = x
    for a, b, c in COEFFICIENTS:
        y = polar_step_oracle(y, a, b, c)
    torch.testing.assert_close(y.float(), y_ref.float(), rtol=6e-2, atol=6e-2)


def test_transpose_policy_equivalence():
    """M > N goes through the transpose (ops.py:26-33): the result equals the
    formula applied to the untransposed input."""
    x = make_input((1, 140, 130), seed=3)
    a, b, c = COEFFICIENTS[0]
    y = polar_step_oracle(x, a, b, c)
    y32 = reference_formula(x.float(), COEFFICIENTS[:1])
    assert error_stats(y, y32)["rel_fro"] < 1e-2


def test_padding_rule():
    """rows = align(M,128), cols = max(align(N,16), rows) (binding.cpp:630-631)."""
    assert padded_shape(129, 130) == (256, 256)
    assert padded_shape(150, 2050) == (256, 2064)
    assert padded_shape(512, 2048) == (512, 2048)
    assert align_up(1, 128) == 128 and align_up(128, 128) == 128


def test_padding_does_not_change_results():
    """Zero padding of rows/cols leaves the cropped result unchanged."""
    x = make_input((1, 100, 120), seed=5)
    a, b, c = COEFFICIENTS[0]
    y = kernel_dataflow_3d(x, a, b, c)
    xp = torch.zeros((1, 100, 200), dtype=torch.bfloat16)
    xp[:, :, :120] = x
    yp = kernel_dataflow_3d(xp, a, b, c)
    assert torch.equal(yp[:, :, :120].view(torch.int16), y.view(torch.int16))
    assert torch.equal(yp[:, :, 120:].float(), torch.zeros(1, 100, 80))


@pytest.mark.parametrize("d", [1, 2, 3, 4, 16, 32])
def test_upper_tile_enumeration_is_a_bijection(d):
    tiles = upper_tiles(d)
    assert len(tiles) == d * (d + 1) // 2 == len(set(tiles))
    assert all(0 <= tm <= tn < d for tm, tn in tiles)


def test_nominal_flops():
    assert nominal_flops(512, 2048) == 4 * 512 ** 2 * 2048 + 2 * 512 ** 3
    assert nominal_flops(2048, 512) == nominal_flops(512, 2048)
    assert 8 * nominal_flops(512, 2048) == 19327352832
