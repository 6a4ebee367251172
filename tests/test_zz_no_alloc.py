"""GPU test of muon_polar_gram_static_scratch_sm100, the Gram entry point for
callers that cannot allocate device memory (its split-K scratch is an array
built into the library instead of a caller buffer).

It is compared with the regular entry point, muon_polar_gram_sm100, run on the
same CTA-pair split-K path (split-K forced on) with caller-owned scratch, using the tolerance of
the Gram stage tests (one bf16 ulp), on two calls in a row -- the second call
finds the array as the first call left it.  This file sorts last so that a
run stopping at the first failure has already run every other test.
"""
from __future__ import annotations

import pytest
import torch

from oracle.polar_oracle import make_input, ulp_bf16

pytestmark = pytest.mark.gpu


def _within_one_ulp(actual, expected):
    a = actual.cpu().to(torch.float64)
    e = expected.cpu().to(torch.float64)
    assert bool(torch.isfinite(a).all())
    assert bool(((a - e).abs() <= ulp_bf16(e)).all()), float((a - e).abs().max())


def test_static_scratch_gram_matches_regular_entry(cuda_device):
    from muon_fusion_ascend950_b200.capi import capi

    api = capi()
    previous = api.set_kernel_policy(1)  # regular entry on the same CTA-pair path
    previous_split = api.set_split_mode(1)  # split-K (and so the scratch) in use
    try:
        # two calls in a row: a split problem, then a different split problem
        for shape, seed in (((8, 512, 2048), 31), ((2, 300, 1000), 32)):
            bsz, m, n = shape
            x = make_input(shape, seed).to(cuda_device)
            mp = api.padded_rows(m)
            expected = torch.empty((bsz, mp, mp), dtype=torch.bfloat16, device=cuda_device)
            scratch = api.new_scratch(bsz, m, n)
            assert 0 < api.scratch_bytes(bsz, m, n) <= 1024 + 80 * 262144
            api.gram(x, expected, scratch=scratch)
            got = torch.full_like(expected, float("nan"))
            api.gram_static_scratch(x, got)
            torch.cuda.synchronize()
            assert api.read_device_status(torch.cuda.current_device()) == 0
            _within_one_ulp(got, expected)
    finally:
        api.set_kernel_policy(previous)
        api.set_split_mode(previous_split)
