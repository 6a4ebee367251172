"""GPU test of muon_polar_gram_static_scratch_sm100, the Gram entry point for
callers that cannot allocate device memory: a plugin inside a fixed memory
budget, code next to a framework allocator that has reserved the GPU, or a
hot path that must not call cudaMalloc.  Its split-K scratch is an array
built into the library instead of a caller buffer.

It is compared through the C ABI with the regular entry point,
muon_polar_gram_sm100, run on the same CTA-pair split-K path (split-K forced
on) with caller-owned scratch.  The header promises the same tiles, split
plan and reduction order, so the bits must be identical, on two calls in a
row -- the second call finds the array as the first call left it.  A plan
larger than the array's budget must be refused without a launch.  This file
sorts last so that a run stopping at the first failure has already run every
other test.
"""
from __future__ import annotations

import pytest
import torch

from oracle.polar_oracle import make_input

pytestmark = pytest.mark.gpu


def _same_bits(actual, expected):
    assert actual.shape == expected.shape
    assert torch.equal(actual.view(torch.int16), expected.view(torch.int16)), (
        int((actual.view(torch.int16) != expected.view(torch.int16)).sum()))


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
            _same_bits(got, expected)
    finally:
        api.set_kernel_policy(previous)
        api.set_split_mode(previous_split)


def test_static_scratch_refuses_plans_over_budget(cuda_device):
    from muon_fusion_ascend950_b200.capi import MuonPolarError, capi

    api = capi()
    previous_split = api.set_split_mode(1)
    previous_limit = api.set_static_scratch_limit(2 * 2 ** 20)  # 2 MiB: 7 split items
    try:
        x = make_input((8, 512, 2048), 33).to(cuda_device)
        mp = api.padded_rows(512)
        got = torch.zeros((8, mp, mp), dtype=torch.bfloat16, device=cuda_device)
        torch.cuda.synchronize()
        launches = api.launch_count()
        with pytest.raises(MuonPolarError) as err:
            api.gram_static_scratch(x, got)
        assert err.value.status == -7  # MUON_POLAR_ERR_STATIC_SCRATCH
        assert api.launch_count() == launches  # nothing was launched
        torch.cuda.synchronize()
        assert int(got.view(torch.int16).abs().sum()) == 0  # nothing was written
    finally:
        api.set_static_scratch_limit(previous_limit)
        api.set_split_mode(previous_split)
