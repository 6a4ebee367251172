"""GPU tests of the packed upper-triangle entry points used by the
column-sharded multi-GPU path (no counterpart in the reference, which runs
on one device): the packed fp32 Gram, the polynomial on a range of units,
the unpack to the full symmetric matrix, and the whole packed pipeline of
two column slabs emulated on one GPU (the collective replaced by a sum)."""
from __future__ import annotations

import pytest
import torch

from oracle.polar_oracle import COEFFICIENTS, CpuKernels, error_stats, make_input

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def api():
    from muon_fusion_ascend950_b200.capi import capi

    return capi()


def _units(mp):
    return CpuKernels.unit_grid(mp)


@pytest.mark.parametrize("shape", [(1, 1000, 3000), (2, 512, 2048), (1, 300, 8192)])
def test_gram_f32_packed_matches_full_gram(api, cuda_device, shape):
    """Each unit is the full kernel's block, bit for bit (same tiles, same K
    order); on diagonal units the lower-left quarter is unspecified."""
    bsz, m, n = shape
    x = make_input(shape, seed=61).to(cuda_device)
    mp = api.padded_rows(m)
    units = api.packed_units(m)
    assert units == len(_units(mp))
    full = torch.zeros((bsz, mp, mp), dtype=torch.float32, device=cuda_device)
    api.gram_f32(x, full)
    packed = torch.full((bsz, units, 256, 256), float("nan"), device=cuda_device)
    api.gram_f32_packed(x, packed)
    torch.cuda.synchronize()
    for u, (i, j) in enumerate(_units(mp)):
        blk = full[:, 256 * i:256 * i + 256, 256 * j:256 * j + 256]
        got = packed[:, u]
        if i == j:
            for rs, cs in ((slice(0, 128), slice(0, 256)), (slice(128, 256), slice(128, 256))):
                assert torch.equal(got[:, rs, cs], blk[:, rs, cs]), (u, i, j)
        else:
            assert torch.equal(got, blk), (u, i, j)
    assert api.read_device_status(torch.cuda.current_device()) == 0


@pytest.mark.parametrize("shape", [(1, 1000, 3000), (2, 512, 2048)])
def test_poly_packed_ranges_match_full_poly(api, cuda_device, shape):
    """Units computed in two ranges equal the CTA-pair polynomial's blocks,
    bit for bit, and units outside a range are left untouched."""
    bsz, m, n = shape
    x = make_input(shape, seed=62).to(cuda_device)
    mp = api.padded_rows(m)
    units = api.packed_units(m)
    gram = torch.empty((bsz, mp, mp), dtype=torch.bfloat16, device=cuda_device)
    api.gram(x, gram)
    a, b, c = COEFFICIENTS[0]
    prev = api.set_kernel_policy(1)  # the full polynomial on CTA pairs as well
    try:
        full = torch.empty_like(gram)
        api.poly(gram, full, b, c)
    finally:
        api.set_kernel_policy(prev)
    packed = torch.full((bsz, units, 256, 256), float("nan"), dtype=torch.bfloat16,
                        device=cuda_device)
    split = max(1, units // 3)
    api.poly_packed(gram, packed, b, c, 0, split)
    torch.cuda.synchronize()
    if split < units:
        assert torch.isnan(packed[:, split:].float()).all()  # not touched
        api.poly_packed(gram, packed, b, c, split, units - split)
    torch.cuda.synchronize()
    for u, (i, j) in enumerate(_units(mp)):
        blk = full[:, 256 * i:256 * i + 256, 256 * j:256 * j + 256]
        assert torch.equal(packed[:, u].view(torch.int16), blk.view(torch.int16)), (u, i, j)


def test_unpack_builds_the_symmetric_matrix(api, cuda_device):
    """A symmetric matrix packed on the CPU comes back bit for bit; the
    lower-left quarters of diagonal units hold NaN and are never read."""
    bsz, mp = 2, 768
    grid = _units(mp)
    gen = torch.Generator().manual_seed(5)
    r = torch.randn((bsz, mp, mp), generator=gen).to(torch.bfloat16)
    sym = torch.triu(r) + torch.triu(r, 1).mT
    packed = torch.empty((bsz, len(grid), 256, 256), dtype=torch.bfloat16)
    for u, (i, j) in enumerate(grid):
        packed[:, u] = sym[:, 256 * i:256 * i + 256, 256 * j:256 * j + 256]
        if i == j:
            packed[:, u, 128:, :128] = float("nan")
    full = torch.full((bsz, mp, mp), float("nan"), dtype=torch.bfloat16, device=cuda_device)
    api.unpack_sym(packed.to(cuda_device), full)
    torch.cuda.synchronize()
    got = full.cpu()
    assert torch.equal(got.view(torch.int16), sym.view(torch.int16))
    want = torch.zeros_like(sym)
    CpuKernels.unpack_sym(packed, want)  # the CPU stand-in agrees
    assert torch.equal(want.view(torch.int16), sym.view(torch.int16))


@pytest.mark.parametrize("m,n", [(1024, 8192), (520, 3000)])
def test_packed_column_sharded_pipeline_on_one_gpu(api, cuda_device, m, n):
    """Two column slabs' packed partial Grams summed (the reduce-scatter's
    sum), cast once, unpacked; the polynomial's units in two ranges; then the
    apply on each slab: against the single-GPU polar_step chain, with the
    bound of the multi-GPU test."""
    import muon_fusion_ascend950_b200 as pkg
    from oracle.polar_oracle import reference_formula

    x = make_input((m, n), seed=63)
    half = (n // 2 + 7) // 8 * 8
    slabs = [x[:, :half].contiguous(), x[:, half:].contiguous()]
    mp = api.padded_rows(m)
    units = api.packed_units(m)
    dev = cuda_device
    y = [s.clone().unsqueeze(0).to(dev) for s in slabs]
    for a, b, c in COEFFICIENTS:
        parts = []
        for s in y:
            p = torch.zeros((1, units, 256, 256), dtype=torch.float32, device=dev)
            api.gram_f32_packed(s, p)
            parts.append(p)
        summed = parts[0] + parts[1]
        a_packed = torch.empty(summed.shape, dtype=torch.bfloat16, device=dev)
        api.cast_f32_bf16(summed, a_packed)
        gram = torch.empty((1, mp, mp), dtype=torch.bfloat16, device=dev)
        api.unpack_sym(a_packed, gram)
        p_packed = torch.empty_like(a_packed)
        first = (units + 1) // 2
        api.poly_packed(gram, p_packed, b, c, 0, first)
        if units > first:
            api.poly_packed(gram, p_packed, b, c, first, units - first)
        poly = torch.empty_like(gram)
        api.unpack_sym(p_packed, poly)
        outs = []
        for s in y:
            o = torch.empty_like(s)
            api.apply(poly, s, o, a)
            outs.append(o)
        y = outs
    torch.cuda.synchronize()
    got = torch.cat([v.squeeze(0).cpu() for v in y], dim=1)
    single = x.unsqueeze(0).to(dev)
    for a, b, c in COEFFICIENTS:
        single = pkg.polar_step(single, a, b, c)
    single = single.squeeze(0).cpu()
    ref32 = reference_formula(x.float(), COEFFICIENTS)
    torch.testing.assert_close(got.float(), single.float(), rtol=6e-2, atol=6e-2)
    e_got, e_single = error_stats(got, ref32), error_stats(single, ref32)
    assert e_got["rel_fro"] <= 1.5 * e_single["rel_fro"] + 1e-3, (e_got, e_single)
    assert api.read_device_status(torch.cuda.current_device()) == 0
