"""CPU tests of the C ABI library: it loads without a GPU, exports every
entry point declared in include/muon_polar_sm100.h, and rejects bad
arguments before touching a device."""
from __future__ import annotations

import ctypes
import re
from pathlib import Path

import pytest

from muon_fusion_ascend950_b200.capi import CAPI, SIGNATURES

HEADER = Path(__file__).resolve().parent.parent / "include" / "muon_polar_sm100.h"


def header_functions():
    text = HEADER.read_text()
    return sorted(set(re.findall(r"^\w[\w\s\*]*?\b(muon_polar_\w+)\s*\(", text, re.M)))


@pytest.fixture(scope="module")
def api():
    return CAPI()


def test_header_declares_entry_points():
    names = header_functions()
    assert "muon_polar_step_sm100" in names and "muon_polar_gram_sm100" in names
    assert len(names) >= 12


def test_library_exports_every_header_symbol(api):
    for name in header_functions():
        assert hasattr(api.lib, name), name


def test_binding_covers_every_header_symbol():
    assert set(header_functions()) == set(SIGNATURES)


def test_abi_version_and_sizes(api):
    assert api.abi_version() == 1
    assert api.padded_rows(1) == 256 and api.padded_rows(256) == 256
    assert api.padded_rows(257) == 512 and api.padded_rows(0) == 0
    assert api.workspace_bytes(8, 512) == 2 * 8 * 512 * 512 * 2
    assert api.workspace_bytes(0, 5) == 0


def test_status_strings(api):
    assert api.status_string(0) == "success"
    for code in (-1, -2, -3, -4, -5, -6, -7):
        assert api.status_string(code) != "unknown status"


def _vp(v):
    return ctypes.c_void_p(v)


def test_argument_validation_without_device(api):
    lib = api.lib
    # null input / bad sizes are rejected before any CUDA call
    assert lib.muon_polar_gram_sm100(None, _vp(16), 1, 128, 128, 128, None, 0, None) == -1
    assert lib.muon_polar_gram_sm100(_vp(16), _vp(16), 0, 128, 128, 128, None, 0, None) == -1
    assert lib.muon_polar_gram_sm100(_vp(16), _vp(16), 1, 128, 128, 64, None, 0, None) == -1
    # misaligned pointer / leading dimension
    assert lib.muon_polar_gram_sm100(_vp(18), _vp(16), 1, 128, 128, 128, None, 0, None) == -3
    assert lib.muon_polar_gram_sm100(_vp(16), _vp(16), 1, 128, 130, 130, None, 0, None) == -3
    assert lib.muon_polar_poly_sm100(_vp(16), _vp(16), 1, 100, 1.0, 1.0, None, 0, None) == -1
    assert lib.muon_polar_apply_sm100(_vp(16), _vp(16), None, 1, 8, 8, 8, 8, 1.0, None) == -1
    # step: workspace too small, y aliasing x
    assert lib.muon_polar_step_sm100(_vp(16), _vp(32), _vp(16), 8, None, 0, 1, 8, 8, 8, 8,
                                     1.0, 1.0, 1.0, None) == -5
    assert lib.muon_polar_step_sm100(_vp(16), _vp(16), _vp(16), 1 << 30, None, 0, 1, 8, 8, 8, 8,
                                     1.0, 1.0, 1.0, None) == -1
    assert lib.muon_polar_cast_f32_bf16_sm100(None, _vp(16), 4, None) == -1
    assert lib.muon_polar_gram_static_scratch_sm100(None, _vp(16), 1, 8, 8, 8, None) == -1
    assert lib.muon_polar_gram_static_scratch_sm100(_vp(16), _vp(24), 1, 8, 8, 8, None) == -3
    assert lib.muon_polar_set_kernel_policy(7) == -1
    # poly rows: slab not a multiple of 256, or past the end
    assert lib.muon_polar_poly_rows_sm100(_vp(16), _vp(16), 1, 512, 128, 256, 1.0, 1.0, None) == -1
    assert lib.muon_polar_poly_rows_sm100(_vp(16), _vp(16), 1, 512, 256, 512, 1.0, 1.0, None) == -1
    assert lib.muon_polar_poly_rows_sm100(_vp(16), _vp(24), 1, 512, 0, 256, 1.0, 1.0, None) == -3
    assert lib.muon_polar_set_split_mode(3) == -1
    assert lib.muon_polar_set_split_mode(-1) == -1
    assert lib.muon_polar_read_device_status(0, None, 0) == -1


def test_transposed_entry_validation_without_device(api):
    """The M > N entries check their arguments like the plain ones; the
    transposed step sizes its workspace by N (the Gram is N x N)."""
    lib = api.lib
    assert lib.muon_polar_gram_t_sm100(None, _vp(16), 1, 300, 128, 128, None, 0, None) == -1
    assert lib.muon_polar_gram_t_sm100(_vp(16), _vp(24), 1, 300, 128, 128, None, 0, None) == -3
    assert lib.muon_polar_gram_t_sm100(_vp(16), _vp(16), 1, 300, 130, 130, None, 0, None) == -3
    assert lib.muon_polar_apply_t_sm100(_vp(16), _vp(16), None, 1, 300, 8, 8, 8, 1.0, None) == -1
    assert lib.muon_polar_apply_t_sm100(_vp(16), _vp(16), _vp(16), 1, 300, 16, 16, 8, 1.0,
                                        None) == -1
    # workspace for N = 128 rows of the Gram is enough; for M = 300 it is not
    # required
    small = api.workspace_bytes(1, 128) - 1
    assert lib.muon_polar_step_t_sm100(_vp(16), _vp(32), _vp(16), small, None, 0, 1, 300, 128,
                                       128, 128, 1.0, 1.0, 1.0, None) == -5
    assert lib.muon_polar_step_t_sm100(_vp(16), _vp(16), _vp(16), 1 << 30, None, 0, 1, 300, 128,
                                       128, 128, 1.0, 1.0, 1.0, None) == -1


def test_caller_side_entry_validation_without_device(api):
    """The multi-step and Muon-update entries reject bad arguments before
    touching a device."""
    lib = api.lib
    coeffs = (ctypes.c_float * 3)(1.0, 1.0, 1.0)
    ws = api.express_workspace_bytes(1, 128, 256)
    assert ws > api.workspace_bytes(1, 128)
    assert api.express_workspace_bytes(0, 128, 256) == 0
    # x aliases y; zero steps; unknown dtype; fp32 without normalisation
    assert lib.muon_polar_express_sm100(_vp(16), 1, 256, _vp(16), 256, _vp(16), ws, None, 0, 1,
                                        128, 256, coeffs, 1, 1, None) == -1
    assert lib.muon_polar_express_sm100(_vp(16), 1, 256, _vp(32), 256, _vp(16), ws, None, 0, 1,
                                        128, 256, coeffs, 0, 1, None) == -1
    assert lib.muon_polar_express_sm100(_vp(16), 2, 256, _vp(32), 256, _vp(16), ws, None, 0, 1,
                                        128, 256, coeffs, 1, 1, None) == -1
    assert lib.muon_polar_express_sm100(_vp(16), 0, 256, _vp(32), 256, _vp(16), ws, None, 0, 1,
                                        128, 256, coeffs, 1, 0, None) == -1
    # unaligned in-place read; workspace too small
    assert lib.muon_polar_express_sm100(_vp(16), 1, 130, _vp(32), 256, _vp(16), ws, None, 0, 1,
                                        128, 130, coeffs, 1, 0, None) == -3
    assert lib.muon_polar_express_sm100(_vp(16), 1, 256, _vp(32), 256, _vp(16), ws - 1, None, 0,
                                        1, 128, 256, coeffs, 1, 1, None) == -5
    # update: aliasing tensors, bad dtype, misalignment, small workspace
    f32 = ctypes.c_float
    args = (f32(0.1), f32(0.9), 1, f32(0.0), f32(1.0), coeffs, 1, None)
    assert lib.muon_polar_update_sm100(_vp(16), _vp(16), _vp(48), 0, _vp(64), ws, None, 0, 1, 128,
                                       256, *args) == -1
    assert lib.muon_polar_update_sm100(_vp(16), _vp(32), _vp(48), 3, _vp(64), ws, None, 0, 1, 128,
                                       256, *args) == -1
    assert lib.muon_polar_update_sm100(_vp(16), _vp(40), _vp(48), 0, _vp(64), ws, None, 0, 1, 128,
                                       256, *args) == -3
    assert lib.muon_polar_update_sm100(_vp(16), _vp(32), _vp(48), 0, _vp(64), ws - 1, None, 0, 1,
                                       128, 256, *args) == -5


def test_steps_entry_validation_without_device(api):
    """muon_polar_steps_sm100 refuses, before touching a device: no
    coefficients or steps, missing or equal buffers for several steps, a
    first step that would overwrite its input (buf0 == x), a last step that
    would overwrite its own input (y == buf[(steps - 2) % 2]), misaligned
    buffers and a small workspace."""
    lib = api.lib
    coeffs = (ctypes.c_float * 15)(*([1.0] * 15))
    ws = api.workspace_bytes(1, 128)
    x, y, b0, b1 = _vp(16), _vp(32), _vp(48), _vp(64)

    def call(x_, y_, b0_, b1_, ldb, steps, wsb=ws, cf=coeffs):
        return lib.muon_polar_steps_sm100(x_, y_, b0_, b1_, ldb, _vp(16), wsb, None, 0, 1, 128,
                                          256, 256, 256, cf, steps, None)

    assert call(x, y, b0, b1, 256, 0) == -1
    assert call(x, y, b0, b1, 256, 2, cf=None) == -1
    assert call(x, x, b0, b1, 256, 1) == -1
    assert call(x, y, None, b1, 256, 2) == -1
    assert call(x, y, b0, b0, 256, 2) == -1
    assert call(x, y, x, b1, 256, 2) == -1
    assert call(x, y, b0, b1, 128, 2) == -1          # ldb < n
    assert call(x, b0, b0, b1, 256, 2) == -1         # last (2nd) step reads buf0
    assert call(x, b1, b0, b1, 256, 3) == -1         # last (3rd) step reads buf1
    assert call(x, y, _vp(40), b1, 256, 2) == -3
    assert call(x, y, b0, b1, 260, 2) == -3
    assert call(x, y, b0, b1, 256, 2, wsb=ws - 1) == -5


def test_gram_band_validation_without_device(api):
    """The banded fp32 Gram refuses, before touching a device, bands that are
    not 256-row multiples inside the padded rows, and a negative reserve."""
    lib = api.lib

    def call(begin, count, reserve=0, x=_vp(16), m=600):
        return lib.muon_polar_gram_f32_band_sm100(x, _vp(32), 1, m, 512, 512, begin, count,
                                                  reserve, None, 0, None)

    assert call(0, 256, x=None) == -1
    assert call(128, 256) == -1      # not a multiple of 256
    assert call(0, 100) == -1
    assert call(0, 0) == -1
    assert call(512, 512) == -1      # past Mp = 768
    assert call(-256, 256) == -1
    assert call(0, 256, reserve=-1) == -1


# ---------------------------------------------------------------- host logic
@pytest.mark.parametrize("d", [1, 2, 3, 4, 7, 16, 32])
def test_kernel_tile_enumeration_matches_oracle(api, d):
    """The kernels' symmetric work-item order (decode_tile, run on the host)
    visits exactly the oracle's upper-triangle tiles, in its row-major order,
    matrix after matrix (the set the reference enumerates, asc:129-146)."""
    from oracle.polar_oracle import upper_tiles

    per = d * (d + 1) // 2
    expected = upper_tiles(d)
    for batch in (1, 3):
        got = [api.decode_tile(t, True, d, d, per) for t in range(per * batch)]
        assert got == [(b, tm, tn) for b in range(batch) for tm, tn in expected]


@pytest.mark.parametrize("d,first,rows", [(4, 1, 2), (8, 3, 5), (8, 0, 8), (6, 5, 1)])
def test_kernel_band_enumeration_matches_oracle(api, d, first, rows):
    """A band of tile rows [first, first + rows): the upper tiles of those
    rows, in the oracle's order (the row-band Gram of the column-sharded
    driver)."""
    from oracle.polar_oracle import upper_tiles

    expected = [(tm, tn) for tm, tn in upper_tiles(d) if first <= tm < first + rows]
    per = len(expected)
    assert per == rows * d - (2 * first + rows - 1) * rows // 2
    got = [api.decode_tile(t, True, d, d, per, first) for t in range(2 * per)]
    assert got == [(b, tm, tn) for b in range(2) for tm, tn in expected]


def test_kernel_grid_enumeration(api):
    got = [api.decode_tile(t, False, 3, 5, 15) for t in range(30)]
    assert got == [(b, r, c) for b in range(2) for r in range(3) for c in range(5)]


def test_tile_decoder_rejects_bad_arguments(api):
    from muon_fusion_ascend950_b200.capi import MuonPolarError

    with pytest.raises(MuonPolarError):
        api.decode_tile(-1, True, 4, 4, 10)
    with pytest.raises(MuonPolarError):
        api.decode_tile(0, True, 4, 4, 11)  # more tiles than the triangle holds
    with pytest.raises(MuonPolarError):
        api.decode_tile(0, False, 3, 5, 14)


def test_static_scratch_address_cache_keeps_only_success(api):
    """A failed device-address lookup is reported and not cached; the next
    call looks up again, and a success is reused without a new lookup."""
    assert api.check_address_cache() == 0


def test_static_scratch_limit_setter(api):
    full = 1024 + 80 * 262144
    prev = api.set_static_scratch_limit(4096)
    try:
        assert prev == full
        assert api.set_static_scratch_limit(0) == 4096
        assert api.set_static_scratch_limit(10 * full) == full  # clamped to the array
    finally:
        api.set_static_scratch_limit(prev)
    assert api.set_static_scratch_limit(0) == full


def test_wait_limit_setter_validation_without_device(api):
    from muon_fusion_ascend950_b200.capi import MuonPolarError

    for bad in (0, 999, 60_000_000_001):
        with pytest.raises(MuonPolarError):
            api.set_wait_limit_ns(bad)


def test_mode_setters_round_trip_without_device(api):
    """Every process-wide mode setter rejects out-of-range values with
    MUON_POLAR_ERR_INVALID_ARGUMENT, leaves the mode unchanged then, and
    returns the previous mode on a valid call (none needs a GPU)."""
    lib = api.lib
    setters = {  # name: highest valid mode
        "muon_polar_set_kernel_policy": 2,
        "muon_polar_set_split_mode": 2,
        "muon_polar_set_step_mode": 2,
        "muon_polar_set_halves_mode": 2,
        "muon_polar_set_stage_mode": 2,
    }
    for name, hi in setters.items():
        fn = getattr(lib, name)
        start = fn(0)
        assert 0 <= start <= hi, name
        assert fn(hi + 1) == -1, name
        assert fn(-1) == -1, name
        for mode in range(hi + 1):
            assert fn(mode) == (0 if mode == 0 else mode - 1), name
        assert fn(start) == hi, name  # restore
