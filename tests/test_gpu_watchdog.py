"""GPU test of the kernels' failure detection: a bounded wait that can never
end gives up, the kernel drains and returns, the host sees the watchdog bit,
MUON_POLAR_DEBUG_SYNC turns it into a RuntimeError (the reference's stage
localisation, csrc/muon_polar_step_binding.cpp:93-101), and the next step is
unaffected.

The wait that is made to run out: in a two-step fused launch
(muon_polar_steps_sm100, fused mode), every work item of matrix 1 in step 1
waits until step 0's apply tiles of matrix 1 are all counted.  Counts are
compared as sequence numbers (a signed difference), and the test seeds that
counter with 0xFFFFFFFF: it starts five below its target and, once step 0's
four apply parts have added to it, stands one below for good.  Each such wait happens before its item issues
any load (the producers and the epilogue's X tile both wait first), so when
it gives up nothing is in flight; the kernel's waits are limited to 1 ms
for the test (muon_polar_set_wait_limit_ns).  Nothing faults or hangs: every
wait involved is bounded, and the launch ends by itself within milliseconds.
"""
from __future__ import annotations

import pytest
import torch

from oracle.polar_oracle import COEFFICIENTS, make_input

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def api():
    from muon_fusion_ascend950_b200.capi import capi

    return capi()


def _two_fused_steps(api, x, ws, scratch, bufs, y):
    prev = api.set_step_mode(1)
    prev_split = api.set_split_mode(2)
    try:
        api.steps(x, y, bufs[0], bufs[1], ws, COEFFICIENTS[:2], scratch=scratch)
        torch.cuda.synchronize()
    finally:
        api.set_step_mode(prev)
        api.set_split_mode(prev_split)


@pytest.mark.timeout(300)
def test_dependency_wait_gives_up_and_is_reported(api, cuda_device, monkeypatch):
    import muon_fusion_ascend950_b200 as pkg
    from muon_fusion_ascend950_b200.capi import WATCHDOG_DEPENDENCY

    dev = torch.cuda.current_device()
    assert api.read_device_status(dev) == 0
    bsz, m, n = 4, 256, 512
    x = make_input((bsz, m, n), seed=51).to(cuda_device)
    ws = torch.empty(api.workspace_bytes(bsz, m), dtype=torch.uint8, device=cuda_device)
    scratch = api.new_scratch(bsz, m, n)
    bufs = [torch.empty_like(x) for _ in range(2)]
    fresh = torch.full_like(x, float("nan"))
    _two_fused_steps(api, x, ws, scratch, bufs, fresh)
    assert api.read_device_status(dev) == 0
    assert not torch.isnan(fresh.float()).any()

    # counters: [0, B) Gram, [B, 2B) polynomial, [2B, 3B) apply, [3B] exits
    counters = scratch[:1024].view(torch.int32)
    counters[2 * bsz + 1] = -1  # 0xFFFFFFFF: step 1 of matrix 1 never starts
    previous_limit = api.set_wait_limit_ns(1_000_000)
    try:
        failed = torch.full_like(x, float("nan"))
        _two_fused_steps(api, x, ws, scratch, bufs, failed)  # returns
        flags = api.read_device_status(dev, clear=False)
        assert flags & WATCHDOG_DEPENDENCY, flags
        # the last CTA out zeroed the counters, as after any launch
        assert int(scratch[:1024].count_nonzero()) == 0
    finally:
        assert api.set_wait_limit_ns(previous_limit) == 1_000_000

    # the operator's debug sync reports the pending watchdog bits as an error
    monkeypatch.setenv("MUON_POLAR_DEBUG_SYNC", "1")
    a, b, c = COEFFICIENTS[0]
    with pytest.raises(RuntimeError, match="bounded wait"):
        pkg.polar_step(x, a, b, c)
    monkeypatch.delenv("MUON_POLAR_DEBUG_SYNC")
    assert api.read_device_status(dev) == 0  # the debug sync cleared the word

    # the next launch runs normally and gives the bits of the first one
    api.scratch_init(scratch)
    again = torch.full_like(x, float("nan"))
    _two_fused_steps(api, x, ws, scratch, bufs, again)
    assert api.read_device_status(dev) == 0
    assert torch.equal(again.view(torch.int16), fresh.view(torch.int16))
