"""CPU tests of the multi-GPU drivers (muon_fusion_ascend950_b200.distributed):
partitioning, the column-sharded step on 2 gloo ranks against the
single-process oracle, and detection of a rank that dies before the
all-reduce.  The CUDA kernels are replaced by oracle.CpuKernels, passed
explicitly as the backend (the product default is the C ABI)."""
from __future__ import annotations

import multiprocessing as mp
import os
import socket
import sys
import time
from pathlib import Path

import pytest
import torch

REPO = Path(__file__).resolve().parent.parent
sys.path.insert(0, str(REPO))

from muon_fusion_ascend950_b200.distributed import (  # noqa: E402
    batch_sharded_steps,
    column_range,
    nominal_flops,
    partition_items,
)
from oracle.polar_oracle import COEFFICIENTS, kernel_dataflow_3d, make_input  # noqa: E402


def test_partition_covers_and_balances_config4():
    # config 4: 128 attention matrices [4096,4096] + 96 FFN [4096,11008]
    costs = [nominal_flops(4096, 4096)] * 128 + [nominal_flops(4096, 11008)] * 96
    total = sum(costs)
    for world in (1, 2, 4, 8):
        parts = partition_items(costs, world)
        flat = sorted(i for p in parts for i in p)
        assert flat == list(range(len(costs)))
        loads = [sum(costs[i] for i in p) for p in parts]
        assert max(loads) - min(loads) <= max(costs)
        assert max(loads) <= total / world * 1.01


def test_partition_edge_cases():
    assert partition_items([], 3) == [[], [], []]
    assert partition_items([5.0], 2) == [[0], []]
    with pytest.raises(ValueError):
        partition_items([1.0], 0)


@pytest.mark.parametrize("n,world", [(65536, 2), (65536, 8), (130, 2), (2050, 4), (8, 4)])
def test_column_ranges(n, world):
    ranges = [column_range(n, r, world) for r in range(world)]
    covered = [c for r in ranges for c in r]
    assert covered == list(range(n))
    for r in ranges[:-1]:
        assert r.start % 8 == 0 and (r.stop - r.start) % 8 == 0 or len(r) == 0


def test_batch_sharded_steps_no_collective():
    xs = [make_input((64, 96), seed=i) for i in range(5)]

    def step(x, a, b, c):
        return x * 2

    got = {}
    for rank in range(2):
        got.update(batch_sharded_steps(xs, [(1, 1, 1)], rank, 2, step=step))
    assert sorted(got) == list(range(5))
    for i, y in got.items():
        assert torch.equal(y, xs[i] * 2)


# ------------------------------------------------------------ multi-process
def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _column_worker(rank, world, port, m, n, steps, out_dir, shard_poly=False, overlap=0,
                   packed=True):
    import datetime

    import torch.distributed as dist

    from muon_fusion_ascend950_b200.distributed import ColumnShardedPolar, column_range
    from oracle.polar_oracle import COEFFICIENTS, CpuKernels, make_input

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=30))
    x = make_input((m, n), seed=7)
    cols = column_range(n, rank, world)
    x_local = x[:, cols.start:cols.stop].contiguous()
    driver = ColumnShardedPolar(m, "cpu", backend=CpuKernels(), shard_poly=shard_poly,
                                overlap_bands=overlap, packed=packed)
    assert len(driver.bands) == (min(overlap, driver.mp // 256) if overlap > 1 else 0)
    assert driver.packed == (packed and overlap <= 1)
    if driver.packed:
        # units of the upper triangle, cut into equal slabs (the last padded)
        d = driver.mp // 256
        units = d * (d + 1) // 2
        per = -(-units // world)
        assert driver.unit_slab == (rank * per, max(0, min(per, units - rank * per)))
        bytes_ = driver.collective_bytes()
        assert bytes_["reduce_scatter_fp32"] == 4 * per * world * 256 * 256
    elif shard_poly:
        # 2 ranks, Mp = 512: rank r computes polynomial rows [256 r, 256 r + 256)
        assert driver.poly_slab == (256 * rank, 256)
    y = driver.run(x_local, COEFFICIENTS[:steps])
    torch.save(y, os.path.join(out_dir, f"y{rank}.pt"))
    dist.barrier()
    dist.destroy_process_group()


@pytest.mark.parametrize("m,n,steps,shard_poly,overlap,packed,world", [
    (96, 200, 1, False, 0, True, 2),     # one unit: rank 1 has only padding
    (130, 256, 2, False, 0, True, 2),
    (520, 700, 2, False, 0, True, 2),    # 3 x 3 units, 6 of them packed
    (1000, 1200, 1, False, 0, True, 3),  # 10 units on 3 ranks: 4 + 4 + 2
    (300, 320, 2, True, 0, False, 2),    # all-reduce + polynomial row slabs
    (600, 640, 1, False, 0, False, 2),   # all-reduce, polynomial replicated
    (600, 640, 2, False, 3, False, 2)])  # all-reduce band by band
def test_column_sharded_ranks_match_single(tmp_path, m, n, steps, shard_poly, overlap, packed,
                                          world):
    """gloo ranks, each owning a column slab, against the single-process
    dataflow: by default on the packed upper triangle (reduce-scatter of
    the fp32 units, all-gathers of packed A and P); `packed=False` with a
    full all-reduce, `overlap` running the Gram in row bands, each band
    all-reduced on its own."""
    ctx = mp.get_context("spawn")
    port = _free_port()
    procs = [ctx.Process(target=_column_worker,
                         args=(r, world, port, m, n, steps, str(tmp_path), shard_poly, overlap,
                               packed))
             for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0
    y = torch.cat([torch.load(tmp_path / f"y{r}.pt") for r in range(world)], dim=1)
    x = make_input((m, n), seed=7)
    ref = x.unsqueeze(0)
    for a, b, c in COEFFICIENTS[:steps]:
        ref = kernel_dataflow_3d(ref, a, b, c)
    ref = ref.squeeze(0)
    d = (y.to(torch.float64) - ref.to(torch.float64)).abs()
    # only the fp32 order of the Gram sum differs from the single-process run
    assert float(d.max()) <= 2e-2 * steps
    assert float(d.mean()) <= 1e-4 * steps


def test_gram_bands_cover_rows():
    from muon_fusion_ascend950_b200.distributed import gram_bands

    for mp_rows, bands in [(256, 4), (1024, 4), (8192, 4), (8192, 5), (2048, 3)]:
        got = gram_bands(mp_rows, bands)
        assert got[0][0] == 0 and sum(c for _, c in got) == mp_rows
        assert all(b % 256 == 0 and c % 256 == 0 and c > 0 for b, c in got)
        assert all(got[i][0] + got[i][1] == got[i + 1][0] for i in range(len(got) - 1))
        assert len(got) == min(bands, mp_rows // 256)


def _dying_worker(rank, world, port, out_dir):
    import datetime

    import torch.distributed as dist

    from muon_fusion_ascend950_b200.distributed import ColumnShardedPolar
    from oracle.polar_oracle import COEFFICIENTS, CpuKernels, make_input

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=5))
    if rank == 1:
        os._exit(3)  # this rank dies between steps, before its all-reduce
    driver = ColumnShardedPolar(64, "cpu", backend=CpuKernels())
    t0 = time.time()
    try:
        driver.step(make_input((64, 64), seed=1), *COEFFICIENTS[0])
        status = "no error"
    except Exception as exc:  # noqa: BLE001 - the failure is the thing tested
        status = f"error after {time.time() - t0:.1f}s: {type(exc).__name__}"
    with open(os.path.join(out_dir, "rank0.txt"), "w") as f:
        f.write(status)
    os._exit(0)


def test_dead_rank_is_detected_by_the_collective(tmp_path):
    ctx = mp.get_context("spawn")
    port = _free_port()
    procs = [ctx.Process(target=_dying_worker, args=(r, 2, port, str(tmp_path)))
             for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=120)
    assert procs[1].exitcode == 3
    status = (tmp_path / "rank0.txt").read_text()
    assert status.startswith("error after"), status
