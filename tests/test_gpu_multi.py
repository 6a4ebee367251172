"""Multi-GPU tests (need >= 2 GPUs; skipped otherwise): the column-sharded
driver over NCCL against the single-GPU operator, run as child processes,
one per GPU, with NVLink SHARP (NVLS) off."""
from __future__ import annotations

import multiprocessing as mp
import os
import socket
import sys
from pathlib import Path

import pytest
import torch

REPO = Path(__file__).resolve().parent.parent
sys.path.insert(0, str(REPO))

pytestmark = pytest.mark.gpu


def _gpus() -> int:
    return torch.cuda.device_count() if torch.cuda.is_available() else 0


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, m, n, steps, out_dir, shard_poly=False, overlap=0,
            packed=True):
    import datetime

    import torch
    import torch.distributed as dist

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    os.environ["NCCL_NVLS_ENABLE"] = "0"
    sys.path.insert(0, str(REPO))
    from muon_fusion_ascend950_b200.distributed import ColumnShardedPolar, column_range
    from oracle.polar_oracle import COEFFICIENTS, make_input

    device = torch.device("cuda", rank)
    torch.cuda.set_device(device)
    dist.init_process_group("nccl", rank=rank, world_size=world, device_id=device,
                            timeout=datetime.timedelta(seconds=60))
    x = make_input((m, n), seed=9)
    cols = column_range(n, rank, world)
    x_local = x[:, cols.start:cols.stop].contiguous().to(device)
    driver = ColumnShardedPolar(m, device, shard_poly=shard_poly, overlap_bands=overlap,
                                packed=packed)
    assert driver.packed == (packed and overlap <= 1)
    assert (driver.poly_slab is not None) == (shard_poly and not driver.packed)
    y = driver.run(x_local, COEFFICIENTS[:steps])
    torch.cuda.synchronize()
    torch.save(y.cpu(), os.path.join(out_dir, f"y{rank}.pt"))
    dist.barrier()
    dist.destroy_process_group()


@pytest.mark.skipif(_gpus() < 2, reason="needs 2 GPUs")
@pytest.mark.parametrize("m,n,steps,shard_poly,overlap,packed", [
    (512, 4096, 1, False, 0, True),      # packed units: reduce-scatter + all-gathers
    (1024, 8192, 5, False, 0, True),
    (520, 3000, 5, False, 0, True),      # ragged: Mp = 768, slabs of 1504 / 1496 columns
    (1024, 8192, 5, False, 0, False),    # full all-reduce, polynomial replicated
    (1024, 8192, 5, True, 0, False),     # full all-reduce, polynomial row slabs
    (1024, 8192, 5, True, 4, False)])    # all-reduce band by band
def test_column_sharded_nccl_matches_single_gpu(tmp_path, m, n, steps, shard_poly, overlap,
                                                packed):
    import muon_fusion_ascend950_b200 as pkg
    from oracle.polar_oracle import COEFFICIENTS, error_stats, make_input, reference_formula

    ctx = mp.get_context("spawn")
    port = _free_port()
    procs = [ctx.Process(target=_worker,
                         args=(r, 2, port, m, n, steps, str(tmp_path), shard_poly, overlap,
                               packed))
             for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=300)
        assert p.exitcode == 0
    y = torch.cat([torch.load(tmp_path / f"y{r}.pt") for r in range(2)], dim=1)
    x = make_input((m, n), seed=9)
    single = x.cuda()
    for a, b, c in COEFFICIENTS[:steps]:
        single = pkg.polar_step(single, a, b, c)
    single = single.cpu()
    y32 = reference_formula(x.float(), COEFFICIENTS[:steps])
    e_shard = error_stats(y, y32)
    e_single = error_stats(single, y32)
    torch.testing.assert_close(y.float(), single.float(), rtol=6e-2, atol=6e-2)
    assert e_shard["rel_fro"] <= 1.5 * e_single["rel_fro"] + 1e-3, (e_shard, e_single)
