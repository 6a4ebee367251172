"""Benchmark of the Polar Express step on B200 (one JSON line on rank 0).

Workload: one ``polar_step`` on X bf16 [8, 512, 2048]
per GPU, N(0,1) entries from seed (rank), each matrix scaled by
1/(||X||_F*1.01 + 1e-6), step-1 coefficients.  With ``--gpus N`` (torchrun,
one process per GPU) every rank runs its own batch of 8 matrices: the batch
is sharded across GPUs with no collective on the data path (weak scaling).

value     effective TFLOP/s of the whole job: nominal FLOPs
          (4 M^2 N + 2 M^3 per matrix) x matrices x K / max-over-ranks time
          of K steps, inputs resident in HBM, the steps replayed from CUDA
          graphs captured through the public API ``polar_step``: graphs of
          one step per rotating input set in a row (as a training loop
          captures its optimizer step), single-step graphs for the rest of K.
          The same K steps as one single-step graph each are reported too.
e2e       the same metric through the public API without graphs, with each
          step's input copied host->device from pinned memory and its output
          copied back inside the timed region (copies on their own streams,
          overlapping the neighbouring steps' compute).
roofline  the dominant kernel's nominal FLOPs per launch / its CUDA-event
          time (timed alone, same buffers), against the measured bf16 peak.

``--impl reference`` times the reference's PyTorch formula
(tests/test_polar_step.py:22-28 of the reference, restated in
oracle/polar_oracle.py) on the host CPU with every thread, rank 0 only.
"""
from __future__ import annotations

import argparse
import gc
import json
import os
import statistics
import sys
import threading
import time
from pathlib import Path

REPO = Path(__file__).resolve().parent
if str(REPO) not in sys.path:
    sys.path.insert(0, str(REPO))

BATCH, M, N = 8, 512, 2048
COEFFICIENTS = (
    (8.156554524902461, -22.48329292557795, 15.878769915207462),
    (4.042929935166739, -2.808917465908714, 0.5000178451051316),
    (3.8916678022926607, -2.772484153217685, 0.5060648178503393),
    (3.285753657755655, -2.3681294933425376, 0.46449024233003106),
    (2.3465413258596377, -1.7097828382687081, 0.42323551169305323),
)
ROTATION = 8             # input sets cycled through: 8 x 42 MB > 126 MB L2
L2_BYTES = 126 * 2 ** 20
FALLBACK_TFLOPS = 1590.0


def nominal_flops_per_matrix(m: int, n: int) -> int:
    """4 M^2 N + 2 M^3 with M <= N (the operator transposes when M > N)."""
    m, n = min(m, n), max(m, n)
    return 4 * m * m * n + 2 * m ** 3


def parse_args():
    p = argparse.ArgumentParser(description=__doc__.splitlines()[0])
    p.add_argument("--gpus", type=int, default=1)
    p.add_argument("--steps", type=int, default=2000)
    p.add_argument("--warmup", type=int, default=20)
    p.add_argument("--impl", choices=["ours", "reference"], default="ours")
    p.add_argument("--e2e-steps", type=int, default=200,
                   help="steps of the host-buffer end-to-end loop (<= --steps)")
    p.add_argument("--no-cpu-baseline", action="store_true")
    p.add_argument("--shape", default="8,512,2048",
                   help="B,M,N of the `shape` workload (one polar_step per timed step)")
    p.add_argument("--poly", choices=["replicated", "sharded"], default="sharded",
                   help="cfg5 with several GPUs: kernel 2 on every rank (replicated) or "
                        "split into row slabs and all-gathered (sharded)")
    p.add_argument("--overlap-bands", type=int, default=0,
                   help="cfg5 with several GPUs: run the Gram in this many row bands and "
                        "all-reduce each band while the next one computes (0: one all-reduce)")
    p.add_argument("--sm-reserve", type=int, default=16,
                   help="cfg5 with --overlap-bands: SMs the Gram bands leave to NCCL")
    p.add_argument("--sharded", choices=["auto", "on", "off"], default="auto",
                   help="also time the sharded workloads (configs 5 and 4) on the same GPUs "
                        "and check the column-sharded result against one GPU, in the headline "
                        "line under `sharded` (auto: with the default cfg1 workload)")
    p.add_argument("--workload", choices=["cfg1", "cfg3", "cfg4", "cfg5", "shape", "express"],
                   default="cfg1",
                   help="cfg1 (default, the headline): one step on [8,512,2048] per GPU; "
                        "cfg3: the 5-step loop on [8,512,2048] per GPU; cfg4: 5-step Muon "
                        "update of a 32-layer 7B model's matrices, batch-sharded over the "
                        "GPUs; cfg5: 5 steps on one [8192,65536] matrix, column-sharded "
                        "with an NCCL all-reduce of the fp32 Gram per step; shape: one "
                        "step on --shape per GPU (config 2 shapes, profiling cases); "
                        "express: the five steps on --shape as one polar_express call "
                        "(a single fused launch for small matrices)")
    return p.parse_args()


# --------------------------------------------------------------------- clocks
class ClockSampler:
    """Samples SM clock and clock-event reasons through NVML in a thread."""

    REASONS = {
        0x1: "gpu_idle", 0x2: "applications_clocks_setting", 0x4: "sw_power_cap",
        0x8: "hw_slowdown", 0x10: "sync_boost", 0x20: "sw_thermal_slowdown",
        0x40: "hw_thermal_slowdown", 0x80: "hw_power_brake_slowdown",
        0x100: "display_clock_setting",
    }

    def __init__(self, device_index: int, interval_s: float = 0.005):
        self.samples = []
        self.reasons = 0
        self.max_mhz = None
        self._stop = threading.Event()
        self._thread = None
        self._interval = interval_s
        try:
            import pynvml

            pynvml.nvmlInit()
            self._nvml = pynvml
            self._h = pynvml.nvmlDeviceGetHandleByIndex(device_index)
            self.max_mhz = pynvml.nvmlDeviceGetMaxClockInfo(self._h, pynvml.NVML_CLOCK_SM)
        except Exception:  # noqa: BLE001 - clocks are reported as unavailable
            self._nvml = None

    def _sample(self):
        nv = self._nvml
        self.samples.append(nv.nvmlDeviceGetClockInfo(self._h, nv.NVML_CLOCK_SM))
        try:
            r = nv.nvmlDeviceGetCurrentClocksEventReasons(self._h)
        except Exception:  # noqa: BLE001
            r = nv.nvmlDeviceGetCurrentClocksThrottleReasons(self._h)
        self.reasons |= int(r) & ~0x1

    def _run(self):
        self._sample()
        while not self._stop.wait(self._interval):
            self._sample()

    def __enter__(self):
        if self._nvml is not None:
            self._thread = threading.Thread(target=self._run, daemon=True)
            self._thread.start()
        return self

    def __exit__(self, *exc):
        if self._thread is not None:
            self._stop.set()
            self._thread.join()
            self._sample()

    def summary(self):
        if self._nvml is None or not self.samples:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvml unavailable"]}
        return {
            "sm_mhz": statistics.median(self.samples),
            "sm_max_mhz": self.max_mhz,
            "samples": len(self.samples),
            "reasons": [name for bit, name in self.REASONS.items() if self.reasons & bit],
        }


# --------------------------------------------------------------------- helpers
def align_rows(m: int) -> int:
    """Rows of the square Gram / polynomial buffers (a multiple of 256)."""
    return -(-m // 256) * 256


def rotation_sets(batch: int, m: int, n: int) -> int:
    """Rotating input sets of the headline workload: enough that one cycle
    touches more than three times the L2 (X, Y and the step's buffers)."""
    k, g = min(m, n), max(m, n)
    set_bytes = 3 * batch * k * g * 2 + 2 * batch * align_rows(k) ** 2 * 2
    return int(min(8, max(2, -(-3 * L2_BYTES // set_bytes))))


def workload_config(workload: str, world: int) -> dict:
    """The `config` object of the JSON line, identical for both arms."""
    shape_str = f"[{BATCH},{M},{N}]"
    rot = rotation_sets(BATCH, M, N)
    k, g = min(M, N), max(M, N)
    touched = (3 * BATCH * k * g * 2 + 2 * BATCH * align_rows(k) ** 2 * 2) >> 20
    return {
        "workload": ("5-step polar_step loop on [8,512,2048] bf16 (BASELINE config 3) per GPU"
                     if workload == "cfg3" else
                     f"polar_express (5 steps, one call) on {shape_str} bf16 per GPU"
                     if workload == "express" else
                     f"polar_step {shape_str} bf16 single step per GPU" +
                     (" (BASELINE config 1)" if workload == "cfg1" else "")),
        "global_batch": BATCH * world, "m": M, "n": N,
        "parallelism": f"batch-sharded x{world}, no data-path collective",
        "l2": f"inputs larger than L2: {rot} rotating input sets ({rot} x {touched} MB touched "
              f"per cycle > {L2_BYTES >> 20} MB L2)",
    }


def large_workload_config(workload: str, world: int, column_path: str = "packed",
                          bands: int = 0, sm_reserve: int = 16, poly_slabs: bool = True) -> dict:
    """The `config` object of configs 4 and 5, identical for both arms (the
    reference arm describes the GPU arm's default column-sharded path)."""
    if workload == "cfg4":
        return {"workload": ("Muon update of a 32-layer 7B model: 5-step loop on [128,4096,4096] + "
                             "[96,4096,11008] bf16 (BASELINE config 4)"),
                "parallelism": f"batch-sharded x{world} (FLOP-balanced, no data-path collective)",
                "l2": "inputs larger than L2"}
    if world == 1:
        parallelism = "single GPU"
    elif column_path == "packed":
        parallelism = (f"column-sharded x{world}: packed upper-triangle units, NCCL fp32 "
                       "reduce-scatter + bf16 all-gathers of A and P per step")
    else:
        reduce = ("one NCCL fp32 all-reduce of the 8192x8192 partial Gram per step" if not bands
                  else f"the partial Gram in {bands} row bands, each NCCL fp32 all-reduced while "
                       f"the next computes ({sm_reserve} SMs left to NCCL)")
        parallelism = (f"column-sharded x{world}, {reduce}, kernel 2 "
                       + ("in row slabs + NCCL bf16 all-gather" if poly_slabs else "replicated"))
    return {"workload": "5-step loop on one [8192,65536] bf16 matrix (BASELINE config 5)",
            "parallelism": parallelism, "l2": "inputs larger than L2"}


def metric_name(workload: str) -> str:
    shape_str = f"[{BATCH},{M},{N}]"
    if workload == "cfg3":
        return f"5-step Polar Express loop effective TFLOP/s at {shape_str} bf16"
    if workload == "express":
        return f"5-step polar_express call effective TFLOP/s at {shape_str} bf16"
    return f"polar_step effective TFLOP/s at {shape_str} bf16"


def measured_peaks():
    path = REPO / "MEASURED_PEAKS.json"
    if path.is_file():
        peaks = json.loads(path.read_text())
        return float(peaks["bf16_tflops"]), "measured"
    return FALLBACK_TFLOPS, "fallback"


def profiled_traffic():
    """Per-launch DRAM bytes of the dominant kernel from the committed ncu
    summary (profiles/ncu_traffic.json), or None."""
    path = REPO / "profiles" / "ncu_traffic.json"
    if path.is_file():
        return json.loads(path.read_text())
    return None


def dist_env():
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local = int(os.environ.get("LOCAL_RANK", str(rank)))
    return rank, world, local


def cpu_reference_rate(steps: int, warmup: int, budget_s: float, rows: int = 1):
    """Times the reference formula (bf16, CPU, all threads) on a sample of the
    workload.  Returns (TFLOP/s, threads, sample description)."""
    import torch

    from oracle.polar_oracle import make_input, reference_formula

    threads = os.cpu_count() or 1
    torch.set_num_threads(threads)
    coeffs = COEFFICIENTS[:rows]
    probe = make_input((1, M, N), seed=0)
    t0 = time.perf_counter()
    reference_formula(probe, coeffs)
    per_matrix = max(time.perf_counter() - t0, 1e-4)
    total = max(steps + warmup, 1)
    batch = max(1, min(BATCH, int(budget_s / (per_matrix * total))))
    x = make_input((batch, M, N), seed=0)
    for _ in range(warmup):
        reference_formula(x, coeffs)
    times = []
    for _ in range(max(steps, 1)):
        t0 = time.perf_counter()
        reference_formula(x, coeffs)
        times.append(time.perf_counter() - t0)
    med = statistics.median(times)
    rate = rows * batch * nominal_flops_per_matrix(M, N) / med / 1e12
    sample = (f"{len(times)} timed steps (median) of the reference formula "
              f"({rows} coefficient row(s)) on {batch} of the {BATCH} matrices [{M},{N}] "
              f"bf16, after {warmup} warm-up")
    return rate, threads, sample


# --------------------------------------------------------------------- sharded
PARITY_SHAPE = (1024, 8192)


def _max_over_ranks(ms: float, world: int, device) -> float:
    import torch
    import torch.distributed as dist

    if world == 1:
        return ms
    t = torch.tensor([ms], device=device, dtype=torch.float64)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def _timed_updates(fn, updates: int, world: int, device, sync_all) -> float:
    """ms per call of fn (one 5-step update) over `updates` calls, CUDA
    events on the current stream, max over ranks."""
    import torch

    sync_all()
    e0 = torch.cuda.Event(enable_timing=True)
    e1 = torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(updates):
        fn()
    e1.record()
    e1.synchronize()
    return _max_over_ranks(e0.elapsed_time(e1) / updates, world, device)


def run_sharded(rank: int, world: int, device, sync_all) -> dict:
    """The sharded workloads of BASELINE configs 5 and 4 on the job's GPUs,
    each against the same workload on one GPU (rank 0's, timed in the same
    process while the other ranks wait), plus a parity check of the
    column-sharded result against the single-GPU polar_step chain.  Every
    rank runs this (it issues collectives); the result is meaningful on
    rank 0."""
    import torch
    import torch.distributed as dist

    import muon_fusion_ascend950_b200 as pkg
    from muon_fusion_ascend950_b200.distributed import (
        ColumnShardedPolar, column_range, nominal_flops, partition_items)

    gen = torch.Generator(device=device)
    out = {}

    def normalised_slab(m, n, seed):
        """Columns of this rank of one normalised [m, n] matrix (global
        Frobenius norm), generated on the device in slab order."""
        cols = column_range(n, rank, world)
        gen.manual_seed(seed * 1000 + rank)
        x = torch.randn((m, len(cols)), generator=gen, device=device).to(torch.bfloat16)
        sq = (x.float() ** 2).sum().reshape(1)
        if world > 1:
            dist.all_reduce(sq)
        return (x / (sq.sqrt() * 1.01 + 1e-6)).to(torch.bfloat16)

    def single_gpu_updates(x, updates):
        def upd():
            y = x
            for a, b, c in COEFFICIENTS:
                y = pkg.polar_step(y, a, b, c)
        upd()
        torch.cuda.synchronize(device)
        return _timed_updates(upd, updates, 1, device, lambda: torch.cuda.synchronize(device))

    # ---- config 5: one [8192, 65536] matrix, 5 steps, column-sharded
    m5, n5 = 8192, 65536
    flops5 = 5 * nominal_flops(m5, n5)
    x_local = normalised_slab(m5, n5, 5)
    driver = ColumnShardedPolar(m5, device, packed=True) if world > 1 else None
    sampler = ClockSampler(int(device.index))
    if driver is not None:
        driver.run(x_local, COEFFICIENTS)  # warm-up
        with sampler:
            ms_n = _timed_updates(lambda: driver.run(x_local, COEFFICIENTS), 3, world, device,
                                  sync_all)
    sync_all()
    ms_1 = None
    if rank == 0:
        gen.manual_seed(55)
        x_full = torch.randn((1, m5, n5), generator=gen, device=device).to(torch.bfloat16)
        x_full = x_full / (x_full.norm() * 1.01 + 1e-6)
        ms_1 = single_gpu_updates(x_full, 2)
        del x_full
        torch.cuda.empty_cache()
    sync_all()
    cfg5 = {"workload": "5-step loop on one [8192,65536] bf16 matrix (BASELINE config 5)",
            "ms_per_5_steps_1gpu": ms_1,
            "tflops_1gpu": flops5 / (ms_1 * 1e-3) / 1e12 if ms_1 else None}
    if driver is not None:
        cfg5.update({
            "parallelism": f"column-sharded x{world}: packed upper-triangle units, NCCL fp32 "
                           "reduce-scatter + bf16 all-gathers of A and P per step",
            "ms_per_5_steps": ms_n, "tflops": flops5 / (ms_n * 1e-3) / 1e12,
            "efficiency": (ms_1 / (world * ms_n)) if ms_1 else None,
            "collective_bytes_per_step": driver.collective_bytes(),
            "clocks": sampler.summary(),
        })
        del driver
    del x_local
    torch.cuda.empty_cache()
    out["cfg5"] = cfg5

    # ---- config 4: 128 [4096,4096] + 96 [4096,11008], 5 steps, batch-sharded
    kinds = [(4096, 4096)] * 128 + [(4096, 11008)] * 96
    flops4 = 5 * sum(nominal_flops(*k) for k in kinds)

    def cfg4_batches(items, seed):
        gen.manual_seed(seed)
        n_att = sum(1 for i in items if kinds[i] == (4096, 4096))
        xs = []
        for cnt, n in ((n_att, 4096), (len(items) - n_att, 11008)):
            if cnt:
                x = torch.randn((cnt, 4096, n), generator=gen, device=device).to(torch.bfloat16)
                xs.append(x / (x.norm(dim=(-2, -1), keepdim=True) * 1.01 + 1e-6))
        return xs

    def cfg4_update(xs):
        for x in xs:
            y = x
            for a, b, c in COEFFICIENTS:
                y = pkg.polar_step(y, a, b, c)

    ms4_1 = None
    if rank == 0:
        xs = cfg4_batches(list(range(len(kinds))), 44)
        cfg4_update(xs)
        torch.cuda.synchronize(device)
        ms4_1 = _timed_updates(lambda: cfg4_update(xs), 1, 1, device,
                               lambda: torch.cuda.synchronize(device))
        del xs
        torch.cuda.empty_cache()
    sync_all()
    cfg4 = {"workload": "Muon update of a 32-layer 7B model: 5-step loop on [128,4096,4096] + "
                        "[96,4096,11008] bf16 (BASELINE config 4), the whole model",
            "ms_per_update_1gpu": ms4_1,
            "tflops_1gpu": flops4 / (ms4_1 * 1e-3) / 1e12 if ms4_1 else None}
    if world > 1:
        mine = partition_items([float(nominal_flops(*k)) for k in kinds], world)[rank]
        xs = cfg4_batches(mine, 44 + rank)
        cfg4_update(xs)
        ms4_n = _timed_updates(lambda: cfg4_update(xs), 2, world, device, sync_all)
        cfg4.update({"parallelism": f"batch-sharded x{world} (FLOP-balanced, no data-path "
                                    "collective)",
                     "ms_per_update": ms4_n, "tflops": flops4 / (ms4_n * 1e-3) / 1e12,
                     "efficiency": (ms4_1 / (world * ms4_n)) if ms4_1 else None})
        del xs
        torch.cuda.empty_cache()
    out["cfg4"] = cfg4

    # ---- parity: a [1024, 8192] column-sharded 5-step result against the
    # single-GPU polar_step chain and an fp32 evaluation of the reference
    # formula (tests/test_polar_step.py:22-28), with the bound of the
    # multi-GPU test: elementwise within rtol = atol = 6e-2 of the single-GPU
    # chain, and a relative Frobenius error against fp32 at most 1.5x the
    # single GPU's + 1e-3.
    if world > 1:
        mp_, np_ = PARITY_SHAPE
        gen.manual_seed(77)  # the same matrix on every rank
        x = torch.randn((mp_, np_), generator=gen, device=device).to(torch.bfloat16)
        x = x / (x.norm() * 1.01 + 1e-6)
        cols = column_range(np_, rank, world)
        drv = ColumnShardedPolar(mp_, device, packed=True)
        y_local = drv.run(x[:, cols.start:cols.stop].contiguous(), COEFFICIENTS).contiguous()
        parts = [torch.empty_like(y_local) for _ in range(world)]
        dist.all_gather(parts, y_local)
        if rank == 0:
            y = torch.cat(parts, dim=1).double()
            single = x.unsqueeze(0)
            for a, b, c in COEFFICIENTS:
                single = pkg.polar_step(single, a, b, c)
            single = single.squeeze(0).double()
            tf32 = torch.backends.cuda.matmul.allow_tf32
            torch.backends.cuda.matmul.allow_tf32 = False
            ref = x.float()
            for a, b, c in COEFFICIENTS:
                g = ref @ ref.mT
                ref = a * ref + (b * g + c * (g @ g)) @ ref
            torch.backends.cuda.matmul.allow_tf32 = tf32
            ref = ref.double()

            def rel_fro(v):
                return float((v - ref).norm() / ref.norm())

            d = (y - single).abs()
            within = bool((d <= 6e-2 + 6e-2 * single.abs()).all())
            rs, r1 = rel_fro(y), rel_fro(single)
            out["parity"] = {
                "shape": list(PARITY_SHAPE), "steps": len(COEFFICIENTS), "ranks": world,
                "path": "column-sharded, packed reduce-scatter / all-gathers",
                "max_abs_vs_single_gpu": float(d.max()),
                "max_abs_vs_fp32": float((y - ref).abs().max()),
                "mean_abs_vs_fp32": float((y - ref).abs().mean()),
                "rel_fro_vs_fp32": rs, "rel_fro_single_gpu_vs_fp32": r1,
                "bound": "allclose(single, rtol=atol=6e-2) and rel_fro <= 1.5 x single + 1e-3",
                "ok": within and rs <= 1.5 * r1 + 1e-3,
            }
        del drv, x, y_local, parts
        torch.cuda.empty_cache()
        sync_all()
    return out


# --------------------------------------------------------------------- arms
def reference_large_rate(workload: str):
    """The reference formula on the host CPU for configs 4 and 5, too large to
    run whole: one matrix of each shape, extrapolated by count (config 4: the
    5-step loop on one [4096,4096] and one [4096,11008] matrix, x128 and x96;
    config 5: one step of the [8192,65536] matrix, x5).  Returns (TFLOP/s,
    ms per update, threads, sample description)."""
    import torch

    from oracle.polar_oracle import make_input, nominal_flops, reference_formula

    threads = os.cpu_count() or 1
    torch.set_num_threads(threads)
    if workload == "cfg4":
        parts = [((4096, 4096), 128, COEFFICIENTS), ((4096, 11008), 96, COEFFICIENTS)]
        what = "the 5-step loop on one [4096,4096] and one [4096,11008] matrix, x128 and x96"
    else:
        parts = [((8192, 65536), 5, COEFFICIENTS[:1])]
        what = "one step of the [8192,65536] matrix, x5"
    flops = 0.0
    ms = 0.0
    for (m, n), count, rows in parts:
        x = make_input((1, m, n), seed=0)
        t0 = time.perf_counter()
        reference_formula(x, rows)
        ms += count * (time.perf_counter() - t0) * 1e3
        flops += count * len(rows) * nominal_flops(m, n)
        del x
    return flops / (ms * 1e-3) / 1e12, ms, threads, (
        f"{what} (bf16, one timed run each, no warm-up), extrapolated by count")


def run_reference(args):
    rank, world, _ = dist_env()
    if rank != 0:
        return
    global BATCH, M, N
    workload = args.workload
    if workload in ("shape", "express"):
        BATCH, M, N = (int(v) for v in args.shape.split(","))
    if workload in ("cfg4", "cfg5"):
        rate, ms, threads, sample = reference_large_rate(workload)
        metric = f"{workload} effective TFLOP/s (nominal 4M^2N+2M^3 per matrix per step)"
        config = large_workload_config(workload, args.gpus)
    else:
        rows = len(COEFFICIENTS) if workload in ("cfg3", "express") else 1
        rate, threads, sample = cpu_reference_rate(args.steps, args.warmup, budget_s=120.0,
                                                   rows=rows)
        ms = rows * BATCH * nominal_flops_per_matrix(M, N) / (rate * 1e12) * 1e3
        metric = metric_name(workload)
        config = workload_config(workload, args.gpus)
    line = {
        "impl": "reference",
        "metric": metric,
        "value": rate, "unit": "TFLOP/s", "n_gpus": args.gpus, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": ms, "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "bf16", "data": "synthetic",
        "config": config,
        "timing": "host CPU (rank 0 only, every thread): the reference's PyTorch formula on a "
                  "bounded sample of the workload, median of the timed steps",
        "cpu_baseline": {"value": rate, "unit": "TFLOP/s", "cores": threads, "kind": "port",
                         "sample": sample},
        "e2e": {"value": rate, "unit": "TFLOP/s", "h2d_bytes_per_step": 0,
                "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


def run_ours(args):
    import torch
    import torch.distributed as dist

    import muon_fusion_ascend950_b200 as pkg
    from muon_fusion_ascend950_b200.capi import capi

    rank, world, local = dist_env()
    if world != args.gpus:
        raise SystemExit(f"--gpus {args.gpus} but WORLD_SIZE={world}")
    device = torch.device("cuda", local)
    torch.cuda.set_device(device)
    if world > 1:
        from datetime import timedelta

        dist.init_process_group("nccl", device_id=device, timeout=timedelta(seconds=120))
    api = capi()
    global BATCH, M, N
    if args.workload in ("shape", "express"):
        BATCH, M, N = (int(v) for v in args.shape.split(","))
    a, b, c = COEFFICIENTS[0]
    rows = COEFFICIENTS if args.workload in ("cfg3", "express") else COEFFICIENTS[:1]
    flops_step = len(rows) * BATCH * nominal_flops_per_matrix(M, N)

    def full_step(x):
        if args.workload == "express":
            # the five steps as one call (muon_polar_steps_sm100: one fused
            # launch for small matrices)
            return pkg.polar_express(x, rows, normalize=False)
        for ra, rb, rc in rows:
            x = pkg.polar_step(x, ra, rb, rc)
        return x

    # inputs generated on the device (seeded per rank and set), normalised as
    # the reference test does; enough rotating sets that one cycle touches
    # more than three times the L2 (8 sets at [8,512,2048])
    global ROTATION
    ROTATION = rotation_sets(BATCH, M, N)
    gen = torch.Generator(device=device)
    xs = []
    for i in range(ROTATION):
        gen.manual_seed(1000 * rank + i)
        x = torch.randn((BATCH, M, N), generator=gen, device=device, dtype=torch.float32)
        x = x.to(torch.bfloat16)
        xs.append(x / (x.norm(dim=(-2, -1), keepdim=True) * 1.01 + 1e-6))
    stream = torch.cuda.Stream(device)

    def sync_all():
        torch.cuda.synchronize(device)
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize(device)

    # ---- CUDA graphs, one step each, through the public API
    graphs, outs = [], []
    with torch.cuda.stream(stream):
        for x in xs:  # eager warm-up of every set before capture
            full_step(x)
    torch.cuda.synchronize(device)
    launches_before = api.launch_count()
    for x in xs:
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g, stream=stream):
            outs.append(full_step(x))
        graphs.append(g)
    launches_per_step = (api.launch_count() - launches_before) // ROTATION
    # One graph of ROTATION consecutive steps (one per input set), as a
    # training loop captures its optimizer step: inside it the steps are
    # chained by programmatic dependent launch like the kernels of one step.
    cycle = torch.cuda.CUDAGraph()
    with torch.cuda.graph(cycle, stream=stream):
        for x in xs:
            outs.append(full_step(x))

    def run_steps(k, single=False):
        """k steps: whole cycles, then single-step graphs for the rest."""
        q, r = (0, k) if single else divmod(k, ROTATION)
        for _ in range(q):
            cycle.replay()
        for i in range(r):
            graphs[i % ROTATION].replay()

    with torch.cuda.stream(stream):
        run_steps(args.warmup)
        # keep the GPU busy long enough for the clocks to settle
        t_end = time.perf_counter() + 0.3
        while time.perf_counter() < t_end:
            run_steps(ROTATION)
    sync_all()

    def timed(single):
        start = torch.cuda.Event(enable_timing=True)
        stop = torch.cuda.Event(enable_timing=True)
        sync_all()
        with torch.cuda.stream(stream):
            start.record(stream)
            run_steps(args.steps, single)
            stop.record(stream)
        stop.synchronize()
        sync_all()
        ms = start.elapsed_time(stop)
        if world > 1:
            t = torch.tensor([ms], device=device, dtype=torch.float64)
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
            ms = float(t.item())
        return ms

    sampler = ClockSampler(local)
    with sampler:
        elapsed_ms = timed(False)
    ms_per_step = elapsed_ms / args.steps
    value = world * flops_step * args.steps / (elapsed_ms * 1e-3) / 1e12
    # the same K steps as one graph replay each (a graph boundary between steps)
    single_graph_ms = timed(True)

    # ---- per-kernel CUDA-event timing (same buffers, kernels timed alone)
    # The C ABI takes what the operator hands it: M <= N (transposed) and a
    # row stride that is a multiple of 8 (zero-padded columns).
    def kernel_input(x):
        if x.shape[-2] > x.shape[-1]:
            x = x.mT.contiguous()
        if x.shape[-1] % 8:
            xp = x.new_zeros((*x.shape[:-1], -(-x.shape[-1] // 16) * 16))
            xp[..., : x.shape[-1]] = x
            x = xp
        return x

    kn = min(M, N)
    xs_k = [kernel_input(x) for x in xs]
    mp = api.padded_rows(kn)
    gram = torch.empty((BATCH, mp, mp), dtype=torch.bfloat16, device=device)
    poly = torch.empty_like(gram)
    y = torch.empty_like(xs_k[0])
    scratch = api.new_scratch(BATCH, kn, max(M, N), device=device, stream=stream)
    kernel_iters = max(50, min(args.steps, 1000))

    def time_kernel(fn):
        with torch.cuda.stream(stream):
            for i in range(5):
                fn(i)
            e0 = torch.cuda.Event(enable_timing=True)
            e1 = torch.cuda.Event(enable_timing=True)
            e0.record(stream)
            for i in range(kernel_iters):
                fn(i)
            e1.record(stream)
        e1.synchronize()
        return e0.elapsed_time(e1) / kernel_iters * 1e3  # us

    nv = max(M, N)
    with torch.cuda.stream(stream):
        api.gram(xs_k[0], gram, n=nv, scratch=scratch, stream=stream)
        api.poly(gram, poly, b, c, scratch=scratch, stream=stream)
    us = {
        "gram": time_kernel(lambda i: api.gram(xs_k[i % ROTATION], gram, n=nv, scratch=scratch,
                                               stream=stream)),
        "poly": time_kernel(lambda i: api.poly(gram, poly, b, c, scratch=scratch,
                                               stream=stream)),
        "apply": time_kernel(lambda i: api.apply(poly, xs_k[i % ROTATION], y, a, n=nv,
                                                 stream=stream)),
    }
    kernel_flops = {"gram": BATCH * 2 * kn * kn * nv, "poly": BATCH * 2 * kn ** 3,
                    "apply": BATCH * 2 * kn * kn * nv}
    dominant = max(us, key=us.get)
    peak, peak_kind = measured_peaks()
    achieved = kernel_flops[dominant] / (us[dominant] * 1e-6) / 1e12
    traffic_info = profiled_traffic()
    traffic = None
    if traffic_info and dominant in traffic_info.get("kernels", {}):
        traffic = traffic_info["kernels"][dominant].get("dram_bytes_per_launch")
    roofline = {
        "bound": "tensor", "kernel": dominant, "achieved": achieved, "peak": peak,
        "unit": "TFLOP/s", "frac": achieved / peak, "traffic": traffic,
        "peak_source": f"{peak_kind} bf16 dense (burst)",
        "kernel_us": us,
        "kernel_tflops": {k: kernel_flops[k] / (us[k] * 1e-6) / 1e12 for k in us},
    }

    # ---- host-inclusive wall clock of eager public-API calls (the way the
    # reference's README times a step): back-to-back calls, and one call
    # followed by a synchronize
    host_iters = max(20, min(args.steps, 500))
    with torch.cuda.stream(stream):
        for i in range(5):
            full_step(xs[i % ROTATION])
        torch.cuda.synchronize(device)
        t0 = time.perf_counter()
        for i in range(host_iters):
            full_step(xs[i % ROTATION])
        torch.cuda.synchronize(device)
        eager_us = (time.perf_counter() - t0) / host_iters * 1e6
        lat = []
        for i in range(50):
            t0 = time.perf_counter()
            full_step(xs[i % ROTATION])
            torch.cuda.synchronize(device)
            lat.append(time.perf_counter() - t0)
    host_inclusive = {"eager_us_per_step": eager_us,
                      "sync_call_us_median": sorted(lat)[len(lat) // 2] * 1e6,
                      "calls": host_iters}

    # ---- end to end through the public API with host buffers.  Every step
    # copies its input from pinned host memory and its result back; the
    # copies run on their own streams, so the input of step i+1 and the
    # result of step i-1 cross PCIe while step i computes (three device input
    # buffers and three pinned result buffers: with two, the host thread
    # measurably stalled in the allocators).
    e2e_steps = max(1, min(args.e2e_steps, args.steps))
    nbuf = 3
    host_in = [x.cpu().pin_memory() for x in xs]
    host_out = [torch.empty(xs[0].shape, dtype=torch.bfloat16).pin_memory()
                for _ in range(nbuf)]
    dev_in = [torch.empty_like(xs[0]) for _ in range(nbuf)]
    h2d, d2h = torch.cuda.Stream(device), torch.cuda.Stream(device)

    def e2e_run(n, e0=None, e1=None):
        consumed = [None] * nbuf  # compute done with dev_in[j]
        if e0 is not None:
            e0.record(stream)
            h2d.wait_event(e0)
        read = None
        for i in range(n):
            j = i % nbuf
            with torch.cuda.stream(h2d):
                if consumed[j] is not None:
                    h2d.wait_event(consumed[j])
                dev_in[j].copy_(host_in[i % ROTATION], non_blocking=True)
                filled = torch.cuda.Event()
                filled.record(h2d)
            with torch.cuda.stream(stream):
                stream.wait_event(filled)
                out = full_step(dev_in[j])
                done = torch.cuda.Event()
                done.record(stream)
                consumed[j] = done
            with torch.cuda.stream(d2h):
                d2h.wait_event(done)
                host_out[j].copy_(out, non_blocking=True)
                out.record_stream(d2h)
                read = torch.cuda.Event()
                read.record(d2h)
        stream.wait_event(read)
        if e1 is not None:
            e1.record(stream)

    # warm-up long enough for the caching allocators (device outputs, pinned
    # staging) to hold every block the pipeline keeps in flight
    e2e_run(20)
    sync_all()
    # median of three timed runs: the host thread that issues the copies and
    # calls is itself part of this number
    e2e_runs = []
    gc.collect()
    gc.disable()
    try:
        for _ in range(3):
            e0 = torch.cuda.Event(enable_timing=True)
            e1 = torch.cuda.Event(enable_timing=True)
            e2e_run(e2e_steps, e0, e1)
            e1.synchronize()
            e2e_runs.append(e0.elapsed_time(e1))
    finally:
        gc.enable()
    e2e_ms = sorted(e2e_runs)[1]
    if world > 1:
        t = torch.tensor([e2e_ms], device=device, dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        e2e_ms = float(t.item())
    e2e_value = world * flops_step * e2e_steps / (e2e_ms * 1e-3) / 1e12
    step_bytes = xs[0].numel() * xs[0].element_size()

    # ---- CPU baseline (rank 0, N=1 only)
    cpu_baseline = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        rate, threads, sample = cpu_reference_rate(3, 1, budget_s=20.0, rows=len(rows))
        cpu_baseline = {"value": rate, "unit": "TFLOP/s", "cores": threads, "kind": "port",
                        "sample": sample}

    for g in graphs:
        g.reset()
    cycle.reset()
    sharded = None
    if args.sharded == "on" or (args.sharded == "auto" and args.workload == "cfg1"):
        del xs, xs_k, gram, poly, y, scratch, host_in, host_out, dev_in
        gc.collect()
        torch.cuda.empty_cache()
        sharded = run_sharded(rank, world, device, sync_all)
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()
    if rank != 0:
        return
    line = {
        "metric": metric_name(args.workload),
        "value": value,
        "unit": "TFLOP/s",
        "n_gpus": world,
        "steps": args.steps,
        "warmup": args.warmup,
        "ms_per_step": ms_per_step,
        "us_per_step": ms_per_step * 1e3,
        "higher_is_better": True,
        "scaling": "weak",
        "vs_baseline": None,
        "dtype": "bf16",
        "data": "synthetic",
        "pct_of_bf16_peak": 100.0 * value / (world * peak),
        "config": workload_config(args.workload, world),
        "timing": (f"CUDA graphs of {ROTATION} consecutive public-API steps (one per input set; "
                   "single-step graphs for the remainder of K), CUDA events, max over ranks"),
        "roofline": roofline,
        "cpu_baseline": cpu_baseline,
        "e2e": {"value": e2e_value, "unit": "TFLOP/s", "steps": e2e_steps,
                "h2d_bytes_per_step": step_bytes, "d2h_bytes_per_step": step_bytes,
                "ms_per_step": e2e_ms / e2e_steps,
                "ms_per_step_runs": [v / e2e_steps for v in e2e_runs],
                "copies": "pinned host buffers; H2D of step i+1 and D2H of step i-1 on "
                          "their own streams while step i computes"},
        "us_per_step_single_step_graphs": single_graph_ms / args.steps * 1e3,
        "host_inclusive": host_inclusive,
        "clocks": sampler.summary(),
        "gpu_launches": launches_per_step * args.steps,
    }
    if sharded is not None:
        line["sharded"] = sharded
    print(json.dumps(line), flush=True)
    parity = (sharded or {}).get("parity")
    if parity is not None and not parity["ok"]:
        raise SystemExit("column-sharded parity check failed: " + json.dumps(parity))


def run_large(args):
    """Configs 4 and 5: one Muon update (the 5-step loop) per timed step over
    a fixed total problem (strong scaling), eager launches (the host issues a
    few hundred microseconds of launches per ~0.1-1 s step)."""
    import torch
    import torch.distributed as dist

    import muon_fusion_ascend950_b200 as pkg
    from muon_fusion_ascend950_b200.capi import capi
    from muon_fusion_ascend950_b200.distributed import (
        ColumnShardedPolar, column_range, nominal_flops, partition_items)

    rank, world, local = dist_env()
    if world != args.gpus:
        raise SystemExit(f"--gpus {args.gpus} but WORLD_SIZE={world}")
    device = torch.device("cuda", local)
    torch.cuda.set_device(device)
    if world > 1:
        from datetime import timedelta

        dist.init_process_group("nccl", device_id=device, timeout=timedelta(seconds=300))
    api = capi()
    gen = torch.Generator(device=device)
    gen.manual_seed(rank)

    def normalised(shape):
        x = torch.randn(shape, generator=gen, device=device, dtype=torch.float32)
        x = x.to(torch.bfloat16)
        return x / (x.norm(dim=(-2, -1), keepdim=True) * 1.01 + 1e-6)

    if args.workload == "cfg4":
        # 32 layers x (q, k, v, o) = 128 [4096,4096]; 32 x (gate, up, down^T)
        # = 96 [4096,11008]; FLOP-balanced across ranks
        kinds = [(4096, 4096)] * 128 + [(4096, 11008)] * 96
        mine = partition_items([float(nominal_flops(*k)) for k in kinds], world)[rank]
        n_att = sum(1 for i in mine if kinds[i] == (4096, 4096))
        n_ffn = len(mine) - n_att
        batches = [normalised((cnt, 4096, n)) for cnt, n in ((n_att, 4096), (n_ffn, 11008))
                   if cnt > 0]
        job_flops = 5 * sum(nominal_flops(*k) for k in kinds)

        def step():
            for x in batches:
                y = x
                for a, b, c in COEFFICIENTS:
                    y = pkg.polar_step(y, a, b, c)

        config = large_workload_config("cfg4", world)
    else:
        m, n = 8192, 65536
        cols = column_range(n, rank, world)
        x_local = torch.randn((m, len(cols)), generator=gen, device=device,
                              dtype=torch.float32).to(torch.bfloat16)
        sq = (x_local.float() ** 2).sum().reshape(1)
        if world > 1:
            dist.all_reduce(sq)
        x_local = (x_local / (sq.sqrt() * 1.01 + 1e-6)).to(torch.bfloat16)
        driver = ColumnShardedPolar(m, device, shard_poly=args.poly == "sharded",
                                    overlap_bands=args.overlap_bands, sm_reserve=args.sm_reserve)
        job_flops = 5 * nominal_flops(m, n)

        def step():
            driver.run(x_local, COEFFICIENTS)

        config = large_workload_config(
            "cfg5", world, column_path="packed" if driver.packed else "all-reduce",
            bands=len(driver.bands), sm_reserve=args.sm_reserve,
            poly_slabs=driver.poly_slab is not None)

    def sync_all():
        torch.cuda.synchronize(device)
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize(device)

    launches0 = api.launch_count()
    step()
    sync_all()
    launches_per_step = api.launch_count() - launches0
    for _ in range(max(0, args.warmup - 1)):
        step()
    sync_all()
    sampler = ClockSampler(local)
    start = torch.cuda.Event(enable_timing=True)
    stop = torch.cuda.Event(enable_timing=True)
    with sampler:
        sync_all()
        start.record()
        for _ in range(args.steps):
            step()
        stop.record()
        stop.synchronize()
        sync_all()
    elapsed_ms = start.elapsed_time(stop)
    if world > 1:
        t = torch.tensor([elapsed_ms], device=device, dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        elapsed_ms = float(t.item())
        dist.barrier()
        dist.destroy_process_group()
    if rank != 0:
        return
    value = job_flops * args.steps / (elapsed_ms * 1e-3) / 1e12
    peak, peak_kind = measured_peaks()
    line = {
        "metric": f"{args.workload} effective TFLOP/s (nominal 4M^2N+2M^3 per matrix per step)",
        "value": value, "unit": "TFLOP/s", "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": elapsed_ms / args.steps,
        "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "bf16",
        "data": "synthetic",
        "pct_of_bf16_peak": 100.0 * value / (world * peak),
        "config": config,
        "timing": "eager public API / column-sharded driver, CUDA events, max over ranks",
        "roofline": {"bound": "tensor", "kernel": "whole step", "achieved": value / world,
                     "peak": peak, "unit": "TFLOP/s", "frac": value / world / peak,
                     "traffic": None, "peak_source": f"{peak_kind} bf16 dense (burst)"},
        "cpu_baseline": None,
        "e2e": None,
        "clocks": sampler.summary(),
        "gpu_launches": launches_per_step * args.steps,
    }
    print(json.dumps(line), flush=True)


def main():
    args = parse_args()
    if args.impl == "reference":
        run_reference(args)
    elif args.workload in ("cfg4", "cfg5"):
        run_large(args)
    else:
        run_ours(args)


if __name__ == "__main__":
    main()
