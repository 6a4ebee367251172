"""Multi-GPU drivers of the Polar Express step (one process per GPU).

The reference has no distributed code (no HCCL or collective anywhere).  The
workloads it is benchmarked on shard in two ways:

* **Batch sharding** (independent matrices: configs 1, 3 and 4).  Each rank
  owns a FLOP-balanced subset of the matrices and runs the local step on
  them; there is no collective on the data path.  `partition_items` balances
  by nominal FLOPs (4 M^2 N + 2 M^3 per matrix).
* **Column sharding** (one large matrix: config 5).  Rank r owns the column
  slab X[:, r*N/G : (r+1)*N/G] for the whole iteration.  Per step, by
  default (`packed`), on the packed upper triangle of the symmetric
  matrices (256 x 256 units, (d+1)/(2d) of the full matrix's bytes):
    1. partial Gram G_r = X_r X_r^T in fp32, written as packed units
       (kernel 1, muon_polar_gram_f32_packed_sm100),
    2. one reduce-scatter (sum, fp32) of the units over NCCL: rank r
       receives the summed units of its slab [r U/G, (r+1) U/G),
    3. A = bf16(sum) of the slab (cast kernel: the one rounding of A, as on
       one GPU), then an all-gather (bf16) of the packed A and an unpack to
       the full symmetric matrix,
    4. P = b A + c A A on the rank's units only (kernel 2,
       muon_polar_poly_packed_sm100), an all-gather (bf16) of the packed P
       and an unpack,
    5. Y_r = a X_r + P X_r on the local slab (kernel 3).
  Against an fp32 all-reduce of the full Mp x Mp Gram and a gather of P row
  slabs, the collectives move about 3/8 of the bytes, and kernel 2 computes
  each unit once instead of both triangles.  `packed=False` keeps that
  earlier scheme: the all-reduce -- or, with `overlap_bands`, kernel 1 band
  by band over the rows (muon_polar_gram_f32_band_sm100, leaving
  `sm_reserve` SMs free), each band all-reduced on a second stream while the
  next band computes -- then A = bf16(sum), and P replicated or (shard_poly)
  as row slabs [r Mp/G, (r+1) Mp/G) followed by an all-gather.
  Either way the result equals the single-GPU step up to the fp32 summation
  order of the Gram (A is rounded to bf16 once, after the sum, as on one
  GPU).

Kernels are reached through a backend object with the methods of
`capi.CAPI` (gram_f32, gram_f32_packed, cast_f32_bf16, unpack_sym,
poly_packed, poly, apply, ...).  The default backend is
the CUDA C ABI; there is no CPU fallback -- tests on CPU pass their own
backend explicitly.
"""
from __future__ import annotations

import heapq
from typing import List, Optional, Sequence

import torch
import torch.distributed as dist


def nominal_flops(m: int, n: int) -> int:
    """Nominal FLOPs of one step on one [m, n] matrix (M <= N after the
    transpose policy): 4 M^2 N + 2 M^3."""
    m, n = min(m, n), max(m, n)
    return 4 * m * m * n + 2 * m ** 3


def partition_items(costs: Sequence[float], world: int) -> List[List[int]]:
    """Assigns item indices to `world` ranks, balancing the summed cost
    (longest-processing-time greedy: items by decreasing cost, each to the
    currently lightest rank; ties to the lowest rank).  Every item lands on
    exactly one rank; each rank's list is in increasing index order."""
    if world <= 0:
        raise ValueError("world must be positive")
    order = sorted(range(len(costs)), key=lambda i: (-costs[i], i))
    heap = [(0.0, r) for r in range(world)]
    heapq.heapify(heap)
    parts: List[List[int]] = [[] for _ in range(world)]
    for i in order:
        load, r = heapq.heappop(heap)
        parts[r].append(i)
        heapq.heappush(heap, (load + costs[i], r))
    return [sorted(p) for p in parts]


def column_range(n: int, rank: int, world: int, align: int = 8) -> range:
    """Columns of rank `rank` when n columns are cut into `world` slabs whose
    boundaries are multiples of `align` (TMA needs 16-byte row strides for a
    slab stored on its own).  The last slab takes the remainder."""
    if world <= 0 or not 0 <= rank < world:
        raise ValueError("bad rank/world")
    per = -(-n // world)
    per = -(-per // align) * align
    start = min(n, rank * per)
    stop = n if rank == world - 1 else min(n, (rank + 1) * per)
    return range(start, stop)


def gram_bands(mp: int, bands: int) -> List[tuple]:
    """Row bands (begin, count) covering [0, mp), multiples of 256 rows, as
    equal as the 256-row granularity allows (at most `bands` of them)."""
    tiles = mp // 256
    bands = max(1, min(bands, tiles))
    out = []
    begin = 0
    for i in range(bands):
        end = (i + 1) * tiles // bands
        if end > begin:
            out.append((begin * 256, (end - begin) * 256))
        begin = end
    return out


class ColumnShardedPolar:
    """Polar Express steps on a matrix whose columns are split across the
    ranks of `group` (see the module docstring).  Buffers for the replicated
    Mp x Mp Gram / polynomial are allocated once per instance.  With
    `shard_poly`, kernel 2 is split into row slabs across the ranks (when
    Mp divides into equal slabs of 256-row multiples; otherwise replicated).
    With `overlap_bands` > 1 the Gram's all-reduce runs band by band beside
    the computation of the next band (the bands' kernels leave `sm_reserve`
    SMs to the collective)."""

    def __init__(self, m: int, device, group=None, backend=None, shard_poly: bool = False,
                 overlap_bands: int = 0, sm_reserve: int = 16, packed: bool = True):
        if backend is None:
            from .capi import capi

            backend = capi()
        self.backend = backend
        self.group = group
        self.m = m
        self.mp = backend.padded_rows(m)
        self.device = torch.device(device)
        world = dist.get_world_size(group) if dist.is_initialized() else 1
        rank = dist.get_rank(group) if dist.is_initialized() else 0
        self.poly_slab = None
        if shard_poly and world > 1 and self.mp % (256 * world) == 0:
            rows = self.mp // world
            self.poly_slab = (rank * rows, rows)
        self.bands = gram_bands(self.mp, overlap_bands) if overlap_bands > 1 and world > 1 else []
        self.sm_reserve = sm_reserve
        self.world, self.rank = world, rank
        self.packed = bool(packed) and world > 1 and not self.bands
        if self.packed:
            units = backend.packed_units(m)
            per = -(-units // world)
            self.unit_slab = (rank * per, max(0, min(per, units - rank * per)))
            unit = (256, 256)
            # the last slab may end in padding units: zero in the partial Gram
            # (never written), unused in A and P
            self.packed_f32 = torch.zeros((per * world, *unit), dtype=torch.float32,
                                          device=self.device)
            self.slab_f32 = torch.empty((per, *unit), dtype=torch.float32, device=self.device)
            self.slab_bf16 = torch.empty((per, *unit), dtype=torch.bfloat16, device=self.device)
            self.packed_a = torch.empty((per * world, *unit), dtype=torch.bfloat16,
                                        device=self.device)
            self.packed_p = torch.zeros((per * world, *unit), dtype=torch.bfloat16,
                                        device=self.device)
            self.poly_slab = None
        self.comm = (torch.cuda.Stream(self.device)
                     if self.bands and self.device.type == "cuda" else None)
        shape = (1, self.mp, self.mp)
        self.gram_f32 = (torch.empty(shape, dtype=torch.float32, device=self.device)
                         if not self.packed else None)
        self.gram = torch.empty(shape, dtype=torch.bfloat16, device=self.device)
        self.poly = torch.empty(shape, dtype=torch.bfloat16, device=self.device)

    def step(self, x_local: torch.Tensor, a: float, b: float, c: float,
             out: Optional[torch.Tensor] = None) -> torch.Tensor:
        """One step on this rank's slab x_local [m, n_local] (bf16, row
        stride a multiple of 8); returns the slab of Y."""
        if x_local.dim() != 2 or x_local.shape[0] != self.m:
            raise ValueError(f"x_local must be [{self.m}, n_local], got {tuple(x_local.shape)}")
        x3 = x_local.contiguous().unsqueeze(0)
        y3 = torch.empty_like(x3) if out is None else out.view(1, *out.shape[-2:])
        if self.packed:
            self._packed_gram_poly(x3, b, c)
            self.backend.apply(self.poly, x3, y3, a)
            return y3.squeeze(0)
        if self.bands:
            self._gram_reduce_bands(x3)
        else:
            self.backend.gram_f32(x3, self.gram_f32)
            if dist.is_initialized() and dist.get_world_size(self.group) > 1:
                dist.all_reduce(self.gram_f32, op=dist.ReduceOp.SUM, group=self.group)
        self.backend.cast_f32_bf16(self.gram_f32, self.gram)
        if self.poly_slab is None:
            self.backend.poly(self.gram, self.poly, b, c)
        else:
            begin, rows = self.poly_slab
            self.backend.poly_rows(self.gram, self.poly, b, c, begin, rows)
            flat = self.poly.view(-1)
            per = rows * self.mp
            dist.all_gather_into_tensor(flat, flat[begin * self.mp: begin * self.mp + per],
                                        group=self.group)
        self.backend.apply(self.poly, x3, y3, a)
        return y3.squeeze(0)

    def _packed_gram_poly(self, x3: torch.Tensor, b: float, c: float) -> None:
        """A and P on the packed upper triangle (module docstring, steps
        1-4).  Every rank issues the same three collectives in order."""
        be = self.backend
        # the kernels' layout is [batch][units][256][256]: batch 1 here
        be.gram_f32_packed(x3, self.packed_f32.unsqueeze(0))
        dist.reduce_scatter_tensor(self.slab_f32, self.packed_f32, op=dist.ReduceOp.SUM,
                                   group=self.group)
        be.cast_f32_bf16(self.slab_f32, self.slab_bf16)
        dist.all_gather_into_tensor(self.packed_a, self.slab_bf16, group=self.group)
        be.unpack_sym(self.packed_a.unsqueeze(0), self.gram)
        begin, count = self.unit_slab
        if count > 0:
            be.poly_packed(self.gram, self.packed_p.unsqueeze(0), b, c, begin, count)
        per = self.slab_f32.shape[0]
        mine = self.packed_p[self.rank * per:(self.rank + 1) * per]
        dist.all_gather_into_tensor(self.packed_p, mine, group=self.group)
        be.unpack_sym(self.packed_p.unsqueeze(0), self.poly)

    def collective_bytes(self) -> dict:
        """Bytes each rank hands to the collectives per step (NCCL message
        sizes, before any algorithm-dependent factor)."""
        if not self.packed:
            full = self.mp * self.mp
            out = {"all_reduce_fp32": 4 * full}
            if self.poly_slab is not None:
                out["all_gather_bf16"] = 2 * full
            return out
        n = self.packed_f32.numel()
        return {"reduce_scatter_fp32": 4 * n, "all_gather_bf16": 2 * 2 * n}

    def _gram_reduce_bands(self, x3: torch.Tensor) -> None:
        """Kernel 1 band by band; band i's rows are complete after its call
        and are summed across the ranks while band i + 1 computes.  Every
        rank issues the same all-reduces in the same order."""
        cur = torch.cuda.current_stream(self.device) if self.comm is not None else None
        for begin, count in self.bands:
            self.backend.gram_f32_band(x3, self.gram_f32, begin, count, self.sm_reserve)
            rows = self.gram_f32[:, begin:begin + count]  # contiguous rows
            if self.comm is None:
                dist.all_reduce(rows, op=dist.ReduceOp.SUM, group=self.group)
                continue
            done = torch.cuda.Event()
            done.record(cur)
            with torch.cuda.stream(self.comm):
                self.comm.wait_event(done)
                dist.all_reduce(rows, op=dist.ReduceOp.SUM, group=self.group)
        if self.comm is not None:
            cur.wait_stream(self.comm)

    def run(self, x_local: torch.Tensor, coefficients) -> torch.Tensor:
        """The caller-side loop over (a, b, c) rows, slab kept local."""
        y = x_local
        for a, b, c in coefficients:
            y = self.step(y, a, b, c)
        return y


def batch_sharded_steps(xs: Sequence[torch.Tensor], coefficients, rank: int, world: int,
                        step=None) -> dict:
    """Runs the caller-side loop on this rank's share of the matrices `xs`
    (a list of [M, N] or [B, M, N] tensors, all ranks passing the same list
    description).  Returns {index: result} for the items this rank owns.
    No collective is issued."""
    if step is None:
        from .ops import polar_step as step
    costs = [float(nominal_flops(x.shape[-2], x.shape[-1]) * (x.shape[0] if x.dim() == 3 else 1))
             for x in xs]
    mine = partition_items(costs, world)[rank]
    results = {}
    for i in mine:
        y = xs[i]
        for a, b, c in coefficients:
            y = step(y, a, b, c)
        results[i] = y
    return results


__all__ = [
    "nominal_flops",
    "partition_items",
    "column_range",
    "ColumnShardedPolar",
    "gram_bands",
    "batch_sharded_steps",
]
