// muon_polar_sm100.cu -- B200 (sm_100a) kernels and C ABI of one Polar
// Express step:  A = X.X^T,  P = b.A + c.A.A,  Y = a.X + P.X.
//
// One persistent, warp-specialised tcgen05 GEMM template serves all three
// stages; they differ in which operands TMA brings in and in the epilogue
// fused onto the TMEM accumulator:
//
//   kind        A operand (K-major)   B operand               epilogue
//   kGramBf16   X rows tm             X rows tn  (K-major)    bf16(acc), tile + mirror
//   kGramF32    X rows tm             X rows tn  (K-major)    fp32 acc,  tile + mirror
//   kPoly       A rows tm             A rows tn  (K-major)    bf16(b*A + c*acc), tile + mirror
//   kApply      P rows tm             X[k, n-block] (MN-major) bf16(bf16(acc) + bf16(alpha*X))
//
// and, for M > N without transposed copies (the step of X^T, returned in
// X's layout: A = X^T.X, Y = a.X + X.P, P symmetric):
//   kGramT      X[k, tm-block] (MN)   X[k, tn-block] (MN)     as kGramBf16
//   kApplyT     X rows tm             P rows tn  (K-major)    as kApply
//
// Two engines of the same kernel (polar_tile_kernel<KIND, PAIR>): 256 x 256
// tiles on a tcgen05 CTA pair (PAIR = 2) and 128 x 128 tiles on one CTA
// (PAIR = 1), chosen by problem size.  CTA layout (320 threads): warp 0 lane
// 0 issues TMA loads into a ring of shared-memory stages; warp 1 owns the
// tensor memory and its lane 0 (leader CTA) issues tcgen05.mma into one of
// two TMEM accumulators; warps 2-9 drain the other accumulator
// (tcgen05.ld), apply the epilogue and store with TMA, so the epilogue of
// tile i overlaps the main loop of tile i+1.  Every wait is bounded in
// wall-clock time; a kernel that gives up records a watchdog bit and returns.
//
// Reference behaviour restated here (Ascend 950PR AscendC kernels):
//   symmetric upper-tile Gram + mirror ........ asc:129-146, 376-474
//   P epilogue, fp32 b*A + c*A2, RINT -> bf16 . asc:929-940
//   Y epilogue, bf16(T) + bf16(alpha_bf16*X) .. asc:1454-1476
//   alpha rounded to bf16 on the host ......... binding.cpp:156-162, 470

#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include <atomic>
#include <cstdlib>
#include <cstring>
#include <mutex>

#include "muon_polar_sm100.h"
#include "sm100_ptx.cuh"

namespace muon_sm100 {

enum Kind : int { kGramBf16 = 0, kGramF32 = 1, kPoly = 2, kApply = 3, kGramT = 4, kApplyT = 5 };
constexpr int kNumKinds = 6;

// The transposed kinds share the epilogue of their plain counterparts.
__host__ __device__ constexpr int epi_kind(int kind) {
  return kind == kGramT ? kGramBf16 : (kind == kApplyT ? kApply : kind);
}
// Operand layouts in global memory: K-major unless stated.
__host__ __device__ constexpr bool a_mn_major(int kind) { return kind == kGramT; }
__host__ __device__ constexpr bool b_mn_major(int kind) { return kind == kApply || kind == kGramT; }

__device__ uint32_t g_watchdog = 0;

struct EpiParams {
  int32_t tiles_m;
  int32_t tiles_n;
  int32_t tiles_per_batch;
  int32_t total_tiles;
  int32_t k_blocks;
  float coef_b;
  float coef_c;
  float alpha;  // kApply: a already rounded to bf16
  // kPoly only: compute whole rows of tile blocks [row_tile_begin,
  // row_tile_begin + tiles_m) -- both triangles, no mirror -- instead of the
  // upper triangle (a row slab of P for a multi-GPU caller).
  int32_t rows_mode;
  // Without rows_mode, symmetric kinds compute the upper tiles of the tile
  // rows from row_tile_begin on (tiles_per_batch of them: a band of rows,
  // each tile stored with its mirror); 0 for the whole triangle.
  int32_t row_tile_begin;
  // At most this many clusters (0: as many as fit), leaving SMs free for
  // kernels that run beside this one (a collective on another stream).
  int32_t max_units;
  // Split-K (symmetric kinds): each tile's K range is cut into `splits`
  // work items of (nearly) equal length; item = tile * splits + split.
  int32_t splits;
  int32_t total_items;
  float* partial;      // [total_items][PAIR][128][tile width] fp32 partial sums
  uint32_t* counters;  // [total_tiles][PAIR] arrivals, zero between launches
  // Packed output (kGramF32, kPoly): the upper-triangle 256 x 256 units of
  // each matrix stored one after another in row-major upper order, unit
  // (I, J >= I) at index upper_index(I, J, packed_d); no mirror.  Tiles are
  // visited from index tile_offset of the upper enumeration on.
  int32_t packed;
  int32_t packed_d;      // units per side: mp / 256
  int32_t packed_units;  // units per matrix: packed_d (packed_d + 1) / 2
  int32_t tile_offset;
  // Gram kinds with K-major X: X itself (rows of prefetch_row_bytes, matrices
  // prefetch_batch_bytes apart, prefetch_rows rows of prefetch_lines 128-byte
  // lines), for the L2 prefetch of the diagonal tiles' row blocks; null
  // otherwise.
  const uint8_t* prefetch_base;
  int64_t prefetch_row_bytes;
  int64_t prefetch_batch_bytes;
  int32_t prefetch_rows;
  int32_t prefetch_lines;
  // Column halves (PAIR = 1 symmetric kinds): item (i, j) of each matrix's
  // tiles_m x tiles_m grid is the diagonal tile (i, i) for i == j, the left
  // 64 columns of tile (i, j) for i < j and the right 64 columns of tile
  // (j, i) for i > j, so every element of the upper triangle is computed
  // once, by tiles_m^2 items of at most 128 x 128.
  int32_t halves;
};

struct TileCoord {
  int b, tm, tn;
};

// Index of unit (i, j), i <= j, in the row-major walk of the upper triangle
// of a d x d grid (row i holds (i, i .. d - 1)).
__host__ __device__ __forceinline__ int upper_index(int i, int j, int d) {
  return i * d - i * (i - 1) / 2 + (j - i);
}

// Linear tile index -> (batch, tile row, tile col).  Symmetric kinds walk the
// upper triangle row by row: row tm holds tiles (tm, tm..d-1) (the
// reference enumerates the same set, asc:129-146, 609-630).
__host__ __device__ __forceinline__ TileCoord decode_tile(int tile, bool sym,
                                                          int tiles_m,
                                                          int tiles_n,
                                                          int tiles_per_batch,
                                                          int first_row = 0,
                                                          int offset = 0) {
  TileCoord t;
  t.b = tile / tiles_per_batch;
  int r = tile - t.b * tiles_per_batch + offset;
  if (!sym) {
    t.tm = r / tiles_n;
    t.tn = r - t.tm * tiles_n;
  } else {
    const int d = tiles_m;
    int tm = first_row;
    while (r >= d - tm) {
      r -= d - tm;
      ++tm;
    }
    t.tm = tm;
    t.tn = tm + r;
  }
  return t;
}

// One work item: its tile, its K range (k-blocks [kb_begin, kb_end)), its
// place among the tile's splits, and which column half of the tile it
// computes (-1: the whole tile).
struct WorkItem {
  int tile, b, tm, tn;
  int split, nsplit;
  int kb_begin, kb_end;
  int half;
};

// Work item `item` of the column-halves layout (EpiParams::halves).
__host__ __device__ __forceinline__ WorkItem decode_halves_item(const EpiParams& p, int item) {
  WorkItem w;
  const int d = p.tiles_m;
  w.b = item / (d * d);
  const int r = item - w.b * d * d;
  const int i = r / d, j = r - (r / d) * d;
  w.tm = i < j ? i : j;
  w.tn = i < j ? j : i;
  w.half = i == j ? -1 : (i < j ? 0 : 1);
  w.tile = item;
  w.split = 0;
  w.nsplit = 1;
  w.kb_begin = 0;
  w.kb_end = p.k_blocks;
  return w;
}

// Work item `item` of the tile layouts: whole tiles (the upper triangle of
// symmetric kinds), each cut into p.splits K ranges (SPLIT; otherwise one
// item per tile).
template <bool SPLIT>
__host__ __device__ __forceinline__ WorkItem decode_tile_item(const EpiParams& p, int item,
                                                              bool sym) {
  WorkItem w;
  w.half = -1;
  const int tile = SPLIT ? item / p.splits : item;
  const bool walk = sym && !p.rows_mode;
  const TileCoord tc = decode_tile(tile, walk, p.tiles_m, p.tiles_n, p.tiles_per_batch,
                                   walk ? p.row_tile_begin : 0, walk ? p.tile_offset : 0);
  w.tile = tile;
  w.b = tc.b;
  w.tm = walk ? tc.tm : tc.tm + p.row_tile_begin;
  w.tn = tc.tn;
  if constexpr (SPLIT) {
    w.split = item - tile * p.splits;
    w.nsplit = p.splits;
    w.kb_begin = w.split * p.k_blocks / w.nsplit;
    w.kb_end = (w.split + 1) * p.k_blocks / w.nsplit;
  } else {
    w.split = 0;
    w.nsplit = 1;
    w.kb_begin = 0;
    w.kb_end = p.k_blocks;
  }
  return w;
}

__device__ __forceinline__ uint32_t float_to_bf16_bits(float v) {
  __nv_bfloat16 h = __float2bfloat16_rn(v);
  return static_cast<uint32_t>(*reinterpret_cast<uint16_t*>(&h));
}

// ============================================================ tile engine
// PAIR = 2: 256 x 256 tiles computed by a cluster of two CTAs with
// tcgen05.mma.cta_group::2 (M = 256, N = 256, K = 16): CTA r of the pair
// loads its own 128 rows of the A operand and its own half (128 rows, or 128
// columns when MN-major) of the B operand with plain TMA loads; the leader
// CTA (r = 0) issues the MMAs, which read both CTAs' shared memory and write
// each CTA's 128 x 256 fp32 slice into its own tensor memory.  Per k-block
// each SM ingests 32 KB for 128x256x64 MACs -- half the bytes per FLOP of a
// 128 x 128 single-CTA tile.
// PAIR = 1: 128 x 128 tiles on one CTA (M = 128, N = 128), the same
// pipeline and epilogue; twice the tiles for a given problem, so small
// problems keep more SMs busy.
//
// Epilogue: 64-column chunks staged in shared memory (128-byte swizzle) and
// written with TMA stores; symmetric kinds also stage the transposed chunk
// (64 rows x 128 columns) for the mirror tile.
constexpr int kPairM = 256;
constexpr int kPairN = 256;
constexpr int kHalf = 128;
constexpr int kChunkCols = 64;
constexpr int kMaxSplits = 4;  // split-K items per tile, at most
// One 64-column chunk of a CTA band's fp32 partial sums (split-K).
constexpr uint32_t kPartChunkBytes = 128 * 64 * 4;
constexpr int kAtom = 64;  // bf16 elements per 128-byte swizzle row

constexpr uint32_t kAtomBytes = kHalf * kAtom * 2;  // one [128 x 64] box, 16 KiB

// K depth of one pipeline stage: two 128-byte swizzle atoms (64 KiB stages)
// for single-CTA tiles and for the bf16 Gram on CTA pairs, one (32 KiB) for
// the other pair kinds.  Every stage costs the MMA thread a handshake (wait,
// commit, refill) of about 200 cycles that eight MMAs hide better than four:
// measured on B200, 64 KiB stages make the pair Gram 7-12% faster at
// 4096-8192 rows; the polynomial and the apply keep 32 KiB stages, which
// leave room for four or five of them beside their larger epilogue buffers.
// The single-CTA bf16 Gram also comes with three atoms per stage (kDeepBK:
// 96 KiB stages, two in flight), chosen by size in gram_launch.
template <int KIND, int PAIR>
constexpr int stage_k() {
  return (PAIR == 1 || KIND == kGramBf16 || KIND == kGramT) ? 128 : 64;
}
constexpr int kDeepBK = 192;
template <int KIND, int PAIR>
constexpr int64_t k_blocks_of(int64_t k) {
  return (k + stage_k<KIND, PAIR>() - 1) / stage_k<KIND, PAIR>();
}

// Shared-memory and tensor-memory plan of one CTA of polar_tile_kernel.
// PAIR = 2: a 256 x 256 tile on a tcgen05 CTA pair (each CTA owns a 128 x 256
// band); PAIR = 1: a 128 x 128 tile on one CTA.  HALVES (PAIR = 1, symmetric
// kinds, one work item per CTA): off-diagonal tiles are computed as two
// 128 x 64 column halves, diagonal tiles whole (see decode_item); a half has
// one epilogue chunk and a diagonal tile no mirror, so the polynomial's
// epilogue needs two chunk regions (the mirror of a half shares the second).
template <int KIND, int PAIR = 2, bool HALVES = false, int BK = 0>
struct PairCfg {
  static constexpr bool kSym = KIND != kApply && KIND != kApplyT;
  static constexpr bool kAux = KIND == kPoly || KIND == kApply || KIND == kApplyT;
  static constexpr bool kF32 = KIND == kGramF32;
  static constexpr int kTileM = kHalf * PAIR;
  static constexpr int kTileN = PAIR == 2 ? kPairN : kHalf;
  static constexpr int kElem = kF32 ? 4 : 2;
  static constexpr int kBoxCols = 128 / kElem;  // columns of one 128-byte box row
  static constexpr int kChunks = kTileN / kChunkCols;
  static constexpr uint32_t kOutChunkBytes = kHalf * kChunkCols * kElem;
  static constexpr uint32_t kMirChunkBytes = kSym ? kChunkCols * kHalf * kElem : 0;
  static constexpr int kBK = BK > 0 ? BK : stage_k<KIND, PAIR>();  // K per stage
  // Output regions: kAux kinds keep the whole 128 x kTileN input band (updated
  // in place, one region per chunk, never reused within a tile); the Gram
  // single-buffers its chunk region.
  static constexpr int kOutRegions = kAux ? kChunks : 1;
  // The polynomial double-buffers its mirror chunk (it still fits four
  // stages); the Gram single-buffers it.
  static constexpr int kMirRegions = kSym ? ((kAux && !HALVES) ? 2 : 1) : 0;
  // Store groups that may still read shared memory when a chunk starts: the
  // region a chunk writes was last used by the chunk kMirRegions before it.
  static constexpr int kPending = (kSym && kAux && !HALVES) ? 1 : 0;
  static constexpr bool kWaitPerChunk = kSym;
  static constexpr uint32_t kEpiBytes =
      (HALVES && kAux) ? kOutRegions * kOutChunkBytes
                       : kOutRegions * kOutChunkBytes + kMirRegions * kMirChunkBytes;
  static constexpr uint32_t kAHalfBytes = kHalf * kBK * 2;
  static constexpr uint32_t kBHalfBytes = kHalf * kBK * 2;
  static constexpr uint32_t kStageBytes = kAHalfBytes + kBHalfBytes;
  static constexpr uint32_t kFixedBytes = 1024 + kEpiBytes + 256;
  static constexpr int kStagesFit =
      static_cast<int>((232448u - kFixedBytes) / kStageBytes);
  static constexpr int kStages = kStagesFit > 8 ? 8 : kStagesFit;
  // TMA producers: two threads fill every stage together, one the A
  // operand's boxes, the other the B operand's (a diagonal tile's A boxes
  // are shared out between them), each arriving on the stage's full barrier
  // with its own byte count.  Measured on B200, one thread's loads into
  // successive mbarrier phases reach about 90 GB/s per SM with 32 KiB
  // phases, two threads about 150 GB/s, the per-SM limit.
  static constexpr int kProducers = 2;
  static constexpr uint32_t kSmemBytes = kFixedBytes + kStages * kStageBytes;
  // Split-K stages partial sums in the pipeline stages: a whole band to
  // publish, or two buffers of (splits - 1) chunks to reduce.
  static constexpr uint32_t kRingBytes = kStages * kStageBytes;
  static constexpr int kSplitsFit = 1 + static_cast<int>(kRingBytes / (2 * kPartChunkBytes));
  static constexpr int kMaxSplitsHere = kSplitsFit < kMaxSplits ? kSplitsFit : kMaxSplits;
  static_assert(kChunks * kPartChunkBytes <= kRingBytes, "split-K staging");
  static constexpr uint32_t kTmemCols = 2 * kTileN;
  static constexpr uint32_t kBandFloats = kHalf * kTileN;  // one CTA's fp32 band
  static_assert(kStages >= 2, "pipeline depth");
  static_assert(kSmemBytes <= 232448, "shared memory budget");
};

// Offset inside a TMA box of 128-byte rows with the 128-byte swizzle.
__device__ __forceinline__ uint32_t swz_box(int row, int byte) {
  return static_cast<uint32_t>(row * 128 +
                               ((((byte >> 4) ^ (row & 7))) << 4) + (byte & 15));
}

__device__ __forceinline__ uint32_t bf162_bits(__nv_bfloat162 v) {
  return *reinterpret_cast<uint32_t*>(&v);
}
__device__ __forceinline__ __nv_bfloat162 bits_bf162(uint32_t u) {
  return *reinterpret_cast<__nv_bfloat162*>(&u);
}

// Epilogue of 32 accumulator columns (half `h` of a 64-column chunk) for
// band row `row`, with packed bf16x2 arithmetic where the reference's
// dataflow is bf16 (kApply) and fp32 where it is fp32 (kPoly).
template <int KIND>
__device__ __forceinline__ void pair_epilogue_half(const EpiParams& p, uint32_t out,
                                                   uint32_t mir, bool mirror, int row,
                                                   int h, const float (&v)[32]) {
  using Cfg = PairCfg<KIND>;
  if constexpr (KIND == kGramF32) {
    // out: box h of [128 x 32 fp32]; mirror rows h*32.. of 4 boxes [64 x 32]
    const uint32_t ob = out + h * (kHalf * 128);
#pragma unroll
    for (int u = 0; u < 8; ++u)
      st_shared_v4(ob + swz_box(row, u * 16),
                   make_uint4(__float_as_uint(v[4 * u]), __float_as_uint(v[4 * u + 1]),
                              __float_as_uint(v[4 * u + 2]), __float_as_uint(v[4 * u + 3])));
    if (mirror) {
      const uint32_t mbase = mir + (row / 32) * (kChunkCols * 128);
#pragma unroll
      for (int j = 0; j < 32; ++j)
        st_shared_f32(mbase + swz_box(h * 32 + j, (row % 32) * 4), v[j]);
    }
  } else {
    // out: columns h*32.. of one box [128 x 64 bf16] = 4 16-byte units
    uint32_t w[16];
#pragma unroll
    for (int u = 0; u < 4; ++u) {
      const uint32_t addr = out + swz_box(row, h * 64 + u * 16);
      if constexpr (KIND == kGramBf16) {
#pragma unroll
        for (int e = 0; e < 4; ++e)
          w[4 * u + e] = bf162_bits(__floats2bfloat162_rn(v[8 * u + 2 * e], v[8 * u + 2 * e + 1]));
      } else {
        const uint4 qv = ld_shared_v4(addr);
        const uint32_t in[4] = {qv.x, qv.y, qv.z, qv.w};
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const int j = 8 * u + 2 * e;
          if constexpr (KIND == kPoly) {
            // P = bf16( fl(b*A) + fl(c*acc) ), no fused multiply-add
            // (asc:929-940).
            const float2 a2 = __bfloat1622float2(bits_bf162(in[e]));
            w[4 * u + e] = bf162_bits(__floats2bfloat162_rn(
                __fadd_rn(__fmul_rn(p.coef_b, a2.x), __fmul_rn(p.coef_c, v[j])),
                __fadd_rn(__fmul_rn(p.coef_b, a2.y), __fmul_rn(p.coef_c, v[j + 1]))));
          } else {
            // Y = bf16( bf16(T) + bf16(alpha*x) ) (asc:1472-1476): bf16 x bf16
            // is exact before its single rounding, and the bf16 add rounds
            // the exact sum once.  The _rn forms keep the multiply and the
            // add separately rounded (no contraction into one fma).
            const __nv_bfloat162 alpha2 = __float2bfloat162_rn(p.alpha);
            const __nv_bfloat162 ax = __hmul2_rn(bits_bf162(in[e]), alpha2);
            const __nv_bfloat162 t = __floats2bfloat162_rn(v[j], v[j + 1]);
            w[4 * u + e] = bf162_bits(__hadd2_rn(t, ax));
          }
        }
      }
      st_shared_v4(addr, make_uint4(w[4 * u], w[4 * u + 1], w[4 * u + 2], w[4 * u + 3]));
    }
    if constexpr (Cfg::kSym) {
      if (mirror) {
        const uint32_t mbase = mir + (row / 64) * (kChunkCols * 128);
#pragma unroll
        for (int j = 0; j < 32; ++j) {
          const uint16_t hv = static_cast<uint16_t>((j & 1) ? (w[j >> 1] >> 16)
                                                            : (w[j >> 1] & 0xFFFFu));
          st_shared_u16(mbase + swz_box(h * 32 + j, (row % 64) * 2), hv);
        }
      }
    }
  }
}

// Threads of polar_tile_kernel and polar_fused_kernel: warps 0 and 10 TMA
// producers, warp 1 MMA issuer and tensor-memory owner, warps 2..9 epilogue
// (two per tensor-memory lane quarter, each taking 32 of a chunk's 64
// columns).
constexpr int kPairEpiThreads = 256;
constexpr int kTileThreads = 352;
constexpr int kProducerWarp2 = 10;

// SPLIT: the launch has split-K items (symmetric kinds only).  Compiling the
// split-K paths out of the other launches cuts the kernel's registers (the
// single-CTA Gram from 145 to 77, the pair apply from 158 to 101); measured
// on B200 the config-1 step 38.9 -> 37.5 us.
// HALVES: the column-halves decomposition (PAIR = 1, symmetric kinds, one
// item per CTA, no split-K; see EpiParams::halves).  tmap_b then has boxes
// of 64 rows, the B operand of a half.
// BK: K per pipeline stage if not the kind's default (stage_k); kDeepBK for
// the single-CTA bf16 Gram on long rows.
template <int KIND, int PAIR, bool SPLIT, bool HALVES = false, int BK = 0>
__global__ void __launch_bounds__(kTileThreads, 1)
    polar_tile_kernel(const __grid_constant__ CUtensorMap tmap_a,
                      const __grid_constant__ CUtensorMap tmap_b,
                      const __grid_constant__ CUtensorMap tmap_aux,
                      const __grid_constant__ CUtensorMap tmap_out,
                      const __grid_constant__ CUtensorMap tmap_mir,
                      const EpiParams p) {
  using Cfg = PairCfg<KIND, PAIR, HALVES, BK>;
  static_assert(!HALVES || (PAIR == 1 && Cfg::kSym && !SPLIT && KIND != kGramT),
                "column halves: single-CTA symmetric kinds without split-K");
  static_assert(BK == 0 || (PAIR == 1 && KIND == kGramBf16 && !SPLIT),
                "deep stages: the single-CTA bf16 Gram without split-K");
  constexpr int kTileM = Cfg::kTileM;
  constexpr int kTileN = Cfg::kTileN;
  constexpr int S = Cfg::kStages;
  constexpr bool kAmn = a_mn_major(KIND);
  constexpr bool kBmn = b_mn_major(KIND);
  constexpr bool kSym = Cfg::kSym;
  // Each launch compiles in only the work-item decode of its layout, and the
  // column-halves kernels no packed or rows-mode paths: code a kernel never
  // runs still costs time (measured on B200, dropping the tile-walk decode
  // and the packed paths from the halves kernels made the config-1 step
  // 32.1 -> 31.0 us, [1,129,130] 13.3 -> 12.9 us; the split-K arithmetic
  // from the decode of launches without it, 31.0 -> 30.8 us).
  auto decode = [](const EpiParams& q, int item, bool sym) {
    if constexpr (HALVES)
      return decode_halves_item(q, item);
    else
      return decode_tile_item<SPLIT>(q, item, sym);
  };

  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw_addr = smem_addr(smem_raw);
  uint8_t* smem = smem_raw + ((1024u - (raw_addr & 1023u)) & 1023u);
  uint8_t* sOut = smem;
  // (HALVES polynomial: a half's mirror shares the second chunk region,
  // which only a diagonal tile uses as a chunk)
  uint8_t* sMir = sOut + ((HALVES && Cfg::kAux) ? 1 : Cfg::kOutRegions) * Cfg::kOutChunkBytes;
  uint8_t* sA = smem + Cfg::kEpiBytes;
  uint8_t* sB = sA + S * Cfg::kAHalfBytes;
  uint64_t* full = reinterpret_cast<uint64_t*>(sB + S * Cfg::kBHalfBytes);
  uint64_t* empty = full + S;
  uint64_t* tfull = empty + S;
  uint64_t* tempty = tfull + 2;
  uint64_t* drain = tempty + 2;
  uint64_t* aux_full = drain + 1;      // epilogue input, one per chunk
  uint64_t* part_full = aux_full + 4;  // split-K partial chunks, two buffers
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(part_full + 2);
  volatile uint32_t* last_flag = tmem_slot + 1;

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const uint32_t rank = PAIR == 2 ? cluster_cta_rank() : 0u;
  const int cluster = static_cast<int>(blockIdx.x) / PAIR;
  const int nclusters = static_cast<int>(gridDim.x) / PAIR;
  constexpr int kEpiLeader = 64;

  if (threadIdx.x == 0) {
    for (int s = 0; s < S; ++s) {
      mbar_init(&full[s], Cfg::kProducers);  // the leader CTA's producers
      mbar_init(&empty[s], 1);
    }
    for (int a = 0; a < 2; ++a) {
      mbar_init(&tfull[a], 1);
      mbar_init(&tempty[a], 8 * PAIR);  // 8 epilogue warps in each CTA
    }
    mbar_init(drain, 1);
    for (int c = 0; c < 4; ++c) mbar_init(&aux_full[c], 1);
    mbar_init(&part_full[0], 1);
    mbar_init(&part_full[1], 1);
    fence_mbar_init();
    prefetch_tensor_map(&tmap_a);
    prefetch_tensor_map(&tmap_b);
    prefetch_tensor_map(&tmap_aux);
    prefetch_tensor_map(&tmap_out);
    prefetch_tensor_map(&tmap_mir);
  }
  if (warp == 1) {
    if constexpr (PAIR == 2) {
      tmem_alloc_pair(tmem_slot, Cfg::kTmemCols);
      tmem_relinquish_pair();
    } else {
      tmem_alloc(tmem_slot, Cfg::kTmemCols);
      tmem_relinquish();
    }
  }
  tc_fence_before();
  __syncthreads();
  if constexpr (PAIR == 2) cluster_sync();  // the peer's barriers exist first
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  // Every thread passes the grid dependency wait before it touches data the
  // previous kernel may write, and lets dependents launch only after it.

  if (warp == 0 || warp == kProducerWarp2) {
    if (lane == 0) {
      // ---------------- TMA producers (both CTAs): producer 0 loads the A
      // operand of every stage, producer 1 the B operand; on a diagonal
      // tile of a symmetric kind (A only) they split A's boxes.
      const uint32_t pid = warp == 0 ? 0u : 1u;
      // Boxes [j0, j1) of one operand into stage s; PAIR = 2 counts the
      // bytes on the leader's barrier, PAIR = 1 on its own.
      // K-major: [128 rows x 64 k] boxes; MN-major: one [kBK k x 64 rows] box
      // per 64-row chunk.
      constexpr int kBoxesA = kAmn ? kHalf / kAtom : Cfg::kBK / kAtom;
      constexpr int kBoxesB = kBmn ? kHalf / kAtom : Cfg::kBK / kAtom;
      constexpr uint32_t kBoxBytesA = Cfg::kAHalfBytes / kBoxesA;
      auto load_a = [&](uint32_t s, const WorkItem& w, int kb, int j0, int j1) {
        const uint32_t bar = PAIR == 2 ? map_to_cta(smem_addr(&full[s]), 0) : 0u;
        const int a_row = w.tm * kTileM + static_cast<int>(rank) * kHalf;
#pragma unroll
        for (int j = 0; j < kBoxesA; ++j) {
          if (j < j0 || j >= j1) continue;
          void* dst = sA + s * Cfg::kAHalfBytes + j * (kAmn ? Cfg::kBK * 128 : kAtomBytes);
          const int c0 = kAmn ? a_row + j * kAtom : kb * Cfg::kBK + j * kAtom;
          const int c1 = kAmn ? kb * Cfg::kBK : a_row;
          if constexpr (PAIR == 2)
            tma_load_3d_pair(dst, &tmap_a, bar, c0, c1, w.b);
          else
            tma_load_3d(dst, &tmap_a, &full[s], c0, c1, w.b);
        }
      };
      auto load_b = [&](uint32_t s, const WorkItem& w, int kb) {
        const uint32_t bar = PAIR == 2 ? map_to_cta(smem_addr(&full[s]), 0) : 0u;
        const int b_row = w.tn * kTileN + static_cast<int>(rank) * kHalf +
                          (HALVES && w.half > 0 ? kChunkCols : 0);
        // K-major: [128 n x 64 k] boxes; MN-major: one [kBK k x 64 n] box per
        // 64-column chunk
#pragma unroll
        for (int j = 0; j < kBoxesB; ++j) {
          void* dst = sB + s * Cfg::kBHalfBytes + j * (kBmn ? Cfg::kBK * 128 : kAtomBytes);
          const int c0 = kBmn ? b_row + j * kAtom : kb * Cfg::kBK + j * kAtom;
          const int c1 = kBmn ? kb * Cfg::kBK : b_row;
          if constexpr (PAIR == 2)
            tma_load_3d_pair(dst, &tmap_b, bar, c0, c1, w.b);
          else
            tma_load_3d(dst, &tmap_b, &full[s], c0, c1, w.b);
        }
      };
      // This producer's share of an item: a diagonal tile of a symmetric
      // kind multiplies a row block by itself, so only the A operand is
      // loaded (the MMA reads it twice) and the producers split its boxes;
      // otherwise producer 0 loads all of A, producer 1 all of B.
      struct Share {
        bool diag;
        int a0, a1;
        uint32_t bytes;
      };
      auto share_of = [&](const WorkItem& w) {
        constexpr int kHalfA = kBoxesA / 2;
        Share sh;
        sh.diag = kSym && w.tm == w.tn;
        sh.a0 = sh.diag ? (pid == 0 ? 0 : kHalfA) : 0;
        sh.a1 = sh.diag ? (pid == 0 ? kHalfA : kBoxesA) : (pid == 0 ? kBoxesA : 0);
        // (a column half's B operand is 64 rows: half the bytes)
        sh.bytes = static_cast<uint32_t>(sh.a1 - sh.a0) * kBoxBytesA +
                   (!sh.diag && pid == 1
                        ? (HALVES && w.half >= 0 ? Cfg::kBHalfBytes / 2 : Cfg::kBHalfBytes)
                        : 0u);
        return sh;
      };
      // The first stage's bookkeeping (decode, expected bytes) runs before
      // the grid dependency wait, so that the loads follow the wait at once:
      // measured on B200, code first executed after the wait stalls on
      // instruction fetch (0.2-0.3 us per miss), about 0.8 us before the
      // first load of each kernel; moving it ahead made the config-1 step
      // 0.6 us faster.
      uint32_t it = 0;
      bool ok = true;
      WorkItem w_first = {};
      bool prepared = false;  // stage 0 is free and its bytes are expected
      if (cluster < p.total_items) {
        w_first = decode(p, cluster, kSym);
        if (w_first.kb_begin < w_first.kb_end) {
          if (rank == 0) mbar_arrive_expect_tx(&full[0], PAIR * share_of(w_first).bytes);
          prepared = true;
        }
      }
      grid_dependency_wait();
      grid_launch_dependents();
      for (int item = cluster; ok && item < p.total_items; item += nclusters) {
        const WorkItem w = item == cluster ? w_first : decode(p, item, kSym);
        const Share sh = share_of(w);
        for (int kb = w.kb_begin; kb < w.kb_end; ++kb, ++it) {
          const uint32_t s = it % S;
          const uint32_t ph = (it / S) & 1u;
          if (!prepared) {
            if (!mbar_wait_bounded(&empty[s], ph ^ 1u)) {
              ok = false;
              break;
            }
            if (rank == 0) mbar_arrive_expect_tx(&full[s], PAIR * sh.bytes);
          }
          prepared = false;
          load_a(s, w, kb, sh.a0, sh.a1);
          if (!sh.diag && pid == 1) load_b(s, w, kb);
        }
      }
      if (!ok) atomicOr(&g_watchdog, MUON_POLAR_WATCHDOG_PRODUCER);
      if (rank == 0) {
        // Drain: the pair's last loads land before the CTAs exit.
        const uint32_t inflight = it < static_cast<uint32_t>(S) ? it : S;
        for (uint32_t i = it - inflight; i < it; ++i) {
          if (!mbar_wait_bounded(&full[i % S], (i / S) & 1u)) {
            atomicOr(&g_watchdog, MUON_POLAR_WATCHDOG_DRAIN);
            break;
          }
        }
      }
    } else {
      grid_dependency_wait();
      grid_launch_dependents();
    }
  } else if (warp == 1) {
    // The MMA warp reads no global memory (only shared memory that the
    // producers fill after their dependency wait), so it does not wait for
    // the previous grid.
    grid_launch_dependents();
    if (lane == 0 && rank == 0) {
      // ---------------- tcgen05 MMA issuer (leader CTA only)
      constexpr uint32_t idesc_full =
          idesc_bf16_f32(kTileN, kBmn ? 1u : 0u, kTileM, kAmn ? 1u : 0u);
      constexpr uint32_t idesc_half =
          idesc_bf16_f32(kChunkCols, kBmn ? 1u : 0u, kTileM, kAmn ? 1u : 0u);
      uint32_t it = 0;
      uint32_t t = 0;
      bool ok = true;
      for (int item = cluster; ok && item < p.total_items; item += nclusters, ++t) {
        const WorkItem w = decode(p, item, kSym);
        const bool diag = kSym && w.tm == w.tn;
        const uint32_t idesc = (HALVES && w.half >= 0) ? idesc_half : idesc_full;
        const uint32_t acc = t & 1u;
        const uint32_t uph = (t >> 1) & 1u;
        if (!mbar_wait_bounded(&tempty[acc], uph ^ 1u)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + acc * kTileN;
        for (int kb = w.kb_begin; kb < w.kb_end; ++kb, ++it) {
          const uint32_t s = it % S;
          const uint32_t ph = (it / S) & 1u;
          if (!mbar_wait_bounded(&full[s], ph)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t a_base = smem_addr(sA + s * Cfg::kAHalfBytes);
          const uint32_t b_base = diag ? a_base : smem_addr(sB + s * Cfg::kBHalfBytes);
#pragma unroll
          for (int k = 0; k < Cfg::kBK / 16; ++k) {
            // K-major: K step k lies in swizzle atom k/4 (16 KiB apart), 32
            // bytes per step inside the atom's 128-byte rows.
            const uint32_t koff = (k / 4) * kAtomBytes + (k % 4) * 32;
            // MN-major: 16 k-rows of 128 bytes per step; 64-column chunks are
            // Cfg::kBK*128 bytes apart (leading offset).
            const uint64_t ad = kAmn ? smem_desc_sw128(a_base + k * 2048, Cfg::kBK * 128, 1024)
                                     : smem_desc_sw128(a_base + koff, 16, 1024);
            const uint64_t bd = kBmn ? smem_desc_sw128(b_base + k * 2048, Cfg::kBK * 128, 1024)
                                     : smem_desc_sw128(b_base + koff, 16, 1024);
            if constexpr (PAIR == 2)
              umma_bf16_pair(d_tmem, ad, bd, idesc, (kb > w.kb_begin || k > 0) ? 1u : 0u);
            else
              umma_bf16(d_tmem, ad, bd, idesc, (kb > w.kb_begin || k > 0) ? 1u : 0u);
          }
          if constexpr (PAIR == 2) {
            umma_commit_pair(map_to_cta(smem_addr(&empty[s]), 0));
            umma_commit_pair(map_to_cta(smem_addr(&empty[s]), 1));
          } else {
            umma_commit(&empty[s]);
          }
        }
        if (!ok) break;
        if constexpr (PAIR == 2) {
          umma_commit_pair(map_to_cta(smem_addr(&tfull[acc]), 0));
          umma_commit_pair(map_to_cta(smem_addr(&tfull[acc]), 1));
        } else {
          umma_commit(&tfull[acc]);
        }
      }
      if (!ok) atomicOr(&g_watchdog, MUON_POLAR_WATCHDOG_MMA);
      if constexpr (PAIR == 2)
        umma_commit_pair(map_to_cta(smem_addr(drain), 0));
      else
        umma_commit(drain);
      if (!mbar_wait_bounded(drain, 0)) atomicOr(&g_watchdog, MUON_POLAR_WATCHDOG_DRAIN);
    }
  } else {
    // ---------------- epilogue warps 2..9 (both CTAs)
    const int q = warp & 3;          // tensor-memory lane quarter of this warp
    const int hc = (warp - 2) >> 2;  // which 32 columns of each 64-column chunk
    const int row = q * 32 + lane;
    const uint32_t out_base = smem_addr(sOut);
    const uint32_t mir_base = smem_addr(sMir);
    const bool leader = threadIdx.x == kEpiLeader;
    const uint32_t tempty_leader0 = PAIR == 2 ? map_to_cta(smem_addr(&tempty[0]), 0) : 0u;
    const uint32_t tempty_leader1 = PAIR == 2 ? map_to_cta(smem_addr(&tempty[1]), 0) : 0u;
    // Epilogue input tile (kAux kinds), one region and one barrier per
    // chunk; the leader reloads chunk c for the next item as soon as the TMA
    // store of this item's chunk c has read the region.
    uint32_t aux_issued[4] = {0u, 0u, 0u, 0u};
    auto load_aux_chunk = [&](int item, int c) {
      const WorkItem w = decode(p, item, kSym);
      mbar_arrive_expect_tx(&aux_full[c], Cfg::kOutChunkBytes);
      tma_load_3d(sOut + c * Cfg::kOutChunkBytes, &tmap_aux, &aux_full[c],
                  w.tn * kTileN + (HALVES && w.half > 0 ? kChunkCols : 0) + c * kChunkCols,
                  w.tm * kTileM + static_cast<int>(rank) * kHalf, w.b);
      ++aux_issued[c];
    };
    // Chunks of an item's epilogue: one for a column half.
    auto chunks_of = [&](int item) {
      if constexpr (HALVES) return decode(p, item, kSym).half >= 0 ? 1 : Cfg::kChunks;
      return Cfg::kChunks;
    };
    auto release_accumulator = [&](uint32_t acc) {
      tc_fence_before();
      __syncwarp();
      if (lane == 0) {
        if (PAIR == 1 || rank == 0)
          mbar_arrive(&tempty[acc]);
        else
          mbar_arrive_cluster(acc ? tempty_leader1 : tempty_leader0);
      }
    };
    if constexpr (KIND == kGramBf16 || KIND == kGramF32) {
      // X is usually not written by the kernel this one waits for, and its
      // first touch comes from DRAM: before the dependency wait the
      // epilogue threads of each diagonal tile's CTA bring that tile's row
      // block of X (every row block has one) into L2, so that each byte is
      // fetched once.  Plain prefetch instructions leave the CTA's TMA unit
      // to its operand loads; issuing the same prefetch as TMA boxes held
      // a diagonal CTA's first loads back by up to 3 us when it started
      // late (measured on B200 at [8,512,2048], where this form is 0.7 us
      // faster per step).  Prefetching into L2, the point of coherence, is
      // safe even while the previous kernel still writes X.
      if (p.prefetch_base != nullptr && cluster < p.total_items) {
        const WorkItem w = decode(p, cluster, kSym);
        if (w.tm == w.tn) {
          const int r0 = w.tm * kTileM + static_cast<int>(rank) * kHalf;
          const int total = kHalf * p.prefetch_lines;
          // line-major order: the first k-blocks of every row come first
          for (int l = static_cast<int>(threadIdx.x) - kEpiLeader; l < total;
               l += kPairEpiThreads) {
            const int row = r0 + (l % kHalf);
            if (row < p.prefetch_rows)
              prefetch_l2(p.prefetch_base + w.b * p.prefetch_batch_bytes +
                          row * p.prefetch_row_bytes + (l / kHalf) * 128);
          }
        }
      }
    }
    // Everything, X included, is loaded after the grid dependency wait:
    // measured on B200, loading the apply's X (operand stages and epilogue
    // tile) before it delayed the P loads queued behind it and made the
    // config-1 step 0.6 us slower.
    grid_dependency_wait();
    grid_launch_dependents();
    if constexpr (Cfg::kAux) {
      if (leader && cluster < p.total_items) {
        const int nch0 = chunks_of(cluster);
        for (int c = 0; c < nch0; ++c) load_aux_chunk(cluster, c);
      }
    }
    uint32_t t = 0;
    for (int item = cluster; item < p.total_items; item += nclusters, ++t) {
      const WorkItem tc = decode(p, item, kSym);
      const uint32_t acc = t & 1u;
      const uint32_t uph = (t >> 1) & 1u;
      const int next = item + nclusters;
      int ok = 1;
      if (lane == 0) ok = mbar_wait_bounded(&tfull[acc], uph) ? 1 : 0;
      ok = __shfl_sync(0xffffffffu, ok, 0);
      if (!ok) {
        if (lane == 0) atomicOr(&g_watchdog, MUON_POLAR_WATCHDOG_EPILOGUE);
        break;
      }
      tc_fence_after();
      bool mirror = kSym && (HALVES || !p.rows_mode) && tc.tm != tc.tn;
      if constexpr ((KIND == kGramF32 || KIND == kPoly) && !HALVES) {
        if (p.packed) mirror = false;
      }
      const int row0 = tc.tm * kTileM + static_cast<int>(rank) * kHalf;
      const int col0 = tc.tn * kTileN + (HALVES && tc.half > 0 ? kChunkCols : 0);
      const int nch = (HALVES && tc.half >= 0) ? 1 : Cfg::kChunks;
      const uint32_t t_row = tmem_base + (static_cast<uint32_t>(q * 32) << 16) + acc * kTileN;
      bool reduce = false;
      // Other splits' partial chunks c into buffer c % 2 of the (free)
      // pipeline stages; issued by the leader of the last split.
      auto load_parts = [&](int c) {
        uint64_t* bar = &part_full[c & 1];
        mbar_arrive_expect_tx(bar, (tc.nsplit - 1) * kPartChunkBytes);
        int o = 0;
        for (int i = 0; i < tc.nsplit; ++i) {
          if (i == tc.split) continue;
          const float* src =
              p.partial +
              (static_cast<size_t>(tc.tile * tc.nsplit + i) * PAIR + rank) * Cfg::kBandFloats +
              static_cast<size_t>(c) * (kPartChunkBytes / 4);
          bulk_load(sA + ((c & 1) * (tc.nsplit - 1) + o) * kPartChunkBytes, src, kPartChunkBytes,
                    bar);
          ++o;
        }
      };
      if (SPLIT && tc.nsplit > 1) {
        // Split-K.  A launch with splits has one work item per cluster, so
        // once the accumulator is complete the pipeline stages are free and
        // serve as staging for partial sums.  The split that arrives last
        // (per CTA band) takes the others' partial bands and sums all of them
        // in split order -- the same order whichever split is last -- and
        // runs the epilogue; the others publish their band and leave.
        // Partial band layout: float4 slots [chunk][vec 0..15][row 0..127],
        // 32 KiB per chunk, moved as whole chunks by bulk copies.
        uint32_t* ctr = p.counters + (static_cast<size_t>(tc.tile) * PAIR + rank) * 2;
        if (leader) {
          if (p.total_items > nclusters) atomicOr(&g_watchdog, MUON_POLAR_WATCHDOG_EPILOGUE);
          *last_flag = atomicAdd(ctr, 1u) + 1u == static_cast<uint32_t>(tc.nsplit) ? 1u : 0u;
        }
        named_barrier(1, kPairEpiThreads);
        reduce = *last_flag != 0u;
        if (!reduce) {
          const uint32_t stage = smem_addr(sA) + static_cast<uint32_t>(row) * 16u;
#pragma unroll 1
          for (int c = 0; c < Cfg::kChunks; ++c) {
            uint32_t r0[32];
            tmem_ld_32x32b_x32(t_row + c * kChunkCols + hc * 32, r0);
            tmem_wait_ld(r0);
#pragma unroll
            for (int u = 0; u < 8; ++u)
              st_shared_v4(stage + static_cast<uint32_t>((c * 16 + hc * 8 + u) * kHalf) * 16u,
                           make_uint4(r0[4 * u], r0[4 * u + 1], r0[4 * u + 2], r0[4 * u + 3]));
          }
          release_accumulator(acc);
          fence_proxy_async_smem();
          named_barrier(1, kPairEpiThreads);
          if (leader) {
            float* dst = p.partial + (static_cast<size_t>(item) * PAIR + rank) * Cfg::kBandFloats;
#pragma unroll
            for (int c = 0; c < Cfg::kChunks; ++c)
              bulk_store(dst + c * (kPartChunkBytes / 4), sA + c * kPartChunkBytes,
                         kPartChunkBytes);
            bulk_commit_group();
            bulk_wait_group0();
            fence_proxy_async_global();
            __threadfence();
            red_release_gpu_add(ctr + 1, 1u);
          }
          continue;
        }
        if (leader) {
          // Last split: no other split touches the ticket counter again, and
          // once every other band has been published, nor the other one.
          ctr[0] = 0u;
          if (!wait_counter_bounded(ctr + 1, static_cast<uint32_t>(tc.nsplit - 1)))
            atomicOr(&g_watchdog, MUON_POLAR_WATCHDOG_EPILOGUE);
          ctr[1] = 0u;
          fence_proxy_async_global();
          load_parts(0);
          if (Cfg::kChunks > 1) load_parts(1);
        }
      }
      // Accumulator chunk c + 1 is read from tensor memory while chunk c is
      // processed (two register buffers, loop fully unrolled).
      uint32_t rbuf[2][32];
      tmem_ld_32x32b_x32(t_row + hc * 32, rbuf[0]);
#pragma unroll
      for (int c = 0; c < Cfg::kChunks; ++c) {
        if (HALVES && c >= nch) break;
        const int ro = c % Cfg::kOutRegions;
        const uint32_t out = out_base + ro * Cfg::kOutChunkBytes;
        constexpr int kMR = Cfg::kMirRegions > 0 ? Cfg::kMirRegions : 1;
        const int rm = c % kMR;
        const uint32_t mir = mir_base + rm * Cfg::kMirChunkBytes;
        if constexpr (Cfg::kWaitPerChunk) {
          if (leader) bulk_wait_group_read<Cfg::kPending>();
          named_barrier(1, kPairEpiThreads);
        }
        tmem_wait_ld(rbuf[c & 1]);
        if (c + 1 < nch)
          tmem_ld_32x32b_x32(t_row + (c + 1) * kChunkCols + hc * 32, rbuf[(c + 1) & 1]);
        else
          release_accumulator(acc);
        float v[32];
#pragma unroll
        for (int j = 0; j < 32; ++j) v[j] = __uint_as_float(rbuf[c & 1][j]);
        if constexpr (Cfg::kAux) {
          if (!mbar_wait_bounded(&aux_full[c], t & 1u))
            atomicOr(&g_watchdog, MUON_POLAR_WATCHDOG_EPILOGUE);
        }
        if (SPLIT && reduce) {
          // v <- sum over splits i = 0..nsplit-1, in that order, of the
          // split's partial (this split's own from tensor memory).
          if (!mbar_wait_bounded(&part_full[c & 1], (c >> 1) & 1))
            atomicOr(&g_watchdog, MUON_POLAR_WATCHDOG_EPILOGUE);
          const uint32_t buf = smem_addr(sA) + (c & 1) * (tc.nsplit - 1) * kPartChunkBytes +
                               static_cast<uint32_t>(row) * 16u;
#pragma unroll
          for (int u = 0; u < 8; ++u) {
            const uint32_t off = static_cast<uint32_t>((hc * 8 + u) * kHalf) * 16u;
            float4 sum = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
            for (int i = 0; i < kMaxSplits; ++i) {
              if (i >= tc.nsplit) break;
              float4 x;
              if (i == tc.split) {
                x = make_float4(v[4 * u], v[4 * u + 1], v[4 * u + 2], v[4 * u + 3]);
              } else {
                const int o = i < tc.split ? i : i - 1;
                const uint4 w4 = ld_shared_v4(buf + o * kPartChunkBytes + off);
                x = make_float4(__uint_as_float(w4.x), __uint_as_float(w4.y),
                                __uint_as_float(w4.z), __uint_as_float(w4.w));
              }
              if (i == 0) {
                sum = x;
              } else {
                sum.x = __fadd_rn(sum.x, x.x);
                sum.y = __fadd_rn(sum.y, x.y);
                sum.z = __fadd_rn(sum.z, x.z);
                sum.w = __fadd_rn(sum.w, x.w);
              }
            }
            v[4 * u] = sum.x;
            v[4 * u + 1] = sum.y;
            v[4 * u + 2] = sum.z;
            v[4 * u + 3] = sum.w;
          }
        }
        pair_epilogue_half<epi_kind(KIND)>(p, out, mir, mirror, row, hc, v);
        fence_proxy_async_smem();
        named_barrier(1, kPairEpiThreads);
        if (leader) {
          // every thread is done with partial buffer c % 2: refill it
          if (SPLIT && reduce && c + 2 < Cfg::kChunks) load_parts(c + 2);
          const uint8_t* so = sOut + ro * Cfg::kOutChunkBytes;
          const uint8_t* sm = sMir + rm * Cfg::kMirChunkBytes;
          bool packed = false;
          if constexpr ((KIND == kGramF32 || KIND == kPoly) && !HALVES) packed = p.packed != 0;
          if (packed) {
            // the chunk's 128 x 64 block inside its 256 x 256 unit
            const int col = col0 + c * kChunkCols;
            const int unit = tc.b * p.packed_units +
                             upper_index(row0 / kPairM, col / kPairN, p.packed_d);
#pragma unroll
            for (int h = 0; h < kChunkCols / Cfg::kBoxCols; ++h)
              tma_store_3d(&tmap_out, so + h * (kHalf * 128), col % kPairN + h * Cfg::kBoxCols,
                           row0 % kPairM, unit);
          } else {
#pragma unroll
            for (int h = 0; h < kChunkCols / Cfg::kBoxCols; ++h)
              tma_store_3d(&tmap_out, so + h * (kHalf * 128),
                           col0 + c * kChunkCols + h * Cfg::kBoxCols, row0, tc.b);
          }
          if (mirror) {
#pragma unroll
            for (int h = 0; h < kHalf / Cfg::kBoxCols; ++h)
              tma_store_3d(&tmap_mir, sm + h * (kChunkCols * 128), row0 + h * Cfg::kBoxCols,
                           col0 + c * kChunkCols, tc.b);
          }
          bulk_commit_group();
          if constexpr (Cfg::kAux && !HALVES) {
            // region c - 1 has been read by its store: next item's chunk c - 1
            if (c >= 1 && next < p.total_items) {
              bulk_wait_group_read<1>();
              load_aux_chunk(next, c - 1);
            }
          }
        }
      }
      if constexpr (Cfg::kAux && !HALVES) {
        if (leader && next < p.total_items) {
          bulk_wait_group_read<0>();
          load_aux_chunk(next, Cfg::kChunks - 1);
        }
      }
    }
    if (leader) {
      bulk_wait_group0();
      // input chunks still in flight (an item that was not processed) land
      // before the CTA exits
      for (int c = 0; c < Cfg::kChunks; ++c) {
        if (aux_issued[c] > 0u && !mbar_wait_bounded(&aux_full[c], (aux_issued[c] - 1u) & 1u))
          atomicOr(&g_watchdog, MUON_POLAR_WATCHDOG_DRAIN);
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  if constexpr (PAIR == 2) cluster_sync();  // the leader's MMAs are done with both CTAs
  if (warp == 1) {
    tc_fence_after();
    if constexpr (PAIR == 2)
      tmem_dealloc_pair(tmem_base, Cfg::kTmemCols);
    else
      tmem_dealloc(tmem_base, Cfg::kTmemCols);
  }
}

// ============================================================ fused step
// One launch for a whole Polar Express step on tcgen05 CTA pairs.  The work
// items of the step -- Gram regions of every matrix, then polynomial
// regions, then apply tiles -- are dealt round-robin to the co-resident
// pairs; an item waits (bounded) until the items it reads are complete:
//   polynomial region of matrix b  <- every Gram region of b
//   apply tile of matrix b         <- every polynomial region of b
// Completion is counted per matrix in scratch (one increment per CTA and
// item, released after the CTA's TMA stores have completed; acquired with a
// proxy fence before the TMA loads of the dependent item).  Every dependency
// has a lower item index than its dependent and items of a pair run in
// index order, so every wait ends.  The last CTA to exit resets the
// counters, so each launch starts from zero.
//
// Tile shapes, all cta_group::2 (M = 256):
//  * Gram and polynomial items: 256 x 128 regions (N = 128).  A region
//    (I, j) covers 128-row blocks 2I and 2I+1 against 128-column block j,
//    j >= 2I: every block on or above the diagonal exactly once (block
//    (2I+1, 2I), below it, is computed and not stored; the mirror of block
//    (2I, 2I+1) writes it).  Per SM a 128 x 128 x 16 MMA reads 6 KiB of
//    shared memory (A: 128 rows, B: 64 rows) instead of the single-CTA
//    engine's 8 KiB, and twice as many SMs work on the Gram.
//  * Or (polar_fused_kernel<true>, when regions would take about three
//    rounds of the pairs) 256 x 256 tiles (N = 256) of the upper triangle:
//    half as many items; the blocks below the diagonal of a diagonal tile
//    are computed and not stored.
//  * Apply items: 256 x 256 tiles (N = 256), as the apply kernel.
// The stage ring (192 KiB) is cut per item kind: four 48 KiB stages of
// K = 128 for regions (three 64 KiB ones for wide tiles); four 32 KiB
// stages of K = 64 for apply items, whose epilogue tile (X, 64 KiB) takes
// the rest of the ring.  At a
// change of layout the producers wait until the previous item's MMAs have
// completed (its accumulator barrier), then restart the ring; each stage's
// barriers keep their own phase.  The Gram / polynomial epilogue stages its
// output and mirror chunks in two dedicated 16 KiB regions; the polynomial
// reads its A tile (the b*A term) straight from global memory into
// registers before its accumulator is ready.  An apply item's X operand and
// epilogue tile do not depend on the polynomial: they are loaded before the
// item waits for it (in steps after the first, once X -- the previous
// step's output for the matrix -- is complete).
enum FusedKind : int { kFGram = 0, kFPoly = 1, kFApply = 2 };

// Several Polar Express steps in one launch (muon_polar_express_sm100): the
// items of step s+1 follow those of step s, and a Gram region of matrix b in
// step s+1 waits for every apply tile of b in step s (its input).  X of step
// s is the launch input for s = 0, else one of two ping-pong buffers; Y of
// the last step is the launch output.  A, P and the buffers are per matrix,
// and every write to one of them waits (through the chain of per-matrix
// dependencies) until the previous step's readers of that matrix are done.
constexpr int kMaxFusedSteps = 8;

struct FusedParams {
  int32_t batch;
  int32_t d2;           // Mp / 256: row blocks of a region
  int32_t regions;      // Gram / polynomial items per matrix: d2 (d2 + 1)
                        // regions, or d2 (d2 + 1) / 2 wide 256 x 256 tiles
                        // (polar_fused_kernel<true>)
  int32_t apply_tn;     // ceil(n / 256)
  int32_t n_gram;       // batch * regions
  int32_t n_poly;       // batch * regions
  int32_t total;        // n_gram + n_poly + batch * d2 * apply_tn
  int32_t kb_gram;      // K-blocks of each kind (128 deep for Gram / poly,
  int32_t kb_poly;      // 64 for the apply)
  int32_t kb_apply;
  int32_t steps;        // Polar Express steps of this launch
  int32_t per_step;     // items of one step
  uint32_t apply_bands; // apply CTA bands per matrix (two per tile)
  float coef[kMaxFusedSteps][3];  // per step: b, c, a rounded to bf16
  // per matrix, counted over all steps: [0, batch) Gram, [batch, 2 batch)
  // poly, [2 batch, 3 batch) apply CTA parts done; [3 batch]: exits.  A
  // step's items of a matrix start only after the previous step's apply of
  // it is complete, so after step s the Gram and poly counts of the matrix
  // are exactly 2 regions (s + 1) and the apply count apply_bands (s + 1).
  uint32_t* counters;
  const uint16_t* gram; // A, [batch][mp][mp] bf16 (the polynomial's epilogue input)
  int32_t mp;
};

// X of a step (index 0: the launch input; 1, 2: ping-pong buffers) and Y
// (index 0: the launch output; 1, 2: the same buffers).
struct FusedMaps {
  CUtensorMap x_k[3];   // X, box {64, 128}: Gram A operand, apply epilogue tile
  CUtensorMap x_mn[3];  // X, box {64, 64}: Gram B operand (K-major), apply B operand (MN-major)
  CUtensorMap a128;     // A, box {64, 128}: Gram output, poly A operand and tile
  CUtensorMap a64;      // A, box {64, 64}: Gram mirror, poly B operand
  CUtensorMap p128;     // P, box {64, 128}: poly output, apply A operand
  CUtensorMap p64;      // P, box {64, 64}: poly mirror
  CUtensorMap y128[3];  // Y, box {64, 128}: apply output
};

__device__ __forceinline__ int fused_src(int step) { return step == 0 ? 0 : 1 + ((step - 1) & 1); }
__device__ __forceinline__ int fused_dst(int step, int steps) {
  return step == steps - 1 ? 0 : 1 + (step & 1);
}

struct FusedItem {
  int kind, b, tm, tn, k_blocks, step;
};

template <bool WIDE>
__device__ __forceinline__ FusedItem fused_item(int w_all, const FusedParams& p) {
  FusedItem it;
  it.step = w_all / p.per_step;
  const int w = w_all - it.step * p.per_step;
  int r;
  if (w < p.n_gram + p.n_poly) {
    it.kind = w < p.n_gram ? kFGram : kFPoly;
    it.k_blocks = w < p.n_gram ? p.kb_gram : p.kb_poly;
    r = w < p.n_gram ? w : w - p.n_gram;
    it.b = r / p.regions;
    r -= it.b * p.regions;
    int tm = 0;
    if (WIDE) {
      // row I holds tiles (I, I .. d2 - 1)
      while (r >= p.d2 - tm) {
        r -= p.d2 - tm;
        ++tm;
      }
      it.tn = tm + r;
    } else {
      // row I holds regions (I, 2I .. 2 d2 - 1)
      while (r >= 2 * p.d2 - 2 * tm) {
        r -= 2 * p.d2 - 2 * tm;
        ++tm;
      }
      it.tn = 2 * tm + r;
    }
    it.tm = tm;
  } else {
    it.kind = kFApply;
    it.k_blocks = p.kb_apply;
    r = w - p.n_gram - p.n_poly;
    const int per = p.d2 * p.apply_tn;
    it.b = r / per;
    r -= it.b * per;
    it.tm = r / p.apply_tn;
    it.tn = r - it.tm * p.apply_tn;
  }
  return it;
}

// Count of a matrix's Gram or poly CTA parts once `step` is complete.
__device__ __forceinline__ uint32_t fused_sym_done(const FusedParams& p, int step) {
  return 2u * static_cast<uint32_t>(p.regions) * static_cast<uint32_t>(step + 1);
}

// Waits (bounded) until X of the item's step -- the previous step's output
// for steps after the first -- is complete.
__device__ __forceinline__ bool fused_wait_x(const FusedItem& it, const FusedParams& p) {
  bool ok = true;
  if (it.step > 0) {
    ok = wait_counter_bounded(p.counters + 2 * p.batch + it.b,
                              p.apply_bands * static_cast<uint32_t>(it.step));
    fence_proxy_async_global();
  }
  return ok;
}

// Waits (bounded) until the item's inputs from this launch are complete.
__device__ __forceinline__ bool fused_wait_inputs(const FusedItem& it, const FusedParams& p) {
  bool ok = true;
  if (it.kind == kFGram)
    return fused_wait_x(it, p);
  if (it.kind == kFPoly)
    ok = wait_counter_bounded(p.counters + it.b, fused_sym_done(p, it.step));
  else
    ok = wait_counter_bounded(p.counters + p.batch + it.b, fused_sym_done(p, it.step));
  fence_proxy_async_global();
  return ok;
}

struct FusedCfg {
  static constexpr uint32_t kRegionBytes = kHalf * kChunkCols * 2;  // 16 KiB
  static constexpr uint32_t kEpiBytes = 2 * kRegionBytes;           // sym output + mirror
  static constexpr uint32_t kSymA = kHalf * 128 * 2;                // 32 KiB
  static constexpr uint32_t kSymB = 64 * 128 * 2;                   // 16 KiB
  static constexpr uint32_t kSymStage = kSymA + kSymB;
  static constexpr uint32_t kSymBW = 128 * 128 * 2;                 // 32 KiB, wide tiles
  static constexpr uint32_t kSymStageW = kSymA + kSymBW;            // 64 KiB
  static constexpr int kSymStagesW = 3;
  static constexpr uint32_t kApA = kHalf * kAtom * 2;               // 16 KiB
  static constexpr uint32_t kApB = kAtom * kHalf * 2;               // 16 KiB
  static constexpr uint32_t kApStage = kApA + kApB;
  static constexpr int kSymStages = 4;
  static constexpr int kApStages = 4;
  static constexpr uint32_t kRingBytes = kSymStages * kSymStage;    // 192 KiB
  static constexpr uint32_t kApAux = kApStages * kApStage;          // apply tile at 128 KiB
  static constexpr int kMaxStages = 4;
  static constexpr uint32_t kSmemBytes = 1024 + kEpiBytes + kRingBytes + 256;
  static constexpr uint32_t kTmemCols = 2 * kPairN;
  static_assert(kApAux + 4 * kRegionBytes <= kRingBytes, "apply layout");
  static_assert(kSymStagesW * kSymStageW <= kRingBytes, "wide layout");
  static_assert(kSmemBytes <= 232448, "shared memory budget");
};

// Polynomial epilogue of 32 accumulator columns with the A values (the b*A
// term) from registers: eight bf16 per 16-byte unit, in column order.  The
// arithmetic and staging are those of pair_epilogue_half<kPoly>.
__device__ __forceinline__ void fused_poly_half(const EpiParams& p, uint32_t out, uint32_t mir,
                                                bool mirror, int row, int h,
                                                const float (&v)[32], const uint4 (&aux)[4]) {
  uint32_t w[16];
#pragma unroll
  for (int u = 0; u < 4; ++u) {
    const uint32_t in[4] = {aux[u].x, aux[u].y, aux[u].z, aux[u].w};
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      const int j = 8 * u + 2 * e;
      const float2 a2 = __bfloat1622float2(bits_bf162(in[e]));
      w[4 * u + e] = bf162_bits(__floats2bfloat162_rn(
          __fadd_rn(__fmul_rn(p.coef_b, a2.x), __fmul_rn(p.coef_c, v[j])),
          __fadd_rn(__fmul_rn(p.coef_b, a2.y), __fmul_rn(p.coef_c, v[j + 1]))));
    }
    st_shared_v4(out + swz_box(row, h * 64 + u * 16),
                 make_uint4(w[4 * u], w[4 * u + 1], w[4 * u + 2], w[4 * u + 3]));
  }
  if (mirror) {
    const uint32_t mbase = mir + (row / 64) * (kChunkCols * 128);
#pragma unroll
    for (int j = 0; j < 32; ++j) {
      const uint16_t hv = static_cast<uint16_t>((j & 1) ? (w[j >> 1] >> 16) : (w[j >> 1] & 0xFFFFu));
      st_shared_u16(mbase + swz_box(h * 32 + j, (row % 64) * 2), hv);
    }
  }
}

// Stage ring of one role: the current layout (0 none yet, 1 Gram /
// polynomial, 2 apply), its stage count, the position in it and, per stage,
// the parity of the barrier phase it waits for next.
struct FusedRing {
  int layout;
  int stages;
  int pos;
  uint32_t parity;  // bit s: phases of stage s used so far, mod 2
};

template <bool WIDE>
__global__ void __launch_bounds__(kTileThreads, 1)
    polar_fused_kernel(const __grid_constant__ FusedMaps maps, const FusedParams p) {
  using Cfg = FusedCfg;
  constexpr int S = Cfg::kMaxStages;

  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw_addr = smem_addr(smem_raw);
  uint8_t* smem = smem_raw + ((1024u - (raw_addr & 1023u)) & 1023u);
  uint8_t* sReg = smem;  // sym epilogue: output chunk, mirror chunk
  uint8_t* sRing = smem + Cfg::kEpiBytes;
  uint8_t* sAux = sRing + Cfg::kApAux;  // apply epilogue tile (apply layout only)
  uint64_t* full = reinterpret_cast<uint64_t*>(sRing + Cfg::kRingBytes);
  uint64_t* empty = full + S;
  uint64_t* tfull = empty + S;
  uint64_t* tempty = tfull + 2;
  uint64_t* drain = tempty + 2;
  uint64_t* aux_full = drain + 1;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(aux_full + 1);
  // Items of this cluster whose epilogue is finished with the apply tile
  // area (the epilogue leader writes it, the producers poll it).
  uint32_t* epi_done = tmem_slot + 1;

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const uint32_t rank = cluster_cta_rank();
  const int cluster = static_cast<int>(blockIdx.x >> 1);
  const int nclusters = static_cast<int>(gridDim.x >> 1);
  constexpr int kEpiLeader = 64;

  if (threadIdx.x == 0) {
    for (int s = 0; s < S; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int a = 0; a < 2; ++a) {
      mbar_init(&tfull[a], 1);
      mbar_init(&tempty[a], 16);  // 8 epilogue warps in each CTA
    }
    mbar_init(drain, 1);
    mbar_init(aux_full, 1);
    *epi_done = 0u;
    fence_mbar_init();
    for (int i = 0; i < 3; ++i) {
      prefetch_tensor_map(&maps.x_k[i]);
      prefetch_tensor_map(&maps.x_mn[i]);
      prefetch_tensor_map(&maps.y128[i]);
    }
    prefetch_tensor_map(&maps.a128);
    prefetch_tensor_map(&maps.a64);
    prefetch_tensor_map(&maps.p128);
    prefetch_tensor_map(&maps.p64);
  }
  if (warp == 1) {
    tmem_alloc_pair(tmem_slot, Cfg::kTmemCols);
    tmem_relinquish_pair();
  }
  tc_fence_before();
  __syncthreads();
  cluster_sync();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  grid_dependency_wait();
  grid_launch_dependents();

  if (warp == 0 || warp == kProducerWarp2) {
    if (lane == 0) {
      // ---------------- TMA producers (both CTAs): producer `pid` owns the
      // stages s with s % 2 == pid in either layout.
      const uint32_t pid = warp == 0 ? 0u : 1u;
      FusedRing ring = {0, 0, 0, 0u};
      uint32_t t = 0;
      int started = 0;  // items whose loads this producer has begun
      // Sym stages 2 and 3 overlap the apply tile area: after an apply item
      // they are loaded only once the epilogue is done with items < aux_wait.
      uint32_t aux_wait = 0;
      bool ok = true;
      for (int w = cluster; ok && w < p.total; w += nclusters, ++t) {
        const FusedItem item = fused_item<WIDE>(w, p);
        const bool ap = item.kind == kFApply;
        const int layout = ap ? 2 : 1;
        if (layout != ring.layout) {
          // new layout: the previous item's MMAs have read every stage
          if (t > 0 && !mbar_wait_bounded(&tfull[(t - 1) & 1u], ((t - 1) >> 1) & 1u)) {
            ok = false;
            break;
          }
          if (!ap && ring.layout == 2) aux_wait = t;
          ring.layout = layout;
          ring.stages = ap ? Cfg::kApStages : (WIDE ? Cfg::kSymStagesW : Cfg::kSymStages);
          ring.pos = 0;
        }
        started = static_cast<int>(t) + 1;
        const uint32_t stage_bytes =
            ap ? Cfg::kApStage : (WIDE ? Cfg::kSymStageW : Cfg::kSymStage);
        const uint32_t a_bytes = ap ? Cfg::kApA : Cfg::kSymA;
        const int a_row = item.tm * kPairM + static_cast<int>(rank) * kHalf;
        // Apply: X (B operand) of the first stages before the dependency
        // wait; Gram: no dependency; polynomial: A only after it.
        const int src = fused_src(item.step);
        FusedRing pre = ring;
        int n_pre = 0;
        if (ap) {
          // X of a later step is the previous step's output
          if (!fused_wait_x(item, p)) {
            atomicOr(&g_watchdog, MUON_POLAR_WATCHDOG_DEPENDENCY);
            ok = false;
            break;
          }
          for (int kb = 0; kb < item.k_blocks && kb < ring.stages; ++kb, ++n_pre) {
            const int s = pre.pos;
            pre.pos = pre.pos + 1 == pre.stages ? 0 : pre.pos + 1;
            if ((s & 1) != static_cast<int>(pid)) continue;
            const uint32_t par = (pre.parity >> s) & 1u;
            if (!mbar_wait_bounded(&empty[s], par ^ 1u)) {
              ok = false;
              break;
            }
            if (rank == 0) mbar_arrive_expect_tx(&full[s], 2 * stage_bytes);
            const uint32_t bar = map_to_cta(smem_addr(&full[s]), 0);
            uint8_t* sb = sRing + s * stage_bytes + a_bytes;
#pragma unroll
            for (int j = 0; j < kHalf / kAtom; ++j)
              tma_load_3d_pair(sb + j * (kAtom * 128), &maps.x_mn[src], bar,
                               item.tn * kPairN + static_cast<int>(rank) * kHalf + j * kAtom,
                               kb * kAtom, item.b);
          }
          if (!ok) break;
        }
        if (!fused_wait_inputs(item, p)) {
          atomicOr(&g_watchdog, MUON_POLAR_WATCHDOG_DEPENDENCY);
          ok = false;
          break;
        }
        for (int kb = 0; kb < item.k_blocks; ++kb) {
          const int s = ring.pos;
          ring.pos = ring.pos + 1 == ring.stages ? 0 : ring.pos + 1;
          if ((s & 1) != static_cast<int>(pid)) continue;
          const uint32_t par = (ring.parity >> s) & 1u;
          ring.parity ^= 1u << s;
          const uint32_t bar = map_to_cta(smem_addr(&full[s]), 0);
          uint8_t* sa = sRing + s * stage_bytes;
          if (ap) {
            if (kb >= n_pre) {
              if (!mbar_wait_bounded(&empty[s], par ^ 1u)) {
                ok = false;
                break;
              }
              if (rank == 0) mbar_arrive_expect_tx(&full[s], 2 * stage_bytes);
#pragma unroll
              for (int j = 0; j < kHalf / kAtom; ++j)
                tma_load_3d_pair(sa + a_bytes + j * (kAtom * 128), &maps.x_mn[src], bar,
                                 item.tn * kPairN + static_cast<int>(rank) * kHalf + j * kAtom,
                                 kb * kAtom, item.b);
            }
            tma_load_3d_pair(sa, &maps.p128, bar, kb * kAtom, a_row, item.b);
          } else {
            if (aux_wait > 0 && s >= 2) {
              if (!wait_shared_bounded(smem_addr(epi_done), aux_wait)) {
                ok = false;
                break;
              }
              aux_wait = 0;
            }
            if (!mbar_wait_bounded(&empty[s], par ^ 1u)) {
              ok = false;
              break;
            }
            if (rank == 0) mbar_arrive_expect_tx(&full[s], 2 * stage_bytes);
            const CUtensorMap* ma = item.kind == kFGram ? &maps.x_k[src] : &maps.a128;
            // B: this CTA's half of the item's columns -- 64 rows of a
            // region, 128 of a wide tile (the same maps as A)
            const CUtensorMap* mb =
                WIDE ? ma : (item.kind == kFGram ? &maps.x_mn[src] : &maps.a64);
            const int b_row = WIDE ? item.tn * kPairN + static_cast<int>(rank) * kHalf
                                     : item.tn * kHalf + static_cast<int>(rank) * 64;
            const uint32_t b_atom = WIDE ? kAtomBytes : 64 * 128;
#pragma unroll
            for (int j = 0; j < 2; ++j) {
              tma_load_3d_pair(sa + j * kAtomBytes, ma, bar, kb * 128 + j * kAtom, a_row, item.b);
              tma_load_3d_pair(sa + a_bytes + j * b_atom, mb, bar, kb * 128 + j * kAtom, b_row,
                               item.b);
            }
          }
        }
      }
      if (!ok) atomicOr(&g_watchdog, MUON_POLAR_WATCHDOG_PRODUCER);
      if (rank == 0 && started > 0) {
        // Drain: the pair's last loads land before the CTAs exit (the last
        // item's accumulator completes only after every one of its stages).
        const uint32_t last = static_cast<uint32_t>(started - 1);
        if (!mbar_wait_bounded(&tfull[last & 1u], (last >> 1) & 1u))
          atomicOr(&g_watchdog, MUON_POLAR_WATCHDOG_DRAIN);
      }
    }
  } else if (warp == 1) {
    if (lane == 0 && rank == 0) {
      // ---------------- tcgen05 MMA issuer (leader CTA only)
      constexpr uint32_t idesc_sym = idesc_bf16_f32(kHalf, 0u, kPairM);
      constexpr uint32_t idesc_sym_w = idesc_bf16_f32(kPairN, 0u, kPairM);
      constexpr uint32_t idesc_ap = idesc_bf16_f32(kPairN, 1u, kPairM);
      const uint32_t idesc_s = WIDE ? idesc_sym_w : idesc_sym;
      const uint32_t b_atom = WIDE ? kAtomBytes : 64 * 128;
      FusedRing ring = {0, 0, 0, 0u};
      uint32_t t = 0;
      bool ok = true;
      for (int w = cluster; ok && w < p.total; w += nclusters, ++t) {
        const FusedItem item = fused_item<WIDE>(w, p);
        const bool ap = item.kind == kFApply;
        const int layout = ap ? 2 : 1;
        if (layout != ring.layout) {
          ring.layout = layout;
          ring.stages = ap ? Cfg::kApStages : (WIDE ? Cfg::kSymStagesW : Cfg::kSymStages);
          ring.pos = 0;
        }
        const uint32_t stage_bytes =
            ap ? Cfg::kApStage : (WIDE ? Cfg::kSymStageW : Cfg::kSymStage);
        const uint32_t a_bytes = ap ? Cfg::kApA : Cfg::kSymA;
        const uint32_t acc = t & 1u;
        if (!mbar_wait_bounded(&tempty[acc], ((t >> 1) & 1u) ^ 1u)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + acc * kPairN;
        for (int kb = 0; kb < item.k_blocks; ++kb) {
          const int s = ring.pos;
          ring.pos = ring.pos + 1 == ring.stages ? 0 : ring.pos + 1;
          const uint32_t par = (ring.parity >> s) & 1u;
          ring.parity ^= 1u << s;
          if (!mbar_wait_bounded(&full[s], par)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t a_base = smem_addr(sRing + s * stage_bytes);
          const uint32_t b_base = a_base + a_bytes;
          if (ap) {
#pragma unroll
            for (int k = 0; k < kAtom / 16; ++k)
              umma_bf16_pair(d_tmem, smem_desc_sw128(a_base + k * 32, 16, 1024),
                             smem_desc_sw128(b_base + k * 2048, kAtom * 128, 1024), idesc_ap,
                             (kb > 0 || k > 0) ? 1u : 0u);
          } else {
            // K-major: step k lies in swizzle atom k/4 (A atoms of 128 rows,
            // 16 KiB apart; B atoms of 64 rows, 8 KiB apart, or of 128 rows
            // for wide tiles)
#pragma unroll
            for (int k = 0; k < 128 / 16; ++k)
              umma_bf16_pair(d_tmem,
                             smem_desc_sw128(a_base + (k / 4) * kAtomBytes + (k % 4) * 32, 16,
                                             1024),
                             smem_desc_sw128(b_base + (k / 4) * b_atom + (k % 4) * 32, 16,
                                             1024),
                             idesc_s, (kb > 0 || k > 0) ? 1u : 0u);
          }
          umma_commit_pair(map_to_cta(smem_addr(&empty[s]), 0));
          umma_commit_pair(map_to_cta(smem_addr(&empty[s]), 1));
        }
        if (!ok) break;
        umma_commit_pair(map_to_cta(smem_addr(&tfull[acc]), 0));
        umma_commit_pair(map_to_cta(smem_addr(&tfull[acc]), 1));
      }
      if (!ok) atomicOr(&g_watchdog, MUON_POLAR_WATCHDOG_MMA);
      umma_commit_pair(map_to_cta(smem_addr(drain), 0));
      if (!mbar_wait_bounded(drain, 0)) atomicOr(&g_watchdog, MUON_POLAR_WATCHDOG_DRAIN);
    }
  } else {
    // ---------------- epilogue warps 2..9 (both CTAs)
    const int q = warp & 3;
    const int hc = (warp - 2) >> 2;
    const int row = q * 32 + lane;
    const uint32_t reg_base = smem_addr(sReg);
    const bool leader = threadIdx.x == kEpiLeader;
    const uint32_t tempty_leader0 = map_to_cta(smem_addr(&tempty[0]), 0);
    const uint32_t tempty_leader1 = map_to_cta(smem_addr(&tempty[1]), 0);
    EpiParams ep = {};
    bool aux_inflight = false;
    // Failures never change the epilogue's control flow: every thread runs
    // the same named barriers for every item, and after a failed wait it only
    // skips its waits, reads and stores (the watchdog word records why).
    bool failed = false;
    // This CTA's 128-row block of a Gram / polynomial item against the
    // 128-column block of chunk c: above the diagonal (stored with its
    // mirror), on it (stored), or below it (not stored).  Along an item's
    // chunks the relation never decreases.
    auto chunk_rel = [&](const FusedItem& it, int c) {
      const int br = 2 * it.tm + static_cast<int>(rank);
      const int bc = WIDE ? 2 * it.tn + (c >> 1) : it.tn;
      return br < bc ? 1 : (br == bc ? 0 : -1);
    };
    // Leader: the epilogue tile of apply item w (X: no wait), into the
    // ring's apply tile area -- free once the previous item's MMAs and
    // stores are done with it.  If X's wait gives up, nothing is loaded:
    // the epilogue skips every later wait and load, so no copy is left in
    // flight when the CTA exits.
    auto load_aux = [&](int w) {
      const FusedItem item = fused_item<WIDE>(w, p);
      if (item.kind != kFApply) return;
      if (!fused_wait_x(item, p)) {
        atomicOr(&g_watchdog, MUON_POLAR_WATCHDOG_DEPENDENCY);
        failed = true;
        return;
      }
      mbar_arrive_expect_tx(aux_full, 4 * Cfg::kRegionBytes);
#pragma unroll
      for (int c = 0; c < 4; ++c)
        tma_load_3d(sAux + c * Cfg::kRegionBytes, &maps.x_k[fused_src(item.step)], aux_full,
                    item.tn * kPairN + c * kChunkCols,
                    item.tm * kPairM + static_cast<int>(rank) * kHalf, item.b);
      aux_inflight = true;
    };
    auto release_accumulator = [&](uint32_t acc) {
      tc_fence_before();
      __syncwarp();
      if (lane == 0) {
        if (rank == 0)
          mbar_arrive(&tempty[acc]);
        else
          mbar_arrive_cluster(acc ? tempty_leader1 : tempty_leader0);
      }
    };
    if (leader && cluster < p.total) load_aux(cluster);
    uint32_t t = 0;
    uint32_t aux_uses = 0;  // completed aux_full phases
    for (int w = cluster; w < p.total; w += nclusters, ++t) {
      const FusedItem item = fused_item<WIDE>(w, p);
      const bool ap = item.kind == kFApply;
      // chunks [c_first, chunks) of this CTA's band are stored
      const int chunks = (ap || WIDE) ? 4 : 2;
      int c_first = 0;
      if (!ap)
        while (c_first < chunks && chunk_rel(item, c_first) < 0) ++c_first;
      const bool has_aux = ap;
      const uint32_t acc = t & 1u;
      ep.coef_b = p.coef[item.step][0];
      ep.coef_c = p.coef[item.step][1];
      ep.alpha = p.coef[item.step][2];
      const int row0 = item.tm * kPairM + static_cast<int>(rank) * kHalf;
      const int col0 = item.tn * ((ap || WIDE) ? kPairN : kHalf);
      // Polynomial: this thread's A values (row `row`, columns hc*32.. of
      // a chunk) from global memory, the first two chunks' requested before
      // the accumulator is ready, chunk c + 2's once chunk c is done.  The
      // Gram of the matrix is complete (acquired per warp).
      uint4 pa[2][4];
      const uint16_t* psrc = nullptr;
      if (item.kind == kFPoly && c_first < chunks && !failed) {
        int dep = 1;
        if (lane == 0)
          dep = wait_counter_bounded(p.counters + item.b, fused_sym_done(p, item.step)) ? 1 : 0;
        dep = __shfl_sync(0xffffffffu, dep, 0);
        if (!dep) {
          if (lane == 0) atomicOr(&g_watchdog, MUON_POLAR_WATCHDOG_DEPENDENCY);
          failed = true;
        } else {
          psrc = p.gram + (static_cast<size_t>(item.b) * p.mp + row0 + row) * p.mp + col0 +
                 hc * 32;
          // (constant indices into pa: it stays in registers)
#pragma unroll
          for (int c = 0; c < 4; ++c) {
            if (c >= c_first && c < c_first + 2 && c < chunks) {
#pragma unroll
              for (int u = 0; u < 4; ++u)
                pa[c & 1][u] = __ldcg(reinterpret_cast<const uint4*>(psrc + c * kChunkCols + u * 8));
            }
          }
        }
      }
      int ok = failed ? 0 : 1;
      if (lane == 0 && ok) {
        ok = mbar_wait_bounded(&tfull[acc], (t >> 1) & 1u) ? 1 : 0;
        if (has_aux && ok) ok = mbar_wait_bounded(aux_full, aux_uses & 1u) ? 1 : 0;
        if (!ok) atomicOr(&g_watchdog, MUON_POLAR_WATCHDOG_EPILOGUE);
      }
      ok = __shfl_sync(0xffffffffu, ok, 0);
      if (!ok) failed = true;
      if (has_aux) {
        // every thread acquires the epilogue input the TMA wrote
        if (!failed) (void)mbar_try_wait(aux_full, aux_uses & 1u);
        ++aux_uses;
        if (leader) aux_inflight = false;
      }
      tc_fence_after();
      const uint32_t t_row = tmem_base + (static_cast<uint32_t>(q * 32) << 16) + acc * kPairN;
      const CUtensorMap* m_out = item.kind == kFGram   ? &maps.a128
                                 : item.kind == kFPoly ? &maps.p128
                                                       : &maps.y128[fused_dst(item.step, p.steps)];
      const CUtensorMap* m_mir = item.kind == kFGram ? &maps.a64 : &maps.p64;
      if (c_first >= chunks) release_accumulator(acc);
      // Accumulator chunk c + 1 is read from tensor memory while chunk c is
      // processed.  Apply: chunk c in place of its X chunk in the tile area.
      // Gram / polynomial: output chunk in region 0, mirror chunk in region
      // 1, reused by chunk 1 once chunk 0's stores have read them.
      const uint32_t aux_base = smem_addr(sAux);
      uint32_t rbuf[2][32];
      if (c_first < chunks && !failed) {
        if (c_first & 1)
          tmem_ld_32x32b_x32(t_row + c_first * kChunkCols + hc * 32, rbuf[1]);
        else
          tmem_ld_32x32b_x32(t_row + c_first * kChunkCols + hc * 32, rbuf[0]);
      }
#pragma unroll
      for (int c = 0; c < 4; ++c) {
        if (c < c_first) continue;
        if (c >= chunks) break;
        const bool mirror = !ap && chunk_rel(item, c) > 0;
        const uint32_t out = ap ? aux_base + c * Cfg::kRegionBytes : reg_base;
        const uint32_t mir = reg_base + Cfg::kRegionBytes;
        if (!ap && c > c_first) {
          if (leader) bulk_wait_group_read<0>();
          named_barrier(1, kPairEpiThreads);
        }
        if (!failed) {
          tmem_wait_ld(rbuf[c & 1]);
          if (c + 1 < chunks)
            tmem_ld_32x32b_x32(t_row + (c + 1) * kChunkCols + hc * 32, rbuf[(c + 1) & 1]);
        }
        if (c + 1 == chunks) release_accumulator(acc);
        if (!failed) {
          float v[32];
#pragma unroll
          for (int j = 0; j < 32; ++j) v[j] = __uint_as_float(rbuf[c & 1][j]);
          if (item.kind == kFGram)
            pair_epilogue_half<kGramBf16>(ep, out, mir, mirror, row, hc, v);
          else if (item.kind == kFPoly)
            fused_poly_half(ep, out, mir, mirror, row, hc, v, pa[c & 1]);
          else
            pair_epilogue_half<kApply>(ep, out, mir, false, row, hc, v);
          if (item.kind == kFPoly && psrc != nullptr && c + 2 < chunks) {
#pragma unroll
            for (int u = 0; u < 4; ++u)
              pa[c & 1][u] =
                  __ldcg(reinterpret_cast<const uint4*>(psrc + (c + 2) * kChunkCols + u * 8));
          }
        }
        fence_proxy_async_smem();
        named_barrier(1, kPairEpiThreads);
        if (leader && !failed) {
          tma_store_3d(m_out, ap ? sAux + c * Cfg::kRegionBytes : sReg, col0 + c * kChunkCols,
                       row0, item.b);
          if (mirror) {
#pragma unroll
            for (int h = 0; h < kHalf / kChunkCols; ++h)
              tma_store_3d(m_mir, sReg + Cfg::kRegionBytes + h * (kChunkCols * 128),
                           row0 + h * kChunkCols, col0 + c * kChunkCols, item.b);
          }
          bulk_commit_group();
        }
      }
      if (leader) {
        if (!ap || item.step + 1 < p.steps) {
          // Publish this CTA's part of the item once its stores have landed
          // (also when it stored nothing or gave up: the count is per CTA
          // and item).  An apply tile is waited for only by the next step.
          bulk_wait_group0();
          fence_proxy_async_global();
          const int slot = item.kind == kFGram ? 0 : (item.kind == kFPoly ? 1 : 2);
          red_release_gpu_add(p.counters + slot * p.batch + item.b, 1u);
        } else {
          bulk_wait_group_read<0>();
        }
        // every epilogue thread has read the apply tile (named barrier before
        // the last store) and the stores have read it
        st_release_cta_shared(smem_addr(epi_done), t + 1);
        const int next = w + nclusters;
        if (next < p.total && !failed) load_aux(next);
      }
      // the regions are free (stores have read them) before the next item
      // writes them
      named_barrier(1, kPairEpiThreads);
    }
    if (leader) {
      bulk_wait_group0();
      if (aux_inflight && !mbar_wait_bounded(aux_full, aux_uses & 1u))
        atomicOr(&g_watchdog, MUON_POLAR_WATCHDOG_DRAIN);
    }
  }

  tc_fence_before();
  __syncthreads();
  cluster_sync();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc_pair(tmem_base, Cfg::kTmemCols);
  }
  // The last CTA out resets the dependency counters for the next launch.
  if (threadIdx.x == 0) {
    __threadfence();
    const int n_ctr = 3 * p.batch;
    const uint32_t exits = atomicAdd(p.counters + n_ctr, 1u);
    if (exits == gridDim.x - 1) {
      for (int i = 0; i <= n_ctr; ++i) p.counters[i] = 0u;
      __threadfence();
    }
  }
}

__global__ void cast_f32_bf16_kernel(const float* __restrict__ src,
                                     uint16_t* __restrict__ dst,
                                     int64_t count) {
  grid_dependency_wait();
  grid_launch_dependents();
  const int64_t stride = static_cast<int64_t>(gridDim.x) * blockDim.x;
  for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
       i < count; i += stride)
    dst[i] = static_cast<uint16_t>(float_to_bf16_bits(src[i]));
}

// Packed upper-triangle units -> full symmetric matrix, bf16.  One CTA per
// 128 x 128 quarter (r, s) of unit (I, J) of matrix b: the quarter goes to
// rows I*256 + r*128, columns J*256 + s*128 of `full`, and its transpose to
// the mirrored place unless it lies on the diagonal.  The lower-left
// quarter of a diagonal unit is not read: it is the mirror of the upper
// right one (the Gram on single-CTA tiles never writes it).
__global__ void __launch_bounds__(256) unpack_sym_kernel(const uint16_t* __restrict__ packed,
                                                         uint16_t* __restrict__ full, int d2,
                                                         int units, int64_t mp) {
  __shared__ uint32_t tile[128][65];  // 128 rows x 128 bf16, one word of padding
  grid_dependency_wait();
  grid_launch_dependents();
  const int u = static_cast<int>(blockIdx.x) >> 2;
  const int r = (blockIdx.x >> 1) & 1, sq = blockIdx.x & 1;
  const int b = blockIdx.y;
  int I = 0, rem = u;
  while (rem >= d2 - I) {
    rem -= d2 - I;
    ++I;
  }
  const int J = I + rem;
  if (I == J && r == 1 && sq == 0) return;
  const int64_t R0 = static_cast<int64_t>(I) * 256 + r * 128;
  const int64_t C0 = static_cast<int64_t>(J) * 256 + sq * 128;
  const uint16_t* src = packed + ((static_cast<int64_t>(b) * units + u) * 256 + r * 128) * 256 + sq * 128;
  uint16_t* dst = full + static_cast<int64_t>(b) * mp * mp;
  const bool mirror = !(I == J && r == sq);
#pragma unroll 2
  for (int i = 0; i < 8; ++i) {
    const int e = i * 256 + threadIdx.x;  // 16-byte unit: row e / 16, column (e % 16) * 8
    const int row = e >> 4, q = e & 15;
    const uint4 v = *reinterpret_cast<const uint4*>(src + row * 256 + q * 8);
    *reinterpret_cast<uint4*>(dst + (R0 + row) * mp + C0 + q * 8) = v;
    if (mirror) {
      tile[row][q * 4 + 0] = v.x;
      tile[row][q * 4 + 1] = v.y;
      tile[row][q * 4 + 2] = v.z;
      tile[row][q * 4 + 3] = v.w;
    }
  }
  if (!mirror) return;
  __syncthreads();
  const uint16_t* t16 = reinterpret_cast<const uint16_t*>(&tile[0][0]);
#pragma unroll 2
  for (int i = 0; i < 8; ++i) {
    const int e = i * 256 + threadIdx.x;  // output row rr = column rr of the quarter
    const int rr = e >> 4, q = e & 15;
    uint32_t w[4];
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      const uint32_t lo = t16[(q * 8 + 2 * k) * 130 + rr];
      const uint32_t hi = t16[(q * 8 + 2 * k + 1) * 130 + rr];
      w[k] = lo | (hi << 16);
    }
    *reinterpret_cast<uint4*>(dst + (C0 + rr) * mp + R0 + q * 8) = make_uint4(w[0], w[1], w[2], w[3]);
  }
}

// ============================================================== host side

namespace {

std::atomic<uint64_t> g_launch_count{0};

constexpr int kMaxDevices = 64;
constexpr int kNumInstances = 2 * kNumKinds;

struct DeviceState {
  std::once_flag once;
  int sms = 0;
  int cc_major = 0, cc_minor = 0;
  bool smem_attr_set[kNumInstances] = {};
  bool smem_attr_set_halves[kNumInstances] = {};  // the HALVES kernels
  bool smem_attr_set_deep[2] = {};  // the kDeepBK Gram kernels: whole tiles, halves
  int capacity[kNumInstances] = {};  // tiles worked on at once (tile_capacity)
};
DeviceState g_devices[kMaxDevices];
std::mutex g_attr_mutex;

typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t,
                                  void*, const cuuint64_t*, const cuuint64_t*,
                                  const cuuint32_t*, const cuuint32_t*,
                                  CUtensorMapInterleave, CUtensorMapSwizzle,
                                  CUtensorMapL2promotion,
                                  CUtensorMapFloatOOBfill);
std::once_flag g_encode_once;
EncodeTiledFn g_encode = nullptr;

EncodeTiledFn encode_fn() {
  std::call_once(g_encode_once, [] {
    void* fn = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &fn, cudaEnableDefault,
                                &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      g_encode = reinterpret_cast<EncodeTiledFn>(fn);
  });
  return g_encode;
}

int current_device_state(DeviceState** out) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return static_cast<int>(e);
  if (dev < 0 || dev >= kMaxDevices) return MUON_POLAR_ERR_UNSUPPORTED_DEVICE;
  DeviceState* st = &g_devices[dev];
  std::call_once(st->once, [st, dev] {
    cudaDeviceGetAttribute(&st->sms, cudaDevAttrMultiProcessorCount, dev);
    cudaDeviceGetAttribute(&st->cc_major, cudaDevAttrComputeCapabilityMajor, dev);
    cudaDeviceGetAttribute(&st->cc_minor, cudaDevAttrComputeCapabilityMinor, dev);
  });
  if (st->cc_major != 10 || st->cc_minor != 0 || st->sms <= 0)
    return MUON_POLAR_ERR_UNSUPPORTED_DEVICE;
  *out = st;
  return MUON_POLAR_OK;
}

// 3-D tiled map over a row-major [d2][d1][d0] tensor (d0 innermost), 128-byte
// swizzle, out-of-bounds elements read as zero.
// Encoded maps, memoised.  A map is a pure function of the arguments of
// encode_3d (the address is part of the key, and device addresses are unique
// across devices), so an entry stays valid even after its buffer is freed
// and another takes the same address: it is what encoding again would give.
// 4-way set-associative on a mixed hash of the key, round-robin replacement
// within a set; a step launches three to five maps per kernel, and a hit
// replaces the driver's encode by a compare and a copy.
struct MapKey {
  uint64_t v[7];
  bool operator==(const MapKey& o) const {
    for (int i = 0; i < 7; ++i)
      if (v[i] != o.v[i]) return false;
    return true;
  }
};
struct MapCacheEntry {
  MapKey key;
  CUtensorMap map;
  bool valid;
};
constexpr int kMapCacheSets = 128;
constexpr int kMapCacheWays = 4;
std::mutex g_map_mutex;
MapCacheEntry g_map_cache[kMapCacheSets][kMapCacheWays];
uint8_t g_map_victim[kMapCacheSets];
std::atomic<uint64_t> g_map_encodes{0};

uint64_t mix64(uint64_t z) {  // splitmix64 finaliser
  z = (z ^ (z >> 30)) * 0xbf58476d1ce4e5b9ull;
  z = (z ^ (z >> 27)) * 0x94d049bb133111ebull;
  return z ^ (z >> 31);
}

int encode_3d(CUtensorMap* map, CUtensorMapDataType dtype, size_t elem_bytes,
              const void* base, uint64_t d0, uint64_t d1, uint64_t d2,
              uint64_t stride1_elems, uint64_t stride2_elems, uint32_t box0,
              uint32_t box1) {
  const MapKey key = {{reinterpret_cast<uintptr_t>(base), d0, d1, d2, stride1_elems,
                       stride2_elems,
                       (static_cast<uint64_t>(dtype) << 48) |
                           (static_cast<uint64_t>(elem_bytes) << 40) |
                           (static_cast<uint64_t>(box0) << 20) | box1}};
  uint64_t h = 0;
  for (uint64_t w : key.v) h = mix64(h ^ w);
  const int set = static_cast<int>(h % kMapCacheSets);
  {
    std::lock_guard<std::mutex> lock(g_map_mutex);
    for (MapCacheEntry& e : g_map_cache[set]) {
      if (e.valid && e.key == key) {
        *map = e.map;
        return MUON_POLAR_OK;
      }
    }
  }
  EncodeTiledFn fn = encode_fn();
  if (fn == nullptr) return MUON_POLAR_ERR_DRIVER;
  const cuuint64_t dims[3] = {d0, d1, d2};
  const cuuint64_t strides[2] = {stride1_elems * elem_bytes,
                                 stride2_elems * elem_bytes};
  const cuuint32_t box[3] = {box0, box1, 1};
  const cuuint32_t estr[3] = {1, 1, 1};
  CUresult r = fn(map, dtype, 3, const_cast<void*>(base), dims, strides, box,
                  estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                  CU_TENSOR_MAP_SWIZZLE_128B,
                  CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                  CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return MUON_POLAR_ERR_TENSOR_MAP;
  g_map_encodes.fetch_add(1, std::memory_order_relaxed);
  std::lock_guard<std::mutex> lock(g_map_mutex);
  MapCacheEntry& slot = g_map_cache[set][g_map_victim[set]];
  g_map_victim[set] = static_cast<uint8_t>((g_map_victim[set] + 1) % kMapCacheWays);
  slot.key = key;
  slot.map = *map;
  slot.valid = true;
  return MUON_POLAR_OK;
}

bool aligned16(const void* p) {
  return (reinterpret_cast<uintptr_t>(p) & 15u) == 0;
}

// Rows of the square A / P buffers: a multiple of the 256-row pair tile.
int64_t padded_rows(int64_t m) { return (m + kPairM - 1) / kPairM * kPairM; }

struct TileMaps {
  CUtensorMap a, b, aux, out, mir;
};

// Slot of (KIND, PAIR) in the per-device caches.
template <int KIND, int PAIR>
constexpr int instance_of() {
  return (PAIR - 1) * kNumKinds + KIND;
}
static_assert(instance_of<kNumKinds - 1, 2>() < kNumInstances, "instance slots");

// Kernel choice: 0 = by size (the engine with the smaller estimated time,
// see use_pairs), 1 = always CTA pairs, 2 = never.  Initial value from
// MUON_POLAR_PAIR.
std::atomic<int> g_policy{[] {
  const char* s = std::getenv("MUON_POLAR_PAIR");
  if (s == nullptr) return 0;
  const int v = std::atoi(s);
  return v == 1 ? 1 : (v == 0 ? 2 : 0);
}()};

// Estimated time of a launch: rounds of tiles over the device, times the
// pipeline iterations per tile, times the measured cost of one iteration
// (B200: a CTA pair's 256 x 256 x 64 step about 0.33 us, a single CTA's
// 128 x 128 x 128 step about 0.45 us; the latter is bound by shared-memory
// bandwidth, both operands of every MMA being read from it).
double engine_cost(int64_t tiles, int units, int64_t k_blocks, int pair) {
  // (k_blocks: K / 64 on pairs, K / 128 on single CTAs; see cost_blocks)
  const int64_t rounds = (tiles + units - 1) / units;
  return static_cast<double>(rounds) * static_cast<double>(k_blocks) * (pair == 2 ? 1.0 : 1.36);
}

template <int PAIR>
int64_t cost_blocks(int64_t k) {
  return PAIR == 2 ? (k + 63) / 64 : (k + 127) / 128;
}

// Whether a launch runs on CTA pairs, given each engine's tile count, the
// tiles it works on at once and its K steps per tile (64 deep on pairs, 128
// on single CTAs).
bool use_pairs(int64_t tiles2, int units2, int64_t kb2, int64_t tiles1, int units1,
               int64_t kb1) {
  const int policy = g_policy.load(std::memory_order_relaxed);
  if (policy == 1) return true;
  if (policy == 2) return false;
  return engine_cost(tiles2, units2, kb2, 2) <= engine_cost(tiles1, units1, kb1, 1);
}

// Split-K of the symmetric kinds: when a problem has fewer tiles than the
// device works on at once, each tile's K range is cut into up to kMaxSplits
// work items.  Scratch layout: kCounterBytes of arrival counters (one per
// tile and CTA band, zero between launches) followed by the fp32 partial
// bands, PAIR bands of 128 x tile-width floats per item.
constexpr size_t kCounterBytes = 1024;

template <int PAIR>
constexpr size_t partial_item_bytes() {
  return static_cast<size_t>(PAIR) * kHalf * PairCfg<kGramBf16, PAIR>::kTileN * sizeof(float);
}
constexpr size_t kPartialItemBytes = partial_item_bytes<2>();

// `units`: tiles the device works on at once (CTA pairs, or single CTAs);
// at most one work item per cluster (the kernel stages partial sums in its
// pipeline stages, free only then), two counters per tile and CTA band, and
// every split gets two k-blocks or more.
// A split also has to save more pipeline iterations than its partial-sum
// round trip through L2 costs: measured on B200 about 10 us for a pair band
// (128 KiB) and 5 us for a single-CTA band (64 KiB), i.e. about 30 pair
// iterations of K = 64 (17 of K = 128) and 12 single-CTA iterations.
// Split mode (muon_polar_set_split_mode): 0 by size, 1 whenever possible,
// 2 never.
std::atomic<int> g_split_mode{0};

template <int KIND, int PAIR>
int choose_splits(int64_t tiles, int64_t k_blocks, int units) {
  const int mode = g_split_mode.load(std::memory_order_relaxed);
  if (mode == 2) return 1;
  if (tiles <= 0 || tiles * PAIR * 2 > static_cast<int64_t>(kCounterBytes / 4)) return 1;
  int64_t s = units / tiles;
  if (s > PairCfg<KIND, PAIR>::kMaxSplitsHere) s = PairCfg<KIND, PAIR>::kMaxSplitsHere;
  if (s > k_blocks / 2) s = k_blocks / 2;
  constexpr int64_t kMinSaved =
      PAIR == 1 ? 12 : (PairCfg<KIND, PAIR>::kBK == 128 ? 17 : 30);
  while (mode == 0 && s >= 2 && k_blocks - k_blocks / s < kMinSaved) --s;
  return s < 2 ? 1 : static_cast<int>(s);
}

template <int PAIR>
size_t split_scratch_bytes(int64_t tiles, int splits) {
  return splits > 1 ? kCounterBytes + static_cast<size_t>(tiles) * splits *
                                          partial_item_bytes<PAIR>()
                    : 0;
}

void plan_no_splits(EpiParams& p) {
  p.splits = 1;
  p.total_items = p.total_tiles;
  p.partial = nullptr;
  p.counters = nullptr;
}

// Column halves (single-CTA symmetric launches): tiles_m^2 items per matrix
// of at most 128 x 128 instead of tiles_m (tiles_m + 1) / 2 whole tiles, when
// all of them fit on the device at once and no split-K is planned.  Measured
// on B200, a single CTA's 128 x 128 tile is bound by shared-memory bandwidth
// (the TMA writes and both MMA operand reads, about 125 cycles per
// 128 x 128 x 16 MMA), and its time hardly depends on how many CTAs run (the
// config-1 Gram: 11.6 us for 10 tiles, 12.6 us for 120): a half reads
// 6 KiB and writes 6 KiB per 128 x 64 x 16 MMA, and twice as many CTAs share
// the work.  Mode (muon_polar_set_halves_mode): 0 by size, 1 whenever the
// items fit (tests), 2 never.
std::atomic<int> g_halves_mode{0};

void plan_halves(EpiParams& p, int64_t batch, int units) {
  p.halves = 0;
  const int mode = g_halves_mode.load(std::memory_order_relaxed);
  if (mode == 2 || p.splits != 1 || p.rows_mode || p.packed || p.row_tile_begin != 0 ||
      p.tile_offset != 0 || p.max_units > 0)
    return;
  const int64_t d = p.tiles_m;
  const int64_t items = d * d * batch;
  if (d < 2 || items > units) return;
  p.halves = 1;
  p.total_items = static_cast<int32_t>(items);
}

// Stage depth of the single-CTA bf16 Gram (muon_polar_set_stage_mode): 0 by
// size, 1 whenever it runs without split-K (see gram_launch), 2 never.  By size, kDeepBK
// stages when they cover at most 4% more K than two-atom stages: fewer,
// larger stages for the K loop, with the last one's columns past n read as
// zeros.  Measured on B200 (steps chained in CUDA graphs): [8,512,2048]
// 30.74 -> 30.48 us, [2,150,2064] 21.8 -> 19.9 us; with 12.5% more K,
// [4,512,1024] 19.3 -> 19.7 us and [1,1024,512] 19.7 -> 19.8 us.
std::atomic<int> g_stage_mode{0};

bool use_deep_stages(int64_t n) {
  const int mode = g_stage_mode.load(std::memory_order_relaxed);
  if (mode != 0) return mode == 1;
  const int64_t k2 = (n + 127) / 128 * 128;
  const int64_t k3 = (n + kDeepBK - 1) / kDeepBK * kDeepBK;
  return k3 * 100 <= k2 * 104;
}

// Applies split-K to `p` if the scratch buffer allows it.
template <int KIND, int PAIR>
void plan_splits(EpiParams& p, void* scratch, size_t scratch_bytes, int units) {
  plan_no_splits(p);
  if (scratch == nullptr || !aligned16(scratch)) return;
  const int s = choose_splits<KIND, PAIR>(p.total_tiles, p.k_blocks, units);
  if (s < 2 || split_scratch_bytes<PAIR>(p.total_tiles, s) > scratch_bytes) return;
  p.splits = s;
  p.total_items = p.total_tiles * s;
  p.counters = static_cast<uint32_t*>(scratch);
  p.partial = reinterpret_cast<float*>(static_cast<uint8_t*>(scratch) + kCounterBytes);
}

// How many tiles of polar_tile_kernel<KIND, PAIR> the device works on at
// once, after raising the kernel's shared-memory limit: co-resident clusters
// of two CTAs for PAIR = 2 (a tcgen05 CTA pair needs both SMs of a TPC; a TPC
// with one usable SM cannot host one), co-resident CTAs for PAIR = 1.
// Cached per device.
template <int KIND, int PAIR>
int tile_capacity(DeviceState* st, int* capacity) {
  constexpr int inst = instance_of<KIND, PAIR>();
  std::lock_guard<std::mutex> lock(g_attr_mutex);
  if (st->capacity[inst] > 0) {
    *capacity = st->capacity[inst];
    return MUON_POLAR_OK;
  }
  auto kern = polar_tile_kernel<KIND, PAIR, false>;
  const uint32_t smem = PairCfg<KIND, PAIR>::kSmemBytes;
  if (!st->smem_attr_set[inst]) {
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
    if (e != cudaSuccess) return static_cast<int>(e);
    if constexpr (PairCfg<KIND, PAIR>::kSym) {
      e = cudaFuncSetAttribute(polar_tile_kernel<KIND, PAIR, true>,
                               cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
      if (e != cudaSuccess) return static_cast<int>(e);
    }
    st->smem_attr_set[inst] = true;
  }
  int units = 0;
  if constexpr (PAIR == 2) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(2 * (st->sms / 2), 1, 1);
    cfg.blockDim = dim3(kTileThreads, 1, 1);
    cfg.dynamicSmemBytes = smem;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = 2;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    if (cudaOccupancyMaxActiveClusters(&units, kern, &cfg) != cudaSuccess || units <= 0) {
      (void)cudaGetLastError();
      units = st->sms / 2;
    }
    if (units > st->sms / 2) units = st->sms / 2;
  } else {
    int per_sm = 0;
    if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kern, kTileThreads, smem) !=
            cudaSuccess ||
        per_sm <= 0) {
      (void)cudaGetLastError();
      per_sm = 1;
    }
    units = per_sm * st->sms;
    // launched as clusters of two (launch_tile): count whole co-resident
    // clusters, so that every CTA of a launch with split-K items is resident
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(2 * (st->sms / 2), 1, 1);
    cfg.blockDim = dim3(kTileThreads, 1, 1);
    cfg.dynamicSmemBytes = smem;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = 2;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    int clusters = 0;
    if (cudaOccupancyMaxActiveClusters(&clusters, kern, &cfg) == cudaSuccess && clusters > 0) {
      if (2 * clusters < units) units = 2 * clusters;
    } else {
      (void)cudaGetLastError();
    }
  }
  st->capacity[inst] = units;
  *capacity = units;
  return MUON_POLAR_OK;
}

// `deep`: the single-CTA bf16 Gram with kDeepBK stages (p.k_blocks counted
// in them; no split-K).
template <int KIND, int PAIR>
int launch_tile(DeviceState* st, const TileMaps& maps, const EpiParams& p,
                cudaStream_t stream, bool deep = false) {
  int units = 0;
  int rc = tile_capacity<KIND, PAIR>(st, &units);
  if (rc != MUON_POLAR_OK) return rc;
  constexpr bool kCanDeepen = PAIR == 1 && KIND == kGramBf16;
  if (deep && (!kCanDeepen || p.splits != 1)) return MUON_POLAR_ERR_INVALID_ARGUMENT;
  constexpr bool kCanHalve = PAIR == 1 && PairCfg<KIND, PAIR>::kSym && KIND != kGramT;
  if constexpr (kCanHalve) {
    if (p.halves) {
      // one work item per CTA (the kernel's column-halves layout needs it)
      if (p.total_items > units || p.splits != 1) return MUON_POLAR_ERR_INVALID_ARGUMENT;
      constexpr int inst = instance_of<KIND, PAIR>();
      {
        std::lock_guard<std::mutex> lock(g_attr_mutex);
        if (!st->smem_attr_set_halves[inst]) {
          cudaError_t e = cudaFuncSetAttribute(polar_tile_kernel<KIND, PAIR, false, true>,
                                               cudaFuncAttributeMaxDynamicSharedMemorySize,
                                               PairCfg<KIND, PAIR, true>::kSmemBytes);
          if (e != cudaSuccess) return static_cast<int>(e);
          st->smem_attr_set_halves[inst] = true;
        }
      }
    }
  }
  if (p.max_units > 0 && units > p.max_units) units = p.max_units;
  int ctas = PAIR * (p.total_items < units ? p.total_items : units);
  // Single-CTA tiles launch as clusters of two independent CTAs as well, so
  // they occupy whole TPCs and leave whole TPCs free for the CTA pairs of
  // the next kernel to start early (measured on B200: 0.1-0.2 us per
  // config-1 step).  An extra CTA past the last item exits at once.
  if (PAIR == 1 && (ctas & 1)) ++ctas;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(ctas, 1, 1);
  cfg.blockDim = dim3(kTileThreads, 1, 1);
  cfg.dynamicSmemBytes = PairCfg<KIND, PAIR>::kSmemBytes;
  cfg.stream = stream;
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  attr[1].id = cudaLaunchAttributeClusterDimension;
  attr[1].val.clusterDim.x = 2;
  attr[1].val.clusterDim.y = 1;
  attr[1].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 2;
  cudaError_t e;
  if constexpr (kCanDeepen) {
    if (deep) {
      const bool h = p.halves != 0;
      {
        std::lock_guard<std::mutex> lock(g_attr_mutex);
        if (!st->smem_attr_set_deep[h]) {
          e = h ? cudaFuncSetAttribute(polar_tile_kernel<KIND, PAIR, false, true, kDeepBK>,
                                       cudaFuncAttributeMaxDynamicSharedMemorySize,
                                       PairCfg<KIND, PAIR, true, kDeepBK>::kSmemBytes)
                : cudaFuncSetAttribute(polar_tile_kernel<KIND, PAIR, false, false, kDeepBK>,
                                       cudaFuncAttributeMaxDynamicSharedMemorySize,
                                       PairCfg<KIND, PAIR, false, kDeepBK>::kSmemBytes);
          if (e != cudaSuccess) return static_cast<int>(e);
          st->smem_attr_set_deep[h] = true;
        }
      }
      if (h) {
        cfg.dynamicSmemBytes = PairCfg<KIND, PAIR, true, kDeepBK>::kSmemBytes;
        e = cudaLaunchKernelEx(&cfg, polar_tile_kernel<KIND, PAIR, false, true, kDeepBK>,
                               maps.a, maps.b, maps.aux, maps.out, maps.mir, p);
      } else {
        cfg.dynamicSmemBytes = PairCfg<KIND, PAIR, false, kDeepBK>::kSmemBytes;
        e = cudaLaunchKernelEx(&cfg, polar_tile_kernel<KIND, PAIR, false, false, kDeepBK>,
                               maps.a, maps.b, maps.aux, maps.out, maps.mir, p);
      }
      if (e != cudaSuccess) return static_cast<int>(e);
      g_launch_count.fetch_add(1, std::memory_order_relaxed);
      return MUON_POLAR_OK;
    }
  }
  if constexpr (kCanHalve) {
    if (p.halves) {
      cfg.dynamicSmemBytes = PairCfg<KIND, PAIR, true>::kSmemBytes;
      e = cudaLaunchKernelEx(&cfg, polar_tile_kernel<KIND, PAIR, false, true>, maps.a, maps.b,
                             maps.aux, maps.out, maps.mir, p);
      if (e != cudaSuccess) return static_cast<int>(e);
      g_launch_count.fetch_add(1, std::memory_order_relaxed);
      return MUON_POLAR_OK;
    }
  }
  if constexpr (PairCfg<KIND, PAIR>::kSym) {
    if (p.splits > 1)
      e = cudaLaunchKernelEx(&cfg, polar_tile_kernel<KIND, PAIR, true>, maps.a, maps.b, maps.aux,
                             maps.out, maps.mir, p);
    else
      e = cudaLaunchKernelEx(&cfg, polar_tile_kernel<KIND, PAIR, false>, maps.a, maps.b,
                             maps.aux, maps.out, maps.mir, p);
  } else {
    e = cudaLaunchKernelEx(&cfg, polar_tile_kernel<KIND, PAIR, false>, maps.a, maps.b, maps.aux,
                           maps.out, maps.mir, p);
  }
  if (e != cudaSuccess) return static_cast<int>(e);
  g_launch_count.fetch_add(1, std::memory_order_relaxed);
  return MUON_POLAR_OK;
}

int check_x_args(const void* x, int64_t batch, int64_t m, int64_t n,
                 int64_t ldx) {
  if (x == nullptr || batch <= 0 || m <= 0 || n <= 0 || ldx < n)
    return MUON_POLAR_ERR_INVALID_ARGUMENT;
  if (batch > INT32_MAX || m > (1 << 24) || ldx > (1ll << 31))
    return MUON_POLAR_ERR_INVALID_ARGUMENT;
  if (!aligned16(x) || (ldx % 8) != 0) return MUON_POLAR_ERR_ALIGNMENT;
  return MUON_POLAR_OK;
}

// Square [batch][mp][mp] buffer, bf16 or fp32, boxes of `box_rows` rows x
// 128 bytes.
int encode_square(CUtensorMap* map, const void* base, int64_t batch, int64_t mp,
                  bool f32, uint32_t box_rows) {
  return f32 ? encode_3d(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 4, base, mp, mp,
                         batch, mp, mp * mp, 32, box_rows)
             : encode_3d(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, base, mp, mp,
                         batch, mp, mp * mp, kAtom, box_rows);
}

// Upper-triangle units (256 x 256) of an mp x mp matrix.
int64_t packed_units_of(int64_t mp) {
  const int64_t d2 = mp / kPairM;
  return d2 * (d2 + 1) / 2;
}

// Packed upper-triangle units, [batch][units][256][256] bf16 or fp32, boxes
// of 128 rows x 128 bytes.
int encode_packed(CUtensorMap* map, const void* base, int64_t batch, int64_t mp, bool f32) {
  const int64_t units = packed_units_of(mp) * batch;
  return f32 ? encode_3d(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 4, base, kPairN, kPairM, units,
                         kPairN, kPairM * kPairN, 32, kHalf)
             : encode_3d(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, base, kPairN, kPairM, units,
                         kPairN, kPairM * kPairN, kAtom, kHalf);
}

// Upper-triangle tile grid of a symmetric kind: d x d tiles of kHalf * PAIR
// rows per matrix, d (d + 1) / 2 of them computed.
template <int PAIR>
void sym_grid(EpiParams& p, int64_t batch, int64_t mp) {
  const int64_t d = mp / (kHalf * PAIR);
  p.tiles_m = static_cast<int32_t>(d);
  p.tiles_n = static_cast<int32_t>(d);
  p.tiles_per_batch = static_cast<int32_t>(d * (d + 1) / 2);
  p.total_tiles = static_cast<int32_t>(d * (d + 1) / 2 * batch);
}

// Kernel (1) on one engine.  `fixed_scratch`: the scratch is a fixed buffer
// that keeps the previous call's contents -- a plan that needs more than it
// holds is refused, and the arrival counters are cleared before the launch.
// kGramT: the Gram of X^T, [batch][align(n, 256)]^2, contracting over the m
// rows of X.
template <int KIND, int PAIR>
int gram_launch(DeviceState* st, const void* x, void* gram, int64_t batch, int64_t m,
                int64_t n, int64_t ldx, void* scratch, size_t scratch_bytes,
                bool fixed_scratch, cudaStream_t stream, int64_t band_begin = 0,
                int64_t band_rows = 0, int sm_reserve = 0, bool packed = false) {
  constexpr bool kT = KIND == kGramT;
  const int64_t mp = padded_rows(kT ? n : m);
  int units = 0;
  int rc = tile_capacity<KIND, PAIR>(st, &units);
  if (rc != MUON_POLAR_OK) return rc;
  // SMs left free: whole clusters of two
  const int keep_units = units - (sm_reserve + 1) / 2 * (PAIR == 2 ? 1 : 2);
  if (sm_reserve > 0) units = keep_units > 0 ? keep_units : 1;
  TileMaps tm;
  // X: rows beyond m and columns beyond n read as zero.  K-major boxes of
  // [128 rows x 64 columns]; MN-major (kGramT) boxes of [kBK rows x 64
  // columns].
  rc = encode_3d(&tm.a, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, x, n, m, batch, ldx, m * ldx,
                 kAtom, kT ? PairCfg<KIND, PAIR>::kBK : kHalf);
  if (rc != MUON_POLAR_OK) return rc;
  tm.b = tm.a;
  tm.aux = tm.a;
  EpiParams p = {};
  if (packed) {
    rc = encode_packed(&tm.out, gram, batch, mp, KIND == kGramF32);
    tm.mir = tm.out;
    p.packed = 1;
    p.packed_d = static_cast<int32_t>(mp / kPairM);
    p.packed_units = static_cast<int32_t>(packed_units_of(mp));
  } else {
    rc = encode_square(&tm.out, gram, batch, mp, KIND == kGramF32, kHalf);
    if (rc != MUON_POLAR_OK) return rc;
    rc = encode_square(&tm.mir, gram, batch, mp, KIND == kGramF32, kChunkCols);
  }
  if (rc != MUON_POLAR_OK) return rc;
  sym_grid<PAIR>(p, batch, mp);
  if (!kT) {
    p.prefetch_base = static_cast<const uint8_t*>(x);
    p.prefetch_row_bytes = ldx * 2;
    p.prefetch_batch_bytes = m * ldx * 2;
    p.prefetch_rows = static_cast<int32_t>(m);
    p.prefetch_lines = static_cast<int32_t>((n * 2 + 127) / 128);
  }
  if (band_rows > 0) {
    // the upper tiles of tile rows [t0, t0 + nt)
    const int64_t th = kHalf * PAIR;
    const int64_t d = mp / th, t0 = band_begin / th, nt = band_rows / th;
    const int64_t count = nt * d - (2 * t0 + nt - 1) * nt / 2;
    p.tiles_per_batch = static_cast<int32_t>(count);
    p.total_tiles = static_cast<int32_t>(count * batch);
    p.row_tile_begin = static_cast<int32_t>(t0);
  }
  if (sm_reserve > 0) p.max_units = units;
  p.k_blocks = static_cast<int32_t>(k_blocks_of<KIND, PAIR>(kT ? m : n));
  if (fixed_scratch &&
      split_scratch_bytes<PAIR>(p.total_tiles,
                                choose_splits<KIND, PAIR>(p.total_tiles, p.k_blocks, units)) >
          scratch_bytes)
    return MUON_POLAR_ERR_STATIC_SCRATCH;
  // Deep stages (single-CTA bf16 Gram) are chosen before split-K: counted in
  // kDeepBK blocks the K loop is shorter, and when the split planner then
  // plans no split the launch runs unsplit on deep stages (measured on B200,
  // [2,150,2064] 21.8 -> 19.9 us against four splits of K = 128 stages).
  bool deep = false;
  if constexpr (PAIR == 1 && KIND == kGramBf16) {
    const int64_t kb3 = (n + kDeepBK - 1) / kDeepBK;
    deep = !fixed_scratch && use_deep_stages(n) &&
           (scratch == nullptr || choose_splits<KIND, PAIR>(p.total_tiles, kb3, units) == 1);
  }
  if (deep)
    plan_no_splits(p);
  else
    plan_splits<KIND, PAIR>(p, scratch, scratch_bytes, units);
  if constexpr (PAIR == 1 && !kT) {
    if (!fixed_scratch) plan_halves(p, batch, units);
    if (p.halves) {
      rc = encode_3d(&tm.b, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, x, n, m, batch, ldx, m * ldx,
                     kAtom, kChunkCols);
      if (rc != MUON_POLAR_OK) return rc;
    }
  }
  if (fixed_scratch && p.splits > 1) {
    cudaError_t e = cudaMemsetAsync(scratch, 0, kCounterBytes, stream);
    if (e != cudaSuccess) return static_cast<int>(e);
  }
  if (deep) p.k_blocks = static_cast<int32_t>((n + kDeepBK - 1) / kDeepBK);
  return launch_tile<KIND, PAIR>(st, tm, p, stream, deep);
}

// `fixed_scratch` callers always run the CTA-pair engine (the size of their
// buffer is stated in pair split items).
template <int KIND>
int gram_impl(const void* x, void* gram, int64_t batch, int64_t m, int64_t n,
              int64_t ldx, void* scratch, size_t scratch_bytes,
              cudaStream_t stream, bool fixed_scratch = false, bool packed = false) {
  int rc = check_x_args(x, batch, m, n, ldx);
  if (rc != MUON_POLAR_OK) return rc;
  if (gram == nullptr) return MUON_POLAR_ERR_INVALID_ARGUMENT;
  if (!aligned16(gram)) return MUON_POLAR_ERR_ALIGNMENT;
  // rows of the Gram and the contraction length
  const int64_t rows = KIND == kGramT ? n : m;
  const int64_t depth = KIND == kGramT ? m : n;
  if (rows > (1 << 24)) return MUON_POLAR_ERR_INVALID_ARGUMENT;
  DeviceState* st = nullptr;
  rc = current_device_state(&st);
  if (rc != MUON_POLAR_OK) return rc;
  const int64_t d = padded_rows(rows) / kHalf;
  if (d * (d + 1) / 2 * batch > INT32_MAX) return MUON_POLAR_ERR_INVALID_ARGUMENT;
  const int64_t dp = padded_rows(rows) / kPairM;
  int pairs = 0, ctas = 0;
  rc = tile_capacity<KIND, 2>(st, &pairs);
  if (rc != MUON_POLAR_OK) return rc;
  rc = tile_capacity<KIND, 1>(st, &ctas);
  if (rc != MUON_POLAR_OK) return rc;
  if (fixed_scratch || use_pairs(dp * (dp + 1) / 2 * batch, pairs, cost_blocks<2>(depth),
                                 d * (d + 1) / 2 * batch, ctas, cost_blocks<1>(depth)))
    return gram_launch<KIND, 2>(st, x, gram, batch, m, n, ldx, scratch, scratch_bytes,
                                fixed_scratch, stream, 0, 0, 0, packed);
  return gram_launch<KIND, 1>(st, x, gram, batch, m, n, ldx, scratch, scratch_bytes,
                              fixed_scratch, stream, 0, 0, 0, packed);
}

// Kernel (1), fp32 output, on the upper tiles of the rows [row_begin,
// row_begin + row_count) of the Gram (multiples of 256), each stored with its
// mirror; `sm_reserve` SMs stay free.  Run for consecutive bands in order,
// the rows of a band are complete (both triangles) once it has run.
int gram_f32_band_impl(const void* x, void* gram, int64_t batch, int64_t m, int64_t n,
                       int64_t ldx, int64_t row_begin, int64_t row_count, int sm_reserve,
                       void* scratch, size_t scratch_bytes, cudaStream_t stream) {
  int rc = check_x_args(x, batch, m, n, ldx);
  if (rc != MUON_POLAR_OK) return rc;
  if (gram == nullptr) return MUON_POLAR_ERR_INVALID_ARGUMENT;
  if (!aligned16(gram)) return MUON_POLAR_ERR_ALIGNMENT;
  const int64_t mp = padded_rows(m);
  if (row_begin < 0 || row_count <= 0 || row_begin % kPairM != 0 || row_count % kPairM != 0 ||
      row_begin + row_count > mp || sm_reserve < 0 || sm_reserve > 1024)
    return MUON_POLAR_ERR_INVALID_ARGUMENT;
  DeviceState* st = nullptr;
  rc = current_device_state(&st);
  if (rc != MUON_POLAR_OK) return rc;
  int pairs = 0, ctas = 0;
  rc = tile_capacity<kGramF32, 2>(st, &pairs);
  if (rc != MUON_POLAR_OK) return rc;
  rc = tile_capacity<kGramF32, 1>(st, &ctas);
  if (rc != MUON_POLAR_OK) return rc;
  auto band_tiles = [&](int64_t th) {
    const int64_t d = mp / th, t0 = row_begin / th, nt = row_count / th;
    return (nt * d - (2 * t0 + nt - 1) * nt / 2) * batch;
  };
  if (band_tiles(kHalf) > INT32_MAX) return MUON_POLAR_ERR_INVALID_ARGUMENT;
  if (use_pairs(band_tiles(kPairM), pairs, cost_blocks<2>(n), band_tiles(kHalf), ctas,
                cost_blocks<1>(n)))
    return gram_launch<kGramF32, 2>(st, x, gram, batch, m, n, ldx, scratch, scratch_bytes, false,
                                    stream, row_begin, row_count, sm_reserve);
  return gram_launch<kGramF32, 1>(st, x, gram, batch, m, n, ldx, scratch, scratch_bytes, false,
                                  stream, row_begin, row_count, sm_reserve);
}

template <int PAIR>
int poly_launch(DeviceState* st, const void* gram, void* poly, int64_t batch, int64_t mp,
                float b, float c, void* scratch, size_t scratch_bytes, cudaStream_t stream) {
  int units = 0;
  int rc = tile_capacity<kPoly, PAIR>(st, &units);
  if (rc != MUON_POLAR_OK) return rc;
  TileMaps tm;
  rc = encode_square(&tm.a, gram, batch, mp, false, kHalf);
  if (rc != MUON_POLAR_OK) return rc;
  tm.b = tm.a;
  tm.aux = tm.a;
  rc = encode_square(&tm.out, poly, batch, mp, false, kHalf);
  if (rc != MUON_POLAR_OK) return rc;
  rc = encode_square(&tm.mir, poly, batch, mp, false, kChunkCols);
  if (rc != MUON_POLAR_OK) return rc;
  EpiParams p = {};
  sym_grid<PAIR>(p, batch, mp);
  p.k_blocks = static_cast<int32_t>(k_blocks_of<kPoly, PAIR>(mp));
  p.coef_b = b;
  p.coef_c = c;
  plan_splits<kPoly, PAIR>(p, scratch, scratch_bytes, units);
  if constexpr (PAIR == 1) {
    plan_halves(p, batch, units);
    if (p.halves) {
      rc = encode_square(&tm.b, gram, batch, mp, false, kChunkCols);
      if (rc != MUON_POLAR_OK) return rc;
    }
  }
  return launch_tile<kPoly, PAIR>(st, tm, p, stream);
}

int poly_impl(const void* gram, void* poly, int64_t batch, int64_t mp, float b,
              float c, void* scratch, size_t scratch_bytes, cudaStream_t stream) {
  if (gram == nullptr || poly == nullptr || batch <= 0 || mp <= 0 ||
      (mp % kHalf) != 0 || batch > INT32_MAX || mp > (1 << 24))
    return MUON_POLAR_ERR_INVALID_ARGUMENT;
  if (!aligned16(gram) || !aligned16(poly)) return MUON_POLAR_ERR_ALIGNMENT;
  DeviceState* st = nullptr;
  int rc = current_device_state(&st);
  if (rc != MUON_POLAR_OK) return rc;
  const int64_t d = mp / kHalf;
  if (d * (d + 1) / 2 * batch > INT32_MAX) return MUON_POLAR_ERR_INVALID_ARGUMENT;
  const int64_t dp = mp / kPairM;
  int pairs = 0, ctas = 0;
  rc = tile_capacity<kPoly, 2>(st, &pairs);
  if (rc != MUON_POLAR_OK) return rc;
  rc = tile_capacity<kPoly, 1>(st, &ctas);
  if (rc != MUON_POLAR_OK) return rc;
  if ((mp % kPairM) == 0 && use_pairs(dp * (dp + 1) / 2 * batch, pairs,
                                      cost_blocks<2>(mp), d * (d + 1) / 2 * batch, ctas,
                                      cost_blocks<1>(mp)))
    return poly_launch<2>(st, gram, poly, batch, mp, b, c, scratch, scratch_bytes, stream);
  return poly_launch<1>(st, gram, poly, batch, mp, b, c, scratch, scratch_bytes, stream);
}

// Rows [row_begin, row_begin + row_count) of P into the full [batch][mp][mp]
// buffer `poly` (whole rows, both triangles), for callers that split kernel
// (2) over GPUs by row slabs.
template <int PAIR>
int poly_rows_launch(DeviceState* st, const void* gram, void* poly, int64_t batch, int64_t mp,
                     int64_t row_begin, int64_t row_count, float b, float c,
                     cudaStream_t stream) {
  using Cfg = PairCfg<kPoly, PAIR>;
  TileMaps tm;
  int rc = encode_square(&tm.a, gram, batch, mp, false, kHalf);
  if (rc != MUON_POLAR_OK) return rc;
  tm.b = tm.a;
  tm.aux = tm.a;
  rc = encode_square(&tm.out, poly, batch, mp, false, kHalf);
  if (rc != MUON_POLAR_OK) return rc;
  tm.mir = tm.out;
  EpiParams p = {};
  p.tiles_m = static_cast<int32_t>(row_count / Cfg::kTileM);
  p.tiles_n = static_cast<int32_t>(mp / Cfg::kTileN);
  p.tiles_per_batch = p.tiles_m * p.tiles_n;
  p.total_tiles = static_cast<int32_t>(p.tiles_per_batch * batch);
  p.rows_mode = 1;
  p.row_tile_begin = static_cast<int32_t>(row_begin / Cfg::kTileM);
  p.k_blocks = static_cast<int32_t>(k_blocks_of<kPoly, PAIR>(mp));
  p.coef_b = b;
  p.coef_c = c;
  plan_no_splits(p);
  return launch_tile<kPoly, PAIR>(st, tm, p, stream);
}

int poly_rows_impl(const void* gram, void* poly, int64_t batch, int64_t mp, int64_t row_begin,
                   int64_t row_count, float b, float c, cudaStream_t stream) {
  if (gram == nullptr || poly == nullptr || batch <= 0 || mp <= 0 || (mp % kPairM) != 0 ||
      batch > INT32_MAX || mp > (1 << 24) || row_begin < 0 || row_count <= 0 ||
      (row_begin % kPairM) != 0 || (row_count % kPairM) != 0 || row_begin + row_count > mp)
    return MUON_POLAR_ERR_INVALID_ARGUMENT;
  if (!aligned16(gram) || !aligned16(poly)) return MUON_POLAR_ERR_ALIGNMENT;
  if ((row_count / kHalf) * (mp / kHalf) * batch > INT32_MAX)
    return MUON_POLAR_ERR_INVALID_ARGUMENT;
  DeviceState* st = nullptr;
  int rc = current_device_state(&st);
  if (rc != MUON_POLAR_OK) return rc;
  int pairs = 0, ctas = 0;
  rc = tile_capacity<kPoly, 2>(st, &pairs);
  if (rc != MUON_POLAR_OK) return rc;
  rc = tile_capacity<kPoly, 1>(st, &ctas);
  if (rc != MUON_POLAR_OK) return rc;
  if (use_pairs(row_count / kPairM * (mp / kPairN) * batch, pairs, cost_blocks<2>(mp),
                row_count / kHalf * (mp / kHalf) * batch, ctas, cost_blocks<1>(mp)))
    return poly_rows_launch<2>(st, gram, poly, batch, mp, row_begin, row_count, b, c, stream);
  return poly_rows_launch<1>(st, gram, poly, batch, mp, row_begin, row_count, b, c, stream);
}

// Units [unit_begin, unit_begin + unit_count) of the upper triangle of P,
// each written into its place in the packed buffer (CTA-pair tiles: one
// tile per unit).
int poly_packed_impl(const void* gram, void* packed, int64_t batch, int64_t mp,
                     int64_t unit_begin, int64_t unit_count, float b, float c,
                     cudaStream_t stream) {
  if (gram == nullptr || packed == nullptr || batch <= 0 || mp <= 0 || (mp % kPairM) != 0 ||
      batch > INT32_MAX || mp > (1 << 24))
    return MUON_POLAR_ERR_INVALID_ARGUMENT;
  const int64_t units = packed_units_of(mp);
  if (unit_begin < 0 || unit_count <= 0 || unit_begin + unit_count > units ||
      unit_count * batch > INT32_MAX)
    return MUON_POLAR_ERR_INVALID_ARGUMENT;
  if (!aligned16(gram) || !aligned16(packed)) return MUON_POLAR_ERR_ALIGNMENT;
  DeviceState* st = nullptr;
  int rc = current_device_state(&st);
  if (rc != MUON_POLAR_OK) return rc;
  int pairs = 0;
  rc = tile_capacity<kPoly, 2>(st, &pairs);
  if (rc != MUON_POLAR_OK) return rc;
  TileMaps tm;
  rc = encode_square(&tm.a, gram, batch, mp, false, kHalf);
  if (rc != MUON_POLAR_OK) return rc;
  tm.b = tm.a;
  tm.aux = tm.a;
  rc = encode_packed(&tm.out, packed, batch, mp, false);
  if (rc != MUON_POLAR_OK) return rc;
  tm.mir = tm.out;
  EpiParams p = {};
  sym_grid<2>(p, batch, mp);
  p.tiles_per_batch = static_cast<int32_t>(unit_count);
  p.total_tiles = static_cast<int32_t>(unit_count * batch);
  p.tile_offset = static_cast<int32_t>(unit_begin);
  p.packed = 1;
  p.packed_d = static_cast<int32_t>(mp / kPairM);
  p.packed_units = static_cast<int32_t>(units);
  p.k_blocks = static_cast<int32_t>(k_blocks_of<kPoly, 2>(mp));
  p.coef_b = b;
  p.coef_c = c;
  plan_no_splits(p);
  return launch_tile<kPoly, 2>(st, tm, p, stream);
}

int unpack_sym_impl(const void* packed, void* full, int64_t batch, int64_t mp,
                    cudaStream_t stream) {
  if (packed == nullptr || full == nullptr || batch <= 0 || mp <= 0 || (mp % kPairM) != 0 ||
      batch > 65535 || mp > (1 << 24))
    return MUON_POLAR_ERR_INVALID_ARGUMENT;
  if (!aligned16(packed) || !aligned16(full)) return MUON_POLAR_ERR_ALIGNMENT;
  DeviceState* st = nullptr;
  int rc = current_device_state(&st);
  if (rc != MUON_POLAR_OK) return rc;
  const int64_t units = packed_units_of(mp);
  if (units * 4 > INT32_MAX) return MUON_POLAR_ERR_INVALID_ARGUMENT;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(static_cast<unsigned>(units * 4), static_cast<unsigned>(batch), 1);
  cfg.blockDim = dim3(256, 1, 1);
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  cudaError_t e = cudaLaunchKernelEx(&cfg, unpack_sym_kernel, static_cast<const uint16_t*>(packed),
                                     static_cast<uint16_t*>(full), static_cast<int>(mp / kPairM),
                                     static_cast<int>(units), mp);
  if (e != cudaSuccess) return static_cast<int>(e);
  g_launch_count.fetch_add(1, std::memory_order_relaxed);
  return MUON_POLAR_OK;
}

// Host-side fp32 -> bf16 round-to-nearest-even, the same rule as the
// reference's FloatToBf16Bits (binding.cpp:156-162).
float round_to_bf16(float v) {
  uint32_t raw;
  std::memcpy(&raw, &v, 4);
  const uint32_t rounded = (raw + 0x7FFFu + ((raw >> 16) & 1u)) & 0xFFFF0000u;
  float out;
  std::memcpy(&out, &rounded, 4);
  return out;
}

template <int PAIR>
int apply_launch(DeviceState* st, const void* poly, const void* x, void* y, int64_t batch,
                 int64_t m, int64_t n, int64_t ldx, int64_t ldy, float a,
                 cudaStream_t stream) {
  using Cfg = PairCfg<kApply, PAIR>;
  const int64_t mp = padded_rows(m);
  const int64_t tiles_m = (m + Cfg::kTileM - 1) / Cfg::kTileM;
  const int64_t tiles_n = (n + Cfg::kTileN - 1) / Cfg::kTileN;
  if (tiles_m * tiles_n * batch > INT32_MAX) return MUON_POLAR_ERR_INVALID_ARGUMENT;
  TileMaps tm;
  int rc = encode_square(&tm.a, poly, batch, mp, false, kHalf);
  if (rc != MUON_POLAR_OK) return rc;
  // X as the B operand: rows are K, a 64-column box is the MN extent.
  rc = encode_3d(&tm.b, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, x, n, m, batch, ldx, m * ldx,
                 kAtom, Cfg::kBK);
  if (rc != MUON_POLAR_OK) return rc;
  // X as the epilogue input tile, Y as the output tile (rows >= m and
  // columns >= n are neither read nor written).
  rc = encode_3d(&tm.aux, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, x, n, m, batch, ldx, m * ldx,
                 kAtom, kHalf);
  if (rc != MUON_POLAR_OK) return rc;
  rc = encode_3d(&tm.out, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, y, n, m, batch, ldy, m * ldy,
                 kAtom, kHalf);
  if (rc != MUON_POLAR_OK) return rc;
  tm.mir = tm.out;
  EpiParams p = {};
  p.tiles_m = static_cast<int32_t>(tiles_m);
  p.tiles_n = static_cast<int32_t>(tiles_n);
  p.tiles_per_batch = static_cast<int32_t>(tiles_m * tiles_n);
  p.total_tiles = static_cast<int32_t>(tiles_m * tiles_n * batch);
  // P's columns >= m are zero and X's rows >= m read as zero: stop at m.
  p.k_blocks = static_cast<int32_t>(k_blocks_of<kApply, PAIR>(m));
  p.alpha = round_to_bf16(a);
  plan_no_splits(p);
  return launch_tile<kApply, PAIR>(st, tm, p, stream);
}

int apply_impl(const void* poly, const void* x, void* y, int64_t batch,
               int64_t m, int64_t n, int64_t ldx, int64_t ldy, float a,
               cudaStream_t stream) {
  int rc = check_x_args(x, batch, m, n, ldx);
  if (rc != MUON_POLAR_OK) return rc;
  if (poly == nullptr || y == nullptr || ldy < n)
    return MUON_POLAR_ERR_INVALID_ARGUMENT;
  if (!aligned16(poly) || !aligned16(y) || (ldy % 8) != 0)
    return MUON_POLAR_ERR_ALIGNMENT;
  DeviceState* st = nullptr;
  rc = current_device_state(&st);
  if (rc != MUON_POLAR_OK) return rc;
  int pairs = 0, ctas = 0;
  rc = tile_capacity<kApply, 2>(st, &pairs);
  if (rc != MUON_POLAR_OK) return rc;
  rc = tile_capacity<kApply, 1>(st, &ctas);
  if (rc != MUON_POLAR_OK) return rc;
  // By size, a short apply (K = m <= 512) that the pairs finish in at most two
  // rounds runs on single CTAs: its four rounds of 128 x 128 tiles end more
  // evenly and store half the bytes per CTA in the last epilogue, which the
  // pair engine's higher per-SM rate does not make up for.  Measured on B200
  // (steps chained in CUDA graphs): [8,512,2048] 32.4 -> 31.9 us,
  // [4,512,2048] 27.2 -> 26.0, [4,256,4096] 29.9 -> 28.2, [16,256,2048]
  // 28.8 -> 28.0; with K = 1024 the pairs stay ahead ([2,1024,4096] 47.0
  // against 49.2 us).
  const int64_t tiles2 = padded_rows(m) / kPairM * ((n + kPairN - 1) / kPairN) * batch;
  const bool short_apply =
      g_policy.load(std::memory_order_relaxed) == 0 && m <= 512 && tiles2 <= 2 * pairs;
  if (!short_apply && use_pairs(tiles2, pairs, cost_blocks<2>(m),
                                (m + kHalf - 1) / kHalf * ((n + kHalf - 1) / kHalf) * batch,
                                ctas, cost_blocks<1>(m)))
    return apply_launch<2>(st, poly, x, y, batch, m, n, ldx, ldy, a, stream);
  return apply_launch<1>(st, poly, x, y, batch, m, n, ldx, ldy, a, stream);
}

// Kernel (3) of the step of X^T returned in X's layout (M > N without
// transposed copies): y = bf16( bf16(X.P) + bf16(alpha*X) ), X and Y
// [batch][m][ld], P [batch][align(n, 256)]^2 -- symmetric, so its rows serve
// as the K-major B operand of X.P.
template <int PAIR>
int apply_t_launch(DeviceState* st, const void* poly, const void* x, void* y, int64_t batch,
                   int64_t m, int64_t n, int64_t ldx, int64_t ldy, float a,
                   cudaStream_t stream) {
  using Cfg = PairCfg<kApplyT, PAIR>;
  const int64_t np = padded_rows(n);
  const int64_t tiles_m = (m + Cfg::kTileM - 1) / Cfg::kTileM;
  const int64_t tiles_n = (n + Cfg::kTileN - 1) / Cfg::kTileN;
  if (tiles_m * tiles_n * batch > INT32_MAX) return MUON_POLAR_ERR_INVALID_ARGUMENT;
  TileMaps tm;
  // X rows: the A operand (K = its columns) and the epilogue input tile.
  int rc = encode_3d(&tm.a, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, x, n, m, batch, ldx, m * ldx,
                     kAtom, kHalf);
  if (rc != MUON_POLAR_OK) return rc;
  tm.aux = tm.a;
  rc = encode_square(&tm.b, poly, batch, np, false, kHalf);
  if (rc != MUON_POLAR_OK) return rc;
  rc = encode_3d(&tm.out, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, y, n, m, batch, ldy, m * ldy,
                 kAtom, kHalf);
  if (rc != MUON_POLAR_OK) return rc;
  tm.mir = tm.out;
  EpiParams p = {};
  p.tiles_m = static_cast<int32_t>(tiles_m);
  p.tiles_n = static_cast<int32_t>(tiles_n);
  p.tiles_per_batch = static_cast<int32_t>(tiles_m * tiles_n);
  p.total_tiles = static_cast<int32_t>(tiles_m * tiles_n * batch);
  // X's columns >= n read as zero and P's rows/columns >= n are zero.
  p.k_blocks = static_cast<int32_t>(k_blocks_of<kApplyT, PAIR>(n));
  p.alpha = round_to_bf16(a);
  plan_no_splits(p);
  return launch_tile<kApplyT, PAIR>(st, tm, p, stream);
}

int apply_t_impl(const void* poly, const void* x, void* y, int64_t batch, int64_t m,
                 int64_t n, int64_t ldx, int64_t ldy, float a, cudaStream_t stream) {
  int rc = check_x_args(x, batch, m, n, ldx);
  if (rc != MUON_POLAR_OK) return rc;
  if (poly == nullptr || y == nullptr || ldy < n || n > (1 << 24))
    return MUON_POLAR_ERR_INVALID_ARGUMENT;
  if (!aligned16(poly) || !aligned16(y) || (ldy % 8) != 0)
    return MUON_POLAR_ERR_ALIGNMENT;
  DeviceState* st = nullptr;
  rc = current_device_state(&st);
  if (rc != MUON_POLAR_OK) return rc;
  int pairs = 0, ctas = 0;
  rc = tile_capacity<kApplyT, 2>(st, &pairs);
  if (rc != MUON_POLAR_OK) return rc;
  rc = tile_capacity<kApplyT, 1>(st, &ctas);
  if (rc != MUON_POLAR_OK) return rc;
  if (use_pairs((m + kPairM - 1) / kPairM * ((n + kPairN - 1) / kPairN) * batch, pairs,
                cost_blocks<2>(n),
                (m + kHalf - 1) / kHalf * ((n + kHalf - 1) / kHalf) * batch, ctas,
                cost_blocks<1>(n)))
    return apply_t_launch<2>(st, poly, x, y, batch, m, n, ldx, ldy, a, stream);
  return apply_t_launch<1>(st, poly, x, y, batch, m, n, ldx, ldy, a, stream);
}

// ---------------------------------------------------------------- fused step
// Step mode: 0 = by size (see fused_steps_impl), 1 = always fused, 2 = three
// kernels.  Initial value from MUON_POLAR_FUSED (1 -> 1, 0 -> 2).
std::atomic<int> g_step_mode{[] {
  const char* s = std::getenv("MUON_POLAR_FUSED");
  if (s == nullptr) return 0;
  const int v = std::atoi(s);
  return v == 1 ? 1 : (v == 0 ? 2 : 0);
}()};

struct FusedDeviceState {
  std::once_flag once;
  cudaError_t err = cudaSuccess;
  int capacity = 0;
};
FusedDeviceState g_fused_state[kMaxDevices];

int fused_capacity(DeviceState* st, int dev, int* capacity) {
  FusedDeviceState& fs = g_fused_state[dev];
  std::call_once(fs.once, [&fs, st] {
    fs.err = cudaFuncSetAttribute(polar_fused_kernel<false>,
                                  cudaFuncAttributeMaxDynamicSharedMemorySize,
                                  FusedCfg::kSmemBytes);
    if (fs.err != cudaSuccess) return;
    fs.err = cudaFuncSetAttribute(polar_fused_kernel<true>,
                                  cudaFuncAttributeMaxDynamicSharedMemorySize,
                                  FusedCfg::kSmemBytes);
    if (fs.err != cudaSuccess) return;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(2 * (st->sms / 2), 1, 1);
    cfg.blockDim = dim3(kTileThreads, 1, 1);
    cfg.dynamicSmemBytes = FusedCfg::kSmemBytes;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = 2;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    int clusters = 0;
    if (cudaOccupancyMaxActiveClusters(&clusters, polar_fused_kernel<false>, &cfg) !=
            cudaSuccess ||
        clusters <= 0) {
      (void)cudaGetLastError();
      clusters = st->sms / 2;
    }
    fs.capacity = clusters < st->sms / 2 ? clusters : st->sms / 2;
  });
  if (fs.err != cudaSuccess) return static_cast<int>(fs.err);
  *capacity = fs.capacity;
  return MUON_POLAR_OK;
}

// Runs `steps` Polar Express steps (coefficient rows coefs[3 s .. 3 s + 2] =
// a, b, c) as one fused launch if the mode and sizes allow it; *done = false
// means the caller should run the three kernels instead.  Step 0 reads x
// (row stride ldx), step s > 0 reads the previous step's output in buffer
// buf[(s - 1) % 2] (row stride ldb), the last step writes y (ldy), the
// others buf[s % 2].  buf may be null when steps == 1.
int fused_steps_impl(const void* x, void* y, void* const* buf, int64_t ldb, void* gram,
                     void* poly, void* scratch, size_t scratch_bytes, int64_t batch, int64_t m,
                     int64_t n, int64_t ldx, int64_t ldy, const float* coefs, int steps,
                     cudaStream_t stream, bool* done) {
  *done = false;
  const int mode = g_step_mode.load(std::memory_order_relaxed);
  if (mode == 2 || steps < 1 || steps > kMaxFusedSteps || scratch == nullptr ||
      !aligned16(scratch) ||
      static_cast<size_t>(3 * batch + 1) * 4 > kCounterBytes || scratch_bytes < kCounterBytes)
    return MUON_POLAR_OK;
  if (steps > 1 && (buf == nullptr || buf[0] == nullptr || buf[1] == nullptr)) return MUON_POLAR_OK;
  DeviceState* st = nullptr;
  int rc = current_device_state(&st);
  if (rc != MUON_POLAR_OK) return rc;
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return static_cast<int>(e);
  int capacity = 0;
  rc = fused_capacity(st, dev, &capacity);
  if (rc != MUON_POLAR_OK) return rc;
  const int64_t mp = padded_rows(m);
  const int64_t d2 = mp / kPairM;
  const int64_t regions_r = d2 * (d2 + 1);  // 256 x 128 regions per matrix
  const int64_t regions_w = regions_r / 2;  // 256 x 256 tiles per matrix
  // Item shape of the Gram and the polynomial.  Wide tiles halve the items
  // but run a 3-stage ring and a 4-chunk epilogue; measured on B200 (five
  // steps in one launch) they win only when regions would take about three
  // rounds of the pairs: [32,512,2048] 418.5 -> 403.7 us, [16,768,3072]
  // 565.8 -> 529.6 us, [32,384,1024] even; and lose at two rounds:
  // [16,512,2048] 231.5 -> 261.8 us, [8,768,3072] 296.6 -> 327.3 us,
  // [64,256,1024] 203.2 -> 207.6 us.
  const bool wide = 2 * batch * regions_r >= 5 * static_cast<int64_t>(capacity);
  const int64_t regions = wide ? regions_w : regions_r;
  const int64_t tn = (n + kPairN - 1) / kPairN;
  const int64_t per_step = 2 * batch * regions + batch * d2 * tn;
  if (per_step * steps > INT32_MAX) return MUON_POLAR_OK;
  // By size, from measurements on B200 (muon_polar_step_sm100, 15 shapes;
  // muon_polar_steps_sm100, 7 more): the fused launch wins for many small
  // matrices -- more Gram regions than pairs, up to three rounds of them, and
  // Mp <= 768: 4-21% faster at [16|32,512,2048], [8,768,3072],
  // [64,256,1024] -- and loses where the three kernels run a Gram of one
  // round (config 1 [8,512,2048]: 38.5 vs 36.8 us), a large one on 256 x
  // 256 pair tiles (Mp >= 1024, N >= 4096: up to 12% slower) or many rounds
  // of items (five steps at [64,512,2048]: 896 vs 740 us).
  const int64_t sym_items = batch * regions_r;
  if (mode == 0 && !(sym_items > capacity && sym_items <= 3 * static_cast<int64_t>(capacity) &&
                     mp <= 768))
    return MUON_POLAR_OK;

  FusedMaps maps;
  // X of each step and Y: the input / output and the two buffers
  const void* xs[3] = {x, steps > 1 ? buf[0] : x, steps > 1 ? buf[1] : x};
  void* ys[3] = {y, steps > 1 ? buf[0] : y, steps > 1 ? buf[1] : y};
  const int64_t lds_x[3] = {ldx, steps > 1 ? ldb : ldx, steps > 1 ? ldb : ldx};
  const int64_t lds_y[3] = {ldy, steps > 1 ? ldb : ldy, steps > 1 ? ldb : ldy};
  for (int k = 0; k < 3; ++k) {
    rc = encode_3d(&maps.x_k[k], CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, xs[k], n, m, batch,
                   lds_x[k], m * lds_x[k], kAtom, kHalf);
    if (rc != MUON_POLAR_OK) return rc;
    rc = encode_3d(&maps.x_mn[k], CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, xs[k], n, m, batch,
                   lds_x[k], m * lds_x[k], kAtom, kAtom);
    if (rc != MUON_POLAR_OK) return rc;
    rc = encode_3d(&maps.y128[k], CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, ys[k], n, m, batch,
                   lds_y[k], m * lds_y[k], kAtom, kHalf);
    if (rc != MUON_POLAR_OK) return rc;
  }
  rc = encode_square(&maps.a128, gram, batch, mp, false, kHalf);
  if (rc != MUON_POLAR_OK) return rc;
  rc = encode_square(&maps.a64, gram, batch, mp, false, kChunkCols);
  if (rc != MUON_POLAR_OK) return rc;
  rc = encode_square(&maps.p128, poly, batch, mp, false, kHalf);
  if (rc != MUON_POLAR_OK) return rc;
  rc = encode_square(&maps.p64, poly, batch, mp, false, kChunkCols);
  if (rc != MUON_POLAR_OK) return rc;

  FusedParams p = {};
  p.batch = static_cast<int32_t>(batch);
  p.d2 = static_cast<int32_t>(d2);
  p.regions = static_cast<int32_t>(regions);
  p.apply_tn = static_cast<int32_t>(tn);
  p.n_gram = static_cast<int32_t>(batch * regions);
  p.n_poly = static_cast<int32_t>(batch * regions);
  p.per_step = static_cast<int32_t>(per_step);
  p.steps = steps;
  p.total = static_cast<int32_t>(per_step * steps);
  p.apply_bands = static_cast<uint32_t>(2 * d2 * tn);
  p.kb_gram = static_cast<int32_t>((n + 127) / 128);
  p.kb_poly = static_cast<int32_t>(mp / 128);
  p.kb_apply = static_cast<int32_t>((m + kAtom - 1) / kAtom);
  for (int k = 0; k < steps; ++k) {
    p.coef[k][0] = coefs[3 * k + 1];
    p.coef[k][1] = coefs[3 * k + 2];
    p.coef[k][2] = round_to_bf16(coefs[3 * k]);
  }
  p.counters = static_cast<uint32_t*>(scratch);
  p.gram = static_cast<const uint16_t*>(gram);
  p.mp = static_cast<int32_t>(mp);

  const int pairs = p.total < capacity ? p.total : capacity;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(2 * pairs, 1, 1);
  cfg.blockDim = dim3(kTileThreads, 1, 1);
  cfg.dynamicSmemBytes = FusedCfg::kSmemBytes;
  cfg.stream = stream;
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = 2;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[1].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 2;
  e = wide ? cudaLaunchKernelEx(&cfg, polar_fused_kernel<true>, maps, p)
           : cudaLaunchKernelEx(&cfg, polar_fused_kernel<false>, maps, p);
  if (e != cudaSuccess) return static_cast<int>(e);
  g_launch_count.fetch_add(1, std::memory_order_relaxed);
  *done = true;
  return MUON_POLAR_OK;
}

}  // namespace
}  // namespace muon_sm100

using namespace muon_sm100;

// ============================================================ no allocation
// Split-K scratch of muon_polar_gram_static_scratch_sm100, for callers that
// cannot allocate device memory themselves: a file-scope device array (1 KiB
// of arrival counters + fp32 partial bands for 80 split items, 20 MiB +
// 1 KiB in all).  Every GPU that loads this library holds it until the
// process exits.  Host code must not hand `g_static_scratch` to a kernel:
// on the host that name is only a stand-in for the device symbol; the
// device address comes from cudaGetSymbolAddress below.
constexpr size_t kStaticScratchItems = 80;
constexpr size_t kStaticScratchBytes =
    muon_sm100::kCounterBytes + kStaticScratchItems * muon_sm100::kPartialItemBytes;
static_assert(kStaticScratchBytes == MUON_POLAR_STATIC_SCRATCH_BYTES,
              "header and library agree on the static scratch size");
static __device__ __align__(256) uint8_t g_static_scratch[kStaticScratchBytes];

namespace {
// A device address looked up once per device.  Only a successful lookup is
// kept: a failed one (say, made during a stream capture, or with another
// error pending) is reported to that caller and tried again by the next.
struct AddressSlot {
  std::mutex mu;
  void* ptr = nullptr;
};

typedef cudaError_t (*AddressLookup)(void** out);

int cached_address(AddressSlot& slot, AddressLookup lookup, void** out) {
  std::lock_guard<std::mutex> lock(slot.mu);
  if (slot.ptr == nullptr) {
    void* p = nullptr;
    const cudaError_t e = lookup(&p);
    if (e != cudaSuccess || p == nullptr) {
      (void)cudaGetLastError();  // leave no error behind for later calls
      return e != cudaSuccess ? static_cast<int>(e) : MUON_POLAR_ERR_DRIVER;
    }
    slot.ptr = p;
  }
  *out = slot.ptr;
  return MUON_POLAR_OK;
}

cudaError_t lookup_static_scratch(void** out) {
  return cudaGetSymbolAddress(out, g_static_scratch);
}

AddressSlot g_static_scratch_address[muon_sm100::kMaxDevices];

// Device address of g_static_scratch on the current device `dev` (looked up
// with that device current).
int static_scratch_address(int dev, void** out) {
  return cached_address(g_static_scratch_address[dev], lookup_static_scratch, out);
}

// Bytes of the array a plan may use (muon_polar_set_static_scratch_limit).
std::atomic<size_t> g_static_scratch_limit{kStaticScratchBytes};

int gram_static_scratch_impl(const void* x, void* gram, int64_t batch, int64_t m,
                             int64_t n, int64_t ldx, cudaStream_t stream) {
  int rc = check_x_args(x, batch, m, n, ldx);
  if (rc != MUON_POLAR_OK) return rc;
  if (gram == nullptr) return MUON_POLAR_ERR_INVALID_ARGUMENT;
  if (!aligned16(gram)) return MUON_POLAR_ERR_ALIGNMENT;
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return static_cast<int>(e);
  if (dev < 0 || dev >= kMaxDevices) return MUON_POLAR_ERR_UNSUPPORTED_DEVICE;
  void* scratch = nullptr;
  rc = static_scratch_address(dev, &scratch);
  if (rc != MUON_POLAR_OK) return rc;
  // The split plan of muon_polar_gram_sm100 on the CTA-pair path with enough
  // scratch; a plan that needs more than the static array is refused, and the
  // array's arrival counters (left as the previous call left them) are
  // cleared before the launch.
  return gram_impl<kGramBf16>(x, gram, batch, m, n, ldx, scratch,
                              g_static_scratch_limit.load(std::memory_order_relaxed), stream,
                              /*fixed_scratch=*/true);
}
}  // namespace

extern "C" {

int muon_polar_abi_version(void) { return MUON_POLAR_ABI_VERSION; }

const char* muon_polar_status_string(int status) {
  switch (status) {
    case MUON_POLAR_OK:
      return "success";
    case MUON_POLAR_ERR_INVALID_ARGUMENT:
      return "invalid argument (null pointer, non-positive size, ld < n or size limit)";
    case MUON_POLAR_ERR_UNSUPPORTED_DEVICE:
      return "current device is not an sm_100 (B200-class) GPU";
    case MUON_POLAR_ERR_ALIGNMENT:
      return "pointer not 16-byte aligned or leading dimension not a multiple of 8";
    case MUON_POLAR_ERR_TENSOR_MAP:
      return "cuTensorMapEncodeTiled rejected the tensor layout";
    case MUON_POLAR_ERR_WORKSPACE:
      return "workspace too small or misaligned";
    case MUON_POLAR_ERR_DRIVER:
      return "CUDA driver entry point cuTensorMapEncodeTiled unavailable";
    case MUON_POLAR_ERR_STATIC_SCRATCH:
      return "problem needs more split-K scratch than the library's static "
             "buffer holds (MUON_POLAR_STATIC_SCRATCH_BYTES); use "
             "muon_polar_gram_sm100 with caller-owned scratch";
    default:
      break;
  }
  if (status > 0) return cudaGetErrorString(static_cast<cudaError_t>(status));
  return "unknown status";
}

int64_t muon_polar_padded_rows(int64_t m) { return m <= 0 ? 0 : padded_rows(m); }

size_t muon_polar_workspace_bytes(int64_t batch, int64_t m) {
  if (batch <= 0 || m <= 0) return 0;
  const int64_t mp = padded_rows(m);
  return static_cast<size_t>(2 * batch * mp * mp * 2);
}

int muon_polar_gram_sm100(const void* x, void* gram, int64_t batch, int64_t m,
                          int64_t n, int64_t ldx, void* scratch,
                          size_t scratch_bytes, void* stream) {
  return gram_impl<kGramBf16>(x, gram, batch, m, n, ldx, scratch, scratch_bytes,
                              static_cast<cudaStream_t>(stream));
}

int muon_polar_gram_f32_band_sm100(const void* x, void* gram_f32, int64_t batch, int64_t m,
                                   int64_t n, int64_t ldx, int64_t row_begin, int64_t row_count,
                                   int sm_reserve, void* scratch, size_t scratch_bytes,
                                   void* stream) {
  return gram_f32_band_impl(x, gram_f32, batch, m, n, ldx, row_begin, row_count, sm_reserve,
                            scratch, scratch_bytes, static_cast<cudaStream_t>(stream));
}

int muon_polar_gram_f32_sm100(const void* x, void* gram_f32, int64_t batch,
                              int64_t m, int64_t n, int64_t ldx, void* scratch,
                              size_t scratch_bytes, void* stream) {
  return gram_impl<kGramF32>(x, gram_f32, batch, m, n, ldx, scratch,
                             scratch_bytes, static_cast<cudaStream_t>(stream));
}

int muon_polar_poly_sm100(const void* gram, void* poly, int64_t batch,
                          int64_t mp, float b, float c, void* scratch,
                          size_t scratch_bytes, void* stream) {
  return poly_impl(gram, poly, batch, mp, b, c, scratch, scratch_bytes,
                   static_cast<cudaStream_t>(stream));
}

int muon_polar_poly_rows_sm100(const void* gram, void* poly, int64_t batch, int64_t mp,
                               int64_t row_begin, int64_t row_count, float b, float c,
                               void* stream) {
  return poly_rows_impl(gram, poly, batch, mp, row_begin, row_count, b, c,
                        static_cast<cudaStream_t>(stream));
}

int muon_polar_apply_sm100(const void* poly, const void* x, void* y,
                           int64_t batch, int64_t m, int64_t n, int64_t ldx,
                           int64_t ldy, float a, void* stream) {
  return apply_impl(poly, x, y, batch, m, n, ldx, ldy, a,
                    static_cast<cudaStream_t>(stream));
}

int muon_polar_step_sm100(const void* x, void* y, void* workspace,
                          size_t workspace_bytes, void* scratch,
                          size_t scratch_bytes, int64_t batch, int64_t m,
                          int64_t n, int64_t ldx, int64_t ldy, float a,
                          float b, float c, void* stream) {
  int rc = check_x_args(x, batch, m, n, ldx);
  if (rc != MUON_POLAR_OK) return rc;
  if (y == nullptr || y == x || ldy < n) return MUON_POLAR_ERR_INVALID_ARGUMENT;
  if (workspace == nullptr || !aligned16(workspace) ||
      workspace_bytes < muon_polar_workspace_bytes(batch, m))
    return MUON_POLAR_ERR_WORKSPACE;
  const int64_t mp = padded_rows(m);
  uint8_t* ws = static_cast<uint8_t*>(workspace);
  void* gram = ws;
  void* poly = ws + static_cast<size_t>(batch * mp * mp * 2);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  bool fused = false;
  const float coefs[3] = {a, b, c};
  rc = fused_steps_impl(x, y, nullptr, 0, gram, poly, scratch, scratch_bytes, batch, m, n, ldx,
                        ldy, coefs, 1, s, &fused);
  if (rc != MUON_POLAR_OK || fused) return rc;
  rc = gram_impl<kGramBf16>(x, gram, batch, m, n, ldx, scratch, scratch_bytes, s);
  if (rc != MUON_POLAR_OK) return rc;
  rc = poly_impl(gram, poly, batch, mp, b, c, scratch, scratch_bytes, s);
  if (rc != MUON_POLAR_OK) return rc;
  return apply_impl(poly, x, y, batch, m, n, ldx, ldy, a, s);
}

int muon_polar_gram_t_sm100(const void* x, void* gram, int64_t batch, int64_t m,
                            int64_t n, int64_t ldx, void* scratch, size_t scratch_bytes,
                            void* stream) {
  return gram_impl<kGramT>(x, gram, batch, m, n, ldx, scratch, scratch_bytes,
                           static_cast<cudaStream_t>(stream));
}

int muon_polar_apply_t_sm100(const void* poly, const void* x, void* y, int64_t batch,
                             int64_t m, int64_t n, int64_t ldx, int64_t ldy, float a,
                             void* stream) {
  return apply_t_impl(poly, x, y, batch, m, n, ldx, ldy, a, static_cast<cudaStream_t>(stream));
}

int muon_polar_step_t_sm100(const void* x, void* y, void* workspace, size_t workspace_bytes,
                            void* scratch, size_t scratch_bytes, int64_t batch, int64_t m,
                            int64_t n, int64_t ldx, int64_t ldy, float a, float b, float c,
                            void* stream) {
  int rc = check_x_args(x, batch, m, n, ldx);
  if (rc != MUON_POLAR_OK) return rc;
  if (y == nullptr || y == x || ldy < n || n > (1 << 24)) return MUON_POLAR_ERR_INVALID_ARGUMENT;
  if (workspace == nullptr || !aligned16(workspace) ||
      workspace_bytes < muon_polar_workspace_bytes(batch, n))
    return MUON_POLAR_ERR_WORKSPACE;
  const int64_t np = padded_rows(n);
  uint8_t* ws = static_cast<uint8_t*>(workspace);
  void* gram = ws;
  void* poly = ws + static_cast<size_t>(batch * np * np * 2);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  rc = gram_impl<kGramT>(x, gram, batch, m, n, ldx, scratch, scratch_bytes, s);
  if (rc != MUON_POLAR_OK) return rc;
  rc = poly_impl(gram, poly, batch, np, b, c, scratch, scratch_bytes, s);
  if (rc != MUON_POLAR_OK) return rc;
  return apply_t_impl(poly, x, y, batch, m, n, ldx, ldy, a, s);
}

int muon_polar_steps_sm100(const void* x, void* y, void* buf0, void* buf1, int64_t ldb,
                           void* workspace, size_t workspace_bytes, void* scratch,
                           size_t scratch_bytes, int64_t batch, int64_t m, int64_t n,
                           int64_t ldx, int64_t ldy, const float* coefficients, int steps,
                           void* stream) {
  int rc = check_x_args(x, batch, m, n, ldx);
  if (rc != MUON_POLAR_OK) return rc;
  if (y == nullptr || y == x || ldy < n || coefficients == nullptr || steps < 1 ||
      n > (1 << 24))
    return MUON_POLAR_ERR_INVALID_ARGUMENT;
  if (steps > 1) {
    // step 0 must not overwrite its input, nor the last step its own input
    if (buf0 == nullptr || buf1 == nullptr || buf0 == buf1 || ldb < n || buf0 == x ||
        y == ((steps & 1) ? buf1 : buf0))
      return MUON_POLAR_ERR_INVALID_ARGUMENT;
    if (!aligned16(buf0) || !aligned16(buf1) || (ldb % 8) != 0) return MUON_POLAR_ERR_ALIGNMENT;
  }
  const bool tall = m > n;
  const int64_t g = tall ? n : m;
  if (workspace == nullptr || !aligned16(workspace) ||
      workspace_bytes < muon_polar_workspace_bytes(batch, g))
    return MUON_POLAR_ERR_WORKSPACE;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  void* buf[2] = {buf0, buf1};
  // step i reads x (i = 0) or buf[(i - 1) % 2] and writes buf[i % 2], the
  // last step y
  int i = 0;
  while (i < steps) {
    const void* in = i == 0 ? x : buf[(i - 1) & 1];
    const int64_t ld_in = i == 0 ? ldx : ldb;
    if (!tall) {
      // as many steps as one fused launch takes
      const int cnt = steps - i < kMaxFusedSteps ? steps - i : kMaxFusedSteps;
      const bool last = i + cnt == steps;
      void* out = last ? y : buf[(i + cnt - 1) & 1];
      void* local[2] = {buf[i & 1], buf[(i + 1) & 1]};
      const int64_t mp = padded_rows(m);
      uint8_t* ws = static_cast<uint8_t*>(workspace);
      bool fused = false;
      rc = fused_steps_impl(in, out, local, ldb, ws, ws + static_cast<size_t>(batch * mp * mp * 2),
                            scratch, scratch_bytes, batch, m, n, ld_in, last ? ldy : ldb,
                            coefficients + 3 * i, cnt, s, &fused);
      if (rc != MUON_POLAR_OK) return rc;
      if (fused) {
        i += cnt;
        continue;
      }
    }
    const bool last = i == steps - 1;
    void* out = last ? y : buf[i & 1];
    const float* cf = coefficients + 3 * i;
    rc = tall ? muon_polar_step_t_sm100(in, out, workspace, workspace_bytes, scratch,
                                        scratch_bytes, batch, m, n, ld_in, last ? ldy : ldb,
                                        cf[0], cf[1], cf[2], stream)
              : muon_polar_step_sm100(in, out, workspace, workspace_bytes, scratch, scratch_bytes,
                                      batch, m, n, ld_in, last ? ldy : ldb, cf[0], cf[1], cf[2],
                                      stream);
    if (rc != MUON_POLAR_OK) return rc;
    ++i;
  }
  return MUON_POLAR_OK;
}

size_t muon_polar_scratch_bytes(int64_t batch, int64_t m, int64_t n) {
  if (batch <= 0 || m <= 0 || n <= 0) return 0;
  int pairs = 0, ctas = 0;
  DeviceState* st = nullptr;
  if (current_device_state(&st) != MUON_POLAR_OK ||
      tile_capacity<kGramBf16, 2>(st, &pairs) != MUON_POLAR_OK || pairs <= 0 ||
      tile_capacity<kGramBf16, 1>(st, &ctas) != MUON_POLAR_OK || ctas <= 0) {
    (void)cudaGetLastError();
    pairs = 512;  // no usable device: the largest the split planner could use
    ctas = 1024;
  }
  const int64_t mp = padded_rows(m);

  const int64_t d2 = mp / kPairM, d1 = mp / kHalf;
  const int64_t t2 = d2 * (d2 + 1) / 2 * batch, t1 = d1 * (d1 + 1) / 2 * batch;
  // The largest plan either engine makes for kernels (1) and (2); the fused
  // step's dependency counters live in the counter area.
  size_t need = kCounterBytes;
  const size_t plans[6] = {
      split_scratch_bytes<2>(
          t2, choose_splits<kGramBf16, 2>(t2, k_blocks_of<kGramBf16, 2>(n), pairs)),
      split_scratch_bytes<2>(t2, choose_splits<kGramF32, 2>(t2, k_blocks_of<kGramF32, 2>(n), pairs)),
      split_scratch_bytes<2>(t2, choose_splits<kPoly, 2>(t2, k_blocks_of<kPoly, 2>(mp), pairs)),
      split_scratch_bytes<1>(
          t1, choose_splits<kGramBf16, 1>(t1, k_blocks_of<kGramBf16, 1>(n), ctas)),
      split_scratch_bytes<1>(t1, choose_splits<kGramF32, 1>(t1, k_blocks_of<kGramF32, 1>(n), ctas)),
      split_scratch_bytes<1>(t1, choose_splits<kPoly, 1>(t1, k_blocks_of<kPoly, 1>(mp), ctas))};
  for (size_t v : plans) need = v > need ? v : need;
  return need;
}

int muon_polar_scratch_init(void* scratch, size_t scratch_bytes, void* stream) {
  if (scratch == nullptr) return MUON_POLAR_ERR_INVALID_ARGUMENT;
  if (scratch_bytes == 0) return MUON_POLAR_OK;
  const size_t n = scratch_bytes < kCounterBytes ? scratch_bytes : kCounterBytes;
  cudaError_t e = cudaMemsetAsync(scratch, 0, n, static_cast<cudaStream_t>(stream));
  return e == cudaSuccess ? MUON_POLAR_OK : static_cast<int>(e);
}

int muon_polar_gram_static_scratch_sm100(const void* x, void* gram, int64_t batch,
                                         int64_t m, int64_t n, int64_t ldx,
                                         void* stream) {
  return gram_static_scratch_impl(x, gram, batch, m, n, ldx,
                                  static_cast<cudaStream_t>(stream));
}

int64_t muon_polar_packed_units(int64_t m) { return m <= 0 ? 0 : packed_units_of(padded_rows(m)); }

int muon_polar_gram_f32_packed_sm100(const void* x, void* packed_f32, int64_t batch, int64_t m,
                                     int64_t n, int64_t ldx, void* scratch, size_t scratch_bytes,
                                     void* stream) {
  return gram_impl<kGramF32>(x, packed_f32, batch, m, n, ldx, scratch, scratch_bytes,
                             static_cast<cudaStream_t>(stream), false, /*packed=*/true);
}

int muon_polar_poly_packed_sm100(const void* gram, void* packed_poly, int64_t batch, int64_t mp,
                                 int64_t unit_begin, int64_t unit_count, float b, float c,
                                 void* stream) {
  return poly_packed_impl(gram, packed_poly, batch, mp, unit_begin, unit_count, b, c,
                          static_cast<cudaStream_t>(stream));
}

int muon_polar_unpack_sym_sm100(const void* packed, void* full, int64_t batch, int64_t mp,
                                void* stream) {
  return unpack_sym_impl(packed, full, batch, mp, static_cast<cudaStream_t>(stream));
}

int muon_polar_cast_f32_bf16_sm100(const void* src, void* dst, int64_t count,
                                   void* stream) {
  if (src == nullptr || dst == nullptr || count <= 0)
    return MUON_POLAR_ERR_INVALID_ARGUMENT;
  DeviceState* st = nullptr;
  int rc = current_device_state(&st);
  if (rc != MUON_POLAR_OK) return rc;
  const int64_t want = (count + 255) / 256;
  const int grid = static_cast<int>(want < st->sms * 8 ? want : st->sms * 8);
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(grid, 1, 1);
  cfg.blockDim = dim3(256, 1, 1);
  cfg.stream = static_cast<cudaStream_t>(stream);
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  cudaError_t e = cudaLaunchKernelEx(&cfg, cast_f32_bf16_kernel,
                                     static_cast<const float*>(src),
                                     static_cast<uint16_t*>(dst), count);
  if (e != cudaSuccess) return static_cast<int>(e);
  g_launch_count.fetch_add(1, std::memory_order_relaxed);
  return MUON_POLAR_OK;
}

int muon_polar_read_device_status(int device, uint32_t* flags, int clear) {
  if (flags == nullptr) return MUON_POLAR_ERR_INVALID_ARGUMENT;
  int prev = 0;
  cudaError_t e = cudaGetDevice(&prev);
  if (e != cudaSuccess) return static_cast<int>(e);
  if (device != prev) {
    e = cudaSetDevice(device);
    if (e != cudaSuccess) return static_cast<int>(e);
  }
  uint32_t v = 0;
  e = cudaDeviceSynchronize();
  if (e == cudaSuccess) e = cudaMemcpyFromSymbol(&v, g_watchdog, sizeof(v));
  if (e == cudaSuccess && clear) {
    const uint32_t zero = 0;
    e = cudaMemcpyToSymbol(g_watchdog, &zero, sizeof(zero));
  }
  if (device != prev) cudaSetDevice(prev);
  if (e != cudaSuccess) return static_cast<int>(e);
  *flags = v;
  return MUON_POLAR_OK;
}

int muon_polar_set_kernel_policy(int policy) {
  if (policy < 0 || policy > 2) return MUON_POLAR_ERR_INVALID_ARGUMENT;
  return g_policy.exchange(policy);
}

int muon_polar_set_step_mode(int mode) {
  if (mode < 0 || mode > 2) return MUON_POLAR_ERR_INVALID_ARGUMENT;
  return g_step_mode.exchange(mode);
}

int muon_polar_set_stage_mode(int mode) {
  if (mode < 0 || mode > 2) return MUON_POLAR_ERR_INVALID_ARGUMENT;
  return g_stage_mode.exchange(mode);
}

int muon_polar_set_halves_mode(int mode) {
  if (mode < 0 || mode > 2) return MUON_POLAR_ERR_INVALID_ARGUMENT;
  return g_halves_mode.exchange(mode);
}

int muon_polar_set_split_mode(int mode) {
  if (mode < 0 || mode > 2) return MUON_POLAR_ERR_INVALID_ARGUMENT;
  return g_split_mode.exchange(mode);
}

int muon_polar_device_pairs(int* pairs) {
  if (pairs == nullptr) return MUON_POLAR_ERR_INVALID_ARGUMENT;
  DeviceState* st = nullptr;
  int rc = current_device_state(&st);
  if (rc != MUON_POLAR_OK) return rc;
  return tile_capacity<kGramBf16, 2>(st, pairs);
}

uint64_t muon_polar_launch_count(void) {
  return g_launch_count.load(std::memory_order_relaxed);
}

uint64_t muon_polar_tensor_map_encodes(void) {
  return g_map_encodes.load(std::memory_order_relaxed);
}

int muon_polar_set_wait_limit_ns(uint64_t limit_ns, uint64_t* previous) {
  if (limit_ns < 1000ull || limit_ns > 60000000000ull) return MUON_POLAR_ERR_INVALID_ARGUMENT;
  DeviceState* st = nullptr;
  int rc = current_device_state(&st);
  if (rc != MUON_POLAR_OK) return rc;
  uint64_t old = 0;
  cudaError_t e = cudaMemcpyFromSymbol(&old, g_wait_limit_ns, sizeof(old));
  if (e == cudaSuccess) e = cudaMemcpyToSymbol(g_wait_limit_ns, &limit_ns, sizeof(limit_ns));
  if (e != cudaSuccess) return static_cast<int>(e);
  if (previous != nullptr) *previous = old;
  return MUON_POLAR_OK;
}

size_t muon_polar_set_static_scratch_limit(size_t bytes) {
  const size_t v = (bytes == 0 || bytes > kStaticScratchBytes) ? kStaticScratchBytes : bytes;
  return g_static_scratch_limit.exchange(v);
}

int muon_polar_decode_tile(int64_t tile, int symmetric, int64_t tiles_m, int64_t tiles_n,
                           int64_t tiles_per_batch, int64_t first_row, int64_t* out) {
  if (out == nullptr || tile < 0 || tiles_m <= 0 || tiles_n <= 0 || tiles_per_batch <= 0 ||
      first_row < 0 || first_row >= tiles_m || tile > INT32_MAX || tiles_m > INT32_MAX ||
      tiles_n > INT32_MAX || tiles_per_batch > INT32_MAX)
    return MUON_POLAR_ERR_INVALID_ARGUMENT;
  if (symmetric) {
    // the tiles (tm, tn >= tm) of rows first_row .. tiles_m - 1
    const int64_t rows = tiles_m - first_row;
    if (tiles_per_batch > rows * (rows + 1) / 2) return MUON_POLAR_ERR_INVALID_ARGUMENT;
  } else if (tiles_per_batch != tiles_m * tiles_n) {
    return MUON_POLAR_ERR_INVALID_ARGUMENT;
  }
  const TileCoord t = decode_tile(static_cast<int>(tile), symmetric != 0,
                                  static_cast<int>(tiles_m), static_cast<int>(tiles_n),
                                  static_cast<int>(tiles_per_batch), static_cast<int>(first_row));
  out[0] = t.b;
  out[1] = t.tm;
  out[2] = t.tn;
  return MUON_POLAR_OK;
}

namespace {
int g_fake_lookups = 0;
cudaError_t fake_lookup_fails_once(void** out) {
  static char target;
  if (g_fake_lookups++ == 0) return cudaErrorStreamCaptureUnsupported;
  *out = &target;
  return cudaSuccess;
}
}  // namespace

int muon_polar_check_address_cache(void) {
  AddressSlot slot;
  g_fake_lookups = 0;
  void* p = nullptr;
  // 1: the first lookup fails and is reported; nothing is cached
  if (cached_address(slot, fake_lookup_fails_once, &p) != cudaErrorStreamCaptureUnsupported ||
      p != nullptr || slot.ptr != nullptr)
    return 1;
  // 2: the next call looks up again and succeeds
  if (cached_address(slot, fake_lookup_fails_once, &p) != MUON_POLAR_OK || p == nullptr ||
      g_fake_lookups != 2)
    return 2;
  // 3: a later call uses the cached address without another lookup
  void* q = nullptr;
  if (cached_address(slot, fake_lookup_fails_once, &q) != MUON_POLAR_OK || q != p ||
      g_fake_lookups != 2)
    return 3;
  return 0;
}

}  // extern "C"
