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
// CTA layout (192 threads): warp 0 lane 0 issues TMA loads into a ring of
// shared-memory stages; warp 1 owns the tensor memory and its lane 0 issues
// tcgen05.mma (128 x BN x 16 per instruction) into one of two TMEM
// accumulators; warps 2-5 drain the other accumulator (tcgen05.ld), apply
// the epilogue and store to global memory, so the epilogue of tile i
// overlaps the main loop of tile i+1.  Every wait is bounded in wall-clock
// time; a kernel that gives up records a watchdog bit and returns.
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

constexpr int kBM = 128;        // tile rows = TMEM lanes
constexpr int kBK = 64;         // bf16 elements per 128-byte swizzle row
constexpr int kThreads = 192;   // 6 warps
constexpr uint32_t kABytes = kBM * kBK * 2;  // 16 KiB per stage

enum Kind : int { kGramBf16 = 0, kGramF32 = 1, kPoly = 2, kApply = 3 };

__device__ uint32_t g_watchdog = 0;

struct EpiParams {
  void* out;
  const void* aux;            // kPoly: A (bf16); kApply: X (bf16)
  int64_t out_batch_stride;   // elements
  int64_t aux_batch_stride;   // elements
  int32_t out_ld;             // elements
  int32_t aux_ld;             // elements
  int32_t rows;               // valid rows of the output (kApply: m)
  int32_t cols;               // valid cols of the output (kApply: n)
  int32_t tiles_m;
  int32_t tiles_n;
  int32_t tiles_per_batch;
  int32_t total_tiles;
  int32_t k_blocks;
  float coef_b;
  float coef_c;
  float alpha;                // kApply: a already rounded to bf16
};

template <int BN>
struct Config {
  static constexpr int kStages = BN == 256 ? 4 : 6;
  static constexpr uint32_t kBBytes = BN * kBK * 2;
  static constexpr uint32_t kStageBytes = kABytes + kBBytes;
  static constexpr uint32_t kTmemCols = 2 * BN;  // two accumulators
  static constexpr uint32_t kBarrierBytes = 256;
  static constexpr uint32_t kSmemBytes =
      1024 + kStages * kStageBytes + kBarrierBytes;
  static_assert(kSmemBytes <= 232448, "shared memory budget");
};

struct TileCoord {
  int b, tm, tn;
};

// Linear tile index -> (batch, tile row, tile col).  Symmetric kinds walk the
// upper triangle row by row: row tm holds tiles (tm, tm..d-1) (the
// reference enumerates the same set, asc:129-146, 609-630).
template <int KIND>
__device__ __forceinline__ TileCoord decode_tile(int tile, const EpiParams& p) {
  TileCoord t;
  t.b = tile / p.tiles_per_batch;
  int r = tile - t.b * p.tiles_per_batch;
  if constexpr (KIND == kApply) {
    t.tm = r / p.tiles_n;
    t.tn = r - t.tm * p.tiles_n;
  } else {
    const int d = p.tiles_m;
    int tm = 0;
    while (r >= d - tm) {
      r -= d - tm;
      ++tm;
    }
    t.tm = tm;
    t.tn = tm + r;
  }
  return t;
}

__device__ __forceinline__ float bf16_bits_to_float(uint32_t bits16) {
  return __uint_as_float(bits16 << 16);
}
__device__ __forceinline__ uint32_t float_to_bf16_bits(float v) {
  __nv_bfloat16 h = __float2bfloat16_rn(v);
  return static_cast<uint32_t>(*reinterpret_cast<uint16_t*>(&h));
}
__device__ __forceinline__ uint32_t pack_bf16x2(float lo, float hi) {
  return float_to_bf16_bits(lo) | (float_to_bf16_bits(hi) << 16);
}

// Writes 32 values of tile row `row` (columns c0..c0+31 of the tile) of a
// symmetric output at (tm,tn) and, off the diagonal, the mirrored column at
// (tn,tm).  In the mirror, lanes of a warp hold consecutive rows, so each
// column store of the warp is one contiguous 64-byte (bf16) or 128-byte
// (fp32) segment.
template <bool kF32>
__device__ __forceinline__ void store_symmetric(const EpiParams& p,
                                                const TileCoord& tc, int row,
                                                int c0, const float (&v)[32]) {
  const int64_t ld = p.out_ld;
  const int64_t grow = static_cast<int64_t>(tc.tm) * kBM + row;
  const int64_t gcol = static_cast<int64_t>(tc.tn) * kBM + c0;
  if constexpr (kF32) {
    float* base = static_cast<float*>(p.out) + tc.b * p.out_batch_stride;
    float4* dst = reinterpret_cast<float4*>(base + grow * ld + gcol);
#pragma unroll
    for (int i = 0; i < 8; ++i)
      dst[i] = make_float4(v[4 * i], v[4 * i + 1], v[4 * i + 2], v[4 * i + 3]);
    if (tc.tm != tc.tn) {
#pragma unroll
      for (int j = 0; j < 32; ++j) base[(gcol + j) * ld + grow] = v[j];
    }
  } else {
    uint16_t* base = static_cast<uint16_t*>(p.out) + tc.b * p.out_batch_stride;
    uint32_t packed[16];
#pragma unroll
    for (int i = 0; i < 16; ++i) packed[i] = pack_bf16x2(v[2 * i], v[2 * i + 1]);
    uint4* dst = reinterpret_cast<uint4*>(base + grow * ld + gcol);
#pragma unroll
    for (int i = 0; i < 4; ++i)
      dst[i] = make_uint4(packed[4 * i], packed[4 * i + 1], packed[4 * i + 2],
                          packed[4 * i + 3]);
    if (tc.tm != tc.tn) {
#pragma unroll
      for (int j = 0; j < 32; ++j) {
        const uint16_t h = static_cast<uint16_t>(
            (j & 1) ? (packed[j >> 1] >> 16) : (packed[j >> 1] & 0xFFFFu));
        base[(gcol + j) * ld + grow] = h;
      }
    }
  }
}

template <int BN, int KIND>
__device__ __forceinline__ void epilogue_chunk(const EpiParams& p,
                                               const TileCoord& tc, int row,
                                               int chunk,
                                               const uint32_t (&r)[32]) {
  float v[32];
#pragma unroll
  for (int j = 0; j < 32; ++j) v[j] = __uint_as_float(r[j]);
  const int c0 = chunk * 32;
  if constexpr (KIND == kGramBf16) {
    store_symmetric<false>(p, tc, row, c0, v);
  } else if constexpr (KIND == kGramF32) {
    store_symmetric<true>(p, tc, row, c0, v);
  } else if constexpr (KIND == kPoly) {
    // P = bf16( fl(b*A) + fl(c*acc) ), the reference's separate Muls/Add
    // (asc:929-940): no fused multiply-add.
    const int64_t grow = static_cast<int64_t>(tc.tm) * kBM + row;
    const int64_t gcol = static_cast<int64_t>(tc.tn) * kBM + c0;
    const uint16_t* ab = static_cast<const uint16_t*>(p.aux) +
                         tc.b * p.aux_batch_stride + grow * p.aux_ld + gcol;
    const uint4* src = reinterpret_cast<const uint4*>(ab);
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const uint4 q = src[i];
      const uint32_t w[4] = {q.x, q.y, q.z, q.w};
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const float a_lo = bf16_bits_to_float(w[e] & 0xFFFFu);
        const float a_hi = bf16_bits_to_float(w[e] >> 16);
        const int j = 8 * i + 2 * e;
        v[j] = __fadd_rn(__fmul_rn(p.coef_b, a_lo), __fmul_rn(p.coef_c, v[j]));
        v[j + 1] = __fadd_rn(__fmul_rn(p.coef_b, a_hi),
                             __fmul_rn(p.coef_c, v[j + 1]));
      }
    }
    store_symmetric<false>(p, tc, row, c0, v);
  } else {  // kApply
    const int64_t grow = static_cast<int64_t>(tc.tm) * kBM + row;
    if (grow >= p.rows) return;
    const int64_t gcol = static_cast<int64_t>(tc.tn) * BN + c0;
    if (gcol >= p.cols) return;
    const uint16_t* xr = static_cast<const uint16_t*>(p.aux) +
                         tc.b * p.aux_batch_stride + grow * p.aux_ld + gcol;
    uint16_t* yr = static_cast<uint16_t*>(p.out) + tc.b * p.out_batch_stride +
                   grow * p.out_ld + gcol;
    // Y = bf16( bf16(T) + bf16(alpha*x) ), alpha already a bf16 value.
    if (gcol + 32 <= p.cols) {
      const uint4* src = reinterpret_cast<const uint4*>(xr);
      uint4* dst = reinterpret_cast<uint4*>(yr);
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const uint4 q = src[i];
        uint32_t w[4] = {q.x, q.y, q.z, q.w};
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const int j = 8 * i + 2 * e;
          const float ax_lo = bf16_bits_to_float(float_to_bf16_bits(
              p.alpha * bf16_bits_to_float(w[e] & 0xFFFFu)));
          const float ax_hi = bf16_bits_to_float(
              float_to_bf16_bits(p.alpha * bf16_bits_to_float(w[e] >> 16)));
          const float t_lo = bf16_bits_to_float(float_to_bf16_bits(v[j]));
          const float t_hi = bf16_bits_to_float(float_to_bf16_bits(v[j + 1]));
          w[e] = pack_bf16x2(t_lo + ax_lo, t_hi + ax_hi);
        }
        dst[i] = make_uint4(w[0], w[1], w[2], w[3]);
      }
    } else {
      const int nvalid = static_cast<int>(p.cols - gcol);
#pragma unroll
      for (int j = 0; j < 32; ++j) {
        if (j < nvalid) {
          const float ax = bf16_bits_to_float(
              float_to_bf16_bits(p.alpha * bf16_bits_to_float(xr[j])));
          const float t = bf16_bits_to_float(float_to_bf16_bits(v[j]));
          yr[j] = static_cast<uint16_t>(float_to_bf16_bits(t + ax));
        }
      }
    }
  }
}

template <int BN, int KIND>
__global__ void __launch_bounds__(kThreads, 1)
    polar_gemm_kernel(const __grid_constant__ CUtensorMap tmap_a,
                      const __grid_constant__ CUtensorMap tmap_b,
                      const EpiParams p) {
  using Cfg = Config<BN>;
  constexpr int S = Cfg::kStages;
  constexpr bool kBmn = (KIND == kApply);

  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw_addr = smem_addr(smem_raw);
  uint8_t* smem = smem_raw + ((1024u - (raw_addr & 1023u)) & 1023u);
  uint8_t* sA = smem;
  uint8_t* sB = smem + S * kABytes;
  uint64_t* full = reinterpret_cast<uint64_t*>(sB + S * Cfg::kBBytes);
  uint64_t* empty = full + S;
  uint64_t* tfull = empty + S;
  uint64_t* tempty = tfull + 2;
  uint64_t* drain = tempty + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(drain + 1);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;

  if (threadIdx.x == 0) {
    for (int s = 0; s < S; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int a = 0; a < 2; ++a) {
      mbar_init(&tfull[a], 1);
      mbar_init(&tempty[a], 4);
    }
    mbar_init(drain, 1);
    fence_mbar_init();
    prefetch_tensor_map(&tmap_a);
    prefetch_tensor_map(&tmap_b);
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, Cfg::kTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  // Inputs may come from the kernel launched just before this one.
  grid_dependency_wait();
  grid_launch_dependents();

  if (warp == 0) {
    if (lane == 0) {
      // ---------------- TMA producer
      uint32_t it = 0;
      bool ok = true;
      for (int tile = blockIdx.x; ok && tile < p.total_tiles;
           tile += gridDim.x) {
        const TileCoord tc = decode_tile<KIND>(tile, p);
        for (int kb = 0; kb < p.k_blocks; ++kb, ++it) {
          const uint32_t s = it % S;
          const uint32_t ph = (it / S) & 1u;
          if (!mbar_wait_bounded(&empty[s], ph ^ 1u)) {
            ok = false;
            break;
          }
          mbar_arrive_expect_tx(&full[s], Cfg::kStageBytes);
          tma_load_3d(sA + s * kABytes, &tmap_a, &full[s], kb * kBK,
                      tc.tm * kBM, tc.b);
          if constexpr (!kBmn) {
            tma_load_3d(sB + s * Cfg::kBBytes, &tmap_b, &full[s], kb * kBK,
                        tc.tn * BN, tc.b);
          } else {
#pragma unroll
            for (int j = 0; j < BN / 64; ++j)
              tma_load_3d(sB + s * Cfg::kBBytes + j * (64 * kBK * 2), &tmap_b,
                          &full[s], tc.tn * BN + j * 64, kb * kBK, tc.b);
          }
        }
      }
      if (!ok) atomicOr(&g_watchdog, MUON_POLAR_WATCHDOG_PRODUCER);
      // Drain: the loads of the last stages must land before the CTA exits.
      const uint32_t inflight = it < static_cast<uint32_t>(S) ? it : S;
      for (uint32_t i = it - inflight; i < it; ++i) {
        if (!mbar_wait_bounded(&full[i % S], (i / S) & 1u)) {
          atomicOr(&g_watchdog, MUON_POLAR_WATCHDOG_DRAIN);
          break;
        }
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      // ---------------- tcgen05 MMA issuer
      constexpr uint32_t idesc = idesc_bf16_f32(BN, kBmn ? 1u : 0u);
      uint32_t it = 0;
      uint32_t t = 0;
      bool ok = true;
      for (int tile = blockIdx.x; ok && tile < p.total_tiles;
           tile += gridDim.x, ++t) {
        const uint32_t acc = t & 1u;
        const uint32_t uph = (t >> 1) & 1u;
        if (!mbar_wait_bounded(&tempty[acc], uph ^ 1u)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + acc * BN;
        for (int kb = 0; kb < p.k_blocks; ++kb, ++it) {
          const uint32_t s = it % S;
          const uint32_t ph = (it / S) & 1u;
          if (!mbar_wait_bounded(&full[s], ph)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t a_base = smem_addr(sA + s * kABytes);
          const uint32_t b_base = smem_addr(sB + s * Cfg::kBBytes);
#pragma unroll
          for (int k = 0; k < kBK / 16; ++k) {
            // K-major, 128B swizzle: a K step of 16 bf16 is 32 bytes inside
            // the swizzle row; 8-row groups are 1024 bytes apart.
            const uint64_t ad = smem_desc_sw128(a_base + k * 32, 16, 1024);
            uint64_t bd;
            if constexpr (kBmn) {
              // MN-major, 128B swizzle: 64-column chunks are kBK*128 bytes
              // apart (leading offset), 8-row K groups 1024 bytes (stride
              // offset); a K step of 16 rows is 2048 bytes.
              bd = smem_desc_sw128(b_base + k * 2048, kBK * 128, 1024);
            } else {
              bd = smem_desc_sw128(b_base + k * 32, 16, 1024);
            }
            umma_bf16(d_tmem, ad, bd, idesc, (kb > 0 || k > 0) ? 1u : 0u);
          }
          umma_commit(&empty[s]);
        }
        if (!ok) break;
        umma_commit(&tfull[acc]);
      }
      if (!ok) atomicOr(&g_watchdog, MUON_POLAR_WATCHDOG_MMA);
      // Drain: every MMA issued above completes before TMEM is released.
      umma_commit(drain);
      if (!mbar_wait_bounded(drain, 0))
        atomicOr(&g_watchdog, MUON_POLAR_WATCHDOG_DRAIN);
    }
  } else {
    // ---------------- epilogue warps 2..5
    const int q = warp & 3;  // TMEM lane quarter this warp may access
    const int row = q * 32 + lane;
    uint32_t t = 0;
    for (int tile = blockIdx.x; tile < p.total_tiles;
         tile += gridDim.x, ++t) {
      const TileCoord tc = decode_tile<KIND>(tile, p);
      const uint32_t acc = t & 1u;
      const uint32_t uph = (t >> 1) & 1u;
      int ok = 1;
      if (lane == 0) ok = mbar_wait_bounded(&tfull[acc], uph) ? 1 : 0;
      ok = __shfl_sync(0xffffffffu, ok, 0);
      if (!ok) {
        if (lane == 0) atomicOr(&g_watchdog, MUON_POLAR_WATCHDOG_EPILOGUE);
        break;
      }
      tc_fence_after();
      const uint32_t t_row =
          tmem_base + (static_cast<uint32_t>(q * 32) << 16) + acc * BN;
#pragma unroll 1
      for (int c = 0; c < BN / 32; ++c) {
        uint32_t r[32];
        tmem_ld_32x32b_x32(t_row + c * 32, r);
        tmem_wait_ld();
        epilogue_chunk<BN, KIND>(p, tc, row, c, r);
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&tempty[acc]);
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem_base, Cfg::kTmemCols);
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

// ============================================================== host side

namespace {

std::atomic<uint64_t> g_launch_count{0};

constexpr int kMaxDevices = 64;
constexpr int kNumInstances = 8;

struct DeviceState {
  std::once_flag once;
  int sms = 0;
  int cc_major = 0, cc_minor = 0;
  bool smem_attr_set[kNumInstances] = {};
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
int encode_3d(CUtensorMap* map, CUtensorMapDataType dtype, size_t elem_bytes,
              const void* base, uint64_t d0, uint64_t d1, uint64_t d2,
              uint64_t stride1_elems, uint64_t stride2_elems, uint32_t box0,
              uint32_t box1) {
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
  return r == CUDA_SUCCESS ? MUON_POLAR_OK : MUON_POLAR_ERR_TENSOR_MAP;
}

bool aligned16(const void* p) {
  return (reinterpret_cast<uintptr_t>(p) & 15u) == 0;
}

template <int BN, int KIND>
int launch_gemm(DeviceState* st, int instance, const CUtensorMap& ta,
                const CUtensorMap& tb, const EpiParams& p,
                cudaStream_t stream) {
  auto kern = polar_gemm_kernel<BN, KIND>;
  const uint32_t smem = Config<BN>::kSmemBytes;
  if (!st->smem_attr_set[instance]) {
    std::lock_guard<std::mutex> lock(g_attr_mutex);
    if (!st->smem_attr_set[instance]) {
      cudaError_t e = cudaFuncSetAttribute(
          kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
      if (e != cudaSuccess) return static_cast<int>(e);
      st->smem_attr_set[instance] = true;
    }
  }
  const int grid = p.total_tiles < st->sms ? p.total_tiles : st->sms;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(grid, 1, 1);
  cfg.blockDim = dim3(kThreads, 1, 1);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  cudaError_t e = cudaLaunchKernelEx(&cfg, kern, ta, tb, p);
  if (e != cudaSuccess) return static_cast<int>(e);
  g_launch_count.fetch_add(1, std::memory_order_relaxed);
  return MUON_POLAR_OK;
}

int64_t padded_rows(int64_t m) { return (m + kBM - 1) / kBM * kBM; }

int check_x_args(const void* x, int64_t batch, int64_t m, int64_t n,
                 int64_t ldx) {
  if (x == nullptr || batch <= 0 || m <= 0 || n <= 0 || ldx < n)
    return MUON_POLAR_ERR_INVALID_ARGUMENT;
  if (batch > INT32_MAX || m > (1 << 24) || ldx > (1ll << 31))
    return MUON_POLAR_ERR_INVALID_ARGUMENT;
  if (!aligned16(x) || (ldx % 8) != 0) return MUON_POLAR_ERR_ALIGNMENT;
  return MUON_POLAR_OK;
}

template <int KIND>
int gram_impl(const void* x, void* gram, int64_t batch, int64_t m, int64_t n,
              int64_t ldx, cudaStream_t stream) {
  int rc = check_x_args(x, batch, m, n, ldx);
  if (rc != MUON_POLAR_OK) return rc;
  if (gram == nullptr) return MUON_POLAR_ERR_INVALID_ARGUMENT;
  if (!aligned16(gram)) return MUON_POLAR_ERR_ALIGNMENT;
  DeviceState* st = nullptr;
  rc = current_device_state(&st);
  if (rc != MUON_POLAR_OK) return rc;
  const int64_t mp = padded_rows(m);
  const int64_t d = mp / kBM;
  const int64_t tiles_per_batch = d * (d + 1) / 2;
  if (tiles_per_batch * batch > INT32_MAX) return MUON_POLAR_ERR_INVALID_ARGUMENT;
  CUtensorMap tx;
  rc = encode_3d(&tx, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, x, n, m, batch, ldx,
                 m * ldx, kBK, kBM);
  if (rc != MUON_POLAR_OK) return rc;
  EpiParams p = {};
  p.out = gram;
  p.aux = nullptr;
  p.out_batch_stride = mp * mp;
  p.out_ld = static_cast<int32_t>(mp);
  p.rows = static_cast<int32_t>(mp);
  p.cols = static_cast<int32_t>(mp);
  p.tiles_m = static_cast<int32_t>(d);
  p.tiles_n = static_cast<int32_t>(d);
  p.tiles_per_batch = static_cast<int32_t>(tiles_per_batch);
  p.total_tiles = static_cast<int32_t>(tiles_per_batch * batch);
  p.k_blocks = static_cast<int32_t>((n + kBK - 1) / kBK);
  return launch_gemm<128, KIND>(st, KIND, tx, tx, p, stream);
}

int poly_impl(const void* gram, void* poly, int64_t batch, int64_t mp, float b,
              float c, cudaStream_t stream) {
  if (gram == nullptr || poly == nullptr || batch <= 0 || mp <= 0 ||
      (mp % kBM) != 0 || batch > INT32_MAX || mp > (1 << 24))
    return MUON_POLAR_ERR_INVALID_ARGUMENT;
  if (!aligned16(gram) || !aligned16(poly)) return MUON_POLAR_ERR_ALIGNMENT;
  DeviceState* st = nullptr;
  int rc = current_device_state(&st);
  if (rc != MUON_POLAR_OK) return rc;
  const int64_t d = mp / kBM;
  const int64_t tiles_per_batch = d * (d + 1) / 2;
  if (tiles_per_batch * batch > INT32_MAX) return MUON_POLAR_ERR_INVALID_ARGUMENT;
  CUtensorMap ta;
  rc = encode_3d(&ta, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, gram, mp, mp, batch,
                 mp, mp * mp, kBK, kBM);
  if (rc != MUON_POLAR_OK) return rc;
  EpiParams p = {};
  p.out = poly;
  p.aux = gram;
  p.out_batch_stride = mp * mp;
  p.aux_batch_stride = mp * mp;
  p.out_ld = static_cast<int32_t>(mp);
  p.aux_ld = static_cast<int32_t>(mp);
  p.rows = static_cast<int32_t>(mp);
  p.cols = static_cast<int32_t>(mp);
  p.tiles_m = static_cast<int32_t>(d);
  p.tiles_n = static_cast<int32_t>(d);
  p.tiles_per_batch = static_cast<int32_t>(tiles_per_batch);
  p.total_tiles = static_cast<int32_t>(tiles_per_batch * batch);
  p.k_blocks = static_cast<int32_t>(mp / kBK);
  p.coef_b = b;
  p.coef_c = c;
  return launch_gemm<128, kPoly>(st, 2, ta, ta, p, stream);
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

int apply_bn_override() {
  static int value = [] {
    const char* s = std::getenv("MUON_POLAR_APPLY_BN");
    if (s == nullptr) return 0;
    const int v = std::atoi(s);
    return (v == 128 || v == 256) ? v : 0;
  }();
  return value;
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
  const int64_t mp = padded_rows(m);
  const int64_t tiles_m = mp / kBM;
  // Tile width: fewest rounds of BN-column work over the SMs.
  const int64_t t128 = tiles_m * ((n + 127) / 128) * batch;
  const int64_t t256 = tiles_m * ((n + 255) / 256) * batch;
  const int64_t cost128 = (t128 + st->sms - 1) / st->sms * 128;
  const int64_t cost256 = (t256 + st->sms - 1) / st->sms * 256;
  int bn = (n > 128 && cost256 <= cost128) ? 256 : 128;
  if (apply_bn_override() != 0) bn = apply_bn_override();
  const int64_t tiles_n = (n + bn - 1) / bn;
  if (tiles_m * tiles_n * batch > INT32_MAX) return MUON_POLAR_ERR_INVALID_ARGUMENT;
  CUtensorMap tp, tx;
  rc = encode_3d(&tp, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, poly, mp, mp, batch,
                 mp, mp * mp, kBK, kBM);
  if (rc != MUON_POLAR_OK) return rc;
  // X as the B operand: rows are K, the 64-column box is the MN extent.
  rc = encode_3d(&tx, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, x, n, m, batch, ldx,
                 m * ldx, 64, kBK);
  if (rc != MUON_POLAR_OK) return rc;
  EpiParams p = {};
  p.out = y;
  p.aux = x;
  p.out_batch_stride = m * ldy;
  p.aux_batch_stride = m * ldx;
  p.out_ld = static_cast<int32_t>(ldy);
  p.aux_ld = static_cast<int32_t>(ldx);
  p.rows = static_cast<int32_t>(m);
  p.cols = static_cast<int32_t>(n);
  p.tiles_m = static_cast<int32_t>(tiles_m);
  p.tiles_n = static_cast<int32_t>(tiles_n);
  p.tiles_per_batch = static_cast<int32_t>(tiles_m * tiles_n);
  p.total_tiles = static_cast<int32_t>(tiles_m * tiles_n * batch);
  // P's columns >= m are zero and X's rows >= m read as zero: stop at m.
  p.k_blocks = static_cast<int32_t>((m + kBK - 1) / kBK);
  p.alpha = round_to_bf16(a);
  if (bn == 256) return launch_gemm<256, kApply>(st, 3, tp, tx, p, stream);
  return launch_gemm<128, kApply>(st, 4, tp, tx, p, stream);
}

}  // namespace
}  // namespace muon_sm100

using namespace muon_sm100;

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
                          int64_t n, int64_t ldx, void* stream) {
  return gram_impl<kGramBf16>(x, gram, batch, m, n, ldx,
                              static_cast<cudaStream_t>(stream));
}

int muon_polar_gram_f32_sm100(const void* x, void* gram_f32, int64_t batch,
                              int64_t m, int64_t n, int64_t ldx, void* stream) {
  return gram_impl<kGramF32>(x, gram_f32, batch, m, n, ldx,
                             static_cast<cudaStream_t>(stream));
}

int muon_polar_poly_sm100(const void* gram, void* poly, int64_t batch,
                          int64_t mp, float b, float c, void* stream) {
  return poly_impl(gram, poly, batch, mp, b, c,
                   static_cast<cudaStream_t>(stream));
}

int muon_polar_apply_sm100(const void* poly, const void* x, void* y,
                           int64_t batch, int64_t m, int64_t n, int64_t ldx,
                           int64_t ldy, float a, void* stream) {
  return apply_impl(poly, x, y, batch, m, n, ldx, ldy, a,
                    static_cast<cudaStream_t>(stream));
}

int muon_polar_step_sm100(const void* x, void* y, void* workspace,
                          size_t workspace_bytes, int64_t batch, int64_t m,
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
  rc = gram_impl<kGramBf16>(x, gram, batch, m, n, ldx, s);
  if (rc != MUON_POLAR_OK) return rc;
  rc = poly_impl(gram, poly, batch, mp, b, c, s);
  if (rc != MUON_POLAR_OK) return rc;
  return apply_impl(poly, x, y, batch, m, n, ldx, ldy, a, s);
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

uint64_t muon_polar_launch_count(void) {
  return g_launch_count.load(std::memory_order_relaxed);
}

}  // extern "C"
