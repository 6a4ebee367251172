// muon_polar_update_sm100.cu -- the caller side of the Polar Express step, on the
// device: a whole Muon update (momentum, Frobenius normalisation, several
// Polar Express steps, scaled parameter update) and a multi-step Polar
// Express entry, both without a host round trip.
//
// The reference leaves all of this to its caller ("the five-step loop, input
// normalisation and the optimizer's parameter update are done by the
// caller", README.md:5; examples/five_steps.py:18-21 normalises with
// x / (||x||_F * 1.01 + 1e-6) and loops over the five coefficient rows).
// Here the loop runs inside one C-ABI call: the elementwise stages are
// HBM-bound kernels chained with programmatic dependent launch to the
// tensor-core kernels of muon_polar_sm100.cu.
//
// Elementwise kernels (HBM-bound; grid = blocks_per_matrix x batch, about
// eight 256-thread blocks per SM; 16-byte vector accesses on rows whose
// length is a multiple of 8):
//   momentum_sumsq_kernel  buf <- lerp(buf, g, 1 - mu); v = nesterov ?
//                          lerp(g, buf, mu) : buf; per-block sum of v^2
//   normalize_kernel       s = sqrt(sum v^2) * 1.01 + 1e-6 (partials summed
//                          in a fixed order: deterministic); X = bf16(v / s)
//   update_kernel          p <- round(p * (1 - lr*wd) - lr*scale*Y)
// Arithmetic is fp32 with one rounding to the storage type per output.
#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include <atomic>

#include "muon_polar_sm100.h"
#include "sm100_ptx.cuh"

namespace muon_update {
namespace {

using muon_sm100::grid_dependency_wait;
using muon_sm100::grid_launch_dependents;

constexpr int kThreads = 256;
constexpr int kMaxBlocksPerMatrix = 1184;  // 8 blocks per SM on 148 SMs

// ------------------------------------------------------------ element I/O
__device__ __forceinline__ float load1(const float* p) { return *p; }
__device__ __forceinline__ float load1(const __nv_bfloat16* p) { return __bfloat162float(*p); }
__device__ __forceinline__ void store1(float* p, float v) { *p = v; }
__device__ __forceinline__ void store1(__nv_bfloat16* p, float v) { *p = __float2bfloat16_rn(v); }
// v rounded to the storage type T, as an fp32 value.
template <typename T>
__device__ __forceinline__ float rounded(float v) {
  if constexpr (sizeof(T) == 2)
    return __bfloat162float(__float2bfloat16_rn(v));
  else
    return v;
}

// Eight consecutive elements at a 16-byte aligned address.
__device__ __forceinline__ void load8(const float* p, float (&v)[8]) {
  const float4 a = reinterpret_cast<const float4*>(p)[0];
  const float4 b = reinterpret_cast<const float4*>(p)[1];
  v[0] = a.x; v[1] = a.y; v[2] = a.z; v[3] = a.w;
  v[4] = b.x; v[5] = b.y; v[6] = b.z; v[7] = b.w;
}
__device__ __forceinline__ void load8(const __nv_bfloat16* p, float (&v)[8]) {
  const uint4 u = *reinterpret_cast<const uint4*>(p);
  const uint32_t w[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    __nv_bfloat162 h = *reinterpret_cast<const __nv_bfloat162*>(&w[i]);
    const float2 f = __bfloat1622float2(h);
    v[2 * i] = f.x;
    v[2 * i + 1] = f.y;
  }
}
__device__ __forceinline__ void store8(float* p, const float (&v)[8]) {
  reinterpret_cast<float4*>(p)[0] = make_float4(v[0], v[1], v[2], v[3]);
  reinterpret_cast<float4*>(p)[1] = make_float4(v[4], v[5], v[6], v[7]);
}
__device__ __forceinline__ void store8(__nv_bfloat16* p, const float (&v)[8]) {
  uint32_t w[4];
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    __nv_bfloat162 h = __floats2bfloat162_rn(v[2 * i], v[2 * i + 1]);
    w[i] = *reinterpret_cast<uint32_t*>(&h);
  }
  *reinterpret_cast<uint4*>(p) = make_uint4(w[0], w[1], w[2], w[3]);
}

// torch.lerp's formula: a + w (b - a) for |w| < 0.5, else b - (b - a)(1 - w).
__device__ __forceinline__ float lerp(float a, float b, float w) {
  const float d = __fsub_rn(b, a);
  return fabsf(w) < 0.5f ? __fadd_rn(a, __fmul_rn(w, d))
                         : __fsub_rn(b, __fmul_rn(d, __fsub_rn(1.0f, w)));
}

// Rows [r0, r1) of matrix b for block x of `blocks` blocks per matrix.
__device__ __forceinline__ void block_rows(int64_t m, int blocks, int64_t* r0, int64_t* r1) {
  *r0 = static_cast<int64_t>(blockIdx.x) * m / blocks;
  *r1 = static_cast<int64_t>(blockIdx.x + 1) * m / blocks;
}

// Sum over the block in a fixed order (warp shuffles, then warp 0 over the
// warps' sums); the result is valid in thread 0.
__device__ __forceinline__ float block_sum(float v, float* red) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_down_sync(0xffffffffu, v, o);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (lane == 0) red[warp] = v;
  __syncthreads();
  float s = 0.f;
  if (warp == 0) {
    s = lane < kThreads / 32 ? red[lane] : 0.f;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) s += __shfl_down_sync(0xffffffffu, s, o);
  }
  return s;
}

// The update direction v from the gradient and the (already updated and
// stored) momentum buffer, rounded to the storage type as a tensor
// g.lerp(buf, mu) of that type would be.
template <typename T>
__device__ __forceinline__ float direction(float g, float buf, float mu, int nesterov) {
  return nesterov ? rounded<T>(lerp(g, buf, mu)) : buf;
}

// ------------------------------------------------------------ kernels
// With `buf` null: v = g (normalisation of a plain input).  With `buf`:
// buf <- lerp(buf, g, 1 - mu) stored back, v = direction(g, buf).  Writes
// the block's sum of v^2 to partial[b * gridDim.x + blockIdx.x].
template <typename T>
__global__ void __launch_bounds__(kThreads)
    momentum_sumsq_kernel(const T* __restrict__ grad, T* __restrict__ buf,
                          float* __restrict__ partial, int64_t m, int64_t n, int64_t ldg,
                          float mu, int nesterov) {
  __shared__ float red[kThreads / 32];
  grid_dependency_wait();
  grid_launch_dependents();
  const int64_t b = blockIdx.y;
  int64_t r0, r1;
  block_rows(m, gridDim.x, &r0, &r1);
  const bool vec = (n % 8) == 0 && (ldg % 8) == 0;
  float acc = 0.f;
  for (int64_t r = r0; r < r1; ++r) {
    const int64_t base = (b * m + r) * ldg;
    if (vec) {
      for (int64_t c = threadIdx.x * 8; c < n; c += kThreads * 8) {
        float g[8], v[8];
        load8(grad + base + c, g);
        if (buf != nullptr) {
          float u[8];
          load8(buf + base + c, u);
#pragma unroll
          for (int i = 0; i < 8; ++i) u[i] = rounded<T>(lerp(u[i], g[i], 1.0f - mu));
          store8(buf + base + c, u);
#pragma unroll
          for (int i = 0; i < 8; ++i) v[i] = direction<T>(g[i], u[i], mu, nesterov);
        } else {
#pragma unroll
          for (int i = 0; i < 8; ++i) v[i] = g[i];
        }
#pragma unroll
        for (int i = 0; i < 8; ++i) acc = fmaf(v[i], v[i], acc);
      }
    } else {
      for (int64_t c = threadIdx.x; c < n; c += kThreads) {
        const float g = load1(grad + base + c);
        float v = g;
        if (buf != nullptr) {
          const float u = rounded<T>(lerp(load1(buf + base + c), g, 1.0f - mu));
          store1(buf + base + c, u);
          v = direction<T>(g, u, mu, nesterov);
        }
        acc = fmaf(v, v, acc);
      }
    }
  }
  const float s = block_sum(acc, red);
  if (threadIdx.x == 0) partial[b * gridDim.x + blockIdx.x] = s;
}

// x[b] = bf16( v / (||v||_F * 1.01 + 1e-6) ), x with row stride ldx.  Every
// block sums the matrix's partials in the same order, so all blocks use the
// same s.
template <typename T>
__global__ void __launch_bounds__(kThreads)
    normalize_kernel(const T* __restrict__ grad, const T* __restrict__ buf,
                     const float* __restrict__ partial, __nv_bfloat16* __restrict__ x,
                     int64_t m, int64_t n, int64_t ldg, int64_t ldx, float mu, int nesterov) {
  __shared__ float red[kThreads / 32];
  __shared__ float s_shared;
  grid_dependency_wait();
  grid_launch_dependents();
  const int64_t b = blockIdx.y;
  const int blocks = gridDim.x;
  float p = 0.f;
  for (int i = threadIdx.x; i < blocks; i += kThreads) p += partial[b * blocks + i];
  const float total = block_sum(p, red);
  if (threadIdx.x == 0) s_shared = __fadd_rn(__fmul_rn(sqrtf(total), 1.01f), 1e-6f);
  __syncthreads();
  const float s = s_shared;
  int64_t r0, r1;
  block_rows(m, blocks, &r0, &r1);
  const bool vec = (n % 8) == 0 && (ldg % 8) == 0 && (ldx % 8) == 0;
  for (int64_t r = r0; r < r1; ++r) {
    const int64_t base = (b * m + r) * ldg;
    __nv_bfloat16* xr = x + (b * m + r) * ldx;
    if (vec) {
      for (int64_t c = threadIdx.x * 8; c < n; c += kThreads * 8) {
        float g[8], v[8];
        load8(grad + base + c, g);
        if (buf != nullptr) {
          float u[8];
          load8(buf + base + c, u);
#pragma unroll
          for (int i = 0; i < 8; ++i) v[i] = direction<T>(g[i], u[i], mu, nesterov);
        } else {
#pragma unroll
          for (int i = 0; i < 8; ++i) v[i] = g[i];
        }
#pragma unroll
        for (int i = 0; i < 8; ++i) v[i] = __fdiv_rn(v[i], s);
        store8(xr + c, v);
      }
    } else {
      for (int64_t c = threadIdx.x; c < n; c += kThreads) {
        const float g = load1(grad + base + c);
        const float v = buf != nullptr ? direction<T>(g, load1(buf + base + c), mu, nesterov) : g;
        xr[c] = __float2bfloat16_rn(__fdiv_rn(v, s));
      }
    }
  }
}

// p <- round( p * (1 - lr*wd) - (lr*scale) * y ), y bf16 with row stride ldy.
template <typename T>
__global__ void __launch_bounds__(kThreads)
    update_kernel(T* __restrict__ param, const __nv_bfloat16* __restrict__ y, int64_t m,
                  int64_t n, int64_t ldy, float decay, float step) {
  grid_dependency_wait();
  grid_launch_dependents();
  const int64_t b = blockIdx.y;
  int64_t r0, r1;
  block_rows(m, gridDim.x, &r0, &r1);
  const bool vec = (n % 8) == 0 && (ldy % 8) == 0;
  for (int64_t r = r0; r < r1; ++r) {
    T* pr = param + (b * m + r) * n;
    const __nv_bfloat16* yr = y + (b * m + r) * ldy;
    if (vec) {
      for (int64_t c = threadIdx.x * 8; c < n; c += kThreads * 8) {
        float p[8], u[8];
        load8(pr + c, p);
        load8(yr + c, u);
#pragma unroll
        for (int i = 0; i < 8; ++i) p[i] = __fsub_rn(__fmul_rn(p[i], decay), __fmul_rn(step, u[i]));
        store8(pr + c, p);
      }
    } else {
      for (int64_t c = threadIdx.x; c < n; c += kThreads) {
        const float p = load1(pr + c);
        store1(pr + c, __fsub_rn(__fmul_rn(p, decay), __fmul_rn(step, __bfloat162float(yr[c]))));
      }
    }
  }
}

// ------------------------------------------------------------ host side
std::atomic<uint64_t>* launch_counter() {
  static std::atomic<uint64_t> count{0};
  return &count;
}

int sm_count(int* sms) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e == cudaSuccess) e = cudaDeviceGetAttribute(sms, cudaDevAttrMultiProcessorCount, dev);
  return e == cudaSuccess ? MUON_POLAR_OK : static_cast<int>(e);
}

int blocks_per_matrix(int64_t batch, int64_t m, int sms) {
  int64_t want = (static_cast<int64_t>(sms) * 8 + batch - 1) / batch;
  if (want > m) want = m;
  if (want > kMaxBlocksPerMatrix) want = kMaxBlocksPerMatrix;
  return want < 1 ? 1 : static_cast<int>(want);
}

template <typename Kernel, typename... Args>
int launch(Kernel kernel, int blocks, int64_t batch, cudaStream_t stream, Args... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(static_cast<unsigned>(blocks), static_cast<unsigned>(batch), 1);
  cfg.blockDim = dim3(kThreads, 1, 1);
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  cudaError_t e = cudaLaunchKernelEx(&cfg, kernel, args...);
  if (e != cudaSuccess) return static_cast<int>(e);
  launch_counter()->fetch_add(1, std::memory_order_relaxed);
  return MUON_POLAR_OK;
}

size_t align256(size_t v) { return (v + 255) / 256 * 256; }

// Row stride of the bf16 iterate buffers: n when the TMA stride rule allows
// it, else n rounded up to 16.
int64_t iterate_ld(int64_t n) { return (n % 8) == 0 ? n : (n + 15) / 16 * 16; }

// Workspace plan of muon_polar_express_sm100 / muon_polar_update_sm100:
// [ polar workspace (A, P) | iterate 0 | iterate 1 | partial sums ].
struct ExpressPlan {
  size_t polar_bytes, iter_bytes, partial_bytes, total;
};

ExpressPlan express_plan(int64_t batch, int64_t m, int64_t n) {
  ExpressPlan pl;
  const int64_t g = m > n ? n : m;  // rows of the Gram (tall X: its columns)
  pl.polar_bytes = align256(muon_polar_workspace_bytes(batch, g));
  pl.iter_bytes = align256(static_cast<size_t>(batch * m * iterate_ld(n) * 2));
  pl.partial_bytes = align256(static_cast<size_t>(batch * kMaxBlocksPerMatrix) * sizeof(float));
  pl.total = pl.polar_bytes + 2 * pl.iter_bytes + pl.partial_bytes;
  return pl;
}

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

// `steps` Polar Express steps from the bf16 iterate `src` (row stride
// ld_src) into `dst` through the two iterate buffers (muon_polar_steps_sm100:
// one fused launch for small matrices, else three kernels a step; tall X
// runs the transposed step, whose Gram is N x N).  When src is iterate 0
// the first step writes iterate 1.
int run_steps(const void* src, int64_t ld_src, void* dst, int64_t ld_dst, uint8_t* ws,
              const ExpressPlan& pl, void* scratch, size_t scratch_bytes, int64_t batch,
              int64_t m, int64_t n, const float* coefficients, int steps, cudaStream_t stream) {
  void* iter[2] = {ws + pl.polar_bytes, ws + pl.polar_bytes + pl.iter_bytes};
  const int first = (src == iter[0]) ? 1 : 0;
  return muon_polar_steps_sm100(src, dst, iter[first], iter[first ^ 1], iterate_ld(n), ws,
                                pl.polar_bytes, scratch, scratch_bytes, batch, m, n, ld_src,
                                ld_dst, coefficients, steps, stream);
}

// input (and momentum) rows of stride ldg -> normalised bf16 x (stride ldx).
template <typename T>
int normalize_into(const T* input, T* momentum, int64_t ldg, float mu, int nesterov, void* x,
                   int64_t ldx, float* partial, int64_t batch, int64_t m, int64_t n, int sms,
                   cudaStream_t stream) {
  const int blocks = blocks_per_matrix(batch, m, sms);
  int rc = launch(momentum_sumsq_kernel<T>, blocks, batch, stream, input, momentum, partial, m, n,
                  ldg, mu, nesterov);
  if (rc != MUON_POLAR_OK) return rc;
  return launch(normalize_kernel<T>, blocks, batch, stream, input,
                static_cast<const T*>(momentum), static_cast<const float*>(partial),
                static_cast<__nv_bfloat16*>(x), m, n, ldg, ldx, mu, nesterov);
}

bool valid_sizes(int64_t batch, int64_t m, int64_t n) {
  return batch > 0 && m > 0 && n > 0 && batch <= 65535 && m <= (1 << 24) && n <= (1 << 24);
}

}  // namespace
}  // namespace muon_update

using namespace muon_update;

extern "C" {

size_t muon_polar_express_workspace_bytes(int64_t batch, int64_t m, int64_t n) {
  if (!valid_sizes(batch, m, n)) return 0;
  return express_plan(batch, m, n).total;
}

int muon_polar_express_sm100(const void* x, int x_dtype, int64_t ldx, void* y, int64_t ldy,
                             void* workspace, size_t workspace_bytes, void* scratch,
                             size_t scratch_bytes, int64_t batch, int64_t m, int64_t n,
                             const float* coefficients, int steps, int normalize, void* stream) {
  if (x == nullptr || y == nullptr || y == x || coefficients == nullptr || steps < 1 ||
      !valid_sizes(batch, m, n) || ldx < n || ldy < n || (x_dtype != 0 && x_dtype != 1))
    return MUON_POLAR_ERR_INVALID_ARGUMENT;
  if (!normalize && x_dtype != 1) return MUON_POLAR_ERR_INVALID_ARGUMENT;
  if (!aligned16(x) || !aligned16(y) || (ldy % 8) != 0) return MUON_POLAR_ERR_ALIGNMENT;
  // without normalisation the first step reads x in place (TMA stride rule)
  if (!normalize && (ldx % 8) != 0) return MUON_POLAR_ERR_ALIGNMENT;
  const ExpressPlan pl = express_plan(batch, m, n);
  if (workspace == nullptr || !aligned16(workspace) || workspace_bytes < pl.total)
    return MUON_POLAR_ERR_WORKSPACE;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  uint8_t* ws = static_cast<uint8_t*>(workspace);
  void* iter0 = ws + pl.polar_bytes;
  float* partial = reinterpret_cast<float*>(ws + pl.polar_bytes + 2 * pl.iter_bytes);
  const void* src = x;
  int64_t ld_src = ldx;
  if (normalize) {
    int sms = 0;
    int rc = sm_count(&sms);
    if (rc != MUON_POLAR_OK) return rc;
    rc = x_dtype == 0
             ? normalize_into(static_cast<const float*>(x), static_cast<float*>(nullptr), ldx,
                              0.f, 0, iter0, iterate_ld(n), partial, batch, m, n, sms, s)
             : normalize_into(static_cast<const __nv_bfloat16*>(x),
                              static_cast<__nv_bfloat16*>(nullptr), ldx, 0.f, 0, iter0,
                              iterate_ld(n), partial, batch, m, n, sms, s);
    if (rc != MUON_POLAR_OK) return rc;
    src = iter0;
    ld_src = iterate_ld(n);
  }
  return run_steps(src, ld_src, y, ldy, ws, pl, scratch, scratch_bytes, batch, m, n, coefficients,
                   steps, s);
}

int muon_polar_update_sm100(void* param, const void* grad, void* momentum, int dtype, void* workspace,
                      size_t workspace_bytes, void* scratch, size_t scratch_bytes, int64_t batch,
                      int64_t m, int64_t n, float lr, float momentum_coef, int nesterov,
                      float weight_decay, float scale, const float* coefficients, int steps,
                      void* stream) {
  if (param == nullptr || grad == nullptr || momentum == nullptr || coefficients == nullptr ||
      steps < 1 || !valid_sizes(batch, m, n) || (dtype != 0 && dtype != 1) || param == grad ||
      param == momentum || grad == momentum)
    return MUON_POLAR_ERR_INVALID_ARGUMENT;
  if (!aligned16(param) || !aligned16(grad) || !aligned16(momentum)) return MUON_POLAR_ERR_ALIGNMENT;
  const ExpressPlan pl = express_plan(batch, m, n);
  if (workspace == nullptr || !aligned16(workspace) || workspace_bytes < pl.total)
    return MUON_POLAR_ERR_WORKSPACE;
  int sms = 0;
  int rc = sm_count(&sms);
  if (rc != MUON_POLAR_OK) return rc;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  uint8_t* ws = static_cast<uint8_t*>(workspace);
  void* iter[2] = {ws + pl.polar_bytes, ws + pl.polar_bytes + pl.iter_bytes};
  float* partial = reinterpret_cast<float*>(ws + pl.polar_bytes + 2 * pl.iter_bytes);
  const int64_t ld = iterate_ld(n);
  rc = dtype == 0 ? normalize_into(static_cast<const float*>(grad), static_cast<float*>(momentum),
                                   n, momentum_coef, nesterov, iter[0], ld, partial, batch, m, n,
                                   sms, s)
                  : normalize_into(static_cast<const __nv_bfloat16*>(grad),
                                   static_cast<__nv_bfloat16*>(momentum), n, momentum_coef,
                                   nesterov, iter[0], ld, partial, batch, m, n, sms, s);
  if (rc != MUON_POLAR_OK) return rc;
  // The last step writes the other iterate buffer (odd step counts) or the
  // first one: never the step's own input.
  void* out = (steps % 2 == 1) ? iter[1] : iter[0];
  rc = run_steps(iter[0], ld, out, ld, ws, pl, scratch, scratch_bytes, batch, m, n, coefficients,
                 steps, s);
  if (rc != MUON_POLAR_OK) return rc;
  const int blocks = blocks_per_matrix(batch, m, sms);
  const float decay = 1.0f - lr * weight_decay;
  const float step = lr * scale;
  const __nv_bfloat16* yb = static_cast<const __nv_bfloat16*>(out);
  return dtype == 0 ? launch(update_kernel<float>, blocks, batch, s, static_cast<float*>(param),
                             yb, m, n, ld, decay, step)
                    : launch(update_kernel<__nv_bfloat16>, blocks, batch, s,
                             static_cast<__nv_bfloat16*>(param), yb, m, n, ld, decay, step);
}

uint64_t muon_polar_update_launch_count(void) {
  return launch_counter()->load(std::memory_order_relaxed);
}

}  // extern "C"
