// polar_step_op.cpp -- PyTorch operator muon_ascend950::polar_step on CUDA.
//
// Host side of the drop-in boundary: the same schema, checks, error texts,
// padding/crop contract and debug-sync switch as the reference binding
// (csrc/muon_polar_step_binding.cpp:613-685), dispatching to the sm_100a
// C ABI (include/muon_polar_sm100.h) instead of three AscendC launchers.
//
// Differences from the reference binding, none visible in results:
//   * rows are never padded: the kernels read rows >= M as zeros through
//     the TMA bounds check and mask their stores, so A/P get align(M,256)
//     rows (the CTA-pair tile height) without a padded copy of X;
//   * columns are padded (to a multiple of 16, zero filled) only when N is
//     not a multiple of 8 or the data pointer is not 16-byte aligned -- the
//     TMA row-stride rule -- instead of always to max(align16(N), rows);
//   * tiling is derived from sizes inside the library, so there is no
//     tiling cache to key on stream/shape/coefficients (binding.cpp:103-611);
//     what is cached per (device, stream) -- the role of the reference's
//     LaunchState maps -- is the split-K scratch buffer, whose arrival
//     counters must be zero before a launch and are left zero by it.
#include <ATen/ATen.h>
#include <c10/core/DeviceGuard.h>
#include <c10/cuda/CUDAFunctions.h>
#include <c10/cuda/CUDAGuard.h>
#include <c10/cuda/CUDAStream.h>
#include <torch/library.h>

#include <cstdint>
#include <cstdlib>
#include <mutex>
#include <unordered_map>
#include <vector>

#include "muon_polar_sm100.h"

namespace {

int64_t AlignUp(int64_t value, int64_t alignment) {
  return (value + alignment - 1) / alignment * alignment;
}

bool DebugSyncEnabled() {
  // Read on every call, as the reference does (binding.cpp:93-101).
  return std::getenv("MUON_POLAR_DEBUG_SYNC") != nullptr;
}

void CheckStatus(int rc, const char* stage) {
  TORCH_CHECK(rc == MUON_POLAR_OK, "muon_polar_step: stage ", stage,
              " failed, status=", rc, ", detail=", muon_polar_status_string(rc));
}

// Synchronises and surfaces asynchronous faults and watchdog trips per stage.
void DebugSync(int device, const char* stage) {
  uint32_t flags = 0;
  const int rc = muon_polar_read_device_status(device, &flags, /*clear=*/1);
  TORCH_CHECK(rc == MUON_POLAR_OK, "muon_polar_step: stage ", stage,
              " failed, status=", rc, ", detail=", muon_polar_status_string(rc));
  TORCH_CHECK(flags == 0, "muon_polar_step: stage ", stage,
              " gave up on a bounded wait, watchdog=", flags);
}

// Split-K scratch per (device, stream), zero-initialised once.  Buffers are
// never freed while the process lives (a CUDA graph captured earlier may
// still point at one); a larger problem allocates a larger buffer.
struct ScratchKey {
  int device;
  uintptr_t stream;
  bool operator==(const ScratchKey& o) const {
    return device == o.device && stream == o.stream;
  }
};
struct ScratchKeyHash {
  size_t operator()(const ScratchKey& k) const {
    return std::hash<uintptr_t>()(k.stream) * 31u + static_cast<size_t>(k.device);
  }
};
std::mutex gScratchMutex;
std::unordered_map<ScratchKey, at::Tensor, ScratchKeyHash> gScratch;
std::vector<at::Tensor> gRetiredScratch;

// Returns (pointer, bytes) of a zeroed scratch buffer of at least `bytes`,
// or (nullptr, 0) -- split-K off -- when none is cached and the stream is
// being captured into a CUDA graph (no allocation may happen then).
std::pair<void*, size_t> GetScratch(const at::Tensor& like, int device,
                                    cudaStream_t stream, size_t bytes) {
  if (bytes == 0) return {nullptr, 0};
  std::lock_guard<std::mutex> lock(gScratchMutex);
  const ScratchKey key{device, reinterpret_cast<uintptr_t>(stream)};
  auto it = gScratch.find(key);
  if (it != gScratch.end() && static_cast<size_t>(it->second.numel()) >= bytes)
    return {it->second.data_ptr(), static_cast<size_t>(it->second.numel())};
  cudaStreamCaptureStatus capture = cudaStreamCaptureStatusNone;
  if (cudaStreamIsCapturing(stream, &capture) != cudaSuccess ||
      capture != cudaStreamCaptureStatusNone)
    return {nullptr, 0};
  at::Tensor fresh = at::empty({static_cast<int64_t>(bytes)}, like.options().dtype(at::kByte));
  CheckStatus(muon_polar_scratch_init(fresh.data_ptr(), bytes, stream), "scratch_init");
  if (it != gScratch.end()) {
    gRetiredScratch.push_back(it->second);
    it->second = fresh;
  } else {
    gScratch.emplace(key, fresh);
  }
  return {fresh.data_ptr(), bytes};
}

// `transposed` = false: the reference operator (M <= N).  true: the step of
// X^T returned in X's layout, for tall X (M > N), without the two transposed
// copies the reference's wrapper makes (ops.py:27-32).
at::Tensor RunPolarStep(const at::Tensor& x, double a, double b, double c, bool transposed) {
  TORCH_CHECK(x.defined(), "muon_polar_step: x must be defined");
  TORCH_CHECK(x.device().is_cuda(), "muon_polar_step: x must be a CUDA tensor");
  TORCH_CHECK(x.scalar_type() == at::kBFloat16,
              "muon_polar_step: only bfloat16 is supported");
  TORCH_CHECK(x.dim() == 3, "muon_polar_step: x must have shape [batch, M, N]");
  TORCH_CHECK(x.size(0) > 0 && x.size(1) > 0 && x.size(2) > 0,
              "muon_polar_step: all dimensions must be positive");
  if (!transposed)
    TORCH_CHECK(x.size(1) <= x.size(2),
                "muon_polar_step: expects M <= N; transpose policy stays outside "
                "this op");
  const c10::cuda::CUDAGuard deviceGuard(x.device());
  at::Tensor input = x.contiguous();
  const int64_t batch = input.size(0);
  const int64_t rows = input.size(1);
  const int64_t cols = input.size(2);
  const bool aligned =
      (cols % 8) == 0 &&
      (reinterpret_cast<uintptr_t>(input.data_ptr()) % 16) == 0;
  int64_t ld = cols;
  if (!aligned) {
    ld = AlignUp(cols, 16);
    // one kernel: a fresh (aligned) buffer with zero-filled pad columns
    input = ld == cols ? input.clone() : at::constant_pad_nd(input, {0, ld - cols}, 0);
  }
  const auto stream = c10::cuda::getCurrentCUDAStream(x.device().index());
  void* raw_stream = static_cast<void*>(stream.stream());
  // The Gram is [batch][g][g]: g = M, or N for the transposed step.
  const int64_t g = transposed ? cols : rows;
  const int64_t depth = transposed ? rows : cols;
  const size_t wsBytes = muon_polar_workspace_bytes(batch, g);
  at::Tensor workspace =
      at::empty({static_cast<int64_t>(wsBytes)}, input.options().dtype(at::kByte));
  at::Tensor out = at::empty({batch, rows, ld}, input.options());
  const float fa = static_cast<float>(a);
  const float fb = static_cast<float>(b);
  const float fc = static_cast<float>(c);
  const auto scratch = GetScratch(input, x.device().index(), stream.stream(),
                                  muon_polar_scratch_bytes(batch, g, depth));

  if (!DebugSyncEnabled()) {
    if (transposed)
      CheckStatus(muon_polar_step_t_sm100(input.data_ptr(), out.data_ptr(),
                                          workspace.data_ptr(), wsBytes, scratch.first,
                                          scratch.second, batch, rows, cols, ld, ld,
                                          fa, fb, fc, raw_stream),
                  "polar_step_t_sm100");
    else
      CheckStatus(muon_polar_step_sm100(input.data_ptr(), out.data_ptr(),
                                        workspace.data_ptr(), wsBytes, scratch.first,
                                        scratch.second, batch, rows, cols, ld, ld,
                                        fa, fb, fc, raw_stream),
                  "polar_step_sm100");
  } else {
    const int device = x.device().index();
    const int64_t mp = muon_polar_padded_rows(g);
    uint8_t* ws = static_cast<uint8_t*>(workspace.data_ptr());
    void* gram = ws;
    void* poly = ws + static_cast<size_t>(batch * mp * mp * 2);
    if (transposed)
      CheckStatus(muon_polar_gram_t_sm100(input.data_ptr(), gram, batch, rows, cols, ld,
                                          scratch.first, scratch.second, raw_stream),
                  "gram_t_sm100");
    else
      CheckStatus(muon_polar_gram_sm100(input.data_ptr(), gram, batch, rows,
                                        cols, ld, scratch.first, scratch.second,
                                        raw_stream),
                  "gram_sm100");
    DebugSync(device, "gram_sm100");
    CheckStatus(muon_polar_poly_sm100(gram, poly, batch, mp, fb, fc,
                                      scratch.first, scratch.second, raw_stream),
                "poly_sm100");
    DebugSync(device, "poly_sm100");
    if (transposed)
      CheckStatus(muon_polar_apply_t_sm100(poly, input.data_ptr(), out.data_ptr(), batch,
                                           rows, cols, ld, ld, fa, raw_stream),
                  "apply_t_sm100");
    else
      CheckStatus(muon_polar_apply_sm100(poly, input.data_ptr(), out.data_ptr(),
                                         batch, rows, cols, ld, ld, fa,
                                         raw_stream),
                  "apply_sm100");
    DebugSync(device, "apply_sm100");
  }
  if (aligned) return out;
  return out.narrow(2, 0, cols).contiguous();
}

at::Tensor MuonPolarStepCuda(const at::Tensor& x, double a, double b, double c) {
  return RunPolarStep(x, a, b, c, /*transposed=*/false);
}

at::Tensor MuonPolarStepTCuda(const at::Tensor& x, double a, double b, double c) {
  return RunPolarStep(x, a, b, c, /*transposed=*/true);
}

std::vector<float> CoefficientRows(at::ArrayRef<double> coefficients, const char* who) {
  TORCH_CHECK(!coefficients.empty() && coefficients.size() % 3 == 0, who,
              ": coefficients must hold (a, b, c) rows, got ", coefficients.size(), " values");
  return std::vector<float>(coefficients.begin(), coefficients.end());
}

// Several Polar Express steps (one C-ABI call), optionally after the
// normalisation x / (||x||_F * 1.01 + 1e-6).  x: [B, M, N] fp32 or bf16.
at::Tensor PolarExpressCuda(const at::Tensor& x, at::ArrayRef<double> coefficients,
                            bool normalize) {
  TORCH_CHECK(x.defined() && x.device().is_cuda(), "polar_express: x must be a CUDA tensor");
  TORCH_CHECK(x.dim() == 3, "polar_express: x must have shape [batch, M, N]");
  TORCH_CHECK(x.size(0) > 0 && x.size(1) > 0 && x.size(2) > 0,
              "polar_express: all dimensions must be positive");
  TORCH_CHECK(x.scalar_type() == at::kBFloat16 || (normalize && x.scalar_type() == at::kFloat),
              "polar_express: x must be bfloat16 (or float32 with normalize=True)");
  const std::vector<float> coeffs = CoefficientRows(coefficients, "polar_express");
  const c10::cuda::CUDAGuard deviceGuard(x.device());
  at::Tensor input = x.contiguous();
  const int64_t batch = input.size(0), rows = input.size(1), cols = input.size(2);
  int64_t ldx = cols;
  if (!normalize && ((cols % 8) != 0 ||
                     (reinterpret_cast<uintptr_t>(input.data_ptr()) % 16) != 0)) {
    // read in place by the first step: the TMA row-stride rule needs a copy
    ldx = AlignUp(cols, 16);
    input = ldx == cols ? input.clone() : at::constant_pad_nd(input, {0, ldx - cols}, 0);
  } else if ((reinterpret_cast<uintptr_t>(input.data_ptr()) % 16) != 0) {
    input = input.clone();
  }
  const int64_t ld = (cols % 8) == 0 ? cols : AlignUp(cols, 16);
  const auto stream = c10::cuda::getCurrentCUDAStream(x.device().index());
  const size_t wsBytes = muon_polar_express_workspace_bytes(batch, rows, cols);
  at::Tensor workspace =
      at::empty({static_cast<int64_t>(wsBytes)}, input.options().dtype(at::kByte));
  at::Tensor out = at::empty({batch, rows, ld}, input.options().dtype(at::kBFloat16));
  const int64_t g = rows < cols ? rows : cols;
  const int64_t depth = rows < cols ? cols : rows;
  const auto scratch = GetScratch(input, x.device().index(), stream.stream(),
                                  muon_polar_scratch_bytes(batch, g, depth));
  CheckStatus(muon_polar_express_sm100(input.data_ptr(), input.scalar_type() == at::kFloat ? 0 : 1,
                                       ldx, out.data_ptr(), ld, workspace.data_ptr(), wsBytes,
                                       scratch.first, scratch.second, batch, rows, cols,
                                       coeffs.data(), static_cast<int>(coeffs.size() / 3),
                                       normalize ? 1 : 0, stream.stream()),
              "polar_express_sm100");
  if (ld == cols) return out;
  return out.narrow(2, 0, cols).contiguous();
}

// One Muon update, in place on param and momentum_buffer.
void MuonUpdateCuda(const at::Tensor& param, const at::Tensor& grad,
                    const at::Tensor& momentum_buffer, double lr, double momentum,
                    bool nesterov, double weight_decay, double scale,
                    at::ArrayRef<double> coefficients) {
  TORCH_CHECK(param.device().is_cuda() && grad.device() == param.device() &&
                  momentum_buffer.device() == param.device(),
              "muon_update: tensors must be on one CUDA device");
  TORCH_CHECK(param.dim() == 2 || param.dim() == 3,
              "muon_update: param must have shape [M, N] or [batch, M, N]");
  TORCH_CHECK(grad.sizes() == param.sizes() && momentum_buffer.sizes() == param.sizes(),
              "muon_update: grad and momentum_buffer must have param's shape");
  TORCH_CHECK(param.scalar_type() == at::kFloat || param.scalar_type() == at::kBFloat16,
              "muon_update: param must be float32 or bfloat16");
  TORCH_CHECK(grad.scalar_type() == param.scalar_type() &&
                  momentum_buffer.scalar_type() == param.scalar_type(),
              "muon_update: grad and momentum_buffer must have param's dtype");
  TORCH_CHECK(param.is_contiguous() && grad.is_contiguous() && momentum_buffer.is_contiguous(),
              "muon_update: tensors must be contiguous");
  TORCH_CHECK(param.numel() > 0, "muon_update: empty parameter");
  const std::vector<float> coeffs = CoefficientRows(coefficients, "muon_update");
  const c10::cuda::CUDAGuard deviceGuard(param.device());
  const int64_t batch = param.dim() == 3 ? param.size(0) : 1;
  const int64_t rows = param.size(-2), cols = param.size(-1);
  const auto stream = c10::cuda::getCurrentCUDAStream(param.device().index());
  const size_t wsBytes = muon_polar_express_workspace_bytes(batch, rows, cols);
  at::Tensor workspace =
      at::empty({static_cast<int64_t>(wsBytes)}, param.options().dtype(at::kByte));
  const int64_t g = rows < cols ? rows : cols;
  const int64_t depth = rows < cols ? cols : rows;
  const auto scratch = GetScratch(param, param.device().index(), stream.stream(),
                                  muon_polar_scratch_bytes(batch, g, depth));
  CheckStatus(muon_polar_update_sm100(param.data_ptr(), grad.data_ptr(), momentum_buffer.data_ptr(),
                                      param.scalar_type() == at::kFloat ? 0 : 1,
                                      workspace.data_ptr(), wsBytes, scratch.first, scratch.second,
                                      batch, rows, cols, static_cast<float>(lr),
                                      static_cast<float>(momentum), nesterov ? 1 : 0,
                                      static_cast<float>(weight_decay), static_cast<float>(scale),
                                      coeffs.data(), static_cast<int>(coeffs.size() / 3),
                                      stream.stream()),
              "muon_update_sm100");
}

}  // namespace

TORCH_LIBRARY(muon_ascend950, m) {
  m.def("polar_step(Tensor x, float a, float b, float c) -> Tensor");
  // Extension (no counterpart in the reference): the step of x^T for tall
  // x, returned in x's layout -- polar_step(x.mT).mT without the copies.
  m.def("polar_step_t(Tensor x, float a, float b, float c) -> Tensor");
  // Extensions: the caller side of the step on the device (several steps
  // with normalisation; a whole Muon update of one parameter).
  m.def("polar_express(Tensor x, float[] coefficients, bool normalize=True) -> Tensor");
  m.def("muon_update_(Tensor(a!) param, Tensor grad, Tensor(b!) momentum_buffer, float lr, "
        "float momentum, bool nesterov, float weight_decay, float scale, "
        "float[] coefficients) -> ()");
}

TORCH_LIBRARY_IMPL(muon_ascend950, CUDA, m) {
  m.impl("polar_step", &MuonPolarStepCuda);
  m.impl("polar_step_t", &MuonPolarStepTCuda);
  m.impl("polar_express", &PolarExpressCuda);
  m.impl("muon_update_", &MuonUpdateCuda);
}
