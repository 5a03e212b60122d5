// Torch operator library `sdc_cutlass` over the sdc_b200 C ABI.
//
// Registers the operator schemas of the reference extension
// (src/cutlass_gemm/csrc/bindings.cpp:45-62) with the same argument checks
// and error messages, so the reference's Python engine and tests can call
// torch.ops.sdc_cutlass.* unchanged. Each op validates, allocates its outputs
// and per-call scratch with the caching allocator on the operand device, and
// enqueues the C ABI on the current CUDA stream (no host synchronisation).
// Extensions beyond the reference schemas are trailing defaulted arguments
// (`layout`) and the extra ops at the end of the registration block.
#include <ATen/ATen.h>
#include <ATen/MemoryOverlap.h>
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>
#include <torch/library.h>

#include <cmath>
#include <limits>
#include <optional>
#include <tuple>

#include "sdc_b200.h"

namespace {

using at::Tensor;
using OptTensor = const std::optional<Tensor>&;
using Out3 = std::tuple<Tensor, Tensor, Tensor>;
using Out5 = std::tuple<Tensor, Tensor, Tensor, Tensor, Tensor>;
using Out6 = std::tuple<Tensor, Tensor, Tensor, Tensor, Tensor, Tensor>;

void check_status(int rc) { TORCH_CHECK(rc == SDC_OK, sdc_last_error()); }

cudaStream_t stream_of(const Tensor& t) { return at::cuda::getCurrentCUDAStream(t.get_device()).stream(); }

int channels_of(int64_t algorithm) {
  // Rejected before any narrowing conversion of the 64-bit schema integer.
  if (algorithm == 0) return 2;
  if (algorithm == 1) return 1;
  TORCH_CHECK(false, "Unknown compiled ABFT algorithm ID");
}

Tensor workspace(const Tensor& like, size_t bytes) {
  return at::empty({static_cast<int64_t>(std::max<size_t>(bytes, 16))}, like.options().dtype(at::kByte));
}

void check_alpha(const Tensor& alpha, const Tensor& a) {
  TORCH_CHECK(alpha.is_cuda() && alpha.device() == a.device() && alpha.layout() == at::kStrided &&
                  alpha.scalar_type() == at::kFloat && alpha.dim() == 0,
              "alpha must be a CUDA FP32 scalar tensor on the operand device");
}

void check_fp8_operands(const Tensor& a, const Tensor& b, const Tensor& alpha) {
  TORCH_CHECK(a.is_cuda() && b.is_cuda() && a.device() == b.device(), "A and B must be on the same CUDA device");
  TORCH_CHECK(a.layout() == at::kStrided && b.layout() == at::kStrided && a.dim() == 2 && b.dim() == 2 &&
                  a.is_contiguous() && b.is_contiguous(),
              "A and B_rows must be contiguous row-major matrices");
  TORCH_CHECK(a.scalar_type() == at::ScalarType::Float8_e4m3fn && b.scalar_type() == at::ScalarType::Float8_e4m3fn,
              "FP8 GEMM requires E4M3FN operands");
  TORCH_CHECK(a.size(1) == b.size(1), "A and B_rows K dimensions must match");
  for (auto d : {a.size(0), b.size(0), a.size(1)}) {
    TORCH_CHECK(d > 0 && d <= std::numeric_limits<int>::max() - 128,
                "Matrix dimensions must be positive and allow int32 tile padding");
  }
  check_alpha(alpha, a);
}

void check_nvfp4_operands(const Tensor& a, const Tensor& b, const Tensor& sfa, const Tensor& sfb, int64_t k,
                          const Tensor& alpha) {
  for (const Tensor* t : {&a, &b, &sfa, &sfb}) {
    TORCH_CHECK(t->is_cuda() && t->device() == a.device(), "All NVFP4 tensors must be on the same CUDA device");
    TORCH_CHECK(t->layout() == at::kStrided && t->is_contiguous(), "NVFP4 storage tensors must be contiguous");
    TORCH_CHECK(t->scalar_type() == at::kByte, "NVFP4 storage tensors must be uint8");
  }
  TORCH_CHECK(a.dim() == 2 && b.dim() == 2, "Packed A and B_rows must be matrices");
  for (auto d : {a.size(0), b.size(0), k}) {
    TORCH_CHECK(d > 0 && d <= std::numeric_limits<int>::max() - 128,
                "NVFP4 dimensions must be positive and allow int32 tile padding");
  }
  TORCH_CHECK(k % 32 == 0, "NVFP4 K must be a multiple of 32");
  TORCH_CHECK(a.size(1) == k / 2 && b.size(1) == k / 2, "Packed operands must contain K/2 bytes per row");
  TORCH_CHECK(sfa.dim() == 1 && sfb.dim() == 1, "Scale buffers must be one-dimensional");
  check_alpha(alpha, a);
  TORCH_CHECK(sfa.numel() == sdc_nvfp4_scale_size(a.size(0), k) && sfb.numel() == sdc_nvfp4_scale_size(b.size(0), k),
              "Scale buffers must match the official CUTLASS scale layout sizes");
}

// Restates check_projection_arguments (src/cutlass_gemm/csrc/abft/common/sm120_epilogue.cuh:153-177).
void check_projection(const Tensor& a, const Tensor& weights, int channels, int64_t m, int64_t n, int64_t row,
                      int64_t col, int64_t bit, OptTensor nonfinite) {
  TORCH_CHECK(weights.is_cuda() && weights.device() == a.device() && weights.layout() == at::kStrided &&
                  weights.scalar_type() == at::kFloat && weights.is_contiguous() && weights.dim() == 2 &&
                  weights.size(0) == channels && weights.size(1) == m,
              "ABFT weights must be contiguous CUDA FP32 [", channels, ",M] on the operand device");
  TORCH_CHECK((row == -1 && col == -1 && bit == -1) ||
                  (row >= 0 && row < m && col >= 0 && col < n && bit >= 0 && bit < 32),
              "ABFT fault must be all -1, or a valid output row/column and FP32 bit [0,31]");
  if (nonfinite.has_value()) {
    const Tensor& flag = *nonfinite;
    TORCH_CHECK(flag.is_cuda() && flag.device() == a.device() && flag.layout() == at::kStrided &&
                    flag.scalar_type() == at::kInt && flag.is_contiguous() && flag.dim() == 1 && flag.size(0) == 1,
                "ABFT nonfinite must be contiguous CUDA int32 [1] on the operand device");
    at::assert_no_overlap(flag, a);
    at::assert_no_overlap(flag, weights);
  }
}

// Block-scaled FP8 (an extension: the reference has no such operator): E4M3
// codes, fp32 scales [M, K/128] for A and [ceil(N/128), K/128] for B_rows.
void check_fp8_block_operands(const Tensor& a, const Tensor& b, const Tensor& scale_a, const Tensor& scale_b) {
  TORCH_CHECK(a.is_cuda() && b.is_cuda() && a.device() == b.device(), "A and B must be on the same CUDA device");
  TORCH_CHECK(a.layout() == at::kStrided && b.layout() == at::kStrided && a.dim() == 2 && b.dim() == 2 &&
                  a.is_contiguous() && b.is_contiguous(),
              "A and B_rows must be contiguous row-major matrices");
  TORCH_CHECK(a.scalar_type() == at::ScalarType::Float8_e4m3fn && b.scalar_type() == at::ScalarType::Float8_e4m3fn,
              "block-scaled FP8 GEMM requires E4M3FN operands");
  TORCH_CHECK(a.size(1) == b.size(1), "A and B_rows K dimensions must match");
  for (auto d : {a.size(0), b.size(0), a.size(1)}) {
    TORCH_CHECK(d > 0 && d <= std::numeric_limits<int>::max() - 128,
                "Matrix dimensions must be positive and allow int32 tile padding");
  }
  TORCH_CHECK(a.size(1) % 128 == 0, "block-scaled FP8 K must be a multiple of 128");
  const int64_t kb = a.size(1) / 128;
  for (const Tensor* t : {&scale_a, &scale_b}) {
    TORCH_CHECK(t->is_cuda() && t->device() == a.device() && t->layout() == at::kStrided &&
                    t->scalar_type() == at::kFloat && t->is_contiguous() && t->dim() == 2,
                "block scales must be contiguous CUDA FP32 matrices on the operand device");
  }
  TORCH_CHECK(scale_a.size(0) == a.size(0) && scale_a.size(1) == kb, "scale_a must be [M, K/128]");
  TORCH_CHECK(scale_b.size(0) == (b.size(0) + 127) / 128 && scale_b.size(1) == kb,
              "scale_b must be [ceil(N/128), K/128]");
}

const uint8_t* u8(const Tensor& t) { return static_cast<const uint8_t*>(t.const_data_ptr()); }
int32_t* opt_i32(OptTensor t) { return t.has_value() ? t->data_ptr<int32_t>() : nullptr; }

// ---------------------------------------------------------------- GEMMs ----

Tensor fp8_mm(const Tensor& a, const Tensor& b, const Tensor& alpha) {
  check_fp8_operands(a, b, alpha);
  const c10::cuda::CUDAGuard guard(a.device());
  const int64_t m = a.size(0), n = b.size(0), k = a.size(1);
  auto out = at::empty_strided({m, n}, {1, m}, a.options().dtype(at::kFloat));
  check_status(sdc_fp8_gemm(u8(a), u8(b), m, n, k, alpha.const_data_ptr<float>(), out.data_ptr<float>(), stream_of(a)));
  return out;
}

Tensor nvfp4_mm(const Tensor& a, const Tensor& b, const Tensor& sfa, const Tensor& sfb, int64_t k,
                const Tensor& alpha) {
  check_nvfp4_operands(a, b, sfa, sfb, k, alpha);
  const c10::cuda::CUDAGuard guard(a.device());
  const int64_t m = a.size(0), n = b.size(0);
  auto out = at::empty({m, n}, a.options().dtype(at::kBFloat16));
  check_status(sdc_nvfp4_gemm(u8(a), u8(b), u8(sfa), u8(sfb), m, n, k, alpha.const_data_ptr<float>(),
                              static_cast<uint16_t*>(out.data_ptr()), stream_of(a)));
  return out;
}

Out3 abft_fp8_mm(const Tensor& a, const Tensor& b, const Tensor& alpha, const Tensor& weights, int64_t row,
                 int64_t col, int64_t bit, int64_t algorithm, OptTensor nonfinite) {
  const int c = channels_of(algorithm);
  check_fp8_operands(a, b, alpha);
  const c10::cuda::CUDAGuard guard(a.device());
  const int64_t m = a.size(0), n = b.size(0), k = a.size(1);
  if (nonfinite.has_value()) {
    at::assert_no_overlap(*nonfinite, b);
    at::assert_no_overlap(*nonfinite, alpha);
  }
  check_projection(a, weights, c, m, n, row, col, bit, nonfinite);
  const int64_t tm = (m + 127) / 128, np = ((n + 63) / 64) * 64;
  auto out = at::empty_strided({m, n}, {1, m}, a.options().dtype(at::kFloat));
  auto observed = at::empty({c, tm, np}, a.options().dtype(at::kFloat));
  auto hit = at::empty({1}, a.options().dtype(at::kInt));
  check_status(sdc_abft_fp8_gemm(u8(a), u8(b), m, n, k, alpha.const_data_ptr<float>(), static_cast<int>(algorithm),
                                 weights.const_data_ptr<float>(), row, col, bit, opt_i32(nonfinite),
                                 out.data_ptr<float>(), observed.data_ptr<float>(), hit.data_ptr<int32_t>(),
                                 stream_of(a)));
  return {out, observed, hit};
}

Out5 abft_fp8_reference_mm(const Tensor& a, const Tensor& b, const Tensor& alpha, const Tensor& weights,
                           int64_t row, int64_t col, int64_t bit, int64_t algorithm, OptTensor nonfinite,
                           int64_t layout) {
  const int c = channels_of(algorithm);
  TORCH_CHECK(layout == SDC_LAYOUT_TILE || layout == SDC_LAYOUT_KSLICE, "ABFT reference layout must be 0 or 1");
  check_fp8_operands(a, b, alpha);
  const c10::cuda::CUDAGuard guard(a.device());
  const int64_t m = a.size(0), n = b.size(0), k = a.size(1);
  if (nonfinite.has_value()) {
    at::assert_no_overlap(*nonfinite, b);
    at::assert_no_overlap(*nonfinite, alpha);
  }
  check_projection(a, weights, c, m, n, row, col, bit, nonfinite);
  const int64_t tm = (m + 127) / 128, np = ((n + 63) / 64) * 64;
  auto out = at::empty_strided({m, n}, {1, m}, a.options().dtype(at::kFloat));
  auto observed = at::empty({c, tm, np}, a.options().dtype(at::kFloat));
  auto predicted = at::empty_like(observed);
  auto magnitude = at::empty_like(observed);
  auto hit = at::empty({1}, a.options().dtype(at::kInt));
  const size_t ws_bytes = sdc_abft_workspace_bytes(static_cast<int>(algorithm), m, n, k, static_cast<int>(layout));
  auto ws = workspace(a, ws_bytes);
  check_status(sdc_abft_fp8_reference_gemm(
      u8(a), u8(b), m, n, k, alpha.const_data_ptr<float>(), static_cast<int>(algorithm),
      weights.const_data_ptr<float>(), row, col, bit, opt_i32(nonfinite), out.data_ptr<float>(),
      observed.data_ptr<float>(), hit.data_ptr<int32_t>(), predicted.data_ptr<float>(), magnitude.data_ptr<float>(),
      static_cast<int>(layout), ws.data_ptr(), ws_bytes, stream_of(a)));
  return {out, observed, hit, predicted, magnitude};
}

Out3 abft_nvfp4_mm(const Tensor& a, const Tensor& b, const Tensor& sfa, const Tensor& sfb, int64_t k,
                   const Tensor& alpha, const Tensor& weights, int64_t row, int64_t col, int64_t bit,
                   int64_t algorithm, OptTensor nonfinite) {
  const int c = channels_of(algorithm);
  check_nvfp4_operands(a, b, sfa, sfb, k, alpha);
  const c10::cuda::CUDAGuard guard(a.device());
  const int64_t m = a.size(0), n = b.size(0);
  if (nonfinite.has_value() && nonfinite->defined()) {
    for (const Tensor* t : {&b, &sfa, &sfb, &alpha}) at::assert_no_overlap(*nonfinite, *t);
  }
  check_projection(a, weights, c, m, n, row, col, bit, nonfinite);
  const int64_t tm = (m + 127) / 128, np = ((n + 127) / 128) * 128;
  auto out = at::empty({m, n}, a.options().dtype(at::kBFloat16));
  auto observed = at::empty({c, tm, np}, a.options().dtype(at::kFloat));
  auto hit = at::empty({1}, a.options().dtype(at::kInt));
  check_status(sdc_abft_nvfp4_gemm(u8(a), u8(b), u8(sfa), u8(sfb), m, n, k, alpha.const_data_ptr<float>(),
                                   static_cast<int>(algorithm), weights.const_data_ptr<float>(), row, col, bit,
                                   opt_i32(nonfinite), static_cast<uint16_t*>(out.data_ptr()),
                                   observed.data_ptr<float>(), hit.data_ptr<int32_t>(), stream_of(a)));
  return {out, observed, hit};
}

Out5 abft_nvfp4_reference_mm(const Tensor& a, const Tensor& b, const Tensor& sfa, const Tensor& sfb, int64_t k,
                             const Tensor& alpha, const Tensor& weights, int64_t row, int64_t col, int64_t bit,
                             int64_t algorithm, OptTensor nonfinite, int64_t layout) {
  const int c = channels_of(algorithm);
  TORCH_CHECK(layout == SDC_LAYOUT_TILE || layout == SDC_LAYOUT_KSLICE, "ABFT reference layout must be 0 or 1");
  check_nvfp4_operands(a, b, sfa, sfb, k, alpha);
  const c10::cuda::CUDAGuard guard(a.device());
  const int64_t m = a.size(0), n = b.size(0);
  if (nonfinite.has_value() && nonfinite->defined()) {
    for (const Tensor* t : {&b, &sfa, &sfb, &alpha}) at::assert_no_overlap(*nonfinite, *t);
  }
  check_projection(a, weights, c, m, n, row, col, bit, nonfinite);
  const int64_t tm = (m + 127) / 128, np = ((n + 127) / 128) * 128;
  auto out = at::empty({m, n}, a.options().dtype(at::kBFloat16));
  auto observed = at::empty({c, tm, np}, a.options().dtype(at::kFloat));
  auto predicted = at::empty_like(observed);
  auto magnitude = at::empty_like(observed);
  auto hit = at::empty({1}, a.options().dtype(at::kInt));
  const size_t ws_bytes = sdc_abft_workspace_bytes(static_cast<int>(algorithm), m, n, k, static_cast<int>(layout));
  auto ws = workspace(a, ws_bytes);
  check_status(sdc_abft_nvfp4_reference_gemm(
      u8(a), u8(b), u8(sfa), u8(sfb), m, n, k, alpha.const_data_ptr<float>(), static_cast<int>(algorithm),
      weights.const_data_ptr<float>(), row, col, bit, opt_i32(nonfinite), static_cast<uint16_t*>(out.data_ptr()),
      observed.data_ptr<float>(), hit.data_ptr<int32_t>(), predicted.data_ptr<float>(), magnitude.data_ptr<float>(),
      static_cast<int>(layout), ws.data_ptr(), ws_bytes, stream_of(a)));
  return {out, observed, hit, predicted, magnitude};
}

Tensor fp8_block_mm(const Tensor& a, const Tensor& b, const Tensor& scale_a, const Tensor& scale_b) {
  check_fp8_block_operands(a, b, scale_a, scale_b);
  const c10::cuda::CUDAGuard guard(a.device());
  const int64_t m = a.size(0), n = b.size(0), k = a.size(1);
  auto out = at::empty({m, n}, a.options().dtype(at::kBFloat16));
  check_status(sdc_fp8_block_gemm(u8(a), u8(b), scale_a.const_data_ptr<float>(), scale_b.const_data_ptr<float>(), m,
                                  n, k, static_cast<uint16_t*>(out.data_ptr()), stream_of(a)));
  return out;
}

Out3 abft_fp8_block_mm(const Tensor& a, const Tensor& b, const Tensor& scale_a, const Tensor& scale_b,
                       const Tensor& weights, int64_t row, int64_t col, int64_t bit, int64_t algorithm,
                       OptTensor nonfinite) {
  const int c = channels_of(algorithm);
  check_fp8_block_operands(a, b, scale_a, scale_b);
  const c10::cuda::CUDAGuard guard(a.device());
  const int64_t m = a.size(0), n = b.size(0), k = a.size(1);
  if (nonfinite.has_value()) {
    for (const Tensor* t : {&b, &scale_a, &scale_b}) at::assert_no_overlap(*nonfinite, *t);
  }
  check_projection(a, weights, c, m, n, row, col, bit, nonfinite);
  const int64_t tm = (m + 127) / 128, np = ((n + 127) / 128) * 128;
  auto out = at::empty({m, n}, a.options().dtype(at::kBFloat16));
  auto observed = at::empty({c, tm, np}, a.options().dtype(at::kFloat));
  auto hit = at::empty({1}, a.options().dtype(at::kInt));
  check_status(sdc_abft_fp8_block_gemm(u8(a), u8(b), scale_a.const_data_ptr<float>(), scale_b.const_data_ptr<float>(),
                                       m, n, k, static_cast<int>(algorithm), weights.const_data_ptr<float>(), row, col,
                                       bit, opt_i32(nonfinite), static_cast<uint16_t*>(out.data_ptr()),
                                       observed.data_ptr<float>(), hit.data_ptr<int32_t>(), stream_of(a)));
  return {out, observed, hit};
}

Out5 abft_fp8_block_reference_mm(const Tensor& a, const Tensor& b, const Tensor& scale_a, const Tensor& scale_b,
                                 const Tensor& weights, int64_t row, int64_t col, int64_t bit, int64_t algorithm,
                                 OptTensor nonfinite) {
  const int c = channels_of(algorithm);
  check_fp8_block_operands(a, b, scale_a, scale_b);
  const c10::cuda::CUDAGuard guard(a.device());
  const int64_t m = a.size(0), n = b.size(0), k = a.size(1);
  if (nonfinite.has_value()) {
    for (const Tensor* t : {&b, &scale_a, &scale_b}) at::assert_no_overlap(*nonfinite, *t);
  }
  check_projection(a, weights, c, m, n, row, col, bit, nonfinite);
  const int64_t tm = (m + 127) / 128, np = ((n + 127) / 128) * 128;
  auto out = at::empty({m, n}, a.options().dtype(at::kBFloat16));
  auto observed = at::empty({c, tm, np}, a.options().dtype(at::kFloat));
  auto predicted = at::empty_like(observed);
  auto magnitude = at::empty_like(observed);
  auto hit = at::empty({1}, a.options().dtype(at::kInt));
  const size_t ws_bytes =
      sdc_abft_workspace_bytes(static_cast<int>(algorithm), m, n, k, static_cast<int>(SDC_LAYOUT_KSLICE));
  auto ws = workspace(a, ws_bytes);
  check_status(sdc_abft_fp8_block_reference_gemm(
      u8(a), u8(b), scale_a.const_data_ptr<float>(), scale_b.const_data_ptr<float>(), m, n, k,
      static_cast<int>(algorithm), weights.const_data_ptr<float>(), row, col, bit, opt_i32(nonfinite),
      static_cast<uint16_t*>(out.data_ptr()), observed.data_ptr<float>(), hit.data_ptr<int32_t>(),
      predicted.data_ptr<float>(), magnitude.data_ptr<float>(), ws.data_ptr(), ws_bytes, stream_of(a)));
  return {out, observed, hit, predicted, magnitude};
}

// ---------------------------------------------------- row checksums (ext) ----

using Out8 = std::tuple<Tensor, Tensor, Tensor, Tensor, Tensor, Tensor, Tensor, Tensor>;
void check_common(int64_t n, double atol, double rtol);  // finalize's checks (below)

// The input-fused GEMM of `kind` with its row checksums: the reference op's
// five outputs plus row_observed [ceil(N/64), M] and the row prediction and
// magnitude [M]. Operands as the kind's own op takes them (a_scales/b_scales:
// NVFP4 scale atoms or block-scaled FP8 fp32 scales; alpha: FP8 and NVFP4).
Out8 abft_reference_rows_mm(int64_t kind, const Tensor& a, OptTensor a_scales, const Tensor& b, OptTensor b_scales,
                            int64_t k, OptTensor alpha, const Tensor& weights, int64_t row, int64_t col, int64_t bit,
                            int64_t algorithm, OptTensor nonfinite, int64_t layout) {
  const int c = channels_of(algorithm);
  TORCH_CHECK(kind == SDC_KIND_FP8 || kind == SDC_KIND_NVFP4 || kind == SDC_KIND_FP8_BLOCK,
              "row checksums: kind must be 0 (FP8), 1 (NVFP4) or 2 (block-scaled FP8)");
  TORCH_CHECK(layout == SDC_LAYOUT_TILE || layout == SDC_LAYOUT_KSLICE, "ABFT reference layout must be 0 or 1");
  const void* sa = nullptr;
  const void* sb = nullptr;
  const float* al = nullptr;
  if (kind == SDC_KIND_FP8) {
    TORCH_CHECK(alpha.has_value(), "FP8 row checksums need alpha");
    check_fp8_operands(a, b, *alpha);
    TORCH_CHECK(a.size(1) == k, "K must equal the operands' K");
    al = alpha->const_data_ptr<float>();
  } else if (kind == SDC_KIND_NVFP4) {
    TORCH_CHECK(alpha.has_value() && a_scales.has_value() && b_scales.has_value(),
                "NVFP4 row checksums need both scale tensors and alpha");
    check_nvfp4_operands(a, b, *a_scales, *b_scales, k, *alpha);
    sa = a_scales->const_data_ptr();
    sb = b_scales->const_data_ptr();
    al = alpha->const_data_ptr<float>();
  } else {
    TORCH_CHECK(a_scales.has_value() && b_scales.has_value(), "block-scaled FP8 row checksums need both scales");
    check_fp8_block_operands(a, b, *a_scales, *b_scales);
    TORCH_CHECK(a.size(1) == k, "K must equal the operands' K");
    sa = a_scales->const_data_ptr();
    sb = b_scales->const_data_ptr();
  }
  const c10::cuda::CUDAGuard guard(a.device());
  const int64_t m = a.size(0), n = b.size(0);
  check_projection(a, weights, c, m, n, row, col, bit, nonfinite);
  const int64_t tm = (m + 127) / 128, np = kind == SDC_KIND_FP8 ? ((n + 63) / 64) * 64 : ((n + 127) / 128) * 128;
  Tensor out = kind == SDC_KIND_FP8 ? at::empty_strided({m, n}, {1, m}, a.options().dtype(at::kFloat))
                                    : at::empty({m, n}, a.options().dtype(at::kBFloat16));
  const auto f32 = a.options().dtype(at::kFloat);
  auto observed = at::empty({c, tm, np}, f32);
  auto predicted = at::empty_like(observed);
  auto magnitude = at::empty_like(observed);
  auto hit = at::empty({1}, a.options().dtype(at::kInt));
  auto row_observed = at::empty({(n + 63) / 64, m}, f32);
  auto row_predicted = at::empty({m}, f32);
  auto row_magnitude = at::empty({m}, f32);
  const size_t ws_bytes = sdc_abft_workspace_bytes(static_cast<int>(algorithm), m, n, k, static_cast<int>(layout));
  auto ws = workspace(a, ws_bytes);
  check_status(sdc_abft_reference_gemm_rows(
      static_cast<int>(kind), u8(a), sa, u8(b), sb, m, n, k, al, static_cast<int>(algorithm),
      weights.const_data_ptr<float>(), row, col, bit, opt_i32(nonfinite), out.data_ptr(), observed.data_ptr<float>(),
      hit.data_ptr<int32_t>(), predicted.data_ptr<float>(), magnitude.data_ptr<float>(), static_cast<int>(layout),
      row_observed.data_ptr<float>(), ws.data_ptr(), ws_bytes, stream_of(a)));
  const size_t row_ws_bytes = sdc_abft_row_workspace_bytes(n, k);
  auto row_ws = workspace(a, row_ws_bytes);
  check_status(sdc_abft_row_reference(static_cast<int>(kind), u8(a), sa, u8(b), sb, m, n, k, al,
                                      row_predicted.data_ptr<float>(), row_magnitude.data_ptr<float>(),
                                      row_ws.data_ptr(), row_ws_bytes, stream_of(a)));
  return {out, observed, hit, predicted, magnitude, row_observed, row_predicted, row_magnitude};
}

Out5 abft_locate2d(const Tensor& row_observed, const Tensor& row_predicted, const Tensor& row_magnitude, double atol,
                   double rtol, const Tensor& residual, const Tensor& threshold, const Tensor& flags,
                   int64_t algorithm) {
  const int c = channels_of(algorithm);
  for (const Tensor* t : {&row_observed, &row_predicted, &row_magnitude, &residual, &threshold}) {
    TORCH_CHECK(t->is_cuda() && t->device() == row_observed.device() && t->is_contiguous() &&
                    t->scalar_type() == at::kFloat,
                "locate2d tensors must be contiguous CUDA float32 on one device");
  }
  TORCH_CHECK(row_observed.dim() == 2 && row_predicted.dim() == 1 && row_magnitude.sizes() == row_predicted.sizes() &&
                  row_observed.size(1) == row_predicted.size(0),
              "locate2d: row_observed [ceil(N/64), M] and row prediction/magnitude [M]");
  TORCH_CHECK(residual.dim() == 2 && residual.size(0) == c && threshold.sizes() == residual.sizes(),
              "locate2d: residual and threshold must be finalize's diagnostics [channels, N]");
  TORCH_CHECK(flags.is_cuda() && flags.scalar_type() == at::kBool && flags.numel() == 5,
              "locate2d: flags must be finalize's bool[5]");
  check_common(residual.size(1), atol, rtol);
  const c10::cuda::CUDAGuard guard(row_observed.device());
  const int64_t m = row_predicted.size(0), n = residual.size(1);
  const auto f32 = row_observed.options();
  auto row_residual = at::empty({m}, f32);
  auto row_threshold = at::empty({m}, f32);
  auto location = at::empty({2}, f32.dtype(at::kLong));
  auto located = at::empty({}, f32.dtype(at::kBool));
  auto row_flags = at::empty({2}, f32.dtype(at::kBool));
  const size_t ws_bytes = sdc_abft_locate2d_workspace_bytes();
  auto ws = workspace(row_observed, ws_bytes);
  check_status(sdc_abft_locate2d(
      row_observed.const_data_ptr<float>(), row_observed.size(0), row_predicted.const_data_ptr<float>(),
      row_magnitude.const_data_ptr<float>(), m, static_cast<float>(atol), static_cast<float>(rtol),
      residual.const_data_ptr<float>(), threshold.const_data_ptr<float>(), static_cast<int>(algorithm), n,
      static_cast<const uint8_t*>(flags.const_data_ptr()), row_residual.data_ptr<float>(),
      row_threshold.data_ptr<float>(), location.data_ptr<int64_t>(), static_cast<uint8_t*>(located.data_ptr()),
      static_cast<uint8_t*>(row_flags.data_ptr()), ws.data_ptr(), ws_bytes, stream_of(row_observed)));
  return {location, located, row_flags, row_residual, row_threshold};
}

// -------------------------------------------------------------- finalize ----
// Restates the checks of src/cutlass_gemm/csrc/abft/common/finalize.cu:154-319.

void check_common(int64_t n, double atol, double rtol) {
  TORCH_CHECK(n > 0 && n <= std::numeric_limits<int>::max() - 128,
              "ABFT finalize N must be positive and fit padded int32 extents");
  const double fmax = std::numeric_limits<float>::max();
  TORCH_CHECK(std::isfinite(atol) && std::isfinite(rtol) && atol >= 0. && rtol >= 0. && atol <= fmax && rtol <= fmax,
              "ABFT finalize tolerances must be finite nonnegative float32 values");
}

void check_reference(OptTensor reference, const Tensor& proto, int channels, int64_t n) {
  if (!reference.has_value()) return;
  const Tensor& r = *reference;
  TORCH_CHECK(r.is_cuda() && r.device() == proto.device() && r.layout() == at::kStrided && r.is_contiguous() &&
                  r.scalar_type() == at::kFloat && r.dim() == 3 && r.size(0) == 2 && r.size(1) == channels &&
                  r.size(2) == n,
              "ABFT finalize reference must be contiguous float32 [2,channels,N] on the same CUDA device");
}

void check_thresholds(OptTensor thresholds, const Tensor& proto, int channels, int64_t n) {
  if (!thresholds.has_value()) return;
  const Tensor& t = *thresholds;
  TORCH_CHECK(t.is_cuda() && t.device() == proto.device() && t.layout() == at::kStrided && t.is_contiguous() &&
                  t.scalar_type() == at::kFloat &&
                  ((t.dim() == 1 && t.size(0) == 1) || (t.dim() == 2 && t.size(0) == channels && t.size(1) == n)),
              "ABFT finalize thresholds must be contiguous CUDA float32 [1] or [channels,N] on the same CUDA device");
}

Out6 run_finalize(const Tensor& proto, int64_t algorithm, int channels, const float* observed,
                  const float* predicted, const float* magnitude, int64_t m_tiles, int64_t padded_n, int64_t n,
                  const int32_t* tile_flags, int64_t flag_count, const int32_t* hit_in, const int32_t* nonfinite_in,
                  double atol, double rtol, OptTensor reference, bool diagnostics, OptTensor thresholds) {
  const c10::cuda::CUDAGuard guard(proto.device());
  Tensor out_ref = reference.has_value() ? *reference : at::empty({2, channels, n}, proto.options());
  if (thresholds.has_value()) at::assert_no_overlap(*thresholds, out_ref);
  Tensor residual = diagnostics ? at::empty({channels, n}, proto.options()) : at::empty({0}, proto.options());
  Tensor threshold = diagnostics ? at::empty({channels, n}, proto.options()) : at::empty({0}, proto.options());
  Tensor flags = at::empty({5}, proto.options().dtype(at::kBool));
  Tensor hit = at::empty({1}, proto.options().dtype(at::kInt));
  Tensor location = at::empty({2}, proto.options().dtype(at::kLong));
  const size_t ws_bytes = sdc_abft_finalize_workspace_bytes(static_cast<int>(algorithm), n, m_tiles);
  Tensor ws = workspace(proto, ws_bytes);
  check_status(sdc_abft_finalize(
      static_cast<int>(algorithm), observed, predicted, magnitude, m_tiles, padded_n, n, tile_flags, flag_count,
      hit_in, nonfinite_in, static_cast<float>(atol), static_cast<float>(rtol), out_ref.data_ptr<float>(),
      reference.has_value() ? 1 : 0, diagnostics ? 1 : 0, diagnostics ? residual.data_ptr<float>() : nullptr,
      diagnostics ? threshold.data_ptr<float>() : nullptr,
      thresholds.has_value() ? thresholds->const_data_ptr<float>() : nullptr,
      thresholds.has_value() && thresholds->numel() == 1 ? 1 : 0, static_cast<uint8_t*>(flags.data_ptr()),
      hit.data_ptr<int32_t>(), location.data_ptr<int64_t>(), ws.data_ptr(), ws_bytes, stream_of(proto)));
  return {out_ref, residual, threshold, flags, hit, location};
}

Out6 abft_finalize(const Tensor& partials, const Tensor& tile_flags, int64_t n, double atol, double rtol,
                   OptTensor reference, bool diagnostics, int64_t algorithm, OptTensor thresholds) {
  const int c = channels_of(algorithm);
  check_common(n, atol, rtol);
  TORCH_CHECK(partials.is_cuda() && tile_flags.is_cuda() && partials.device() == tile_flags.device(),
              "ABFT finalize tensors must be on the same CUDA device");
  TORCH_CHECK(partials.layout() == at::kStrided && partials.is_contiguous() && partials.scalar_type() == at::kFloat &&
                  partials.dim() == 4 && partials.size(0) == 3 && partials.size(1) == c && partials.size(2) > 0,
              "ABFT finalize partials must be contiguous float32 [3,channels,T,padded_N] with T>0");
  const int64_t n_tiles = (n + 127) / 128, padded_n = n_tiles * 128, m_tiles = partials.size(2);
  TORCH_CHECK(partials.size(3) == padded_n, "ABFT finalize padded_N must equal ceil(N/128)*128");
  TORCH_CHECK(tile_flags.layout() == at::kStrided && tile_flags.is_contiguous() && tile_flags.scalar_type() == at::kInt &&
                  tile_flags.dim() == 2 && tile_flags.size(0) == m_tiles && tile_flags.size(1) == n_tiles,
              "ABFT finalize tile_flags must be contiguous int32 [T,ceil(N/128)]");
  check_reference(reference, partials, c, n);
  check_thresholds(thresholds, partials, c, n);
  const int64_t field = c * m_tiles * padded_n;
  const float* obs = partials.const_data_ptr<float>();
  return run_finalize(partials, algorithm, c, obs, obs + field, obs + 2 * field, m_tiles, padded_n, n,
                      tile_flags.const_data_ptr<int32_t>(), m_tiles * n_tiles, nullptr, nullptr, atol, rtol, reference,
                      diagnostics, thresholds);
}

Out6 abft_finalize_reference(const Tensor& observed, const Tensor& predicted, const Tensor& magnitude,
                             const Tensor& hit, const Tensor& nonfinite, int64_t n, double atol, double rtol,
                             OptTensor reference, bool diagnostics, int64_t algorithm, OptTensor thresholds) {
  const int c = channels_of(algorithm);
  check_common(n, atol, rtol);
  TORCH_CHECK(observed.is_cuda(), "ABFT finalize observed must be a CUDA tensor");
  for (const Tensor* t : {&predicted, &magnitude, &hit, &nonfinite}) {
    TORCH_CHECK(t->is_cuda() && t->device() == observed.device(), "ABFT finalize inputs must be on the same CUDA device");
  }
  TORCH_CHECK(observed.layout() == at::kStrided && observed.is_contiguous() && observed.scalar_type() == at::kFloat &&
                  observed.dim() == 3 && observed.size(0) == c && observed.size(1) > 0,
              "ABFT finalize observed must be contiguous float32 [channels,T,padded_N] with T>0");
  for (const Tensor* t : {&predicted, &magnitude}) {
    TORCH_CHECK(t->layout() == at::kStrided && t->is_contiguous() && t->scalar_type() == at::kFloat &&
                    t->sizes() == observed.sizes(),
                "ABFT finalize predicted/magnitude must match observed's contiguous float32 layout and shape");
  }
  const int64_t padded_n = observed.size(2);
  TORCH_CHECK(padded_n == ((n + 63) / 64) * 64 || padded_n == ((n + 127) / 128) * 128,
              "ABFT finalize padded_N must equal ceil(N/64)*64 or ceil(N/128)*128");
  for (const Tensor* t : {&hit, &nonfinite}) {
    TORCH_CHECK(t->layout() == at::kStrided && t->is_contiguous() && t->scalar_type() == at::kInt && t->dim() == 1 &&
                    t->size(0) == 1,
                "ABFT finalize hit/nonfinite must be contiguous CUDA int32 [1] tensors");
  }
  check_reference(reference, observed, c, n);
  check_thresholds(thresholds, observed, c, n);
  return run_finalize(observed, algorithm, c, observed.const_data_ptr<float>(), predicted.const_data_ptr<float>(),
                      magnitude.const_data_ptr<float>(), observed.size(1), padded_n, n, nullptr, 0,
                      hit.const_data_ptr<int32_t>(), nonfinite.const_data_ptr<int32_t>(), atol, rtol, reference,
                      diagnostics, thresholds);
}

// ---------------------------------------------------------- quantisation ----

int dtype_code(const Tensor& x) {
  TORCH_CHECK(x.scalar_type() == at::kFloat || x.scalar_type() == at::kBFloat16, "quantize requires FP32 or BF16 input");
  return x.scalar_type() == at::kFloat ? 0 : 1;
}

// `amax`: optional device fp32 scalar, max |x| of the whole (row-sharded)
// matrix; when given, the "amax" multiplier comes from it instead of x.
void check_global_amax(OptTensor amax, const Tensor& x, std::optional<double> global_scale) {
  if (!amax.has_value()) return;
  TORCH_CHECK(!global_scale.has_value(), "quantize takes a fixed global_scale or a global amax, not both");
  TORCH_CHECK(amax->is_cuda() && amax->device() == x.device() && amax->scalar_type() == at::kFloat &&
                  amax->numel() == 1 && amax->is_contiguous(),
              "global amax must be a CUDA fp32 scalar on the input device");
}

std::tuple<Tensor, Tensor> quantize_fp8(const Tensor& x, std::optional<double> global_scale, OptTensor amax) {
  TORCH_CHECK(x.is_cuda() && x.dim() == 2, "quantize requires a two-dimensional CUDA tensor");
  const int dt = dtype_code(x);
  TORCH_CHECK(x.size(0) > 0 && x.size(1) > 0 && x.size(1) % 4 == 0, "nonempty input columns must be divisible by 4");
  check_global_amax(amax, x, global_scale);
  const c10::cuda::CUDAGuard guard(x.device());
  Tensor xc = x.contiguous();
  auto codes = at::empty(x.sizes(), x.options().dtype(at::kByte));
  auto st = at::empty({}, x.options().dtype(at::kFloat));
  if (amax.has_value()) {
    check_status(sdc_quantize_fp8_global_amax(xc.const_data_ptr(), dt, x.size(0), x.size(1),
                                              amax->const_data_ptr<float>(), codes.data_ptr<uint8_t>(),
                                              st.data_ptr<float>(), stream_of(x)));
    return {codes, st};
  }
  const size_t ws_bytes = sdc_quantize_workspace_bytes(x.size(0), x.size(1));
  Tensor ws = workspace(x, ws_bytes);
  check_status(sdc_quantize_fp8(xc.const_data_ptr(), dt, x.size(0), x.size(1), global_scale.has_value() ? 0 : 1,
                                static_cast<float>(global_scale.value_or(1.0)), codes.data_ptr<uint8_t>(),
                                st.data_ptr<float>(), ws.data_ptr(), ws_bytes, stream_of(x)));
  return {codes, st};
}

std::tuple<Tensor, Tensor> quantize_fp8_block(const Tensor& x, int64_t block_rows) {
  TORCH_CHECK(x.is_cuda() && x.dim() == 2, "quantize requires a two-dimensional CUDA tensor");
  const int dt = dtype_code(x);
  TORCH_CHECK(block_rows == 1 || block_rows == 128, "block_rows must be 1 (activations) or 128 (weights)");
  TORCH_CHECK(x.size(0) > 0 && x.size(1) > 0 && x.size(1) % 128 == 0,
              "nonempty input columns must be divisible by 128");
  const c10::cuda::CUDAGuard guard(x.device());
  Tensor xc = x.contiguous();
  auto codes = at::empty(x.sizes(), x.options().dtype(at::kByte));
  auto scales = at::empty({(x.size(0) + block_rows - 1) / block_rows, x.size(1) / 128}, x.options().dtype(at::kFloat));
  check_status(sdc_quantize_fp8_block(xc.const_data_ptr(), dt, x.size(0), x.size(1), static_cast<int>(block_rows),
                                      codes.data_ptr<uint8_t>(), scales.data_ptr<float>(), stream_of(x)));
  return {codes, scales};
}

std::tuple<Tensor, Tensor, Tensor, Tensor> quantize_nvfp4(const Tensor& x, std::optional<double> global_scale,
                                                          OptTensor amax) {
  TORCH_CHECK(x.is_cuda() && x.dim() == 2, "quantize requires a two-dimensional CUDA tensor");
  const int dt = dtype_code(x);
  const int64_t rows = x.size(0), cols = x.size(1);
  TORCH_CHECK(rows > 0 && cols > 0 && cols % 16 == 0, "nonempty input columns must be divisible by 16");
  check_global_amax(amax, x, global_scale);
  const c10::cuda::CUDAGuard guard(x.device());
  Tensor xc = x.contiguous();
  auto codes = at::empty({rows, cols / 2}, x.options().dtype(at::kByte));
  auto scales = at::empty({rows, cols / 16}, x.options().dtype(at::kByte));
  auto packed = at::empty({sdc_nvfp4_scale_size(rows, cols)}, x.options().dtype(at::kByte));
  auto st = at::empty({}, x.options().dtype(at::kFloat));
  if (amax.has_value()) {
    check_status(sdc_quantize_nvfp4_global_amax(xc.const_data_ptr(), dt, rows, cols, amax->const_data_ptr<float>(),
                                                codes.data_ptr<uint8_t>(), scales.data_ptr<uint8_t>(),
                                                packed.data_ptr<uint8_t>(), st.data_ptr<float>(), stream_of(x)));
    return {codes, scales, packed, st};
  }
  const size_t ws_bytes = sdc_quantize_workspace_bytes(rows, cols);
  Tensor ws = workspace(x, ws_bytes);
  check_status(sdc_quantize_nvfp4(xc.const_data_ptr(), dt, rows, cols, global_scale.has_value() ? 0 : 1,
                                  static_cast<float>(global_scale.value_or(1.0)), codes.data_ptr<uint8_t>(),
                                  scales.data_ptr<uint8_t>(), packed.data_ptr<uint8_t>(), st.data_ptr<float>(),
                                  ws.data_ptr(), ws_bytes, stream_of(x)));
  return {codes, scales, packed, st};
}

// Host-only layout helper (CPU catch-all), as sdc_cutlass_nvfp4_scale_layout.
std::tuple<Tensor, Tensor, int64_t, int64_t> nvfp4_scale_layout(int64_t m, int64_t n, int64_t k) {
  for (auto d : {m, n, k}) {
    TORCH_CHECK(d > 0 && d <= std::numeric_limits<int>::max() - 128,
                "NVFP4 dimensions must be positive and allow int32 tile padding");
  }
  TORCH_CHECK(k % 32 == 0, "NVFP4 K must be a multiple of 32");
  auto opts = at::TensorOptions().device(at::kCPU).dtype(at::kLong);
  auto ia = at::empty({m, k / 16}, opts), ib = at::empty({n, k / 16}, opts);
  check_status(sdc_nvfp4_scale_layout(m, k, ia.data_ptr<int64_t>()));
  check_status(sdc_nvfp4_scale_layout(n, k, ib.data_ptr<int64_t>()));
  return {ia, ib, sdc_nvfp4_scale_size(m, k), sdc_nvfp4_scale_size(n, k)};
}

Tensor nvfp4_pack_scales(const Tensor& scales, int64_t k) {
  TORCH_CHECK(scales.is_cuda() && scales.dim() == 2 && scales.scalar_type() == at::kByte && scales.is_contiguous(),
              "scales must be contiguous CUDA uint8 [rows, K/16]");
  TORCH_CHECK(k % 16 == 0 && scales.size(1) == k / 16, "scales must hold K/16 blocks per row");
  const c10::cuda::CUDAGuard guard(scales.device());
  auto packed = at::empty({sdc_nvfp4_scale_size(scales.size(0), k)}, scales.options());
  check_status(sdc_nvfp4_pack_scales(scales.const_data_ptr<uint8_t>(), scales.size(0), k, packed.data_ptr<uint8_t>(),
                                     stream_of(scales)));
  return packed;
}

// --------------------------------------------------- locate and correct ----

std::tuple<Tensor, Tensor> abft_locate(const Tensor& residual, const Tensor& threshold, const Tensor& flags, int64_t m) {
  TORCH_CHECK(residual.is_cuda() && residual.dim() == 2 && residual.size(0) == 2 && residual.is_contiguous() &&
                  residual.scalar_type() == at::kFloat,
              "abft_locate needs a contiguous CUDA float32 [2,N] residual (Classic policy)");
  TORCH_CHECK(threshold.sizes() == residual.sizes() && threshold.is_contiguous() && threshold.device() == residual.device() &&
                  threshold.scalar_type() == at::kFloat,
              "abft_locate threshold must match residual");
  TORCH_CHECK(flags.device() == residual.device() && flags.scalar_type() == at::kBool && flags.numel() == 5,
              "abft_locate flags must be the finalize bool[5] on the same device");
  const c10::cuda::CUDAGuard guard(residual.device());
  auto location = at::empty({2}, residual.options().dtype(at::kLong));
  auto located = at::empty({}, residual.options().dtype(at::kBool));
  check_status(sdc_abft_locate(residual.const_data_ptr<float>(), threshold.const_data_ptr<float>(),
                               static_cast<const uint8_t*>(flags.const_data_ptr()), m, residual.size(1),
                               location.data_ptr<int64_t>(), static_cast<uint8_t*>(located.data_ptr()),
                               stream_of(residual)));
  return {location, located};
}

Tensor abft_fp8_correct(const Tensor& a, const Tensor& b, const Tensor& alpha, const Tensor& location,
                        const Tensor& located, const Tensor& output) {
  check_fp8_operands(a, b, alpha);
  TORCH_CHECK(output.scalar_type() == at::kFloat && output.dim() == 2 && output.stride(0) == 1 &&
                  output.stride(1) == a.size(0) && output.size(0) == a.size(0) && output.size(1) == b.size(0),
              "abft_fp8_correct output must be the fp32 column-major GEMM output");
  const c10::cuda::CUDAGuard guard(a.device());
  auto corrected = at::empty({}, a.options().dtype(at::kBool));
  check_status(sdc_abft_correct_fp8(u8(a), u8(b), a.size(0), b.size(0), a.size(1), alpha.const_data_ptr<float>(),
                                    location.const_data_ptr<int64_t>(), static_cast<const uint8_t*>(located.const_data_ptr()),
                                    output.data_ptr<float>(), static_cast<uint8_t*>(corrected.data_ptr()), stream_of(a)));
  return corrected;
}

Tensor abft_nvfp4_correct(const Tensor& a, const Tensor& b, const Tensor& sfa, const Tensor& sfb, int64_t k,
                          const Tensor& alpha, const Tensor& location, const Tensor& located, const Tensor& output) {
  check_nvfp4_operands(a, b, sfa, sfb, k, alpha);
  TORCH_CHECK(output.scalar_type() == at::kBFloat16 && output.is_contiguous() && output.size(0) == a.size(0) &&
                  output.size(1) == b.size(0),
              "abft_nvfp4_correct output must be the bf16 row-major GEMM output");
  const c10::cuda::CUDAGuard guard(a.device());
  auto corrected = at::empty({}, a.options().dtype(at::kBool));
  check_status(sdc_abft_correct_nvfp4(u8(a), u8(b), u8(sfa), u8(sfb), a.size(0), b.size(0), k,
                                      alpha.const_data_ptr<float>(), location.const_data_ptr<int64_t>(),
                                      static_cast<const uint8_t*>(located.const_data_ptr()),
                                      static_cast<uint16_t*>(output.data_ptr()), static_cast<uint8_t*>(corrected.data_ptr()),
                                      stream_of(a)));
  return corrected;
}

// Out-of-scope reference precisions (FP32/BF16 SM80 paths) keep their
Tensor abft_fp8_block_correct(const Tensor& a, const Tensor& b, const Tensor& scale_a, const Tensor& scale_b,
                              const Tensor& location, const Tensor& located, const Tensor& output) {
  check_fp8_block_operands(a, b, scale_a, scale_b);
  TORCH_CHECK(output.scalar_type() == at::kBFloat16 && output.is_contiguous() && output.size(0) == a.size(0) &&
                  output.size(1) == b.size(0),
              "abft_fp8_block_correct output must be the bf16 row-major GEMM output");
  const c10::cuda::CUDAGuard guard(a.device());
  auto corrected = at::empty({}, a.options().dtype(at::kBool));
  check_status(sdc_abft_correct_fp8_block(u8(a), u8(b), scale_a.const_data_ptr<float>(),
                                          scale_b.const_data_ptr<float>(), a.size(0), b.size(0), a.size(1),
                                          location.const_data_ptr<int64_t>(),
                                          static_cast<const uint8_t*>(located.const_data_ptr()),
                                          static_cast<uint16_t*>(output.data_ptr()),
                                          static_cast<uint8_t*>(corrected.data_ptr()), stream_of(a)));
  return corrected;
}

// schemas so callers fail with a clear message instead of a missing op.
[[noreturn]] void out_of_scope(const char* name) {
  TORCH_CHECK(false, "sdc_cutlass::", name,
              " (FP32/BF16 legacy kernels) is not part of the sdc_b200 FP8/NVFP4 hot path");
}
// ------------------------------------------------------ bf16 / augmented ----

// A [M,K] and B [K,N], each packed row-major or column-major (the layouts the
// reference accepts); the sm_100a kernels take A row-major and B as rows
// [N,K] (K-major), so the other layouts are repacked first.
std::pair<Tensor, Tensor> bf16_operands(const Tensor& a, const Tensor& b, const char* what) {
  for (const Tensor* t : {&a, &b}) {
    for (int dim = 0; dim < 2; ++dim) {
      TORCH_CHECK(t->size(dim) > 0 && t->size(dim) <= std::numeric_limits<int>::max() - 128, what,
                  " dimensions must be positive and fit padded int32 extents");
    }
  }
  const bool a_row = a.stride(1) == 1 && a.stride(0) == a.size(1);
  const bool a_col = a.stride(0) == 1 && a.stride(1) == a.size(0);
  const bool b_row = b.stride(1) == 1 && b.stride(0) == b.size(1);
  const bool b_col = b.stride(0) == 1 && b.stride(1) == b.size(0);
  TORCH_CHECK(a_row || a_col, what, " A requires packed row-major or column-major storage");
  TORCH_CHECK(b_row || b_col, what, " B requires packed row-major or column-major storage");
  TORCH_CHECK(a.size(1) % 8 == 0, what, " K must be a multiple of 8 on sm_100a (16-byte operand rows)");
  // B column-major [K,N] is already B^T row-major [N,K].
  return {a_row ? a : a.contiguous(), b_col ? b.t() : b.t().contiguous()};
}

const uint16_t* u16(const Tensor& t) { return static_cast<const uint16_t*>(t.const_data_ptr()); }

Tensor mm(const Tensor& a, const Tensor& b) {
  TORCH_CHECK(a.is_cuda() && b.is_cuda(), "A and B must be CUDA tensors");
  TORCH_CHECK(a.device() == b.device(), "A and B must be on the same CUDA device");
  TORCH_CHECK(a.layout() == at::kStrided && b.layout() == at::kStrided, "A and B must be strided tensors");
  TORCH_CHECK(a.dim() == 2 && b.dim() == 2, "A and B must be two-dimensional");
  TORCH_CHECK(a.scalar_type() == b.scalar_type(), "A and B must have the same dtype");
  TORCH_CHECK(a.scalar_type() == at::kBFloat16,
              "sdc_b200 mm computes BF16 operands on the tensor cores (the reference's FP32 SIMT GEMM is not "
              "part of this library)");
  TORCH_CHECK(a.size(1) == b.size(0), "A and B inner dimensions must match");
  const c10::cuda::CUDAGuard guard(a.device());
  auto [ar, br] = bf16_operands(a, b, "BF16 GEMM");
  const int64_t m = a.size(0), n = b.size(1), k = a.size(1);
  auto out = at::empty({m, n}, a.options());
  check_status(sdc_bf16_gemm(u16(ar), u16(br), m, n, k, static_cast<uint16_t*>(out.data_ptr()), stream_of(a)));
  return out;
}

struct AugmentedOut {
  Tensor d, observed, predicted, magnitude, hit, partials, tile_flags;
};

AugmentedOut run_augmented(const Tensor& a, const Tensor& b, const Tensor& weights, int64_t row, int64_t col,
                           int64_t bit, int64_t algorithm, bool compact) {
  const int c = channels_of(algorithm);
  TORCH_CHECK(a.is_cuda() && b.is_cuda() && weights.is_cuda() && a.device() == b.device() &&
                  a.device() == weights.device(),
              "Augmented ABFT tensors must be on the same CUDA device");
  TORCH_CHECK(a.layout() == at::kStrided && b.layout() == at::kStrided && a.dim() == 2 && b.dim() == 2,
              "Augmented ABFT operands must be strided matrices");
  TORCH_CHECK(a.scalar_type() == at::kBFloat16 && b.scalar_type() == at::kBFloat16,
              "Augmented ABFT currently requires BF16 operands");
  TORCH_CHECK(a.size(1) == b.size(0), "Augmented ABFT inner dimensions must match");
  TORCH_CHECK(weights.layout() == at::kStrided && weights.scalar_type() == at::kBFloat16 && weights.dim() == 2 &&
                  weights.size(0) == c && weights.size(1) == a.size(0) && weights.is_contiguous(),
              "Augmented ABFT weights must be contiguous BF16 [", c, ",M]");
  TORCH_CHECK((row == -1 && col == -1 && bit == -1) ||
                  (row >= 0 && row < a.size(0) && col >= 0 && col < b.size(1) && bit >= 0 && bit < 32),
              "Augmented ABFT fault must be all -1, or a valid row/column and FP32 bit 0..31");
  const c10::cuda::CUDAGuard guard(a.device());
  auto [ar, br] = bf16_operands(a, b, "Augmented ABFT");
  const int64_t m = a.size(0), n = b.size(1), k = a.size(1);
  const int64_t tm = (m + 127) / 128, nt = (n + 127) / 128, np = nt * 128;
  AugmentedOut o;
  o.d = at::empty({m, n}, a.options());
  const auto f32 = a.options().dtype(at::kFloat);
  if (compact) {
    o.partials = at::empty({3, c, tm, np}, f32);
    o.observed = o.partials.select(0, 0);
    o.predicted = o.partials.select(0, 1);
    o.magnitude = o.partials.select(0, 2);
    o.tile_flags = at::empty({tm, nt}, a.options().dtype(at::kInt));
  } else {
    o.observed = at::empty({c, tm, np}, f32);
    o.predicted = at::empty_like(o.observed);
    o.magnitude = at::empty_like(o.observed);
    o.hit = at::empty({1}, a.options().dtype(at::kInt));
  }
  const size_t ws_bytes = sdc_abft_augmented_workspace_bytes(static_cast<int>(algorithm), m, k);
  Tensor ws = workspace(a, ws_bytes + 256);
  void* base = reinterpret_cast<void*>((reinterpret_cast<uintptr_t>(ws.data_ptr()) + 255) & ~uintptr_t{255});
  check_status(sdc_abft_bf16_augmented_gemm(
      u16(ar), u16(br), m, n, k, static_cast<int>(algorithm), u16(weights), row, col, bit,
      static_cast<uint16_t*>(o.d.data_ptr()), o.observed.data_ptr<float>(), o.predicted.data_ptr<float>(),
      o.magnitude.data_ptr<float>(), compact ? nullptr : o.hit.data_ptr<int32_t>(),
      compact ? o.tile_flags.data_ptr<int32_t>() : nullptr, base, ws_bytes, stream_of(a)));
  return o;
}

Out5 abft_augmented_mm(const Tensor& a, const Tensor& b, const Tensor& weights, int64_t row, int64_t col, int64_t bit,
                       int64_t algorithm) {
  AugmentedOut o = run_augmented(a, b, weights, row, col, bit, algorithm, false);
  return {o.d, o.observed, o.hit, o.predicted, o.magnitude};
}

Out3 abft_augmented_compact(const Tensor& a, const Tensor& b, const Tensor& weights, int64_t row, int64_t col,
                            int64_t bit, int64_t algorithm) {
  AugmentedOut o = run_augmented(a, b, weights, row, col, bit, algorithm, true);
  return {o.d, o.partials, o.tile_flags};
}

Out3 abft_mm_stub(const Tensor&, const Tensor&, const Tensor&, int64_t, int64_t, int64_t, int64_t, OptTensor) {
  out_of_scope("abft_mm");
}
Out5 abft_reference_mm_stub(const Tensor&, const Tensor&, const Tensor&, int64_t, int64_t, int64_t, int64_t, OptTensor) {
  out_of_scope("abft_reference_mm");
}

}  // namespace

TORCH_LIBRARY(sdc_cutlass, lib) {
  lib.def("mm(Tensor a, Tensor b) -> Tensor");
  lib.def("fp8_mm(Tensor a, Tensor b_rows, Tensor alpha) -> Tensor");
  lib.def("nvfp4_mm(Tensor a_packed, Tensor b_packed, Tensor sfa, Tensor sfb, int k, Tensor alpha) -> Tensor");
  lib.def("abft_mm(Tensor a, Tensor b, Tensor weights, int row, int col, int bit, int algorithm=0, Tensor(a!)? nonfinite=None) -> (Tensor, Tensor, Tensor)");
  lib.def("abft_reference_mm(Tensor a, Tensor b, Tensor weights, int row, int col, int bit, int algorithm=0, Tensor(a!)? nonfinite=None) -> (Tensor, Tensor, Tensor, Tensor, Tensor)");
  lib.def("abft_augmented_mm(Tensor a, Tensor b, Tensor weights, int row, int col, int bit, int algorithm=0) -> (Tensor, Tensor, Tensor, Tensor, Tensor)");
  lib.def("abft_augmented_compact(Tensor a, Tensor b, Tensor weights, int row, int col, int bit, int algorithm=0) -> (Tensor, Tensor, Tensor)");
  lib.def("abft_finalize(Tensor partials, Tensor tile_flags, int n, float atol, float rtol, Tensor(a)? reference, bool diagnostics, int algorithm=0, Tensor? thresholds=None) -> (Tensor(a), Tensor, Tensor, Tensor, Tensor, Tensor)");
  lib.def("abft_finalize_reference(Tensor observed, Tensor predicted, Tensor magnitude, Tensor hit, Tensor nonfinite, int n, float atol, float rtol, Tensor(a)? reference, bool diagnostics, int algorithm=0, Tensor? thresholds=None) -> (Tensor(a), Tensor, Tensor, Tensor, Tensor, Tensor)");
  lib.def("abft_fp8_mm(Tensor a, Tensor b_rows, Tensor alpha, Tensor weights, int row, int col, int bit, int algorithm=0, Tensor(a!)? nonfinite=None) -> (Tensor, Tensor, Tensor)");
  lib.def("abft_fp8_reference_mm(Tensor a, Tensor b_rows, Tensor alpha, Tensor weights, int row, int col, int bit, int algorithm=0, Tensor(a!)? nonfinite=None, int layout=0) -> (Tensor, Tensor, Tensor, Tensor, Tensor)");
  lib.def("abft_nvfp4_mm(Tensor a_packed, Tensor b_packed, Tensor sfa, Tensor sfb, int k, Tensor alpha, Tensor weights, int row, int col, int bit, int algorithm=0, Tensor(a!)? nonfinite=None) -> (Tensor, Tensor, Tensor)");
  lib.def("abft_nvfp4_reference_mm(Tensor a_packed, Tensor b_packed, Tensor sfa, Tensor sfb, int k, Tensor alpha, Tensor weights, int row, int col, int bit, int algorithm=0, Tensor(a!)? nonfinite=None, int layout=0) -> (Tensor, Tensor, Tensor, Tensor, Tensor)");
  lib.def("fp8_block_mm(Tensor a, Tensor b_rows, Tensor scale_a, Tensor scale_b) -> Tensor");
  lib.def("abft_fp8_block_mm(Tensor a, Tensor b_rows, Tensor scale_a, Tensor scale_b, Tensor weights, int row, int col, int bit, int algorithm=0, Tensor(a!)? nonfinite=None) -> (Tensor, Tensor, Tensor)");
  lib.def("abft_fp8_block_reference_mm(Tensor a, Tensor b_rows, Tensor scale_a, Tensor scale_b, Tensor weights, int row, int col, int bit, int algorithm=0, Tensor(a!)? nonfinite=None) -> (Tensor, Tensor, Tensor, Tensor, Tensor)");
  lib.def("quantize_fp8_block(Tensor x, int block_rows) -> (Tensor, Tensor)");
  lib.def("abft_fp8_block_correct(Tensor a, Tensor b_rows, Tensor scale_a, Tensor scale_b, Tensor location, Tensor located, Tensor(a!) output) -> Tensor");
  lib.def("nvfp4_scale_layout(int m, int n, int k) -> (Tensor, Tensor, int, int)", &nvfp4_scale_layout);
  // sdc_b200 extensions.
  lib.def("quantize_fp8(Tensor x, float? global_scale=None, Tensor? amax=None) -> (Tensor, Tensor)");
  lib.def("quantize_nvfp4(Tensor x, float? global_scale=None, Tensor? amax=None) -> (Tensor, Tensor, Tensor, Tensor)");
  lib.def("nvfp4_pack_scales(Tensor scales, int k) -> Tensor");
  lib.def("abft_locate(Tensor residual, Tensor threshold, Tensor flags, int m) -> (Tensor, Tensor)");
  lib.def("abft_reference_rows_mm(int kind, Tensor a, Tensor? a_scales, Tensor b_rows, Tensor? b_scales, int k, Tensor? alpha, Tensor weights, int row, int col, int bit, int algorithm=0, Tensor(a!)? nonfinite=None, int layout=1) -> (Tensor, Tensor, Tensor, Tensor, Tensor, Tensor, Tensor, Tensor)");
  lib.def("abft_locate2d(Tensor row_observed, Tensor row_predicted, Tensor row_magnitude, float atol, float rtol, Tensor residual, Tensor threshold, Tensor flags, int algorithm=0) -> (Tensor, Tensor, Tensor, Tensor, Tensor)");
  lib.def("abft_fp8_correct(Tensor a, Tensor b_rows, Tensor alpha, Tensor location, Tensor located, Tensor(a!) output) -> Tensor");
  lib.def("abft_nvfp4_correct(Tensor a_packed, Tensor b_packed, Tensor sfa, Tensor sfb, int k, Tensor alpha, Tensor location, Tensor located, Tensor(a!) output) -> Tensor");
}

TORCH_LIBRARY_IMPL(sdc_cutlass, CUDA, lib) {
  lib.impl("mm", &mm);
  lib.impl("abft_mm", &abft_mm_stub);
  lib.impl("abft_reference_mm", &abft_reference_mm_stub);
  lib.impl("abft_augmented_mm", &abft_augmented_mm);
  lib.impl("abft_augmented_compact", &abft_augmented_compact);
  lib.impl("fp8_mm", &fp8_mm);
  lib.impl("nvfp4_mm", &nvfp4_mm);
  lib.impl("abft_fp8_mm", &abft_fp8_mm);
  lib.impl("abft_fp8_reference_mm", &abft_fp8_reference_mm);
  lib.impl("abft_nvfp4_mm", &abft_nvfp4_mm);
  lib.impl("abft_nvfp4_reference_mm", &abft_nvfp4_reference_mm);
  lib.impl("abft_finalize", &abft_finalize);
  lib.impl("abft_finalize_reference", &abft_finalize_reference);
  lib.impl("quantize_fp8", &quantize_fp8);
  lib.impl("quantize_nvfp4", &quantize_nvfp4);
  lib.impl("fp8_block_mm", &fp8_block_mm);
  lib.impl("abft_fp8_block_mm", &abft_fp8_block_mm);
  lib.impl("abft_fp8_block_reference_mm", &abft_fp8_block_reference_mm);
  lib.impl("quantize_fp8_block", &quantize_fp8_block);
  lib.impl("abft_fp8_block_correct", &abft_fp8_block_correct);
  lib.impl("nvfp4_pack_scales", &nvfp4_pack_scales);
  lib.impl("abft_locate", &abft_locate);
  lib.impl("abft_reference_rows_mm", &abft_reference_rows_mm);
  lib.impl("abft_locate2d", &abft_locate2d);
  lib.impl("abft_fp8_correct", &abft_fp8_correct);
  lib.impl("abft_nvfp4_correct", &abft_nvfp4_correct);
}
