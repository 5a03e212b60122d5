// extern "C" GEMM entry points: argument contracts of the reference
// operators (src/cutlass_gemm/csrc/gemm/{fp8,nvfp4}.cu and
// abft/{fp8,nvfp4}/*.cu), then the sm_100a launchers in gemm.cu and
// tile_reference.cu.
#include <climits>

#include "gemm.cuh"

namespace sdc {
namespace {

int check_dims(int64_t m, int64_t n, int64_t k) {
  for (int64_t d : {m, n, k}) {
    if (d <= 0 || d > static_cast<int64_t>(INT_MAX) - 128) {
      return fail(SDC_ERR_INVALID, "Matrix dimensions must be positive and allow int32 tile padding");
    }
  }
  if (m * n > static_cast<int64_t>(INT_MAX) * 4) {
    return fail(SDC_ERR_INVALID, "Output has too many elements for this kernel");
  }
  return SDC_OK;
}

int check_fp8(const uint8_t* a, const uint8_t* b, int64_t m, int64_t n, int64_t k,
              const float* alpha, const void* d) {
  int rc = check_dims(m, n, k);
  if (rc != SDC_OK) return rc;
  SDC_REQUIRE(a != nullptr && b != nullptr && alpha != nullptr && d != nullptr,
              "FP8 GEMM pointers must not be null");
  SDC_REQUIRE(k % 16 == 0, "FP8 K must be a multiple of 16 (16-byte operand rows)");
  SDC_REQUIRE(reinterpret_cast<uintptr_t>(a) % 16 == 0 && reinterpret_cast<uintptr_t>(b) % 16 == 0,
              "FP8 operands must be 16-byte aligned");
  return SDC_OK;
}

int check_nvfp4(const uint8_t* a, const uint8_t* b, const uint8_t* sfa, const uint8_t* sfb,
                int64_t m, int64_t n, int64_t k, const float* alpha, const void* d) {
  int rc = check_dims(m, n, k);
  if (rc != SDC_OK) return rc;
  SDC_REQUIRE(a != nullptr && b != nullptr && sfa != nullptr && sfb != nullptr && alpha != nullptr &&
                  d != nullptr,
              "NVFP4 GEMM pointers must not be null");
  SDC_REQUIRE(k % 32 == 0, "NVFP4 K must be a multiple of 32");
  SDC_REQUIRE(reinterpret_cast<uintptr_t>(a) % 16 == 0 && reinterpret_cast<uintptr_t>(b) % 16 == 0 &&
                  reinterpret_cast<uintptr_t>(sfa) % 16 == 0 && reinterpret_cast<uintptr_t>(sfb) % 16 == 0,
              "NVFP4 operands and scale buffers must be 16-byte aligned");
  return SDC_OK;
}

int check_fp8_block(const uint8_t* a, const uint8_t* b, const float* sa, const float* sb, int64_t m, int64_t n,
                    int64_t k, const void* d) {
  int rc = check_dims(m, n, k);
  if (rc != SDC_OK) return rc;
  SDC_REQUIRE(a != nullptr && b != nullptr && sa != nullptr && sb != nullptr && d != nullptr,
              "block-scaled FP8 GEMM pointers must not be null");
  SDC_REQUIRE(k % 128 == 0, "block-scaled FP8 K must be a multiple of 128 (one scale per 128-wide block)");
  SDC_REQUIRE(reinterpret_cast<uintptr_t>(a) % 16 == 0 && reinterpret_cast<uintptr_t>(b) % 16 == 0 &&
                  reinterpret_cast<uintptr_t>(sa) % 4 == 0 && reinterpret_cast<uintptr_t>(sb) % 4 == 0,
              "block-scaled FP8 operands must be 16-byte aligned and scales 4-byte aligned");
  return SDC_OK;
}

int check_abft(int algorithm, const float* weights, int64_t m, int64_t n, int64_t row, int64_t col,
               int64_t bit, const float* observed, const int32_t* hit) {
  if (policy_channels(algorithm) == 0) return fail(SDC_ERR_UNKNOWN_ALGORITHM, "Unknown compiled ABFT algorithm ID");
  SDC_REQUIRE(weights != nullptr && observed != nullptr && hit != nullptr,
              "ABFT weights/observed/hit must not be null");
  SDC_REQUIRE((row == -1 && col == -1 && bit == -1) ||
                  (row >= 0 && row < m && col >= 0 && col < n && bit >= 0 && bit < 32),
              "ABFT fault must be all -1, or a valid output row/column and FP32 bit [0,31]");
  return SDC_OK;
}

GemmProblem make_problem(Kind kind, const uint8_t* a, const uint8_t* b, const uint8_t* sfa,
                         const uint8_t* sfb, int64_t m, int64_t n, int64_t k, const float* alpha,
                         bool bf16, void* d) {
  GemmProblem g{};
  g.kind = kind;
  g.a = a;
  g.b = b;
  g.sfa = sfa;
  g.sfb = sfb;
  g.m = m;
  g.n = n;
  g.k = k;
  g.alpha = alpha;
  g.out_bf16_rowmajor = bf16;
  g.d = d;
  g.channels = 0;
  g.fault_row = g.fault_col = g.fault_bit = -1;
  return g;
}

void set_abft(GemmProblem& g, int algorithm, const float* weights, int64_t row, int64_t col,
              int64_t bit, int32_t* nonfinite, float* observed, int32_t* hit, int64_t tile_n) {
  g.channels = policy_channels(algorithm);
  g.weights = weights;
  g.fault_row = row;
  g.fault_col = col;
  g.fault_bit = bit;
  g.nonfinite = nonfinite;
  g.observed = observed;
  g.hit = hit;
  g.padded_n = ceil_div(g.n, tile_n) * tile_n;
}

ReferenceProblem reference_problem(const GemmProblem& g, float* predicted, float* magnitude, int layout,
                                   void* workspace, size_t workspace_bytes) {
  ReferenceProblem r{};
  r.kind = g.kind;
  r.a = g.a;
  r.b = g.b;
  r.sfa = g.sfa;
  r.sfb = g.sfb;
  r.m = g.m;
  r.n = g.n;
  r.k = g.k;
  r.alpha = g.alpha;
  r.channels = g.channels;
  r.weights = g.weights;
  r.predicted = predicted;
  r.magnitude = magnitude;
  r.padded_n = g.padded_n;
  r.layout = layout;
  r.workspace = workspace;
  r.workspace_bytes = workspace_bytes;
  return r;
}

// Input-fused ABFT GEMM: TILE layout = per-tile projection, GEMM, then the
// propagation on CUDA cores; K-SLICE layout = one GEMM launch whose
// prediction warps compute the projection of A and the propagation, or, for
// a short M, the two standalone K-slice kernels and an observed-only GEMM.
int run_input_fused(GemmProblem g, float* predicted, float* magnitude, int layout, void* workspace,
                    size_t workspace_bytes, cudaStream_t stream) {
  SDC_REQUIRE(predicted != nullptr && magnitude != nullptr, "predicted/magnitude must not be null");
  const ReferenceProblem r = reference_problem(g, predicted, magnitude, layout, workspace, workspace_bytes);
  if (layout == SDC_LAYOUT_KSLICE) {
    int rc = check_problem(r);
    if (rc != SDC_OK) return rc;
    const KsliceScratch scratch = kslice_scratch(r);
    if (kslice_standalone(r)) {
      rc = check_current_device();
      if (rc != SDC_OK) return rc;
      rc = launch_kslice_standalone(r, scratch, stream);
      if (rc != SDC_OK) return rc;
      return launch_gemm(g, stream);  // q_full unset: observed-only epilogue
    }
    g.q_full = scratch.q_full;
    g.q_part = scratch.q_part;
    g.grid_sync = scratch.grid_sync;
    g.predicted = predicted;
    g.magnitude = magnitude;
    if (kslice_preproject(r)) {
      rc = check_current_device();
      if (rc != SDC_OK) return rc;
      rc = launch_kslice_projection(r, scratch, stream);
      if (rc != SDC_OK) return rc;
      g.q_ready = true;
      g.grid_sync = nullptr;  // no grid barriers in the launch
    }
    return launch_gemm(g, stream);
  }
  int rc = launch_projection(r, stream);
  if (rc != SDC_OK) return rc;
  rc = launch_gemm(g, stream);
  if (rc != SDC_OK) return rc;
  return launch_tile_propagate(r, stream);
}

}  // namespace
}  // namespace sdc

extern "C" {

int sdc_fp8_gemm(const uint8_t* a, const uint8_t* b_rows, int64_t m, int64_t n, int64_t k,
                 const float* alpha, float* d, sdc_stream_t stream) {
  using namespace sdc;
  int rc = check_fp8(a, b_rows, m, n, k, alpha, d);
  if (rc != SDC_OK) return rc;
  return launch_gemm(make_problem(Kind::kFp8, a, b_rows, nullptr, nullptr, m, n, k, alpha, false, d), stream);
}

int sdc_nvfp4_gemm(const uint8_t* a_packed, const uint8_t* b_packed, const uint8_t* sfa,
                   const uint8_t* sfb, int64_t m, int64_t n, int64_t k, const float* alpha,
                   uint16_t* d, sdc_stream_t stream) {
  using namespace sdc;
  int rc = check_nvfp4(a_packed, b_packed, sfa, sfb, m, n, k, alpha, d);
  if (rc != SDC_OK) return rc;
  return launch_gemm(make_problem(Kind::kNvf4, a_packed, b_packed, sfa, sfb, m, n, k, alpha, true, d), stream);
}

size_t sdc_abft_workspace_bytes(int algorithm, int64_t m, int64_t n, int64_t k, int reference_layout) {
  const int channels = sdc::policy_channels(algorithm);
  if (channels == 0) return 0;
  return sdc::reference_workspace_bytes(channels, m, n, k, reference_layout);
}

int sdc_abft_fp8_gemm(const uint8_t* a, const uint8_t* b_rows, int64_t m, int64_t n, int64_t k,
                      const float* alpha, int algorithm, const float* weights, int64_t row,
                      int64_t col, int64_t bit, int32_t* nonfinite, float* d, float* observed,
                      int32_t* hit, sdc_stream_t stream) {
  using namespace sdc;
  int rc = check_fp8(a, b_rows, m, n, k, alpha, d);
  if (rc == SDC_OK) rc = check_abft(algorithm, weights, m, n, row, col, bit, observed, hit);
  if (rc != SDC_OK) return rc;
  GemmProblem g = make_problem(Kind::kFp8, a, b_rows, nullptr, nullptr, m, n, k, alpha, false, d);
  set_abft(g, algorithm, weights, row, col, bit, nonfinite, observed, hit, 64);
  return launch_gemm(g, stream);
}

int sdc_abft_fp8_reference_gemm(const uint8_t* a, const uint8_t* b_rows, int64_t m, int64_t n,
                                int64_t k, const float* alpha, int algorithm, const float* weights,
                                int64_t row, int64_t col, int64_t bit, int32_t* nonfinite, float* d,
                                float* observed, int32_t* hit, float* predicted, float* magnitude,
                                int reference_layout, void* workspace, size_t workspace_bytes,
                                sdc_stream_t stream) {
  using namespace sdc;
  int rc = check_fp8(a, b_rows, m, n, k, alpha, d);
  if (rc == SDC_OK) rc = check_abft(algorithm, weights, m, n, row, col, bit, observed, hit);
  if (rc != SDC_OK) return rc;
  GemmProblem g = make_problem(Kind::kFp8, a, b_rows, nullptr, nullptr, m, n, k, alpha, false, d);
  set_abft(g, algorithm, weights, row, col, bit, nonfinite, observed, hit, 64);
  return run_input_fused(g, predicted, magnitude, reference_layout, workspace, workspace_bytes, stream);
}

int sdc_abft_nvfp4_gemm(const uint8_t* a_packed, const uint8_t* b_packed, const uint8_t* sfa,
                        const uint8_t* sfb, int64_t m, int64_t n, int64_t k, const float* alpha,
                        int algorithm, const float* weights, int64_t row, int64_t col, int64_t bit,
                        int32_t* nonfinite, uint16_t* d, float* observed, int32_t* hit,
                        sdc_stream_t stream) {
  using namespace sdc;
  int rc = check_nvfp4(a_packed, b_packed, sfa, sfb, m, n, k, alpha, d);
  if (rc == SDC_OK) rc = check_abft(algorithm, weights, m, n, row, col, bit, observed, hit);
  if (rc != SDC_OK) return rc;
  GemmProblem g = make_problem(Kind::kNvf4, a_packed, b_packed, sfa, sfb, m, n, k, alpha, true, d);
  set_abft(g, algorithm, weights, row, col, bit, nonfinite, observed, hit, 128);
  return launch_gemm(g, stream);
}

int sdc_abft_nvfp4_reference_gemm(const uint8_t* a_packed, const uint8_t* b_packed,
                                  const uint8_t* sfa, const uint8_t* sfb, int64_t m, int64_t n,
                                  int64_t k, const float* alpha, int algorithm,
                                  const float* weights, int64_t row, int64_t col, int64_t bit,
                                  int32_t* nonfinite, uint16_t* d, float* observed, int32_t* hit,
                                  float* predicted, float* magnitude, int reference_layout,
                                  void* workspace, size_t workspace_bytes, sdc_stream_t stream) {
  using namespace sdc;
  int rc = check_nvfp4(a_packed, b_packed, sfa, sfb, m, n, k, alpha, d);
  if (rc == SDC_OK) rc = check_abft(algorithm, weights, m, n, row, col, bit, observed, hit);
  if (rc != SDC_OK) return rc;
  GemmProblem g = make_problem(Kind::kNvf4, a_packed, b_packed, sfa, sfb, m, n, k, alpha, true, d);
  set_abft(g, algorithm, weights, row, col, bit, nonfinite, observed, hit, 128);
  return run_input_fused(g, predicted, magnitude, reference_layout, workspace, workspace_bytes, stream);
}

// ---- block-scaled FP8 (extension: no reference operator) ----

int sdc_fp8_block_gemm(const uint8_t* a, const uint8_t* b_rows, const float* scale_a, const float* scale_b,
                       int64_t m, int64_t n, int64_t k, uint16_t* d, sdc_stream_t stream) {
  using namespace sdc;
  int rc = check_fp8_block(a, b_rows, scale_a, scale_b, m, n, k, d);
  if (rc != SDC_OK) return rc;
  return launch_gemm(make_problem(Kind::kFp8Block, a, b_rows, reinterpret_cast<const uint8_t*>(scale_a),
                                  reinterpret_cast<const uint8_t*>(scale_b), m, n, k, nullptr, true, d),
                     stream);
}

int sdc_abft_fp8_block_gemm(const uint8_t* a, const uint8_t* b_rows, const float* scale_a,
                            const float* scale_b, int64_t m, int64_t n, int64_t k, int algorithm,
                            const float* weights, int64_t row, int64_t col, int64_t bit, int32_t* nonfinite,
                            uint16_t* d, float* observed, int32_t* hit, sdc_stream_t stream) {
  using namespace sdc;
  int rc = check_fp8_block(a, b_rows, scale_a, scale_b, m, n, k, d);
  if (rc == SDC_OK) rc = check_abft(algorithm, weights, m, n, row, col, bit, observed, hit);
  if (rc != SDC_OK) return rc;
  GemmProblem g = make_problem(Kind::kFp8Block, a, b_rows, reinterpret_cast<const uint8_t*>(scale_a),
                               reinterpret_cast<const uint8_t*>(scale_b), m, n, k, nullptr, true, d);
  set_abft(g, algorithm, weights, row, col, bit, nonfinite, observed, hit, 128);
  return launch_gemm(g, stream);
}

int sdc_abft_fp8_block_reference_gemm(const uint8_t* a, const uint8_t* b_rows, const float* scale_a,
                                      const float* scale_b, int64_t m, int64_t n, int64_t k, int algorithm,
                                      const float* weights, int64_t row, int64_t col, int64_t bit,
                                      int32_t* nonfinite, uint16_t* d, float* observed, int32_t* hit,
                                      float* predicted, float* magnitude, void* workspace,
                                      size_t workspace_bytes, sdc_stream_t stream) {
  using namespace sdc;
  int rc = check_fp8_block(a, b_rows, scale_a, scale_b, m, n, k, d);
  if (rc == SDC_OK) rc = check_abft(algorithm, weights, m, n, row, col, bit, observed, hit);
  if (rc != SDC_OK) return rc;
  GemmProblem g = make_problem(Kind::kFp8Block, a, b_rows, reinterpret_cast<const uint8_t*>(scale_a),
                               reinterpret_cast<const uint8_t*>(scale_b), m, n, k, nullptr, true, d);
  set_abft(g, algorithm, weights, row, col, bit, nonfinite, observed, hit, 128);
  return run_input_fused(g, predicted, magnitude, SDC_LAYOUT_KSLICE, workspace, workspace_bytes, stream);
}

// ---- row checksums (extension) ----

int sdc_abft_reference_gemm_rows(int kind, const uint8_t* a, const void* a_scales, const uint8_t* b_rows,
                                 const void* b_scales, int64_t m, int64_t n, int64_t k, const float* alpha,
                                 int algorithm, const float* weights, int64_t row, int64_t col, int64_t bit,
                                 int32_t* nonfinite, void* d, float* observed, int32_t* hit, float* predicted,
                                 float* magnitude, int reference_layout, float* row_observed, void* workspace,
                                 size_t workspace_bytes, sdc_stream_t stream) {
  using namespace sdc;
  SDC_REQUIRE(row_observed != nullptr, "row checksums need row_observed [ceil(N/64)][M]");
  int rc = SDC_OK;
  GemmProblem g{};
  int tile = 128;
  if (kind == SDC_KIND_FP8) {
    rc = check_fp8(a, b_rows, m, n, k, alpha, d);
    g = make_problem(Kind::kFp8, a, b_rows, nullptr, nullptr, m, n, k, alpha, false, d);
    tile = 64;
  } else if (kind == SDC_KIND_NVFP4) {
    const uint8_t* sfa = static_cast<const uint8_t*>(a_scales);
    const uint8_t* sfb = static_cast<const uint8_t*>(b_scales);
    rc = check_nvfp4(a, b_rows, sfa, sfb, m, n, k, alpha, d);
    g = make_problem(Kind::kNvf4, a, b_rows, sfa, sfb, m, n, k, alpha, true, d);
  } else if (kind == SDC_KIND_FP8_BLOCK) {
    const float* sa = static_cast<const float*>(a_scales);
    const float* sb = static_cast<const float*>(b_scales);
    rc = check_fp8_block(a, b_rows, sa, sb, m, n, k, d);
    g = make_problem(Kind::kFp8Block, a, b_rows, reinterpret_cast<const uint8_t*>(sa),
                     reinterpret_cast<const uint8_t*>(sb), m, n, k, nullptr, true, d);
    SDC_REQUIRE(reference_layout == SDC_LAYOUT_KSLICE, "block-scaled FP8 offers the K-slice layout only");
  } else {
    return fail(SDC_ERR_INVALID, "row checksums: kind must be SDC_KIND_FP8, SDC_KIND_NVFP4 or SDC_KIND_FP8_BLOCK");
  }
  if (rc == SDC_OK) rc = check_abft(algorithm, weights, m, n, row, col, bit, observed, hit);
  if (rc != SDC_OK) return rc;
  set_abft(g, algorithm, weights, row, col, bit, nonfinite, observed, hit, tile);
  g.row_observed = row_observed;
  return run_input_fused(g, predicted, magnitude, reference_layout, workspace, workspace_bytes, stream);
}

}  // extern "C"
