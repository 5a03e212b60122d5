// Internal interface of the tcgen05 GEMM kernels (FP8 e4m3 and NVFP4).
#pragma once

#include "common.cuh"

namespace sdc {

enum class Kind : int { kFp8 = 0, kNvf4 = 1 };

struct GemmProblem {
  Kind kind;
  const uint8_t* a;    // [M, K] e4m3 or [M, K/2] packed e2m1
  const uint8_t* b;    // [N, K] e4m3 or [N, K/2] packed e2m1
  const uint8_t* sfa;  // NVFP4 scale atoms of A
  const uint8_t* sfb;  // NVFP4 scale atoms of B
  int64_t m, n, k;
  const float* alpha;  // device scalar
  // Epilogue
  bool out_bf16_rowmajor;  // else fp32 column-major
  void* d;
  int channels;            // 0 = unprotected
  const float* weights;    // [C, M]
  int64_t fault_row, fault_col, fault_bit;
  int32_t* nonfinite;      // nullable
  float* observed;         // [C, Tm, Np]
  int32_t* hit;
  int64_t padded_n;
  // K-slice input prediction fused into the GEMM (all null: not fused).
  const float* q_full;     // [K][C][2], from launch_projection
  float* predicted;        // [C, Tm, Np]
  float* magnitude;
  // hit/nonfinite were already zeroed earlier on the stream.
  bool flags_zeroed;
  // Launch as a programmatic dependent of the kernel just before it on the
  // stream (the K-slice projection): only the prediction warps wait for it.
  bool dependent_launch;
};

// Launches the GEMM (and its fused epilogue) on `stream`. Zeroes hit/nonfinite
// first unless flags_zeroed. Returns an SDC_* status.
int launch_gemm(const GemmProblem& p, cudaStream_t stream);

// Input-side checksum partials (predicted, magnitude), reference layouts.
struct ReferenceProblem {
  Kind kind;
  const uint8_t* a;
  const uint8_t* b;
  const uint8_t* sfa;
  const uint8_t* sfb;
  int64_t m, n, k;
  const float* alpha;
  int channels;
  const float* weights;
  float* predicted;  // [C, Tm, Np]
  float* magnitude;
  int64_t padded_n;
  int layout;        // sdc_reference_layout
  void* workspace;
  size_t workspace_bytes;
};

size_t reference_workspace_bytes(int channels, int64_t m, int64_t n, int64_t k, int layout);
// Per-tile projections q[c][h][t][k] of A (and, for the K-slice layout, their
// ascending-tile sum q_full[k][c][h] at the end of the workspace). Must run
// before the GEMM when the prediction is fused into it.
int launch_projection(const ReferenceProblem& p, cudaStream_t stream);
// TILE layout: per-tile propagation against B on CUDA cores (after projection).
int launch_tile_propagate(const ReferenceProblem& p, cudaStream_t stream);
// Device pointer of q_full inside the workspace of a K-slice problem.
const float* kslice_q_full(const ReferenceProblem& p);

}  // namespace sdc
