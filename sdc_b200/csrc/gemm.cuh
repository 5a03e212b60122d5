// Internal interface of the tcgen05 GEMM kernels (FP8 e4m3 and NVFP4).
#pragma once

#include "common.cuh"

namespace sdc {

// kFp8Block: e4m3 codes with fp32 dequantisation scales per 1 x 128 block of
// A (sfa: float [M][K/128]) and per 128 x 128 block of B rows (sfb: float
// [ceil(N/128)][K/128]); bf16 row-major output.
enum class Kind : int { kFp8 = 0, kNvf4 = 1, kFp8Block = 2 };
__host__ __device__ constexpr bool is_e4m3(Kind k) { return k != Kind::kNvf4; }

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
  // Scratch from kslice_scratch(): q_full [K_pad][C][2], per-band partials
  // and the grid-barrier counter (zeroed by launch_gemm).
  float* q_full;
  float* q_part;
  uint32_t* grid_sync;
  float* predicted;        // [C, Tm, Np]
  float* magnitude;
};

// Launches the GEMM (and its fused epilogue) on `stream`. Zeroes hit/nonfinite
// first. Returns an SDC_* status. A launch that gave up a bounded wait sets bit
// 1 of `hit` (and `nonfinite` when given), which finalize reports as detected.
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
// Checks the layout id and the workspace size/alignment of `p`.
int check_problem(const ReferenceProblem& p);
// TILE layout: per-tile projections q[c][h][t][k] of A (before the GEMM) and
// their propagation against B on CUDA cores (after it).
int launch_projection(const ReferenceProblem& p, cudaStream_t stream);
int launch_tile_propagate(const ReferenceProblem& p, cudaStream_t stream);
// K-slice layout: the GEMM's scratch inside the workspace.
struct KsliceScratch {
  uint32_t* grid_sync;  // 256 bytes, zeroed by launch_gemm
  float* q_full;        // [K_pad][C][2]
  float* q_part;        // [ceil(M / 512)][K_pad][C][2]
};
KsliceScratch kslice_scratch(const ReferenceProblem& p);

}  // namespace sdc
