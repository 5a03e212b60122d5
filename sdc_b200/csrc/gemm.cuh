// Internal interface of the tcgen05 GEMM kernels (FP8 e4m3 and NVFP4).
#pragma once

#include "common.cuh"

namespace sdc {

// kFp8Block: e4m3 codes with fp32 dequantisation scales per 1 x 128 block of
// A (sfa: float [M][K/128]) and per 128 x 128 block of B rows (sfb: float
// [ceil(N/128)][K/128]); bf16 row-major output.
// kBf16: bf16 operands (kind::f16 MMA, fp32 accumulation), bf16 row-major
// output; its protected form is the augmented GEMM (checksum rows of A as
// extra M-tiles, see GemmProblem::q).
enum class Kind : int { kFp8 = 0, kNvf4 = 1, kFp8Block = 2, kBf16 = 3 };
__host__ __device__ constexpr bool is_e4m3(Kind k) { return k == Kind::kFp8 || k == Kind::kFp8Block; }
// Bytes of one operand row of K elements.
__host__ __device__ constexpr int64_t row_bytes_of(Kind k, int64_t elems) {
  return k == Kind::kNvf4 ? elems / 2 : k == Kind::kBf16 ? 2 * elems : elems;
}

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
  // Augmented bf16 GEMM (kBf16 with channels > 0): q holds the bf16 checksum
  // rows of A, row t * C + c = bf16(w_c^T A over M-tile t), [aug_rows, K].
  // They run as extra M-tiles after the data tiles; their fp32 results are
  // written to `predicted`, and the data tiles' epilogue also writes the
  // output-side magnitude sum_rows |w_c v| to `magnitude`. tile_flags
  // (nullable, zeroed by launch_gemm): int32 [Tm, flag_cols] of bit 0 fault
  // applied, bit 1 non-finite output, per 128-column block.
  const uint8_t* q;
  int64_t aug_rows;
  int32_t* tile_flags;
  int64_t flag_cols;
  // The caller zeroed hit and tile_flags on this stream already (launch_gemm
  // then issues no memsets for them).
  bool status_zeroed;
  // Row checksums (nullable): fp32 [ceil(N/64)][M] row sums of the output
  // per 64-column block, after the fault (FP8 and NVFP4 kinds).
  float* row_observed;
  // q_full already holds the projection of A (computed by the standalone
  // projection kernels before this launch): the prediction warps go straight
  // to the per-tile prediction.
  bool q_ready;
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
  float* q_part;        // [ceil(M / 128)][K_pad][C][2]
};
KsliceScratch kslice_scratch(const ReferenceProblem& p);
// NVFP4 with a short M (rows <= kStandaloneMaxRows) and N >= 16 M, unless
// kslice_preproject takes it: the projection and the K-slice prediction run
// as two kernels spread over the whole GPU before an observed-only GEMM, with
// bit-identical partials (kslice.cu); otherwise they stay inside the GEMM,
// behind its tiles.
constexpr int64_t kStandaloneMaxRows = 4096;
bool kslice_standalone(const ReferenceProblem& p);
int launch_kslice_standalone(const ReferenceProblem& p, const KsliceScratch& s, cudaStream_t stream);
// The projection of A alone, by the standalone kernels, into s.q_full (the
// partials bit-identical to the in-GEMM projection's). Chosen by
// kslice_preproject when the GEMM has too few tiles per CTA to hide the
// in-GEMM projection behind its mainloop.
bool kslice_preproject(const ReferenceProblem& p);
int launch_kslice_projection(const ReferenceProblem& p, const KsliceScratch& s, cudaStream_t stream);

}  // namespace sdc
