// Augmented BF16 ABFT GEMM on sm_100a (the reference's augmented reference
// mode, src/cutlass_gemm/csrc/abft/fp32_bf16/bf16_augmented.{h,cu}).
//
// The checksum of a 128-row M-tile t is carried as extra GEMM rows: for each
// channel c, q[t * C + c][k] = bf16(sum over the tile's rows of w_c[r] *
// A[r][k]) (fp32 sum, one rounding to bf16). All tiles' checksum rows are
// packed densely into ceil(C * Tm / 128) extra M-tiles of the same tcgen05
// GEMM (gemm.cu, Kind::kBf16), so the tensor cores compute
//   predicted[c][t][n] = sum_k q[t * C + c][k] * B[n][k]   (fp32)
// at C / 128 extra rows per data row, instead of padding every 128-row tile
// with C rows as a per-tile MMA fragment would. The data tiles' epilogue forms
// observed = sum_rows w_c v and the output-side magnitude sum_rows |w_c v|
// (the augmented mode's threshold scale), after the optional fault XOR.
//
// Fixed summation order of the encoding (mirrored by the C oracle): per
// (tile, channel, k), eight fp32 fma chains over 16-row segments (rows
// ascending), added in ascending segment order, one rounding to bf16.
#include <algorithm>

#include "gemm.cuh"

namespace sdc {
namespace {

constexpr int kSegments = 8;                   // warps per block: row segments of a tile
constexpr int kSegmentRows = 128 / kSegments;  // 16 rows per segment
constexpr int kEncodeThreads = 32 * kSegments;
constexpr int kEncodeK = 8;                    // k per lane: one 16-byte bf16 load per row
constexpr int kBlockK = 32 * kEncodeK;         // 256 columns per block

// Grid (ceil(K / 256), Tm), 256 threads. Warp s forms, for the block's 256
// columns, the fp32 fma chain over rows [16 s, 16 s + 16) of the tile in
// ascending order (its 16 row loads all in flight at once); the eight
// segment sums are then added in ascending segment order (an empty segment
// adds +0) and rounded once to bf16. Blocks x == 0 also write the tile's
// weights as fp32 for the GEMM epilogue (when w32 is not null) and zero the
// tile's status words (tile_flags row t, and hit once) that the GEMM ORs into.
template <int C>
__global__ void __launch_bounds__(kEncodeThreads)
    augment_encode(const uint16_t* a, int64_t m, int64_t k, const uint16_t* w, uint16_t* q, float* w32,
                   int32_t* tile_flags, int64_t flag_cols, int32_t* hit) {
  __shared__ float part[kSegments][C][kBlockK];
  // The GEMM launched next may begin its data tiles now (it waits for this
  // grid before it reads anything this kernel writes).
  griddep_launch_dependents();
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int64_t t = blockIdx.y;
  const int64_t row0 = t * 128;
  const int rows = static_cast<int>(std::min<int64_t>(128, m - row0));
  if (blockIdx.x == 0) {
    if (w32 != nullptr) {
      for (int i = threadIdx.x; i < C * rows; i += kEncodeThreads) {
        const int64_t c = i / rows, r = row0 + i % rows;
        w32[c * m + r] = bf16_bits_to_float(w[c * m + r]);
      }
    }
    if (tile_flags != nullptr) {
      for (int64_t i = threadIdx.x; i < flag_cols; i += kEncodeThreads) tile_flags[t * flag_cols + i] = 0;
    }
    if (hit != nullptr && t == 0 && threadIdx.x == 0) *hit = 0;
  }
  const int64_t kb = static_cast<int64_t>(blockIdx.x) * kBlockK;
  const int64_t k0 = kb + lane * kEncodeK;
  // acc[c][j]: channel c, columns (k0 + 2j, k0 + 2j + 1) as one f32x2 lane pair.
  float2 acc[C][kEncodeK / 2];
#pragma unroll
  for (int c = 0; c < C; ++c)
#pragma unroll
    for (int j = 0; j < kEncodeK / 2; ++j) acc[c][j] = make_float2(0.f, 0.f);
  const int seg0 = warp * kSegmentRows;
  if (k0 < k) {  // K % 8 == 0: a lane's 8 columns are all inside or all outside
    uint4 raw[kSegmentRows];
    float wv[kSegmentRows][C];
#pragma unroll
    for (int i = 0; i < kSegmentRows; ++i) {
      const bool in = seg0 + i < rows;
      const int64_t r = row0 + seg0 + i;
      raw[i] = in ? __ldg(reinterpret_cast<const uint4*>(a + r * k + k0)) : make_uint4(0, 0, 0, 0);
#pragma unroll
      for (int c = 0; c < C; ++c) wv[i][c] = in ? bf16_bits_to_float(__ldg(w + c * m + r)) : 0.f;
    }
#pragma unroll
    for (int i = 0; i < kSegmentRows; ++i) {
      if (seg0 + i >= rows) break;  // rows past M are not terms (keeps a -0 chain -0)
      const uint32_t words[4] = {raw[i].x, raw[i].y, raw[i].z, raw[i].w};
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const float2 v = make_float2(__uint_as_float(words[j] << 16), __uint_as_float(words[j] & 0xFFFF0000u));
#pragma unroll
        for (int c = 0; c < C; ++c) acc[c][j] = fma2(make_float2(wv[i][c], wv[i][c]), v, acc[c][j]);
      }
    }
  }
#pragma unroll
  for (int c = 0; c < C; ++c) {
    float4* dst = reinterpret_cast<float4*>(&part[warp][c][lane * kEncodeK]);
    dst[0] = make_float4(acc[c][0].x, acc[c][0].y, acc[c][1].x, acc[c][1].y);
    dst[1] = make_float4(acc[c][2].x, acc[c][2].y, acc[c][3].x, acc[c][3].y);
  }
  __syncthreads();
  // Column pairs: (channel, pair) = i over C * 128; segments added ascending.
  for (int i = threadIdx.x; i < C * (kBlockK / 2); i += kEncodeThreads) {
    const int c = i / (kBlockK / 2), col = 2 * (i % (kBlockK / 2));
    if (kb + col >= k) continue;
    float lo = part[0][c][col], hi = part[0][c][col + 1];
#pragma unroll
    for (int seg = 1; seg < kSegments; ++seg) {
      lo = lo + part[seg][c][col];
      hi = hi + part[seg][c][col + 1];
    }
    *reinterpret_cast<uint32_t*>(q + (t * C + c) * k + kb + col) = bf16x2_bits(lo, hi);
  }
}

constexpr size_t kAlign = 256;
size_t align_up(size_t bytes) { return (bytes + kAlign - 1) / kAlign * kAlign; }

struct AugmentedScratch {
  uint16_t* q;    // [C * Tm, K] bf16
  float* w32;     // [C, M] fp32
  int32_t* hit;   // 1 word, used when the caller passes none
};

size_t scratch_bytes(int channels, int64_t m, int64_t k) {
  const int64_t tiles = ceil_div(m, 128);
  return align_up(static_cast<size_t>(channels) * tiles * k * 2) + align_up(static_cast<size_t>(channels) * m * 4) +
         kAlign;
}

AugmentedScratch carve(void* workspace, int channels, int64_t m, int64_t k) {
  const int64_t tiles = ceil_div(m, 128);
  uint8_t* base = static_cast<uint8_t*>(workspace);
  AugmentedScratch s{};
  s.q = reinterpret_cast<uint16_t*>(base);
  base += align_up(static_cast<size_t>(channels) * tiles * k * 2);
  s.w32 = reinterpret_cast<float*>(base);
  base += align_up(static_cast<size_t>(channels) * m * 4);
  s.hit = reinterpret_cast<int32_t*>(base);
  return s;
}

int check_bf16(const uint16_t* a, const uint16_t* b, int64_t m, int64_t n, int64_t k, const void* d) {
  for (int64_t v : {m, n, k}) {
    if (v <= 0 || v > static_cast<int64_t>(INT32_MAX) - 256) {
      return fail(SDC_ERR_INVALID, "Matrix dimensions must be positive and allow int32 tile padding");
    }
  }
  SDC_REQUIRE(a != nullptr && b != nullptr && d != nullptr, "BF16 GEMM pointers must not be null");
  SDC_REQUIRE(k % 8 == 0, "BF16 K must be a multiple of 8 (16-byte operand rows)");
  SDC_REQUIRE(reinterpret_cast<uintptr_t>(a) % 16 == 0 && reinterpret_cast<uintptr_t>(b) % 16 == 0,
              "BF16 operands must be 16-byte aligned");
  return SDC_OK;
}

GemmProblem bf16_problem(const uint16_t* a, const uint16_t* b, int64_t m, int64_t n, int64_t k, uint16_t* d) {
  GemmProblem g{};
  g.kind = Kind::kBf16;
  g.a = reinterpret_cast<const uint8_t*>(a);
  g.b = reinterpret_cast<const uint8_t*>(b);
  g.m = m;
  g.n = n;
  g.k = k;
  g.out_bf16_rowmajor = true;
  g.d = d;
  g.fault_row = g.fault_col = g.fault_bit = -1;
  return g;
}

int launch_encode(const uint16_t* a, int64_t m, int64_t k, int channels, const uint16_t* weights, uint16_t* q,
                  float* w32, int32_t* tile_flags, int64_t flag_cols, int32_t* hit, cudaStream_t stream) {
  const dim3 grid(static_cast<unsigned>(ceil_div(k, kBlockK)), static_cast<unsigned>(ceil_div(m, 128)));
  if (channels == 2) {
    augment_encode<2><<<grid, kEncodeThreads, 0, stream>>>(a, m, k, weights, q, w32, tile_flags, flag_cols, hit);
  } else {
    augment_encode<1><<<grid, kEncodeThreads, 0, stream>>>(a, m, k, weights, q, w32, tile_flags, flag_cols, hit);
  }
  SDC_CUDA_CHECK(cudaGetLastError());
  return SDC_OK;
}

}  // namespace
}  // namespace sdc

extern "C" {

int sdc_bf16_gemm(const uint16_t* a, const uint16_t* b_rows, int64_t m, int64_t n, int64_t k, uint16_t* d,
                  sdc_stream_t stream) {
  using namespace sdc;
  int rc = check_bf16(a, b_rows, m, n, k, d);
  if (rc != SDC_OK) return rc;
  return launch_gemm(bf16_problem(a, b_rows, m, n, k, d), stream);
}

int sdc_abft_augment_encode(const uint16_t* a, int64_t m, int64_t k, int algorithm, const uint16_t* weights,
                            uint16_t* q, sdc_stream_t stream) {
  using namespace sdc;
  const int channels = policy_channels(algorithm);
  if (channels == 0) return fail(SDC_ERR_UNKNOWN_ALGORITHM, "Unknown compiled ABFT algorithm ID");
  for (int64_t v : {m, k}) {
    if (v <= 0 || v > static_cast<int64_t>(INT32_MAX) - 256) {
      return fail(SDC_ERR_INVALID, "Matrix dimensions must be positive and allow int32 tile padding");
    }
  }
  SDC_REQUIRE(a != nullptr && weights != nullptr && q != nullptr, "Augmented encode pointers must not be null");
  SDC_REQUIRE(k % 8 == 0, "BF16 K must be a multiple of 8 (16-byte operand rows)");
  SDC_REQUIRE(reinterpret_cast<uintptr_t>(a) % 16 == 0 && reinterpret_cast<uintptr_t>(q) % 16 == 0,
              "Augmented encode A and q must be 16-byte aligned");
  int rc = check_current_device();
  if (rc != SDC_OK) return rc;
  return launch_encode(a, m, k, channels, weights, q, nullptr, nullptr, 0, nullptr, stream);
}

size_t sdc_abft_augmented_workspace_bytes(int algorithm, int64_t m, int64_t k) {
  const int channels = sdc::policy_channels(algorithm);
  if (channels == 0 || m <= 0 || k <= 0) return 0;
  return sdc::scratch_bytes(channels, m, k);
}

int sdc_abft_bf16_augmented_gemm(const uint16_t* a, const uint16_t* b_rows, int64_t m, int64_t n, int64_t k,
                                 int algorithm, const uint16_t* weights, int64_t row, int64_t col, int64_t bit,
                                 uint16_t* d, float* observed, float* predicted, float* magnitude, int32_t* hit,
                                 int32_t* tile_flags, void* workspace, size_t workspace_bytes, sdc_stream_t stream) {
  using namespace sdc;
  const int channels = policy_channels(algorithm);
  if (channels == 0) return fail(SDC_ERR_UNKNOWN_ALGORITHM, "Unknown compiled ABFT algorithm ID");
  int rc = check_bf16(a, b_rows, m, n, k, d);
  if (rc != SDC_OK) return rc;
  SDC_REQUIRE(weights != nullptr && observed != nullptr && predicted != nullptr && magnitude != nullptr,
              "Augmented ABFT weights/observed/predicted/magnitude must not be null");
  SDC_REQUIRE((row == -1 && col == -1 && bit == -1) ||
                  (row >= 0 && row < m && col >= 0 && col < n && bit >= 0 && bit < 32),
              "Augmented ABFT fault must be all -1, or a valid row/column and FP32 bit 0..31");
  const size_t need = scratch_bytes(channels, m, k);
  if (workspace == nullptr || workspace_bytes < need || reinterpret_cast<uintptr_t>(workspace) % 256 != 0) {
    return fail(SDC_ERR_WORKSPACE, "Augmented ABFT workspace too small or not 256-byte aligned");
  }
  const AugmentedScratch s = carve(workspace, channels, m, k);
  const int64_t tiles = ceil_div(m, 128);
  // The encode kernel also zeroes hit and tile_flags (no memset launches).
  rc = launch_encode(a, m, k, channels, weights, s.q, s.w32, tile_flags, ceil_div(n, 128),
                     hit != nullptr ? hit : s.hit, stream);
  if (rc != SDC_OK) return rc;
  GemmProblem g = bf16_problem(a, b_rows, m, n, k, d);
  g.channels = channels;
  g.weights = s.w32;
  g.fault_row = row;
  g.fault_col = col;
  g.fault_bit = bit;
  g.observed = observed;
  g.predicted = predicted;
  g.magnitude = magnitude;
  g.hit = hit != nullptr ? hit : s.hit;
  g.padded_n = ceil_div(n, 128) * 128;
  g.q = reinterpret_cast<const uint8_t*>(s.q);
  g.aug_rows = channels * tiles;
  g.tile_flags = tile_flags;
  g.flag_cols = ceil_div(n, 128);
  g.status_zeroed = true;
  return launch_gemm(g, stream);
}

}  // extern "C"
