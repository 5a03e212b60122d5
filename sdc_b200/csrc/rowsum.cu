// Row checksums and two-dimensional localisation (extension; the reference
// checks column sums only and locates with the two-channel ratio).
//
// The epilogue of the GEMM (gemm.cu) forms the row sums of the fp32 output
// C = alpha * A B^T per 64-column block; this file forms their input-side
// prediction and decides:
//
//   u = e^T B, u_abs = e^T |B|          projection of the B rows with unit
//                                       weights (launch_projection_sums, the
//                                       column checksums' own projection code)
//   predicted_rows[m] = alpha * A[m] . u,   magnitude_rows[m] = |alpha| * |A[m]| . u_abs
//   residual_rows[m] = sum of the row's 64-column blocks (ascending) - predicted
//   threshold_rows[m] = atol + rtol * magnitude (no FMA), as for the columns
//
// A single faulty element (r, c) changes row r's sum and column c's sums by
// the same amount, so one failing row and one failing column locate it
// exactly, however small the error is next to the ratio locator's tolerance.
//
// Fixed summation orders (restated by oracle/cref.c): u as the K-slice
// projection (128-row bands, 8 row lanes, pairwise lane combine, bands
// ascending); A[m] . u by one warp per row: lane j runs the fma chain over the
// 16-element groups g = j, j + 32, ... (k ascending), the lanes combine by a
// butterfly (xor 16, 8, 4, 2, 1); a row block sum runs its 64 columns in
// ascending order from +0.
#include <algorithm>
#include <atomic>
#include <cfloat>
#include <mutex>

#include "kslice.cuh"

namespace sdc {
namespace {

constexpr int kRowWarps = 8;       // warps per block of the row prediction
constexpr int kRowsPerWarp = 4;    // rows per warp (their chains interleave)
constexpr int kPanelGroups = 32;   // 16-element groups per staged panel of u (512 k)
constexpr int kPanelStride = 33;   // float2 per panel row e (32 groups + 1 pad)
constexpr int kPanelFloat2 = 16 * kPanelStride;
constexpr int kMaxStagedPanels = 48;  // 48 * 528 * 8 B = 198 KiB of shared memory
constexpr int kLocate2dThreads = 64;  // small blocks: the rows spread over every SM
constexpr int kLocate2dBlocks = 4 * 148;
constexpr int kLocateBatch = 32;  // row blocks loaded ahead of their adds
constexpr int kBlockState = 5;    // per block: failing rows, first row, status bits, failing columns, first column
constexpr unsigned kRowFailed = 1u;
constexpr unsigned kRowNonfinite = 2u;

// The raw bytes of one row's 16-element group: codes (FP8: 16 bytes; NVFP4:
// 8 bytes in x, y) and the scale (block-scaled FP8: the fp32 block scale;
// NVFP4: the e4m3 scale byte), loaded ahead of their use.
struct GroupRaw {
  uint4 codes;
  uint32_t scale;
};

template <Kind KIND>
__device__ __forceinline__ GroupRaw load_group(const uint8_t* a, const float* sa, const uint8_t* sfa, int64_t k,
                                               int64_t k_blocks, int64_t row, int64_t k0, bool in) {
  GroupRaw raw{make_uint4(0, 0, 0, 0), 0u};
  if (!in) return raw;
  if constexpr (is_e4m3(KIND)) {
    raw.codes = __ldg(reinterpret_cast<const uint4*>(a + row * k + k0));
    if constexpr (KIND == Kind::kFp8Block) raw.scale = __float_as_uint(__ldg(sa + row * k_blocks + (k0 >> 7)));
  } else {
    const uint2 u = __ldg(reinterpret_cast<const uint2*>(a + row * (k / 2) + k0 / 2));
    raw.codes = make_uint4(u.x, u.y, 0, 0);
    const int64_t k_atoms = (k + 63) / 64;
    const int64_t off =
        ((row >> 7) * k_atoms + (k0 >> 6)) * 512 + (row & 31) * 16 + ((row >> 5) & 3) * 4 + ((k0 >> 4) & 3);
    raw.scale = __ldg(sfa + off);
  }
  return raw;
}

// Elements 8h .. 8h + 7 of a loaded group, decoded (times the block scale).
template <Kind KIND>
__device__ __forceinline__ void decode_half(const GroupRaw& raw, int h, float (&v)[8]) {
  if constexpr (is_e4m3(KIND)) {
    const uint32_t w0 = h == 0 ? raw.codes.x : raw.codes.z, w1 = h == 0 ? raw.codes.y : raw.codes.w;
    const uint32_t words[2] = {w0, w1};
#pragma unroll
    for (int j = 0; j < 2; ++j) {
      const float2 lo = e4m3x2_to_float2(words[j] & 0xFFFFu), hi = e4m3x2_to_float2(words[j] >> 16);
      v[4 * j] = lo.x;
      v[4 * j + 1] = lo.y;
      v[4 * j + 2] = hi.x;
      v[4 * j + 3] = hi.y;
    }
    if constexpr (KIND == Kind::kFp8Block) {
      const float scale = __uint_as_float(raw.scale);
#pragma unroll
      for (int e = 0; e < 8; ++e) v[e] = __fmul_rn(v[e], scale);
    }
  } else {
    e2m1x8_to_float(h == 0 ? raw.codes.x : raw.codes.y, v);
    const float scale = decode_e4m3(raw.scale);
#pragma unroll
    for (int e = 0; e < 8; ++e) v[e] = __fmul_rn(v[e], scale);
  }
}

// predicted_rows[m] = alpha * A[m] . u and magnitude_rows[m] = |alpha| *
// |A[m]| . u_abs, with u as [K_pad][2] (value, abs). A warp holds
// kRowsPerWarp rows; lane j of the warp runs each row's fma chain over the
// 16-element groups g = j, j + 32, ... (k ascending) and the lanes combine by
// a butterfly. u is staged in shared memory in panels of 512 k (32 groups):
// panel[e][g_local] with a padded row, so that the 32 lanes reading element e
// of their groups touch consecutive words. When K is longer than the staged
// chunk, the block walks the chunks for each tile of rows and the rows'
// chains carry across chunks, in the same order. The next panel's bytes are
// loaded while the current panel is summed.
template <Kind KIND>
__global__ void __launch_bounds__(32 * kRowWarps, KIND == Kind::kNvf4 ? 2 : 3)
    row_predict(const uint8_t* a, const float* sa, const uint8_t* sfa, int64_t m, int64_t k, const float* u,
                const float* alpha, float* predicted, float* magnitude, int chunk_panels) {
  extern __shared__ float2 staged_u[];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int64_t groups = k / 16;  // K % 16 == 0
  const int64_t k_blocks = k / 128;
  const int64_t panels = (groups + kPanelGroups - 1) / kPanelGroups;
  const int64_t chunks = (panels + chunk_panels - 1) / chunk_panels;
  constexpr int64_t kTileRows = kRowWarps * kRowsPerWarp;
  const int64_t tiles = (m + kTileRows - 1) / kTileRows;
  const float2* u2 = reinterpret_cast<const float2*>(u);
  for (int64_t tile = blockIdx.x; tile < tiles; tile += gridDim.x) {
    const int64_t row0 = tile * kTileRows + warp * kRowsPerWarp;
    float acc[kRowsPerWarp], acc_m[kRowsPerWarp];
#pragma unroll
    for (int r = 0; r < kRowsPerWarp; ++r) acc[r] = acc_m[r] = 0.f;
    for (int64_t c = 0; c < chunks; ++c) {
      const int64_t p0 = c * chunk_panels, p1 = min(panels, p0 + chunk_panels);
      GroupRaw cur[kRowsPerWarp];
      {
        const int64_t g = p0 * kPanelGroups + lane;
#pragma unroll
        for (int r = 0; r < kRowsPerWarp; ++r) {
          cur[r] = load_group<KIND>(a, sa, sfa, k, k_blocks, row0 + r, g * 16, row0 + r < m && g < groups);
        }
      }
      if (chunks > 1 || tile == blockIdx.x) {
        __syncthreads();
        const int64_t count = (p1 - p0) * kPanelGroups * 16;
        constexpr int kFillBatch = 8;
        for (int64_t base = threadIdx.x; base < count; base += kFillBatch * 32 * kRowWarps) {
          float2 t[kFillBatch];
#pragma unroll
          for (int j = 0; j < kFillBatch; ++j) {
            const int64_t i = base + static_cast<int64_t>(j) * 32 * kRowWarps;
            const int64_t kk = p0 * kPanelGroups * 16 + i;
            t[j] = i < count && kk < k ? __ldg(u2 + kk) : make_float2(0.f, 0.f);
          }
#pragma unroll
          for (int j = 0; j < kFillBatch; ++j) {
            const int64_t i = base + static_cast<int64_t>(j) * 32 * kRowWarps;
            if (i < count) {
              const int64_t pl = i / (kPanelGroups * 16);
              const int gl = static_cast<int>((i >> 4) & (kPanelGroups - 1)), e = static_cast<int>(i & 15);
              staged_u[pl * kPanelFloat2 + e * kPanelStride + gl] = t[j];
            }
          }
        }
        __syncthreads();
      }
      for (int64_t p = p0; p < p1; ++p) {
        const int64_t g = p * kPanelGroups + lane;
        GroupRaw next[kRowsPerWarp];
        const int64_t gn = g + kPanelGroups;
#pragma unroll
        for (int r = 0; r < kRowsPerWarp; ++r) {
          next[r] = load_group<KIND>(a, sa, sfa, k, k_blocks, row0 + r, gn * 16,
                                     p + 1 < p1 && row0 + r < m && gn < groups);
        }
        if (g < groups) {
          const float2* panel = staged_u + (p - p0) * kPanelFloat2 + lane;
#pragma unroll
          for (int h = 0; h < 2; ++h) {
            float v[kRowsPerWarp][8];
#pragma unroll
            for (int r = 0; r < kRowsPerWarp; ++r) decode_half<KIND>(cur[r], h, v[r]);
#pragma unroll
            for (int e = 0; e < 8; ++e) {
              const float2 uk = panel[(8 * h + e) * kPanelStride];
#pragma unroll
              for (int r = 0; r < kRowsPerWarp; ++r) {
                acc[r] = fmaf(v[r][e], uk.x, acc[r]);
                acc_m[r] = fmaf(fabsf(v[r][e]), uk.y, acc_m[r]);
              }
            }
          }
        }
#pragma unroll
        for (int r = 0; r < kRowsPerWarp; ++r) cur[r] = next[r];
      }
    }
    const float al = alpha != nullptr ? __ldg(alpha) : 1.f;
#pragma unroll
    for (int r = 0; r < kRowsPerWarp; ++r) {
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) {
        acc[r] = __fadd_rn(acc[r], __shfl_xor_sync(0xffffffffu, acc[r], o));
        acc_m[r] = __fadd_rn(acc_m[r], __shfl_xor_sync(0xffffffffu, acc_m[r], o));
      }
      if (lane == 0 && row0 + r < m) {
        predicted[row0 + r] = __fmul_rn(al, acc[r]);
        magnitude[row0 + r] = __fmul_rn(fabsf(al), acc_m[r]);
      }
    }
  }
}

struct Locate2dArgs {
  const float* row_observed;   // [row_blocks][m]
  int64_t row_blocks;
  const float* predicted;      // [m]
  const float* magnitude;      // [m]
  int64_t m;
  float atol, rtol;
  const float* col_residual;   // [C][n]
  const float* col_threshold;  // [C][n]
  int channels;
  int64_t n;
  const uint8_t* col_flags;    // finalize flags: [0] detected, [1] nonfinite
  float* row_residual;         // [m], nullable
  float* row_threshold;        // [m], nullable
  int64_t* location;           // [2]
  uint8_t* located;            // [1]
  uint8_t* row_flags;          // [2]: a row failed, a row was non-finite
  int64_t* block_state;        // [gridDim][kBlockState]
  uint32_t* ticket;
};

constexpr int kTicketSlots = 1024;
static __device__ uint32_t g_locate2d_tickets[kTicketSlots];

__device__ __forceinline__ void block_reduce(int64_t& count, int64_t& first, unsigned& bits) {
  for (int o = 16; o > 0; o >>= 1) {
    count += __shfl_xor_sync(0xffffffffu, count, o);
    first = min(first, __shfl_xor_sync(0xffffffffu, first, o));
    bits |= __shfl_xor_sync(0xffffffffu, bits, o);
  }
  __shared__ int64_t s_count[kLocate2dThreads / 32], s_first[kLocate2dThreads / 32];
  __shared__ unsigned s_bits[kLocate2dThreads / 32];
  const int warp = threadIdx.x >> 5;
  if ((threadIdx.x & 31) == 0) {
    s_count[warp] = count;
    s_first[warp] = first;
    s_bits[warp] = bits;
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    count = 0;
    first = INT64_MAX;
    bits = 0;
    for (int w = 0; w < kLocate2dThreads / 32; ++w) {
      count += s_count[w];
      first = min(first, s_first[w]);
      bits |= s_bits[w];
    }
  }
  __syncthreads();
}

// Row residuals and thresholds, and the failing columns (any channel over
// its threshold, the finalize's rule), both grid-stride; the last block to
// finish combines the blocks' counts and decides: exactly one failing row and
// one failing column with nothing non-finite locate the element.
__global__ void __launch_bounds__(kLocate2dThreads) locate2d(Locate2dArgs p) {
  int64_t count = 0, first = INT64_MAX;
  unsigned bits = 0;
  const int64_t stride = static_cast<int64_t>(gridDim.x) * kLocate2dThreads;
  for (int64_t row = static_cast<int64_t>(blockIdx.x) * kLocate2dThreads + threadIdx.x; row < p.m; row += stride) {
    // The row's blocks in ascending order; loads batched ahead of the adds.
    float sum = 0.f;
    int64_t b = 0;
    for (; b + kLocateBatch <= p.row_blocks; b += kLocateBatch) {
      float x[kLocateBatch];
#pragma unroll
      for (int i = 0; i < kLocateBatch; ++i) x[i] = __ldg(p.row_observed + (b + i) * p.m + row);
#pragma unroll
      for (int i = 0; i < kLocateBatch; ++i) sum = __fadd_rn(sum, x[i]);
    }
    for (; b < p.row_blocks; ++b) sum = __fadd_rn(sum, __ldg(p.row_observed + b * p.m + row));
    const float pred = p.predicted[row], mag = p.magnitude[row];
    const float residual = __fsub_rn(sum, pred);
    const float threshold = __fadd_rn(p.atol, __fmul_rn(p.rtol, mag));
    const bool nonfinite = !isfinite(sum) || !isfinite(pred) || !isfinite(mag) || !isfinite(residual) ||
                           !isfinite(threshold);
    if (nonfinite) bits |= kRowNonfinite;
    if (nonfinite || threshold < 0.f || fabsf(residual) > threshold) {
      bits |= kRowFailed;
      ++count;
      first = min(first, row);
    }
    if (p.row_residual != nullptr) p.row_residual[row] = residual;
    if (p.row_threshold != nullptr) p.row_threshold[row] = threshold;
  }
  int64_t cols = 0, col_first = INT64_MAX;
  unsigned unused = 0;
  for (int64_t col = static_cast<int64_t>(blockIdx.x) * kLocate2dThreads + threadIdx.x; col < p.n; col += stride) {
    bool failed = false;
    for (int c = 0; c < p.channels; ++c) {
      failed |= fabsf(__ldg(p.col_residual + c * p.n + col)) > __ldg(p.col_threshold + c * p.n + col);
    }
    if (failed) {
      ++cols;
      col_first = min(col_first, col);
    }
  }
  block_reduce(count, first, bits);
  block_reduce(cols, col_first, unused);
  __shared__ bool last;
  if (threadIdx.x == 0) {
    int64_t* state = p.block_state + blockIdx.x * kBlockState;
    state[0] = count;
    state[1] = first;
    state[2] = static_cast<int64_t>(bits);
    state[3] = cols;
    state[4] = col_first;
    __threadfence();
    last = atomicAdd(p.ticket, 1u) == gridDim.x - 1;
  }
  __syncthreads();
  if (!last) return;
  __threadfence();
  int64_t rows = 0, row_first = INT64_MAX, all_cols = 0, all_col_first = INT64_MAX;
  unsigned row_bits = 0;
  for (int64_t i = threadIdx.x; i < gridDim.x; i += kLocate2dThreads) {
    const int64_t* state = p.block_state + i * kBlockState;
    rows += __ldcg(state + 0);
    row_first = min(row_first, static_cast<int64_t>(__ldcg(state + 1)));
    row_bits |= static_cast<unsigned>(__ldcg(state + 2));
    all_cols += __ldcg(state + 3);
    all_col_first = min(all_col_first, static_cast<int64_t>(__ldcg(state + 4)));
  }
  block_reduce(rows, row_first, row_bits);
  block_reduce(all_cols, all_col_first, unused);
  if (threadIdx.x == 0) {
    const bool col_nonfinite = p.col_flags[1] != 0;
    const bool located = rows == 1 && all_cols == 1 && !(row_bits & kRowNonfinite) && !col_nonfinite;
    p.location[0] = located ? row_first : -1;
    p.location[1] = located ? all_col_first : -1;
    *p.located = located ? 1 : 0;
    p.row_flags[0] = (row_bits & kRowFailed) ? 1 : 0;
    p.row_flags[1] = (row_bits & kRowNonfinite) ? 1 : 0;
    *p.ticket = 0;  // clean for the slot's next launch
  }
}

int locate2d_ticket(uint32_t** out) {
  constexpr int kMaxDevices = 64;
  static std::mutex lock;
  static uint32_t* base[kMaxDevices] = {};
  static std::atomic<uint64_t> sequence{0};
  int device = 0;
  SDC_CUDA_CHECK(cudaGetDevice(&device));
  if (device < 0 || device >= kMaxDevices) return fail(SDC_ERR_INVALID, "device index out of range");
  uint32_t* slots = nullptr;
  {
    std::lock_guard<std::mutex> guard(lock);
    if (base[device] == nullptr) {
      void* ptr = nullptr;
      SDC_CUDA_CHECK(cudaGetSymbolAddress(&ptr, g_locate2d_tickets));
      base[device] = static_cast<uint32_t*>(ptr);
    }
    slots = base[device];
  }
  *out = slots + sequence.fetch_add(1, std::memory_order_relaxed) % kTicketSlots;
  return SDC_OK;
}

// Grid: as many blocks as fit on the SMs (shared memory for the staged u,
// registers), at most one per tile of rows.
template <Kind KIND>
int launch_row_predict(const uint8_t* a, const float* sa, const uint8_t* sfa, int64_t m, int64_t k, const float* u,
                       const float* alpha, float* predicted, float* magnitude, cudaStream_t stream) {
  const int64_t panels = ceil_div(k / 16, kPanelGroups);
  const int chunk_panels = static_cast<int>(std::min<int64_t>(panels, kMaxStagedPanels));
  const size_t smem = static_cast<size_t>(chunk_panels) * kPanelFloat2 * sizeof(float2);
  auto kernel = row_predict<KIND>;
  SDC_CUDA_CHECK(cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                      static_cast<int>(kMaxStagedPanels * kPanelFloat2 * sizeof(float2))));
  int per_sm = 0;
  SDC_CUDA_CHECK(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kernel, 32 * kRowWarps, smem));
  const int64_t tiles = ceil_div(m, kRowWarps * kRowsPerWarp);
  const int64_t blocks = std::min<int64_t>(tiles, static_cast<int64_t>(std::max(per_sm, 1)) * sm_count());
  kernel<<<static_cast<unsigned>(blocks), 32 * kRowWarps, smem, stream>>>(a, sa, sfa, m, k, u, alpha, predicted,
                                                                          magnitude, chunk_panels);
  SDC_CUDA_CHECK(cudaGetLastError());
  return SDC_OK;
}

Kind row_kind(int kind) {
  return kind == SDC_KIND_NVFP4 ? Kind::kNvf4 : kind == SDC_KIND_FP8_BLOCK ? Kind::kFp8Block : Kind::kFp8;
}

}  // namespace
}  // namespace sdc

extern "C" {

size_t sdc_abft_row_workspace_bytes(int64_t n, int64_t k) {
  if (n <= 0 || k <= 0) return 0;
  // u [K_pad][2], then the projection's band partials [ceil(N/128)][K_pad][2].
  const int64_t floats = sdc::ceil_div(k, 64) * 64 * 2;
  return static_cast<size_t>(floats * (1 + sdc::ceil_div(n, sdc::kBandRows))) * sizeof(float);
}

int sdc_abft_row_reference(int kind, const uint8_t* a, const void* a_scales, const uint8_t* b_rows,
                           const void* b_scales, int64_t m, int64_t n, int64_t k, const float* alpha,
                           float* predicted_rows, float* magnitude_rows, void* workspace, size_t workspace_bytes,
                           sdc_stream_t stream) {
  using namespace sdc;
  SDC_REQUIRE(kind == SDC_KIND_FP8 || kind == SDC_KIND_NVFP4 || kind == SDC_KIND_FP8_BLOCK,
              "row checksums: kind must be SDC_KIND_FP8, SDC_KIND_NVFP4 or SDC_KIND_FP8_BLOCK");
  SDC_REQUIRE(m > 0 && n > 0 && k > 0 && m <= INT32_MAX && n <= INT32_MAX, "row checksums need positive sizes");
  SDC_REQUIRE(a != nullptr && b_rows != nullptr && predicted_rows != nullptr && magnitude_rows != nullptr,
              "row checksum pointers must not be null");
  SDC_REQUIRE(kind == SDC_KIND_FP8 || (a_scales != nullptr && b_scales != nullptr),
              "row checksums of scaled kinds need both operands' scales");
  SDC_REQUIRE(kind == SDC_KIND_FP8_BLOCK || alpha != nullptr, "row checksums need alpha (FP8, NVFP4)");
  SDC_REQUIRE(k % (kind == SDC_KIND_FP8_BLOCK ? 128 : kind == SDC_KIND_NVFP4 ? 32 : 16) == 0,
              "row checksums: K must be a multiple of 16 (FP8), 32 (NVFP4) or 128 (block-scaled FP8)");
  if (workspace == nullptr || workspace_bytes < sdc_abft_row_workspace_bytes(n, k) ||
      reinterpret_cast<uintptr_t>(workspace) % 16 != 0) {
    return fail(SDC_ERR_WORKSPACE, "row checksum workspace too small or not 16-byte aligned");
  }
  int rc = check_current_device();
  if (rc != SDC_OK) return rc;
  const Kind kd = row_kind(kind);
  float* u = static_cast<float*>(workspace);
  // u = e^T B, u_abs = e^T |B| over the N rows of B (unit weights).
  ProjectionView view{b_rows,
                      kd == Kind::kFp8Block ? static_cast<const float*>(b_scales) : nullptr,
                      kd == Kind::kNvf4 ? static_cast<const uint8_t*>(b_scales) : nullptr,
                      nullptr,
                      n,
                      k,
                      k / 128,
                      ceil_div(k, 64),
                      u + ceil_div(k, 64) * 64 * 2};
  view.scale_shift = 7;  // B's block scales cover 128 rows
  rc = launch_projection_sums(kd, 1, view, u, stream);
  if (rc != SDC_OK) return rc;
  const float* sa = kd == Kind::kFp8Block ? static_cast<const float*>(a_scales) : nullptr;
  const uint8_t* sfa = kd == Kind::kNvf4 ? static_cast<const uint8_t*>(a_scales) : nullptr;
  const float* al = kd == Kind::kFp8Block ? nullptr : alpha;
  return kd == Kind::kFp8    ? launch_row_predict<Kind::kFp8>(a, sa, sfa, m, k, u, al, predicted_rows,
                                                              magnitude_rows, stream)
         : kd == Kind::kNvf4 ? launch_row_predict<Kind::kNvf4>(a, sa, sfa, m, k, u, al, predicted_rows,
                                                               magnitude_rows, stream)
                             : launch_row_predict<Kind::kFp8Block>(a, sa, sfa, m, k, u, al, predicted_rows,
                                                                   magnitude_rows, stream);
}

size_t sdc_abft_locate2d_workspace_bytes(void) {
  return static_cast<size_t>(sdc::kLocate2dBlocks) * sdc::kBlockState * sizeof(int64_t);
}

int sdc_abft_locate2d(const float* row_observed, int64_t row_blocks, const float* predicted_rows,
                      const float* magnitude_rows, int64_t m, float atol, float rtol, const float* col_residual,
                      const float* col_threshold, int algorithm, int64_t n, const uint8_t* col_flags,
                      float* row_residual, float* row_threshold, int64_t* location, uint8_t* located,
                      uint8_t* row_flags, void* workspace, size_t workspace_bytes, sdc_stream_t stream) {
  using namespace sdc;
  const int channels = policy_channels(algorithm);
  if (channels == 0) return fail(SDC_ERR_UNKNOWN_ALGORITHM, "Unknown compiled ABFT algorithm ID");
  SDC_REQUIRE(m > 0 && n > 0 && row_blocks == ceil_div(n, 64), "locate2d: row_blocks must be ceil(n / 64)");
  SDC_REQUIRE(row_observed && predicted_rows && magnitude_rows && col_residual && col_threshold && col_flags &&
                  location && located && row_flags,
              "locate2d pointers must not be null");
  SDC_REQUIRE(std::isfinite(atol) && std::isfinite(rtol) && atol >= 0.f && rtol >= 0.f,
              "ABFT tolerances must be finite and nonnegative");
  if (workspace == nullptr || workspace_bytes < sdc_abft_locate2d_workspace_bytes() ||
      reinterpret_cast<uintptr_t>(workspace) % 8 != 0) {
    return fail(SDC_ERR_WORKSPACE, "locate2d workspace too small or not 8-byte aligned");
  }
  Locate2dArgs p{};
  p.row_observed = row_observed;
  p.row_blocks = row_blocks;
  p.predicted = predicted_rows;
  p.magnitude = magnitude_rows;
  p.m = m;
  p.atol = atol;
  p.rtol = rtol;
  p.col_residual = col_residual;
  p.col_threshold = col_threshold;
  p.channels = channels;
  p.n = n;
  p.col_flags = col_flags;
  p.row_residual = row_residual;
  p.row_threshold = row_threshold;
  p.location = location;
  p.located = located;
  p.row_flags = row_flags;
  p.block_state = static_cast<int64_t*>(workspace);
  int rc = locate2d_ticket(&p.ticket);
  if (rc != SDC_OK) return rc;
  const int64_t blocks = std::min<int64_t>(kLocate2dBlocks, ceil_div(std::max(m, n), kLocate2dThreads));
  locate2d<<<static_cast<unsigned>(blocks), kLocate2dThreads, 0, stream>>>(p);
  SDC_CUDA_CHECK(cudaGetLastError());
  return SDC_OK;
}

}  // extern "C"
