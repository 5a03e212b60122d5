// ABFT checksum finalize: merge per-tile partials and decide.
//
// Semantics follow src/cutlass_gemm/csrc/abft/common/finalize.cu:55-153 and
// policy.cuh:54-63 of the reference: each (channel, column) is reduced by one
// thread in ascending tile order with round-to-nearest adds, the threshold is
// a separate multiply then add (never an FMA), and only exact integer status
// bits cross thread-block boundaries. Work is memory bound (3 partial planes
// read once); the grid is one thread per (channel, column) so loads of
// consecutive columns coalesce, and a second one-block kernel ORs the
// per-block status words into the five flags: the last block of the grid to
// finish (an atomic ticket) does it, so the finalize is one launch, with no
// float atomics and no host syncs.
// The partials are staged through shared memory by all warps of a block so
// that many loads are in flight, while the additions stay serial per column.
#include <algorithm>
#include <atomic>
#include <mutex>

#include "common.cuh"

namespace sdc {
namespace {

constexpr int kFinalizeThreads = 64;   // columns per block (and threads of the flags kernel)
constexpr int kColumnThreads = 256;    // threads of a finalize_columns block
constexpr int kTileChunk = 32;         // tiles staged in shared memory per round
constexpr unsigned kDetected = 1u;
constexpr unsigned kNonfinite = 2u;
constexpr unsigned kHit = 4u;

struct FinalizeParams {
  const float* observed;
  const float* predicted;
  const float* magnitude;
  int64_t m_tiles, padded_n, n;
  const int32_t* tile_flags;
  int64_t flag_count;
  const int32_t* hit_in;
  const int32_t* nonfinite_in;
  float atol, rtol;
  float* reference;
  bool use_reference;
  bool diagnostics;
  float* residual;
  float* threshold;
  const float* thresholds;
  bool scalar_threshold;
  int32_t* block_states;
  int64_t blocks;            // grid size: the ticket value of the last block
  uint32_t* ticket;          // this launch's arrival counter, zero on entry
  uint8_t* flags;
  int32_t* hit_out;
  int64_t* location;
};

// Arrival counters of the finalize launches on a device. A launch takes the
// slot its host-side sequence number selects (mod kTicketSlots); its last
// block returns the counter to zero, so a slot is clean again before it
// comes round (far more launches than that are never in flight at once; a
// captured graph replays its slot sequentially).
constexpr int kTicketSlots = 4096;
static __device__ uint32_t g_finalize_tickets[kTicketSlots];

// Block = 64 columns of one channel. All 8 warps stage the partials of 32
// tiles at a time in shared memory (warp w stages column group w % 2 of the
// tiles t with t % 4 == w / 2), so many loads are in flight; then warps 0 and
// 1 add them, one thread per column, in ascending tile order.
template <int C>
__global__ void __launch_bounds__(kColumnThreads) finalize_columns(FinalizeParams p) {
  __shared__ float staged[3][kTileChunk][kFinalizeThreads];
  __shared__ unsigned warp_state[kColumnThreads / 32];
  unsigned state = 0;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int group = warp & 1;                 // column group of 32
  const int phase = warp >> 1;                // tiles t with t % 4 == phase
  const int channel = blockIdx.y;
  const int64_t block = static_cast<int64_t>(blockIdx.y) * gridDim.x + blockIdx.x;
  const int local = group * 32 + lane;        // column within the block
  const int64_t col = static_cast<int64_t>(blockIdx.x) * kFinalizeThreads + local;
  const bool col_in = col < p.n;

  // Status inputs: each packed tile flag is read by exactly one thread of the grid.
  if (p.tile_flags != nullptr) {
    const int64_t stride = static_cast<int64_t>(gridDim.x) * gridDim.y * kColumnThreads;
    for (int64_t i = block * kColumnThreads + threadIdx.x; i < p.flag_count; i += stride) {
      const int32_t t = p.tile_flags[i];
      if (t & 1) state |= kHit;
      if (t & 2) state |= kDetected | kNonfinite;
    }
  } else if (block == 0 && threadIdx.x == 0) {
    // hit bit 0: the fault was applied; bit 1: the GEMM launch gave up a
    // bounded wait, so its partials are incomplete and the call must not pass.
    const int32_t hit = *p.hit_in;
    if (hit & 1) state |= kHit;
    if (hit & 2) state |= kDetected | kNonfinite;
    if (*p.nonfinite_in != 0) state |= kDetected | kNonfinite;
  }

  const int64_t base = static_cast<int64_t>(channel) * p.m_tiles * p.padded_n + col;
  float observed = 0.f, predicted = 0.f, magnitude = 0.f;
  for (int64_t t0 = 0; t0 < p.m_tiles; t0 += kTileChunk) {
    // All 24 loads of this thread are issued before any lands in shared memory.
    constexpr int kPerWarp = kTileChunk / 4;
    float v[3][kPerWarp];
#pragma unroll
    for (int j = 0; j < kPerWarp; ++j) {
      const int i = phase + 4 * j;
      const bool in = col_in && t0 + i < p.m_tiles;
      const int64_t off = base + (t0 + i) * p.padded_n;
      v[0][j] = in ? __ldg(p.observed + off) : 0.f;
      v[1][j] = (in && !p.use_reference) ? __ldg(p.predicted + off) : 0.f;
      v[2][j] = (in && !p.use_reference) ? __ldg(p.magnitude + off) : 0.f;
    }
#pragma unroll
    for (int j = 0; j < kPerWarp; ++j) {
#pragma unroll
      for (int plane = 0; plane < 3; ++plane) staged[plane][phase + 4 * j][local] = v[plane][j];
    }
    __syncthreads();
    if (warp < 2) {
      const int64_t count = p.m_tiles - t0 < kTileChunk ? p.m_tiles - t0 : kTileChunk;
      for (int i = 0; i < count; ++i) {
        observed = __fadd_rn(observed, staged[0][i][local]);
        predicted = __fadd_rn(predicted, staged[1][i][local]);
        magnitude = __fadd_rn(magnitude, staged[2][i][local]);
      }
    }
    __syncthreads();
  }

  if (warp < 2 && col_in) {
    const int64_t out = static_cast<int64_t>(channel) * p.n + col;
    if (p.use_reference) {
      predicted = p.reference[out];
      magnitude = p.reference[static_cast<int64_t>(C) * p.n + out];
    } else {
      p.reference[out] = predicted;
      p.reference[static_cast<int64_t>(C) * p.n + out] = magnitude;
    }
    const float residual = __fsub_rn(observed, predicted);
    const float threshold =
        p.thresholds != nullptr ? p.thresholds[p.scalar_threshold ? 0 : out]
                                : __fadd_rn(p.atol, __fmul_rn(p.rtol, magnitude));
    const bool nonfinite = !isfinite(observed) || !isfinite(predicted) || !isfinite(magnitude) ||
                           !isfinite(residual) || !isfinite(threshold);
    if (nonfinite) state |= kDetected | kNonfinite;
    if (threshold < 0.f || fabsf(residual) > threshold) state |= kDetected;
    if (p.diagnostics) {
      p.residual[out] = residual;
      p.threshold[out] = threshold;
    }
  }

  // Deterministic OR across the block: warp shuffle, then shared memory.
  for (int offset = 16; offset > 0; offset >>= 1) state |= __shfl_xor_sync(0xffffffffu, state, offset);
  if (lane == 0) warp_state[warp] = state;
  __syncthreads();
  __shared__ bool last;
  if (threadIdx.x == 0) {
    unsigned combined = 0;
    for (int w = 0; w < kColumnThreads / 32; ++w) combined |= warp_state[w];
    p.block_states[block] = static_cast<int32_t>(combined);
    // Publish the state before taking a ticket; the block that takes the
    // last ticket sees every other block's state.
    __threadfence();
    last = atomicAdd(p.ticket, 1u) == static_cast<uint32_t>(p.blocks - 1);
  }
  __syncthreads();
  if (!last) return;
  __threadfence();
  unsigned all = 0;
  for (int64_t i = threadIdx.x; i < p.blocks; i += kColumnThreads) {
    all |= static_cast<unsigned>(__ldcg(p.block_states + i));
  }
  for (int offset = 16; offset > 0; offset >>= 1) all |= __shfl_xor_sync(0xffffffffu, all, offset);
  if (lane == 0) warp_state[warp] = all;
  __syncthreads();
  if (threadIdx.x == 0) {
    unsigned combined = 0;
    for (int w = 0; w < kColumnThreads / 32; ++w) combined |= warp_state[w];
    p.flags[0] = (combined & kDetected) ? 1 : 0;
    p.flags[1] = (combined & kNonfinite) ? 1 : 0;
    p.flags[2] = 0;  // located: reported by sdc_abft_locate, not by the policy decision
    p.flags[3] = 0;  // recovered: owned by the caller's retry transaction
    p.flags[4] = 0;  // recheck_failed: owned by the caller's retry transaction
    p.hit_out[0] = (combined & kHit) ? 1 : 0;
    p.location[0] = -1;
    p.location[1] = -1;
    *p.ticket = 0;  // the slot is clean for its next launch
  }
}

// The device address of this launch's ticket (slot chosen on the host).
int finalize_ticket(uint32_t** out) {
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
      SDC_CUDA_CHECK(cudaGetSymbolAddress(&ptr, g_finalize_tickets));
      base[device] = static_cast<uint32_t*>(ptr);
    }
    slots = base[device];
  }
  *out = slots + sequence.fetch_add(1, std::memory_order_relaxed) % kTicketSlots;
  return SDC_OK;
}

int64_t finalize_blocks(int channels, int64_t n) {
  return static_cast<int64_t>(channels) * ceil_div(n, kFinalizeThreads);
}

}  // namespace
}  // namespace sdc

extern "C" {

size_t sdc_abft_finalize_workspace_bytes(int algorithm, int64_t n, int64_t m_tiles) {
  (void)m_tiles;
  const int channels = sdc::policy_channels(algorithm);
  if (channels == 0 || n <= 0) return 0;
  return static_cast<size_t>(sdc::finalize_blocks(channels, n)) * sizeof(int32_t);
}

int sdc_abft_finalize(int algorithm, const float* observed, const float* predicted,
                      const float* magnitude, int64_t m_tiles, int64_t padded_n, int64_t n,
                      const int32_t* tile_flags, int64_t flag_count, const int32_t* hit_in,
                      const int32_t* nonfinite_in, float atol, float rtol, float* reference,
                      int use_reference, int diagnostics, float* residual, float* threshold,
                      const float* thresholds, int scalar_threshold, uint8_t* flags,
                      int32_t* hit_out, int64_t* location, void* workspace,
                      size_t workspace_bytes, sdc_stream_t stream) {
  using namespace sdc;
  const int channels = policy_channels(algorithm);
  if (channels == 0) return fail(SDC_ERR_UNKNOWN_ALGORITHM, "Unknown compiled ABFT algorithm ID");
  SDC_REQUIRE(n > 0 && m_tiles > 0 && padded_n >= n, "ABFT finalize requires n > 0, m_tiles > 0, padded_n >= n");
  SDC_REQUIRE(observed != nullptr && reference != nullptr && flags != nullptr &&
                  hit_out != nullptr && location != nullptr,
              "ABFT finalize pointers must not be null");
  SDC_REQUIRE(use_reference || (predicted != nullptr && magnitude != nullptr),
              "ABFT finalize needs predicted/magnitude partials without a reference");
  SDC_REQUIRE(tile_flags != nullptr || (hit_in != nullptr && nonfinite_in != nullptr),
              "ABFT finalize needs tile_flags or hit/nonfinite inputs");
  SDC_REQUIRE(!diagnostics || (residual != nullptr && threshold != nullptr),
              "ABFT finalize diagnostics need residual and threshold outputs");
  const int64_t blocks = finalize_blocks(channels, n);
  if (workspace == nullptr || workspace_bytes < static_cast<size_t>(blocks) * sizeof(int32_t)) {
    return fail(SDC_ERR_WORKSPACE, "ABFT finalize workspace too small");
  }
  FinalizeParams p{};
  p.observed = observed;
  p.predicted = predicted;
  p.magnitude = magnitude;
  p.m_tiles = m_tiles;
  p.padded_n = padded_n;
  p.n = n;
  p.tile_flags = tile_flags;
  p.flag_count = flag_count;
  p.hit_in = hit_in;
  p.nonfinite_in = nonfinite_in;
  p.atol = atol;
  p.rtol = rtol;
  p.reference = reference;
  p.use_reference = use_reference != 0;
  p.diagnostics = diagnostics != 0;
  p.residual = residual;
  p.threshold = threshold;
  p.thresholds = thresholds;
  p.scalar_threshold = scalar_threshold != 0;
  p.block_states = static_cast<int32_t*>(workspace);
  p.blocks = blocks;
  p.flags = flags;
  p.hit_out = hit_out;
  p.location = location;
  const int rc = finalize_ticket(&p.ticket);
  if (rc != SDC_OK) return rc;
  const dim3 grid(static_cast<unsigned>(ceil_div(n, kFinalizeThreads)), channels);
  if (channels == 2) {
    finalize_columns<2><<<grid, kColumnThreads, 0, stream>>>(p);
  } else {
    finalize_columns<1><<<grid, kColumnThreads, 0, stream>>>(p);
  }
  SDC_CUDA_CHECK(cudaGetLastError());
  return SDC_OK;
}

// ---------------------------------------------------------------------------
// Allocation-free finalize. Some hosts that bind this ABI have no device
// allocator they may call at this point (a plain C or FFI host driving the
// check from a monitoring hook, or code that must not grow device memory
// between steps), so they cannot hand finalize its per-block scratch. This
// variant takes the scratch from a fixed, file-scope device array instead.
// ---------------------------------------------------------------------------
namespace sdc {
namespace {

// 16384 int32 status words (64 KiB per GPU that loads the library, held until
// the process exits): channels * ceil(n / 64) <= 16384, i.e. n <= 524288 for
// the two-channel Classic policy.
constexpr int64_t kNoAllocMaxBlocks = 16384;
static __device__ __align__(256) int32_t g_finalize_noalloc_scratch[kNoAllocMaxBlocks];

// In host code the array's name is only a host-side stand-in, so its device
// address is looked up once per device (with that device current) and cached.
int noalloc_scratch(int32_t** out) {
  constexpr int kMaxDevices = 64;
  static std::mutex lock;
  static int32_t* cached[kMaxDevices] = {};
  int device = 0;
  SDC_CUDA_CHECK(cudaGetDevice(&device));
  if (device < 0 || device >= kMaxDevices) return fail(SDC_ERR_INVALID, "device index out of range");
  std::lock_guard<std::mutex> guard(lock);
  if (cached[device] == nullptr) {
    void* ptr = nullptr;
    SDC_CUDA_CHECK(cudaGetSymbolAddress(&ptr, g_finalize_noalloc_scratch));
    cached[device] = static_cast<int32_t*>(ptr);
  }
  *out = cached[device];
  return SDC_OK;
}

}  // namespace
}  // namespace sdc

int sdc_abft_finalize_noalloc(int algorithm, const float* observed, const float* predicted,
                              const float* magnitude, int64_t m_tiles, int64_t padded_n, int64_t n,
                              const int32_t* tile_flags, int64_t flag_count, const int32_t* hit_in,
                              const int32_t* nonfinite_in, float atol, float rtol, float* reference,
                              int use_reference, int diagnostics, float* residual, float* threshold,
                              const float* thresholds, int scalar_threshold, uint8_t* flags,
                              int32_t* hit_out, int64_t* location, sdc_stream_t stream) {
  using namespace sdc;
  const int channels = policy_channels(algorithm);
  if (channels == 0) return fail(SDC_ERR_UNKNOWN_ALGORITHM, "Unknown compiled ABFT algorithm ID");
  if (n <= 0 || finalize_blocks(channels, n) > kNoAllocMaxBlocks) {
    return fail(SDC_ERR_INVALID,
                "sdc_abft_finalize_noalloc supports channels * ceil(n/64) <= 16384 status words "
                "(n <= 524288 for Classic); use sdc_abft_finalize with a caller workspace");
  }
  int32_t* scratch = nullptr;
  const int rc = noalloc_scratch(&scratch);
  if (rc != SDC_OK) return rc;
  // The status words are written by every block before they are read, so the
  // shared array needs no clearing between calls.
  return sdc_abft_finalize(algorithm, observed, predicted, magnitude, m_tiles, padded_n, n, tile_flags,
                           flag_count, hit_in, nonfinite_in, atol, rtol, reference, use_reference,
                           diagnostics, residual, threshold, thresholds, scalar_threshold, flags, hit_out,
                           location, scratch, static_cast<size_t>(kNoAllocMaxBlocks) * sizeof(int32_t),
                           stream);
}

}  // extern "C"
