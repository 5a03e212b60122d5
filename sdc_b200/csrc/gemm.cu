// Persistent tcgen05 GEMMs for sm_100a with the ABFT checksums fused.
//
// One CTA (or CTA pair, cta_group::2, when M > 128) per SM loops over output
// tiles of 128 rows per CTA (one reference M-tile, so every observed-checksum
// partial comes from one CTA) in a grouped raster order that keeps a band of
// A and the B tiles resident in L2. Tile widths: 256 columns (FP8, NVFP4),
// 128 (block-scaled FP8). Warp roles:
//   warp 0      TMA producer: 128-byte-swizzled K-major A/B stages (and the
//               512-byte NVFP4 scale atoms) into a ring; in pairs each CTA
//               loads its A rows and half of the tile's B rows, completing
//               on the leader's barrier.
//   warp 1      allocates tensor memory; one thread (the leader's, in pairs)
//               issues tcgen05.mma: kind::f8f6f4 e4m3, or kind::mxf4nvf4.block16
//               with scales copied to TMEM by tcgen05.cp. FP8 double-buffers
//               a 256-column fp32 accumulator so a tile's epilogue overlaps
//               the next mainloop; NVFP4 has one (the scales take the rest of
//               TMEM); block-scaled FP8 writes one partial per 128-wide K
//               block into four rotating 128-column buffers.
//   epilogue    FP8: warps 2-5, one per TMEM lane quarter, 32 columns at a
//               time. NVFP4 and block-scaled FP8 ("wide" kinds): warps 4-11,
//               two per lane quarter, each owning half of the tile's columns;
//               NVFP4's warps load their whole half before the math, so the
//               next tile's MMAs only wait for the loads; block-scaled FP8's
//               warps first promote every partial into register-resident
//               totals (total += fl(sa * sb) * partial). Then per 32-column
//               chunk: alpha * acc, optional accumulator bit flip, column
//               checksums sum_rows w_c[row] * v (butterfly transpose-reduce
//               across lanes, fixed-order sum across the four row quarters),
//               non-finite check of the converted output, output store.
//   prediction  (K-slice layout only; warps 6-9, wide kinds 12-15)
//               input-side prediction, independent of the MMA pipeline, in
//               three phases separated by grid-wide barriers (every CTA is
//               resident; each wait is bounded):
//                 1. projection partials of A: each warp takes (64-wide K
//                    chunk, 512-row band) items and writes
//                    part[band][k][c][h] = sum over the band's rows of
//                    w_c[row] * A[row, k] (h = 0) and |w_c| |A| (h = 1);
//                 2. q_full[k][c][h] = sum over bands (ascending);
//                 3. for the 64-wide K slices assigned to each of this CTA's
//                    tiles (slice % Tm == tile row), fma chains of q_full
//                    with B[n, k] and |q|, |B| (B rows read from L2).
//               In total one extra pass over A and one over B, overlapped
//               with the tensor-core mainloop.
// Wide kinds run their roles on warpgroup boundaries and move registers with
// setmaxnreg (warpgroup 0 down, the epilogue warpgroups up).
// Epilogue semantics follow src/cutlass_gemm/csrc/abft/common/
// sm120_epilogue.cuh:52-151 of the reference (inject after alpha, observe
// before the output cast). Every wait is bounded (common.cuh).
#include <algorithm>
#include <atomic>

#include "kslice.cuh"

namespace sdc {
namespace {

constexpr int kBM = 128;
constexpr int kBN = 256;
constexpr int kBKBytes = 128;  // one 128-byte swizzle atom of K per stage
constexpr int kStages = 4;
constexpr uint32_t kTmemCols = 512;
// Tile width in output columns. NVFP4 keeps 256 as well: a 128-wide tile
// would leave room for two accumulators next to the block scales, but the
// extra operand traffic per MAC costs more (measured: 2.2 vs 3.1 PF/s
// unprotected at 16384^3) than the exposed epilogue of one accumulator.
__host__ __device__ constexpr int tile_n(Kind k) { return k == Kind::kFp8Block ? kBN / 2 : kBN; }
__host__ __device__ constexpr int chunks(Kind k) { return tile_n(k) / 32; }
// NVFP4 block scales in TMEM after the accumulator(s): per 64-wide k-step,
// 4 columns per 128 rows of A (the CTA's M-tile) and of B (the tile's rows).
__host__ __device__ constexpr int sfb_groups(Kind k) { return tile_n(k) / 128; }
constexpr uint32_t kSfaCol = 256;  // 4 k-steps x 4 columns
constexpr uint32_t kSfbCol = 272;  // 4 k-steps x 4 columns x B row groups
constexpr int kChunks = kBN / 32;  // the widest tile's 32-column chunks
constexpr int kGroupM = 16;        // M-tiles per raster group
constexpr int64_t kPacedItems = 4;  // projection items per warp above which they are paced

constexpr int kABytes = kBM * kBKBytes;
constexpr int kSfaBytes = 4 * 512;
constexpr int kSfbBytes = 4 * 512 * (kBN / 128);  // per k-block: 4 k-steps x the tile's B row groups
// Reduced channels of the epilogue per 32-column chunk and row quarter: the
// checksum channels (<= 2), plus as many output-magnitude channels for the
// augmented bf16 GEMM.
__host__ __device__ constexpr int red_channels(Kind k) { return k == Kind::kBf16 ? 4 : 2; }
__host__ __device__ constexpr int red_floats(Kind k) { return kChunks * 4 * red_channels(k) * 32; }

// CTA pairs: each CTA stages its 128 rows of A and 128 of the tile's 256 B
// rows (NVFP4: plus its own A scales and all 256 rows' B scales); one
// cta_group::2 MMA covers the 256 x 256 pair tile.
__host__ __device__ constexpr int b_stage_bytes(Kind k, bool pair) {
  return (pair ? tile_n(k) / 2 : tile_n(k)) * kBKBytes;
}
__host__ __device__ constexpr int stage_bytes(Kind k, bool pair = false) {
  return kABytes + b_stage_bytes(k, pair) + (k == Kind::kNvf4 ? kSfaBytes + kSfbBytes : 0);
}
__host__ __device__ constexpr int num_stages(Kind k, bool pair) {
  return pair ? (k == Kind::kFp8 || k == Kind::kBf16 ? 6 : k == Kind::kFp8Block ? 8 : 5) : kStages;
}
// Checked e4m3 launches stage the prediction's B slices (tile rows x one
// 64-byte K slice) in shared memory with their own TMA copies: a warp-wide
// read there costs 4 shared-memory wavefronts where a global load of 32 rows
// cost 32 L1 sectors (measured: most of the protected FP8 kernel's overhead).
__host__ __device__ constexpr int pred_slice_bytes(Kind k, bool chk) {
  return (chk && is_e4m3(k)) ? tile_n(k) * 64 : 0;
}
// Checked launches stage each K slice's q (64 k x 2 channels x value and
// magnitude, fp32) for the prediction warps: one batch of loads per slice.
__host__ __device__ constexpr int pred_q_bytes(bool chk) { return chk ? 64 * 2 * 2 * 4 : 0; }
__host__ __device__ constexpr int smem_bytes(Kind k, bool pair = false, bool chk = false) {
  return 1024 + num_stages(k, pair) * stage_bytes(k, pair) + red_floats(k) * 4 + pred_slice_bytes(k, chk) +
         pred_q_bytes(chk) + 512;
}
__host__ __device__ constexpr int num_acc(Kind k) { return k == Kind::kNvf4 ? 1 : 2; }
// Warp roles. Tensorwise FP8: 0 TMA, 1 MMA, 2-5 epilogue, 6-9 prediction
// (checked K-slice launches). Wide kinds (NVFP4, block-scaled FP8): 0 TMA,
// 1 MMA, 2-3 idle, 4-11 epilogue (block-scaled: promotion + epilogue), two
// warps per TMEM lane quarter, each owning one half of the tile's columns,
// 12-15 prediction: roles on warpgroup boundaries, so that registers can move
// from warpgroup 0 to the epilogue warps (setmaxnreg). NVFP4 has a single
// accumulator: its epilogue warps load their whole half of it before the
// math, so the next tile's MMAs start after the loads, not after the stores.
__host__ __device__ constexpr bool is_wide(Kind k) { return k != Kind::kFp8 && k != Kind::kBf16; }
__host__ __device__ constexpr int epi_warp0(bool wide) { return wide ? 4 : 2; }
__host__ __device__ constexpr int acc_warps(bool wide) { return wide ? 8 : 4; }
__host__ __device__ constexpr int pred_warp0(bool wide) { return epi_warp0(wide) + acc_warps(wide); }
// Register split of the wide kinds (registers per thread, by warpgroup):
// checked launches start 512 threads with 128 each (the whole register file);
// warpgroup 0 drops to 40, the two epilogue warpgroups rise to 168 and the
// prediction warpgroup keeps 128: 40 + 168 + 168 + 128 = 504 <= 4 x 128.
// Unchecked launches start 384 threads with 168: 40 + 224 + 224 = 488 <= 3 x 168.
// launch_impl checks the launch's register count against this before
// launching (an increase that does not fit would wait forever).
constexpr uint32_t kLowRegs = 40;
__host__ __device__ constexpr uint32_t epilogue_regs(bool chk) { return chk ? 168 : 224; }
__host__ __device__ constexpr uint32_t required_regs_per_thread(bool chk) {
  // Registers of the whole CTA after the split, divided by its threads (rounded up).
  return chk ? (kLowRegs + 2 * epilogue_regs(true) + 128 + 3) / 4 : (kLowRegs + 2 * epilogue_regs(false) + 2) / 3;
}
__host__ __device__ constexpr int num_threads(bool chk, bool wide = false) {
  return 32 * (pred_warp0(wide) + (chk ? 4 : 0));
}
template <bool WIDE>
__device__ __forceinline__ bool is_prediction_warp(int warp) {
  return warp >= pred_warp0(WIDE) && warp < pred_warp0(WIDE) + 4;
}
template <bool WIDE>
__device__ __forceinline__ int prediction_index(int warp) { return warp - pred_warp0(WIDE); }
// Block-scaled FP8: 4 partial accumulators of 128 columns fill the 512 TMEM
// columns; the promotion warps keep the tile totals in registers. The MMA and
// promotion warps hand partials over in groups of 2 K blocks (one commit and
// one release per group), so 2 groups are in flight.
constexpr int kPartBufs = 4;
constexpr int kGroupKb = 2;
constexpr int kGroupSlots = kPartBufs / kGroupKb;

struct Params {
  int32_t m, n, k, num_kb, tiles_m, tiles_n, num_tiles;
  int32_t num_work;  // tiles, or 256-row pair tiles when CTAs are paired
  const float* sa;   // block-scaled FP8: A scales [M][K/128], B scales [ceil(N/128)][K/128]
  const float* sb;
  int32_t k_blocks;
  const float* alpha;
  void* d;
  const float* weights;
  int32_t frow, fcol, fbit;
  int32_t* nonfinite;
  float* observed;
  int32_t* hit;
  int32_t padded_n;
  float* q_full;        // [K_pad][C][2]: full-M projection (h=0) and magnitude (h=1)
  float* q_part;        // [bands][K_pad][C][2]: per-band partials
  uint32_t* grid_sync;  // arrival counter of the prediction warpgroups (zeroed per launch)
  int32_t q_bands;
  int32_t q_ready;      // q_full computed before the launch: no projection phases
  const uint8_t* a;     // A operand rows (projection) and B rows (prediction),
  const uint8_t* sfa;   // read directly by the prediction warps
  const uint8_t* b;
  const uint8_t* sfb;
  float* predicted;
  float* magnitude;
  int32_t* watchdog;
  uint64_t wait_limit_ns;  // every bounded wait gives up after this long
  int32_t pace_extra;      // test hook: added to every pacing target (0 in use)
  // Augmented bf16 GEMM: M-tiles tiles_m .. tiles_m_all - 1 hold the
  // checksum rows (aug_rows of them, row t * C + c); tile_flags (nullable)
  // [tiles_m][flag_cols] collects per-128-column status bits (ORed).
  int32_t tiles_m_all;
  int32_t aug_rows;
  int32_t* tile_flags;
  // Row checksums (extension, nullable): sum over each 64-column block of
  // every output row's fp32 values (after the fault), [ceil(N/64)][M].
  float* row_observed;
  int32_t flag_cols;
};

__device__ __forceinline__ void raster(int t, int rows, int group_rows, int tiles_n, int& r, int& nt) {
  const int group_tiles = group_rows * tiles_n;
  const int group = t / group_tiles;
  const int first = group * group_rows;
  const int gm = min(group_rows, rows - first);
  const int in_group = t - group * group_tiles;
  r = first + in_group % gm;
  nt = in_group / gm;
}

// Work item -> this CTA's (M-tile, N-tile). With CTA pairs an item is a
// 256-row pair tile and the CTA of rank r owns its 128-row half r (which may
// lie beyond M when M % 256 <= 128).
template <bool PAIR>
__device__ __forceinline__ void work_coords(int w, const Params& p, uint32_t rank, int& mt, int& nt) {
  if constexpr (PAIR) {
    int mt2;
    raster(w, (p.tiles_m_all + 1) / 2, kGroupM / 2, p.tiles_n, mt2, nt);
    mt = 2 * mt2 + static_cast<int>(rank);
  } else {
    raster(w, p.tiles_m_all, kGroupM, p.tiles_n, mt, nt);
  }
}

// Butterfly transpose-reduce over the lane bits below N: lane j returns the
// sum, over the lanes that differ from it only in those bits, of x[j % N]
// (x is consumed). With N = 32 that is the sum over the warp of x[j].
template <int N>
__device__ __forceinline__ float transpose_reduce(float (&x)[N], int lane) {
#pragma unroll
  for (int width = N / 2; width >= 1; width >>= 1) {
    const bool upper = (lane & width) != 0;
#pragma unroll
    for (int i = 0; i < width; ++i) {
      const float send = upper ? x[i] : x[i + width];
      const float keep = upper ? x[i + width] : x[i];
      x[i] = keep + __shfl_xor_sync(0xffffffffu, send, width);
    }
  }
  return x[0];
}


__device__ __forceinline__ uint32_t ld_acquire_u32(const uint32_t* p) {
  uint32_t v;
  asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

// Grid-wide barrier of the prediction warpgroups (thread ct == 0 of each CTA
// arrives; all 128 threads leave together). Bounded: on timeout the CTA's
// abort flag and the watchdog are set. Returns false when aborted.
__device__ __forceinline__ bool prediction_grid_barrier(uint32_t* counter, uint32_t target, int ct,
                                                        volatile int32_t* abort_flag, int32_t* watchdog,
                                                        uint64_t limit_ns) {
  named_barrier(2, 128);
  if (ct == 0) {
    __threadfence();
    atomicAdd(counter, 1u);
    const uint64_t start = global_ns();
    while (ld_acquire_u32(counter) < target) {
      if (*abort_flag) break;
      if (global_ns() - start > limit_ns) {
        atomicCAS(watchdog, 0, kWaitGrid);
        *abort_flag = kWaitGrid;
        break;
      }
      // Every CTA polls the same word; at a short M the wait is on the
      // launch's critical path, so the poll is frequent.
      __nanosleep(256);
    }
    __threadfence();
  }
  named_barrier(2, 128);
  return *abort_flag == 0;
}

// Scale-factor atom (32 rows x 16 bytes, contiguous) as a tcgen05.cp source.
__device__ __forceinline__ uint64_t sf_desc(uint32_t addr) { return smem_desc(addr, 0, 128, 0); }

template <Kind KIND, int C, bool BF16OUT, bool CHK, bool PAIR>
__global__ void __launch_bounds__(num_threads(CHK, is_wide(KIND)), 1)
    gemm_kernel(const __grid_constant__ CUtensorMap tm_a, const __grid_constant__ CUtensorMap tm_b,
                const __grid_constant__ CUtensorMap tm_sfa,
                const __grid_constant__ CUtensorMap tm_sfb, const Params p) {
  constexpr int kS = num_stages(KIND, PAIR);
  constexpr int kBStage = b_stage_bytes(KIND, PAIR);
  constexpr int kTN = tile_n(KIND);
  constexpr int kTileChunks = chunks(KIND);
  constexpr int kStageBytes = stage_bytes(KIND, PAIR);
  constexpr int kAcc = num_acc(KIND);
  // Block-scaled FP8: the MMA writes each 128-wide K block into one of four
  // partial accumulators (TMEM columns 0..511); the promotion warps add
  // scale_a * scale_b * partial into tile totals held in their registers and
  // run the epilogue from there.
  constexpr bool BLK = KIND == Kind::kFp8Block;
  // Augmented bf16 GEMM: checksum-row M-tiles, and the epilogue also reduces
  // the output-side magnitude |w_c| |v| (R reduced channels in all).
  constexpr bool AUG = KIND == Kind::kBf16 && C > 0;
  constexpr int R = AUG ? 2 * C : C;
  constexpr bool WIDE = is_wide(KIND);
  constexpr int kAccWarps = acc_warps(WIDE);
  constexpr int kEpi0 = epi_warp0(WIDE);
  constexpr uint32_t kAccThreads = 32 * kAccWarps;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~static_cast<uintptr_t>(1023));
  float* red = reinterpret_cast<float*>(smem + kS * kStageBytes);
  // 1024-byte aligned: the stages and the reduction area are multiples of 1 KiB.
  uint8_t* pred_slice = reinterpret_cast<uint8_t*>(red + red_floats(KIND));
  float* pred_q = reinterpret_cast<float*>(pred_slice + pred_slice_bytes(KIND, CHK));
  uint64_t* full = reinterpret_cast<uint64_t*>(reinterpret_cast<uint8_t*>(pred_q) + pred_q_bytes(CHK));
  uint64_t* empty = full + kS;
  uint64_t* acc_full = empty + kS;
  uint64_t* acc_empty = acc_full + 2;
  uint64_t* part_full = acc_empty + 2;
  uint64_t* part_empty = part_full + kPartBufs;
  uint64_t* mma_done = part_empty + kPartBufs;  // the MMA thread's final commit (teardown)
  uint64_t* pred_full = mma_done + 1;            // the prediction's B slice has landed
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(pred_full + 1);
  volatile int32_t* abort_flag = reinterpret_cast<volatile int32_t*>(tmem_slot + 1);
  // Tiles whose epilogue has finished: paces the prediction warps.
  volatile uint32_t* tiles_done = tmem_slot + 2;

  // Warp-uniform by construction (setmaxnreg needs provably uniform branches).
  const int warp = __shfl_sync(0xffffffffu, static_cast<int>(threadIdx.x >> 5), 0);
  const int lane = threadIdx.x & 31;
  // CTA pairs: rank 0 (the leader) issues the MMAs for both CTAs; its
  // barriers count both CTAs' loads and epilogues.
  const uint32_t rank = PAIR ? cluster_ctarank() : 0u;
  const bool leader = rank == 0;
  const int work_first = PAIR ? static_cast<int>(blockIdx.x >> 1) : static_cast<int>(blockIdx.x);
  const int work_step = PAIR ? static_cast<int>(gridDim.x >> 1) : static_cast<int>(gridDim.x);

  if (threadIdx.x == 0) {
    for (int s = 0; s < kS; ++s) {
      mbar_init(full + s, 1);
      mbar_init(empty + s, 1);
    }
    for (int b = 0; b < 2; ++b) {
      // The (leader's) MMA waits for both CTAs' epilogues.
      mbar_init(acc_full + b, 1);
      mbar_init(acc_empty + b, PAIR ? 2 * kAccWarps : kAccWarps);
    }
    for (int b = 0; b < kGroupSlots; ++b) {
      // Block-scaled partial groups: the leader's MMA waits for both CTAs'
      // promotion warps.
      mbar_init(part_full + b, 1);
      mbar_init(part_empty + b, PAIR ? 2 * kAccWarps : kAccWarps);
    }
    mbar_init(mma_done, 1);
    mbar_init(pred_full, 1);
    *abort_flag = 0;
    *tiles_done = 0;
    fence_barrier_init();
  }
  if (warp == 0 && lane == 0) {
    tma_prefetch(&tm_a);
    tma_prefetch(&tm_b);
    if constexpr (KIND == Kind::kNvf4) {
      tma_prefetch(&tm_sfa);
      tma_prefetch(&tm_sfb);
    } else if constexpr (CHK) {
      tma_prefetch(&tm_sfb);  // e4m3: the prediction's B-slice map
    }
  }
  if (warp == 1) {
    if constexpr (PAIR) {
      tmem_alloc_pair(tmem_slot, kTmemCols);
      tmem_relinquish_pair();
    } else {
      tmem_alloc(tmem_slot, kTmemCols);
      tmem_relinquish();
    }
  }
  tc_fence_before();
  __syncthreads();
  // Both CTAs' barriers must be initialised before either touches the other's.
  if constexpr (PAIR) cluster_sync();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  // One 32-column chunk of a finished tile (values after alpha), by the
  // thread owning output row `row`: fault injection, nonfinite check, the
  // observed checksum partials of the warp's 32 rows into `red`, the store.
  auto emit_chunk = [&](float (&v)[32], int q, int row, bool row_ok, int c0, int chunk, const float* w,
                        uint32_t& nonfinite, uint32_t& faulted, float& row_acc) {
    if (C > 0 && p.fbit >= 0 && row == p.frow && p.fcol >= c0 && p.fcol < c0 + 32) {
#pragma unroll
      for (int j = 0; j < 32; ++j) {
        if (c0 + j == p.fcol) v[j] = __uint_as_float(__float_as_uint(v[j]) ^ (1u << p.fbit));
      }
      atomicOr(p.hit, 1);
      faulted |= 1u << (chunk >> 2);  // bit per 128-column block of the tile
    }
    if constexpr (C > 0) {
      if (p.row_observed != nullptr) {
        // Row sums per 64-column block (chunks 2b and 2b + 1): columns in
        // ascending order from +0, only those < n.
        float sum = (chunk & 1) ? row_acc : 0.f;
#pragma unroll
        for (int j = 0; j < 32; ++j) {
          if (c0 + j < p.n) sum = __fadd_rn(sum, v[j]);
        }
        if (chunk & 1) {
          if (row_ok && c0 - 32 < p.n) p.row_observed[static_cast<int64_t>(c0 >> 6) * p.m + row] = sum;
        } else {
          row_acc = sum;
        }
      }
    }
    if constexpr (BF16OUT) {
      // The output as stored first: one round-to-nearest conversion per
      // column pair. Its words also give the non-finite test: a bf16 exponent
      // of all ones is inf or NaN as stored (the cast overflows from
      // |x| >= 0x7F7F8000, the tie above the largest finite bf16 rounding to
      // the even pattern, +inf); adding 0x80 to an all-ones exponent field
      // sets the half's top bit, and no other exponent does.
      uint32_t packed[16];
#pragma unroll
      for (int j = 0; j < 16; ++j) packed[j] = bf16x2_bits(v[2 * j], v[2 * j + 1]);
      const bool full = c0 + 32 <= p.n;
      if (C > 0 && (AUG || p.nonfinite != nullptr) && row_ok) {
        uint32_t flag = 0;
        if (full) {
#pragma unroll
          for (int j = 0; j < 16; ++j) flag |= (packed[j] & 0x7F807F80u) + 0x00800080u;
        } else {
#pragma unroll
          for (int j = 0; j < 16; ++j) {
            const uint32_t keep = (c0 + 2 * j < p.n ? 0x0000FFFFu : 0u) | (c0 + 2 * j + 1 < p.n ? 0xFFFF0000u : 0u);
            flag |= ((packed[j] & keep) & 0x7F807F80u) + 0x00800080u;
          }
        }
        if (flag & 0x80008000u) nonfinite |= 1u << (chunk >> 2);
      }
      if (row_ok) {
        uint16_t* d = static_cast<uint16_t*>(p.d) + static_cast<int64_t>(row) * p.n;
        if (full && (p.n & 7) == 0) {
          uint4* dst = reinterpret_cast<uint4*>(d + c0);
#pragma unroll
          for (int j = 0; j < 4; ++j) {
            dst[j] = make_uint4(packed[4 * j], packed[4 * j + 1], packed[4 * j + 2], packed[4 * j + 3]);
          }
        } else {
#pragma unroll
          for (int j = 0; j < 32; ++j) {
            if (c0 + j < p.n) d[c0 + j] = static_cast<uint16_t>((j & 1) ? packed[j >> 1] >> 16 : packed[j >> 1]);
          }
        }
      }
    } else if (C > 0 && p.nonfinite != nullptr && row_ok) {
      // Non-finite as stored: fp32 from 0x7F800000 up.
      uint32_t largest = 0;
#pragma unroll
      for (int j = 0; j < 32; ++j) {
        if (c0 + j < p.n) largest = max(largest, __float_as_uint(v[j]) & 0x7FFFFFFFu);
      }
      if (largest >= 0x7F800000u) nonfinite |= 1u << (chunk >> 2);
    }
    if constexpr (C > 0) {
      // Column sums of w_c[row] * v over the warp's 32 rows. The first
      // butterfly level (lane bit 16) runs for all channels at once: the
      // selects of v are shared, and the kept half's weight fuses into the
      // add. Lane j ends with column j.
      const bool upper = (lane & 16) != 0;
      float x[C][16];
#pragma unroll
      for (int i = 0; i < 16; ++i) {
        const float sent = upper ? v[i] : v[i + 16];
        const float kept = upper ? v[i + 16] : v[i];
#pragma unroll
        for (int c = 0; c < C; ++c) x[c][i] = fmaf(w[c], kept, __shfl_xor_sync(0xffffffffu, w[c] * sent, 16));
      }
#pragma unroll
      for (int c = 0; c < C; ++c) red[((chunk * 4 + q) * R + c) * 32 + lane] = transpose_reduce(x[c], lane);
      if constexpr (AUG) {
        // Output-side magnitude sum_rows |w_c v| = sum_rows |w_c| |v|, in the
        // same butterfly order as the observed sum.
#pragma unroll
        for (int i = 0; i < 16; ++i) {
          const float sent = fabsf(upper ? v[i] : v[i + 16]);
          const float kept = fabsf(upper ? v[i + 16] : v[i]);
#pragma unroll
          for (int c = 0; c < C; ++c) {
            const float wa = fabsf(w[c]);
            x[c][i] = fmaf(wa, kept, __shfl_xor_sync(0xffffffffu, wa * sent, 16));
          }
        }
#pragma unroll
        for (int c = 0; c < C; ++c) red[((chunk * 4 + q) * R + C + c) * 32 + lane] = transpose_reduce(x[c], lane);
      }
    }
    if constexpr (!BF16OUT) {
      if (row_ok) {
        float* d = static_cast<float*>(p.d);
#pragma unroll
        for (int j = 0; j < 32; ++j) {
          if (c0 + j < p.n) d[static_cast<int64_t>(c0 + j) * p.m + row] = v[j];
        }
      }
    }
  };
  // After every chunk of a tile: the observed checksum of each column is the
  // sum of the four lane quarters' 32-row partials (all epilogue threads).
  auto store_observed = [&](int mt, int n0, bool live) {
    if constexpr (C > 0) {
      named_barrier(1, kAccThreads);
      if (live) {
        const int e = static_cast<int>(threadIdx.x) - 32 * kEpi0;
        for (int idx = e; idx < kTileChunks * R * 32; idx += kAccThreads) {
          const int chunk = idx / (R * 32);
          const int rem = idx - chunk * R * 32;
          const int r = rem >> 5;
          const int col = rem & 31;
          float sum = 0.f;
#pragma unroll
          for (int qq = 0; qq < 4; ++qq) sum += red[((chunk * 4 + qq) * R + r) * 32 + col];
          const int gcol = n0 + chunk * 32 + col;
          if (gcol < p.padded_n && mt < p.tiles_m) {
            // Channels r >= C (augmented only) are the output magnitudes.
            float* plane = r < C ? p.observed : p.magnitude;
            const int c = r < C ? r : r - C;
            plane[(static_cast<int64_t>(c) * p.tiles_m + mt) * p.padded_n + gcol] = sum;
          }
        }
      }
      named_barrier(1, kAccThreads);
    }
  };
  // Augmented bf16: the status (bit 0 fault applied, bit 1 non-finite
  // output) of each 128 x 128 block of this CTA's tile, ORed into its flag
  // word. Every epilogue thread takes part (the decisions are CTA-uniform).
  auto store_tile_flags = [&](int mt, int nt, uint32_t faulted, uint32_t nonfinite) {
    if constexpr (AUG) {
#pragma unroll
      for (int block = 0; block < kTN / 128; ++block) {
        const bool any_fault = named_barrier_or(1, kAccThreads, (faulted >> block) & 1u);
        const bool any_nonfinite = named_barrier_or(1, kAccThreads, (nonfinite >> block) & 1u);
        const int col_block = nt * (kTN / 128) + block;
        const int32_t word = (any_fault ? 1 : 0) | (any_nonfinite ? 2 : 0);
        if (p.tile_flags != nullptr && threadIdx.x == 32 * kEpi0 && mt < p.tiles_m && word != 0 &&
            col_block < p.flag_cols) {
          atomicOr(p.tile_flags + static_cast<int64_t>(mt) * p.flag_cols + col_block, word);
        }
      }
    }
  };

  if (warp < kEpi0) {
    // Warps 0-1 (wide kinds: warpgroup 0, warps 2-3 idle).
    if constexpr (WIDE) setmaxnreg_dec<kLowRegs>();
  if (warp == 0) {
    // ---------------- TMA producer ----------------
    if (lane == 0) {
      uint32_t kbg = 0;
      bool stop = false;
      bool encoded = false;  // augmented: the encode grid's rows are visible
      for (int t = work_first; t < p.num_work && !stop; t += work_step) {
        int mt, nt;
        work_coords<PAIR>(t, p, rank, mt, nt);
        for (int kb = 0; kb < p.num_kb; ++kb, ++kbg) {
          const int s = kbg % kS;
          if (kbg >= kS &&
              !mbar_wait_own_limit(empty + s, ((kbg / kS) - 1) & 1, kWaitEmpty, abort_flag, p.watchdog,
                                   p.wait_limit_ns)) {
            stop = true;
            break;
          }
          uint8_t* sa = smem + s * kStageBytes;
          uint8_t* sb = sa + kABytes;
          // Augmented bf16: the M-tiles after the data tiles read the checksum
          // rows (tensor map tm_sfa), from row 0 of that matrix.
          const bool aug_tile = AUG && mt >= p.tiles_m;
          if (aug_tile && !encoded) {
            // Launched as a programmatic dependent of the encode kernel: the
            // checksum rows exist once that grid has completed.
            griddep_wait();
            encoded = true;
          }
          const CUtensorMap* map_a = aug_tile ? &tm_sfa : &tm_a;
          const int32_t row_a = (aug_tile ? mt - p.tiles_m : mt) * kBM;
          if constexpr (PAIR) {
            // Both halves complete on the leader's barrier, which expects both.
            const uint32_t bar = mapa_shared(full + s, 0);
            if (leader) mbar_arrive_expect_tx(full + s, 2 * kStageBytes);
            tma_load_2d_pair(sa, map_a, bar, kb * kBKBytes, row_a);
            tma_load_2d_pair(sb, &tm_b, bar, kb * kBKBytes, nt * kTN + static_cast<int>(rank) * (kTN / 2));
            if constexpr (KIND == Kind::kNvf4) {
              // Own A scales; the B scales of all the tile's rows (each CTA's
              // accumulator spans every column of the tile).
              uint8_t* ssfa = sb + kBStage;
              uint8_t* ssfb = ssfa + kSfaBytes;
              tma_load_4d_pair(ssfa, &tm_sfa, bar, 0, 0, kb * 4, mt);
              tma_load_4d_pair(ssfb, &tm_sfb, bar, 0, 0, kb * 4, nt * sfb_groups(KIND));
            }
            continue;
          }
          mbar_arrive_expect_tx(full + s, kStageBytes);
          tma_load_2d(sa, map_a, full + s, kb * kBKBytes, row_a);
          tma_load_2d(sb, &tm_b, full + s, kb * kBKBytes, nt * kTN);
          if constexpr (KIND == Kind::kNvf4) {
            uint8_t* ssfa = sb + kBStage;
            uint8_t* ssfb = ssfa + kSfaBytes;
            tma_load_4d(ssfa, &tm_sfa, full + s, 0, 0, kb * 4, mt);
            tma_load_4d(ssfb, &tm_sfb, full + s, 0, 0, kb * 4, nt * sfb_groups(KIND));
          }
        }
      }
      // Teardown: the last stages issued have landed (after a clean run the
      // MMA already consumed them), so no copy writes shared memory after
      // the CTA leaves. A pair's loads all complete on the leader's barriers.
      if (leader) {
        for (uint32_t j = kbg > static_cast<uint32_t>(kS) ? kbg - kS : 0u; j < kbg; ++j) {
          if (!mbar_drain(full + j % kS, (j / kS) & 1)) *abort_flag = kWaitOther;
        }
      }
    }
  } else if (warp == 1 && BLK) {
    // ---------------- MMA issuer, block-scaled: one partial per K block ----------------
    if (lane == 0 && leader) {
      constexpr uint32_t idesc = idesc_e4m3(PAIR ? 2 * kBM : kBM, kTN);
      uint32_t kbg = 0, gg = 0;
      bool stop = false;
      for (int t = work_first; t < p.num_work && !stop; t += work_step) {
        // Groups of kGroupKb K blocks of one tile (the last may be shorter).
        for (int kb0 = 0; kb0 < p.num_kb && !stop; kb0 += kGroupKb, ++gg) {
          const uint32_t gs = gg % kGroupSlots;
          if (gg >= kGroupSlots &&
              !mbar_wait(part_empty + gs, ((gg / kGroupSlots) - 1) & 1, kWaitAccumFree, abort_flag, p.watchdog, p.wait_limit_ns)) {
            stop = true;
            break;
          }
          const int kb_end = min(kb0 + kGroupKb, p.num_kb);
          for (int kb = kb0; kb < kb_end; ++kb, ++kbg) {
            const int s = kbg % kS;
            if (!mbar_wait(full + s, (kbg / kS) & 1, kWaitFull, abort_flag, p.watchdog, p.wait_limit_ns)) {
              stop = true;
              break;
            }
            tc_fence_after();
            const uint32_t sa = smem_u32(smem + s * kStageBytes);
            const uint32_t sb = sa + kABytes;
            const uint32_t d_tmem = tmem + (gs * kGroupKb + (kb - kb0)) * kTN;
#pragma unroll
            for (int j = 0; j < 4; ++j) {
              const uint32_t acc = j > 0 ? 1u : 0u;
              if constexpr (PAIR) {
                mma_f8f6f4_pair(d_tmem, sw128_desc(sa + 32 * j), sw128_desc(sb + 32 * j), idesc, acc);
              } else {
                mma_f8f6f4(d_tmem, sw128_desc(sa + 32 * j), sw128_desc(sb + 32 * j), idesc, acc);
              }
            }
            if constexpr (PAIR) {
              tc_commit_pair(empty + s, 0x3);
            } else {
              tc_commit(empty + s);
            }
          }
          if (stop) break;
          if constexpr (PAIR) {
            tc_commit_pair(part_full + gs, 0x3);
          } else {
            tc_commit(part_full + gs);
          }
        }
      }
      // Teardown: every MMA issued has completed before TMEM is released.
      if constexpr (PAIR) {
        tc_commit_pair(mma_done, 0x1);
      } else {
        tc_commit(mma_done);
      }
      if (!mbar_drain(mma_done, 0)) *abort_flag = kWaitOther;
    }
  } else if (warp == 1) {
    // ---------------- MMA issuer ----------------
    if (lane == 0 && leader) {
      constexpr int kMmaM = PAIR ? 2 * kBM : kBM;
      constexpr uint32_t idesc = KIND == Kind::kFp8    ? idesc_e4m3(kMmaM, kTN)
                                 : KIND == Kind::kBf16 ? idesc_bf16(kMmaM, kTN)
                                                       : idesc_nvf4(kMmaM, kTN);
      uint32_t kbg = 0;
      int i = 0;
      for (int t = work_first; t < p.num_work && !*abort_flag; t += work_step, ++i) {
        const int b = i % kAcc;
        if (i >= kAcc) {
          if (!mbar_wait(acc_empty + b, ((i / kAcc) - 1) & 1, kWaitAccumFree, abort_flag, p.watchdog, p.wait_limit_ns)) break;
          tc_fence_after();
        }
        const uint32_t d_tmem = tmem + b * kTN;
        for (int kb = 0; kb < p.num_kb; ++kb, ++kbg) {
          const int s = kbg % kS;
          if (!mbar_wait(full + s, (kbg / kS) & 1, kWaitFull, abort_flag, p.watchdog, p.wait_limit_ns)) break;
          tc_fence_after();
          const uint32_t sa = smem_u32(smem + s * kStageBytes);
          const uint32_t sb = sa + kABytes;
          if constexpr (KIND == Kind::kNvf4) {
            // Pairs: one copy moves each CTA's staged scales into its own TMEM.
            const uint32_t ssfa = sb + kBStage;
            const uint32_t ssfb = ssfa + kSfaBytes;
#pragma unroll
            for (int j = 0; j < 4; ++j) {
              tmem_cp_32x128b_x4<PAIR>(tmem + kSfaCol + 4 * j, sf_desc(ssfa + 512 * j));
#pragma unroll
              for (int g = 0; g < sfb_groups(KIND); ++g) {
                tmem_cp_32x128b_x4<PAIR>(tmem + kSfbCol + 4 * (sfb_groups(KIND) * j + g),
                                         sf_desc(ssfb + 2048 * g + 512 * j));
              }
            }
          }
#pragma unroll
          for (int j = 0; j < 4; ++j) {
            const uint64_t adesc = sw128_desc(sa + 32 * j);
            const uint64_t bdesc = sw128_desc(sb + 32 * j);
            const uint32_t acc = (kb > 0 || j > 0) ? 1u : 0u;
            if constexpr (KIND == Kind::kFp8) {
              if constexpr (PAIR) {
                mma_f8f6f4_pair(d_tmem, adesc, bdesc, idesc, acc);
              } else {
                mma_f8f6f4(d_tmem, adesc, bdesc, idesc, acc);
              }
            } else if constexpr (KIND == Kind::kBf16) {
              // 16 bf16 K per MMA: 32 bytes of the swizzle atom, as for e4m3.
              mma_bf16<PAIR>(d_tmem, adesc, bdesc, idesc, acc);
            } else {
              mma_nvf4<PAIR>(d_tmem, adesc, bdesc, idesc, tmem + kSfaCol + 4 * j,
                             tmem + kSfbCol + 4 * sfb_groups(KIND) * j, acc);
            }
          }
          // Frees the stage in both CTAs (pairs) once these MMAs have read it.
          if constexpr (PAIR) {
            tc_commit_pair(empty + s, 0x3);
          } else {
            tc_commit(empty + s);
          }
        }
        if constexpr (PAIR) {
          tc_commit_pair(acc_full + b, 0x3);
        } else {
          tc_commit(acc_full + b);
        }
      }
      // Teardown: every MMA issued has completed before TMEM is released.
      if constexpr (PAIR) {
        tc_commit_pair(mma_done, 0x1);
      } else {
        tc_commit(mma_done);
      }
      if (!mbar_drain(mma_done, 0)) *abort_flag = kWaitOther;
    }
    }
  } else if (BLK && warp < kEpi0 + kAccWarps) {
    // ------- promotion + epilogue (block-scaled): total += sa * sb * partial -------
    if constexpr (BLK) {
      setmaxnreg_inc<epilogue_regs(CHK)>();
      constexpr int kHalfCols = kTN / 2;
      const int q = warp & 3;                // TMEM lane quarter this warp may access
      const int half = (warp - kEpi0) >> 2;  // 64-column half of the tile
      const uint32_t lane_base = (static_cast<uint32_t>(q * 32) << 16) + static_cast<uint32_t>(half * kHalfCols);
      uint32_t gg = 0;
      int i = 0;
      for (int t = work_first; t < p.num_work; t += work_step, ++i) {
        int mt, nt;
        work_coords<PAIR>(t, p, rank, mt, nt);
        const int n0 = nt * kTN;
        const int row = mt * kBM + q * 32 + lane;
        const bool row_ok = row < p.m;
        float w[C > 0 ? C : 1];
#pragma unroll
        for (int c = 0; c < C; ++c) w[c] = row_ok ? p.weights[static_cast<int64_t>(c) * p.m + row] : 0.f;
        const float* sa_row = p.sa + static_cast<int64_t>(row_ok ? row : 0) * p.k_blocks;
        const float* sb_blk = p.sb + static_cast<int64_t>(nt) * p.k_blocks;  // 128-wide tile = one B block
        // Column pairs (2j, 2j + 1) of this warp's half; -0 keeps
        // fma(s, x, total) equal to s * x (sign of zero included) on the first block.
        float2 total[kHalfCols / 2];
#pragma unroll
        for (int j = 0; j < kHalfCols / 2; ++j) total[j] = make_float2(-0.f, -0.f);
        // This group's scales; the next group's load under this group's wait.
        float sa_next[kGroupKb], sb_next[kGroupKb];
#pragma unroll
        for (int e = 0; e < kGroupKb; ++e) {
          const bool in = e < p.num_kb;
          sa_next[e] = in && row_ok ? __ldg(sa_row + e) : 0.f;
          sb_next[e] = in ? __ldg(sb_blk + e) : 0.f;
        }
        bool ok = !*abort_flag;
        for (int kb0 = 0; kb0 < p.num_kb && ok; kb0 += kGroupKb, ++gg) {
          float2 s2[kGroupKb];
#pragma unroll
          for (int e = 0; e < kGroupKb; ++e) {
            const float scale = __fmul_rn(sa_next[e], sb_next[e]);
            s2[e] = make_float2(scale, scale);
            const int kn = kb0 + kGroupKb + e;
            if (kn < p.num_kb) {
              sa_next[e] = row_ok ? __ldg(sa_row + kn) : 0.f;
              sb_next[e] = __ldg(sb_blk + kn);
            }
          }
          const int n_in = min(kGroupKb, p.num_kb - kb0);
          const uint32_t gs = gg % kGroupSlots;
          if (!mbar_wait(part_full + gs, (gg / kGroupSlots) & 1, kWaitAccum, abort_flag, p.watchdog, p.wait_limit_ns)) {
            ok = false;
            break;
          }
          tc_fence_after();
#pragma unroll
          for (int e = 0; e < kGroupKb; ++e) {
            if (e < n_in) {
              const uint32_t col = lane_base + static_cast<uint32_t>((gs * kGroupKb + e) * kTN);
              uint32_t lo[32], hi[32];
              tmem_ld_32x32b_x32(tmem + col, lo);
              tmem_ld_32x32b_x32(tmem + col + 32, hi);
              tmem_ld_wait();
#pragma unroll
              for (int j = 0; j < 16; ++j) {
                total[j] =
                    fma2(s2[e], make_float2(__uint_as_float(lo[2 * j]), __uint_as_float(lo[2 * j + 1])), total[j]);
                total[16 + j] = fma2(s2[e], make_float2(__uint_as_float(hi[2 * j]), __uint_as_float(hi[2 * j + 1])),
                                     total[16 + j]);
              }
            }
          }
          // The group's partials are in registers: hand the buffers back to
          // the (leader's) MMA warp.
          tc_fence_before();
          __syncwarp();
          if (lane == 0) {
            if constexpr (PAIR) {
              mbar_arrive_cluster(mapa_shared(part_empty + gs, 0));
            } else {
              mbar_arrive(part_empty + gs);
            }
          }
        }
        const bool live = !named_barrier_or(1, kAccThreads, !ok || *abort_flag != 0);
        if (live) {
          uint32_t nonfinite = 0, faulted = 0;
          float row_acc = 0.f;  // row sum of the current 64-column block
#pragma unroll
          for (int cc = 0; cc < kHalfCols / 32; ++cc) {
            float v[32];
#pragma unroll
            for (int j = 0; j < 16; ++j) {
              v[2 * j] = total[cc * 16 + j].x;
              v[2 * j + 1] = total[cc * 16 + j].y;
            }
            const int chunk = half * (kHalfCols / 32) + cc;
            emit_chunk(v, q, row, row_ok, n0 + chunk * 32, chunk, w, nonfinite, faulted, row_acc);
          }
          if (nonfinite) atomicExch(p.nonfinite, 1);
        }
        store_observed(mt, n0, live);
        if (threadIdx.x == 32 * kEpi0) *tiles_done = static_cast<uint32_t>(i + 1);
        if (!live) break;
      }
    }
  } else if (!BLK && warp < kEpi0 + kAccWarps) {
    // ---------------- epilogue ----------------
    if constexpr (WIDE) setmaxnreg_inc<epilogue_regs(CHK)>();
    const int q = warp & 3;  // TMEM lane quarter this warp may access
    constexpr int kWarpChunks = kTileChunks * 4 / kAccWarps;  // 32-column chunks per warp
    const int first_chunk = ((warp - kEpi0) >> 2) * kWarpChunks;
    // bf16 GEMMs have no alpha: the fp32 accumulator is the value (times 1).
    const float alpha = KIND == Kind::kBf16 ? 1.f : *p.alpha;
    // Augmented: the weights and the zeroed status words come from the encode
    // grid this launch may overlap (programmatic dependent launch).
    if constexpr (AUG) griddep_wait();
    int i = 0;
    for (int t = work_first; t < p.num_work; t += work_step, ++i) {
      int mt, nt;
      work_coords<PAIR>(t, p, rank, mt, nt);
      const int m0 = mt * kBM, n0 = nt * kTN;
      const int row = m0 + q * 32 + lane;
      const bool row_ok = row < p.m;
      // Augmented bf16: tiles past the data tiles hold checksum rows, whose
      // results are the predicted partials (row t * C + c -> predicted[c][t]).
      const bool checksum_tile = AUG && mt >= p.tiles_m;
      const int aug_row = (mt - p.tiles_m) * kBM + q * 32 + lane;
      float w[C > 0 ? C : 1];
#pragma unroll
      for (int c = 0; c < C; ++c) w[c] = row_ok ? p.weights[static_cast<int64_t>(c) * p.m + row] : 0.f;
      const int b = i % kAcc;
      const bool ready = mbar_wait(acc_full + b, (i / kAcc) & 1, kWaitAccum, abort_flag, p.watchdog, p.wait_limit_ns);
      const bool live = !named_barrier_or(1, kAccThreads, !ready || *abort_flag != 0);
      tc_fence_after();
      const uint32_t acc_col = (static_cast<uint32_t>(q * 32) << 16) + b * kTN;
      // All of this warp's accumulator columns are in registers: hand the
      // buffer back to the (leader's) MMA warp before the remaining math.
      auto release = [&]() {
        tc_fence_before();
        __syncwarp();
        if (lane == 0) {
          if constexpr (PAIR) {
            mbar_arrive_cluster(mapa_shared(acc_empty + b, 0));  // the leader's MMA waits on both CTAs
          } else {
            mbar_arrive(acc_empty + b);
          }
        }
      };
      uint32_t nonfinite = 0, faulted = 0;
      float row_acc = 0.f;  // row sum of the current 64-column block
      if (live) {
        if constexpr (WIDE) {
          uint32_t r[kWarpChunks][32];
#pragma unroll
          for (int cc = 0; cc < kWarpChunks; ++cc) tmem_ld_32x32b_x32(tmem + acc_col + (first_chunk + cc) * 32, r[cc]);
          tmem_ld_wait();
          release();
#pragma unroll
          for (int cc = 0; cc < kWarpChunks; ++cc) {
            float v[32];
#pragma unroll
            for (int j = 0; j < 32; ++j) v[j] = __fmul_rn(alpha, __uint_as_float(r[cc][j]));
            const int chunk = first_chunk + cc;
            emit_chunk(v, q, row, row_ok, n0 + chunk * 32, chunk, w, nonfinite, faulted, row_acc);
          }
        } else {
#pragma unroll 1
          for (int chunk = 0; chunk < kTileChunks; ++chunk) {
            uint32_t r[32];
            tmem_ld_32x32b_x32(tmem + acc_col + chunk * 32, r);
            tmem_ld_wait();
            if (chunk == kTileChunks - 1) release();
            float v[32];
#pragma unroll
            for (int j = 0; j < 32; ++j) v[j] = __fmul_rn(alpha, __uint_as_float(r[j]));
            if (checksum_tile) {
              if (aug_row < p.aug_rows) {
                const int c = aug_row % (C > 0 ? C : 1), tile = aug_row / (C > 0 ? C : 1);
                float* dst = p.predicted + (static_cast<int64_t>(c) * p.tiles_m + tile) * p.padded_n;
#pragma unroll
                for (int j = 0; j < 32; ++j) {
                  const int col = n0 + chunk * 32 + j;
                  if (col < p.padded_n) dst[col] = v[j];
                }
              }
            } else {
              emit_chunk(v, q, row, row_ok, n0 + chunk * 32, chunk, w, nonfinite, faulted, row_acc);
            }
          }
        }
        if (nonfinite && p.nonfinite != nullptr) atomicExch(p.nonfinite, 1);
      }
      store_tile_flags(mt, nt, faulted, nonfinite);
      store_observed(mt, n0, live && !checksum_tile);
      if (threadIdx.x == 32 * kEpi0) *tiles_done = static_cast<uint32_t>(i + 1);
      if (!live) break;
    }
  } else if constexpr (CHK) {
    if (is_prediction_warp<WIDE>(warp)) {
      // ---------------- input-side prediction (4 warps) ----------------
      // Independent of the MMA pipeline: for each of this CTA's tiles, the
      // slices s = mt, mt + Tm, ... (ascending) of the tile's 256 B rows are
      // read from global memory (hot in L2: the same column block is streaming
      // through this SM) and folded into fma chains with q_full.
      // 0..127: the tile's B rows ct (and ct + 128 for 256-wide tiles).
      const int ct = prediction_index<WIDE>(warp) * 32 + lane;
      constexpr int kRowsPerThread = kTN / 128;
      const float alpha = BLK ? 1.f : *p.alpha;
      const int num_slices = (p.k + kSliceK - 1) / kSliceK;
      const int64_t row_bytes = is_e4m3(KIND) ? p.k : p.k / 2;
      const int64_t k_atoms = (p.k + 63) / 64;
      const int64_t k_pad = static_cast<int64_t>(num_slices) * kSliceK;
      // Pacing: this work is spread over the CTA's tiles (projection during
      // the first half, prediction during the second) instead of running in
      // bursts, which would take L2 bandwidth from the TMA loads feeding the
      // tensor cores. A wait returns false once the CTA has aborted.
      const uint32_t my_tiles =
          work_first < p.num_work ? static_cast<uint32_t>((p.num_work - 1 - work_first) / work_step + 1) : 0u;
      const uint32_t half = my_tiles / 2;
      auto pace = [&](uint32_t target) -> bool {
        target += static_cast<uint32_t>(p.pace_extra);
        if (*tiles_done >= target) return true;
        const uint64_t start = global_ns();
        while (*tiles_done < target) {
          if (*abort_flag) return false;
          if (global_ns() - start > p.wait_limit_ns) {
            atomicCAS(p.watchdog, 0, kWaitPace);
            *abort_flag = kWaitPace;
            return false;
          }
          __nanosleep(500);
        }
        return true;
      };
      if (!p.q_ready) {
        // ---- phase 1: per-band projection partials (project_item, kslice.cuh),
        // spread over the first half of the CTA's tiles.
        {
          const ProjectionView view{p.a, p.sa, p.sfa, p.weights, p.m, p.k, p.k_blocks, num_slices, p.q_part};
          const int64_t items = static_cast<int64_t>(num_slices) * p.q_bands;
          const int64_t first_item = static_cast<int64_t>(blockIdx.x) * 4 + prediction_index<WIDE>(warp);
          const int64_t item_step = static_cast<int64_t>(gridDim.x) * 4;
          const int64_t my_items = first_item < items ? (items - 1 - first_item) / item_step + 1 : 0;
          int64_t j = 0;
          for (int64_t item = first_item; item < items && !*abort_flag; item += item_step, ++j) {
            // A few items (a short M) run at once: pacing only matters when
            // the projection is large enough to take L2 bandwidth from the
            // mainloop's loads.
            if (my_items > kPacedItems && !pace(static_cast<uint32_t>(j * half / my_items))) break;
            const int64_t band = item / num_slices, chunk = item % num_slices;
            project_item<KIND, C>(view, band, chunk, lane, band_partial<C>(view, band, chunk));
          }
        }
        // ---- phase 2: q_full = sum over bands (ascending) ----
        if (prediction_grid_barrier(p.grid_sync, gridDim.x, ct, abort_flag, p.watchdog, p.wait_limit_ns)) {
          const int64_t entries = k_pad * C * 2;
          for (int64_t e = static_cast<int64_t>(blockIdx.x) * 128 + ct; e < entries;
               e += static_cast<int64_t>(gridDim.x) * 128) {
            // Bands in ascending order; their loads batched ahead of the adds.
            float acc = __ldcg(p.q_part + e);
            int b = 1;
            for (; b + 8 <= p.q_bands; b += 8) {
              float x[8];
#pragma unroll
              for (int i = 0; i < 8; ++i) x[i] = __ldcg(p.q_part + (b + i) * entries + e);
#pragma unroll
              for (int i = 0; i < 8; ++i) acc = __fadd_rn(acc, x[i]);
            }
            for (; b < p.q_bands; ++b) acc = __fadd_rn(acc, __ldcg(p.q_part + b * entries + e));
            p.q_full[e] = acc;
          }
        }
        prediction_grid_barrier(p.grid_sync, 2 * gridDim.x, ct, abort_flag, p.watchdog, p.wait_limit_ns);
      } else {
        // q_full was written by the kernels before this launch.
        griddep_wait();
      }
      // ---- phase 3: predictions of this CTA's tiles ----
      const uint32_t last = my_tiles > 0 ? my_tiles - 1 : 0u;
      const uint32_t start = min(static_cast<uint32_t>(*tiles_done), last);
      uint32_t jt = 0;
      uint32_t slices_staged = 0;  // B slices copied to shared memory (e4m3)
      bool copy_in_flight = false;  // thread ct == 0: a slice copy not yet seen landing
      bool stopped = false;
      // Every decision to leave is taken by all 128 prediction threads
      // together (named_barrier_or), since the slice loop synchronises them.
      for (int t = work_first; t < p.num_work; t += work_step, ++jt) {
        // Spread over the tiles still to come when the projection finished
        // (the second half for a long M, almost all of them for a short one).
        const bool paced = pace(start + jt * (last > start ? last - start : 0u) / (my_tiles > 0 ? my_tiles : 1u));
        if (named_barrier_or(2, 128, !paced || *abort_flag != 0)) break;
        int mt, nt;
        work_coords<PAIR>(t, p, rank, mt, nt);
        if (mt >= p.tiles_m) continue;
        // Per row and channel: the value chain (.x) and the magnitude chain
        // (.y), advanced together by one f32x2 fma (two independent fmas).
        float2 acc[kRowsPerThread][C];
#pragma unroll
        for (int h = 0; h < kRowsPerThread; ++h)
#pragma unroll
          for (int c = 0; c < C; ++c) acc[h][c] = make_float2(0.f, 0.f);
        // e4m3: one thread copies each slice of the tile's B rows into
        // shared memory (rows past N and K past the row read as zeros); the
        // next slice's copy is issued as soon as every prediction thread holds
        // the current one in registers, so it lands while that one is summed.
        auto copy_slice = [&](int sl_copy) {
          if (ct == 0) {
            fence_proxy_async_smem();
            mbar_arrive_expect_tx(pred_full, static_cast<uint32_t>(pred_slice_bytes(KIND, CHK)));
            tma_load_2d(pred_slice, &tm_sfb, pred_full, sl_copy * kSliceK, nt * kTN);
            copy_in_flight = true;
          }
        };
        if constexpr (is_e4m3(KIND)) {
          if (mt < num_slices) copy_slice(mt);
        }
        for (int sl = mt; sl < num_slices; sl += p.tiles_m) {
          const int k0 = sl * kSliceK;
          constexpr int kChunksPerSlice = is_e4m3(KIND) ? 4 : 2;  // 16-byte chunks per row
          uint4 raw[kRowsPerThread][kChunksPerSlice];
          uint32_t sfw[kRowsPerThread];
          bool landed = true;
          if constexpr (is_e4m3(KIND)) {
            landed = mbar_wait(pred_full, slices_staged & 1u, kWaitProjection, abort_flag, p.watchdog, p.wait_limit_ns);
            if (ct == 0 && landed) copy_in_flight = false;
            ++slices_staged;
          }
#pragma unroll
          for (int h = 0; h < kRowsPerThread; ++h) {
            const int64_t r = static_cast<int64_t>(nt) * kTN + ct + 128 * h;
            const bool row_in = r < p.n;
            if constexpr (is_e4m3(KIND)) {
              // 64-byte swizzle: chunk c of slice row q sits at q*64 + ((c ^ ((q >> 1) & 3)) << 4).
              const int q = ct + 128 * h;
#pragma unroll
              for (int ch = 0; ch < kChunksPerSlice; ++ch) {
                raw[h][ch] = landed ? *reinterpret_cast<const uint4*>(pred_slice + q * 64 + ((ch ^ ((q >> 1) & 3)) << 4))
                                    : make_uint4(0, 0, 0, 0);
              }
            } else {
              const uint8_t* src = p.b + r * row_bytes + k0 / 2;
#pragma unroll
              for (int ch = 0; ch < kChunksPerSlice; ++ch) {
                const int byte = k0 / 2 + ch * 16;
                raw[h][ch] = (row_in && byte < row_bytes) ? __ldg(reinterpret_cast<const uint4*>(src) + ch)
                                                           : make_uint4(0, 0, 0, 0);
              }
            }
            if constexpr (KIND == Kind::kNvf4) {
              const int64_t off = ((r >> 7) * k_atoms + (k0 >> 6)) * 512 + (r & 31) * 16 + ((r >> 5) & 3) * 4;
              sfw[h] = row_in ? __ldg(reinterpret_cast<const uint32_t*>(p.sfb + off)) : 0u;
            } else if constexpr (BLK) {
              // The scale of this row's 128 x 128 block holding the slice.
              sfw[h] = row_in ? __float_as_uint(__ldg(p.sb + (r >> 7) * p.k_blocks + (k0 >> 7))) : 0u;
            }
          }
          if constexpr (is_e4m3(KIND)) {
            // The slice is in registers (or its copy failed everywhere).
            if (named_barrier_or(2, 128, !landed)) {
              stopped = true;
              break;
            }
            // No thread reads this slice's buffer any more: it takes the next.
            if (sl + p.tiles_m < num_slices) copy_slice(sl + p.tiles_m);
          }
          // The slice's q in shared memory: one batch of L2 loads (q_full was
          // written by other CTAs during this launch, so they bypass L1)
          // instead of a round trip per 8 k. q_full is zero-padded to a
          // multiple of 64 K, so the loads need no guard.
          named_barrier(2, 128);  // the previous slice's reads of pred_q are done
          if (ct < kSliceK * C * 2 / 4) {
            reinterpret_cast<float4*>(pred_q)[ct] =
                __ldcg(reinterpret_cast<const float4*>(p.q_full + static_cast<int64_t>(k0) * C * 2) + ct);
          }
          named_barrier(2, 128);
          // NVFP4: each row's four block scales of the slice as fp16 pairs (s, s).
          uint32_t scale_h2[kRowsPerThread][4];
          if constexpr (KIND == Kind::kNvf4) {
#pragma unroll
            for (int h = 0; h < kRowsPerThread; ++h) {
              const uint32_t lo = e4m3x2_to_h2(sfw[h] & 0xFFFFu), hi = e4m3x2_to_h2(sfw[h] >> 16);
              scale_h2[h][0] = __byte_perm(lo, 0, 0x1010);
              scale_h2[h][1] = __byte_perm(lo, 0, 0x3232);
              scale_h2[h][2] = __byte_perm(hi, 0, 0x1010);
              scale_h2[h][3] = __byte_perm(hi, 0, 0x3232);
            }
          }
#pragma unroll
          for (int e0 = 0; e0 < kSliceK; e0 += 8) {
            float2 qv[8][C];  // (q, q magnitude) per element and channel
#pragma unroll
            for (int e = 0; e < 8; ++e) {
              const float* qk = pred_q + (e0 + e) * C * 2;
              if constexpr (C == 2) {
                const float4 f = *reinterpret_cast<const float4*>(qk);
                qv[e][0] = make_float2(f.x, f.y);
                qv[e][1] = make_float2(f.z, f.w);
              } else {
                qv[e][0] = *reinterpret_cast<const float2*>(qk);
              }
            }
#pragma unroll
            for (int h = 0; h < kRowsPerThread; ++h) {
              float value[8];
              if constexpr (is_e4m3(KIND)) {
                const uint4 chunk = raw[h][e0 >> 4];
                const uint32_t w0 = (e0 & 8) ? chunk.z : chunk.x;
                const uint32_t w1 = (e0 & 8) ? chunk.w : chunk.y;
                const float2 v01 = e4m3x2_to_float2(w0 & 0xFFFFu), v23 = e4m3x2_to_float2(w0 >> 16);
                const float2 v45 = e4m3x2_to_float2(w1 & 0xFFFFu), v67 = e4m3x2_to_float2(w1 >> 16);
                value[0] = v01.x; value[1] = v01.y; value[2] = v23.x; value[3] = v23.y;
                value[4] = v45.x; value[5] = v45.y; value[6] = v67.x; value[7] = v67.y;
                if constexpr (BLK) {
                  const float scale = __uint_as_float(sfw[h]);
#pragma unroll
                  for (int e = 0; e < 8; ++e) value[e] = __fmul_rn(value[e], scale);
                }
              } else {
                const uint4 chunk = raw[h][e0 >> 5];
                const int wi = (e0 >> 3) & 3;
                const uint32_t word = wi == 0 ? chunk.x : wi == 1 ? chunk.y : wi == 2 ? chunk.z : chunk.w;
                // code x block scale, two at a time in fp16: exact (at most
                // 6 significant bits), so the same values as in fp32.
                const uint32_t sh2 = scale_h2[h][e0 >> 4];
#pragma unroll
                for (int i = 0; i < 4; ++i) {
                  const float2 v = h2_to_float2(hmul2_rn(e2m1x2_to_h2((word >> (8 * i)) & 0xFFu), sh2));
                  value[2 * i] = v.x;
                  value[2 * i + 1] = v.y;
                }
              }
#pragma unroll
              for (int e = 0; e < 8; ++e) {
                const float2 vv = make_float2(value[e], fabsf(value[e]));
#pragma unroll
                for (int c = 0; c < C; ++c) acc[h][c] = fma2(qv[e][c], vv, acc[h][c]);
              }
            }
          }
        }
        if (stopped) break;
#pragma unroll
        for (int h = 0; h < kRowsPerThread; ++h) {
          const int col = nt * kTN + ct + 128 * h;
          if (col < p.padded_n) {
            const bool in = col < p.n;
#pragma unroll
            for (int c = 0; c < C; ++c) {
              const int64_t off = (static_cast<int64_t>(c) * p.tiles_m + mt) * p.padded_n + col;
              p.predicted[off] = alpha * (in ? acc[h][c].x : 0.f);
              p.magnitude[off] = fabsf(alpha) * (in ? acc[h][c].y : 0.f);
            }
          }
        }
      }
      // Teardown: a slice copy that was never seen landing lands before the
      // CTA releases its shared memory.
      if (copy_in_flight && !mbar_drain(pred_full, (slices_staged - 1u) & 1u)) *abort_flag = kWaitOther;
    }
  }

  __syncthreads();
  // A CTA that gave up a bounded wait left its tiles incomplete: bit 1 of
  // `hit` (and the non-finite flag) carry that to finalize, which reports the
  // launch as detected, so an aborted GEMM can never pass as clean.
  if constexpr (C > 0) {
    if (threadIdx.x == 0 && *abort_flag != 0) {
      if constexpr (AUG) griddep_wait();  // after the encode grid zeroed the status
      atomicOr(p.hit, 2);
      // Augmented calls report through their tile flags: the non-finite bit
      // of the first entry makes the packed finalize report detected.
      if (AUG && p.tile_flags != nullptr) atomicOr(p.tile_flags, 2);
      if (p.nonfinite != nullptr) atomicExch(p.nonfinite, 1);
    }
  }
  // No CTA of a pair leaves while the other may still signal its barriers.
  if constexpr (PAIR) cluster_sync();
  if (warp == 1) {
    __syncwarp();
    tc_fence_after();
    if constexpr (PAIR) {
      tmem_dealloc_pair(tmem, kTmemCols);
    } else {
      tmem_dealloc(tmem, kTmemCols);
    }
  }
}

template <Kind KIND, int C, bool BF16OUT, bool CHK, bool PAIR>
int launch_impl(const GemmProblem& g, cudaStream_t stream) {
  constexpr bool AUG = KIND == Kind::kBf16 && C > 0;
  const int64_t k_bytes = row_bytes_of(KIND, g.k);
  CUtensorMap ta{}, tb{}, tsa{}, tsb{};
  {
    const uint64_t dims[2] = {static_cast<uint64_t>(k_bytes), static_cast<uint64_t>(g.m)};
    const uint64_t strides[1] = {static_cast<uint64_t>(k_bytes)};
    const uint32_t box[2] = {kBKBytes, kBM};
    int rc = encode_tensor_map(&ta, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<uint8_t*>(g.a), dims,
                               strides, box, CU_TENSOR_MAP_SWIZZLE_128B);
    if (rc != SDC_OK) return rc;
  }
  {
    const uint64_t dims[2] = {static_cast<uint64_t>(k_bytes), static_cast<uint64_t>(g.n)};
    const uint64_t strides[1] = {static_cast<uint64_t>(k_bytes)};
    // Pairs: each CTA stages half of the tile's B rows.
    const uint32_t box[2] = {kBKBytes, static_cast<uint32_t>(PAIR ? tile_n(KIND) / 2 : tile_n(KIND))};
    int rc = encode_tensor_map(&tb, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<uint8_t*>(g.b), dims,
                               strides, box, CU_TENSOR_MAP_SWIZZLE_128B);
    if (rc != SDC_OK) return rc;
  }
  if constexpr (KIND == Kind::kNvf4) {
    const uint64_t k_atoms = static_cast<uint64_t>(ceil_div(g.k, 64));
    {
      const uint64_t dims[4] = {16, 32, k_atoms, static_cast<uint64_t>(ceil_div(g.m, 128))};
      const uint64_t strides[3] = {16, 512, 512 * k_atoms};
      const uint32_t box[4] = {16, 32, 4, 1};
      int rc = encode_tensor_map(&tsa, CU_TENSOR_MAP_DATA_TYPE_UINT8, 4, const_cast<uint8_t*>(g.sfa),
                                 dims, strides, box, CU_TENSOR_MAP_SWIZZLE_NONE);
      if (rc != SDC_OK) return rc;
    }
    {
      const uint64_t dims[4] = {16, 32, k_atoms, static_cast<uint64_t>(ceil_div(g.n, 128))};
      const uint64_t strides[3] = {16, 512, 512 * k_atoms};
      const uint32_t box[4] = {16, 32, 4, static_cast<uint32_t>(tile_n(KIND) / 128)};  // the tile's B row groups
      int rc = encode_tensor_map(&tsb, CU_TENSOR_MAP_DATA_TYPE_UINT8, 4, const_cast<uint8_t*>(g.sfb),
                                 dims, strides, box, CU_TENSOR_MAP_SWIZZLE_NONE);
      if (rc != SDC_OK) return rc;
    }
  } else {
    tsa = ta;
    tsb = tb;
    if constexpr (AUG) {
      // The checksum rows of A, read by the M-tiles after the data tiles.
      const uint64_t dims[2] = {static_cast<uint64_t>(k_bytes), static_cast<uint64_t>(g.aug_rows)};
      const uint64_t strides[1] = {static_cast<uint64_t>(k_bytes)};
      const uint32_t box[2] = {kBKBytes, kBM};
      int rc = encode_tensor_map(&tsa, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<uint8_t*>(g.q), dims, strides,
                                 box, CU_TENSOR_MAP_SWIZZLE_128B);
      if (rc != SDC_OK) return rc;
    }
    if constexpr (CHK) {
      // The prediction's B slices: the tile's rows x 64 bytes of K, 64-byte
      // swizzle (conflict-free 16-byte reads of 8 consecutive rows).
      const uint64_t dims[2] = {static_cast<uint64_t>(k_bytes), static_cast<uint64_t>(g.n)};
      const uint64_t strides[1] = {static_cast<uint64_t>(k_bytes)};
      const uint32_t box[2] = {static_cast<uint32_t>(kSliceK), static_cast<uint32_t>(tile_n(KIND))};
      int rc = encode_tensor_map(&tsb, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<uint8_t*>(g.b), dims, strides,
                                 box, CU_TENSOR_MAP_SWIZZLE_64B);
      if (rc != SDC_OK) return rc;
    }
  }
  Params p{};
  p.m = static_cast<int32_t>(g.m);
  p.n = static_cast<int32_t>(g.n);
  p.k = static_cast<int32_t>(g.k);
  p.num_kb = static_cast<int32_t>(ceil_div(k_bytes, kBKBytes));
  p.tiles_m = static_cast<int32_t>(ceil_div(g.m, kBM));
  p.tiles_m_all = p.tiles_m + (AUG ? static_cast<int32_t>(ceil_div(g.aug_rows, kBM)) : 0);
  p.aug_rows = AUG ? static_cast<int32_t>(g.aug_rows) : 0;
  p.tile_flags = g.tile_flags;
  p.row_observed = g.row_observed;
  p.flag_cols = static_cast<int32_t>(g.flag_cols);
  p.tiles_n = static_cast<int32_t>(ceil_div(g.n, tile_n(KIND)));
  p.num_tiles = p.tiles_m_all * p.tiles_n;
  p.num_work = PAIR ? static_cast<int32_t>(ceil_div(p.tiles_m_all, 2)) * p.tiles_n : p.num_tiles;
  if constexpr (KIND == Kind::kFp8Block) {
    p.sa = reinterpret_cast<const float*>(g.sfa);
    p.sb = reinterpret_cast<const float*>(g.sfb);
    p.k_blocks = static_cast<int32_t>(g.k / 128);
  }
  p.alpha = g.alpha;
  p.d = g.d;
  p.weights = g.weights;
  p.frow = static_cast<int32_t>(g.fault_row);
  p.fcol = static_cast<int32_t>(g.fault_col);
  p.fbit = static_cast<int32_t>(g.fault_bit);
  p.nonfinite = g.nonfinite;
  p.observed = g.observed;
  p.hit = g.hit;
  p.padded_n = static_cast<int32_t>(g.padded_n);
  p.q_full = g.q_full;
  p.q_part = g.q_part;
  p.grid_sync = g.grid_sync;
  p.q_bands = static_cast<int32_t>(ceil_div(g.m, kBandRows));
  p.q_ready = g.q_ready ? 1 : 0;
  p.a = g.a;
  p.sfa = g.sfa;
  p.b = g.b;
  p.sfb = g.sfb;
  p.predicted = g.predicted;
  p.magnitude = g.magnitude;
  p.watchdog = watchdog_ptr();
  if (p.watchdog == nullptr) return fail(SDC_ERR_CUDA, "watchdog symbol unavailable");
  const WatchdogSettings watch = watchdog_settings();
  p.wait_limit_ns = watch.wait_limit_ns;
  p.pace_extra = watch.pace_extra;
  auto kernel = gemm_kernel<KIND, C, BF16OUT, CHK, PAIR>;
  constexpr int smem = smem_bytes(KIND, PAIR, CHK);
  static_assert(smem <= 232448, "shared memory beyond the 227 KiB per-CTA limit");
  cudaLaunchConfig_t config{};
  config.blockDim = dim3(num_threads(CHK, is_wide(KIND)));
  config.dynamicSmemBytes = smem;
  config.stream = stream;
  cudaLaunchAttribute attribute[3];
  int attrs = 0;
  if constexpr (PAIR) {
    attribute[attrs].id = cudaLaunchAttributeClusterDimension;
    attribute[attrs].val.clusterDim.x = 2;
    attribute[attrs].val.clusterDim.y = 1;
    attribute[attrs].val.clusterDim.z = 1;
    ++attrs;
  }
  if constexpr (AUG) {
    // The augmented GEMM follows its encode kernel on the stream and may
    // start while that grid finishes: its data tiles need nothing from it,
    // and the warps that do (checksum-row loads, epilogue) wait for it.
    attribute[attrs].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attribute[attrs].val.programmaticStreamSerializationAllowed = 1;
    ++attrs;
  }
  config.attrs = attribute;
  config.numAttrs = attrs;
  // Per device: the shared-memory opt-in and how many CTAs (pairs) fit at
  // once. Concurrent first launches from several host threads may both run
  // the set-up (it is idempotent); the cached count is published atomically.
  static std::atomic<int> resident[64] = {};
  int device = 0;
  SDC_CUDA_CHECK(cudaGetDevice(&device));
  int fit = device >= 0 && device < 64 ? resident[device].load(std::memory_order_acquire) : 0;
  if (fit == 0) {
    if constexpr (is_wide(KIND)) {
      // The register split (setmaxnreg) must fit in what the kernel is
      // launched with, or the increasing warps would wait forever.
      cudaFuncAttributes attr{};
      SDC_CUDA_CHECK(cudaFuncGetAttributes(&attr, kernel));
      if (attr.numRegs < static_cast<int>(required_regs_per_thread(CHK))) {
        return fail(SDC_ERR_CUDA, "GEMM kernel was built with too few registers for its register split");
      }
    }
    SDC_CUDA_CHECK(cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, smem));
    if constexpr (PAIR) {
      config.gridDim = dim3(2);
      SDC_CUDA_CHECK(cudaOccupancyMaxActiveClusters(&fit, kernel, &config));
    } else {
      fit = sm_count();
    }
    if (fit <= 0) return fail(SDC_ERR_CUDA, "GEMM kernel does not fit on this device");
    if (device >= 0 && device < 64) resident[device].store(fit, std::memory_order_release);
  }
  const int units = std::min(p.num_work, fit);  // persistent: at most one wave
  config.gridDim = dim3(static_cast<unsigned>(PAIR ? 2 * units : units));
  // The prediction warps synchronise across CTAs (two grid barriers around
  // the projection), so every CTA must be resident: the grid never exceeds
  // one wave of the occupancy computed above and single CTAs additionally
  // launch cooperatively (a guarantee that cluster launches cannot combine
  // with under the profiler). A CTA that cannot start because another kernel
  // holds its SM (e.g. a second protected GEMM launched concurrently on
  // another stream) leaves the others waiting at the barrier; every wait is
  // bounded, and a launch that gives up is reported in-band as detected.
  if constexpr (CHK && !PAIR) {
    attribute[attrs].id = cudaLaunchAttributeCooperative;
    attribute[attrs].val.cooperative = 1;
    config.numAttrs = ++attrs;
  }
  SDC_CUDA_CHECK(cudaLaunchKernelEx(&config, kernel, ta, tb, tsa, tsb, p));
  return SDC_OK;
}

template <Kind KIND, int C, bool BF16OUT, bool CHK>
int dispatch_pair(const GemmProblem& g, cudaStream_t stream) {
  // CTA pairs (256-row tiles) whenever there are two M-tiles (checksum-row
  // tiles of the augmented bf16 GEMM included).
  const int64_t rows = ceil_div(g.m, kBM) * kBM + (KIND == Kind::kBf16 && C > 0 ? g.aug_rows : 0);
  if (rows > kBM) return launch_impl<KIND, C, BF16OUT, CHK, true>(g, stream);
  return launch_impl<KIND, C, BF16OUT, CHK, false>(g, stream);
}

template <Kind KIND, int C>
int dispatch_out(const GemmProblem& g, cudaStream_t stream) {
  const bool chk = g.q_full != nullptr;
  if constexpr (C == 0) {
    return g.out_bf16_rowmajor ? dispatch_pair<KIND, 0, true, false>(g, stream)
                               : dispatch_pair<KIND, 0, false, false>(g, stream);
  } else {
    if (g.out_bf16_rowmajor) {
      return chk ? dispatch_pair<KIND, C, true, true>(g, stream) : dispatch_pair<KIND, C, true, false>(g, stream);
    }
    return chk ? dispatch_pair<KIND, C, false, true>(g, stream) : dispatch_pair<KIND, C, false, false>(g, stream);
  }
}

}  // namespace

int launch_gemm(const GemmProblem& g, cudaStream_t stream) {
  int rc = check_current_device();
  if (rc != SDC_OK) return rc;
  if (g.channels > 0) {
    if (!g.status_zeroed) SDC_CUDA_CHECK(cudaMemsetAsync(g.hit, 0, sizeof(int32_t), stream));
    if (g.nonfinite != nullptr) SDC_CUDA_CHECK(cudaMemsetAsync(g.nonfinite, 0, sizeof(int32_t), stream));
    if (g.grid_sync != nullptr) SDC_CUDA_CHECK(cudaMemsetAsync(g.grid_sync, 0, sizeof(uint32_t), stream));
    if (g.tile_flags != nullptr && !g.status_zeroed) {
      SDC_CUDA_CHECK(cudaMemsetAsync(g.tile_flags, 0, sizeof(int32_t) * ceil_div(g.m, kBM) * g.flag_cols, stream));
    }
  }
  if (g.kind == Kind::kFp8) {
    if (g.channels == 0) return dispatch_out<Kind::kFp8, 0>(g, stream);
    if (g.channels == 1) return dispatch_out<Kind::kFp8, 1>(g, stream);
    return dispatch_out<Kind::kFp8, 2>(g, stream);
  }
  if (g.kind == Kind::kFp8Block) {
    if (g.channels == 0) return dispatch_out<Kind::kFp8Block, 0>(g, stream);
    if (g.channels == 1) return dispatch_out<Kind::kFp8Block, 1>(g, stream);
    return dispatch_out<Kind::kFp8Block, 2>(g, stream);
  }
  if (g.kind == Kind::kBf16) {
    // bf16 row-major output only; the protected form is the augmented GEMM.
    if (g.channels == 0) return dispatch_pair<Kind::kBf16, 0, true, false>(g, stream);
    if (g.channels == 1) return dispatch_pair<Kind::kBf16, 1, true, false>(g, stream);
    return dispatch_pair<Kind::kBf16, 2, true, false>(g, stream);
  }
  if (g.channels == 0) return dispatch_out<Kind::kNvf4, 0>(g, stream);
  if (g.channels == 1) return dispatch_out<Kind::kNvf4, 1>(g, stream);
  return dispatch_out<Kind::kNvf4, 2>(g, stream);
}

}  // namespace sdc
