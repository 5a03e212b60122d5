// Standalone K-slice prediction: two kernels before an observed-only GEMM.
//
// The fused path (gemm.cu) computes the projection q = w^T A and the K-slice
// prediction on four warps of every GEMM CTA, paced across the CTA's tiles.
// That hides both when each CTA has many tiles, but the prediction reads all
// of B (N x K) whatever M is, so when N dwarfs a short M it can outlast the
// GEMM. This path spreads the same arithmetic over the whole GPU instead
// (chosen by kslice_standalone):
//
//   kslice_project  one warp per (128-row band, slice) item: project_item,
//                   the same device function the fused path runs, into the
//                   band partials;
//   kslice_fold     one thread per entry: the bands added in ascending order
//                   into q_full (the fused path's phase 2);
//   kslice_predict  one thread per (slot t, column n): each slice's q staged
//                   in shared memory, the column's fma chains over the slices
//                   s % Tm == t (ascending), k ascending, exactly as the fused
//                   path does (the next slice of B loaded under the current);
//
// so predicted and magnitude are bit-identical between the two paths (and to
// oracle/cref.c). The GEMM launched after them has no prediction warps, no
// grid barriers and the full register budget of the observed-only epilogue.
#include <atomic>

#include "kslice.cuh"

namespace sdc {
namespace {

constexpr int kProjectWarps = 8;
constexpr int kItemBatch = 4;     // rows of a row lane loaded ahead of their fma chains
constexpr int kFoldThreads = 64;  // small blocks: the entries spread over every SM
constexpr int kFoldBatch = 32;    // band partials loaded ahead of their adds
constexpr int kPredictThreads = 128;

// Test hook: 0 = choose by size, 1 = always fused (projection inside the
// GEMM), 2 = always standalone, 3 = always fused with the projection
// computed before the GEMM.
std::atomic<int> g_kslice_mode{0};

// One warp per item (band, slice), items in band-major order so that a
// block's warps read neighbouring slices of the same rows: the band's partial
// of the slice (project_item, as in the fused path) into q_part.
template <Kind KIND, int C>
__global__ void __launch_bounds__(32 * kProjectWarps, 2) kslice_project(ProjectionView v, int64_t items) {
  griddep_launch_dependents();
  const int64_t item = static_cast<int64_t>(blockIdx.x) * kProjectWarps + (threadIdx.x >> 5);
  if (item >= items) return;
  const int64_t band = item / v.num_slices, chunk = item % v.num_slices;
  project_item<KIND, C, kItemBatch>(v, band, chunk, static_cast<int>(threadIdx.x & 31),
                                    band_partial<C>(v, band, chunk));
}

// q_full[e] = the bands' partials of entry e added in ascending band order
// (the fused path's phase 2), the loads batched ahead of the adds.
__global__ void __launch_bounds__(kFoldThreads) kslice_fold(const float* q_part, int64_t entries, int64_t bands,
                                                           float* q_full) {
  griddep_launch_dependents();
  const int64_t e = static_cast<int64_t>(blockIdx.x) * kFoldThreads + threadIdx.x;
  if (e >= entries) return;
  float q = __ldg(q_part + e);
  int64_t b = 1;
  for (; b + kFoldBatch <= bands; b += kFoldBatch) {
    float x[kFoldBatch];
#pragma unroll
    for (int i = 0; i < kFoldBatch; ++i) x[i] = __ldg(q_part + (b + i) * entries + e);
#pragma unroll
    for (int i = 0; i < kFoldBatch; ++i) q = __fadd_rn(q, x[i]);
  }
  for (; b < bands; ++b) q = __fadd_rn(q, __ldg(q_part + b * entries + e));
  q_full[e] = q;
}

struct PredictArgs {
  const uint8_t* b;        // B rows [N][K] (e4m3) or [N][K/2] (packed e2m1)
  const uint8_t* sfb;      // NVFP4: B scale atoms
  const float* sb;         // block-scaled FP8: B scales [ceil(N/128)][K/128]
  const float* alpha;      // device scalar; null = 1 (block-scaled)
  const float* q_full;     // [K_pad][C][2]
  int64_t n, k, k_blocks, num_slices, tiles_m, padded_n;
  float* predicted;        // [C][Tm][padded_n]
  float* magnitude;
};

// Grid (ceil(padded_n / 128), Tm): slot t = blockIdx.y, column (B row)
// n = blockIdx.x * 128 + threadIdx.x.
template <Kind KIND, int C>
__global__ void __launch_bounds__(kPredictThreads) kslice_predict(PredictArgs p) {
  constexpr bool BLK = KIND == Kind::kFp8Block;
  constexpr int kChunks = is_e4m3(KIND) ? 4 : 2;  // 16-byte chunks of a slice row
  constexpr int kEntries = kSliceK * C * 2;       // q floats of one slice
  constexpr int kStageSlices = 16;  // slices of q staged in shared memory at a time
  __shared__ __align__(16) float qs[kStageSlices][kEntries];
  const int64_t t = blockIdx.y;
  const int64_t r = static_cast<int64_t>(blockIdx.x) * kPredictThreads + threadIdx.x;
  const bool row_in = r < p.n;
  const int64_t row_bytes = is_e4m3(KIND) ? p.k : p.k / 2;
  const int64_t k_atoms = (p.k + 63) / 64;
  // Channel c: value chain in acc[c].x, magnitude chain in acc[c].y.
  float2 acc[C];
#pragma unroll
  for (int c = 0; c < C; ++c) acc[c] = make_float2(0.f, 0.f);
  // The column's slice of B (zeros past N and past K) and its scales; the
  // next slice's are loaded while this one is folded in.
  auto load_slice = [&](int64_t sl, uint4 (&raw)[kChunks], uint32_t& sfw) {
    const int64_t k0 = sl * kSliceK;
#pragma unroll
    for (int ch = 0; ch < kChunks; ++ch) {
      const int64_t byte = (is_e4m3(KIND) ? k0 : k0 / 2) + ch * 16;
      raw[ch] = (row_in && sl < p.num_slices && byte < row_bytes)
                    ? __ldg(reinterpret_cast<const uint4*>(p.b + r * row_bytes + byte))
                    : make_uint4(0, 0, 0, 0);
    }
    sfw = 0;
    if (row_in && sl < p.num_slices) {
      if constexpr (KIND == Kind::kNvf4) {
        const int64_t off = ((r >> 7) * k_atoms + (k0 >> 6)) * 512 + (r & 31) * 16 + ((r >> 5) & 3) * 4;
        sfw = __ldg(reinterpret_cast<const uint32_t*>(p.sfb + off));
      } else if constexpr (BLK) {
        sfw = __float_as_uint(__ldg(p.sb + (r >> 7) * p.k_blocks + (k0 >> 7)));
      }
    }
  };
  uint4 next[kChunks];
  uint32_t next_sfw = 0;
  load_slice(t, next, next_sfw);
  // Launched as a programmatic dependent of kslice_project: B above needs
  // nothing from it, q_full below does.
  griddep_wait();
  int64_t staged_end = t;  // first slice of this slot not yet staged
  int staged_first = 0;     // index in qs of the next slice to fold in
  for (int64_t sl = t; sl < p.num_slices; sl += p.tiles_m) {
    uint4 raw[kChunks];
#pragma unroll
    for (int ch = 0; ch < kChunks; ++ch) raw[ch] = next[ch];
    const uint32_t sfw = next_sfw;
    load_slice(sl + p.tiles_m, next, next_sfw);
    if (sl == staged_end) {
      // q of the slot's next kStageSlices slices, in one round of loads.
      __syncthreads();  // the previous group's reads of qs are done
      for (int i = threadIdx.x; i < kStageSlices * kEntries; i += kPredictThreads) {
        const int64_t s_i = sl + (i / kEntries) * p.tiles_m;
        qs[i / kEntries][i % kEntries] = s_i < p.num_slices ? __ldg(p.q_full + s_i * kEntries + i % kEntries) : 0.f;
      }
      __syncthreads();
      staged_end = sl + kStageSlices * p.tiles_m;
      staged_first = 0;
    }
    const float* q_slice = qs[staged_first++];
    // NVFP4: the slice's four block scales as fp16 pairs (s, s).
    uint32_t scale_h2[4] = {0, 0, 0, 0};
    if constexpr (KIND == Kind::kNvf4) {
      const uint32_t lo = e4m3x2_to_h2(sfw & 0xFFFFu), hi = e4m3x2_to_h2(sfw >> 16);
      scale_h2[0] = __byte_perm(lo, 0, 0x1010);
      scale_h2[1] = __byte_perm(lo, 0, 0x3232);
      scale_h2[2] = __byte_perm(hi, 0, 0x1010);
      scale_h2[3] = __byte_perm(hi, 0, 0x3232);
    }
#pragma unroll
    for (int e0 = 0; e0 < kSliceK; e0 += 8) {
      float2 value[4];  // elements e0 + 2i, e0 + 2i + 1
      if constexpr (is_e4m3(KIND)) {
        const uint4 chunk = raw[e0 >> 4];
        const uint32_t w0 = (e0 & 8) ? chunk.z : chunk.x;
        const uint32_t w1 = (e0 & 8) ? chunk.w : chunk.y;
        value[0] = h2_to_float2(e4m3x2_to_h2(w0 & 0xFFFFu));
        value[1] = h2_to_float2(e4m3x2_to_h2(w0 >> 16));
        value[2] = h2_to_float2(e4m3x2_to_h2(w1 & 0xFFFFu));
        value[3] = h2_to_float2(e4m3x2_to_h2(w1 >> 16));
        if constexpr (BLK) {
          const float scale = __uint_as_float(sfw);
#pragma unroll
          for (int i = 0; i < 4; ++i) value[i] = make_float2(__fmul_rn(value[i].x, scale), __fmul_rn(value[i].y, scale));
        }
      } else {
        const uint4 chunk = raw[e0 >> 5];
        const int wi = (e0 >> 3) & 3;
        const uint32_t word = wi == 0 ? chunk.x : wi == 1 ? chunk.y : wi == 2 ? chunk.z : chunk.w;
        const uint32_t sh2 = scale_h2[e0 >> 4];
#pragma unroll
        for (int i = 0; i < 4; ++i) value[i] = h2_to_float2(hmul2_rn(e2m1x2_to_h2((word >> (8 * i)) & 0xFFu), sh2));
      }
#pragma unroll
      for (int e = 0; e < 8; ++e) {
        const float v = (e & 1) ? value[e >> 1].y : value[e >> 1].x;
        // (value, |value|) against channel c's (q, q_magnitude): the value and
        // magnitude chains of one channel in one f32x2 fma (two independent
        // fmas), operands in the [k][c][2] order of q.
        const float2 vv = make_float2(v, fabsf(v));
        if constexpr (C == 2) {
          const float4 qk = reinterpret_cast<const float4*>(q_slice)[e0 + e];
          acc[0] = fma2(make_float2(qk.x, qk.y), vv, acc[0]);
          acc[1] = fma2(make_float2(qk.z, qk.w), vv, acc[1]);
        } else {
          const float2 qk = reinterpret_cast<const float2*>(q_slice)[e0 + e];
          acc[0] = fma2(qk, vv, acc[0]);
        }
      }
    }
  }
  if (r < p.padded_n) {
    const float alpha = p.alpha != nullptr ? *p.alpha : 1.f;
#pragma unroll
    for (int c = 0; c < C; ++c) {
      const int64_t off = (static_cast<int64_t>(c) * p.tiles_m + t) * p.padded_n + r;
      p.predicted[off] = alpha * (row_in ? acc[c].x : 0.f);
      p.magnitude[off] = fabsf(alpha) * (row_in ? acc[c].y : 0.f);
    }
  }
}

template <Kind KIND, int C>
int standalone_impl(const ReferenceProblem& r, const KsliceScratch& s, cudaStream_t stream) {
  constexpr bool BLK = KIND == Kind::kFp8Block;
  const int64_t num_slices = ceil_div(r.k, kSliceK);
  const int64_t bands = ceil_div(r.m, kBandRows);
  const ProjectionView view{r.a,
                            BLK ? reinterpret_cast<const float*>(r.sfa) : nullptr,
                            KIND == Kind::kNvf4 ? r.sfa : nullptr,
                            r.weights,
                            r.m,
                            r.k,
                            r.k / 128,
                            num_slices,
                            s.q_part};
  (void)bands;
  const int rc = launch_projection_sums(KIND, C, view, s.q_full, stream);
  if (rc != SDC_OK) return rc;
  PredictArgs pa{};
  pa.b = r.b;
  pa.sfb = KIND == Kind::kNvf4 ? r.sfb : nullptr;
  pa.sb = BLK ? reinterpret_cast<const float*>(r.sfb) : nullptr;
  pa.alpha = BLK ? nullptr : r.alpha;
  pa.q_full = s.q_full;
  pa.n = r.n;
  pa.k = r.k;
  pa.k_blocks = r.k / 128;
  pa.num_slices = num_slices;
  pa.tiles_m = ceil_div(r.m, 128);
  pa.padded_n = r.padded_n;
  pa.predicted = r.predicted;
  pa.magnitude = r.magnitude;
  cudaLaunchConfig_t config{};
  config.gridDim = dim3(static_cast<unsigned>(ceil_div(r.padded_n, kPredictThreads)), static_cast<unsigned>(pa.tiles_m));
  config.blockDim = dim3(kPredictThreads);
  config.stream = stream;
  cudaLaunchAttribute attribute[1];
  attribute[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attribute[0].val.programmaticStreamSerializationAllowed = 1;
  config.attrs = attribute;
  config.numAttrs = 1;
  SDC_CUDA_CHECK(cudaLaunchKernelEx(&config, kslice_predict<KIND, C>, pa));
  return SDC_OK;
}

template <Kind KIND>
int standalone_kind(const ReferenceProblem& r, const KsliceScratch& s, cudaStream_t stream) {
  return r.channels == 2 ? standalone_impl<KIND, 2>(r, s, stream) : standalone_impl<KIND, 1>(r, s, stream);
}

}  // namespace

int launch_projection_sums(Kind kind, int channels, const ProjectionView& view, float* q_full, cudaStream_t stream) {
  if (channels != 1 && channels != 2) return fail(SDC_ERR_INVALID, "projection sums need 1 or 2 channels");
  const int64_t bands = ceil_div(view.m, kBandRows);
  ProjectionView v = view;
  // One band: its partial is the sum, written straight into q_full.
  if (bands == 1) v.q_part = q_full;
  if (v.q_part == nullptr) return fail(SDC_ERR_WORKSPACE, "projection sums need band scratch");
  const int64_t items = bands * v.num_slices;
  const dim3 grid(static_cast<unsigned>(ceil_div(items, kProjectWarps)));
  const dim3 block(32 * kProjectWarps);
  switch (kind) {
    case Kind::kFp8:
      if (channels == 2) kslice_project<Kind::kFp8, 2><<<grid, block, 0, stream>>>(v, items);
      else kslice_project<Kind::kFp8, 1><<<grid, block, 0, stream>>>(v, items);
      break;
    case Kind::kNvf4:
      if (channels == 2) kslice_project<Kind::kNvf4, 2><<<grid, block, 0, stream>>>(v, items);
      else kslice_project<Kind::kNvf4, 1><<<grid, block, 0, stream>>>(v, items);
      break;
    case Kind::kFp8Block:
      if (channels == 2) kslice_project<Kind::kFp8Block, 2><<<grid, block, 0, stream>>>(v, items);
      else kslice_project<Kind::kFp8Block, 1><<<grid, block, 0, stream>>>(v, items);
      break;
    default:
      return fail(SDC_ERR_INVALID, "projection sums are defined for the FP8 and NVFP4 kinds");
  }
  SDC_CUDA_CHECK(cudaGetLastError());
  if (bands > 1) {
    const int64_t entries = v.num_slices * kSliceK * channels * 2;
    kslice_fold<<<static_cast<unsigned>(ceil_div(entries, kFoldThreads)), kFoldThreads, 0, stream>>>(
        v.q_part, entries, bands, q_full);
    SDC_CUDA_CHECK(cudaGetLastError());
  }
  return SDC_OK;
}

// Measured on B200 over the Qwen2.5-7B linear shapes at M = 2048 / 4096 /
// 8192 (protected step over the unprotected GEMM): the projection computed
// before the GEMM wins only at M <= 2048 when the in-GEMM projection has many
// items per prediction warp next to few tiles per CTA, i.e. a long K
// (down, K = 18944: NVFP4 57 vs 70 %, FP8 36 vs 53 %), and for NVFP4 with
// N >= 16 M (gate/up: 57 vs 61 % standalone, 68 % in-GEMM). It loses for
// block-scaled FP8 (whose 128-wide tiles give the in-GEMM projection twice
// the tiles to hide behind) and at M >= 4096 everywhere.
static bool kslice_preproject_auto(const ReferenceProblem& r) {
  if (r.kind == Kind::kFp8Block || r.m > 2048) return false;
  return r.k >= 4 * r.n || (r.kind == Kind::kNvf4 && r.n >= 16 * r.m);
}

bool kslice_standalone(const ReferenceProblem& r) {
  const int mode = g_kslice_mode.load(std::memory_order_relaxed);
  if (mode == 1 || mode == 3) return false;
  if (mode == 2) return true;
  // Measured on B200 over the Qwen2.5-7B linear shapes at M = 2048 / 4096 /
  // 8192: the in-GEMM path wins except for NVFP4 (whose in-GEMM prediction
  // reads B with plain loads) when N dwarfs a short M; up to M = 2048 the
  // projection computed before the GEMM does better still.
  return r.kind == Kind::kNvf4 && r.m <= kStandaloneMaxRows && r.n >= 16 * r.m && !kslice_preproject_auto(r);
}

bool kslice_preproject(const ReferenceProblem& r) {
  const int mode = g_kslice_mode.load(std::memory_order_relaxed);
  if (mode == 1 || mode == 2) return false;
  if (mode == 3) return true;
  return kslice_preproject_auto(r);
}

int launch_kslice_projection(const ReferenceProblem& r, const KsliceScratch& s, cudaStream_t stream) {
  const Kind kind = r.kind;
  if (kind != Kind::kFp8 && kind != Kind::kNvf4 && kind != Kind::kFp8Block) {
    return fail(SDC_ERR_INVALID, "K-slice prediction is defined for the FP8 and NVFP4 kinds");
  }
  const bool blk = kind == Kind::kFp8Block;
  const ProjectionView view{r.a,
                            blk ? reinterpret_cast<const float*>(r.sfa) : nullptr,
                            kind == Kind::kNvf4 ? r.sfa : nullptr,
                            r.weights,
                            r.m,
                            r.k,
                            r.k / 128,
                            ceil_div(r.k, kSliceK),
                            s.q_part};
  return launch_projection_sums(kind, r.channels, view, s.q_full, stream);
}

int launch_kslice_standalone(const ReferenceProblem& r, const KsliceScratch& s, cudaStream_t stream) {
  switch (r.kind) {
    case Kind::kFp8:
      return standalone_kind<Kind::kFp8>(r, s, stream);
    case Kind::kNvf4:
      return standalone_kind<Kind::kNvf4>(r, s, stream);
    case Kind::kFp8Block:
      return standalone_kind<Kind::kFp8Block>(r, s, stream);
    default:
      return fail(SDC_ERR_INVALID, "K-slice prediction is defined for the FP8 and NVFP4 kinds");
  }
}

}  // namespace sdc

extern "C" int sdc_test_set_kslice_path(int mode) {
  if (mode < 0 || mode > 3) return sdc::fail(SDC_ERR_INVALID, "kslice path mode must be 0 (auto), 1, 2 or 3");
  sdc::g_kslice_mode.store(mode, std::memory_order_relaxed);
  return SDC_OK;
}
