// Input-side ABFT checksums: predicted = alpha * w^T A B and
// magnitude = |alpha| * |w|^T |A| |B| partials.
//
// TILE layout (reference parity). Restates the arithmetic of
// src/cutlass_gemm/csrc/abft/fp8/fp8_reference.cuh:31-83 and
// nvfp4/nvfp4_reference.cuh:31-84 of the reference: per 128-row M-tile,
//   q_c[k]  = fma over rows (ascending) of w_c[row] * A[row, k]
//   |q|_c[k] likewise with |w|, |A|
//   r_c[n] = fma over k (ascending) of q_c[k] * B[n, k];  a_c[n] with |q|, |B|
//   predicted = alpha * r, magnitude = |alpha| * a   (columns < padded N)
// with the same fp32 operation order, so results match the reference's
// mainloop bit for bit. Cost is ~C/32 of the GEMM on CUDA cores, so this
// layout is the parity path, not the fast path.
//
// KSLICE layout (fast path). q is the projection over ALL rows, and the
// 64-wide K slice s contributes to slot s % Tm:
//   predicted[c, t, n] = alpha * sum_{s % Tm == t} sum_{k in s} q_c[k] B[n,k]
// Both q and the propagation run inside the GEMM (gemm.cu, prediction
// warps); this file only sizes and lays out their scratch. The per-column
// sum over slots equals the TILE layout's sum over tiles up to fp32
// rounding, so finalize is unchanged.
#include <algorithm>

#include "kslice.cuh"

namespace sdc {
namespace {

constexpr int kTileRows = 128;
constexpr int kRefThreads = 128;
constexpr int kTilesPerBlock = 8;
constexpr int kChunkK = 64;

__device__ __forceinline__ int64_t sf_off(int64_t row, int64_t block, int64_t k_atoms) {
  return ((row >> 7) * k_atoms + (block >> 2)) * 512 + (row & 31) * 16 + ((row >> 5) & 3) * 4 +
         (block & 3);
}

// Decoded operand value at (row, k): e4m3 byte, or e2m1 nibble times its ue4m3 scale.
template <Kind KIND>
__device__ __forceinline__ float operand_value(const uint8_t* x, const uint8_t* sf, int64_t row,
                                               int64_t k, int64_t kdim) {
  if constexpr (KIND == Kind::kFp8) {
    return decode_e4m3(x[row * kdim + k]);
  } else {
    const uint32_t byte = x[row * (kdim / 2) + (k >> 1)];
    const float code = decode_e2m1((k & 1) ? (byte >> 4) : (byte & 15u));
    const float scale = decode_e4m3(sf[sf_off(row, k >> 4, (kdim + 63) / 64)]);
    return code * scale;
  }
}

// q[(c*2 + h) * Tm * K + t * K + k]: h = 0 signed projection, h = 1 magnitude.
// Each thread owns 8 consecutive k of one tile and walks the tile's rows in
// ascending order (the reference's fma order); loads of 8 rows are issued
// ahead of their fma chains so enough bytes are in flight to stream A at
// HBM speed. A warp reads 256 contiguous bytes (FP8) or 128 (NVFP4) per row.
template <Kind KIND, int C>
__global__ void __launch_bounds__(kRefThreads)
    q_encode(const uint8_t* a, const uint8_t* sfa, int64_t m, int64_t k, const float* weights,
             float* q, int64_t tiles_m) {
  const int64_t k0 = (static_cast<int64_t>(blockIdx.x) * kRefThreads + threadIdx.x) * 8;
  const int64_t t = blockIdx.y;
  if (k0 >= k) return;
  // acc[e] = {enc_c0, enc_c1} and {mag_c0, mag_c1} pairs for packed f32x2 fmas
  // (C == 1 keeps the second lane at zero weight).
  float2 enc[8], mag[8];
#pragma unroll
  for (int e = 0; e < 8; ++e) enc[e] = mag[e] = make_float2(0.f, 0.f);
  const int64_t rows = std::min<int64_t>(kTileRows, m - t * kTileRows);
  const int64_t k_atoms = (k + 63) / 64;
  constexpr int kBatch = 8;
  for (int64_t r0 = 0; r0 < rows; r0 += kBatch) {
    uint2 u8[kBatch];
    uint32_t u4[kBatch];
    uint32_t sfb[kBatch];
    float w[kBatch][C];
#pragma unroll
    for (int i = 0; i < kBatch; ++i) {
      const int64_t row = t * kTileRows + r0 + i;
      const bool in = r0 + i < rows;
      if constexpr (KIND == Kind::kFp8) {
        u8[i] = in ? __ldg(reinterpret_cast<const uint2*>(a + row * k + k0)) : make_uint2(0, 0);
      } else {
        u4[i] = in ? __ldg(reinterpret_cast<const uint32_t*>(a + row * (k / 2) + k0 / 2)) : 0u;
        sfb[i] = in ? sfa[sf_off(row, k0 >> 4, k_atoms)] : 0u;
      }
#pragma unroll
      for (int c = 0; c < C; ++c) w[i][c] = in ? __ldg(weights + c * m + row) : 0.f;
    }
#pragma unroll
    for (int i = 0; i < kBatch; ++i) {
      if (r0 + i >= rows) break;
      float v[8];
      if constexpr (KIND == Kind::kFp8) {
        const float2 v01 = e4m3x2_to_float2(u8[i].x & 0xFFFFu), v23 = e4m3x2_to_float2(u8[i].x >> 16);
        const float2 v45 = e4m3x2_to_float2(u8[i].y & 0xFFFFu), v67 = e4m3x2_to_float2(u8[i].y >> 16);
        v[0] = v01.x; v[1] = v01.y; v[2] = v23.x; v[3] = v23.y;
        v[4] = v45.x; v[5] = v45.y; v[6] = v67.x; v[7] = v67.y;
      } else {
        const float scale = decode_e4m3(sfb[i]);
        e2m1x8_to_float(u4[i], v);
#pragma unroll
        for (int e = 0; e < 8; ++e) v[e] *= scale;
      }
      const float2 wv = make_float2(w[i][0], C == 2 ? w[i][C - 1] : 0.f);
      const float2 wa = make_float2(fabsf(wv.x), fabsf(wv.y));
#pragma unroll
      for (int e = 0; e < 8; ++e) {
        enc[e] = fma2(wv, make_float2(v[e], v[e]), enc[e]);
        const float av = fabsf(v[e]);
        mag[e] = fma2(wa, make_float2(av, av), mag[e]);
      }
    }
  }
#pragma unroll
  for (int c = 0; c < C; ++c) {
    float4* pe = reinterpret_cast<float4*>(q + ((c * 2 + 0) * tiles_m + t) * k + k0);
    float4* pm = reinterpret_cast<float4*>(q + ((c * 2 + 1) * tiles_m + t) * k + k0);
    float e8[8], m8[8];
#pragma unroll
    for (int e = 0; e < 8; ++e) {
      e8[e] = c == 0 ? enc[e].x : enc[e].y;
      m8[e] = c == 0 ? mag[e].x : mag[e].y;
    }
    pe[0] = make_float4(e8[0], e8[1], e8[2], e8[3]);
    pe[1] = make_float4(e8[4], e8[5], e8[6], e8[7]);
    pm[0] = make_float4(m8[0], m8[1], m8[2], m8[3]);
    pm[1] = make_float4(m8[4], m8[5], m8[6], m8[7]);
  }
}

// Loads the B operand values of columns k0..k0+63 of `row` (k0 % 64 == 0).
template <Kind KIND>
__device__ __forceinline__ void load_b_chunk(const uint8_t* b, const uint8_t* sfb, int64_t row,
                                             int64_t k0, int64_t kdim, int kc, float (&v)[kChunkK]) {
  if (kc == kChunkK) {
    if constexpr (KIND == Kind::kFp8) {
      const uint4* p = reinterpret_cast<const uint4*>(b + row * kdim + k0);
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const uint4 u = __ldg(p + i);
        const uint32_t w[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
        for (int j = 0; j < 16; ++j) v[16 * i + j] = decode_e4m3((w[j >> 2] >> (8 * (j & 3))) & 0xFFu);
      }
    } else {
      const uint4* p = reinterpret_cast<const uint4*>(b + row * (kdim / 2) + k0 / 2);
      const uint32_t sf_word =
          *reinterpret_cast<const uint32_t*>(sfb + sf_off(row, k0 >> 4, (kdim + 63) / 64));
#pragma unroll
      for (int i = 0; i < 2; ++i) {
        const uint4 u = __ldg(p + i);
        const uint32_t w[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
        for (int j = 0; j < 32; ++j) {
          const int kk = 32 * i + j;
          const uint32_t byte = (w[j >> 3] >> (8 * ((j >> 1) & 3))) & 0xFFu;
          const float code = decode_e2m1((j & 1) ? (byte >> 4) : (byte & 15u));
          v[kk] = code * decode_e4m3((sf_word >> (8 * (kk >> 4))) & 0xFFu);
        }
      }
    }
  } else {
#pragma unroll
    for (int j = 0; j < kChunkK; ++j) v[j] = j < kc ? operand_value<KIND>(b, sfb, row, k0 + j, kdim) : 0.f;
  }
}

template <Kind KIND, int C>
__global__ void __launch_bounds__(kRefThreads)
    propagate_tiles(const uint8_t* b, const uint8_t* sfb, int64_t n, int64_t k, const float* q,
                    int64_t tiles_m, const float* alpha_ptr, float* pred, float* mag,
                    int64_t padded_n) {
  __shared__ float qs[kTilesPerBlock][C][2][kChunkK];
  const int64_t col = static_cast<int64_t>(blockIdx.x) * kRefThreads + threadIdx.x;
  const int64_t t0 = static_cast<int64_t>(blockIdx.y) * kTilesPerBlock;
  const int nt = static_cast<int>(std::min<int64_t>(kTilesPerBlock, tiles_m - t0));
  float r[kTilesPerBlock][C], a[kTilesPerBlock][C];
#pragma unroll
  for (int t = 0; t < kTilesPerBlock; ++t) {
#pragma unroll
    for (int c = 0; c < C; ++c) r[t][c] = a[t][c] = 0.f;
  }
  for (int64_t k0 = 0; k0 < k; k0 += kChunkK) {
    const int kc = static_cast<int>(std::min<int64_t>(kChunkK, k - k0));
    __syncthreads();
    for (int idx = threadIdx.x; idx < kTilesPerBlock * C * 2 * kChunkK; idx += kRefThreads) {
      const int kk = idx % kChunkK;
      const int h = (idx / kChunkK) % 2;
      const int c = (idx / (2 * kChunkK)) % C;
      const int t = idx / (C * 2 * kChunkK);
      qs[t][c][h][kk] = (t < nt && kk < kc) ? q[((c * 2 + h) * tiles_m + t0 + t) * k + k0 + kk] : 0.f;
    }
    __syncthreads();
    if (col < n) {
      float v[kChunkK];
      load_b_chunk<KIND>(b, sfb, col, k0, k, kc, v);
#pragma unroll
      for (int kk = 0; kk < kChunkK; ++kk) {
        if (kk >= kc) break;
        const float value = v[kk];
        const float av = fabsf(value);
#pragma unroll
        for (int t = 0; t < kTilesPerBlock; ++t) {
          if (t < nt) {
#pragma unroll
            for (int c = 0; c < C; ++c) {
              r[t][c] = fmaf(qs[t][c][0][kk], value, r[t][c]);
              a[t][c] = fmaf(qs[t][c][1][kk], av, a[t][c]);
            }
          }
        }
      }
    }
  }
  if (col < padded_n) {
    const float alpha = *alpha_ptr;
#pragma unroll
    for (int t = 0; t < kTilesPerBlock; ++t) {
      if (t < nt) {
#pragma unroll
        for (int c = 0; c < C; ++c) {
          const int64_t off = (c * tiles_m + t0 + t) * padded_n + col;
          pred[off] = alpha * r[t][c];
          mag[off] = fabsf(alpha) * a[t][c];
        }
      }
    }
  }
}

int64_t q_floats(int channels, int64_t m, int64_t k) { return static_cast<int64_t>(channels) * 2 * ceil_div(m, kTileRows) * k; }

template <Kind KIND, int C>
int projection_impl(const ReferenceProblem& p, cudaStream_t stream) {
  float* q = static_cast<float*>(p.workspace);
  const int64_t tiles_m = ceil_div(p.m, kTileRows);
  q_encode<KIND, C><<<dim3(static_cast<unsigned>(ceil_div(p.k, kRefThreads * 8)), static_cast<unsigned>(tiles_m)),
                      kRefThreads, 0, stream>>>(p.a, p.sfa, p.m, p.k, p.weights, q, tiles_m);
  SDC_CUDA_CHECK(cudaGetLastError());
  return SDC_OK;
}

template <Kind KIND, int C>
int tile_propagate_impl(const ReferenceProblem& p, cudaStream_t stream) {
  const int64_t tiles_m = ceil_div(p.m, kTileRows);
  const float* q = static_cast<const float*>(p.workspace);
  const unsigned col_blocks = static_cast<unsigned>(ceil_div(p.padded_n, kRefThreads));
  propagate_tiles<KIND, C><<<dim3(col_blocks, static_cast<unsigned>(ceil_div(tiles_m, kTilesPerBlock))),
                             kRefThreads, 0, stream>>>(p.b, p.sfb, p.n, p.k, q, tiles_m, p.alpha, p.predicted,
                                                       p.magnitude, p.padded_n);
  SDC_CUDA_CHECK(cudaGetLastError());
  return SDC_OK;
}


}  // namespace

namespace {
constexpr int64_t kSyncBytes = 256;
int64_t kslice_q_floats(int channels, int64_t k) { return static_cast<int64_t>(channels) * 2 * ceil_div(k, 64) * 64; }
}  // namespace

size_t reference_workspace_bytes(int channels, int64_t m, int64_t n, int64_t k, int layout) {
  (void)n;
  if (layout == SDC_LAYOUT_KSLICE) {
    const int64_t floats = kslice_q_floats(channels, k) * (1 + ceil_div(m, kBandRows));
    return static_cast<size_t>(kSyncBytes + floats * static_cast<int64_t>(sizeof(float)));
  }
  return static_cast<size_t>(q_floats(channels, m, k)) * sizeof(float);
}

KsliceScratch kslice_scratch(const ReferenceProblem& p) {
  uint8_t* base = static_cast<uint8_t*>(p.workspace);
  float* q_full = reinterpret_cast<float*>(base + kSyncBytes);
  return {reinterpret_cast<uint32_t*>(base), q_full, q_full + kslice_q_floats(p.channels, p.k)};
}

int check_problem(const ReferenceProblem& p) {
  if (p.layout != SDC_LAYOUT_TILE && p.layout != SDC_LAYOUT_KSLICE) {
    return fail(SDC_ERR_INVALID, "unknown ABFT reference layout");
  }
  const size_t need = reference_workspace_bytes(p.channels, p.m, p.n, p.k, p.layout);
  if (p.workspace == nullptr || p.workspace_bytes < need) {
    return fail(SDC_ERR_WORKSPACE, "ABFT reference workspace too small");
  }
  if (reinterpret_cast<uintptr_t>(p.workspace) % 16 != 0) {
    return fail(SDC_ERR_WORKSPACE, "ABFT reference workspace must be 16-byte aligned");
  }
  return SDC_OK;
}


int launch_projection(const ReferenceProblem& p, cudaStream_t stream) {
  int rc = check_problem(p);
  if (rc != SDC_OK) return rc;
  if (p.kind == Kind::kFp8) {
    return p.channels == 2 ? projection_impl<Kind::kFp8, 2>(p, stream) : projection_impl<Kind::kFp8, 1>(p, stream);
  }
  return p.channels == 2 ? projection_impl<Kind::kNvf4, 2>(p, stream) : projection_impl<Kind::kNvf4, 1>(p, stream);
}

int launch_tile_propagate(const ReferenceProblem& p, cudaStream_t stream) {
  int rc = check_problem(p);
  if (rc != SDC_OK) return rc;
  if (p.kind == Kind::kFp8) {
    return p.channels == 2 ? tile_propagate_impl<Kind::kFp8, 2>(p, stream)
                           : tile_propagate_impl<Kind::kFp8, 1>(p, stream);
  }
  return p.channels == 2 ? tile_propagate_impl<Kind::kNvf4, 2>(p, stream)
                         : tile_propagate_impl<Kind::kNvf4, 1>(p, stream);
}

}  // namespace sdc
