// K-slice input-side prediction: the pieces shared by the fused path (the
// GEMM's prediction warps, gemm.cu) and the standalone kernels (kslice.cu).
//
// predicted[c][t][n] = alpha * sum over the 64-wide K slices s with
// s % Tm == t (ascending) of sum_{k in s} q_c[k] * B[n][k] (one fp32 fma chain
// per (c, t, n), k ascending), magnitude likewise with |q| and |B|; q is the
// projection w_c^T A over all rows. Fixed summation order of q (mirrored by
// oracle/cref.c): bands of kBandRows rows; in a band, 8 row lanes l each run
// an fma chain over rows band_start + l, + 8, ... (ascending), combined as
// ((p0 + p1) + (p2 + p3)) + ((p4 + p5) + (p6 + p7)); the bands are then
// added in ascending order.
#pragma once

#include "gemm.cuh"

namespace sdc {

constexpr int kSliceK = 64;     // K elements per input-checksum slice
constexpr int kBandRows = 128;  // rows per projection band

// What one projection item reads and writes. The projected operand is A for
// the column checksums and B (rows [N][K], unit weights) for the row
// checksums' e^T B.
struct ProjectionView {
  const uint8_t* a;        // codes: e4m3 [M][K] or packed e2m1 [M][K/2]
  const float* sa;         // block-scaled FP8: scales [ceil(M / 2^scale_shift)][K/128]
  const uint8_t* sfa;      // NVFP4: scale atoms
  const float* weights;    // [C][M]; null = every weight 1
  int64_t m, k;
  int64_t k_blocks;        // K / 128 (block-scaled)
  int64_t num_slices;      // ceil(K / 64)
  float* q_part;           // [bands][K_pad][C][2]
  int scale_shift = 0;     // block-scaled FP8: log2 rows per scale row (0 for A, 7 for B)
};

// One item = (band, slice `chunk`) for one warp: lane = 4 * l + g covers
// k-group g (16 consecutive k of the slice) and row lane l. Writes the band's
// partial q (and |w|^T |A|) of the slice's 64 k to dst[64][C][2].
// kBatch rows of each row lane are loaded before their fma chains (a larger
// batch keeps more loads in flight at the cost of registers; the arithmetic
// and its order do not depend on it).
template <Kind KIND, int C, int kBatch = 4>
__device__ __forceinline__ void project_item(const ProjectionView& v, int64_t band, int64_t chunk, int lane,
                                             float* dst) {
  constexpr bool BLK = KIND == Kind::kFp8Block;
  const int g = lane & 3, l = lane >> 2;
  const int64_t row_bytes = is_e4m3(KIND) ? v.k : v.k / 2;
  const int64_t k_atoms = (v.k + 63) / 64;
  const int64_t k0 = chunk * kSliceK + g * 16;
  // K % 16 == 0 (FP8) / % 32 == 0 (NVFP4): a group of 16 is all in or all out.
  const bool k_in = k0 < v.k;
  const int64_t row_end = min(v.m, (band + 1) * kBandRows);
  float2 enc[16], mg[16];
#pragma unroll
  for (int e = 0; e < 16; ++e) enc[e] = mg[e] = make_float2(0.f, 0.f);
  for (int64_t r0 = band * kBandRows + l; r0 < row_end; r0 += 8 * kBatch) {
    uint4 raw[kBatch];
    uint32_t sfv[kBatch];
    float w[kBatch][C];
#pragma unroll
    for (int i = 0; i < kBatch; ++i) {
      const int64_t row = r0 + 8 * i;
      const bool row_in = row < row_end;
      const bool in = row_in && k_in;
      if constexpr (is_e4m3(KIND)) {
        raw[i] = in ? __ldg(reinterpret_cast<const uint4*>(v.a + row * row_bytes + k0)) : make_uint4(0, 0, 0, 0);
        // Block-scaled: the row's scale of the 128-wide block holding these 16 k.
        if constexpr (BLK) {
          sfv[i] = in ? __float_as_uint(__ldg(v.sa + (row >> v.scale_shift) * v.k_blocks + (k0 >> 7))) : 0u;
        }
      } else {
        const uint2 u = in ? __ldg(reinterpret_cast<const uint2*>(v.a + row * row_bytes + k0 / 2)) : make_uint2(0, 0);
        raw[i] = make_uint4(u.x, u.y, 0, 0);
        const int64_t off = ((row >> 7) * k_atoms + (k0 >> 6)) * 512 + (row & 31) * 16 + ((row >> 5) & 3) * 4 +
                            ((k0 >> 4) & 3);
        sfv[i] = in ? __ldg(v.sfa + off) : 0u;
      }
#pragma unroll
      for (int c = 0; c < C; ++c) {
        w[i][c] = !row_in ? 0.f : v.weights != nullptr ? __ldg(v.weights + static_cast<int64_t>(c) * v.m + row) : 1.f;
      }
    }
#pragma unroll
    for (int i = 0; i < kBatch; ++i) {
      if (r0 + 8 * i >= row_end) break;
      float val[16];
      if constexpr (is_e4m3(KIND)) {
        const uint32_t words[4] = {raw[i].x, raw[i].y, raw[i].z, raw[i].w};
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          const float2 lo = e4m3x2_to_float2(words[j] & 0xFFFFu), hi = e4m3x2_to_float2(words[j] >> 16);
          val[4 * j] = lo.x;
          val[4 * j + 1] = lo.y;
          val[4 * j + 2] = hi.x;
          val[4 * j + 3] = hi.y;
        }
        if constexpr (BLK) {
          const float scale = __uint_as_float(sfv[i]);
#pragma unroll
          for (int e = 0; e < 16; ++e) val[e] = __fmul_rn(val[e], scale);
        }
      } else {
        float lo8[8], hi8[8];
        e2m1x8_to_float(raw[i].x, lo8);
        e2m1x8_to_float(raw[i].y, hi8);
        const float scale = decode_e4m3(sfv[i]);
#pragma unroll
        for (int e = 0; e < 8; ++e) {
          val[e] = __fmul_rn(lo8[e], scale);
          val[8 + e] = __fmul_rn(hi8[e], scale);
        }
      }
      const float2 wv = make_float2(w[i][0], C == 2 ? w[i][C - 1] : 0.f);
      const float2 wa = make_float2(fabsf(wv.x), fabsf(wv.y));
#pragma unroll
      for (int e = 0; e < 16; ++e) {
        enc[e] = fma2(wv, make_float2(val[e], val[e]), enc[e]);
        const float av = fabsf(val[e]);
        mg[e] = fma2(wa, make_float2(av, av), mg[e]);
      }
    }
  }
  // Row lanes l = lane >> 2: xor 4, 8, 16 pair (l0,l1), (l0+l1, l2+l3), ...
#pragma unroll
  for (int offset = 4; offset <= 16; offset <<= 1) {
#pragma unroll
    for (int e = 0; e < 16; ++e) {
      enc[e].x = __fadd_rn(enc[e].x, __shfl_xor_sync(0xffffffffu, enc[e].x, offset));
      enc[e].y = __fadd_rn(enc[e].y, __shfl_xor_sync(0xffffffffu, enc[e].y, offset));
      mg[e].x = __fadd_rn(mg[e].x, __shfl_xor_sync(0xffffffffu, mg[e].x, offset));
      mg[e].y = __fadd_rn(mg[e].y, __shfl_xor_sync(0xffffffffu, mg[e].y, offset));
    }
  }
  if (l == 0) {
    float* out = dst + g * 16 * C * 2;
#pragma unroll
    for (int e = 0; e < 16; ++e) {
      if constexpr (C == 2) {
        reinterpret_cast<float4*>(out)[e] = make_float4(enc[e].x, mg[e].x, enc[e].y, mg[e].y);
      } else {
        reinterpret_cast<float2*>(out)[e] = make_float2(enc[e].x, mg[e].x);
      }
    }
  }
}

// Packed decodes for the prediction's inner loop. Every e2m1 code times its
// ue4m3 block scale is exact in fp16 (at most 6 significant bits, magnitudes
// 2^-10 .. 2688), so the product is formed two at a time in fp16 and widened:
// the same fp32 values as code * scale computed in fp32.
__device__ __forceinline__ uint32_t e4m3x2_to_h2(uint32_t two_bytes) {
  uint32_t h2;
  asm("cvt.rn.f16x2.e4m3x2 %0, %1;" : "=r"(h2) : "h"(static_cast<uint16_t>(two_bytes)));
  return h2;
}

__device__ __forceinline__ uint32_t e2m1x2_to_h2(uint32_t byte) {
  uint32_t h2;
  asm("{\n\t.reg .b8 b;\n\tcvt.u8.u32 b, %1;\n\tcvt.rn.f16x2.e2m1x2 %0, b;\n\t}" : "=r"(h2) : "r"(byte));
  return h2;
}

__device__ __forceinline__ uint32_t hmul2_rn(uint32_t a, uint32_t b) {
  uint32_t d;
  asm("mul.rn.f16x2 %0, %1, %2;" : "=r"(d) : "r"(a), "r"(b));
  return d;
}

__device__ __forceinline__ float2 h2_to_float2(uint32_t h2) {
  float2 out;
  asm("{\n\t.reg .f16 lo, hi;\n\tmov.b32 {lo, hi}, %2;\n\t"
      "cvt.f32.f16 %0, lo;\n\tcvt.f32.f16 %1, hi;\n\t}"
      : "=f"(out.x), "=f"(out.y)
      : "r"(h2));
  return out;
}

// q_full [K_pad][C][2] of `view` (bands summed in ascending order) by the
// standalone projection kernels (kslice.cu): the band partials go to
// view.q_part ([bands][K_pad][C][2]; unused when there is one band), then
// they are added in ascending band order.
int launch_projection_sums(Kind kind, int channels, const ProjectionView& view, float* q_full, cudaStream_t stream);

// The band partial of item (band, chunk) in the [bands][K_pad][C][2] layout.
template <int C>
__device__ __forceinline__ float* band_partial(const ProjectionView& v, int64_t band, int64_t chunk) {
  return v.q_part + (band * v.num_slices * kSliceK + chunk * kSliceK) * C * 2;
}

}  // namespace sdc
