// Operand quantisation for the ABFT GEMMs.
//
// Semantics follow src/cutlass_gemm/quantization.py:99-162 of the reference:
//   FP8   st = 448 / amax(|x|)  (1 when amax == 0), codes = e4m3_rn_sat(x * st)
//   NVFP4 st = 2688 / amax; per 16-block s = e4m3(amax16 * (st * (1/6)));
//         codes = e2m1_rn_sat(x * min((1/s) * st, FLT_MAX)), low nibble = even k
// The reference runs a torch amax, a torch multiply and a CuTe conversion
// kernel, plus a host-built index table and a scatter for the NVFP4 scale
// layout. Here it is two memory-bound passes: (1) per-block |x| maxima into a
// small workspace, (2) every block re-reduces those maxima from L2 (no atomics,
// no memset, no host sync), derives st and writes codes, natural scales and
// the MMA-layout scales in one streaming pass with 16-byte accesses.
#include <algorithm>
#include <cfloat>

#include "common.cuh"

namespace sdc {
namespace {

constexpr int kQuantThreads = 256;
constexpr int kMaxAmaxBlocks = 148 * 8;

// |x| as ordered bits: for non-negative floats the unsigned bit pattern is
// monotone, and NaN payloads order above +inf, so the integer max propagates
// NaN the way torch.amax does.
__device__ __forceinline__ uint32_t abs_bits(float v) { return __float_as_uint(v) & 0x7FFFFFFFu; }

template <int DT>
__device__ __forceinline__ float load_elem(const void* x, int64_t i) {
  if constexpr (DT == 0) {
    return static_cast<const float*>(x)[i];
  } else {
    return bf16_bits_to_float(static_cast<const uint16_t*>(x)[i]);
  }
}

// Loads 8 consecutive elements starting at i (i % 8 == 0, base 16-byte aligned).
template <int DT>
__device__ __forceinline__ void load8(const void* x, int64_t i, float (&v)[8]) {
  if constexpr (DT == 0) {
    const float4* p = reinterpret_cast<const float4*>(static_cast<const float*>(x) + i);
    const float4 a = __ldg(p), b = __ldg(p + 1);
    v[0] = a.x; v[1] = a.y; v[2] = a.z; v[3] = a.w;
    v[4] = b.x; v[5] = b.y; v[6] = b.z; v[7] = b.w;
  } else {
    const uint4 a = __ldg(reinterpret_cast<const uint4*>(static_cast<const uint16_t*>(x) + i));
    const uint32_t w[4] = {a.x, a.y, a.z, a.w};
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      v[2 * j] = __uint_as_float(w[j] << 16);
      v[2 * j + 1] = __uint_as_float(w[j] & 0xFFFF0000u);
    }
  }
}

template <int DT>
__global__ void __launch_bounds__(kQuantThreads)
    amax_partials(const void* x, int64_t count, bool vec, uint32_t* partial) {
  uint32_t m = 0;
  const int64_t tid = static_cast<int64_t>(blockIdx.x) * kQuantThreads + threadIdx.x;
  const int64_t stride = static_cast<int64_t>(gridDim.x) * kQuantThreads;
  if (vec) {
    const int64_t groups = count / 8;
    for (int64_t g = tid; g < groups; g += stride) {
      float v[8];
      load8<DT>(x, g * 8, v);
#pragma unroll
      for (int j = 0; j < 8; ++j) m = max(m, abs_bits(v[j]));
    }
    for (int64_t i = groups * 8 + tid; i < count; i += stride) m = max(m, abs_bits(load_elem<DT>(x, i)));
  } else {
    for (int64_t i = tid; i < count; i += stride) m = max(m, abs_bits(load_elem<DT>(x, i)));
  }
  for (int o = 16; o > 0; o >>= 1) m = max(m, __shfl_xor_sync(0xffffffffu, m, o));
  __shared__ uint32_t warp_max[kQuantThreads / 32];
  if ((threadIdx.x & 31) == 0) warp_max[threadIdx.x >> 5] = m;
  __syncthreads();
  if (threadIdx.x == 0) {
    uint32_t r = 0;
    for (int w = 0; w < kQuantThreads / 32; ++w) r = max(r, warp_max[w]);
    partial[blockIdx.x] = r;
  }
}

// Every block derives st from the partial maxima (or the fixed scale).
__device__ __forceinline__ float block_multiplier(const uint32_t* partial, int blocks, bool use_amax,
                                                  float fixed, float limit) {
  __shared__ float s_st;
  if (!use_amax) return fixed;
  uint32_t m = 0;
  for (int i = threadIdx.x; i < blocks; i += kQuantThreads) m = max(m, partial[i]);
  for (int o = 16; o > 0; o >>= 1) m = max(m, __shfl_xor_sync(0xffffffffu, m, o));
  __shared__ uint32_t warp_max[kQuantThreads / 32];
  if ((threadIdx.x & 31) == 0) warp_max[threadIdx.x >> 5] = m;
  __syncthreads();
  if (threadIdx.x == 0) {
    uint32_t r = 0;
    for (int w = 0; w < kQuantThreads / 32; ++w) r = max(r, warp_max[w]);
    const float amax = __uint_as_float(r);
    s_st = (amax == 0.f) ? 1.f : __fdiv_rn(limit, amax);
  }
  __syncthreads();
  return s_st;
}

template <int DT>
__global__ void __launch_bounds__(kQuantThreads)
    fp8_cast(const void* x, int64_t count, bool vec, const uint32_t* partial, int blocks,
             bool use_amax, float fixed, uint8_t* codes, float* multiplier) {
  const float st = block_multiplier(partial, blocks, use_amax, fixed, 448.f);
  if (blockIdx.x == 0 && threadIdx.x == 0) *multiplier = st;
  const int64_t tid = static_cast<int64_t>(blockIdx.x) * kQuantThreads + threadIdx.x;
  const int64_t stride = static_cast<int64_t>(gridDim.x) * kQuantThreads;
  int64_t done = 0;
  if (vec) {
    const int64_t groups = count / 16;
    for (int64_t g = tid; g < groups; g += stride) {
      float v[16];
      load8<DT>(x, g * 16, *reinterpret_cast<float(*)[8]>(&v[0]));
      load8<DT>(x, g * 16 + 8, *reinterpret_cast<float(*)[8]>(&v[8]));
      uint32_t w[4];
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const uint32_t lo = cvt_e4m3x2(__fmul_rn(v[4 * j], st), __fmul_rn(v[4 * j + 1], st));
        const uint32_t hi = cvt_e4m3x2(__fmul_rn(v[4 * j + 2], st), __fmul_rn(v[4 * j + 3], st));
        w[j] = lo | (hi << 16);
      }
      reinterpret_cast<uint4*>(codes)[g] = make_uint4(w[0], w[1], w[2], w[3]);
    }
    done = groups * 16;
  }
  for (int64_t i = done + tid; i < count; i += stride) {
    codes[i] = static_cast<uint8_t>(cvt_e4m3x2(__fmul_rn(load_elem<DT>(x, i), st), 0.f) & 0xFFu);
  }
}

__host__ __device__ __forceinline__ int64_t sf_offset(int64_t row, int64_t block, int64_t k_atoms) {
  // 128 rows x 4 blocks of 16 per 512-byte atom; atoms tile K first, then rows.
  return ((row >> 7) * k_atoms + (block >> 2)) * 512 + (row & 31) * 16 + ((row >> 5) & 3) * 4 +
         (block & 3);
}

template <int DT>
__global__ void __launch_bounds__(kQuantThreads)
    nvfp4_cast(const void* x, int64_t rows, int64_t cols, bool vec, const uint32_t* partial,
               int blocks, bool use_amax, float fixed, uint8_t* codes, uint8_t* scales,
               uint8_t* scales_mma, float* multiplier) {
  const float st = block_multiplier(partial, blocks, use_amax, fixed, 2688.f);
  if (blockIdx.x == 0 && threadIdx.x == 0) *multiplier = st;
  // st * (1/6) in fp32 exactly as the reference's scalar promotion does.
  const float st_sixth = __fmul_rn(st, 0.16666667163372039795f);
  const int64_t per_row = cols / 16;
  const int64_t total = rows * per_row;
  const int64_t k_atoms = (cols + 63) / 64;
  const int64_t tid = static_cast<int64_t>(blockIdx.x) * kQuantThreads + threadIdx.x;
  const int64_t stride = static_cast<int64_t>(gridDim.x) * kQuantThreads;
  for (int64_t b = tid; b < total; b += stride) {
    float v[16];
    if (vec) {
      load8<DT>(x, b * 16, *reinterpret_cast<float(*)[8]>(&v[0]));
      load8<DT>(x, b * 16 + 8, *reinterpret_cast<float(*)[8]>(&v[8]));
    } else {
#pragma unroll
      for (int j = 0; j < 16; ++j) v[j] = load_elem<DT>(x, b * 16 + j);
    }
    uint32_t m = 0;
#pragma unroll
    for (int j = 0; j < 16; ++j) m = max(m, abs_bits(v[j]));
    const float scale_value = __fmul_rn(__uint_as_float(m), st_sixth);
    const uint32_t sbyte = cvt_e4m3x2(scale_value, 0.f) & 0xFFu;
    const float decoded = decode_e4m3(sbyte);
    float acc = __fmul_rn(__frcp_rn(decoded), st);
    acc = acc > FLT_MAX ? FLT_MAX : acc;  // clamp_max(FLT_MAX); NaN passes through
    float lo[8], hi[8];
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      lo[j] = __fmul_rn(v[j], acc);
      hi[j] = __fmul_rn(v[8 + j], acc);
    }
    const uint2 packed = make_uint2(cvt_e2m1x8(lo), cvt_e2m1x8(hi));
    if (vec) {
      reinterpret_cast<uint2*>(codes)[b] = packed;
    } else {
      uint8_t* dst = codes + b * 8;
      for (int j = 0; j < 4; ++j) dst[j] = (packed.x >> (8 * j)) & 0xFF;
      for (int j = 0; j < 4; ++j) dst[4 + j] = (packed.y >> (8 * j)) & 0xFF;
    }
    const int64_t row = b / per_row;
    const int64_t blk = b - row * per_row;
    if (scales != nullptr) scales[b] = static_cast<uint8_t>(sbyte);
    if (scales_mma != nullptr) scales_mma[sf_offset(row, blk, k_atoms)] = static_cast<uint8_t>(sbyte);
  }
}

__global__ void pack_scales_kernel(const uint8_t* scales, int64_t rows, int64_t per_row,
                                   int64_t k_atoms, uint8_t* packed) {
  const int64_t total = rows * per_row;
  for (int64_t b = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; b < total;
       b += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int64_t row = b / per_row;
    packed[sf_offset(row, b - row * per_row, k_atoms)] = scales[b];
  }
}

int amax_blocks(int64_t count) {
  return static_cast<int>(std::max<int64_t>(1, std::min<int64_t>(kMaxAmaxBlocks, ceil_div(count, kQuantThreads * 16))));
}

int grid_for(int64_t work) {
  return static_cast<int>(std::max<int64_t>(1, std::min<int64_t>(148 * 16, ceil_div(work, kQuantThreads))));
}

// ---- block-scaled FP8 (1 x 128 and 128 x 128 fp32 scales) ----------------
// A 128-wide K block of `BR` rows shares one dequantisation scale
// d = amax(|x|) / 448 (1 when amax == 0); codes = e4m3_rn_satfinite(x / d),
// so x ~ code * d. BR = 1 (activations, one warp per block) or 128 (weights,
// one CTA per block).
// Block-scaled FP8 cast: d = amax(|block|) / 448 (1 for an all-zero block),
// code = e4m3_rn_satfinite(x / d).
// BR = 1 (1 x 128 blocks): 16 lanes per block, 8 consecutive elements (one or
// two 16-byte loads) per lane, two blocks per warp.
// BR = 128 (128 x 128 blocks): one CTA per block; every warp-wide load and
// store covers two rows of the block contiguously.
template <int DT, int BR>
__global__ void __launch_bounds__(kQuantThreads)
    fp8_block_cast(const void* x, int64_t rows, int64_t cols, uint8_t* codes, float* scales) {
  const int64_t kblocks = cols / 128;
  const int lane = threadIdx.x & 31;
  if constexpr (BR == 1) {
    const int64_t blk = static_cast<int64_t>(blockIdx.x) * (kQuantThreads / 16) + (threadIdx.x >> 4);
    if (blk >= rows * kblocks) return;  // whole 16-lane groups leave together
    const int64_t r = blk / kblocks, kb = blk - r * kblocks;
    const int64_t base = r * cols + kb * 128 + (threadIdx.x & 15) * 8;
    float v[8];
    load8<DT>(x, base, v);
    uint32_t bits = 0;
#pragma unroll
    for (int e = 0; e < 8; ++e) bits = max(bits, abs_bits(v[e]));
    const uint32_t group = 0xFFFFu << (lane & 16);
#pragma unroll
    for (int o = 8; o > 0; o >>= 1) bits = max(bits, __shfl_xor_sync(group, bits, o));
    const float amax = __uint_as_float(bits);
    const float d = amax == 0.f ? 1.f : __fdiv_rn(amax, 448.f);
    uint32_t w[4];
#pragma unroll
    for (int j = 0; j < 4; ++j) w[j] = cvt_e4m3x2(__fdiv_rn(v[2 * j], d), __fdiv_rn(v[2 * j + 1], d));
    *reinterpret_cast<uint2*>(codes + base) = make_uint2(w[0] | (w[1] << 16), w[2] | (w[3] << 16));
    if ((threadIdx.x & 15) == 0) scales[r * kblocks + kb] = d;
  } else {
    __shared__ uint32_t warp_max[kQuantThreads / 32];
    const int warp = threadIdx.x >> 5;
    const int64_t rb = blockIdx.x / kblocks, kb = blockIdx.x - rb * kblocks;
    // 16 lanes per row (8 columns each, 16-byte loads), two rows per warp and
    // instruction; warp w owns rows 16w..16w+15 of the block.
    const int64_t row0 = rb * 128 + warp * 16 + (lane >> 4);
    const int64_t col = kb * 128 + (lane & 15) * 8;
    float v[8][8];
    uint32_t bits = 0;
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      if (row0 + 2 * i < rows) {
        load8<DT>(x, (row0 + 2 * i) * cols + col, v[i]);
      } else {
#pragma unroll
        for (int e = 0; e < 8; ++e) v[i][e] = 0.f;
      }
#pragma unroll
      for (int e = 0; e < 8; ++e) bits = max(bits, abs_bits(v[i][e]));
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) bits = max(bits, __shfl_xor_sync(0xffffffffu, bits, o));
    if (lane == 0) warp_max[warp] = bits;
    __syncthreads();
    bits = 0;
#pragma unroll
    for (int w = 0; w < kQuantThreads / 32; ++w) bits = max(bits, warp_max[w]);
    const float amax = __uint_as_float(bits);
    const float d = amax == 0.f ? 1.f : __fdiv_rn(amax, 448.f);
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      if (row0 + 2 * i < rows) {
        uint32_t w[4];
#pragma unroll
        for (int j = 0; j < 4; ++j) w[j] = cvt_e4m3x2(__fdiv_rn(v[i][2 * j], d), __fdiv_rn(v[i][2 * j + 1], d));
        *reinterpret_cast<uint2*>(codes + (row0 + 2 * i) * cols + col) = make_uint2(w[0] | (w[1] << 16), w[2] | (w[3] << 16));
      }
    }
    if (threadIdx.x == 0) scales[rb * kblocks + kb] = d;
  }
}

}  // namespace
}  // namespace sdc

extern "C" {

size_t sdc_quantize_workspace_bytes(int64_t rows, int64_t cols) {
  return static_cast<size_t>(sdc::amax_blocks(rows * cols)) * sizeof(uint32_t);
}

int64_t sdc_nvfp4_scale_offset(int64_t row, int64_t block, int64_t k) {
  return sdc::sf_offset(row, block, (k + 63) / 64);
}

int64_t sdc_nvfp4_scale_size(int64_t rows, int64_t k) {
  return sdc::ceil_div(rows, 128) * 128 * sdc::ceil_div(k, 64) * 4;
}

int sdc_nvfp4_scale_layout(int64_t rows, int64_t k, int64_t* indices) {
  SDC_REQUIRE(rows > 0 && k > 0 && k % 16 == 0, "NVFP4 scale layout needs rows > 0 and k % 16 == 0");
  SDC_REQUIRE(indices != nullptr, "indices must not be null");
  const int64_t per_row = k / 16, k_atoms = (k + 63) / 64;
  for (int64_t r = 0; r < rows; ++r) {
    for (int64_t b = 0; b < per_row; ++b) indices[r * per_row + b] = sdc::sf_offset(r, b, k_atoms);
  }
  return SDC_OK;
}

int sdc_nvfp4_pack_scales(const uint8_t* scales, int64_t rows, int64_t k, uint8_t* packed,
                          sdc_stream_t stream) {
  using namespace sdc;
  SDC_REQUIRE(rows > 0 && k > 0 && k % 16 == 0, "NVFP4 scale packing needs rows > 0 and k % 16 == 0");
  SDC_REQUIRE(scales != nullptr && packed != nullptr, "scale pointers must not be null");
  SDC_CUDA_CHECK(cudaMemsetAsync(packed, 0, sdc_nvfp4_scale_size(rows, k), stream));
  const int64_t per_row = k / 16;
  pack_scales_kernel<<<grid_for(rows * per_row), kQuantThreads, 0, stream>>>(
      scales, rows, per_row, (k + 63) / 64, packed);
  SDC_CUDA_CHECK(cudaGetLastError());
  return SDC_OK;
}

int sdc_quantize_fp8(const void* x, int dtype, int64_t rows, int64_t cols, int use_amax,
                     float global_scale, uint8_t* codes, float* multiplier, void* workspace,
                     size_t workspace_bytes, sdc_stream_t stream) {
  using namespace sdc;
  SDC_REQUIRE(dtype == 0 || dtype == 1, "quantize requires FP32 (0) or BF16 (1) input");
  SDC_REQUIRE(rows > 0 && cols > 0, "quantize requires a nonempty matrix");
  SDC_REQUIRE(x != nullptr && codes != nullptr && multiplier != nullptr, "quantize pointers must not be null");
  const int64_t count = rows * cols;
  const int blocks = amax_blocks(count);
  if (use_amax && (workspace == nullptr || workspace_bytes < blocks * sizeof(uint32_t))) {
    return fail(SDC_ERR_WORKSPACE, "quantize workspace too small");
  }
  const bool vec = (reinterpret_cast<uintptr_t>(x) % 16 == 0) && (reinterpret_cast<uintptr_t>(codes) % 16 == 0);
  uint32_t* partial = static_cast<uint32_t*>(workspace);
  if (use_amax) {
    if (dtype == 0) amax_partials<0><<<blocks, kQuantThreads, 0, stream>>>(x, count, vec, partial);
    else amax_partials<1><<<blocks, kQuantThreads, 0, stream>>>(x, count, vec, partial);
    SDC_CUDA_CHECK(cudaGetLastError());
  }
  const int grid = grid_for(ceil_div(count, 16));
  if (dtype == 0) {
    fp8_cast<0><<<grid, kQuantThreads, 0, stream>>>(x, count, vec, partial, blocks, use_amax != 0,
                                                    global_scale, codes, multiplier);
  } else {
    fp8_cast<1><<<grid, kQuantThreads, 0, stream>>>(x, count, vec, partial, blocks, use_amax != 0,
                                                    global_scale, codes, multiplier);
  }
  SDC_CUDA_CHECK(cudaGetLastError());
  return SDC_OK;
}

int sdc_quantize_nvfp4(const void* x, int dtype, int64_t rows, int64_t cols, int use_amax,
                       float global_scale, uint8_t* codes, uint8_t* scales, uint8_t* scales_mma,
                       float* multiplier, void* workspace, size_t workspace_bytes,
                       sdc_stream_t stream) {
  using namespace sdc;
  SDC_REQUIRE(dtype == 0 || dtype == 1, "quantize requires FP32 (0) or BF16 (1) input");
  SDC_REQUIRE(rows > 0 && cols > 0 && cols % 16 == 0, "nonempty input columns must be divisible by 16");
  SDC_REQUIRE(x != nullptr && codes != nullptr && multiplier != nullptr, "quantize pointers must not be null");
  const int64_t count = rows * cols;
  const int blocks = amax_blocks(count);
  if (use_amax && (workspace == nullptr || workspace_bytes < blocks * sizeof(uint32_t))) {
    return fail(SDC_ERR_WORKSPACE, "quantize workspace too small");
  }
  const bool vec = (reinterpret_cast<uintptr_t>(x) % 16 == 0) && (reinterpret_cast<uintptr_t>(codes) % 8 == 0);
  uint32_t* partial = static_cast<uint32_t*>(workspace);
  if (use_amax) {
    if (dtype == 0) amax_partials<0><<<blocks, kQuantThreads, 0, stream>>>(x, count, vec, partial);
    else amax_partials<1><<<blocks, kQuantThreads, 0, stream>>>(x, count, vec, partial);
    SDC_CUDA_CHECK(cudaGetLastError());
  }
  if (scales_mma != nullptr && (rows % 128 != 0 || cols % 64 != 0)) {
    SDC_CUDA_CHECK(cudaMemsetAsync(scales_mma, 0, sdc_nvfp4_scale_size(rows, cols), stream));
  }
  const int grid = grid_for(rows * (cols / 16));
  if (dtype == 0) {
    nvfp4_cast<0><<<grid, kQuantThreads, 0, stream>>>(x, rows, cols, vec, partial, blocks, use_amax != 0,
                                                      global_scale, codes, scales, scales_mma, multiplier);
  } else {
    nvfp4_cast<1><<<grid, kQuantThreads, 0, stream>>>(x, rows, cols, vec, partial, blocks, use_amax != 0,
                                                      global_scale, codes, scales, scales_mma, multiplier);
  }
  SDC_CUDA_CHECK(cudaGetLastError());
  return SDC_OK;
}


// Quantisation of one shard of a row-sharded matrix with the multiplier of
// the whole matrix: `amax` is a device fp32 scalar holding max |x| over every
// shard (e.g. a MAX all-reduce of the shards' maxima). The cast kernels
// derive st from it exactly as from their own partial maxima (a non-negative
// float's bits order like its value), so the codes equal the unsharded
// matrix's rows bit for bit, with no host read of the maximum.
int sdc_quantize_fp8_global_amax(const void* x, int dtype, int64_t rows, int64_t cols, const float* amax,
                                 uint8_t* codes, float* multiplier, sdc_stream_t stream) {
  using namespace sdc;
  SDC_REQUIRE(dtype == 0 || dtype == 1, "quantize requires FP32 (0) or BF16 (1) input");
  SDC_REQUIRE(rows > 0 && cols > 0, "quantize requires a nonempty matrix");
  SDC_REQUIRE(x != nullptr && amax != nullptr && codes != nullptr && multiplier != nullptr,
              "quantize pointers must not be null");
  const int64_t count = rows * cols;
  const bool vec = (reinterpret_cast<uintptr_t>(x) % 16 == 0) && (reinterpret_cast<uintptr_t>(codes) % 16 == 0);
  const uint32_t* bits = reinterpret_cast<const uint32_t*>(amax);
  const int grid = grid_for(ceil_div(count, 16));
  if (dtype == 0) {
    fp8_cast<0><<<grid, kQuantThreads, 0, stream>>>(x, count, vec, bits, 1, true, 1.f, codes, multiplier);
  } else {
    fp8_cast<1><<<grid, kQuantThreads, 0, stream>>>(x, count, vec, bits, 1, true, 1.f, codes, multiplier);
  }
  SDC_CUDA_CHECK(cudaGetLastError());
  return SDC_OK;
}

int sdc_quantize_nvfp4_global_amax(const void* x, int dtype, int64_t rows, int64_t cols, const float* amax,
                                   uint8_t* codes, uint8_t* scales, uint8_t* scales_mma, float* multiplier,
                                   sdc_stream_t stream) {
  using namespace sdc;
  SDC_REQUIRE(dtype == 0 || dtype == 1, "quantize requires FP32 (0) or BF16 (1) input");
  SDC_REQUIRE(rows > 0 && cols > 0 && cols % 16 == 0, "nonempty input columns must be divisible by 16");
  SDC_REQUIRE(x != nullptr && amax != nullptr && codes != nullptr && multiplier != nullptr,
              "quantize pointers must not be null");
  const bool vec = (reinterpret_cast<uintptr_t>(x) % 16 == 0) && (reinterpret_cast<uintptr_t>(codes) % 8 == 0);
  if (scales_mma != nullptr && (rows % 128 != 0 || cols % 64 != 0)) {
    SDC_CUDA_CHECK(cudaMemsetAsync(scales_mma, 0, sdc_nvfp4_scale_size(rows, cols), stream));
  }
  const uint32_t* bits = reinterpret_cast<const uint32_t*>(amax);
  const int grid = grid_for(rows * (cols / 16));
  if (dtype == 0) {
    nvfp4_cast<0><<<grid, kQuantThreads, 0, stream>>>(x, rows, cols, vec, bits, 1, true, 1.f, codes, scales,
                                                      scales_mma, multiplier);
  } else {
    nvfp4_cast<1><<<grid, kQuantThreads, 0, stream>>>(x, rows, cols, vec, bits, 1, true, 1.f, codes, scales,
                                                      scales_mma, multiplier);
  }
  SDC_CUDA_CHECK(cudaGetLastError());
  return SDC_OK;
}

}  // extern "C"

extern "C" int sdc_quantize_fp8_block(const void* x, int dtype, int64_t rows, int64_t cols, int block_rows,
                                      uint8_t* codes, float* scales, sdc_stream_t stream) {
  using namespace sdc;
  SDC_REQUIRE(dtype == 0 || dtype == 1, "quantize requires FP32 (0) or BF16 (1) input");
  SDC_REQUIRE(rows > 0 && cols > 0 && cols % 128 == 0, "block-scaled FP8 needs rows > 0 and cols % 128 == 0");
  SDC_REQUIRE(block_rows == 1 || block_rows == 128, "block-scaled FP8 blocks are 1 x 128 or 128 x 128");
  SDC_REQUIRE(x != nullptr && codes != nullptr && scales != nullptr, "quantize pointers must not be null");
  SDC_REQUIRE(reinterpret_cast<uintptr_t>(x) % 16 == 0 && reinterpret_cast<uintptr_t>(codes) % 8 == 0 &&
                  reinterpret_cast<uintptr_t>(scales) % 4 == 0,
              "block-scaled FP8 input must be 16-byte aligned, codes 8-byte and scales 4-byte aligned");
  const int64_t kblocks = cols / 128;
  if (block_rows == 1) {
    const unsigned grid = static_cast<unsigned>(ceil_div(rows * kblocks, kQuantThreads / 16));
    if (dtype == 0) fp8_block_cast<0, 1><<<grid, kQuantThreads, 0, stream>>>(x, rows, cols, codes, scales);
    else fp8_block_cast<1, 1><<<grid, kQuantThreads, 0, stream>>>(x, rows, cols, codes, scales);
  } else {
    const unsigned grid = static_cast<unsigned>(ceil_div(rows, 128) * kblocks);
    if (dtype == 0) fp8_block_cast<0, 128><<<grid, kQuantThreads, 0, stream>>>(x, rows, cols, codes, scales);
    else fp8_block_cast<1, 128><<<grid, kQuantThreads, 0, stream>>>(x, rows, cols, codes, scales);
  }
  SDC_CUDA_CHECK(cudaGetLastError());
  return SDC_OK;
}
