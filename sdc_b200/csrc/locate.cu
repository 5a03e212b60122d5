// Error localisation (Classic two-channel ratio locator) and single-element
// correction by targeted recomputation.
//
// The locator restates Classic.verify of the reference
// (src/abft/methods.py:201-237) on the device, op for op in fp32 with
// round-to-nearest and no contraction, so its decisions equal the torch
// restatement for the same residual/threshold tensors.
#include <cfloat>

#include "gemm.cuh"

namespace sdc {
namespace {

constexpr int kLocThreads = 256;

__global__ void __launch_bounds__(kLocThreads)
    locate_kernel(const float* residual, const float* threshold, const uint8_t* flags, int64_t m,
                  int64_t n, int64_t* location, uint8_t* located_out) {
  // failed[c, col] = |residual| > threshold; columns = any over channels.
  int64_t first = INT64_MAX;
  int64_t count = 0;
  for (int64_t col = threadIdx.x; col < n; col += kLocThreads) {
    const bool f0 = fabsf(residual[col]) > threshold[col];
    const bool f1 = fabsf(residual[n + col]) > threshold[n + col];
    if (f0 || f1) {
      first = min(first, col);
      ++count;
    }
  }
  for (int o = 16; o > 0; o >>= 1) {
    first = min(first, __shfl_xor_sync(0xffffffffu, first, o));
    count += __shfl_xor_sync(0xffffffffu, count, o);
  }
  __shared__ int64_t s_first[kLocThreads / 32], s_count[kLocThreads / 32];
  if ((threadIdx.x & 31) == 0) {
    s_first[threadIdx.x >> 5] = first;
    s_count[threadIdx.x >> 5] = count;
  }
  __syncthreads();
  if (threadIdx.x != 0) return;
  first = INT64_MAX;
  count = 0;
  for (int w = 0; w < kLocThreads / 32; ++w) {
    first = min(first, s_first[w]);
    count += s_count[w];
  }
  const int64_t col = first == INT64_MAX ? 0 : first;  // argmax of an all-false vector is 0
  const float d0 = residual[col], d1 = residual[n + col];
  const float t0 = threshold[col], t1 = threshold[n + col];
  const bool detected = flags[0] != 0, nonfinite = flags[1] != 0;
  const float ratio = __fdiv_rn(d1, d0 == 0.f ? 1.f : d0);
  bool located = detected && !nonfinite && count == 1 && fabsf(d0) > t0 && isfinite(ratio);
  int64_t row = -1;
  if (located) {
    const float rounded = rintf(ratio);  // round half to even, as torch.round
    row = static_cast<int64_t>(rounded) - 1;
    const float rp1 = static_cast<float>(row + 1);
    const float consistency = fabsf(__fsub_rn(d1, __fmul_rn(rp1, d0)));
    const float allowance = __fadd_rn(t1, __fmul_rn(fabsf(rp1), t0));
    located = row >= 0 && row < m && consistency <= allowance;
    const float denom = fmaxf(__fsub_rn(fabsf(d0), t0), FLT_MIN);
    const float uncertainty = __fdiv_rn(__fadd_rn(t1, __fmul_rn(fabsf(ratio), t0)), denom);
    located = located && __fadd_rn(fabsf(__fsub_rn(ratio, rp1)), uncertainty) < 0.5f;
  }
  location[0] = located ? row : -1;
  location[1] = located ? col : -1;
  *located_out = located ? 1 : 0;
}

template <Kind KIND, bool BF16OUT>
__global__ void __launch_bounds__(kLocThreads)
    correct_kernel(const uint8_t* a, const uint8_t* b, const uint8_t* sfa, const uint8_t* sfb,
                   int64_t m, int64_t n, int64_t k, const float* alpha, const int64_t* location,
                   const uint8_t* located, void* d, uint8_t* corrected) {
  if (*located == 0) {
    if (threadIdx.x == 0) *corrected = 0;
    return;
  }
  const int64_t row = location[0], col = location[1];
  float sum = 0.f;
  for (int64_t kk = threadIdx.x; kk < k; kk += kLocThreads) {
    float av, bv;
    if constexpr (KIND == Kind::kFp8) {
      av = decode_e4m3(a[row * k + kk]);
      bv = decode_e4m3(b[col * k + kk]);
    } else if constexpr (KIND == Kind::kFp8Block) {
      // fp32 scales [m, k/128] (A) and [ceil(n/128), k/128] (B rows).
      const int64_t kb = k / 128;
      av = __fmul_rn(decode_e4m3(a[row * k + kk]), reinterpret_cast<const float*>(sfa)[row * kb + (kk >> 7)]);
      bv = __fmul_rn(decode_e4m3(b[col * k + kk]), reinterpret_cast<const float*>(sfb)[(col >> 7) * kb + (kk >> 7)]);
    } else {
      const int64_t k_atoms = (k + 63) / 64;
      const auto sf_off = [k_atoms](int64_t r, int64_t blk) {
        return ((r >> 7) * k_atoms + (blk >> 2)) * 512 + (r & 31) * 16 + ((r >> 5) & 3) * 4 + (blk & 3);
      };
      const uint32_t ab = a[row * (k / 2) + (kk >> 1)], bb = b[col * (k / 2) + (kk >> 1)];
      av = decode_e2m1((kk & 1) ? (ab >> 4) : (ab & 15u)) * decode_e4m3(sfa[sf_off(row, kk >> 4)]);
      bv = decode_e2m1((kk & 1) ? (bb >> 4) : (bb & 15u)) * decode_e4m3(sfb[sf_off(col, kk >> 4)]);
    }
    sum = fmaf(av, bv, sum);
  }
  __shared__ float partial[kLocThreads];
  partial[threadIdx.x] = sum;
  __syncthreads();
  for (int width = kLocThreads / 2; width > 0; width >>= 1) {
    if (threadIdx.x < width) partial[threadIdx.x] += partial[threadIdx.x + width];
    __syncthreads();
  }
  if (threadIdx.x == 0) {
    const float v = alpha != nullptr ? __fmul_rn(*alpha, partial[0]) : partial[0];
    if constexpr (BF16OUT) {
      static_cast<uint16_t*>(d)[row * n + col] = float_to_bf16_bits(v);
    } else {
      static_cast<float*>(d)[col * m + row] = v;
    }
    *corrected = 1;
  }
}

}  // namespace
}  // namespace sdc

extern "C" {

int sdc_abft_locate(const float* residual, const float* threshold, const uint8_t* flags, int64_t m,
                    int64_t n, int64_t* location, uint8_t* located, sdc_stream_t stream) {
  using namespace sdc;
  SDC_REQUIRE(residual != nullptr && threshold != nullptr && flags != nullptr && location != nullptr &&
                  located != nullptr,
              "locate pointers must not be null");
  SDC_REQUIRE(m > 0 && n > 0, "locate needs m > 0 and n > 0");
  locate_kernel<<<1, kLocThreads, 0, stream>>>(residual, threshold, flags, m, n, location, located);
  SDC_CUDA_CHECK(cudaGetLastError());
  return SDC_OK;
}

int sdc_abft_correct_fp8(const uint8_t* a, const uint8_t* b_rows, int64_t m, int64_t n, int64_t k,
                         const float* alpha, const int64_t* location, const uint8_t* located,
                         float* d_colmajor, uint8_t* corrected, sdc_stream_t stream) {
  using namespace sdc;
  SDC_REQUIRE(a && b_rows && alpha && location && located && d_colmajor && corrected,
              "correct pointers must not be null");
  SDC_REQUIRE(m > 0 && n > 0 && k > 0, "correct needs positive dimensions");
  correct_kernel<Kind::kFp8, false><<<1, kLocThreads, 0, stream>>>(
      a, b_rows, nullptr, nullptr, m, n, k, alpha, location, located, d_colmajor, corrected);
  SDC_CUDA_CHECK(cudaGetLastError());
  return SDC_OK;
}

int sdc_abft_correct_nvfp4(const uint8_t* a_packed, const uint8_t* b_packed, const uint8_t* sfa,
                           const uint8_t* sfb, int64_t m, int64_t n, int64_t k, const float* alpha,
                           const int64_t* location, const uint8_t* located, uint16_t* d_rowmajor,
                           uint8_t* corrected, sdc_stream_t stream) {
  using namespace sdc;
  SDC_REQUIRE(a_packed && b_packed && sfa && sfb && alpha && location && located && d_rowmajor && corrected,
              "correct pointers must not be null");
  SDC_REQUIRE(m > 0 && n > 0 && k > 0 && k % 32 == 0, "correct needs positive dimensions, k % 32 == 0");
  correct_kernel<Kind::kNvf4, true><<<1, kLocThreads, 0, stream>>>(
      a_packed, b_packed, sfa, sfb, m, n, k, alpha, location, located, d_rowmajor, corrected);
  SDC_CUDA_CHECK(cudaGetLastError());
  return SDC_OK;
}

int sdc_abft_correct_fp8_block(const uint8_t* a, const uint8_t* b_rows, const float* scale_a,
                               const float* scale_b, int64_t m, int64_t n, int64_t k, const int64_t* location,
                               const uint8_t* located, uint16_t* d_rowmajor, uint8_t* corrected,
                               sdc_stream_t stream) {
  using namespace sdc;
  SDC_REQUIRE(a && b_rows && scale_a && scale_b && location && located && d_rowmajor && corrected,
              "correct pointers must not be null");
  SDC_REQUIRE(m > 0 && n > 0 && k > 0 && k % 128 == 0, "correct needs positive dimensions, k % 128 == 0");
  correct_kernel<Kind::kFp8Block, true><<<1, kLocThreads, 0, stream>>>(
      a, b_rows, reinterpret_cast<const uint8_t*>(scale_a), reinterpret_cast<const uint8_t*>(scale_b), m, n, k,
      nullptr, location, located, d_rowmajor, corrected);
  SDC_CUDA_CHECK(cudaGetLastError());
  return SDC_OK;
}

}  // extern "C"
