// tcgen05 GEMMs for sm_100a with the ABFT epilogue fused.
//
// One CTA computes a 128 x 256 output tile (one reference M-tile of 128 rows,
// so each observed-checksum partial is produced by exactly one CTA):
//   warp 0     TMA producer: 128-byte-swizzled K-major A/B stages (and, for
//              NVFP4, the 512-byte scale-factor atoms) into a 4-stage ring.
//   warp 1     allocates tensor memory; one thread issues tcgen05.mma
//              (kind::f8f6f4 for e4m3, kind::mxf4nvf4.block16 for NVFP4 with
//              scales copied to TMEM by tcgen05.cp) into a 128x256 fp32
//              accumulator and releases stages with tcgen05.commit.
//   warps 2-5  epilogue: tcgen05.ld 32 columns at a time, alpha * acc,
//              optional accumulator bit flip, column checksums
//              sum_rows w_c[row] * v (butterfly transpose-reduce across lanes,
//              fixed-order sum across the four row quarters), non-finite
//              check of the converted output, and the output store.
// Epilogue semantics follow src/cutlass_gemm/csrc/abft/common/
// sm120_epilogue.cuh:52-151 of the reference (inject after alpha, observe
// before the output cast); every wait is bounded (common.cuh).
#include <algorithm>

#include "gemm.cuh"

namespace sdc {
namespace {

constexpr int kBM = 128;
constexpr int kBN = 256;
constexpr int kBKBytes = 128;  // one 128-byte swizzle atom of K per stage
constexpr int kStages = 4;
constexpr int kThreads = 192;  // 6 warps
constexpr uint32_t kTmemCols = 512;
constexpr uint32_t kSfaCol = 256;  // NVFP4: 4 k-steps x 4 columns
constexpr uint32_t kSfbCol = 272;  // NVFP4: 4 k-steps x 8 columns
constexpr int kChunks = kBN / 32;

constexpr int kABytes = kBM * kBKBytes;
constexpr int kBBytes = kBN * kBKBytes;
constexpr int kSfaBytes = 4 * 512;
constexpr int kSfbBytes = 2 * 4 * 512;
constexpr int kRedFloats = kChunks * 4 * 2 * 32;

__host__ __device__ constexpr int stage_bytes(Kind k) {
  return kABytes + kBBytes + (k == Kind::kNvf4 ? kSfaBytes + kSfbBytes : 0);
}
__host__ __device__ constexpr int smem_bytes(Kind k) {
  return 1024 + kStages * stage_bytes(k) + kRedFloats * 4 + 256;
}

struct Params {
  int32_t m, n, num_kb;
  const float* alpha;
  void* d;
  const float* weights;
  int32_t frow, fcol, fbit;
  int32_t* nonfinite;
  float* observed;
  int32_t* hit;
  int32_t padded_n, tiles_m;
  int32_t* watchdog;
};

// Lane j of the warp returns sum over the 32 lanes of x[j] (x is consumed).
__device__ __forceinline__ float transpose_reduce32(float (&x)[32], int lane) {
#pragma unroll
  for (int width = 16; width >= 1; width >>= 1) {
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

// Scale-factor atom (32 rows x 16 bytes, contiguous) as a tcgen05.cp source.
__device__ __forceinline__ uint64_t sf_desc(uint32_t addr) { return smem_desc(addr, 0, 128, 0); }

template <Kind KIND, int C, bool BF16OUT>
__global__ void __launch_bounds__(kThreads, 1)
    gemm_kernel(const __grid_constant__ CUtensorMap tm_a, const __grid_constant__ CUtensorMap tm_b,
                const __grid_constant__ CUtensorMap tm_sfa,
                const __grid_constant__ CUtensorMap tm_sfb, const Params p) {
  constexpr int kStageBytes = stage_bytes(KIND);
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~static_cast<uintptr_t>(1023));
  float* red = reinterpret_cast<float*>(smem + kStages * kStageBytes);
  uint64_t* full = reinterpret_cast<uint64_t*>(red + kRedFloats);
  uint64_t* empty = full + kStages;
  uint64_t* accum = empty + kStages;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(accum + 1);
  volatile int32_t* abort_flag = reinterpret_cast<volatile int32_t*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int nt = blockIdx.x, mt = blockIdx.y;
  const int m0 = mt * kBM, n0 = nt * kBN;

  if (threadIdx.x == 0) {
    for (int s = 0; s < kStages; ++s) {
      mbar_init(full + s, 1);
      mbar_init(empty + s, 1);
    }
    mbar_init(accum, 1);
    *abort_flag = 0;
    fence_barrier_init();
  }
  if (warp == 0 && lane == 0) {
    tma_prefetch(&tm_a);
    tma_prefetch(&tm_b);
    if constexpr (KIND == Kind::kNvf4) {
      tma_prefetch(&tm_sfa);
      tma_prefetch(&tm_sfb);
    }
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, kTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp == 0) {
    // ---------------- TMA producer ----------------
    if (lane == 0) {
      for (int kb = 0; kb < p.num_kb; ++kb) {
        const int s = kb % kStages;
        if (kb >= kStages &&
            !mbar_wait(empty + s, ((kb / kStages) - 1) & 1, kWaitEmpty, abort_flag, p.watchdog)) {
          break;
        }
        uint8_t* sa = smem + s * kStageBytes;
        uint8_t* sb = sa + kABytes;
        mbar_arrive_expect_tx(full + s, kStageBytes);
        tma_load_2d(sa, &tm_a, full + s, kb * kBKBytes, m0);
        tma_load_2d(sb, &tm_b, full + s, kb * kBKBytes, n0);
        if constexpr (KIND == Kind::kNvf4) {
          uint8_t* ssfa = sb + kBBytes;
          uint8_t* ssfb = ssfa + kSfaBytes;
          tma_load_4d(ssfa, &tm_sfa, full + s, 0, 0, kb * 4, mt);
          tma_load_4d(ssfb, &tm_sfb, full + s, 0, 0, kb * 4, nt * 2);
        }
      }
    }
  } else if (warp == 1) {
    // ---------------- MMA issuer ----------------
    if (lane == 0) {
      constexpr uint32_t idesc = KIND == Kind::kFp8 ? idesc_e4m3(kBM, kBN) : idesc_nvf4(kBM, kBN);
      for (int kb = 0; kb < p.num_kb; ++kb) {
        const int s = kb % kStages;
        if (!mbar_wait(full + s, (kb / kStages) & 1, kWaitFull, abort_flag, p.watchdog)) break;
        tc_fence_after();
        const uint32_t sa = smem_u32(smem + s * kStageBytes);
        const uint32_t sb = sa + kABytes;
        if constexpr (KIND == Kind::kNvf4) {
          const uint32_t ssfa = sb + kBBytes;
          const uint32_t ssfb = ssfa + kSfaBytes;
#pragma unroll
          for (int j = 0; j < 4; ++j) {
            tmem_cp_32x128b_x4(tmem + kSfaCol + 4 * j, sf_desc(ssfa + 512 * j));
            tmem_cp_32x128b_x4(tmem + kSfbCol + 8 * j, sf_desc(ssfb + 512 * j));
            tmem_cp_32x128b_x4(tmem + kSfbCol + 8 * j + 4, sf_desc(ssfb + 2048 + 512 * j));
          }
        }
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          const uint64_t adesc = sw128_desc(sa + 32 * j);
          const uint64_t bdesc = sw128_desc(sb + 32 * j);
          const uint32_t acc = (kb > 0 || j > 0) ? 1u : 0u;
          if constexpr (KIND == Kind::kFp8) {
            mma_f8f6f4(tmem, adesc, bdesc, idesc, acc);
          } else {
            mma_nvf4(tmem, adesc, bdesc, idesc, tmem + kSfaCol + 4 * j, tmem + kSfbCol + 8 * j, acc);
          }
        }
        tc_commit(empty + s);
      }
      tc_commit(accum);
    }
  } else {
    // ---------------- epilogue (warps 2..5) ----------------
    const int q = warp & 3;  // TMEM lane quarter this warp may access
    const int row = m0 + q * 32 + lane;
    const bool row_ok = row < p.m;
    float w[C > 0 ? C : 1];
#pragma unroll
    for (int c = 0; c < C; ++c) w[c] = row_ok ? p.weights[static_cast<int64_t>(c) * p.m + row] : 0.f;
    const bool ready = mbar_wait(accum, 0, kWaitAccum, abort_flag, p.watchdog);
    tc_fence_after();
    if (ready && *abort_flag == 0) {
      const float alpha = *p.alpha;
      bool nonfinite = false;
#pragma unroll 1
      for (int chunk = 0; chunk < kChunks; ++chunk) {
        uint32_t r[32];
        tmem_ld_32x32b_x32(tmem + (static_cast<uint32_t>(q * 32) << 16) + chunk * 32, r);
        tmem_ld_wait();
        const int c0 = n0 + chunk * 32;
        float v[32];
#pragma unroll
        for (int j = 0; j < 32; ++j) v[j] = __fmul_rn(alpha, __uint_as_float(r[j]));
        if (C > 0 && p.fbit >= 0 && row == p.frow && p.fcol >= c0 && p.fcol < c0 + 32) {
#pragma unroll
          for (int j = 0; j < 32; ++j) {
            if (c0 + j == p.fcol) v[j] = __uint_as_float(__float_as_uint(v[j]) ^ (1u << p.fbit));
          }
          *p.hit = 1;
        }
        if (C > 0 && p.nonfinite != nullptr && row_ok) {
#pragma unroll
          for (int j = 0; j < 32; ++j) {
            const float out = BF16OUT ? bf16_bits_to_float(float_to_bf16_bits(v[j])) : v[j];
            if (c0 + j < p.n && !isfinite(out)) nonfinite = true;
          }
        }
        if constexpr (C > 0) {
#pragma unroll
          for (int c = 0; c < C; ++c) {
            float x[32];
#pragma unroll
            for (int j = 0; j < 32; ++j) x[j] = w[c] * v[j];
            red[((chunk * 4 + q) * C + c) * 32 + lane] = transpose_reduce32(x, lane);
          }
        }
        if (row_ok) {
          if constexpr (BF16OUT) {
            uint16_t* d = static_cast<uint16_t*>(p.d) + static_cast<int64_t>(row) * p.n;
            if (c0 + 32 <= p.n && (p.n & 7) == 0) {
              uint32_t packed[16];
#pragma unroll
              for (int j = 0; j < 16; ++j) {
                packed[j] = static_cast<uint32_t>(float_to_bf16_bits(v[2 * j])) |
                            (static_cast<uint32_t>(float_to_bf16_bits(v[2 * j + 1])) << 16);
              }
              uint4* dst = reinterpret_cast<uint4*>(d + c0);
#pragma unroll
              for (int j = 0; j < 4; ++j) {
                dst[j] = make_uint4(packed[4 * j], packed[4 * j + 1], packed[4 * j + 2], packed[4 * j + 3]);
              }
            } else {
#pragma unroll
              for (int j = 0; j < 32; ++j) {
                if (c0 + j < p.n) d[c0 + j] = float_to_bf16_bits(v[j]);
              }
            }
          } else {
            float* d = static_cast<float*>(p.d);
#pragma unroll
            for (int j = 0; j < 32; ++j) {
              if (c0 + j < p.n) d[static_cast<int64_t>(c0 + j) * p.m + row] = v[j];
            }
          }
        }
      }
      if (nonfinite) atomicExch(p.nonfinite, 1);
    }
    tc_fence_before();
    if constexpr (C > 0) {
      named_barrier(1, 128);
      if (ready && *abort_flag == 0) {
        const int e = threadIdx.x - 64;
        for (int idx = e; idx < kChunks * C * 32; idx += 128) {
          const int chunk = idx / (C * 32);
          const int rem = idx - chunk * C * 32;
          const int c = rem >> 5;
          const int col = rem & 31;
          float sum = 0.f;
#pragma unroll
          for (int qq = 0; qq < 4; ++qq) sum += red[((chunk * 4 + qq) * C + c) * 32 + col];
          const int gcol = n0 + chunk * 32 + col;
          if (gcol < p.padded_n) {
            p.observed[(static_cast<int64_t>(c) * p.tiles_m + mt) * p.padded_n + gcol] = sum;
          }
        }
      }
    }
  }

  __syncthreads();
  if (warp == 1) {
    __syncwarp();
    tc_fence_after();
    tmem_dealloc(tmem, kTmemCols);
  }
}

template <Kind KIND, int C, bool BF16OUT>
int launch_impl(const GemmProblem& g, cudaStream_t stream) {
  const int64_t k_bytes = KIND == Kind::kFp8 ? g.k : g.k / 2;
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
    const uint32_t box[2] = {kBKBytes, kBN};
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
      const uint32_t box[4] = {16, 32, 4, 2};
      int rc = encode_tensor_map(&tsb, CU_TENSOR_MAP_DATA_TYPE_UINT8, 4, const_cast<uint8_t*>(g.sfb),
                                 dims, strides, box, CU_TENSOR_MAP_SWIZZLE_NONE);
      if (rc != SDC_OK) return rc;
    }
  } else {
    tsa = ta;
    tsb = tb;
  }
  Params p{};
  p.m = static_cast<int32_t>(g.m);
  p.n = static_cast<int32_t>(g.n);
  p.num_kb = static_cast<int32_t>(ceil_div(k_bytes, kBKBytes));
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
  p.tiles_m = static_cast<int32_t>(ceil_div(g.m, kBM));
  p.watchdog = watchdog_ptr();
  if (p.watchdog == nullptr) return fail(SDC_ERR_CUDA, "watchdog symbol unavailable");
  auto kernel = gemm_kernel<KIND, C, BF16OUT>;
  constexpr int smem = smem_bytes(KIND);
  SDC_CUDA_CHECK(cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, smem));
  const dim3 grid(static_cast<unsigned>(ceil_div(g.n, kBN)), static_cast<unsigned>(ceil_div(g.m, kBM)));
  kernel<<<grid, kThreads, smem, stream>>>(ta, tb, tsa, tsb, p);
  SDC_CUDA_CHECK(cudaGetLastError());
  return SDC_OK;
}

}  // namespace

int launch_gemm(const GemmProblem& g, cudaStream_t stream) {
  int rc = check_current_device();
  if (rc != SDC_OK) return rc;
  if (g.channels > 0) {
    SDC_CUDA_CHECK(cudaMemsetAsync(g.hit, 0, sizeof(int32_t), stream));
    if (g.nonfinite != nullptr) SDC_CUDA_CHECK(cudaMemsetAsync(g.nonfinite, 0, sizeof(int32_t), stream));
  }
  const bool bf16 = g.out_bf16_rowmajor;
#define SDC_DISPATCH(KIND, C)                                                   \
  return bf16 ? launch_impl<KIND, C, true>(g, stream) : launch_impl<KIND, C, false>(g, stream)
  if (g.kind == Kind::kFp8) {
    if (g.channels == 0) SDC_DISPATCH(Kind::kFp8, 0);
    if (g.channels == 1) SDC_DISPATCH(Kind::kFp8, 1);
    SDC_DISPATCH(Kind::kFp8, 2);
  }
  if (g.channels == 0) SDC_DISPATCH(Kind::kNvf4, 0);
  if (g.channels == 1) SDC_DISPATCH(Kind::kNvf4, 1);
  SDC_DISPATCH(Kind::kNvf4, 2);
#undef SDC_DISPATCH
}

}  // namespace sdc
