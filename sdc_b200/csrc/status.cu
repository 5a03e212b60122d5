// Host-side status plumbing, device checks and TMA descriptor encoding.
#include <cudaTypedefs.h>

#include <atomic>
#include <cstdio>
#include <mutex>
#include <string>

#include "common.cuh"

namespace sdc {

__device__ int32_t g_watchdog = 0;

int32_t* watchdog_ptr() {
  static thread_local int cached_device = -1;
  static thread_local int32_t* cached = nullptr;
  int device = -1;
  if (cudaGetDevice(&device) != cudaSuccess) return nullptr;
  if (device != cached_device) {
    void* p = nullptr;
    if (cudaGetSymbolAddress(&p, g_watchdog) != cudaSuccess) return nullptr;
    cached = static_cast<int32_t*>(p);
    cached_device = device;
  }
  return cached;
}

namespace {
thread_local std::string t_last_error;
// Test hook state (sdc_test_set_watchdog): 0 = the production limit.
std::atomic<uint64_t> g_test_wait_limit_ns{0};
std::atomic<int32_t> g_test_pace_extra{0};
}  // namespace

WatchdogSettings watchdog_settings() {
  const uint64_t limit = g_test_wait_limit_ns.load(std::memory_order_relaxed);
  return {limit != 0 ? limit : kWaitLimitNs, g_test_pace_extra.load(std::memory_order_relaxed)};
}

void set_error(const std::string& message) { t_last_error = message; }

int fail(int status, const std::string& message) {
  set_error(message);
  return status;
}

int cuda_fail(cudaError_t error, const char* what) {
  set_error(std::string(what) + ": " + cudaGetErrorString(error));
  return SDC_ERR_CUDA;
}

int check_current_device() {
  // Cached per device: cudaGetDeviceProperties costs milliseconds, which
  // would dominate every launch; the attribute query is cheap.
  constexpr int kMaxDevices = 64;
  static std::atomic<int> verified[kMaxDevices] = {};
  int device = 0;
  SDC_CUDA_CHECK(cudaGetDevice(&device));
  if (device >= 0 && device < kMaxDevices && verified[device].load(std::memory_order_relaxed) == 1) {
    return SDC_OK;
  }
  int rc = sdc_device_check(device);
  if (rc == SDC_OK && device >= 0 && device < kMaxDevices) verified[device].store(1, std::memory_order_relaxed);
  return rc;
}

int sm_count() {
  constexpr int kMaxDevices = 64;
  static std::atomic<int> cached[kMaxDevices] = {};
  int device = 0;
  if (cudaGetDevice(&device) != cudaSuccess || device < 0 || device >= kMaxDevices) return 148;
  int count = cached[device].load(std::memory_order_relaxed);
  if (count == 0) {
    if (cudaDeviceGetAttribute(&count, cudaDevAttrMultiProcessorCount, device) != cudaSuccess || count <= 0) {
      return 148;
    }
    cached[device].store(count, std::memory_order_relaxed);
  }
  return count;
}

namespace {
PFN_cuTensorMapEncodeTiled_v12000 g_encode = nullptr;
std::once_flag g_encode_once;
}  // namespace

int encode_tensor_map(CUtensorMap* map, CUtensorMapDataType type, int rank, void* base,
                      const uint64_t* dims, const uint64_t* strides_bytes, const uint32_t* box,
                      CUtensorMapSwizzle swizzle) {
  std::call_once(g_encode_once, [] {
    void* fn = nullptr;
    cudaDriverEntryPointQueryResult q{};
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &fn, cudaEnableDefault, &q) ==
            cudaSuccess &&
        q == cudaDriverEntryPointSuccess) {
      g_encode = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(fn);
    }
  });
  if (g_encode == nullptr) return fail(SDC_ERR_CUDA, "cuTensorMapEncodeTiled entry point unavailable");
  cuuint64_t gdim[5];
  cuuint64_t gstride[4];
  cuuint32_t bdim[5];
  cuuint32_t estride[5];
  for (int i = 0; i < rank; ++i) {
    gdim[i] = dims[i];
    bdim[i] = box[i];
    estride[i] = 1;
    if (i + 1 < rank) gstride[i] = strides_bytes[i];
  }
  CUresult r = g_encode(map, type, static_cast<cuuint32_t>(rank), base, gdim, gstride, bdim,
                        estride, CU_TENSOR_MAP_INTERLEAVE_NONE, swizzle,
                        CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) {
    char msg[160];
    std::snprintf(msg, sizeof(msg), "cuTensorMapEncodeTiled failed (CUresult %d, rank %d)",
                  static_cast<int>(r), rank);
    return fail(SDC_ERR_CUDA, msg);
  }
  return SDC_OK;
}

}  // namespace sdc

extern "C" {

const char* sdc_last_error(void) { return sdc::t_last_error.c_str(); }

int sdc_device_check(int device) {
  int major = 0, minor = 0;
  cudaError_t e = cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, device);
  if (e == cudaSuccess) e = cudaDeviceGetAttribute(&minor, cudaDevAttrComputeCapabilityMinor, device);
  if (e != cudaSuccess) return sdc::cuda_fail(e, "cudaDeviceGetAttribute");
  if (major != 10 || minor != 0) {
    return sdc::fail(SDC_ERR_UNSUPPORTED_DEVICE,
                     "sdc_b200 kernels are built for sm_100a (B200); device is sm_" +
                         std::to_string(major) + std::to_string(minor));
  }
  return SDC_OK;
}

int sdc_test_set_watchdog(uint64_t wait_limit_ns, int32_t pace_extra) {
  if (pace_extra < 0) return sdc::fail(SDC_ERR_INVALID, "pace_extra must be >= 0");
  sdc::g_test_wait_limit_ns.store(wait_limit_ns, std::memory_order_relaxed);
  sdc::g_test_pace_extra.store(pace_extra, std::memory_order_relaxed);
  return SDC_OK;
}

int sdc_read_device_error(sdc_stream_t stream, int32_t* code) {
  if (code == nullptr) return sdc::fail(SDC_ERR_INVALID, "code must not be null");
  int32_t zero = 0;
  SDC_CUDA_CHECK(cudaStreamSynchronize(stream));
  SDC_CUDA_CHECK(cudaMemcpyFromSymbol(code, sdc::g_watchdog, sizeof(int32_t)));
  SDC_CUDA_CHECK(cudaMemcpyToSymbol(sdc::g_watchdog, &zero, sizeof(int32_t)));
  return SDC_OK;
}

}  // extern "C"
