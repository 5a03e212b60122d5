// Shared host/device utilities of the sdc_b200 library: status plumbing,
// bounded mbarrier waits, TMA and tcgen05 PTX wrappers for sm_100a.
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include <string>

#include "../../include/sdc_b200.h"

namespace sdc {

// ---------------------------------------------------------------------------
// Host status handling.
// ---------------------------------------------------------------------------
void set_error(const std::string& message);
int fail(int status, const std::string& message);
int cuda_fail(cudaError_t error, const char* what);
// Returns SDC_OK when the current device is sm_100.
int check_current_device();
// Streaming multiprocessors of the current device (cached per device).
int sm_count();
// Encodes a tiled TMA descriptor through the driver entry point (no -lcuda).
int encode_tensor_map(CUtensorMap* map, CUtensorMapDataType type, int rank,
                      void* base, const uint64_t* dims,
                      const uint64_t* strides_bytes, const uint32_t* box,
                      CUtensorMapSwizzle swizzle);

#define SDC_CUDA_CHECK(expr)                                 \
  do {                                                       \
    cudaError_t sdc_err_ = (expr);                           \
    if (sdc_err_ != cudaSuccess) return ::sdc::cuda_fail(sdc_err_, #expr); \
  } while (0)

#define SDC_REQUIRE(cond, msg)                                              \
  do {                                                                      \
    if (!(cond)) return ::sdc::fail(SDC_ERR_INVALID, (msg));                \
  } while (0)

inline int64_t ceil_div(int64_t a, int64_t b) { return (a + b - 1) / b; }

// Compiled checksum policies: algorithm id -> channel count.
inline int policy_channels(int64_t algorithm) {
  if (algorithm == 0) return 2;
  if (algorithm == 1) return 1;
  return 0;
}

// ---------------------------------------------------------------------------
// Device watchdog: every spin wait in this library gives up after a bounded
// time, records a code here and lets the kernel unwind instead of hanging.
// ---------------------------------------------------------------------------
// Device address of this library's watchdog word on the current device.
int32_t* watchdog_ptr();

enum WatchdogCode : int32_t {
  kWaitFull = 1,      // consumer waiting for a TMA stage
  kWaitEmpty = 2,     // producer waiting for a free stage
  kWaitAccum = 3,     // epilogue waiting for the accumulator
  kWaitAccumFree = 4, // MMA waiting for the epilogue to drain TMEM
  kWaitOther = 5,
  kWaitProjection = 6, // K-slice projection waiting for its A rows
  kWaitGrid = 7,       // prediction warps waiting at the grid-wide barrier
  kWaitPace = 8,       // prediction warps waiting for the epilogue's progress
};

// 2 seconds of globaltimer nanoseconds; a healthy wait ends in microseconds.
constexpr uint64_t kWaitLimitNs = 2000000000ull;

// Per-launch watchdog parameters: the wait limit, and a pacing offset that
// only the test hook sdc_test_set_watchdog changes (it makes the prediction
// warps' pacing wait unreachable, so a test can watch a bounded wait expire).
struct WatchdogSettings {
  uint64_t wait_limit_ns;
  int32_t pace_extra;
};
WatchdogSettings watchdog_settings();

__device__ __forceinline__ uint64_t global_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

// ---------------------------------------------------------------------------
// mbarrier
// ---------------------------------------------------------------------------
__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count));
}

__device__ __forceinline__ void fence_barrier_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes)
               : "memory");
}

// The waiting thread may be suspended for up to the hint (1 ms) and is woken
// when the phase completes, so waiters do not poll shared memory.
__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t phase) {
  uint32_t done;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, 1000000;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(done)
      : "r"(smem_u32(bar)), "r"(phase)
      : "memory");
  return done != 0;
}

// Teardown wait for this thread's own asynchronous work (copies or MMAs in
// flight) before the CTA releases its shared or tensor memory: ignores the
// abort flag (an aborted CTA must still let its in-flight work land), gives
// up after kDrainLimitNs. Returns whether the phase completed.
constexpr uint64_t kDrainLimitNs = 100000000ull;
__device__ __forceinline__ bool mbar_drain(uint64_t* bar, uint32_t phase) {
  const uint64_t start = global_ns();
  while (!mbar_try_wait(bar, phase)) {
    if (global_ns() - start > kDrainLimitNs) return false;
  }
  return true;
}

// Waits for `phase` of `bar` with a time limit. Returns false (and records
// `code` in the watchdog word and in `*abort`) when the limit expires or when
// another role of the CTA already aborted.
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t phase, int32_t code,
                                          volatile int32_t* abort, int32_t* watchdog,
                                          uint64_t limit_ns = kWaitLimitNs) {
  if (mbar_try_wait(bar, phase)) return true;
  const uint64_t start = global_ns();
  uint32_t spins = 0;
  while (!mbar_try_wait(bar, phase)) {
    if ((++spins & 15u) == 0u) {
      if (*abort) return false;
      if (global_ns() - start > limit_ns) {
        atomicCAS(watchdog, 0, code);
        *abort = code;
        return false;
      }
    }
  }
  return true;
}

// As mbar_wait, but gives up only when its own limit expires, not when
// another role aborted. The TMA producers use it: the two producers of a CTA
// pair receive the same stage releases (the leader's MMA commits to both), so
// as long as neither leaves early they issue exactly the same stages and the
// leader's teardown drain covers every copy still in flight in either CTA.
__device__ __forceinline__ bool mbar_wait_own_limit(uint64_t* bar, uint32_t phase, int32_t code,
                                                    volatile int32_t* abort, int32_t* watchdog,
                                                    uint64_t limit_ns) {
  if (mbar_try_wait(bar, phase)) return true;
  const uint64_t start = global_ns();
  uint32_t spins = 0;
  while (!mbar_try_wait(bar, phase)) {
    if ((++spins & 15u) == 0u && global_ns() - start > limit_ns) {
      atomicCAS(watchdog, 0, code);
      *abort = code;
      return false;
    }
  }
  return true;
}

// ---------------------------------------------------------------------------
// TMA (bulk tensor copies, no multicast)
// ---------------------------------------------------------------------------
__device__ __forceinline__ void tma_prefetch(const CUtensorMap* map) {
  asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(map)) : "memory");
}

__device__ __forceinline__ void tma_load_2d(void* dst, const CUtensorMap* map, uint64_t* bar,
                                            int32_t c0, int32_t c1) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%3, %4}], [%2];" ::"r"(smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(smem_u32(bar)), "r"(c0), "r"(c1)
      : "memory");
}

// Orders this thread's earlier generic-proxy shared-memory accesses before
// later async-proxy (TMA) writes to the same memory.
__device__ __forceinline__ void fence_proxy_async_smem() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

__device__ __forceinline__ void tma_load_4d(void* dst, const CUtensorMap* map, uint64_t* bar,
                                            int32_t c0, int32_t c1, int32_t c2, int32_t c3) {
  asm volatile(
      "cp.async.bulk.tensor.4d.shared::cluster.global.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%3, %4, %5, %6}], [%2];" ::"r"(smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(smem_u32(bar)), "r"(c0), "r"(c1), "r"(c2),
      "r"(c3)
      : "memory");
}

// ---------------------------------------------------------------------------
// tcgen05 (5th-generation tensor core, accumulators in tensor memory)
// ---------------------------------------------------------------------------
__device__ __forceinline__ void tmem_alloc(uint32_t* dst_smem, uint32_t columns) {
  asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                   smem_u32(dst_smem)),
               "r"(columns)
               : "memory");
}

__device__ __forceinline__ void tmem_relinquish() {
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}

__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t columns) {
  asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(columns)
               : "memory");
}

__device__ __forceinline__ void tc_fence_before() {
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}

__device__ __forceinline__ void tc_fence_after() {
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}

// Arrives once on `bar` when all previously issued tcgen05 ops of this thread
// have completed.
__device__ __forceinline__ void tc_commit(uint64_t* bar) {
  asm volatile(
      "tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
          smem_u32(bar))
      : "memory");
}

// ---- CTA pairs (cta_group::2): one MMA spans the two CTAs of a cluster ----
__device__ __forceinline__ uint32_t cluster_ctarank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}

// Every thread of both CTAs; release/acquire at cluster scope.
__device__ __forceinline__ void cluster_sync() {
  asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}

// Address of the same shared-memory object in CTA `rank` of the cluster.
__device__ __forceinline__ uint32_t mapa_shared(const void* p, uint32_t rank) {
  uint32_t out;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(out) : "r"(smem_u32(p)), "r"(rank));
  return out;
}

// Arrive on an mbarrier given by its cluster shared-memory address.
// Arrive on a barrier of another CTA of the cluster (address from mapa).
// Release at CTA scope: a cluster-scope release cost about a microsecond per
// arrive on B200, which throttled every per-K-block handshake.
__device__ __forceinline__ void mbar_arrive_cluster(uint32_t cluster_addr) {
  asm volatile("mbarrier.arrive.shared::cluster.b64 _, [%0];" ::"r"(cluster_addr) : "memory");
}

__device__ __forceinline__ void tmem_alloc_pair(uint32_t* dst_smem, uint32_t columns) {
  asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(dst_smem)),
               "r"(columns)
               : "memory");
}
__device__ __forceinline__ void tmem_relinquish_pair() {
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_dealloc_pair(uint32_t taddr, uint32_t columns) {
  asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(columns) : "memory");
}

// TMA load into this CTA's shared memory whose completion is counted on the
// pair leader's mbarrier (cluster address). No multicast.
__device__ __forceinline__ void tma_load_2d_pair(void* dst, const CUtensorMap* map, uint32_t leader_bar,
                                                 int32_t c0, int32_t c1) {
  asm volatile(
      "cp.async.bulk.tensor.2d.cta_group::2.shared::cluster.global.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%3, %4}], [%2];" ::"r"(smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(leader_bar), "r"(c0), "r"(c1)
      : "memory");
}

__device__ __forceinline__ void tma_load_4d_pair(void* dst, const CUtensorMap* map, uint32_t leader_bar,
                                                 int32_t c0, int32_t c1, int32_t c2, int32_t c3) {
  asm volatile(
      "cp.async.bulk.tensor.4d.cta_group::2.shared::cluster.global.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%3, %4, %5, %6}], [%2];" ::"r"(smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(leader_bar), "r"(c0), "r"(c1), "r"(c2), "r"(c3)
      : "memory");
}

// Arrives once on `bar` in every CTA of `cta_mask` when the pair MMAs issued
// so far have completed.
__device__ __forceinline__ void tc_commit_pair(uint64_t* bar, uint16_t cta_mask) {
  asm volatile(
      "tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.multicast::cluster.b64 [%0], %1;" ::"r"(
          smem_u32(bar)),
      "h"(cta_mask)
      : "memory");
}

// Pair MMA: D (M = 256 across the two CTAs' TMEM) (+)= A . B^T, A split by
// rows and B by columns between the CTAs' shared memory (same offsets).
__device__ __forceinline__ void mma_f8f6f4_pair(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc,
                                                uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::2.kind::f8f6f4 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
      : "memory");
}

// D[tmem] (+)= A[smem] . B[smem]^T, e4m3 x e4m3 -> fp32.
__device__ __forceinline__ void mma_f8f6f4(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc,
                                           uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f8f6f4 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
      : "memory");
}

// D[tmem] (+)= A[smem] . B[smem]^T, bf16 x bf16 -> fp32 (kind::f16);
// PAIR: one MMA over the CTA pair (M = 256), issued by the leader.
template <bool PAIR = false>
__device__ __forceinline__ void mma_bf16(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc, uint32_t idesc,
                                         uint32_t accumulate) {
  if constexpr (PAIR) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::2.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
        "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
        : "memory");
  } else {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
        "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
        : "memory");
  }
}

// Block-scaled e2m1 x e2m1 with ue4m3 scales per 16 K (NVFP4), fp32
// accumulate; PAIR: one MMA over the CTA pair (M = 256), issued by the leader.
template <bool PAIR = false>
__device__ __forceinline__ void mma_nvf4(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc,
                                         uint32_t idesc, uint32_t sfa_tmem, uint32_t sfb_tmem,
                                         uint32_t accumulate) {
  if constexpr (PAIR) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::2.kind::mxf4nvf4.block_scale.block16 [%0], %1, %2, %3, [%5], [%6], "
        "p;\n\t}" ::"r"(d_tmem),
        "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate), "r"(sfa_tmem), "r"(sfb_tmem)
        : "memory");
  } else {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::mxf4nvf4.block_scale.block16 [%0], %1, %2, %3, [%5], [%6], "
        "p;\n\t}" ::"r"(d_tmem),
        "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate), "r"(sfa_tmem), "r"(sfb_tmem)
        : "memory");
  }
}

// Copies 32 rows x 16 bytes of shared memory into 4 TMEM columns of lanes
// 0-31, replicated into the other three 32-lane sub-partitions. PAIR: issued
// by the leader, each CTA of the pair copies from its own shared memory (same
// offset) into its own TMEM.
template <bool PAIR = false>
__device__ __forceinline__ void tmem_cp_32x128b_x4(uint32_t taddr, uint64_t src_desc) {
  if constexpr (PAIR) {
    asm volatile("tcgen05.cp.cta_group::2.32x128b.warpx4 [%0], %1;" ::"r"(taddr), "l"(src_desc) : "memory");
  } else {
    asm volatile("tcgen05.cp.cta_group::1.32x128b.warpx4 [%0], %1;" ::"r"(taddr), "l"(src_desc) : "memory");
  }
}

// Each thread of the warp loads 32 consecutive fp32 columns of its lane.
__device__ __forceinline__ void tmem_ld_32x32b_x32(uint32_t taddr, uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32"
      " {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15,"
      " %16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31}, [%32];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
        "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]),
        "=r"(r[14]), "=r"(r[15]), "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]),
        "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]), "=r"(r[25]),
        "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
      : "r"(taddr));
}

// Each thread of the warp stores 32 consecutive fp32 columns of its lane.
__device__ __forceinline__ void tmem_st_32x32b_x32(uint32_t taddr, const uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0],"
      " {%1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15, %16,"
      " %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31, %32};"
      ::"r"(taddr), "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]),
        "r"(r[7]), "r"(r[8]), "r"(r[9]), "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]),
        "r"(r[14]), "r"(r[15]), "r"(r[16]), "r"(r[17]), "r"(r[18]), "r"(r[19]), "r"(r[20]),
        "r"(r[21]), "r"(r[22]), "r"(r[23]), "r"(r[24]), "r"(r[25]), "r"(r[26]), "r"(r[27]),
        "r"(r[28]), "r"(r[29]), "r"(r[30]), "r"(r[31])
      : "memory");
}

__device__ __forceinline__ void tmem_st_wait() {
  asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
}

__device__ __forceinline__ void tmem_ld_wait() {
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
}

// Shared-memory matrix descriptor (K-major operand) for tcgen05.
//   bits  0-13 start address >> 4, 16-29 leading byte offset >> 4,
//   bits 32-45 stride byte offset >> 4, 46-47 version (1 on sm_100),
//   bits 61-63 layout (2 = 128-byte swizzle, 0 = no swizzle).
__device__ __forceinline__ uint64_t smem_desc(uint32_t addr, uint32_t lbo, uint32_t sbo,
                                              uint32_t layout) {
  uint64_t d = 0;
  d |= static_cast<uint64_t>((addr >> 4) & 0x3FFFu);
  d |= static_cast<uint64_t>((lbo >> 4) & 0x3FFFu) << 16;
  d |= static_cast<uint64_t>((sbo >> 4) & 0x3FFFu) << 32;
  d |= static_cast<uint64_t>(1u) << 46;
  d |= static_cast<uint64_t>(layout & 7u) << 61;
  return d;
}

// K-major tile of rows x 128 bytes written by TMA with 128-byte swizzle:
// 8-row groups of 1024 bytes; advancing K inside the swizzle atom moves the
// start address (the swizzle is a function of absolute address bits).
__device__ __forceinline__ uint64_t sw128_desc(uint32_t addr) { return smem_desc(addr, 16, 1024, 2); }

// Instruction descriptor of kind::f8f6f4 e4m3 x e4m3 -> fp32, K-major A and B.
__host__ __device__ constexpr uint32_t idesc_e4m3(int m, int n) {
  return (1u << 4) /*D fp32*/ | (0u << 7) /*A e4m3*/ | (0u << 10) /*B e4m3*/ |
         (static_cast<uint32_t>(n >> 3) << 17) | (static_cast<uint32_t>(m >> 4) << 24);
}

// Instruction descriptor of kind::f16 bf16 x bf16 -> fp32, K-major A and B.
__host__ __device__ constexpr uint32_t idesc_bf16(int m, int n) {
  return (1u << 4) /*D fp32*/ | (1u << 7) /*A bf16*/ | (1u << 10) /*B bf16*/ |
         (static_cast<uint32_t>(n >> 3) << 17) | (static_cast<uint32_t>(m >> 4) << 24);
}

// Instruction descriptor of kind::mxf4nvf4 e2m1 x e2m1 with ue4m3 scales.
__host__ __device__ constexpr uint32_t idesc_nvf4(int m, int n) {
  return (1u << 7) /*A e2m1*/ | (1u << 10) /*B e2m1*/ | (static_cast<uint32_t>(n >> 3) << 17) |
         (0u << 23) /*scale ue4m3*/ | (static_cast<uint32_t>(m >> 4) << 24);
}

// Programmatic dependent launch. griddep_wait: until the grid this one was
// launched after (as a programmatic dependent) has completed and its writes
// are visible; returns at once for a grid launched normally.
// griddep_launch_dependents: this block allows the next grid on the stream
// (if launched as a dependent) to start launching.
__device__ __forceinline__ void griddep_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void griddep_launch_dependents() { asm volatile("griddepcontrol.launch_dependents;"); }

// Named barrier among `count` threads (ids 1..15; 0 is __syncthreads).
__device__ __forceinline__ void named_barrier(uint32_t id, uint32_t count) {
  asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(count) : "memory");
}

// Per-warpgroup register reallocation: every warp of the warpgroup executes
// the same instruction, in warp-uniform control flow. The increases of a CTA
// must fit in what it was launched with (threads x registers at launch) minus
// what the decreases free, or the increasing warps wait forever.
template <uint32_t N>
__device__ __forceinline__ void setmaxnreg_inc() {
  asm volatile("setmaxnreg.inc.sync.aligned.u32 %0;\n" ::"n"(N));
}
template <uint32_t N>
__device__ __forceinline__ void setmaxnreg_dec() {
  asm volatile("setmaxnreg.dec.sync.aligned.u32 %0;\n" ::"n"(N));
}

// Named barrier that also ORs a predicate across the participating threads,
// so every thread leaves with the same decision (e.g. "some wait failed").
__device__ __forceinline__ bool named_barrier_or(uint32_t id, uint32_t count, bool pred) {
  uint32_t out;
  asm volatile(
      "{\n\t.reg .pred p, q;\n\t"
      "setp.ne.u32 p, %1, 0;\n\t"
      "bar.red.or.pred q, %2, %3, p;\n\t"
      "selp.u32 %0, 1, 0, q;\n\t}"
      : "=r"(out)
      : "r"(static_cast<uint32_t>(pred)), "r"(id), "r"(count)
      : "memory");
  return out != 0;
}

__device__ __forceinline__ bool elect_one() {
  uint32_t pred = 0;
  asm volatile(
      "{\n\t.reg .b32 r;\n\t.reg .pred p;\n\t"
      "elect.sync r|p, 0xffffffff;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(pred));
  return pred != 0;
}

// ---------------------------------------------------------------------------
// Narrow float formats: decode of e4m3 / e2m1 bytes (exact) and RN-satfinite
// encodes through the hardware conversion instructions.
// ---------------------------------------------------------------------------
__device__ __forceinline__ float decode_e4m3(uint32_t byte) {
  const uint32_t sign = (byte & 0x80u) << 24;
  const uint32_t exp = (byte >> 3) & 0xFu;
  const uint32_t man = byte & 0x7u;
  if (exp == 0xFu && man == 0x7u) return __uint_as_float(0x7FC00000u | sign);  // NaN
  float mag;
  if (exp == 0) {
    mag = static_cast<float>(man) * 0.001953125f;  // man * 2^-9 (subnormal)
  } else {
    mag = __uint_as_float(((exp + 120u) << 23) | (man << 20));  // 2^(exp-7) * 1.man
  }
  return __uint_as_float(__float_as_uint(mag) | sign);
}

__device__ __forceinline__ float decode_e2m1(uint32_t nibble) {
  // {0, .5, 1, 1.5, 2, 3, 4, 6} with sign bit 3.
  const uint32_t mag = nibble & 7u;
  float v;
  if (mag < 2u) {
    v = 0.5f * static_cast<float>(mag);
  } else {
    const uint32_t e = mag >> 1;  // 1..3
    v = __uint_as_float(((e + 126u) << 23) | ((mag & 1u) << 22));
  }
  return (nibble & 8u) ? -v : v;
}

// Two fp32 -> two e4m3 (RN, satfinite); `lo` ends in the low byte.
__device__ __forceinline__ uint16_t cvt_e4m3x2(float lo, float hi) {
  uint16_t out;
  asm("cvt.rn.satfinite.e4m3x2.f32 %0, %1, %2;" : "=h"(out) : "f"(hi), "f"(lo));
  return out;
}

// Eight fp32 -> eight e2m1 (RN, satfinite) packed in 4 bytes; v[2i] lands in
// the low nibble of byte i (the operand order of cvt puts `a` in the high half).
__device__ __forceinline__ uint32_t cvt_e2m1x8(const float (&v)[8]) {
  uint32_t out;
  asm("{\n\t.reg .b8 b0, b1, b2, b3;\n\t"
      "cvt.rn.satfinite.e2m1x2.f32 b0, %2, %1;\n\t"
      "cvt.rn.satfinite.e2m1x2.f32 b1, %4, %3;\n\t"
      "cvt.rn.satfinite.e2m1x2.f32 b2, %6, %5;\n\t"
      "cvt.rn.satfinite.e2m1x2.f32 b3, %8, %7;\n\t"
      "mov.b32 %0, {b0, b1, b2, b3};\n\t}"
      : "=r"(out)
      : "f"(v[0]), "f"(v[1]), "f"(v[2]), "f"(v[3]), "f"(v[4]), "f"(v[5]), "f"(v[6]), "f"(v[7]));
  return out;
}

// Exact widening decodes through the hardware conversions (e4m3 and e2m1
// values are all representable in fp16): element 0 in .x.
__device__ __forceinline__ float2 e4m3x2_to_float2(uint32_t two_bytes) {
  uint32_t h2;
  asm("cvt.rn.f16x2.e4m3x2 %0, %1;" : "=r"(h2) : "h"(static_cast<uint16_t>(two_bytes)));
  float2 out;
  asm("{\n\t.reg .f16 lo, hi;\n\tmov.b32 {lo, hi}, %2;\n\t"
      "cvt.f32.f16 %0, lo;\n\tcvt.f32.f16 %1, hi;\n\t}"
      : "=f"(out.x), "=f"(out.y)
      : "r"(h2));
  return out;
}

// Eight e2m1 codes of a 32-bit word (low nibble first) to fp32.
__device__ __forceinline__ void e2m1x8_to_float(uint32_t word, float (&v)[8]) {
  uint32_t h[4];
  asm("{\n\t.reg .b8 b0, b1, b2, b3;\n\t"
      "mov.b32 {b0, b1, b2, b3}, %4;\n\t"
      "cvt.rn.f16x2.e2m1x2 %0, b0;\n\t"
      "cvt.rn.f16x2.e2m1x2 %1, b1;\n\t"
      "cvt.rn.f16x2.e2m1x2 %2, b2;\n\t"
      "cvt.rn.f16x2.e2m1x2 %3, b3;\n\t}"
      : "=r"(h[0]), "=r"(h[1]), "=r"(h[2]), "=r"(h[3])
      : "r"(word));
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    asm("{\n\t.reg .f16 lo, hi;\n\tmov.b32 {lo, hi}, %2;\n\t"
        "cvt.f32.f16 %0, lo;\n\tcvt.f32.f16 %1, hi;\n\t}"
        : "=f"(v[2 * i]), "=f"(v[2 * i + 1])
        : "r"(h[i]));
  }
}

// Two independent IEEE fp32 fused multiply-adds in one sm_100 instruction
// (bit-identical to two fmaf calls): returns {fma(a.x,b.x,c.x), fma(a.y,b.y,c.y)}.
__device__ __forceinline__ float2 fma2(float2 a, float2 b, float2 c) {
  float2 d;
  asm("{\n\t.reg .b64 ra, rb, rc, rd;\n\t"
      "mov.b64 ra, {%2, %3};\n\tmov.b64 rb, {%4, %5};\n\tmov.b64 rc, {%6, %7};\n\t"
      "fma.rn.f32x2 rd, ra, rb, rc;\n\t"
      "mov.b64 {%0, %1}, rd;\n\t}"
      : "=f"(d.x), "=f"(d.y)
      : "f"(a.x), "f"(a.y), "f"(b.x), "f"(b.y), "f"(c.x), "f"(c.y));
  return d;
}

__device__ __forceinline__ float bf16_bits_to_float(uint16_t b) {
  return __uint_as_float(static_cast<uint32_t>(b) << 16);
}

// fp32 -> bf16 bits, round to nearest even (NaN stays NaN).
__device__ __forceinline__ uint16_t float_to_bf16_bits(float f) {
  uint16_t out;
  asm("cvt.rn.bf16.f32 %0, %1;" : "=h"(out) : "f"(f));
  return out;
}

// Two floats to bf16 (round to nearest even) in one instruction: lo in bits
// 0-15, hi in bits 16-31.
__device__ __forceinline__ uint32_t bf16x2_bits(float lo, float hi) {
  uint32_t out;
  asm("cvt.rn.bf16x2.f32 %0, %1, %2;" : "=r"(out) : "f"(hi), "f"(lo));
  return out;
}

}  // namespace sdc
