// Thin inline-PTX wrappers for sm_100a: mbarriers, bulk (TMA) copies, fences.
//
// Every wait is bounded: an mbarrier wait gives up after kWaitNs of global
// time (kSpinLimit polls for the flag spins of the multi-GPU solvers),
// records the cause in the device error word (read by
// trnsparse_device_error) and returns false, so a kernel can never hang the
// GPU on a barrier that is never completed.
#pragma once

#include <stdint.h>

namespace tsb {

// Device-side error word: 0 = fine; otherwise the code of the first wait that
// timed out. Defined in capi.cu.
extern __device__ int g_device_error;

enum DeviceError : int {
  DEVERR_NONE = 0,
  DEVERR_MBAR_TIMEOUT = 1,
  DEVERR_TMEM_ALLOC = 2,
  DEVERR_PEER_TIMEOUT = 3,
  DEVERR_SELFCHECK_SMEM = 4,  // a shared-memory tile failed its alignment self-check
};

constexpr uint32_t kSpinLimit = 1u << 26;
constexpr uint64_t kWaitNs = 1000000000ull;  // 1 s: pipeline stages complete in microseconds

__device__ __forceinline__ uint64_t global_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %globaltimer;" : "=l"(t));
  return t;
}

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ void record_device_error(int code) { atomicCAS(&g_device_error, 0, code); }

__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;\n" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}

__device__ __forceinline__ void fence_mbar_init() {
  asm volatile("fence.mbarrier_init.release.cluster;\n" ::: "memory");
}

__device__ __forceinline__ void fence_proxy_async_smem() {
  asm volatile("fence.proxy.async.shared::cta;\n" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;\n" ::"r"(smem_u32(bar)), "r"(bytes) : "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];\n" ::"r"(smem_u32(bar)) : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n"
      ".reg .pred p;\n"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n"
      "selp.u32 %0, 1, 0, p;\n"
      "}\n"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}

// Non-blocking probe: has the phase with the given parity completed?
__device__ __forceinline__ bool mbar_test_wait(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n"
      ".reg .pred p;\n"
      "mbarrier.test_wait.parity.shared::cta.b64 p, [%1], %2;\n"
      "selp.u32 %0, 1, 0, p;\n"
      "}\n"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}

// Cross-GPU flags (the sharded solvers): wait, bounded by kPeerWaitNs of global
// time, until *f >= seq (acquire at system scope). A peer may launch its side
// late, hence the longer limit; on timeout the error word records
// DEVERR_PEER_TIMEOUT and the caller winds the solve down.
constexpr uint64_t kPeerWaitNs = 10000000000ull;  // 10 s

__device__ __forceinline__ long long ld_acquire_sys_s64(const long long* p) {
  long long v;
  asm volatile("ld.acquire.sys.global.s64 %0, [%1];\n" : "=l"(v) : "l"(p) : "memory");
  return v;
}

__device__ __forceinline__ bool wait_flag_geq(const long long* f, long long seq, unsigned sleep_ns) {
  if (ld_acquire_sys_s64(f) >= seq) return true;
  const uint64_t t0 = global_ns();
  for (uint32_t i = 1;; ++i) {
    __nanosleep(sleep_ns);
    if (ld_acquire_sys_s64(f) >= seq) return true;
    if ((i & 15u) == 0 && global_ns() - t0 > kPeerWaitNs) break;
  }
  record_device_error(DEVERR_PEER_TIMEOUT);
  return false;
}

// Bounded wait for the phase with the given parity to complete.
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity) {
  if (mbar_try_wait(bar, parity)) return true;
  const uint64_t t0 = global_ns();
  for (uint32_t i = 1;; ++i) {
    if (mbar_try_wait(bar, parity)) return true;
    if ((i & 63u) == 0 && global_ns() - t0 > kWaitNs) break;
  }
  record_device_error(DEVERR_MBAR_TIMEOUT);
  return false;
}

// 1-D bulk copy global -> shared, completing `bytes` of transaction on `bar`.
// dst, src 16-byte aligned; bytes a multiple of 16.
__device__ __forceinline__ void bulk_g2s(void* dst, const void* src, uint32_t bytes, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];\n" ::"r"(smem_u32(dst)),
      "l"(src), "r"(bytes), "r"(smem_u32(bar))
      : "memory");
}

}  // namespace tsb
