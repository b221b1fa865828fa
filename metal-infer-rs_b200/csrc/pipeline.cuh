// Asynchronous-copy helpers: mbarriers, bulk (TMA 1-D) copies from global to
// shared memory and 16-byte cp.async, with bounded waits. Every wait gives up
// after kWaitLimit polls, records a code in this translation unit's
// `g_wait_status` (read by the host through the unit's status function) and
// returns false, so a lost completion never hangs the GPU.
#pragma once

#include <cuda_runtime.h>

#include <cstdint>

namespace mi {
namespace k {
namespace pipe {

static __device__ unsigned g_wait_status = 0;

// A wait gives up after kWaitNs nanoseconds of the global timer (one
// try_wait may itself suspend for a while, so the bound is on time, not on
// the number of polls).
constexpr uint64_t kWaitNs = 200ull * 1000 * 1000;

__device__ __forceinline__ uint64_t global_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %globaltimer;" : "=l"(t));
  return t;
}

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count));
}

__device__ __forceinline__ void fence_mbar_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void mbar_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)),
               "r"(bytes)
               : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n .reg .pred p;\n"
      " mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n"
      " selp.u32 %0, 1, 0, p;\n}"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}

__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity, unsigned code) {
  if (mbar_try_wait(bar, parity)) return true;
  const uint64_t start = global_ns();
  while (!mbar_try_wait(bar, parity))
    if (global_ns() - start > kWaitNs) {
      atomicCAS(&g_wait_status, 0u, code);
      return false;
    }
  return true;
}

// 1-D bulk copy global -> shared completing on `bar` (no multicast).
// dst, src 16-byte aligned; bytes a multiple of 16.
__device__ __forceinline__ void bulk_g2s(void* dst, const void* src, uint32_t bytes,
                                         uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
          smem_u32(dst)),
      "l"(src), "r"(bytes), "r"(smem_u32(bar))
      : "memory");
}

__device__ __forceinline__ void cp_async16(void* dst, const void* src) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(smem_u32(dst)), "l"(src)
               : "memory");
}

__device__ __forceinline__ void cp_async_commit() {
  asm volatile("cp.async.commit_group;" ::: "memory");
}

__device__ __forceinline__ void cp_async_wait_all() {
  asm volatile("cp.async.wait_all;" ::: "memory");
}

// Host: this unit's expired-wait code (0 = none), optionally cleared.
static inline unsigned read_status(bool reset) {
  unsigned v = 0;
  cudaMemcpyFromSymbol(&v, g_wait_status, sizeof v);
  if (reset && v) {
    unsigned z = 0;
    cudaMemcpyToSymbol(g_wait_status, &z, sizeof z);
  }
  return v;
}

}  // namespace pipe
}  // namespace k
}  // namespace mi
