// Device-side helpers shared by the kernels.
#pragma once

#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <cstdint>

#include "kernels.h"
#include "mi_internal.h"
#include "numerics.cuh"

namespace mi {
namespace k {

// ---- programmatic dependent launch ------------------------------------------
// Blocks until the predecessor grid has completed and its writes are visible
// (a no-op when the kernel was launched without the PDL attribute).
__device__ __forceinline__ void pdl_wait() {
  asm volatile("griddepcontrol.wait;" ::: "memory");
}
// Lets the dependent grid start launching (its CTAs then run their
// independent prologue while this grid finishes).
__device__ __forceinline__ void pdl_trigger() {
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}

// Prefetch `bytes` (multiple of 16, 16-byte aligned) into L2.
__device__ __forceinline__ void prefetch_l2(const void* p, uint32_t bytes) {
  asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(p), "r"(bytes) : "memory");
}

// Streaming 16-byte load that does not allocate in L1.
__device__ __forceinline__ uint4 ld_stream(const uint4* p) {
  uint4 r;
  asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0,%1,%2,%3}, [%4];"
               : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w)
               : "l"(p));
  return r;
}

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}

// Greedy argmax key of argmax_better (transformer.metal:1396-1411): values
// compare by the sign-flipped bit pattern, ties go to the larger index.
__device__ __forceinline__ uint32_t argmax_key(float v) {
  uint32_t b = __float_as_uint(v);
  return (b & 0x80000000u) ? ~b : (b ^ 0x80000000u);
}
__device__ __forceinline__ bool argmax_better(uint32_t ck, uint32_t ci, uint32_t bk,
                                              uint32_t bi) {
  if (ci == 0xFFFFFFFFu) return false;
  if (bi == 0xFFFFFFFFu) return true;
  return ck > bk || (ck == bk && ci > bi);
}

// Sampling order key of finite FP16 bits: descending key = descending
// total_cmp value (-0 below +0).
__device__ __forceinline__ uint32_t sample_key16(uint16_t b) {
  return (b & 0x8000u) ? (uint32_t)(~b & 0xffffu) : (uint32_t)(b | 0x8000u);
}

__device__ __forceinline__ uint32_t pos_of(const Pos& p) {
  return p.dev ? (*p.dev + p.base) : p.base;
}

}  // namespace k

// Host launch helper: cudaLaunchKernelEx with the PDL attribute when asked.
template <typename... KArgs, typename... Args>
inline void launch_kernel(const k::Launch& l, dim3 grid, dim3 block, size_t smem,
                          void (*kernel)(KArgs...), Args&&... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = l.stream;
  cudaLaunchAttribute attr[1];
  if (l.pdl) {
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
  }
  cudaError_t err = cudaLaunchKernelEx(&cfg, kernel, std::forward<Args>(args)...);
  if (err != cudaSuccess)
    fail(MI_ERR_COMMAND, "kernel launch failed: %s", cudaGetErrorString(err));
}

}  // namespace mi
