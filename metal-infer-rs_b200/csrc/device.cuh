// Device-side helpers shared by the kernels.
#pragma once

#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <cstdint>
#include <mutex>
#include <set>
#include <tuple>

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

// Bitonic sort (ascending) of n 16-bit keys in shared memory, n a power of
// two, by every thread of the block; ends with a barrier.
__device__ __forceinline__ void block_sort_u16(uint16_t* keys, int n) {
  for (int k = 2; k <= n; k <<= 1)
    for (int j = k >> 1; j > 0; j >>= 1) {
      for (int i = threadIdx.x; i < n; i += blockDim.x) {
        const int ixj = i ^ j;
        if (ixj > i) {
          const uint16_t a = keys[i], b = keys[ixj];
          if ((a > b) == ((i & k) == 0)) {
            keys[i] = b;
            keys[ixj] = a;
          }
        }
      }
      __syncthreads();
    }
}

// Adds the run lengths of the sorted keys[0, n) to hist (0xFFFF marks an
// empty slot: it is the key of no finite value): the last element of each
// run finds the run's first by binary search and adds its length, so there
// is one global atomic per distinct key. The run lengths also go to the
// block's coarse counts `coarse_s` (shared, one per 64 keys).
__device__ __forceinline__ void emit_key_runs(const uint16_t* keys, int n, uint32_t* hist,
                                              uint32_t* coarse_s) {
  for (int i = threadIdx.x; i < n; i += blockDim.x) {
    const uint16_t k = keys[i];
    if (k == 0xFFFFu || (i + 1 < n && keys[i + 1] == k)) continue;
    int lo = 0, hi = i;  // first index with keys[index] == k
    while (lo < hi) {
      const int mid = (lo + hi) >> 1;
      if (keys[mid] < k) lo = mid + 1;
      else hi = mid;
    }
    const uint32_t len = (uint32_t)(i + 1 - lo);
    atomicAdd(hist + k, len);
    atomicAdd(coarse_s + (k >> 6), len);
  }
}

// Sampling histogram of logits[first, last) (this block's rows): the keys of
// the finite values are sorted in `scratch` (>= 2 * seg + 4096 bytes of
// shared memory, seg a power of two) segment by segment and added as runs;
// the per-64-key block counts hist[65536 + b] get one atomic per non-empty
// block.
__device__ __forceinline__ void hist_add_rows(const uint16_t* logits, int first, int last,
                                              uint16_t* scratch, int seg, uint32_t* hist) {
  uint32_t* coarse_s = reinterpret_cast<uint32_t*>(scratch + seg);
  for (int b = threadIdx.x; b < 1024; b += blockDim.x) coarse_s[b] = 0;
  for (int base = first; base < last; base += seg) {
    const int n = min(seg, last - base);
    int np2 = 1;
    while (np2 < n) np2 <<= 1;
    for (int i = threadIdx.x; i < np2; i += blockDim.x) {
      uint16_t key = 0xFFFFu;
      if (i < n) {
        const uint16_t b = logits[base + i];
        if ((b & 0x7c00u) != 0x7c00u) key = (uint16_t)sample_key16(b);
      }
      scratch[i] = key;
    }
    __syncthreads();
    block_sort_u16(scratch, np2);
    emit_key_runs(scratch, np2, hist, coarse_s);
    __syncthreads();
  }
  for (int b = threadIdx.x; b < 1024; b += blockDim.x)
    if (coarse_s[b]) atomicAdd(hist + 65536 + b, coarse_s[b]);
  __syncthreads();
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

// Host: raises `kernel`'s dynamic shared-memory limit to `bytes` on the
// current device, once per (kernel, device, bytes). The attribute belongs to
// the device's context, so a process that launches on several devices
// (tensor-parallel ranks as threads, say) sets it on each of them.
template <typename... KArgs>
inline void allow_dynamic_smem(void (*kernel)(KArgs...), size_t bytes) {
  static std::mutex mu;
  static std::set<std::tuple<const void*, int, size_t>> done;
  int device = 0;
  cudaError_t err = cudaGetDevice(&device);
  if (err != cudaSuccess) fail(MI_ERR_COMMAND, "no current device: %s", cudaGetErrorString(err));
  const auto key = std::make_tuple(reinterpret_cast<const void*>(kernel), device, bytes);
  std::lock_guard<std::mutex> lock(mu);
  if (done.count(key)) return;
  err = cudaFuncSetAttribute(reinterpret_cast<const void*>(kernel),
                             cudaFuncAttributeMaxDynamicSharedMemorySize, (int)bytes);
  if (err != cudaSuccess)
    fail(MI_ERR_COMMAND, "kernel configuration failed: %s", cudaGetErrorString(err));
  done.insert(key);
}

}  // namespace mi
