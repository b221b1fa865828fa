// tcgen05 tensor-core GEMM for the prefill projections:
//   out[m, n] = sum_k x[m, k] * w[n, k]   (FP16 in, FP32 accumulate in TMEM,
//                                           one FP16 rounding on store)
// matmul_simd_db_f16 (transformer.metal:174-272) on sm_100a.
//
// One CTA computes a 128 x BN tile with three warp roles:
//   warp 0  TMA producer: 2-D tiled loads (128B swizzle, no multicast) of the
//           x and w K-slices into an S-stage shared-memory ring
//   warp 1  allocates TMEM; one thread issues tcgen05.mma (M=128, N=BN,
//           K=16) and tcgen05.commit frees each stage back to the producer
//   warps 2-5  epilogue: tcgen05.ld of the FP32 accumulator (each warp owns
//           the 32 TMEM lanes of its quadrant), FP16 rounding, global store
// Both operands are K-major, so the canonical K-major SW128 layout produced
// by the TMA box {64, rows} is consumed directly by the MMA descriptors.
// Every mbarrier wait is bounded: on expiry the kernel records an error code
// in mi_tc_status, drains its own copies (bounded) and frees its TMEM.

#include <cuda.h>

#include <algorithm>
#include <mutex>

#include "device.cuh"

namespace mi {
namespace k {

namespace {

__device__ unsigned int mi_tc_status = 0;

constexpr int BM = 128;
constexpr int BK = 64;  // halves per stage = one 128-byte swizzle row
constexpr int kThreads = 192;
constexpr uint64_t kWaitNs = 200ull * 1000 * 1000;  // give up after 200 ms

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count));
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

// Bounded wait; returns false (and records `code`) when the limit expires.
__device__ __forceinline__ uint64_t global_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %globaltimer;" : "=l"(t));
  return t;
}

// Bounded on time (a single try_wait may suspend for a while).
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity, unsigned code) {
  if (mbar_try_wait(bar, parity)) return true;
  const uint64_t start = global_ns();
  while (!mbar_try_wait(bar, parity))
    if (global_ns() - start > kWaitNs) {
      atomicCAS(&mi_tc_status, 0u, code);
      return false;
    }
  return true;
}

__device__ __forceinline__ void tma_load_2d(void* dst, const CUtensorMap* map, uint64_t* bar,
                                            int c0, int c1) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, "
      "{%3, %4}], [%2];" ::"r"(smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(smem_u32(bar)), "r"(c0), "r"(c1)
      : "memory");
}

// Shared-memory matrix descriptor: K-major, 128-byte swizzle, 8-row groups
// 1024 bytes apart (SBO), LBO unused (1), descriptor version 1.
__device__ __forceinline__ uint64_t sw128_desc(uint32_t addr) {
  return (uint64_t)((addr >> 4) & 0x3FFF) | ((uint64_t)1 << 16) | ((uint64_t)(1024 >> 4) << 32) |
         ((uint64_t)1 << 46) | ((uint64_t)2 << 61);
}

// Instruction descriptor of kind::f16: A = B = F16, D = F32, both K-major.
template <int BN>
__host__ __device__ constexpr uint32_t idesc_f16() {
  return (1u << 4) | ((uint32_t)(BN >> 3) << 17) | ((uint32_t)(BM >> 4) << 24);
}

__device__ __forceinline__ void mma_f16(uint32_t tmem_d, uint64_t a, uint64_t b, uint32_t idesc,
                                        uint32_t accumulate) {
  asm volatile(
      "{\n .reg .pred p;\n setp.ne.u32 p, %4, 0;\n"
      " tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n}" ::"r"(tmem_d),
      "l"(a), "l"(b), "r"(idesc), "r"(accumulate)
      : "memory");
}

__device__ __forceinline__ void mma_commit(uint64_t* bar) {
  asm volatile(
      "tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
          smem_u32(bar))
      : "memory");
}

template <int BN>
struct Smem {
  static constexpr int kStages = BN >= 256 ? 4 : 6;
  static constexpr int kABytes = BM * BK * 2;
  static constexpr int kBBytes = BN * BK * 2;
  static constexpr int kStageBytes = kABytes + kBBytes;
  static constexpr int kBytes = 1024 /*align*/ + kStages * kStageBytes + 256;
};

// Epilogue of FP32 outputs (tensor-parallel partials): 32 accumulator
// columns of one row, `left` of them inside the matrix.
__device__ __forceinline__ void store_f32_row(float* dst, const uint32_t (&r)[32], int left) {
  if (left >= 32 && ((reinterpret_cast<uintptr_t>(dst) & 15) == 0)) {
#pragma unroll
    for (int q = 0; q < 8; ++q)
      reinterpret_cast<float4*>(dst)[q] =
          make_float4(__uint_as_float(r[4 * q]), __uint_as_float(r[4 * q + 1]),
                      __uint_as_float(r[4 * q + 2]), __uint_as_float(r[4 * q + 3]));
  } else {
#pragma unroll
    for (int i = 0; i < 32; ++i)
      if (i < left) dst[i] = __uint_as_float(r[i]);
  }
}

template <int BN>
__global__ void __launch_bounds__(kThreads, 1)
    gemm_tc_kernel(const __grid_constant__ CUtensorMap map_x,
                   const __grid_constant__ CUtensorMap map_w, __half* out, int m, int n, int k,
                   int ldo, float* outf) {
  using S = Smem<BN>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~uintptr_t(1023));
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + S::kStages * S::kStageBytes);
  uint64_t* empty = full + S::kStages;
  uint64_t* accum = empty + S::kStages;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(accum + 1);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int n0 = blockIdx.x * BN;
  const int m0 = blockIdx.y * BM;
  const int ktiles = (k + BK - 1) / BK;

  if (threadIdx.x == 0) {
    for (int s = 0; s < S::kStages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    mbar_init(accum, 1);
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&map_x)) : "memory");
    asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&map_w)) : "memory");
  }
  if (warp == 1) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                     smem_u32(tmem_slot)),
                 "r"(BN)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
  __syncthreads();
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
  const uint32_t tmem = *tmem_slot;

  pdl_trigger();
  pdl_wait();

  if (warp == 0 && lane == 0) {
    // TMA producer.
    bool ok = true;
    for (int kt = 0; kt < ktiles; ++kt) {
      int s = kt % S::kStages;
      uint32_t phase = (kt / S::kStages) & 1;
      if (ok) ok = mbar_wait(&empty[s], phase ^ 1, 1);
      uint8_t* a = smem + s * S::kStageBytes;
      uint8_t* b = a + S::kABytes;
      mbar_expect_tx(&full[s], S::kStageBytes);
      tma_load_2d(a, &map_x, &full[s], kt * BK, m0);
      tma_load_2d(b, &map_w, &full[s], kt * BK, n0);
    }
    // Drain: the copies of the last stages must land before the CTA exits.
    int first = ktiles > S::kStages ? ktiles - S::kStages : 0;
    for (int kt = first; kt < ktiles; ++kt)
      mbar_wait(&full[kt % S::kStages], (kt / S::kStages) & 1, 4);
  } else if (warp == 1 && lane == 0) {
    // MMA issuer.
    constexpr uint32_t idesc = idesc_f16<BN>();
    bool ok = true;
    for (int kt = 0; kt < ktiles; ++kt) {
      int s = kt % S::kStages;
      uint32_t phase = (kt / S::kStages) & 1;
      if (ok) ok = mbar_wait(&full[s], phase, 2);
      asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
      uint32_t a_addr = smem_u32(smem + s * S::kStageBytes);
      uint32_t b_addr = a_addr + S::kABytes;
      uint64_t adesc = sw128_desc(a_addr), bdesc = sw128_desc(b_addr);
#pragma unroll
      for (int kk = 0; kk < BK / 16; ++kk)
        mma_f16(tmem, adesc + 2 * kk, bdesc + 2 * kk, idesc, (kt | kk) != 0);
      mma_commit(&empty[s]);
    }
    mma_commit(accum);
  } else if (warp >= 2) {
    // Epilogue: warp w reads TMEM lanes [32 * (w % 4), +32).
    const int quad = warp & 3;
    const int row = m0 + quad * 32 + lane;
    bool ok = mbar_wait(accum, 0, 3);
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
    (void)ok;
#pragma unroll 1
    for (int c = 0; c < BN; c += 32) {
      uint32_t r[32];
      uint32_t taddr = tmem + ((uint32_t)(quad * 32) << 16) + (uint32_t)c;
      asm volatile(
          "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,"
          "%13,%14,%15,%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
          : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
            "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]),
            "=r"(r[13]), "=r"(r[14]), "=r"(r[15]), "=r"(r[16]), "=r"(r[17]), "=r"(r[18]),
            "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]),
            "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]),
            "=r"(r[31])
          : "r"(taddr));
      asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
      if (row < m && outf) {
        store_f32_row(outf + (size_t)row * ldo + n0 + c, r, n - (n0 + c));
      } else if (row < m) {
        int col = n0 + c;
        __half* dst = out + (size_t)row * ldo + col;
        if (col + 32 <= n && ((reinterpret_cast<uintptr_t>(dst) & 15) == 0)) {
#pragma unroll
          for (int q = 0; q < 4; ++q) {
            uint4 v;
            __half2* hv = reinterpret_cast<__half2*>(&v);
#pragma unroll
            for (int i = 0; i < 4; ++i)
              hv[i] = __floats2half2_rn(__uint_as_float(r[q * 8 + 2 * i]),
                                        __uint_as_float(r[q * 8 + 2 * i + 1]));
            reinterpret_cast<uint4*>(dst)[q] = v;
          }
        } else {
#pragma unroll
          for (int i = 0; i < 32; ++i)
            if (col + i < n) dst[i] = __float2half_rn(__uint_as_float(r[i]));
        }
      }
    }
  }
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
  __syncthreads();
  if (warp == 1) {
    __syncwarp();
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(BN)
                 : "memory");
  }
}

// ---- persistent kernel with two TMEM accumulators ---------------------------------
// One CTA per SM walks the output tiles blockIdx.x, blockIdx.x + gridDim.x, ...
// (M fastest, so CTAs running at the same time share the weight tile in L2).
// The producer and the MMA issuer run ahead across tile boundaries; the MMA
// warp alternates between two BN-column TMEM accumulators, so the epilogue
// warps drain tile i while tile i + 1 is being multiplied.
constexpr int kPBN = 256;

struct PSmem {
  static constexpr int kStages = 4;
  static constexpr int kABytes = BM * BK * 2;    // 16 KB
  static constexpr int kBBytes = kPBN * BK * 2;  // 32 KB
  static constexpr int kStageBytes = kABytes + kBBytes;
  static constexpr int kBytes = 1024 /*align*/ + kStages * kStageBytes + 256;
};

__global__ void __launch_bounds__(kThreads, 1)
    gemm_tc_persistent_kernel(const __grid_constant__ CUtensorMap map_x,
                              const __grid_constant__ CUtensorMap map_w, __half* out, int m, int n,
                              int k, int ldo, float* outf) {
  using S = PSmem;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~uintptr_t(1023));
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + S::kStages * S::kStageBytes);
  uint64_t* empty = full + S::kStages;
  uint64_t* acc_full = empty + S::kStages;  // [2] MMA -> epilogue
  uint64_t* acc_empty = acc_full + 2;       // [2] epilogue -> MMA
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(acc_empty + 2);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int tiles_m = (m + BM - 1) / BM;
  const int tiles = tiles_m * ((n + kPBN - 1) / kPBN);
  const int ktiles = (k + BK - 1) / BK;

  if (threadIdx.x == 0) {
    for (int s = 0; s < S::kStages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int a = 0; a < 2; ++a) {
      mbar_init(&acc_full[a], 1);
      mbar_init(&acc_empty[a], 4);  // one arrival per epilogue warp
    }
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&map_x)) : "memory");
    asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&map_w)) : "memory");
  }
  if (warp == 1) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                     smem_u32(tmem_slot)),
                 "r"(2 * kPBN)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
  __syncthreads();
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
  const uint32_t tmem = *tmem_slot;

  pdl_trigger();
  pdl_wait();

  if (warp == 0 && lane == 0) {
    // TMA producer over all of this CTA's tiles.
    bool ok = true;
    uint32_t g = 0;
    for (int tile = blockIdx.x; tile < tiles && ok; tile += gridDim.x) {
      const int m0 = (tile % tiles_m) * BM, n0 = (tile / tiles_m) * kPBN;
      for (int kt = 0; kt < ktiles; ++kt, ++g) {
        const int s = g % S::kStages;
        const uint32_t phase = (g / S::kStages) & 1;
        if (!mbar_wait(&empty[s], phase ^ 1, 1)) {
          ok = false;
          break;
        }
        uint8_t* a = smem + s * S::kStageBytes;
        mbar_expect_tx(&full[s], S::kStageBytes);
        tma_load_2d(a, &map_x, &full[s], kt * BK, m0);
        tma_load_2d(a + S::kABytes, &map_w, &full[s], kt * BK, n0);
      }
    }
    // Drain: the copies into the last stages must land before the CTA exits.
    const uint32_t first = g > (uint32_t)S::kStages ? g - S::kStages : 0u;
    for (uint32_t q = first; q < g; ++q) mbar_wait(&full[q % S::kStages], (q / S::kStages) & 1, 4);
  } else if (warp == 1 && lane == 0) {
    // MMA issuer: accumulator i & 1 for this CTA's i-th tile.
    constexpr uint32_t idesc = idesc_f16<kPBN>();
    bool ok = true;
    uint32_t g = 0;
    int i = 0;
    for (int tile = blockIdx.x; tile < tiles && ok; tile += gridDim.x, ++i) {
      const int a = i & 1;
      if (!mbar_wait(&acc_empty[a], ((i >> 1) & 1) ^ 1, 5)) break;
      asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
      const uint32_t d = tmem + (uint32_t)(a * kPBN);
      for (int kt = 0; kt < ktiles; ++kt, ++g) {
        const int s = g % S::kStages;
        if (!mbar_wait(&full[s], (g / S::kStages) & 1, 2)) {
          ok = false;
          break;
        }
        asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
        const uint32_t a_addr = smem_u32(smem + s * S::kStageBytes);
        const uint64_t adesc = sw128_desc(a_addr), bdesc = sw128_desc(a_addr + S::kABytes);
#pragma unroll
        for (int kk = 0; kk < BK / 16; ++kk)
          mma_f16(d, adesc + 2 * kk, bdesc + 2 * kk, idesc, (kt | kk) != 0);
        mma_commit(&empty[s]);
      }
      mma_commit(&acc_full[a]);
    }
  } else if (warp >= 2) {
    // Epilogue: warp w reads TMEM lanes [32 * (w % 4), +32) of the tile's accumulator.
    const int quad = warp & 3;
    int i = 0;
    for (int tile = blockIdx.x; tile < tiles; tile += gridDim.x, ++i) {
      const int a = i & 1;
      const int m0 = (tile % tiles_m) * BM, n0 = (tile / tiles_m) * kPBN;
      const int row = m0 + quad * 32 + lane;
      if (!mbar_wait(&acc_full[a], (i >> 1) & 1, 3)) break;
      asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
#pragma unroll 1
      for (int c = 0; c < kPBN; c += 32) {
        uint32_t r[32];
        const uint32_t taddr = tmem + ((uint32_t)(quad * 32) << 16) + (uint32_t)(a * kPBN + c);
        asm volatile(
            "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,"
            "%13,%14,%15,%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
            : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
              "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]),
              "=r"(r[13]), "=r"(r[14]), "=r"(r[15]), "=r"(r[16]), "=r"(r[17]), "=r"(r[18]),
              "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]),
              "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]),
              "=r"(r[31])
            : "r"(taddr));
        asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
        if (row < m && outf) {
          store_f32_row(outf + (size_t)row * ldo + n0 + c, r, n - (n0 + c));
        } else if (row < m) {
          const int col = n0 + c;
          __half* dst = out + (size_t)row * ldo + col;
          if (col + 32 <= n && ((reinterpret_cast<uintptr_t>(dst) & 15) == 0)) {
#pragma unroll
            for (int q = 0; q < 4; ++q) {
              uint4 v;
              __half2* hv = reinterpret_cast<__half2*>(&v);
#pragma unroll
              for (int e = 0; e < 4; ++e)
                hv[e] = __floats2half2_rn(__uint_as_float(r[q * 8 + 2 * e]),
                                          __uint_as_float(r[q * 8 + 2 * e + 1]));
              reinterpret_cast<uint4*>(dst)[q] = v;
            }
          } else {
#pragma unroll
            for (int e = 0; e < 32; ++e)
              if (col + e < n) dst[e] = __float2half_rn(__uint_as_float(r[e]));
          }
        }
      }
      // this warp's reads of the accumulator are done: the MMA may reuse it
      asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
      __syncwarp();
      if (lane == 0) asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(
                                      smem_u32(&acc_empty[a]))
                                  : "memory");
    }
  }
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
  __syncthreads();
  if (warp == 1) {
    __syncwarp();
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem),
                 "r"(2 * kPBN)
                 : "memory");
  }
}

// ---- host side ------------------------------------------------------------------
using EncodeTiled = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*,
                                 const cuuint64_t*, const cuuint64_t*, const cuuint32_t*,
                                 const cuuint32_t*, CUtensorMapInterleave, CUtensorMapSwizzle,
                                 CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiled encoder() {
  static EncodeTiled fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    // pinned to the ABI of the signature used here (12.0)
    if (cudaGetDriverEntryPointByVersion("cuTensorMapEncodeTiled", &p, 12000, cudaEnableDefault,
                                         &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeTiled>(p);
  });
  return fn;
}

// [rows, cols] FP16 row-major with a box of {64, box_rows}, 128B swizzle.
bool make_map(CUtensorMap* map, const __half* ptr, int rows, int cols, int box_rows) {
  EncodeTiled enc = encoder();
  if (!enc) return false;
  cuuint64_t dims[2] = {(cuuint64_t)cols, (cuuint64_t)rows};
  cuuint64_t strides[1] = {(cuuint64_t)cols * 2};
  cuuint32_t box[2] = {(cuuint32_t)BK, (cuuint32_t)box_rows};
  cuuint32_t elem[2] = {1, 1};
  return enc(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, const_cast<__half*>(ptr), dims, strides,
             box, elem, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
             CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
             CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

template <int BN>
void launch_tc(const Launch& l, const CUtensorMap& mx, const CUtensorMap& mw, __half* out, int m,
               int n, int k, int ldo, float* outf) {
  auto kernel = gemm_tc_kernel<BN>;
  allow_dynamic_smem(kernel, Smem<BN>::kBytes);
  dim3 grid((n + BN - 1) / BN, (m + BM - 1) / BM);
  launch_kernel(l, grid, dim3(kThreads), Smem<BN>::kBytes, kernel, mx, mw, out, m, n, k, ldo,
                outf);
}

bool enabled() {
  static int on = -1;
  if (on < 0) {
    const char* e = getenv("MI_DISABLE_TCGEN05");
    on = (e && *e == '1') ? 0 : 1;
  }
  return on == 1;
}

// MI_GEMM_PERSISTENT=0 keeps every shape on the one-tile-per-CTA kernel.
bool persistent_enabled() {
  static int on = -1;
  if (on < 0) {
    const char* e = getenv("MI_GEMM_PERSISTENT");
    on = (e && *e == '0') ? 0 : 1;
  }
  return on == 1;
}

}  // namespace

bool gemm_tc_available() { return enabled() && encoder() != nullptr; }

bool make_kv_tile_map(void* map, const __half* cache, int capacity, int kv_heads, int box_rows) {
  EncodeTiled enc = encoder();
  if (!enc) return false;
  cuuint64_t dims[2] = {(cuuint64_t)kv_heads * 128, (cuuint64_t)capacity};
  cuuint64_t strides[1] = {(cuuint64_t)kv_heads * 128 * 2};
  cuuint32_t box[2] = {64, (cuuint32_t)box_rows};
  cuuint32_t elem[2] = {1, 1};
  return enc(static_cast<CUtensorMap*>(map), CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2,
             const_cast<__half*>(cache), dims, strides, box, elem, CU_TENSOR_MAP_INTERLEAVE_NONE,
             CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
             CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

bool gemm_tc(const Launch& l, const __half* x, const __half* w, __half* out, int m, int n, int k,
             int ldo, float* outf) {
  if (!gemm_tc_available()) return false;
  if (m < 2 || k < 8 || (k & 7) || ((reinterpret_cast<uintptr_t>(x) | reinterpret_cast<uintptr_t>(w)) & 15))
    return false;
  int tiles_m = (m + BM - 1) / BM;
  CUtensorMap mx, mw;
  if (persistent_enabled() && tiles_m * ((n + kPBN - 1) / kPBN) >= l.sm_count) {
    // enough 128 x 256 tiles for every SM: the persistent kernel
    if (!make_map(&mx, x, m, k, BM) || !make_map(&mw, w, n, k, kPBN)) return false;
    auto kernel = gemm_tc_persistent_kernel;
    allow_dynamic_smem(kernel, PSmem::kBytes);
    const int tiles = tiles_m * ((n + kPBN - 1) / kPBN);
    launch_kernel(l, dim3(std::min(tiles, l.sm_count)), dim3(kThreads), PSmem::kBytes, kernel, mx,
                  mw, out, m, n, k, ldo, outf);
    return true;
  }
  // Narrow tiles when the grid would not fill the GPU.
  int bn = (tiles_m * ((n + 127) / 128) >= l.sm_count) ? 128 : 64;
  if (!make_map(&mx, x, m, k, BM) || !make_map(&mw, w, n, k, bn)) return false;
  if (bn == 128)
    launch_tc<128>(l, mx, mw, out, m, n, k, ldo, outf);
  else
    launch_tc<64>(l, mx, mw, out, m, n, k, ldo, outf);
  return true;
}

unsigned gemm_tc_status(bool reset) {
  unsigned v = 0;
  cudaMemcpyFromSymbol(&v, mi_tc_status, sizeof v);
  if (reset && v) {
    unsigned z = 0;
    cudaMemcpyToSymbol(mi_tc_status, &z, sizeof z);
  }
  return v;
}

}  // namespace k
}  // namespace mi
