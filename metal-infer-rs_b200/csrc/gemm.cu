// Prefill projections (M > 1): out[m, n] = sum_k x[m, k] * w[n, k] with FP32
// accumulation and one FP16 rounding (matmul_simd_db_f16,
// transformer.metal:174-272).
//
// This file holds the CUDA-core tiled kernel used for ragged shapes; aligned
// shapes go to the tcgen05 tensor-core kernel (gemm_tc.cu) when it is built.

#include "device.cuh"

namespace mi {
namespace k {

namespace {

constexpr int BM = 64, BN = 64, BK = 16;

// 256 threads; each computes a 4x4 block of the 64x64 tile.
__global__ void __launch_bounds__(256) gemm_simt_kernel(const __half* x, const __half* w,
                                                        __half* out, int m, int n, int k,
                                                        int ldo) {
  __shared__ float xs[BK][BM + 4];
  __shared__ float ws[BK][BN + 4];
  pdl_wait();
  const int tid = threadIdx.x;
  const int tx = tid % 16, ty = tid / 16;
  const int m0 = blockIdx.y * BM, n0 = blockIdx.x * BN;
  float acc[4][4] = {};
  for (int k0 = 0; k0 < k; k0 += BK) {
    for (int i = tid; i < BM * BK; i += 256) {
      int r = i / BK, c = i % BK;
      int gm = m0 + r, gk = k0 + c;
      xs[c][r] = (gm < m && gk < k) ? __half2float(x[(size_t)gm * k + gk]) : 0.f;
      int gn = n0 + r;
      ws[c][r] = (gn < n && gk < k) ? __half2float(w[(size_t)gn * k + gk]) : 0.f;
    }
    __syncthreads();
#pragma unroll
    for (int kk = 0; kk < BK; ++kk) {
      float a[4], b[4];
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        a[i] = xs[kk][ty * 4 + i];
        b[i] = ws[kk][tx * 4 + i];
      }
#pragma unroll
      for (int i = 0; i < 4; ++i)
#pragma unroll
        for (int j = 0; j < 4; ++j) acc[i][j] = fmaf(a[i], b[j], acc[i][j]);
    }
    __syncthreads();
  }
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    int gm = m0 + ty * 4 + i;
    if (gm >= m) continue;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      int gn = n0 + tx * 4 + j;
      if (gn < n) out[(size_t)gm * ldo + gn] = __float2half_rn(acc[i][j]);
    }
  }
}

}  // namespace

bool gemm_tc_available();
bool gemm_tc(const Launch& l, const __half* x, const __half* w, __half* out, int m, int n, int k,
             int ldo);

void gemm(const Launch& l, const __half* x, const __half* w, __half* out, int m, int n, int k,
          int ldo) {
  if (m <= 0 || n <= 0) return;
  if (gemm_tc(l, x, w, out, m, n, k, ldo)) return;
  dim3 grid((n + BN - 1) / BN, (m + BM - 1) / BM);
  launch_kernel(l, grid, dim3(256), 0, gemm_simt_kernel, x, w, out, m, n, k, ldo);
}

}  // namespace k
}  // namespace mi
