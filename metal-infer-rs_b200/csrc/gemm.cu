// Prefill projections (M > 1): out[m, n] = sum_k x[m, k] * w[n, k] with FP32
// accumulation and one FP16 rounding (matmul_simd_db_f16,
// transformer.metal:174-272).
//
//   gemm_canon  CUDA-core kernel with the canonical reduction of numerics.cuh
//               (each output is DOT(x[m], w[n]) exactly as the decode GEMV
//               computes it); used for prompts up to kCanonRows rows, where
//               the weight stream, not the arithmetic, bounds the time
//   gemm_tc     tcgen05 tensor-core kernel (gemm_tc.cu) for longer prompts
//   gemm_simt   tiled fallback for ragged K or unaligned operands

#include "device.cuh"

namespace mi {
namespace k {

namespace {

constexpr int kCanonRows = 512;

// Warp tile: 8 rows of x by 8 rows of w; CTA: 2 x 4 warp tiles (16 x 32).
// Lane l reduces chunks l, l + 32, ... of every pair, then the canonical
// butterfly completes each of the 64 dots.
__global__ void __launch_bounds__(256) gemm_canon_kernel(const __half* x, const __half* w,
                                                         __half* out, int m, int n, int k,
                                                         int ldo, float* outf) {
  pdl_wait();
  const int lane = threadIdx.x & 31;
  const int warp = threadIdx.x >> 5;
  const int m0 = blockIdx.y * 16 + (warp & 1) * 8;
  const int n0 = blockIdx.x * 32 + (warp >> 1) * 8;
  const int kc = k >> 3;
  const int lanes = canon_lanes(k);
  float acc[8][8];
#pragma unroll
  for (int i = 0; i < 8; ++i)
#pragma unroll
    for (int j = 0; j < 8; ++j) acc[i][j] = 0.f;
  const uint4 zero = make_uint4(0, 0, 0, 0);
  for (int c = lane; c < kc; c += 32) {
    uint4 xv[8], wv[8];
#pragma unroll
    for (int i = 0; i < 8; ++i)
      xv[i] = m0 + i < m ? __ldg(reinterpret_cast<const uint4*>(x + (size_t)(m0 + i) * k) + c)
                         : zero;
#pragma unroll
    for (int j = 0; j < 8; ++j)
      wv[j] = n0 + j < n ? __ldg(reinterpret_cast<const uint4*>(w + (size_t)(n0 + j) * k) + c)
                         : zero;
#pragma unroll
    for (int i = 0; i < 8; ++i)
#pragma unroll
      for (int j = 0; j < 8; ++j) acc[i][j] = chunk_dot(xv[i], wv[j], acc[i][j]);
  }
#pragma unroll
  for (int i = 0; i < 8; ++i)
#pragma unroll
    for (int j = 0; j < 8; ++j) acc[i][j] = canon_reduce(acc[i][j], lanes);
  // Lane l writes outputs (l / 8, l % 8) and (l / 8 + 4, l % 8).
#pragma unroll
  for (int half = 0; half < 2; ++half) {
    int i = lane / 8 + 4 * half, j = lane % 8;
    float v = 0.f;
#pragma unroll
    for (int ii = 0; ii < 8; ++ii)
#pragma unroll
      for (int jj = 0; jj < 8; ++jj)
        if (ii == i && jj == j) v = acc[ii][jj];
    if (m0 + i < m && n0 + j < n) {
      if (outf) outf[(size_t)(m0 + i) * ldo + n0 + j] = v;
      else out[(size_t)(m0 + i) * ldo + n0 + j] = __float2half_rn(v);
    }
  }
}

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

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15) == 0; }

}  // namespace

bool gemm_tc(const Launch& l, const __half* x, const __half* w, __half* out, int m, int n, int k,
             int ldo);

void gemm(const Launch& l, const __half* x, const __half* w, __half* out, int m, int n, int k,
          int ldo) {
  if (m <= 0 || n <= 0) return;
  const bool vec = k % 8 == 0 && aligned16(x) && aligned16(w);
  if (vec && m <= kCanonRows) {
    dim3 grid((n + 31) / 32, (m + 15) / 16);
    launch_kernel(l, grid, dim3(256), 0, gemm_canon_kernel, x, w, out, m, n, k, ldo,
                  static_cast<float*>(nullptr));
    return;
  }
  if (gemm_tc(l, x, w, out, m, n, k, ldo)) return;
  dim3 grid((n + BN - 1) / BN, (m + BM - 1) / BM);
  launch_kernel(l, grid, dim3(256), 0, gemm_simt_kernel, x, w, out, m, n, k, ldo);
}

void gemm_partial_f32(const Launch& l, const __half* x, const __half* w, float* out, int m, int n,
                      int k) {
  if (m <= 0 || n <= 0) return;
  MI_REQUIRE(k % 8 == 0 && aligned16(x) && aligned16(w), MI_ERR_SHAPE,
             "tensor-parallel partial products need K %% 8 == 0 and 16-byte aligned operands");
  dim3 grid((n + 31) / 32, (m + 15) / 16);
  launch_kernel(l, grid, dim3(256), 0, gemm_canon_kernel, x, w, static_cast<__half*>(nullptr), m,
                n, k, n, out);
}

}  // namespace k
}  // namespace mi
