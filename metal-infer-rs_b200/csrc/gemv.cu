// Decode GEMV family (M = 1): y = x . W^T with FP16 weights streamed by
// 16-byte loads, FP32 accumulation and warp-shuffle reductions, fused with the
// prologues and epilogues of the decode step:
//   kInNorm      matvec3_rms_impl      (transformer.metal:937-1009)
//   kInAddNorm   matvec2_add_rms_impl  (transformer.metal:1091-1160)
//   kOutResidual matmul + add_f16      (transformer.metal:274-347, 61-68)
//   kOutSwiglu   matvec2 + swiglu_f16  (transformer.metal:484-542, 1371-1380)
//   kOutArgmax   matvec_vocab + argmax (transformer.metal:473-482, 1396-1512)
//
// Each warp owns whole rows (no split-K): lane l reads 16-byte chunks
// l, l+32, ... of a row, so a warp-wide load covers 512 contiguous bytes.
// Before waiting on its predecessor (PDL) every warp prefetches its rows into
// L2, so the weight stream overlaps the previous kernel's tail.

#include "device.cuh"

namespace mi {
namespace k {

namespace {

constexpr int kThreads = 256;
constexpr int kWarps = kThreads / 32;

struct RowRef {
  const __half* ptr;
  int seg;
  int row;
};

__device__ __forceinline__ RowRef locate(const GemvProblem& p, int item) {
  int r = item;
  int s = 0;
  if (r >= p.n[0]) {
    r -= p.n[0];
    s = 1;
    if (r >= p.n[1]) {
      r -= p.n[1];
      s = 2;
    }
  }
  return {p.w[s] + (size_t)r * p.k, s, r};
}

// Builds the GEMV input in shared memory (k halves as k/8 uint4 chunks).
template <int IN>
__device__ void build_input(const GemvProblem& p, uint4* xs, float* red) {
  const int tid = threadIdx.x;
  const int kc = p.k >> 3;
  const uint4* src = reinterpret_cast<const uint4*>(p.x);
  if (IN == kInEmbedNorm) {
    uint32_t tok = p.token[p.token_pos ? *p.token_pos : 0u];
    bool zero = tok == 0xFFFFFFFFu || tok >= p.table_rows;
    src = zero ? nullptr : reinterpret_cast<const uint4*>(p.table + (size_t)tok * p.k);
  }
  float ss = 0.f;
  for (int c = tid; c < kc; c += kThreads) {
    uint4 v;
    if (IN == kInAddNorm) {
      uint4 a = src[c];
      uint4 b = reinterpret_cast<const uint4*>(p.x2)[c];
      const __half2* ha = reinterpret_cast<const __half2*>(&a);
      const __half2* hb = reinterpret_cast<const __half2*>(&b);
      __half2* hv = reinterpret_cast<__half2*>(&v);
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        float2 fa = __half22float2(ha[i]);
        float2 fb = __half22float2(hb[i]);
        float s0 = __fadd_rn(fa.x, fb.x), s1 = __fadd_rn(fa.y, fb.y);
        ss = fmaf(s0, s0, ss);
        ss = fmaf(s1, s1, ss);
        hv[i] = __floats2half2_rn(s0, s1);
      }
      if (blockIdx.x == 0 && p.residual_out)
        reinterpret_cast<uint4*>(p.residual_out)[c] = v;
    } else if (IN == kInAddThenNorm) {
      uint4 a = src[c];
      uint4 b = reinterpret_cast<const uint4*>(p.x2)[c];
      const __half2* ha = reinterpret_cast<const __half2*>(&a);
      const __half2* hb = reinterpret_cast<const __half2*>(&b);
      __half2* hv = reinterpret_cast<__half2*>(&v);
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        hv[i] = __hadd2(ha[i], hb[i]);
        float2 f = __half22float2(hv[i]);
        ss = fmaf(f.x, f.x, ss);
        ss = fmaf(f.y, f.y, ss);
      }
      if (blockIdx.x == 0 && p.residual_out)
        reinterpret_cast<uint4*>(p.residual_out)[c] = v;
    } else {
      if (IN == kInEmbedNorm && src == nullptr)
        v = make_uint4(0, 0, 0, 0);
      else
        v = src[c];
      if (IN == kInEmbedNorm && blockIdx.x == 0 && p.embed_out)
        reinterpret_cast<uint4*>(p.embed_out)[c] = v;
      if (IN != kInPlain) {
        const __half2* hv = reinterpret_cast<const __half2*>(&v);
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          float2 f = __half22float2(hv[i]);
          ss = fmaf(f.x, f.x, ss);
          ss = fmaf(f.y, f.y, ss);
        }
      }
    }
    xs[c] = v;
  }
  if (IN == kInPlain) {
    __syncthreads();
    return;
  }
  ss = warp_sum(ss);
  if ((tid & 31) == 0) red[tid >> 5] = ss;
  __syncthreads();
  float total = 0.f;
#pragma unroll
  for (int w = 0; w < kWarps; ++w) total += red[w];
  float scale = rms_scale(total, p.k, p.eps);
  const uint4* g4 = reinterpret_cast<const uint4*>(p.norm_w);
  for (int c = tid; c < kc; c += kThreads) {
    uint4 v = xs[c];
    uint4 g = g4[c];
    const __half2* hv = reinterpret_cast<const __half2*>(&v);
    const __half2* hg = reinterpret_cast<const __half2*>(&g);
    uint4 o;
    __half2* ho = reinterpret_cast<__half2*>(&o);
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      float2 f = __half22float2(hv[i]);
      float2 gg = __half22float2(hg[i]);
      ho[i] = __floats2half2_rn(norm_mul(f.x, scale, gg.x), norm_mul(f.y, scale, gg.y));
    }
    xs[c] = o;
  }
  __syncthreads();
}

__device__ __forceinline__ float silu_mul(float g, float u) {
  // half((g / (1 + exp(-g))) * u) of swiglu_f16, without contraction.
  return __fmul_rn(__fdiv_rn(g, __fadd_rn(1.0f, expf(-g))), u);
}

template <int IN, int OUT>
__global__ void __launch_bounds__(kThreads) gemv_fast_kernel(GemvProblem p) {
  extern __shared__ uint4 xs[];
  __shared__ float red[kWarps];
  __shared__ uint32_t best_key_s[kWarps];
  __shared__ uint32_t best_idx_s[kWarps];
  __shared__ bool is_last;
  const int lane = threadIdx.x & 31;
  const int warp = threadIdx.x >> 5;
  const int warps_total = gridDim.x * kWarps;
  const int gw = blockIdx.x * kWarps + warp;
  const int kc = p.k >> 3;
  const int items = (OUT == kOutSwiglu) ? p.n[0] : p.n[0] + p.n[1] + p.n[2];
  const uint32_t row_bytes = (uint32_t)p.k * 2u;

  // Independent of the predecessor: warm L2 with this warp's first rows.
  {
    int item = gw + lane * warps_total;
    if (item < items) {
      if (OUT == kOutSwiglu) {
        prefetch_l2(p.w[0] + (size_t)item * p.k, row_bytes);
        prefetch_l2(p.w[1] + (size_t)item * p.k, row_bytes);
      } else {
        prefetch_l2(locate(p, item).ptr, row_bytes);
      }
    }
  }
  pdl_trigger();
  pdl_wait();
  build_input<IN>(p, xs, red);

  uint32_t best_key = 0, best_idx = 0xFFFFFFFFu;
  for (int item = gw; item < items; item += 2 * warps_total) {
    const int item_b = item + warps_total;
    const bool has_b = item_b < items;
    const uint4 *r0, *r1, *r2 = nullptr, *r3 = nullptr;
    RowRef ra{}, rb{};
    if (OUT == kOutSwiglu) {
      r0 = reinterpret_cast<const uint4*>(p.w[0] + (size_t)item * p.k);
      r1 = reinterpret_cast<const uint4*>(p.w[1] + (size_t)item * p.k);
      if (has_b) {
        r2 = reinterpret_cast<const uint4*>(p.w[0] + (size_t)item_b * p.k);
        r3 = reinterpret_cast<const uint4*>(p.w[1] + (size_t)item_b * p.k);
      }
    } else {
      ra = locate(p, item);
      r0 = reinterpret_cast<const uint4*>(ra.ptr);
      r1 = nullptr;
      if (has_b) {
        rb = locate(p, item_b);
        r2 = reinterpret_cast<const uint4*>(rb.ptr);
      }
    }
    float a0 = 0.f, a1 = 0.f, a2 = 0.f, a3 = 0.f;
#pragma unroll 4
    for (int c = lane; c < kc; c += 32) {
      uint4 xv = xs[c];
      uint4 w0 = ld_stream(r0 + c);
      uint4 w1, w2, w3;
      if (OUT == kOutSwiglu) w1 = ld_stream(r1 + c);
      if (has_b) {
        w2 = ld_stream(r2 + c);
        if (OUT == kOutSwiglu) w3 = ld_stream(r3 + c);
      }
      a0 = dot8(xv, w0, a0);
      if (OUT == kOutSwiglu) a1 = dot8(xv, w1, a1);
      if (has_b) {
        a2 = dot8(xv, w2, a2);
        if (OUT == kOutSwiglu) a3 = dot8(xv, w3, a3);
      }
    }
    a0 = warp_sum(a0);
    if (OUT == kOutSwiglu) a1 = warp_sum(a1);
    if (has_b) {
      a2 = warp_sum(a2);
      if (OUT == kOutSwiglu) a3 = warp_sum(a3);
    }
    if (lane == 0) {
      if (OUT == kOutSwiglu) {
        float g = __half2float(__float2half_rn(a0));
        float u = __half2float(__float2half_rn(a1));
        p.out[0][item] = __float2half_rn(silu_mul(g, u));
        if (has_b) {
          g = __half2float(__float2half_rn(a2));
          u = __half2float(__float2half_rn(a3));
          p.out[0][item_b] = __float2half_rn(silu_mul(g, u));
        }
      } else if (OUT == kOutResidual) {
        p.out[0][item] = __hadd(p.res[item], __float2half_rn(a0));
        if (has_b) p.out[0][item_b] = __hadd(p.res[item_b], __float2half_rn(a2));
      } else {
        __half h0 = __float2half_rn(a0);
        p.out[ra.seg][ra.row] = h0;
        if (has_b) p.out[rb.seg][rb.row] = __float2half_rn(a2);
        if (OUT == kOutArgmax) {
          float v0 = __half2float(h0);
          if (isfinite(v0) && argmax_better(argmax_key(v0), item, best_key, best_idx)) {
            best_key = argmax_key(v0);
            best_idx = item;
          }
          if (has_b) {
            float v1 = __half2float(__float2half_rn(a2));
            if (isfinite(v1) && argmax_better(argmax_key(v1), item_b, best_key, best_idx)) {
              best_key = argmax_key(v1);
              best_idx = item_b;
            }
          }
        }
      }
    }
  }

  if (OUT == kOutArgmax) {
    if (lane == 0) {
      best_key_s[warp] = best_key;
      best_idx_s[warp] = best_idx;
    }
    __syncthreads();
    if (threadIdx.x == 0) {
      uint32_t bk = 0, bi = 0xFFFFFFFFu;
      for (int w = 0; w < kWarps; ++w)
        if (argmax_better(best_key_s[w], best_idx_s[w], bk, bi)) {
          bk = best_key_s[w];
          bi = best_idx_s[w];
        }
      p.argmax_partial[blockIdx.x] = __uint_as_float(bk);
      p.argmax_index[blockIdx.x] = bi;
      __threadfence();
      uint32_t done = atomicAdd(p.counter, 1u);
      is_last = done == gridDim.x - 1;
    }
    __syncthreads();
    if (is_last) {
      __threadfence();
      uint32_t bk = 0, bi = 0xFFFFFFFFu;
      for (int b = threadIdx.x; b < (int)gridDim.x; b += kThreads) {
        uint32_t ck = __float_as_uint(__ldcg(p.argmax_partial + b));
        uint32_t ci = __ldcg(p.argmax_index + b);
        if (argmax_better(ck, ci, bk, bi)) {
          bk = ck;
          bi = ci;
        }
      }
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) {
        uint32_t ok = __shfl_xor_sync(0xffffffffu, bk, o);
        uint32_t oi = __shfl_xor_sync(0xffffffffu, bi, o);
        if (argmax_better(ok, oi, bk, bi)) {
          bk = ok;
          bi = oi;
        }
      }
      if (lane == 0) {
        best_key_s[warp] = bk;
        best_idx_s[warp] = bi;
      }
      __syncthreads();
      if (threadIdx.x == 0) {
        for (int w = 0; w < kWarps; ++w)
          if (argmax_better(best_key_s[w], best_idx_s[w], bk, bi)) {
            bk = best_key_s[w];
            bi = best_idx_s[w];
          }
        p.token_out[p.token_pos ? *p.token_pos + 1u : 0u] = bi;
        __threadfence();
        if (p.step_counter) *p.step_counter += 1u;
        *p.counter = 0u;
      }
    }
  }
}

// Generic GEMV for any K and alignment (plain input and output only): one
// warp per row, scalar loads.
__global__ void gemv_generic_kernel(const __half* x, const __half* w, __half* out, int n, int k) {
  int warp = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  int lane = threadIdx.x & 31;
  pdl_wait();
  if (warp >= n) return;
  const __half* row = w + (size_t)warp * k;
  float acc = 0.f;
  for (int i = lane; i < k; i += 32) acc = fmaf(__half2float(x[i]), __half2float(row[i]), acc);
  acc = warp_sum(acc);
  if (lane == 0) out[warp] = __float2half_rn(acc);
}

// Reference tiled kernel of matmul_f16 (transformer.metal:70-94): 16x16
// tiles, FP32 accumulate, any shape.
__global__ void matmul_reference_kernel(const __half* x, const __half* w, __half* out, int m,
                                        int n, int k) {
  __shared__ __half xt[16][16];
  __shared__ __half wt[16][16];
  pdl_wait();
  int col = blockIdx.x * 16 + threadIdx.x;
  int row = blockIdx.y * 16 + threadIdx.y;
  float sum = 0.f;
  for (int base = 0; base < k; base += 16) {
    int inner = base + threadIdx.x;
    xt[threadIdx.y][threadIdx.x] = row < m && inner < k ? x[(size_t)row * k + inner] : __half(0.f);
    int wcol = blockIdx.x * 16 + threadIdx.y;
    wt[threadIdx.y][threadIdx.x] =
        wcol < n && inner < k ? w[(size_t)wcol * k + inner] : __half(0.f);
    __syncthreads();
#pragma unroll
    for (int i = 0; i < 16; ++i)
      sum = fmaf(__half2float(xt[threadIdx.y][i]), __half2float(wt[threadIdx.x][i]), sum);
    __syncthreads();
  }
  if (row < m && col < n) out[(size_t)row * n + col] = __float2half_rn(sum);
}

template <int IN, int OUT>
void launch_fast(const Launch& l, const GemvProblem& p) {
  int items = (OUT == kOutSwiglu) ? p.n[0] : p.n[0] + p.n[1] + p.n[2];
  int want = (items + kWarps - 1) / kWarps;
  int cap = l.sm_count * 8;
  if (OUT == kOutArgmax) cap = l.sm_count * 4;  // bounded partial array
  int grid = want < cap ? want : cap;
  if (grid < 1) grid = 1;
  size_t smem = (size_t)p.k * 2;
  auto kernel = gemv_fast_kernel<IN, OUT>;
  if (smem > 48 * 1024) {
    static bool done = false;
    if (!done) {
      cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, 64 * 1024);
      done = true;
    }
  }
  launch_kernel(l, dim3(grid), dim3(kThreads), smem, kernel, p);
}

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15) == 0; }

}  // namespace

bool gemv_fast_ok(const GemvProblem& p) {
  if (p.k <= 0 || (p.k & 7) || p.k > 16384) return false;
  for (int s = 0; s < 3; ++s)
    if (p.n[s] > 0 && !aligned16(p.w[s])) return false;
  const void* ins[] = {p.x, p.x2, p.norm_w, p.table, p.residual_out, p.embed_out};
  for (const void* q : ins)
    if (q && !aligned16(q)) return false;
  return true;
}

int argmax_grid_cap(int sm_count) { return sm_count * 4; }

void gemv(const Launch& l, const GemvProblem& p) {
  if (!gemv_fast_ok(p)) {
    MI_REQUIRE(p.in_mode == kInPlain && p.out_mode == kOutPlain, MI_ERR_SHAPE,
               "fused GEMV needs K %% 8 == 0, K <= 16384 and 16-byte aligned operands");
    for (int s = 0; s < 3; ++s) {
      if (p.n[s] <= 0) continue;
      int grid = (p.n[s] * 32 + 255) / 256;
      launch_kernel(l, dim3(grid), dim3(256), 0, gemv_generic_kernel, p.x, p.w[s], p.out[s],
                    p.n[s], p.k);
    }
    return;
  }
#define MI_GEMV_CASE(IN, OUT)                      \
  if (p.in_mode == IN && p.out_mode == OUT) {      \
    launch_fast<IN, OUT>(l, p);                    \
    return;                                        \
  }
  MI_GEMV_CASE(kInPlain, kOutPlain)
  MI_GEMV_CASE(kInNorm, kOutPlain)
  MI_GEMV_CASE(kInAddNorm, kOutPlain)
  MI_GEMV_CASE(kInEmbedNorm, kOutPlain)
  MI_GEMV_CASE(kInPlain, kOutResidual)
  MI_GEMV_CASE(kInAddNorm, kOutSwiglu)
  MI_GEMV_CASE(kInAddThenNorm, kOutPlain)
  MI_GEMV_CASE(kInAddThenNorm, kOutSwiglu)
  MI_GEMV_CASE(kInPlain, kOutSwiglu)
  MI_GEMV_CASE(kInNorm, kOutArgmax)
  MI_GEMV_CASE(kInPlain, kOutArgmax)
#undef MI_GEMV_CASE
  fail(MI_ERR_SHAPE, "unsupported GEMV fusion (%d, %d)", p.in_mode, p.out_mode);
}

void matmul_reference(const Launch& l, const __half* x, const __half* w, __half* out, int m,
                      int n, int k) {
  dim3 grid((n + 15) / 16, (m + 15) / 16);
  launch_kernel(l, grid, dim3(16, 16), 0, matmul_reference_kernel, x, w, out, m, n, k);
}

}  // namespace k
}  // namespace mi
