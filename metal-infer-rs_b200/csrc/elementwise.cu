// Row and elementwise kernels: residual add, RMSNorm, fused add+RMSNorm,
// SwiGLU, embedding gather, RoPE, fused per-head QK-norm + RoPE + K-cache
// append, V-cache append and the standalone greedy argmax. Row reductions use
// the canonical order of numerics.cuh (one warp per row).

#include "device.cuh"

namespace mi {
namespace k {

namespace {

// Canonical sum of squares of `width` FP16 values (one warp).
__device__ __forceinline__ float row_sumsq(const __half* row, int width) {
  const int lane = threadIdx.x & 31;
  const int lanes = canon_lanes(width);
  const int chunks = (width + 7) / 8;
  float acc = 0.f;
  if (lane < lanes) {
    const bool vec = (width % 8 == 0) && ((reinterpret_cast<uintptr_t>(row) & 15) == 0);
    for (int c = lane; c < chunks; c += lanes) {
      if (vec) {
        acc = chunk_sq(reinterpret_cast<const uint4*>(row)[c], acc);
      } else {
        for (int i = 8 * c; i < min(width, 8 * c + 8); ++i) {
          float v = __half2float(row[i]);
          acc = __fmaf_rn(v, v, acc);
        }
      }
    }
  }
  return canon_reduce(acc, lanes);
}

// add_f16 (transformer.metal:61-68): a correctly rounded half addition.
__global__ void add_kernel(const __half* a, const __half* b, __half* out, size_t n) {
  pdl_wait();
  for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < n;
       i += (size_t)gridDim.x * blockDim.x)
    out[i] = __hadd(a[i], b[i]);
}

// rms_norm_f16 (transformer.metal:1318-1340): one warp per row.
__global__ void rms_norm_kernel(const __half* x, const __half* w, __half* out, int rows,
                                int width, float eps) {
  int row = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  int lane = threadIdx.x & 31;
  pdl_wait();
  if (row >= rows) return;
  const __half* xr = x + (size_t)row * width;
  float scale = rms_scale(row_sumsq(xr, width), width, eps);
  for (int i = lane; i < width; i += 32)
    out[(size_t)row * width + i] =
        __float2half_rn(norm_mul(__half2float(xr[i]), scale, __half2float(w[i])));
}

// add_rms_norm_f16 (transformer.metal:1342-1369): residual = half(l + r);
// squares of the unrounded sums; normalized from the rounded residual.
__global__ void add_rms_norm_kernel(const __half* l, const __half* r, const __half* w,
                                    __half* residual, __half* normalized, int rows, int width,
                                    float eps) {
  int row = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  int lane = threadIdx.x & 31;
  pdl_wait();
  if (row >= rows) return;
  size_t base = (size_t)row * width;
  const int lanes = canon_lanes(width);
  const int chunks = (width + 7) / 8;
  float acc = 0.f;
  if (lane < lanes)
    for (int c = lane; c < chunks; c += lanes)
      for (int i = 8 * c; i < min(width, 8 * c + 8); ++i) {
        float v = __fadd_rn(__half2float(l[base + i]), __half2float(r[base + i]));
        residual[base + i] = __float2half_rn(v);
        acc = __fmaf_rn(v, v, acc);
      }
  float scale = rms_scale(canon_reduce(acc, lanes), width, eps);
  __syncwarp();
  for (int i = lane; i < width; i += 32) {
    float v = __half2float(__float2half_rn(
        __fadd_rn(__half2float(l[base + i]), __half2float(r[base + i]))));
    normalized[base + i] = __float2half_rn(norm_mul(v, scale, __half2float(w[i])));
  }
}

// swiglu_f16 (transformer.metal:1371-1380)
__global__ void swiglu_kernel(const __half* gate, const __half* up, __half* out, size_t n) {
  pdl_wait();
  for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < n;
       i += (size_t)gridDim.x * blockDim.x)
    out[i] = __float2half_rn(silu_mul(__half2float(gate[i]), __half2float(up[i])));
}

// embedding_f16 (transformer.metal:1382-1394); out-of-range ids (including
// the 0xFFFFFFFF "no token" marker) embed as zeros.
__global__ void embedding_kernel(const uint32_t* tokens, const __half* table, __half* out,
                                 int count, int width, uint32_t rows) {
  int t = blockIdx.y;
  pdl_wait();
  if (t >= count) return;
  uint32_t tok = tokens[t];
  bool zero = tok == 0xFFFFFFFFu || tok >= rows;
  for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < width; i += gridDim.x * blockDim.x)
    out[(size_t)t * width + i] = zero ? __half(0.f) : table[(size_t)tok * width + i];
}

// Rotate-half RoPE of one pair with the engine's RoPE terms (from the table
// when one is given).
__device__ __forceinline__ void rope_pair(float x, float y, int pair, int head_dim, uint32_t pos,
                                          float theta, __half* ox, __half* oy,
                                          const float2* table = nullptr) {
  float c, s;
  if (table) {
    float2 cs = table[(size_t)pos * (head_dim / 2) + pair];
    c = cs.x;
    s = cs.y;
  } else {
    rope_cs(pos, pair, head_dim, theta, &c, &s);
  }
  *ox = __float2half_rn(__fsub_rn(__fmul_rn(x, c), __fmul_rn(y, s)));
  *oy = __float2half_rn(__fadd_rn(__fmul_rn(x, s), __fmul_rn(y, c)));
}

// rope_f16 (transformer.metal:1514-1531): one warp per (token, head).
__global__ void rope_kernel(const __half* in, __half* out, int tokens, int heads, int head_dim,
                            Pos pos, float theta) {
  int row = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  int lane = threadIdx.x & 31;
  pdl_wait();
  if (row >= tokens * heads) return;
  int token = row / heads;
  uint32_t p = pos_of(pos) + token;
  size_t base = (size_t)row * head_dim;
  int half_dim = head_dim / 2;
  for (int pair = lane; pair < half_dim; pair += 32)
    rope_pair(__half2float(in[base + pair]), __half2float(in[base + pair + half_dim]), pair,
              head_dim, p, theta, out + base + pair, out + base + pair + half_dim);
}

// qk_norm_rope_cache_f16 (transformer.metal:1533-1577): one warp per
// (token, head) row of Q then K. Per-head RMSNorm and RoPE in FP32 rounded
// once (round_norm adds the FP16 rounding of the unfused rms_norm -> rope
// path); rotated keys go to key_cache[pos + token].
__global__ void qk_norm_rope_cache_kernel(const __half* q, const __half* k, const __half* qw,
                                          const __half* kw, __half* q_out, __half* key_cache,
                                          int tokens, int q_heads, int kv_heads, int head_dim,
                                          Pos pos, float theta, float eps, int round_norm,
                                          const float2* table) {
  int group = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  int lane = threadIdx.x & 31;
  pdl_wait();
  int q_rows = tokens * q_heads;
  bool is_q = group < q_rows;
  int row = is_q ? group : group - q_rows;
  int heads = is_q ? q_heads : kv_heads;
  if (row >= tokens * heads) return;
  int token = row / heads;
  int head = row - token * heads;
  const __half* in = (is_q ? q : k) + (size_t)row * head_dim;
  const __half* w = is_q ? qw : kw;
  float scale = rms_scale(row_sumsq(in, head_dim), head_dim, eps);
  uint32_t p = pos_of(pos) + token;
  __half* dst = is_q ? q_out + (size_t)row * head_dim
                     : key_cache + ((size_t)p * kv_heads + head) * head_dim;
  int half_dim = head_dim / 2;
  for (int pair = lane; pair < half_dim; pair += 32) {
    float x = norm_mul(__half2float(in[pair]), scale, __half2float(w[pair]));
    float y = norm_mul(__half2float(in[pair + half_dim]), scale, __half2float(w[pair + half_dim]));
    if (round_norm) {
      x = __half2float(__float2half_rn(x));
      y = __half2float(__float2half_rn(y));
    }
    rope_pair(x, y, pair, head_dim, p, theta, dst + pair, dst + pair + half_dim, table);
  }
}

__global__ void rope_table_kernel(float2* out, int positions, int head_dim, float theta) {
  const int pairs = head_dim / 2;
  const size_t n = (size_t)positions * pairs;
  for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < n;
       i += (size_t)gridDim.x * blockDim.x) {
    float c, s;
    rope_cs((uint32_t)(i / pairs), (int)(i % pairs), head_dim, theta, &c, &s);
    out[i] = make_float2(c, s);
  }
}

// copy_kv_f16 (transformer.metal:2318-2325)
__global__ void copy_kv_kernel(const __half* src, __half* cache, int tokens, int stride,
                               Pos pos) {
  pdl_wait();
  size_t n = (size_t)tokens * stride;
  size_t base = (size_t)pos_of(pos) * stride;
  for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < n;
       i += (size_t)gridDim.x * blockDim.x)
    cache[base + i] = src[i];
}

// argmax_f16_partial / _reduce (transformer.metal:1396-1512): partials over
// 2048-element blocks, then one block reduces them.
__global__ void argmax_partial_kernel(const __half* logits, size_t n, float* pv, uint32_t* pi) {
  __shared__ uint32_t sk[8], si[8];
  uint32_t bk = 0, bi = 0xFFFFFFFFu;
  pdl_wait();
  for (int j = 0; j < 8; ++j) {
    size_t idx = (size_t)blockIdx.x * 2048 + threadIdx.x + j * 256;
    if (idx < n) {
      float v = __half2float(logits[idx]);
      if (isfinite(v) && argmax_better(argmax_key(v), (uint32_t)idx, bk, bi)) {
        bk = argmax_key(v);
        bi = (uint32_t)idx;
      }
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
  if ((threadIdx.x & 31) == 0) {
    sk[threadIdx.x >> 5] = bk;
    si[threadIdx.x >> 5] = bi;
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    for (int w = 0; w < 8; ++w)
      if (argmax_better(sk[w], si[w], bk, bi)) {
        bk = sk[w];
        bi = si[w];
      }
    pv[blockIdx.x] = __uint_as_float(bk);
    pi[blockIdx.x] = bi;
  }
}

__global__ void argmax_reduce_kernel(const float* pv, const uint32_t* pi, int groups,
                                     uint32_t* out) {
  __shared__ uint32_t sk[8], si[8];
  uint32_t bk = 0, bi = 0xFFFFFFFFu;
  pdl_wait();
  for (int g = threadIdx.x; g < groups; g += 256) {
    uint32_t ck = __float_as_uint(pv[g]);
    if (argmax_better(ck, pi[g], bk, bi)) {
      bk = ck;
      bi = pi[g];
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
  if ((threadIdx.x & 31) == 0) {
    sk[threadIdx.x >> 5] = bk;
    si[threadIdx.x >> 5] = bi;
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    for (int w = 0; w < 8; ++w)
      if (argmax_better(sk[w], si[w], bk, bi)) {
        bk = sk[w];
        bi = si[w];
      }
    *out = bi;
  }
}

int grid_for(size_t n, int threads, int sm_count) {
  size_t g = (n + threads - 1) / threads;
  size_t cap = (size_t)sm_count * 16;
  if (g > cap) g = cap;
  return g < 1 ? 1 : (int)g;
}

}  // namespace

void add(const Launch& l, const __half* a, const __half* b, __half* out, size_t n) {
  if (!n) return;
  launch_kernel(l, dim3(grid_for(n, 256, l.sm_count)), dim3(256), 0, add_kernel, a, b, out, n);
}

void rms_norm(const Launch& l, const __half* x, const __half* w, __half* out, int rows,
              int width, float eps) {
  if (rows <= 0) return;
  launch_kernel(l, dim3((rows + 7) / 8), dim3(256), 0, rms_norm_kernel, x, w, out, rows, width,
                eps);
}

void add_rms_norm(const Launch& l, const __half* left, const __half* right, const __half* w,
                  __half* residual, __half* normalized, int rows, int width, float eps) {
  if (rows <= 0) return;
  launch_kernel(l, dim3((rows + 7) / 8), dim3(256), 0, add_rms_norm_kernel, left, right, w,
                residual, normalized, rows, width, eps);
}

void swiglu(const Launch& l, const __half* gate, const __half* up, __half* out, size_t n) {
  if (!n) return;
  launch_kernel(l, dim3(grid_for(n, 256, l.sm_count)), dim3(256), 0, swiglu_kernel, gate, up,
                out, n);
}

void embedding(const Launch& l, const uint32_t* tokens, const __half* table, __half* out,
               int count, int width, uint32_t rows) {
  if (count <= 0) return;
  int gx = (width + 255) / 256;
  launch_kernel(l, dim3(gx, count), dim3(256), 0, embedding_kernel, tokens, table, out, count,
                width, rows);
}

void rope(const Launch& l, const __half* in, __half* out, int tokens, int heads, int head_dim,
          Pos pos, float theta) {
  int rows = tokens * heads;
  if (rows <= 0) return;
  launch_kernel(l, dim3((rows + 7) / 8), dim3(256), 0, rope_kernel, in, out, tokens, heads,
                head_dim, pos, theta);
}

void qk_norm_rope_cache(const Launch& l, const __half* q, const __half* k, const __half* qw,
                        const __half* kw, __half* q_out, __half* key_cache, int tokens,
                        int q_heads, int kv_heads, int head_dim, Pos pos, float theta,
                        float eps, bool round_norm, const float2* rope) {
  int rows = tokens * (q_heads + kv_heads);
  if (rows <= 0) return;
  launch_kernel(l, dim3((rows + 7) / 8), dim3(256), 0, qk_norm_rope_cache_kernel, q, k, qw, kw,
                q_out, key_cache, tokens, q_heads, kv_heads, head_dim, pos, theta, eps,
                (int)round_norm, rope);
}

void rope_table(cudaStream_t s, float2* out, int positions, int head_dim, float theta) {
  size_t n = (size_t)positions * (head_dim / 2);
  if (!n) return;
  int grid = (int)std::min<size_t>((n + 255) / 256, 4096);
  rope_table_kernel<<<grid, 256, 0, s>>>(out, positions, head_dim, theta);
  MI_CUDA(cudaGetLastError());
}

void copy_kv(const Launch& l, const __half* src, __half* cache, int tokens, int stride,
             Pos pos) {
  size_t n = (size_t)tokens * stride;
  if (!n) return;
  launch_kernel(l, dim3(grid_for(n, 256, l.sm_count)), dim3(256), 0, copy_kv_kernel, src, cache,
                tokens, stride, pos);
}

int argmax_partials(size_t n) { return (int)((n + 2047) / 2048); }

void argmax(const Launch& l, const __half* logits, size_t n, float* pv, uint32_t* pi,
            uint32_t* out) {
  int groups = argmax_partials(n);
  launch_kernel(l, dim3(groups), dim3(256), 0, argmax_partial_kernel, logits, n, pv, pi);
  launch_kernel(l, dim3(1), dim3(256), 0, argmax_reduce_kernel, (const float*)pv,
                (const uint32_t*)pi, groups, out);
}

}  // namespace k
}  // namespace mi
