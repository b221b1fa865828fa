// The engine's arithmetic contract, shared by every kernel on the decode path
// and by the small-prompt prefill path (the CPU oracle states the same
// contract independently, which makes those paths bit-exact):
//
//  * DOT(x, y, n): chunks of 8 consecutive elements; chunk c belongs to lane
//    c mod L, L = min(32, next_pow2(ceil(n / 8))); a lane accumulates its
//    chunks in increasing order with 8 sequential fused multiply-adds per
//    chunk; the L lane sums meet in a butterfly (xor L/2, ..., 1). Sums of
//    squares are DOT(x, x). This is one fixed instance of the reference's
//    lane-strided loops + simd_sum.
//  * exp: Cody-Waite reduction n = rint(x log2 e), r = x - n ln2 (two-part
//    constant), e^r by the degree-7 Taylor polynomial (Horner, fused
//    multiply-adds), scaled by 2^n.
//  * rsqrt(v) = 1 / sqrt(v), both correctly rounded.
//  * RoPE: frequency = float(pow(theta, -2i / d)); cos / sin of the FP32
//    angle pos * frequency in double precision, rounded once to FP32.
#pragma once

#include <cuda_fp16.h>

#include <cstdint>

namespace mi {
namespace k {

__device__ __forceinline__ float mi_exp(float x) {
  // Branch-free: the reduction runs on x clamped to [-104, 89] and the
  // out-of-range / NaN results are selected at the end. 2^n is applied as
  // 2^(n >> 1) * 2^(n - (n >> 1)): the first product is exact, so the result
  // carries the single rounding of p * 2^n, also where it is subnormal.
  const float kLog2e = 0x1.715476p+0f;
  const float kLn2Hi = 0x1.62e4p-1f;
  const float kLn2Lo = 0x1.7f7d1cp-20f;
  const float xc = fminf(fmaxf(x, -104.0f), 89.0f);
  float n = rintf(__fmul_rn(xc, kLog2e));
  float r = __fmaf_rn(n, -kLn2Hi, xc);
  r = __fmaf_rn(n, -kLn2Lo, r);
  float p = 0x1.a01a02p-13f;
  p = __fmaf_rn(p, r, 0x1.6c16c2p-10f);
  p = __fmaf_rn(p, r, 0x1.111112p-7f);
  p = __fmaf_rn(p, r, 0x1.555556p-5f);
  p = __fmaf_rn(p, r, 0x1.555556p-3f);
  p = __fmaf_rn(p, r, 0.5f);
  p = __fmaf_rn(p, r, 1.0f);
  p = __fmaf_rn(p, r, 1.0f);
  const int ni = (int)n;
  const int n1 = ni >> 1;
  const int n2 = ni - n1;
  float res = __fmul_rn(__fmul_rn(p, __int_as_float((n1 + 127) << 23)),
                        __int_as_float((n2 + 127) << 23));
  res = x > 89.0f ? __int_as_float(0x7f800000) : res;
  res = x < -104.0f ? 0.0f : res;
  return x != x ? x : res;
}

// Lanes of the canonical reduction for n elements.
__host__ __device__ __forceinline__ int canon_lanes(int n) {
  int chunks = (n + 7) / 8;
  int l = 1;
  while (l < chunks && l < 32) l <<= 1;
  return l;
}

// Butterfly over `lanes` lanes of a warp (lanes a power of two <= 32); every
// lane of each group ends with the group's sum.
__device__ __forceinline__ float canon_butterfly(float v, int lanes) {
  for (int o = lanes >> 1; o >= 1; o >>= 1) v = __fadd_rn(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}

// One canonical reduction per warp, returned to every lane (lanes outside
// the first group of `lanes` hold other sums after the butterfly alone).
__device__ __forceinline__ float canon_reduce(float v, int lanes) {
  v = canon_butterfly(v, lanes);
  return lanes < 32 ? __shfl_sync(0xffffffffu, v, 0) : v;
}

// The same over a subset of a warp: `mask` names exactly the lanes that
// execute the call (every xor partner must be in it).
__device__ __forceinline__ float canon_butterfly_mask(float v, int lanes, unsigned mask) {
  for (int o = lanes >> 1; o >= 1; o >>= 1) v = __fadd_rn(v, __shfl_xor_sync(mask, v, o));
  return v;
}

// a * b + c for FP16 a, b and FP32 c with one rounding: the mixed-precision
// FMA of sm_100 (the FP16 operands widen exactly, so this equals
// __fmaf_rn(float(a), float(b), c) without the two conversions).
__device__ __forceinline__ float fma_f16_f32(unsigned short a, unsigned short b, float c) {
  float d;
  asm("fma.rn.f32.f16 %0, %1, %2, %3;" : "=f"(d) : "h"(a), "h"(b), "f"(c));
  return d;
}

// 8 sequential fused multiply-adds of one chunk (FP16 x FP16).
__device__ __forceinline__ float chunk_dot(const uint4& a, const uint4& b, float acc) {
  const uint32_t x[4] = {a.x, a.y, a.z, a.w};
  const uint32_t y[4] = {b.x, b.y, b.z, b.w};
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    acc = fma_f16_f32((unsigned short)(x[i] & 0xffffu), (unsigned short)(y[i] & 0xffffu), acc);
    acc = fma_f16_f32((unsigned short)(x[i] >> 16), (unsigned short)(y[i] >> 16), acc);
  }
  return acc;
}

// Sum of squares of one FP16 chunk.
__device__ __forceinline__ float chunk_sq(const uint4& a, float acc) { return chunk_dot(a, a, acc); }

// Single-thread canonical DOT of FP32 q (8 consecutive per chunk) with an
// FP16 row, n % 8 == 0, n <= 256: one partial per chunk, then the butterfly
// tree in registers.
template <int N>
__device__ __forceinline__ float canon_dot_thread(const float* q, const uint4* row) {
  constexpr int kChunks = N / 8;
  constexpr int kLanes = kChunks <= 1 ? 1 : kChunks <= 2 ? 2 : kChunks <= 4 ? 4 : kChunks <= 8 ? 8 : kChunks <= 16 ? 16 : 32;
  float v[kLanes];
#pragma unroll
  for (int c = 0; c < kLanes; ++c) v[c] = 0.f;
#pragma unroll
  for (int c = 0; c < kChunks; ++c) {
    uint4 w = row[c];
    const __half2* hw = reinterpret_cast<const __half2*>(&w);
    float acc = 0.f;
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      float2 f = __half22float2(hw[i]);
      acc = __fmaf_rn(q[8 * c + 2 * i], f.x, acc);
      acc = __fmaf_rn(q[8 * c + 2 * i + 1], f.y, acc);
    }
    v[c] = acc;
  }
#pragma unroll
  for (int step = kLanes / 2; step >= 1; step >>= 1)
#pragma unroll
    for (int l = 0; l < step; ++l) v[l] = __fadd_rn(v[l], v[l + step]);
  return v[0];
}

// RoPE terms of (position, pair).
__device__ __forceinline__ void rope_cs(uint32_t pos, int pair, int head_dim, float theta,
                                        float* c, float* s) {
  float exponent = __fdiv_rn(-(float)(pair * 2), (float)head_dim);
  float frequency = (float)pow((double)theta, (double)exponent);
  float angle = __fmul_rn((float)pos, frequency);
  double sd, cd;
  sincos((double)angle, &sd, &cd);
  *c = (float)cd;
  *s = (float)sd;
}

// x * scale * g with both products rounded.
__device__ __forceinline__ float norm_mul(float x, float scale, float g) {
  return __fmul_rn(__fmul_rn(x, scale), g);
}

// rsqrt(total / width + eps), correctly rounded 1 / sqrt.
__device__ __forceinline__ float rms_scale(float total, int width, float eps) {
  return __frcp_rn(__fsqrt_rn(__fadd_rn(__fdiv_rn(total, (float)width), eps)));
}

// SwiGLU of swiglu_f16: (g / (1 + exp(-g))) * u.
__device__ __forceinline__ float silu_mul(float g, float u) {
  return __fmul_rn(__fdiv_rn(g, __fadd_rn(1.0f, mi_exp(-g))), u);
}

// Per-head RMSNorm + RoPE of one 128-dim head held by a half-warp (lane li
// owns dims 8 li .. 8 li + 7; the rotation partner of dim d is d +- 64, lane
// li ^ 8). Returns the FP16-rounded rotated values as floats. `mask` names
// the lanes of the warp executing the call (one or both half-warps).
__device__ __forceinline__ void norm_rope_half(const uint4& raw, const __half* w, uint32_t pos,
                                               float theta, float eps, bool round_norm,
                                               unsigned mask, const float2* rope,
                                               float (&out)[8]) {
  constexpr int HD = 128;
  const int li = threadIdx.x & 15;
  float total = canon_butterfly_mask(chunk_sq(raw, 0.f), 16, mask);
  float scale = rms_scale(total, HD, eps);
  const __half2* hr = reinterpret_cast<const __half2*>(&raw);
  uint4 wr = reinterpret_cast<const uint4*>(w)[li];
  const __half2* hw = reinterpret_cast<const __half2*>(&wr);
  float nx[8];
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    float2 f = __half22float2(hr[i]);
    float2 g = __half22float2(hw[i]);
    nx[2 * i] = norm_mul(f.x, scale, g.x);
    nx[2 * i + 1] = norm_mul(f.y, scale, g.y);
  }
  if (round_norm)
#pragma unroll
    for (int e = 0; e < 8; ++e) nx[e] = __half2float(__float2half_rn(nx[e]));
  const bool first = li < 8;
#pragma unroll
  for (int e = 0; e < 8; ++e) {
    float partner = __shfl_xor_sync(mask, nx[e], 8);
    int d = 8 * li + e;
    int pair = first ? d : d - HD / 2;
    float c, s;
    if (rope) {
      float2 cs = rope[(size_t)pos * (HD / 2) + pair];
      c = cs.x;
      s = cs.y;
    } else {
      rope_cs(pos, pair, HD, theta, &c, &s);
    }
    float r = first ? __fsub_rn(__fmul_rn(nx[e], c), __fmul_rn(partner, s))
                    : __fadd_rn(__fmul_rn(partner, s), __fmul_rn(nx[e], c));
    out[e] = __half2float(__float2half_rn(r));
  }
}

}  // namespace k
}  // namespace mi
