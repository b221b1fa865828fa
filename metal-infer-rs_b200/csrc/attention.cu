// Causal GQA attention over the contiguous [capacity, kv_heads, head_dim]
// FP16 cache (qwen3.rs:68-117):
//   attention_reference  two-pass FP32 softmax, one thread per output element
//                        (attention_reference_f16, transformer.metal:1579-1612)
//   attention_decode     single query, split-K over key blocks for any GQA
//                        ratio; each CTA keeps FP32 online-softmax states for
//                        the whole query group of one KV head and the last CTA
//                        of the head merges them by log-sum-exp
//                        (attention_flash_decode_*, transformer.metal:1911-2316)
//   attention_decode_fused  the same with the per-head QK RMSNorm + RoPE and
//                        the K/V append of the new token folded in
//                        (qk_norm_rope_cache_f16 + copy_kv_f16)
//   attention_prefill    flash-prefill semantics: 32-key blocks, FP32 scores
//                        and row sums, probabilities rounded to FP16 before
//                        they weight V (transformer.metal:1669-1822)

#include "device.cuh"

namespace mi {
namespace k {

namespace {

__device__ __forceinline__ int kv_len_of(const AttnProblem& p) {
  return p.kv_len_dev ? (int)(*p.kv_len_dev) + p.kv_len_add : p.kv_len;
}

// ---- reference ---------------------------------------------------------------
__global__ void attention_reference_kernel(AttnProblem p) {
  pdl_wait();
  int d = blockIdx.x * blockDim.x + threadIdx.x;
  int h = blockIdx.y;
  int qi = blockIdx.z;
  if (d >= p.hd || h >= p.qh || qi >= p.tokens) return;
  int L = kv_len_of(p);
  int kvh = h / (p.qh / p.kvh);
  int available = p.causal ? min(L, p.query_offset + qi + 1) : L;
  float scale = rsqrtf((float)p.hd);
  scale = __frcp_rn(__fsqrt_rn((float)p.hd));
  const __half* q = p.q + ((size_t)qi * p.qh + h) * p.hd;
  float maximum = -INFINITY;
  for (int j = 0; j < available; ++j) {
    const __half* kr = p.k + ((size_t)j * p.kvh + kvh) * p.hd;
    float s = 0.f;
    for (int x = 0; x < p.hd; ++x) s = fmaf(__half2float(q[x]), __half2float(kr[x]), s);
    maximum = fmaxf(maximum, s * scale);
  }
  float den = 0.f, num = 0.f;
  for (int j = 0; j < available; ++j) {
    const __half* kr = p.k + ((size_t)j * p.kvh + kvh) * p.hd;
    float s = 0.f;
    for (int x = 0; x < p.hd; ++x) s = fmaf(__half2float(q[x]), __half2float(kr[x]), s);
    float prob = expf(s * scale - maximum);
    den += prob;
    num = fmaf(prob, __half2float(p.v[((size_t)j * p.kvh + kvh) * p.hd + d]), num);
  }
  p.out[((size_t)qi * p.qh + h) * p.hd + d] = __float2half_rn(num / den);
}

// ---- split-K decode --------------------------------------------------------------
// CTA (s, g) handles keys [s*chunk, min(L, (s+1)*chunk)) of KV head g for the
// G query heads of its group. Warps stride over keys; each lane owns HD/32
// consecutive dims. Partial state per (split, head): [max, sum, acc[HD]].
constexpr int kDecodeWarps = 4;
constexpr int kMinKeysPerSplit = 32;

template <int HD, int G>
struct DecodeState {
  float m[G], l[G], acc[G][HD / 32];
};

template <int HD, int G>
__device__ __forceinline__ void decode_keys(const float (&q)[G][HD / 32], const __half* K,
                                            const __half* V, int kvh_stride, int begin, int end,
                                            float scale, DecodeState<HD, G>& st) {
  constexpr int E = HD / 32;
  const int lane = threadIdx.x & 31;
  const int warp = threadIdx.x >> 5;
  for (int j = begin + warp; j < end; j += kDecodeWarps) {
    const __half* kr = K + (size_t)j * kvh_stride + lane * E;
    const __half* vr = V + (size_t)j * kvh_stride + lane * E;
    float kf[E], vf[E];
    if (E == 4) {
      uint2 kk = *reinterpret_cast<const uint2*>(kr);
      uint2 vv = *reinterpret_cast<const uint2*>(vr);
      const __half2* hk = reinterpret_cast<const __half2*>(&kk);
      const __half2* hv = reinterpret_cast<const __half2*>(&vv);
      float2 a = __half22float2(hk[0]), b = __half22float2(hk[1]);
      kf[0] = a.x; kf[1] = a.y; kf[2] = b.x; kf[3] = b.y;
      a = __half22float2(hv[0]); b = __half22float2(hv[1]);
      vf[0] = a.x; vf[1] = a.y; vf[2] = b.x; vf[3] = b.y;
    } else {
#pragma unroll
      for (int e = 0; e < E; ++e) {
        kf[e] = __half2float(kr[e]);
        vf[e] = __half2float(vr[e]);
      }
    }
#pragma unroll
    for (int g = 0; g < G; ++g) {
      float part = 0.f;
#pragma unroll
      for (int e = 0; e < E; ++e) part = fmaf(q[g][e], kf[e], part);
      float s = warp_sum(part) * scale;
      float nm = fmaxf(st.m[g], s);
      float prev = expf(st.m[g] - nm);
      float cur = expf(s - nm);
#pragma unroll
      for (int e = 0; e < E; ++e) st.acc[g][e] = fmaf(st.acc[g][e], prev, cur * vf[e]);
      st.l[g] = fmaf(st.l[g], prev, cur);
      st.m[g] = nm;
    }
  }
}

// Combines the warps' states in shared memory and writes the CTA partial;
// the last CTA of the KV head merges all partials into the output.
template <int HD, int G>
__device__ void decode_finish(DecodeState<HD, G>& st, float* scratch, uint32_t* counters,
                              int splits_eff, int split, int g_kv, __half* out) {
  constexpr int E = HD / 32;
  constexpr int stride = HD + 2;
  __shared__ float sm_m[kDecodeWarps][G], sm_l[kDecodeWarps][G];
  __shared__ float sm_acc[kDecodeWarps][G][HD];
  __shared__ bool last;
  const int lane = threadIdx.x & 31;
  const int warp = threadIdx.x >> 5;
#pragma unroll
  for (int g = 0; g < G; ++g) {
    if (lane == 0) {
      sm_m[warp][g] = st.m[g];
      sm_l[warp][g] = st.l[g];
    }
#pragma unroll
    for (int e = 0; e < E; ++e) sm_acc[warp][g][lane * E + e] = st.acc[g][e];
  }
  __syncthreads();
  float* part = scratch + ((size_t)g_kv * gridDim.x + split) * G * stride;
  for (int idx = threadIdx.x; idx < G * HD; idx += blockDim.x) {
    int g = idx / HD, d = idx - g * HD;
    float M = -INFINITY;
#pragma unroll
    for (int w = 0; w < kDecodeWarps; ++w) M = fmaxf(M, sm_m[w][g]);
    float num = 0.f, den = 0.f;
#pragma unroll
    for (int w = 0; w < kDecodeWarps; ++w) {
      float f = sm_m[w][g] == -INFINITY ? 0.f : expf(sm_m[w][g] - M);
      num = fmaf(sm_acc[w][g][d], f, num);
      den = fmaf(sm_l[w][g], f, den);
    }
    part[g * stride + 2 + d] = num;
    if (d == 0) {
      part[g * stride] = M;
      part[g * stride + 1] = den;
    }
  }
  __threadfence();
  __syncthreads();
  if (threadIdx.x == 0) {
    uint32_t done = atomicAdd(counters + g_kv, 1u);
    last = done == (uint32_t)splits_eff - 1;
  }
  __syncthreads();
  if (!last) return;
  __threadfence();
  const float* base = scratch + (size_t)g_kv * gridDim.x * G * stride;
  for (int idx = threadIdx.x; idx < G * HD; idx += blockDim.x) {
    int g = idx / HD, d = idx - g * HD;
    float M = -INFINITY;
    for (int s = 0; s < splits_eff; ++s) M = fmaxf(M, __ldcg(base + (size_t)(s * G + g) * stride));
    float num = 0.f, den = 0.f;
    for (int s = 0; s < splits_eff; ++s) {
      const float* ps = base + (size_t)(s * G + g) * stride;
      float m = __ldcg(ps);
      float f = m == -INFINITY ? 0.f : expf(m - M);
      den = fmaf(__ldcg(ps + 1), f, den);
      num = fmaf(__ldcg(ps + 2 + d), f, num);
    }
    out[(size_t)(g_kv * G + g) * HD + d] = __float2half_rn(num / den);
  }
  if (threadIdx.x == 0) counters[g_kv] = 0u;
}

template <int HD, int G>
__global__ void __launch_bounds__(kDecodeWarps * 32)
    attention_decode_kernel(AttnProblem p, float* scratch, uint32_t* counters, int block_keys) {
  constexpr int E = HD / 32;
  const int lane = threadIdx.x & 31;
  const int g_kv = blockIdx.y;
  const int split = blockIdx.x;
  pdl_wait();
  const int L = kv_len_of(p);
  const int available = p.causal && p.query_offset < L ? p.query_offset + 1 : L;
  int splits_eff = min((int)gridDim.x, (available + block_keys - 1) / block_keys);
  if (splits_eff < 1) splits_eff = 1;
  if (split >= splits_eff) return;
  const int chunk = (available + splits_eff - 1) / splits_eff;
  const int begin = split * chunk;
  const int end = min(available, begin + chunk);
  float q[G][E];
#pragma unroll
  for (int g = 0; g < G; ++g)
#pragma unroll
    for (int e = 0; e < E; ++e)
      q[g][e] = __half2float(p.q[(size_t)(g_kv * G + g) * HD + lane * E + e]);
  DecodeState<HD, G> st;
#pragma unroll
  for (int g = 0; g < G; ++g) {
    st.m[g] = -INFINITY;
    st.l[g] = 0.f;
#pragma unroll
    for (int e = 0; e < E; ++e) st.acc[g][e] = 0.f;
  }
  const float scale = __frcp_rn(__fsqrt_rn((float)HD));
  decode_keys<HD, G>(q, p.k + (size_t)g_kv * HD, p.v + (size_t)g_kv * HD, p.kvh * HD, begin, end,
                     scale, st);
  decode_finish<HD, G>(st, scratch, counters, splits_eff, split, g_kv, p.out);
}

// Per-head RMSNorm + RoPE of one head held as E = HD/32 consecutive dims per
// lane (lane l owns dims [l*E, l*E + E)); the rotation partner of dim d is
// d +- HD/2, which lives in lane l ^ 16.
template <int HD>
__device__ __forceinline__ void norm_rope_lane(float (&x)[HD / 32], const __half* w,
                                               uint32_t pos, float theta, float eps,
                                               bool round_norm, float (&out)[HD / 32]) {
  constexpr int E = HD / 32;
  const int lane = threadIdx.x & 31;
  float ss = 0.f;
#pragma unroll
  for (int e = 0; e < E; ++e) ss = fmaf(x[e], x[e], ss);
  float scale = rms_scale(warp_sum(ss), HD, eps);
  float nx[E];
#pragma unroll
  for (int e = 0; e < E; ++e) {
    nx[e] = norm_mul(x[e], scale, __half2float(w[lane * E + e]));
    if (round_norm) nx[e] = __half2float(__float2half_rn(nx[e]));
  }
  const bool first = lane < 16;
#pragma unroll
  for (int e = 0; e < E; ++e) {
    float partner = __shfl_xor_sync(0xffffffffu, nx[e], 16);
    int d = lane * E + e;
    int pair = first ? d : d - HD / 2;
    float exponent = __fdiv_rn(-(float)(pair * 2), (float)HD);
    float frequency = powf(theta, exponent);
    float angle = __fmul_rn((float)pos, frequency);
    float sn, cs;
    sincosf(angle, &sn, &cs);
    float r = first ? __fsub_rn(__fmul_rn(nx[e], cs), __fmul_rn(partner, sn))
                    : __fadd_rn(__fmul_rn(partner, sn), __fmul_rn(nx[e], cs));
    out[e] = __half2float(__float2half_rn(r));
  }
}

template <int HD, int G>
__global__ void __launch_bounds__(kDecodeWarps * 32)
    attention_decode_fused_kernel(DecodeFused p, float* scratch, uint32_t* counters) {
  constexpr int E = HD / 32;
  const int lane = threadIdx.x & 31;
  const int warp = threadIdx.x >> 5;
  const int g_kv = blockIdx.y;
  const int split = blockIdx.x;
  pdl_trigger();
  pdl_wait();
  const uint32_t pos = pos_of(p.pos);
  const int L = (int)pos + 1;
  int splits_eff = min((int)gridDim.x, (L + kMinKeysPerSplit - 1) / kMinKeysPerSplit);
  if (splits_eff < 1) splits_eff = 1;
  if (split >= splits_eff) return;
  const int chunk = (L + splits_eff - 1) / splits_eff;
  const int begin = split * chunk;
  const int end = min(L, begin + chunk);
  const int kv_stride = p.kvh * HD;

  // Query heads of this group: RMSNorm + RoPE, rounded to FP16.
  float q[G][E];
#pragma unroll
  for (int g = 0; g < G; ++g) {
    float raw[E];
#pragma unroll
    for (int e = 0; e < E; ++e)
      raw[e] = __half2float(p.q_raw[(size_t)(g_kv * G + g) * HD + lane * E + e]);
    norm_rope_lane<HD>(raw, p.q_norm, pos, p.theta, p.eps, p.round_norm, q[g]);
  }
  // The CTA that owns the new position appends the rotated key and the value.
  if (warp == 0 && (int)(pos) >= begin && (int)pos < end) {
    float raw[E], kr[E];
#pragma unroll
    for (int e = 0; e < E; ++e) raw[e] = __half2float(p.k_raw[(size_t)g_kv * HD + lane * E + e]);
    norm_rope_lane<HD>(raw, p.k_norm, pos, p.theta, p.eps, p.round_norm, kr);
    __half* kd = p.key_cache + (size_t)pos * kv_stride + (size_t)g_kv * HD + lane * E;
    __half* vd = p.value_cache + (size_t)pos * kv_stride + (size_t)g_kv * HD + lane * E;
#pragma unroll
    for (int e = 0; e < E; ++e) {
      kd[e] = __float2half_rn(kr[e]);
      vd[e] = p.v_raw[(size_t)g_kv * HD + lane * E + e];
    }
  }
  __syncthreads();
  DecodeState<HD, G> st;
#pragma unroll
  for (int g = 0; g < G; ++g) {
    st.m[g] = -INFINITY;
    st.l[g] = 0.f;
#pragma unroll
    for (int e = 0; e < E; ++e) st.acc[g][e] = 0.f;
  }
  const float scale = __frcp_rn(__fsqrt_rn((float)HD));
  decode_keys<HD, G>(q, p.key_cache + (size_t)g_kv * HD, p.value_cache + (size_t)g_kv * HD,
                     kv_stride, begin, end, scale, st);
  decode_finish<HD, G>(st, scratch, counters, splits_eff, split, g_kv, p.out);
}

// ---- prefill (flash-prefill semantics) ----------------------------------------
// One warp per (query, head). Keys in blocks of 32 from 0: lane j scores key
// (block + j); the block max updates the running max; weights exp(s - max)
// sum unrounded into the row sum and are rounded to FP16 before weighting V.
constexpr int kPrefillWarps = 4;

__global__ void __launch_bounds__(kPrefillWarps * 32) attention_prefill_kernel(AttnProblem p) {
  __shared__ float qs[kPrefillWarps][256];
  const int lane = threadIdx.x & 31;
  const int warp = threadIdx.x >> 5;
  const int row = blockIdx.x * kPrefillWarps + warp;  // qi * qh + h
  pdl_wait();
  if (row >= p.tokens * p.qh) return;
  const int qi = row / p.qh;
  const int h = row - qi * p.qh;
  const int kvh = h / (p.qh / p.kvh);
  const int L = kv_len_of(p);
  const int available = p.causal ? min(L, p.query_offset + qi + 1) : L;
  const int hd = p.hd;
  const int kv_stride = p.kvh * hd;
  for (int d = lane; d < hd; d += 32) qs[warp][d] = __half2float(p.q[(size_t)row * hd + d]);
  __syncwarp();
  const float scale = __frcp_rn(__fsqrt_rn((float)hd));
  float acc[8];
#pragma unroll
  for (int i = 0; i < 8; ++i) acc[i] = 0.f;
  float row_max = -INFINITY, row_sum = 0.f;
  const bool vec = (hd % 8) == 0;
  for (int base = 0; base < available; base += 32) {
    const int key = base + lane;
    const bool valid = key < available;
    float s = -INFINITY;
    if (valid) {
      const __half* kr = p.k + (size_t)key * kv_stride + (size_t)kvh * hd;
      float dot = 0.f;
      if (vec) {
        for (int c = 0; c < hd; c += 8) {
          uint4 kk = *reinterpret_cast<const uint4*>(kr + c);
          const __half2* hk = reinterpret_cast<const __half2*>(&kk);
#pragma unroll
          for (int i = 0; i < 4; ++i) {
            float2 f = __half22float2(hk[i]);
            dot = fmaf(qs[warp][c + 2 * i], f.x, dot);
            dot = fmaf(qs[warp][c + 2 * i + 1], f.y, dot);
          }
        }
      } else {
        for (int c = 0; c < hd; ++c) dot = fmaf(qs[warp][c], __half2float(kr[c]), dot);
      }
      s = dot * scale;
    }
    float block_max = warp_max(s);
    float next_max = fmaxf(row_max, block_max);
    float alpha = isinf(row_max) ? 0.f : expf(row_max - next_max);
    float w = valid ? expf(s - next_max) : 0.f;
    float block_sum = warp_sum(w);
    float prob = p.round_p ? __half2float(__float2half_rn(w)) : w;
    row_sum = fmaf(row_sum, alpha, block_sum);
    row_max = next_max;
#pragma unroll
    for (int i = 0; i < 8; ++i) acc[i] *= alpha;
    const int count = min(32, available - base);
    for (int c = 0; c < count; ++c) {
      float pc = __shfl_sync(0xffffffffu, prob, c);
      const __half* vr = p.v + (size_t)(base + c) * kv_stride + (size_t)kvh * hd;
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        int d = lane + i * 32;
        if (d < hd) acc[i] = fmaf(pc, __half2float(vr[d]), acc[i]);
      }
    }
  }
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    int d = lane + i * 32;
    if (d < hd) p.out[(size_t)row * hd + d] = __float2half_rn(acc[i] / row_sum);
  }
}

template <int HD>
bool launch_decode_hd(const Launch& l, const AttnProblem& p, int splits, int block_keys,
                      float* scratch, uint32_t* counters) {
  int G = p.qh / p.kvh;
  dim3 grid(splits, p.kvh);
  dim3 block(kDecodeWarps * 32);
  switch (G) {
    case 1: launch_kernel(l, grid, block, 0, attention_decode_kernel<HD, 1>, p, scratch, counters, block_keys); return true;
    case 2: launch_kernel(l, grid, block, 0, attention_decode_kernel<HD, 2>, p, scratch, counters, block_keys); return true;
    case 4: launch_kernel(l, grid, block, 0, attention_decode_kernel<HD, 4>, p, scratch, counters, block_keys); return true;
    case 8: launch_kernel(l, grid, block, 0, attention_decode_kernel<HD, 8>, p, scratch, counters, block_keys); return true;
    default: return false;
  }
}

}  // namespace

void attention_reference(const Launch& l, const AttnProblem& p) {
  dim3 grid((p.hd + 127) / 128, p.qh, p.tokens);
  launch_kernel(l, grid, dim3(128), 0, attention_reference_kernel, p);
}

size_t attention_decode_scratch(int kvh, int splits, int group, int hd) {
  return (size_t)kvh * splits * group * (hd + 2) * sizeof(float);
}

int attention_decode_splits(int kv_len_max, int kvh, int sm_count, int block_keys) {
  int by_len = (kv_len_max + block_keys - 1) / block_keys;
  int by_sm = (2 * sm_count + kvh - 1) / kvh;
  int s = by_len < by_sm ? by_len : by_sm;
  return s < 1 ? 1 : s;
}

void attention_decode(const Launch& l, const AttnProblem& p, int splits, int block_keys,
                      float* scratch, uint32_t* counters) {
  bool ok = false;
  if (p.hd == 128) ok = launch_decode_hd<128>(l, p, splits, block_keys, scratch, counters);
  else if (p.hd == 64) ok = launch_decode_hd<64>(l, p, splits, block_keys, scratch, counters);
  else if (p.hd == 256) ok = launch_decode_hd<256>(l, p, splits, block_keys, scratch, counters);
  if (!ok) attention_reference(l, p);
}

void attention_decode_fused(const Launch& l, const DecodeFused& p, int splits, float* scratch,
                            uint32_t* counters) {
  MI_REQUIRE(p.hd == 128, MI_ERR_SHAPE, "fused decode attention needs head_dim 128");
  int G = p.qh / p.kvh;
  dim3 grid(splits, p.kvh);
  dim3 block(kDecodeWarps * 32);
  switch (G) {
    case 1: launch_kernel(l, grid, block, 0, attention_decode_fused_kernel<128, 1>, p, scratch, counters); break;
    case 2: launch_kernel(l, grid, block, 0, attention_decode_fused_kernel<128, 2>, p, scratch, counters); break;
    case 4: launch_kernel(l, grid, block, 0, attention_decode_fused_kernel<128, 4>, p, scratch, counters); break;
    case 8: launch_kernel(l, grid, block, 0, attention_decode_fused_kernel<128, 8>, p, scratch, counters); break;
    default: fail(MI_ERR_SHAPE, "fused decode attention supports GQA ratios 1, 2, 4 and 8");
  }
}

void attention_prefill(const Launch& l, const AttnProblem& p) {
  MI_REQUIRE(p.hd <= 256, MI_ERR_SHAPE, "prefill attention needs head_dim <= 256");
  int rows = p.tokens * p.qh;
  if (rows <= 0) return;
  launch_kernel(l, dim3((rows + kPrefillWarps - 1) / kPrefillWarps), dim3(kPrefillWarps * 32), 0,
                attention_prefill_kernel, p);
}

}  // namespace k
}  // namespace mi
