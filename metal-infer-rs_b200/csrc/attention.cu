// Causal GQA attention over the contiguous [capacity, kv_heads, head_dim]
// FP16 cache (qwen3.rs:68-117):
//   attention_reference  two-pass FP32 softmax, one thread per output element
//                        (attention_reference_f16, transformer.metal:1579-1612)
//   attention_decode     one query, flash decode (transformer.metal:2127-2316)
//                        for any GQA ratio: blocks of B keys, 8 interleaved
//                        online-softmax streams per block (one per half-warp;
//                        a lane owns 8 of the 128 dims), stream then block
//                        log-sum-exp merges in index order; the last CTA of a
//                        KV head merges the blocks
//   attention_decode_fused  the same with the per-head QK RMSNorm + RoPE and
//                        the K/V append of the new token folded in
//                        (qk_norm_rope_cache_f16 + copy_kv_f16); the cached
//                        K/V rows are staged by cp.async before the kernel
//                        waits on its predecessor
//   attention_prefill    32-key blocks per query with the block sums of a
//                        32-lane butterfly; flash prefill rounds the
//                        probabilities to FP16 (transformer.metal:1614-1822)
// All reductions follow numerics.cuh.

#include <cuda.h>
#include <cudaTypedefs.h>

#include <mutex>
#include <utility>
#include <vector>

#include "device.cuh"
#include "pipeline.cuh"

namespace mi {
namespace k {

namespace {

constexpr int HD = 128;
constexpr int kDecodeThreads = 128;  // 4 warps = 8 half-warp streams
constexpr int kStreams = 8;
constexpr int kTile = 64;            // keys staged per shared-memory tile
constexpr int kRowBytes = HD * 2;

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
  float scale = __frcp_rn(__fsqrt_rn((float)p.hd));
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
    float prob = mi_exp(s * scale - maximum);
    den += prob;
    num = fmaf(prob, __half2float(p.v[((size_t)j * p.kvh + kvh) * p.hd + d]), num);
  }
  p.out[((size_t)qi * p.qh + h) * p.hd + d] = __float2half_rn(num / den);
}

// ---- flash decode ----------------------------------------------------------------
struct DecodeArgs {
  const __half* q;        // [qh, 128]: final queries, or raw ones when fused
  const __half* k_cache;  // [*, kvh, 128]
  const __half* v_cache;
  int qh, kvh;
  int length;             // keys when length_dev is null
  const uint32_t* length_dev;  // fused: position of the new token (keys = *dev + 1)
  int block;              // keys per block (multiple of kTile)
  __half* out;            // [qh, 128]
  float* scratch;         // [kvh, gridDim.x, G, 130]
  uint32_t* counters;     // [kvh], zero on entry and exit
  int early;              // the first K/V tile is staged before the dependency wait
  // fused front end
  int fused;
  const __half* k_raw;
  const __half* v_raw;
  const __half* q_norm;
  const __half* k_norm;
  __half* k_cache_w;
  __half* v_cache_w;
  float theta, eps;
  int round_norm;
  const float2* rope;     // RoPE table (null: evaluate the terms)
};

// K / V rows padded to 272 bytes: one thread per key reads its row
// without bank conflicts.
constexpr int kRowP = HD + 8;

struct alignas(16) DecodeTile {
  __half k[kTile][kRowP];
  __half v[kTile][kRowP];
};

// The K/V tiles come last: a launch whose blocks fit one tile (block <=
// kTile) reserves only the first, which doubles the CTAs an SM holds.
template <int G>
struct DecodeSmem {
  __half new_k[HD];
  __half new_v[HD];
  __half q[G][HD];              // FP16-rounded queries (after QK-norm + RoPE when fused)
  float sc[G][kTile];           // scaled scores of the tile
  float pa[G][kTile];           // exp(m_prev - m), exp(s - m) per key
  float pc[G][kTile];
  float mrun[2][kStreams][G];   // running max per stream, by tile parity
  float m[kStreams][G];
  float l[kStreams][G];
  float acc[kStreams][G][HD];
  bool last;
  DecodeTile tile[2];
};

template <int G>
constexpr size_t decode_smem_bytes(bool two_tiles) {
  return sizeof(DecodeSmem<G>) - (two_tiles ? 0 : sizeof(DecodeTile));
}

// Stages keys [j0, j1) of head g into buffer `buf` (cp.async, 16 bytes per
// copy), skipping `skip`.
__device__ __forceinline__ void stage_tile(const DecodeArgs& a, int g, int j0, int j1, int skip,
                                           __half (*kt)[kRowP], __half (*vt)[kRowP]) {
  const int per_row = kRowBytes / 16;
  const int total = (j1 - j0) * per_row;
  const size_t stride = (size_t)a.kvh * HD;
  for (int i = threadIdx.x; i < total; i += kDecodeThreads) {
    int r = i / per_row, c = i - r * per_row;
    int j = j0 + r;
    if (j == skip) continue;
    const __half* ks = a.k_cache + (size_t)j * stride + (size_t)g * HD + 8 * c;
    const __half* vs = a.v_cache + (size_t)j * stride + (size_t)g * HD + 8 * c;
    pipe::cp_async16(&kt[r][8 * c], ks);
    pipe::cp_async16(&vt[r][8 * c], vs);
  }
  pipe::cp_async_commit();
}

template <int G>
__global__ void __launch_bounds__(kDecodeThreads) attention_decode_kernel(DecodeArgs a) {
  extern __shared__ __align__(16) uint8_t raw_smem[];
  DecodeSmem<G>& sm = *reinterpret_cast<DecodeSmem<G>*>(raw_smem);
  const int lane = threadIdx.x & 31;
  const int warp = threadIdx.x >> 5;
  const int li = lane & 15;
  const int hw = warp * 2 + (lane >> 4);  // stream index
  const int g_kv = blockIdx.y;
  const int b = blockIdx.x;

  // Keys and this block's range are fixed before the predecessor finishes:
  // the cache length only changes between decode steps.
  const int pos = a.fused ? (int)*a.length_dev : -1;
  const int L = a.fused ? pos + 1 : a.length;
  const int nb = (L + a.block - 1) / a.block;
  const int begin = b * a.block;
  const int end = min(L, begin + a.block);
  const int ntiles = b < nb ? (end - begin + kTile - 1) / kTile : 0;
  // The cached rows (all but the new one, which this kernel appends) are
  // staged before the dependency wait when no predecessor writes them.
  if (ntiles > 0 && a.early)
    stage_tile(a, g_kv, begin, min(end, begin + kTile), pos, sm.tile[0].k, sm.tile[0].v);
  pdl_trigger();
  pdl_wait();
  if (ntiles > 0 && !a.early)
    stage_tile(a, g_kv, begin, min(end, begin + kTile), pos, sm.tile[0].k, sm.tile[0].v);
  if (b >= nb) return;

  // Queries of this group (and, fused, the new key / value).
  if (hw < G) {
    // Both half-warps of this warp take a head unless G is odd here.
    const unsigned mask = (warp * 2 + 1 < G) ? 0xffffffffu : 0x0000ffffu;
    const __half* qsrc = a.q + (size_t)(g_kv * G + hw) * HD;
    uint4 raw = reinterpret_cast<const uint4*>(qsrc)[li];
    float qv[8];
    if (a.fused) {
      norm_rope_half(raw, a.q_norm, (uint32_t)pos, a.theta, a.eps, a.round_norm != 0, mask,
                     a.rope, qv);
    } else {
      const __half2* hr = reinterpret_cast<const __half2*>(&raw);
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        float2 f = __half22float2(hr[i]);
        qv[2 * i] = f.x;
        qv[2 * i + 1] = f.y;
      }
    }
    // FP16-rounded values (the fused RoPE rounds; raw queries are FP16)
    uint4 qq;
    __half2* hq2 = reinterpret_cast<__half2*>(&qq);
#pragma unroll
    for (int i = 0; i < 4; ++i) hq2[i] = __floats2half2_rn(qv[2 * i], qv[2 * i + 1]);
    reinterpret_cast<uint4*>(sm.q[hw])[li] = qq;
  }
  if (a.fused && pos >= begin && pos < end && warp == 3 && lane >= 16) {
    uint4 raw = reinterpret_cast<const uint4*>(a.k_raw + (size_t)g_kv * HD)[li];
    float kv[8];
    norm_rope_half(raw, a.k_norm, (uint32_t)pos, a.theta, a.eps, a.round_norm != 0, 0xffff0000u,
                   a.rope, kv);
    uint4 kk;
    __half2* hk = reinterpret_cast<__half2*>(&kk);
#pragma unroll
    for (int i = 0; i < 4; ++i) hk[i] = __floats2half2_rn(kv[2 * i], kv[2 * i + 1]);
    uint4 vv = reinterpret_cast<const uint4*>(a.v_raw + (size_t)g_kv * HD)[li];
    const size_t row = (size_t)pos * a.kvh * HD + (size_t)g_kv * HD;
    reinterpret_cast<uint4*>(a.k_cache_w + row)[li] = kk;
    reinterpret_cast<uint4*>(a.v_cache_w + row)[li] = vv;
    reinterpret_cast<uint4*>(sm.new_k)[li] = kk;
    reinterpret_cast<uint4*>(sm.new_v)[li] = vv;
  }

  // Lane per key: one thread per (key, head) score with the canonical tree
  // in registers; a key's running maximum is its stream's prefix maximum
  // (exact in any order), so each key's two exponentials are independent;
  // the accumulations stay sequential in key order, one thread per (stream,
  // head, 8 dims). Stream s takes block-relative keys s, s + 8, ... (tiles
  // are multiples of 8 keys, so the order is the block's).
  constexpr int R = G;  // accumulators per thread: kStreams * G * 16 / 128
  if (threadIdx.x < kStreams * G) sm.mrun[0][threadIdx.x / G][threadIdx.x % G] = -INFINITY;
  float acc[R][8], l[R];
#pragma unroll
  for (int r = 0; r < R; ++r) {
    l[r] = 0.f;
#pragma unroll
    for (int e = 0; e < 8; ++e) acc[r][e] = 0.f;
  }
  const float scale = __frcp_rn(__fsqrt_rn((float)HD));
  const uint4* nk = reinterpret_cast<const uint4*>(sm.new_k);
  const uint4* nv = reinterpret_cast<const uint4*>(sm.new_v);

  for (int t = 0; t < ntiles; ++t) {
    const int buf = t & 1;
    const int j0 = begin + t * kTile;
    const int j1 = min(end, j0 + kTile);
    const int cnt = j1 - j0;
    const int cur = t & 1;
    if (t + 1 < ntiles)
      stage_tile(a, g_kv, j1, min(end, j1 + kTile), pos, sm.tile[buf ^ 1].k, sm.tile[buf ^ 1].v);
    if (t + 1 < ntiles)
      asm volatile("cp.async.wait_group 1;" ::: "memory");
    else
      pipe::cp_async_wait_all();
    __syncthreads();
    // scores
    for (int idx = threadIdx.x; idx < kTile * G; idx += kDecodeThreads) {
      const int jj = idx & (kTile - 1), g = idx / kTile;
      if (jj < cnt) {
        const bool fresh = j0 + jj == pos;
        const uint4* q = reinterpret_cast<const uint4*>(sm.q[g]);
        const uint4* kr = reinterpret_cast<const uint4*>(sm.tile[buf].k[jj]);
        float d[8];
#pragma unroll
        for (int c = 0; c < 8; ++c) d[c] = chunk_dot(q[c], fresh ? nk[c] : kr[c], 0.f);
#pragma unroll
        for (int c = 0; c < 8; ++c)
          d[c] = __fadd_rn(d[c], chunk_dot(q[c + 8], fresh ? nk[c + 8] : kr[c + 8], 0.f));
#pragma unroll
        for (int step = 4; step >= 1; step >>= 1)
#pragma unroll
          for (int c = 0; c < step; ++c) d[c] = __fadd_rn(d[c], d[c + step]);
        sm.sc[g][jj] = __fmul_rn(d[0], scale);
      }
    }
    __syncthreads();
    // prefix maxima and the two exponentials of every key
    for (int idx = threadIdx.x; idx < kTile * G; idx += kDecodeThreads) {
      const int jj = idx & (kTile - 1), g = idx / kTile, st = jj & (kStreams - 1);
      if (jj < cnt) {
        float prev[kTile / kStreams];
#pragma unroll
        for (int i = 0; i < kTile / kStreams; ++i) prev[i] = sm.sc[g][st + kStreams * i];
        float mp = sm.mrun[cur][st][g];
#pragma unroll
        for (int i = 0; i < kTile / kStreams; ++i)
          if (st + kStreams * i < jj) mp = fmaxf(mp, prev[i]);
        const float sc = sm.sc[g][jj];
        const float mn = fmaxf(mp, sc);
        sm.pa[g][jj] = mi_exp(__fsub_rn(mp, mn));
        sm.pc[g][jj] = mi_exp(__fsub_rn(sc, mn));
        if (jj + kStreams >= cnt) sm.mrun[cur ^ 1][st][g] = mn;  // the stream's last key here
      } else if (jj < kStreams) {
        sm.mrun[cur ^ 1][jj][g] = sm.mrun[cur][jj][g];  // a stream with no key in this tile
      }
    }
    __syncthreads();
    // accumulations in key order
#pragma unroll
    for (int r = 0; r < R; ++r) {
      const int idx = threadIdx.x + r * kDecodeThreads;
      const int st = (idx >> 4) & (kStreams - 1), g = idx >> 7;
#pragma unroll
      for (int i = 0; i < kTile / kStreams; ++i) {
        const int jj = st + kStreams * i;
        if (jj >= cnt) break;
        const float pa = sm.pa[g][jj], pc = sm.pc[g][jj];
        const uint4 vv = j0 + jj == pos ? nv[li]
                                        : reinterpret_cast<const uint4*>(sm.tile[buf].v[jj])[li];
        const __half2* hv = reinterpret_cast<const __half2*>(&vv);
#pragma unroll
        for (int e2 = 0; e2 < 4; ++e2) {
          const float2 f = __half22float2(hv[e2]);
          acc[r][2 * e2] = __fmaf_rn(acc[r][2 * e2], pa, __fmul_rn(pc, f.x));
          acc[r][2 * e2 + 1] = __fmaf_rn(acc[r][2 * e2 + 1], pa, __fmul_rn(pc, f.y));
        }
        l[r] = __fmaf_rn(l[r], pa, pc);
      }
    }
    __syncthreads();
  }

  // Stream states -> shared memory for the stream merge (index order).
#pragma unroll
  for (int r = 0; r < R; ++r) {
    const int idx = threadIdx.x + r * kDecodeThreads;
    const int st = (idx >> 4) & (kStreams - 1), g = idx >> 7;
#pragma unroll
    for (int e = 0; e < 8; ++e) sm.acc[st][g][8 * li + e] = acc[r][e];
    if (li == 0) sm.l[st][g] = l[r];
  }
  if (threadIdx.x < kStreams * G)
    sm.m[threadIdx.x / G][threadIdx.x % G] = sm.mrun[ntiles & 1][threadIdx.x / G][threadIdx.x % G];
  __syncthreads();
  const int stride = HD + 2;
  float* part = a.scratch + ((size_t)g_kv * gridDim.x + b) * G * stride;
  for (int idx = threadIdx.x; idx < G * HD; idx += kDecodeThreads) {
    int g = idx / HD, d = idx - g * HD;
    float M = -INFINITY;
#pragma unroll
    for (int s = 0; s < kStreams; ++s) M = fmaxf(M, sm.m[s][g]);
    float num = 0.f, den = 0.f;
#pragma unroll
    for (int s = 0; s < kStreams; ++s) {
      float f = sm.m[s][g] == -INFINITY ? 0.f : mi_exp(__fsub_rn(sm.m[s][g], M));
      num = __fmaf_rn(sm.acc[s][g][d], f, num);
      den = __fmaf_rn(sm.l[s][g], f, den);
    }
    if (nb == 1) {
      a.out[(size_t)(g_kv * G + g) * HD + d] = __float2half_rn(__fdiv_rn(num, den));
    } else {
      part[g * stride + 2 + d] = num;
      if (d == 0) {
        part[g * stride] = M;
        part[g * stride + 1] = den;
      }
    }
  }
  if (nb == 1) return;
  // Release: the barrier orders every thread's partial stores before thread
  // 0's fence, which orders them before its arrival.
  __syncthreads();
  if (threadIdx.x == 0) {
    __threadfence();
    sm.last = atomicAdd(a.counters + g_kv, 1u) == (uint32_t)nb - 1;
  }
  __syncthreads();
  if (!sm.last) return;
  __threadfence();
  // Block merge in index order, staged through shared memory: the K/V tile
  // buffers (free now) take the records of up to `chunk` blocks at a time,
  // copied by every thread with 16-byte cp.async (one L2 round trip per
  // chunk). The arithmetic is the sequential merge: M = the max of the block
  // maxima (exact in any order), then per block f = exp(m - M) and
  // den / num = fma(l / acc, f, den / num) in block order.
  const float* base = a.scratch + (size_t)g_kv * gridDim.x * G * stride;
  float* buf = reinterpret_cast<float*>(&sm.tile[0]);      // the reserved K/V tiles
  const int buf_floats =
      (int)((a.block > kTile ? 2 : 1) * sizeof(DecodeTile) / sizeof(float));
  constexpr int kRec = G * (HD + 2);                        // floats of one block record
  // two halves: chunk c + 1 streams into one while chunk c is merged from the other
  const int half = buf_floats / 2 / 4 * 4;
  const int kChunk = (half - 3) / kRec;                     // blocks per staged chunk
  float* fs = &sm.acc[0][0][0];                             // [kChunk][G] merge factors
  static_assert((2 * sizeof(DecodeTile) / sizeof(float) - 3) / kRec * G <= kStreams * G * HD,
                "factor buffer");
  // Chunk `ci` (blocks [ci * kChunk, +cnt)) into half `hb`: 16-byte cp.async
  // for the aligned middle, plain loads for a misaligned head and the tail.
  auto issue = [&](int ci, int hb) -> float* {
    const int s0 = ci * kChunk;
    const int cnt = min(kChunk, nb - s0);
    const float* src = base + (size_t)s0 * kRec;
    const int n = cnt * kRec;
    const int head = (int)((4 - ((reinterpret_cast<uintptr_t>(src) >> 2) & 3)) & 3);
    const int h = min(n, head);
    float* stage = buf + hb * half + ((4 - h) & 3);  // stage + h is 16-byte aligned
    const int n4 = (n - h) >> 2;
    for (int i2 = threadIdx.x; i2 < n4; i2 += kDecodeThreads)
      pipe::cp_async16(stage + h + 4 * i2, src + h + 4 * i2);
    pipe::cp_async_commit();
    if (threadIdx.x < h) stage[threadIdx.x] = __ldcg(src + threadIdx.x);
    const int t0 = h + 4 * n4;
    if (threadIdx.x < n - t0) stage[t0 + threadIdx.x] = __ldcg(src + t0 + threadIdx.x);
    return stage;
  };
  const int nchunks = (nb + kChunk - 1) / kChunk;
  float* stage_a = issue(0, 0);  // the chunk staged in half 0 / half 1
  float* stage_b = nullptr;
  // M per head of the group (sm.m[0][g]).
  {
    float mloc[G];
#pragma unroll
    for (int g = 0; g < G; ++g) mloc[g] = -INFINITY;
    for (int s0 = threadIdx.x * 8; s0 < nb; s0 += kDecodeThreads * 8) {
#pragma unroll
      for (int u = 0; u < 8; ++u) {
        if (s0 + u < nb) {
#pragma unroll
          for (int g = 0; g < G; ++g)
            mloc[g] = fmaxf(mloc[g], __ldcg(base + (size_t)((s0 + u) * G + g) * stride));
        }
      }
    }
#pragma unroll
    for (int g = 0; g < G; ++g) {
      float v = mloc[g];
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
      if (lane == 0) sm.l[warp][g] = v;
    }
    __syncthreads();
    if (threadIdx.x < G) {
      float v = sm.l[0][threadIdx.x];
#pragma unroll
      for (int w = 1; w < kDecodeThreads / 32; ++w) v = fmaxf(v, sm.l[w][threadIdx.x]);
      sm.m[0][threadIdx.x] = v;
    }
    __syncthreads();
  }
  float num[G], den = 0.f;  // thread t: element t of each head g (t < 128 = HD)
#pragma unroll
  for (int g = 0; g < G; ++g) num[g] = 0.f;
  static_assert(kDecodeThreads == HD, "one thread per head dimension");
  const int d = threadIdx.x;
  for (int ci = 0; ci < nchunks; ++ci) {
    const int cnt = min(kChunk, nb - ci * kChunk);
    if (ci + 1 < nchunks) {
      if ((ci + 1) & 1)
        stage_b = issue(ci + 1, 1);
      else
        stage_a = issue(ci + 1, 0);
      asm volatile("cp.async.wait_group 1;" ::: "memory");
    } else {
      pipe::cp_async_wait_all();
    }
    __syncthreads();
    const float* stage = (ci & 1) ? stage_b : stage_a;
    for (int i2 = threadIdx.x; i2 < cnt * G; i2 += kDecodeThreads) {
      const int g = i2 % G;
      const float mm = stage[i2 * (HD + 2)];
      fs[i2] = mm == -INFINITY ? 0.f : mi_exp(__fsub_rn(mm, sm.m[0][g]));
    }
    __syncthreads();
    // The chains read their operands kMB blocks at a time, loads first.
    constexpr int kMB = G >= 4 ? 4 : 8;
    if (threadIdx.x < G) {
      const int g = threadIdx.x;
      for (int u0 = 0; u0 < cnt; u0 += kMB) {
        float lv[kMB], fv[kMB];
#pragma unroll
        for (int e = 0; e < kMB; ++e) {
          const int u = min(u0 + e, cnt - 1);
          lv[e] = stage[(u * G + g) * (HD + 2) + 1];
          fv[e] = fs[u * G + g];
        }
#pragma unroll
        for (int e = 0; e < kMB; ++e)
          if (u0 + e < cnt) den = __fmaf_rn(lv[e], fv[e], den);
      }
    }
    for (int u0 = 0; u0 < cnt; u0 += kMB) {
      float sv[G][kMB], fv[G][kMB];
#pragma unroll
      for (int g = 0; g < G; ++g)
#pragma unroll
        for (int e = 0; e < kMB; ++e) {
          const int u = min(u0 + e, cnt - 1);
          sv[g][e] = stage[(u * G + g) * (HD + 2) + 2 + d];
          fv[g][e] = fs[u * G + g];
        }
#pragma unroll
      for (int g = 0; g < G; ++g)
#pragma unroll
        for (int e = 0; e < kMB; ++e)
          if (u0 + e < cnt) num[g] = __fmaf_rn(sv[g][e], fv[g][e], num[g]);
    }
    __syncthreads();
  }
  if (threadIdx.x < G) sm.l[0][threadIdx.x] = den;
  __syncthreads();
#pragma unroll
  for (int g = 0; g < G; ++g)
    a.out[(size_t)(g_kv * G + g) * HD + d] = __float2half_rn(__fdiv_rn(num[g], sm.l[0][g]));
  if (threadIdx.x == 0) a.counters[g_kv] = 0u;
}

template <int G>
void launch_decode_g(const Launch& l, const DecodeArgs& a, int blocks) {
  auto kernel = attention_decode_kernel<G>;
  const size_t smem = decode_smem_bytes<G>(a.block > kTile);
  allow_dynamic_smem(kernel, decode_smem_bytes<G>(true));  // the largest layout
  launch_kernel(l, dim3(blocks, a.kvh), dim3(kDecodeThreads), smem, kernel, a);
}

void launch_decode(const Launch& l, const DecodeArgs& args, int blocks) {
  DecodeArgs a = args;
  a.early = l.early ? 1 : 0;
  switch (a.qh / a.kvh) {
    case 1: launch_decode_g<1>(l, a, blocks); break;
    case 2: launch_decode_g<2>(l, a, blocks); break;
    case 4: launch_decode_g<4>(l, a, blocks); break;
    case 8: launch_decode_g<8>(l, a, blocks); break;
    default: fail(MI_ERR_SHAPE, "decode attention supports GQA ratios 1, 2, 4 and 8");
  }
}

// ---- prefill ------------------------------------------------------------------------
// One warp per query row; the 4 warps of a CTA take 4 consecutive queries of
// one head and share 32-key K/V tiles in shared memory (rows padded by 16
// bytes). Lane j scores key j with the canonical DOT computed in-thread.
constexpr int kPrefillWarps = 4;

template <int D>
__global__ void __launch_bounds__(kPrefillWarps * 32) attention_prefill_kernel(AttnProblem p) {
  constexpr int kPad = D * 2 + 16;  // bytes per staged row
  __shared__ __align__(16) uint8_t ks[32 * kPad];
  __shared__ __align__(16) uint8_t vs[32 * kPad];
  __shared__ float qs[kPrefillWarps][D];
  const int lane = threadIdx.x & 31;
  const int warp = threadIdx.x >> 5;
  const int h = blockIdx.y;
  const int kvh = h / (p.qh / p.kvh);
  const int q0 = blockIdx.x * kPrefillWarps;
  const int qi = q0 + warp;
  pdl_wait();
  const int L = kv_len_of(p);
  const int last_q = min(p.tokens, q0 + kPrefillWarps) - 1;
  const int limit = p.causal ? min(L, p.query_offset + last_q + 1) : L;
  const bool active = qi < p.tokens;
  const int available = active ? (p.causal ? min(L, p.query_offset + qi + 1) : L) : 0;
  if (active)
    for (int d = lane; d < D; d += 32) qs[warp][d] = __half2float(p.q[((size_t)qi * p.qh + h) * D + d]);
  const size_t stride = (size_t)p.kvh * D;
  const float scale = __frcp_rn(__fsqrt_rn((float)D));
  constexpr int E = (D + 31) / 32;
  float acc[E];
#pragma unroll
  for (int i = 0; i < E; ++i) acc[i] = 0.f;
  float row_max = -INFINITY, row_sum = 0.f;
  for (int base = 0; base < limit; base += 32) {
    const int count = min(32, limit - base);
    __syncthreads();
    for (int i = threadIdx.x; i < count * (D / 8); i += kPrefillWarps * 32) {
      int r = i / (D / 8), c = i - r * (D / 8);
      const size_t src = (size_t)(base + r) * stride + (size_t)kvh * D + 8 * c;
      *reinterpret_cast<uint4*>(ks + r * kPad + 16 * c) = *reinterpret_cast<const uint4*>(p.k + src);
      *reinterpret_cast<uint4*>(vs + r * kPad + 16 * c) = *reinterpret_cast<const uint4*>(p.v + src);
    }
    __syncthreads();
    if (base >= available) continue;
    const int valid_n = min(32, available - base);
    const bool valid = lane < valid_n;
    float s = -INFINITY;
    if (valid)
      s = __fmul_rn(canon_dot_thread<D>(qs[warp], reinterpret_cast<const uint4*>(ks + lane * kPad)),
                    scale);
    float block_max = warp_max(s);
    float next_max = fmaxf(row_max, block_max);
    float alpha = isinf(row_max) ? 0.f : mi_exp(__fsub_rn(row_max, next_max));
    float w = valid ? mi_exp(__fsub_rn(s, next_max)) : 0.f;
    float block_sum = canon_butterfly(w, 32);
    float prob = p.round_p ? __half2float(__float2half_rn(w)) : w;
    row_sum = __fmaf_rn(row_sum, alpha, block_sum);
    row_max = next_max;
#pragma unroll
    for (int i = 0; i < E; ++i) acc[i] = __fmul_rn(acc[i], alpha);
    for (int c = 0; c < valid_n; ++c) {
      float pc = __shfl_sync(0xffffffffu, prob, c);
      const __half* vr = reinterpret_cast<const __half*>(vs + c * kPad);
#pragma unroll
      for (int i = 0; i < E; ++i) {
        int d = lane + i * 32;
        if (d < D) acc[i] = __fmaf_rn(pc, __half2float(vr[d]), acc[i]);
      }
    }
  }
  if (!active) return;
#pragma unroll
  for (int i = 0; i < E; ++i) {
    int d = lane + i * 32;
    if (d < D) p.out[((size_t)qi * p.qh + h) * D + d] = __float2half_rn(__fdiv_rn(acc[i], row_sum));
  }
}

// Any head_dim <= 256 (test shapes): direct global reads, same arithmetic.
__global__ void attention_prefill_scalar_kernel(AttnProblem p) {
  const int lane = threadIdx.x & 31;
  const int row = blockIdx.x * (blockDim.x / 32) + (threadIdx.x >> 5);
  pdl_wait();
  if (row >= p.tokens * p.qh) return;
  const int qi = row / p.qh, h = row - (row / p.qh) * p.qh;
  const int kvh = h / (p.qh / p.kvh);
  const int L = kv_len_of(p);
  const int available = p.causal ? min(L, p.query_offset + qi + 1) : L;
  const int hd = p.hd;
  const size_t stride = (size_t)p.kvh * hd;
  const float scale = __frcp_rn(__fsqrt_rn((float)hd));
  const __half* q = p.q + (size_t)row * hd;
  const int lanes = canon_lanes(hd);
  const int chunks = (hd + 7) / 8;
  float acc[8];
#pragma unroll
  for (int i = 0; i < 8; ++i) acc[i] = 0.f;
  float row_max = -INFINITY, row_sum = 0.f;
  for (int base = 0; base < available; base += 32) {
    const int valid_n = min(32, available - base);
    const bool valid = lane < valid_n;
    float s = -INFINITY;
    if (valid) {
      const __half* kr = p.k + (size_t)(base + lane) * stride + (size_t)kvh * hd;
      float v[32];
      for (int c = 0; c < 32; ++c) v[c] = 0.f;
      for (int c = 0; c < chunks; ++c)
        for (int i = 8 * c; i < min(hd, 8 * c + 8); ++i)
          v[c % lanes] = __fmaf_rn(__half2float(q[i]), __half2float(kr[i]), v[c % lanes]);
      for (int step = lanes / 2; step >= 1; step /= 2)
        for (int t = 0; t < step; ++t) v[t] = __fadd_rn(v[t], v[t + step]);
      s = __fmul_rn(v[0], scale);
    }
    float block_max = warp_max(s);
    float next_max = fmaxf(row_max, block_max);
    float alpha = isinf(row_max) ? 0.f : mi_exp(__fsub_rn(row_max, next_max));
    float w = valid ? mi_exp(__fsub_rn(s, next_max)) : 0.f;
    float block_sum = canon_butterfly(w, 32);
    float prob = p.round_p ? __half2float(__float2half_rn(w)) : w;
    row_sum = __fmaf_rn(row_sum, alpha, block_sum);
    row_max = next_max;
#pragma unroll
    for (int i = 0; i < 8; ++i) acc[i] = __fmul_rn(acc[i], alpha);
    for (int c = 0; c < valid_n; ++c) {
      float pc = __shfl_sync(0xffffffffu, prob, c);
      const __half* vr = p.v + (size_t)(base + c) * stride + (size_t)kvh * hd;
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        int d = lane + i * 32;
        if (d < hd) acc[i] = __fmaf_rn(pc, __half2float(vr[d]), acc[i]);
      }
    }
  }
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    int d = lane + i * 32;
    if (d < hd) p.out[(size_t)row * hd + d] = __float2half_rn(__fdiv_rn(acc[i], row_sum));
  }
}

}  // namespace

void attention_reference(const Launch& l, const AttnProblem& p) {
  dim3 grid((p.hd + 127) / 128, p.qh, p.tokens);
  launch_kernel(l, grid, dim3(128), 0, attention_reference_kernel, p);
}

int decode_block_for(int capacity) {
  if (capacity <= 8192) return 64;
  int b = 64;
  while ((long long)b * 128 < capacity) b <<= 1;
  return b;
}

size_t attention_decode_scratch(int kvh, int blocks, int group, int hd) {
  return (size_t)kvh * blocks * group * (hd + 2) * sizeof(float);
}

int attention_decode_splits(int kv_len_max, int kvh, int sm_count, int block_keys) {
  (void)kvh;
  (void)sm_count;
  int b = (kv_len_max + block_keys - 1) / block_keys;
  return b < 1 ? 1 : b;
}

void attention_decode(const Launch& l, const AttnProblem& p, int splits, int block_keys,
                      float* scratch, uint32_t* counters) {
  const bool aligned =
      ((reinterpret_cast<uintptr_t>(p.q) | reinterpret_cast<uintptr_t>(p.k) |
        reinterpret_cast<uintptr_t>(p.v)) & 15) == 0;
  if (!aligned || p.hd != 128 || (p.qh / p.kvh) > 8 ||
      ((p.qh / p.kvh) & ((p.qh / p.kvh) - 1)) || block_keys % 8 ||
      (block_keys > kTile && block_keys % kTile)) {
    attention_reference(l, p);
    return;
  }
  DecodeArgs a = {};
  a.q = p.q;
  a.k_cache = p.k;
  a.v_cache = p.v;
  a.qh = p.qh;
  a.kvh = p.kvh;
  const int L = p.kv_len;
  a.length = p.causal && p.query_offset < L ? p.query_offset + 1 : L;
  a.block = block_keys;
  a.out = p.out;
  a.scratch = scratch;
  a.counters = counters;
  launch_decode(l, a, splits);
}

void attention_decode_fused(const Launch& l, const DecodeFused& p, int splits, float* scratch,
                            uint32_t* counters, int block_keys) {
  MI_REQUIRE(p.hd == 128, MI_ERR_SHAPE, "fused decode attention needs head_dim 128");
  DecodeArgs a = {};
  a.q = p.q_raw;
  a.k_cache = p.key_cache;
  a.v_cache = p.value_cache;
  a.k_cache_w = p.key_cache;
  a.v_cache_w = p.value_cache;
  a.qh = p.qh;
  a.kvh = p.kvh;
  a.length_dev = p.pos.dev;
  a.block = block_keys;
  a.out = p.out;
  a.scratch = scratch;
  a.counters = counters;
  a.fused = 1;
  a.k_raw = p.k_raw;
  a.v_raw = p.v_raw;
  a.q_norm = p.q_norm;
  a.k_norm = p.k_norm;
  a.theta = p.theta;
  a.eps = p.eps;
  a.round_norm = p.round_norm ? 1 : 0;
  a.rope = p.rope;
  launch_decode(l, a, splits);
}

void attention_prefill(const Launch& l, const AttnProblem& p) {
  MI_REQUIRE(p.hd <= 256, MI_ERR_SHAPE, "prefill attention needs head_dim <= 256");
  if (p.tokens * p.qh <= 0) return;
  if (attention_prefill_mma(l, p)) return;  // long prompts: tensor cores
  dim3 grid((p.tokens + kPrefillWarps - 1) / kPrefillWarps, p.qh);
  dim3 block(kPrefillWarps * 32);
  const bool aligned =
      ((reinterpret_cast<uintptr_t>(p.k) | reinterpret_cast<uintptr_t>(p.v)) & 15) == 0;
  switch (aligned ? p.hd : 0) {
    case 64: launch_kernel(l, grid, block, 0, attention_prefill_kernel<64>, p); return;
    case 128: launch_kernel(l, grid, block, 0, attention_prefill_kernel<128>, p); return;
    case 256: launch_kernel(l, grid, block, 0, attention_prefill_kernel<256>, p); return;
    default: break;
  }
  int rows = p.tokens * p.qh;
  launch_kernel(l, dim3((rows + 3) / 4), dim3(128), 0, attention_prefill_scalar_kernel, p);
}

unsigned attention_status(bool reset) { return pipe::read_status(reset); }

// ---- flash decode without allocation ------------------------------------------------
// Some callers cannot allocate device memory at the point of the call: hosts
// that reserve the whole device for their own memory pool up front (a
// cudaMalloc there fails or fragments the pool), and latency-critical loops
// where cudaMalloc / cudaFree would stall because they synchronize the
// device. For them, mi_attention_flash_decode_noalloc runs the flash-decode
// kernel with its scratch (per-block softmax partials and per-KV-head merge
// counters) in this file-scope device array instead of allocated memory.
// Every GPU that loads the library holds the array until the process exits.
namespace {

constexpr size_t kNoAllocPartialBytes = size_t(1) << 20;  // FP32 block partials
constexpr size_t kNoAllocMaxKvHeads = 64;                  // one u32 counter each
constexpr size_t kNoAllocBytes = kNoAllocPartialBytes + kNoAllocMaxKvHeads * sizeof(uint32_t);

static __device__ __align__(256) unsigned char g_noalloc_scratch[kNoAllocBytes];

std::mutex g_noalloc_mutex;
std::vector<std::pair<CUcontext, void*>> g_noalloc_ptr;  // per CUDA context

// Driver entry points through the runtime (the library does not link
// libcuda directly, so that it loads on hosts without a driver). Each is
// requested at the ABI version whose signature is used here: the
// unversioned lookup follows the runtime's version, and from CUDA 12.5 on
// that gives cuStreamGetCtx the three-argument form of cuStreamGetCtx_v2.
template <typename F>
F driver_fn(const char* name, unsigned version) {
  void* f = nullptr;
  cudaDriverEntryPointQueryResult q;
  if (cudaGetDriverEntryPointByVersion(name, &f, version, cudaEnableDefault, &q) != cudaSuccess ||
      q != cudaDriverEntryPointSuccess || !f)
    fail(MI_ERR_RESOURCE, "driver entry point %s (ABI %u) is unavailable", name, version);
  return reinterpret_cast<F>(f);
}
CUresult ctx_get_current(CUcontext* c) {
  static const PFN_cuCtxGetCurrent_v4000 fn =
      driver_fn<PFN_cuCtxGetCurrent_v4000>("cuCtxGetCurrent", 4000);
  return fn(c);
}
CUresult stream_get_ctx(CUstream s, CUcontext* c) {
  static const PFN_cuStreamGetCtx_v9020 fn =
      driver_fn<PFN_cuStreamGetCtx_v9020>("cuStreamGetCtx", 9020);
  return fn(s, c);
}

// Device address of the scratch array in the current CUDA context, looked up
// once per context (the array's host-side name is not a device address; the
// module, and so the address, belongs to a context, not to a device ordinal).
// Returns the context too, so that the caller can check its stream against it.
void* noalloc_scratch(CUcontext* ctx_out) {
  std::lock_guard<std::mutex> lock(g_noalloc_mutex);
  CUcontext cur = nullptr;
  if (ctx_get_current(&cur) != CUDA_SUCCESS || !cur) {
    // no context current yet: the runtime call below makes the device's
    // primary context current
    void* ptr = nullptr;
    cudaError_t err = cudaGetSymbolAddress(&ptr, g_noalloc_scratch);
    if (err != cudaSuccess || !ptr || ctx_get_current(&cur) != CUDA_SUCCESS || !cur)
      fail(MI_ERR_RESOURCE, "cannot resolve the decode scratch array: %s",
           cudaGetErrorString(err));
  }
  *ctx_out = cur;
  for (const auto& e : g_noalloc_ptr)
    if (e.first == cur) return e.second;
  void* ptr = nullptr;
  cudaError_t err = cudaGetSymbolAddress(&ptr, g_noalloc_scratch);
  if (err != cudaSuccess || !ptr)
    fail(MI_ERR_RESOURCE, "cannot resolve the decode scratch array: %s", cudaGetErrorString(err));
  g_noalloc_ptr.emplace_back(cur, ptr);
  return ptr;
}

}  // namespace

}  // namespace k
}  // namespace mi

extern "C" mi_status mi_attention_flash_decode_noalloc(const void* query, const void* key,
                                                       const void* value, void* out,
                                                       size_t query_heads, size_t kv_heads,
                                                       size_t head_dim, size_t length,
                                                       size_t block_keys, void* stream) {
  using namespace mi;
  using namespace mi::k;
  return guard([&] {
    MI_REQUIRE(query && key && value && out, MI_ERR_INVALID_ARGUMENT,
               "query, key, value and out must be device pointers");
    MI_REQUIRE(((reinterpret_cast<uintptr_t>(query) | reinterpret_cast<uintptr_t>(key) |
                 reinterpret_cast<uintptr_t>(value) | reinterpret_cast<uintptr_t>(out)) & 15) == 0,
               MI_ERR_INVALID_ARGUMENT, "query, key, value and out must be 16-byte aligned");
    MI_REQUIRE(head_dim == 128, MI_ERR_SHAPE, "flash decode without allocation needs head_dim 128");
    MI_REQUIRE(kv_heads > 0 && query_heads % kv_heads == 0, MI_ERR_SHAPE,
               "query_heads must be divisible by kv_heads");
    const size_t group = query_heads / kv_heads;
    MI_REQUIRE(group == 1 || group == 2 || group == 4 || group == 8, MI_ERR_SHAPE,
               "GQA ratio must be 1, 2, 4 or 8");
    MI_REQUIRE(block_keys == 32 || block_keys == 64 || block_keys == 128 || block_keys == 256,
               MI_ERR_SHAPE, "flash decode block size must be 32, 64, 128, or 256");
    MI_REQUIRE(length > 0 && length < 0x7FFFFFFF, MI_ERR_SHAPE, "length must be positive");
    MI_REQUIRE(kv_heads <= kNoAllocMaxKvHeads, MI_ERR_SHAPE,
               "kv_heads %zu exceeds the scratch limit of %zu", kv_heads, kNoAllocMaxKvHeads);
    const size_t blocks = (length + block_keys - 1) / block_keys;
    const size_t partial_bytes = attention_decode_scratch((int)kv_heads, (int)blocks, (int)group,
                                                          (int)head_dim);
    MI_REQUIRE(partial_bytes <= kNoAllocPartialBytes, MI_ERR_SHAPE,
               "kv_heads x blocks x group x 130 x 4 = %zu bytes exceeds the %zu-byte scratch "
               "(lengthen block_keys or split the call)",
               partial_bytes, kNoAllocPartialBytes);
    CUcontext cur = nullptr;
    uint8_t* scratch = static_cast<uint8_t*>(noalloc_scratch(&cur));
    uint32_t* counters = reinterpret_cast<uint32_t*>(scratch + kNoAllocPartialBytes);
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    // The scratch belongs to the current context: a stream of another
    // context (another device) would have the kernel and the counter reset
    // reach this context's array across devices.
    CUcontext stream_ctx = nullptr;
    MI_REQUIRE(stream_get_ctx(reinterpret_cast<CUstream>(s), &stream_ctx) == CUDA_SUCCESS &&
                   stream_ctx == cur,
               MI_ERR_INVALID_ARGUMENT,
               "the stream must belong to the current device's CUDA context");
    // The merge counters must start at zero (the kernel leaves them at zero,
    // but an interrupted earlier call may not have).
    MI_CUDA(cudaMemsetAsync(counters, 0, kv_heads * sizeof(uint32_t), s));
    Launch l;
    l.stream = s;
    l.pdl = false;
    DecodeArgs a = {};
    a.q = static_cast<const __half*>(query);
    a.k_cache = static_cast<const __half*>(key);
    a.v_cache = static_cast<const __half*>(value);
    a.qh = (int)query_heads;
    a.kvh = (int)kv_heads;
    a.length = (int)length;
    a.block = (int)block_keys;
    a.out = static_cast<__half*>(out);
    a.scratch = reinterpret_cast<float*>(scratch);
    a.counters = counters;
    launch_decode(l, a, (int)blocks);
  });
}
