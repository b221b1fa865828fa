// On-device sampling: sample_token_f16 + sample_candidates
// (crates/metal-infer-models/src/qwen3.rs:927-1005) with the XorShift64
// stream of qwen3.rs:1011-1034, reproducing the reference's sequential FP64
// arithmetic exactly.
//
// The reference sorts the finite logits by descending value, optionally keeps
// the first top_k, weighs each by exp((v - max) / T) in FP32, sums the weights
// in FP64 in sorted order, optionally cuts the prefix whose running sum first
// reaches total * top_p, then walks `target = u * total` down by the weights
// until it is <= 0. Candidates with the same FP16 value share one weight, so
// the sorted sequence is a list of groups (key, count) read from a 65536-bin
// histogram of the logits' order keys, built by the lm_head GEMV as it writes
// the logits (or by logit_histogram below). Equal bit patterns are ordered by
// ascending index.
//
// The FP64 running sums are order dependent, so they are computed as the
// reference's left-to-right loop, but in parallel: while the running value t
// stays in one binade [2^(e+52), 2^(e+53)), t = T * 2^e with an integer T, and
// one step t +- p rounds to T +- round(p / 2^e): a constant for each group,
// except that a tie (fraction exactly 1/2) rounds to the even neighbour and so
// depends on the parity of T. Each group is therefore a map
// T -> T + D[T mod 2] (two integers), maps compose associatively, and a block
// scan gives the exact running value before every group. A group whose steps
// may leave the binade (or reach a stop) is handed to one thread, which runs
// it with real FP64 steps and jumps over the steady stretches; the scan
// resumes behind it. Runs for the total, the top-p cut and the walk.
#include "device.cuh"
#include "kernels.h"

namespace mi {
namespace k {

namespace {

constexpr int kThreads = 1024;
constexpr int kWarps = kThreads / 32;
constexpr int kPerThread = 4;  // groups per thread per chunk
constexpr int kChunk = kThreads * kPerThread;
constexpr int kCheckpoints = 256;
constexpr long long kSat = 1ll << 60;
constexpr long long kTwo52 = 1ll << 52;
constexpr long long kTwo53 = 1ll << 53;

enum PassMode : int { kAdd = 0, kTopP = 1, kSub = 2 };

// Value of an order key (inverse of sample_key16).
__device__ __forceinline__ float key_value(uint32_t key) {
  uint16_t bits = (key & 0x8000u) ? (uint16_t)(key & 0x7fffu) : (uint16_t)(~key & 0xffffu);
  return __half2float(__ushort_as_half(bits));
}
__device__ __forceinline__ uint16_t key_bits(uint32_t key) {
  return (key & 0x8000u) ? (uint16_t)(key & 0x7fffu) : (uint16_t)(~key & 0xffffu);
}

__device__ __forceinline__ long long sat(long long v) {
  return v > kSat ? kSat : (v < -kSat ? -kSat : v);
}
__device__ __forceinline__ long long mul_sat(long long n, long long d) {
  if (d != 0 && n > kSat / d) return kSat;
  return n * d;
}

// t = T * 2^e with T in [2^52, 2^53); false for zero, subnormal, negative or
// non-finite t.
__device__ __forceinline__ bool decode(double t, long long& T, int& e) {
  unsigned long long b = (unsigned long long)__double_as_longlong(t);
  int be = (int)((b >> 52) & 0x7ff);
  if (be == 0 || be == 0x7ff || (b >> 63)) return false;
  T = (long long)((b & ((1ull << 52) - 1)) | (1ull << 52));
  e = be - 1075;
  return true;
}

// p / 2^e = m + f: class 0 (f < 1/2), 1 (f > 1/2), 2 (f == 1/2), 3 (too large).
__device__ __forceinline__ void classify(double p, int e, long long& m, int& cls) {
  double x = scalbn(p, -e);
  if (!(x < 0x1p62)) {
    m = 0;
    cls = 3;
    return;
  }
  double fm = floor(x);
  m = (long long)fm;
  double f = x - fm;
  cls = f < 0.5 ? 0 : (f > 0.5 ? 1 : 2);
}

// T -> T + d[T & 1].
struct Elem {
  long long d0, d1;
};
__device__ __forceinline__ Elem identity() { return Elem{0, 0}; }
// a, then b.
__device__ __forceinline__ Elem compose(Elem a, Elem b) {
  Elem c;
  c.d0 = sat(a.d0 + ((a.d0 & 1) ? b.d1 : b.d0));
  c.d1 = sat(a.d1 + (((a.d1 + 1) & 1) ? b.d1 : b.d0));
  return c;
}
// `c` steps of one weight in the current binade.
__device__ __forceinline__ Elem group_elem(long long m, int cls, uint32_t c, bool sub) {
  Elem r;
  if (cls == 3) {
    r.d0 = r.d1 = kSat;
  } else if (cls == 2) {
    long long even = m + (m & 1);
    long long rest = mul_sat((long long)c - 1, even);
    r.d0 = sat(rest + ((m & 1) ? m + 1 : m));  // T even: T + m even iff m even
    r.d1 = sat(rest + ((m & 1) ? m : m + 1));
  } else {
    r.d0 = r.d1 = mul_sat((long long)c, m + cls);
  }
  if (sub) {
    r.d0 = -r.d0;
    r.d1 = -r.d1;
  }
  return r;
}
__device__ __forceinline__ long long apply(long long T, const Elem& el) {
  return T + ((T & 1) ? el.d1 : el.d0);
}

// `count` steps of weight p from t, one thread: real FP64 steps where the
// binade may change or a stop may come, closed-form jumps over the steady
// stretches. Returns true at a stop (pos = its step), t updated.
__device__ bool run_steps(double& t, double p, uint32_t count, int mode, double thr,
                          uint32_t& pos) {
  uint32_t done = 0;
  while (done < count) {
    if (mode == kSub) {
      if (t <= p) {
        pos = done;
        t = __dsub_rn(t, p);
        return true;
      }
      t = __dsub_rn(t, p);
    } else {
      t = __dadd_rn(t, p);
      if (mode == kTopP && t >= thr) {
        pos = done;
        return true;
      }
    }
    ++done;
    if (done == count) break;
    long long T, m;
    int e, cls;
    if (!decode(t, T, e)) continue;
    classify(p, e, m, cls);
    if (cls == 3) continue;
    long long d;
    if (cls == 2) {
      if (T & 1) continue;  // the parity-dependent step runs for real
      d = m + (m & 1);
    } else {
      d = m + cls;
    }
    const long long rem = (long long)(count - done);
    long long n;
    if (mode == kSub) {
      // every step exact in the binade while the result stays >= 2^52 + 1
      long long room = T - (kTwo52 + 1);
      if (room < 0) continue;
      n = d == 0 ? rem : min(rem, room / d);
      if (n <= 0) continue;
      T -= n * d;
    } else {
      // step j is exact in the binade while T_(j-1) + p / 2^e < 2^53
      long long room = (kTwo53 - 1) - T - m;
      if (room < 0) continue;
      n = d == 0 ? rem : min(rem, room / d + 1);
      if (mode == kTopP && d > 0) {
        double thr_t = scalbn(thr, -e);
        if (thr_t < 0x1p62) {
          long long need = (long long)ceil(thr_t) - T;  // >= 1 since t < thr
          long long jt = (need + d - 1) / d;
          if (jt <= n) {
            T += jt * d;
            t = scalbn((double)T, e);
            done += (uint32_t)jt;
            pos = done - 1;
            return true;
          }
        }
      }
      T += n * d;
    }
    t = scalbn((double)T, e);
    done += (uint32_t)n;
  }
  pos = count;
  return false;
}

struct Shared {
  Elem warp_elem[kWarps];
  unsigned long long warp_u64[kWarps];
  double t;
  long long t_bad;
  int bad;
  int stopped;
  uint32_t stop_group, stop_pos;
  uint32_t ngroups_written;
  uint32_t ckpt_count;
  uint32_t ckpt_group[kCheckpoints];
  double ckpt_t[kCheckpoints];
  uint32_t result;
};

// Exclusive block scan of composable elements; `total` gets the whole block's.
__device__ Elem scan_elems(Elem x, Elem& total, Shared& s) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  Elem inc = x;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    Elem y;
    y.d0 = __shfl_up_sync(0xffffffffu, inc.d0, o);
    y.d1 = __shfl_up_sync(0xffffffffu, inc.d1, o);
    if (lane >= o) inc = compose(y, inc);
  }
  if (lane == 31) s.warp_elem[warp] = inc;
  __syncthreads();
  if (warp == 0) {
    Elem w = s.warp_elem[lane];
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      Elem y;
      y.d0 = __shfl_up_sync(0xffffffffu, w.d0, o);
      y.d1 = __shfl_up_sync(0xffffffffu, w.d1, o);
      if (lane >= o) w = compose(y, w);
    }
    s.warp_elem[lane] = w;
  }
  __syncthreads();
  Elem ex;
  ex.d0 = __shfl_up_sync(0xffffffffu, inc.d0, 1);
  ex.d1 = __shfl_up_sync(0xffffffffu, inc.d1, 1);
  if (lane == 0) ex = identity();
  if (warp > 0) ex = compose(s.warp_elem[warp - 1], ex);
  total = s.warp_elem[kWarps - 1];
  __syncthreads();
  return ex;
}

// Exclusive block scan of u64 sums; `total` gets the block sum.
__device__ unsigned long long scan_u64(unsigned long long x, unsigned long long& total,
                                       Shared& s) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  unsigned long long inc = x;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    unsigned long long y = __shfl_up_sync(0xffffffffu, inc, o);
    if (lane >= o) inc += y;
  }
  if (lane == 31) s.warp_u64[warp] = inc;
  __syncthreads();
  if (warp == 0) {
    unsigned long long w = s.warp_u64[lane];
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      unsigned long long y = __shfl_up_sync(0xffffffffu, w, o);
      if (lane >= o) w += y;
    }
    s.warp_u64[lane] = w;
  }
  __syncthreads();
  unsigned long long ex = inc - x;
  if (warp > 0) ex += s.warp_u64[warp - 1];
  total = s.warp_u64[kWarps - 1];
  __syncthreads();
  return ex;
}

// One sequential FP64 pass over groups [g_start, ngroups) from t_start.
// Leaves the final value in s.t and a stop (kTopP, kSub) in s.stopped /
// s.stop_group / s.stop_pos. `record` keeps chunk-start checkpoints.
__device__ void run_pass(int mode, double t_start, uint32_t g_start, uint32_t ngroups,
                         const uint32_t* g_count, const float* g_p, double thr, bool record,
                         Shared& s) {
  const int tid = threadIdx.x;
  if (tid == 0) {
    s.t = t_start;
    s.stopped = 0;
    if (record) s.ckpt_count = 0;
  }
  __syncthreads();
  const bool sub = mode == kSub;
  uint32_t g0 = g_start;
  while (g0 < ngroups) {
    const double t = s.t;
    if (record && tid == 0 && s.ckpt_count < kCheckpoints) {
      s.ckpt_group[s.ckpt_count] = g0;
      s.ckpt_t[s.ckpt_count] = t;
      ++s.ckpt_count;
    }
    long long T0;
    int e;
    if (!decode(t, T0, e)) {
      // zero or subnormal running value: one group by real steps
      if (tid == 0) {
        double tt = t;
        uint32_t pos;
        if (run_steps(tt, (double)g_p[g0], g_count[g0], mode, thr, pos)) {
          s.stopped = 1;
          s.stop_group = g0;
          s.stop_pos = pos;
        }
        s.t = tt;
      }
      __syncthreads();
      if (s.stopped) return;
      ++g0;
      continue;
    }
    if (tid == 0) s.bad = 0x7fffffff;
    const uint32_t base = g0 + (uint32_t)tid * kPerThread;
    Elem acc = identity();
#pragma unroll
    for (int j = 0; j < kPerThread; ++j) {
      uint32_t g = base + j;
      if (g < ngroups) {
        long long m;
        int cls;
        classify((double)g_p[g], e, m, cls);
        acc = compose(acc, group_elem(m, cls, g_count[g], sub));
      }
    }
    Elem total;
    Elem ex = scan_elems(acc, total, s);  // ends with a barrier (s.bad is set)
    long long T = apply(T0, ex);
    int bad = 0x7fffffff;
    long long t_bad = 0;
#pragma unroll
    for (int j = 0; j < kPerThread; ++j) {
      uint32_t g = base + j;
      if (g < ngroups && bad == 0x7fffffff) {
        long long m;
        int cls;
        classify((double)g_p[g], e, m, cls);
        long long tend = apply(T, group_elem(m, cls, g_count[g], sub));
        bool ok;
        if (cls == 3) {
          ok = false;
        } else if (sub) {
          ok = tend >= kTwo52 + 1;
        } else {
          ok = tend + m <= kTwo53 - 1;
          if (ok && mode == kTopP) ok = scalbn((double)tend, e) < thr;
        }
        if (!ok) {
          bad = (int)g;
          t_bad = T;
        } else {
          T = tend;
        }
      }
    }
    if (bad != 0x7fffffff) atomicMin(&s.bad, bad);
    __syncthreads();
    const int first = s.bad;
    if (first != 0x7fffffff && bad == first) s.t_bad = t_bad;
    __syncthreads();
    if (first == 0x7fffffff) {
      if (tid == 0) s.t = scalbn((double)apply(T0, total), e);
      g0 = min(ngroups, g0 + (uint32_t)kChunk);
    } else {
      if (tid == 0) {
        double tt = scalbn((double)s.t_bad, e);
        uint32_t pos;
        if (run_steps(tt, (double)g_p[first], g_count[first], mode, thr, pos)) {
          s.stopped = 1;
          s.stop_group = (uint32_t)first;
          s.stop_pos = pos;
        }
        s.t = tt;
      }
      g0 = (uint32_t)first + 1;
    }
    __syncthreads();
    if (s.stopped) return;
  }
}

__global__ void __launch_bounds__(kThreads, 1)
    sample_kernel(const __half* logits, uint32_t n, uint32_t* hist, uint32_t* g_key,
                  uint32_t* g_count, float* g_p, const uint32_t* opts,
                  unsigned long long* state, uint32_t* token_out, const uint32_t* token_pos) {
  __shared__ Shared s;
  const int tid = threadIdx.x;
  pdl_wait();
  const float inv_temperature = __uint_as_float(opts[0]);
  const float top_p = __uint_as_float(opts[1]);
  const uint32_t top_k = opts[2];
  if (tid == 0) {
    s.ngroups_written = 0;
    s.result = 0xFFFFFFFFu;
  }
  __syncthreads();

  // 1. Groups in descending key order (first top_k candidates), histogram
  //    cleared for the next use.
  const unsigned long long cut = top_k > 0 ? (unsigned long long)top_k : ~0ull;
  unsigned long long groups_before = 0, cands_before = 0;
  bool cut_done = false;
  for (int r = 0; r < 16; ++r) {
    const int hi = 65535 - 4096 * r - 4 * tid;  // this thread: keys hi, hi-1, hi-2, hi-3
    uint4* slot = reinterpret_cast<uint4*>(hist + (hi - 3));
    if (!cut_done) {
      uint4 v = *slot;
      uint32_t c[4] = {v.w, v.z, v.y, v.x};
      uint32_t ne = 0;
      unsigned long long cc = 0;
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        ne += c[i] != 0;
        cc += c[i];
      }
      unsigned long long tot;
      unsigned long long ex = scan_u64((cc << 13) | ne, tot, s);
      unsigned long long g = groups_before + (ex & 0x1fff);
      unsigned long long cb = cands_before + (ex >> 13);
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        if (c[i] == 0) continue;
        if (cb < cut) {
          unsigned long long keep = cut - cb;
          g_key[g] = (uint32_t)(hi - i);
          g_count[g] = keep < c[i] ? (uint32_t)keep : c[i];
          atomicMax(&s.ngroups_written, (uint32_t)(g + 1));
        }
        ++g;
        cb += c[i];
      }
      groups_before += tot & 0x1fff;
      cands_before += tot >> 13;
      cut_done = cands_before >= cut;
    }
    *slot = make_uint4(0, 0, 0, 0);
  }
  __syncthreads();
  const uint32_t ngroups = s.ngroups_written;
  if (ngroups == 0) {
    if (tid == 0) token_out[token_pos ? *token_pos : 0] = 0xFFFFFFFFu;
    return;
  }

  // 2. Weights exp((v - max) * (1 / T)) in FP32.
  const float max_logit = key_value(g_key[0]);
  for (uint32_t g = tid; g < ngroups; g += kThreads)
    g_p[g] = mi_exp(__fmul_rn(__fsub_rn(key_value(g_key[g]), max_logit), inv_temperature));
  __syncthreads();

  // 3. Total.
  run_pass(kAdd, 0.0, 0, ngroups, g_count, g_p, 0.0, true, s);
  double total = s.t;
  uint32_t kept = ngroups;

  // 4. Top-p: the prefix whose running sum first reaches total * top_p, from
  //    the last checkpoint of the total pass below the threshold.
  if (top_p < 1.0f) {
    const double thr = total * (double)top_p;
    uint32_t g_start = 0;
    double t_start = 0.0;
    for (uint32_t i = 1; i < s.ckpt_count; ++i)
      if (s.ckpt_t[i] < thr) {
        g_start = s.ckpt_group[i];
        t_start = s.ckpt_t[i];
      }
    __syncthreads();
    run_pass(kTopP, t_start, g_start, ngroups, g_count, g_p, thr, false, s);
    if (s.stopped) {  // always, as the full sum reaches the threshold
      kept = s.stop_group + 1;
      if (tid == 0) g_count[s.stop_group] = s.stop_pos + 1;
      total = s.t;
    }
    __syncthreads();
  }

  // 5. XorShift64 draw and the walk.
  __shared__ double s_target;
  if (tid == 0) {
    unsigned long long v = *state;
    v ^= v << 13;
    v ^= v >> 7;
    v ^= v << 17;
    *state = v;
    s_target = __dmul_rn(__ull2double_rn(v) * 0x1p-64, total);
  }
  __syncthreads();
  run_pass(kSub, s_target, 0, kept, g_count, g_p, 0.0, false, s);
  if (!s.stopped) {
    if (tid == 0) token_out[token_pos ? *token_pos : 0] = 0xFFFFFFFEu;
    return;
  }
  const uint32_t key = g_key[s.stop_group];
  const uint32_t want = s.stop_pos;
  const uint16_t bits = key_bits(key);

  // 6. The want-th occurrence (index order) of the chosen value.
  const uint32_t per = (((n + kThreads - 1) / kThreads) + 7) & ~7u;
  const uint32_t begin = min(n, (uint32_t)tid * per);
  const uint32_t end = min(n, begin + per);
  const uint16_t* lb = reinterpret_cast<const uint16_t*>(logits);
  const bool vec = (reinterpret_cast<uintptr_t>(logits) & 15) == 0;
  uint32_t cnt = 0;
  uint32_t i = begin;
  if (vec) {
    for (; i + 8 <= end; i += 8) {
      uint4 v = *reinterpret_cast<const uint4*>(lb + i);
      const uint32_t w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
      for (int q = 0; q < 4; ++q)
        cnt += ((w[q] & 0xffffu) == bits) + ((w[q] >> 16) == bits);
    }
  }
  for (; i < end; ++i) cnt += lb[i] == bits;
  unsigned long long tot;
  const unsigned long long ex = scan_u64(cnt, tot, s);
  if (want >= ex && want < ex + cnt) {
    uint32_t left = want - (uint32_t)ex;
    for (uint32_t j = begin; j < end; ++j)
      if (lb[j] == bits) {
        if (left == 0) {
          s.result = j;
          break;
        }
        --left;
      }
  }
  __syncthreads();
  if (tid == 0) token_out[token_pos ? *token_pos : 0] = s.result;
}

__global__ void logit_histogram_kernel(const __half* logits, uint32_t n, uint32_t* hist) {
  pdl_wait();
  const uint16_t* lb = reinterpret_cast<const uint16_t*>(logits);
  for (uint32_t i = blockIdx.x * blockDim.x + threadIdx.x; i < n; i += gridDim.x * blockDim.x) {
    uint16_t b = lb[i];
    if ((b & 0x7c00u) != 0x7c00u) atomicAdd(hist + sample_key16(b), 1u);
  }
}

}  // namespace

void logit_histogram(const Launch& l, const __half* logits, uint32_t n, uint32_t* hist) {
  int grid = min(l.sm_count * 4, (int)((n + 255) / 256));
  if (grid < 1) grid = 1;
  launch_kernel(l, dim3(grid), dim3(256), 0, logit_histogram_kernel, logits, n, hist);
}

void sample(const Launch& l, const SampleProblem& p) {
  launch_kernel(l, dim3(1), dim3(kThreads), 0, sample_kernel, p.logits, p.n, p.hist,
                p.groups, p.groups + kSampleBins, reinterpret_cast<float*>(p.groups + 2 * kSampleBins),
                p.opts, reinterpret_cast<unsigned long long*>(p.state), p.token_out,
                p.token_pos);
}

}  // namespace k
}  // namespace mi
