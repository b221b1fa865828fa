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
constexpr uint32_t kSeqTail = 64;  // a tail this short runs on one thread
constexpr uint32_t kBurst = 32;    // one-thread run after an event close to the last
constexpr long long kSat = 1ll << 60;
constexpr long long kTwo52 = 1ll << 52;
constexpr long long kTwo53 = 1ll << 53;

enum PassMode : int { kAdd = 0, kTopP = 1, kSub = 2 };

#ifdef MI_SAMPLE_TRACE
// Diagnostic build only: %globaltimer after each phase of the last draw.
static __device__ unsigned long long g_sample_trace[16];
__device__ __forceinline__ void sample_trace(int i) {
  if (threadIdx.x == 0) {
    unsigned long long t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    g_sample_trace[i] = t;
  }
}
#define MI_SAMPLE_TRACE_AT(i) sample_trace(i)
#else
#define MI_SAMPLE_TRACE_AT(i) ((void)0)
#endif

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
// n * d for n, d >= 0, saturated at kSat (no division: the high half of the
// 128-bit product).
__device__ __forceinline__ long long mul_sat(long long n, long long d) {
  const unsigned long long un = (unsigned long long)n, ud = (unsigned long long)d;
  const unsigned long long lo = un * ud;
  return (__umul64hi(un, ud) != 0 || lo > (unsigned long long)kSat) ? kSat : (long long)lo;
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

// v * 2^k, exact: one multiply by a power of two built from its exponent
// bits when 2^k is a normal double, scalbn otherwise.
__device__ __forceinline__ double times_pow2(double v, int k) {
  if (k >= -1022 && k <= 1023) return v * __longlong_as_double((long long)(k + 1023) << 52);
  return scalbn(v, k);
}

// p / 2^e = m + f: class 0 (f < 1/2), 1 (f > 1/2), 2 (f == 1/2), 3 (too large).
__device__ __forceinline__ void classify(double p, int e, long long& m, int& cls) {
  double x = times_pow2(p, -e);
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
        double thr_t = times_pow2(thr, -e);
        if (thr_t < 0x1p62) {
          long long need = (long long)ceil(thr_t) - T;  // >= 1 since t < thr
          long long jt = (need + d - 1) / d;
          if (jt <= n) {
            T += jt * d;
            t = times_pow2((double)T, e);
            done += (uint32_t)jt;
            pos = done - 1;
            return true;
          }
        }
      }
      T += n * d;
    }
    t = times_pow2((double)T, e);
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
  uint32_t next;
  uint2 seq[kSeqTail];  // groups of a one-thread run, staged
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

// Weight of a group: exp((v - max) * (1 / T)) in FP32 (sample_candidates'
// `(value - max_logit) * inverse_temperature).exp()`), from its key.
struct Weights {
  float max_logit, inv_temperature;
  __device__ __forceinline__ double of(uint32_t key) const {
    return (double)mi_exp(__fmul_rn(__fsub_rn(key_value(key), max_logit), inv_temperature));
  }
};

// Groups [g, limit) by thread 0, in order, from s.t, reading the staged
// copies s.seq[g - g_seq]; stops early at a stop (recorded in s).
__device__ void run_sequential(int mode, uint32_t g, uint32_t limit, uint32_t g_seq,
                               const Weights& w, double thr, Shared& s) {
  double t = s.t;
  for (; g < limit; ++g) {
    const uint2 kc = s.seq[g - g_seq];
    uint32_t pos;
    if (run_steps(t, w.of(kc.x), kc.y, mode, thr, pos)) {
      s.stopped = 1;
      s.stop_group = g;
      s.stop_pos = pos;
      break;
    }
  }
  s.t = t;
}

// One sequential FP64 pass over groups [g_start, ngroups) from t_start.
// Leaves the final value in s.t and a stop (kTopP, kSub) in s.stopped /
// s.stop_group / s.stop_pos. `record` keeps checkpoints (group, value).
// Chunks of kChunk groups are loaded once into registers (key, count,
// weight); the block scans the chunk in the current binade, one thread runs
// the first group that may cross the binade or hold the stop, and the scan
// resumes behind it in the new binade. A short tail (top_k lists) runs on
// one thread from shared memory.
__device__ void run_pass(int mode, double t_start, uint32_t g_start, uint32_t ngroups,
                         const uint2* g_kc, const Weights& w, double thr, bool record,
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
  uint32_t last_event = 0xffffffffu;  // where the previous one-thread run began
  while (g0 < ngroups) {
    if (ngroups - g0 <= kSeqTail) {
      if (tid < ngroups - g0) s.seq[tid] = g_kc[g0 + tid];
      if (record && tid == 0 && s.ckpt_count < kCheckpoints) {
        s.ckpt_group[s.ckpt_count] = g0;
        s.ckpt_t[s.ckpt_count] = s.t;
        ++s.ckpt_count;
      }
      __syncthreads();
      if (tid == 0) run_sequential(mode, g0, ngroups, g0, w, thr, s);
      __syncthreads();
      return;
    }
    const uint32_t chunk_end = min(ngroups, g0 + (uint32_t)kChunk);
    const uint32_t base = g0 + (uint32_t)tid * kPerThread;
    uint2 kc[kPerThread];
    double pw[kPerThread];
#pragma unroll
    for (int j = 0; j < kPerThread; ++j) {
      const uint32_t g = base + j;
      kc[j] = g < chunk_end ? g_kc[g] : make_uint2(0, 0);
      pw[j] = g < chunk_end ? w.of(kc[j].x) : 0.0;
    }
    uint32_t start = g0;  // first group of the chunk still to run
    while (start < chunk_end) {
      const double t = s.t;
      if (record && tid == 0 && s.ckpt_count < kCheckpoints) {
        s.ckpt_group[s.ckpt_count] = start;
        s.ckpt_t[s.ckpt_count] = t;
        ++s.ckpt_count;
      }
      long long T0;
      int e;
      const bool normal = decode(t, T0, e);
      if (tid == 0) s.bad = normal ? 0x7fffffff : (int)start;  // zero / subnormal: one thread
      long long gm[kPerThread];
      int gc[kPerThread];
      Elem acc = identity();
#pragma unroll
      for (int j = 0; j < kPerThread; ++j) {
        const uint32_t g = base + j;
        gm[j] = 0;
        gc[j] = 0;
        if (normal && g >= start && g < chunk_end) {
          classify(pw[j], e, gm[j], gc[j]);
          acc = compose(acc, group_elem(gm[j], gc[j], kc[j].y, sub));
        }
      }
      Elem total;
      const Elem ex = scan_elems(acc, total, s);  // ends with a barrier (s.bad is set)
      int bad = 0x7fffffff;
      long long t_bad = 0;
      if (normal) {
        long long T = apply(T0, ex);
#pragma unroll
        for (int j = 0; j < kPerThread; ++j) {
          const uint32_t g = base + j;
          if (g >= start && g < chunk_end && bad == 0x7fffffff) {
            const long long m = gm[j];
            const int cls = gc[j];
            const long long tend = apply(T, group_elem(m, cls, kc[j].y, sub));
            bool ok;
            if (cls == 3) {
              ok = false;
            } else if (sub) {
              ok = tend >= kTwo52 + 1;
            } else {
              ok = tend + m <= kTwo53 - 1;
              if (ok && mode == kTopP) ok = times_pow2((double)tend, e) < thr;
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
      }
      __syncthreads();
      const int first = s.bad;
      if (first == 0x7fffffff) {
        __syncthreads();  // every thread has read s.bad
        if (tid == 0) s.t = times_pow2((double)apply(T0, total), e);
        start = chunk_end;
        __syncthreads();
        break;
      }
      // One thread runs the group, and, where events come close together
      // (the first binades of a sum), the kBurst groups after it: a block
      // scan per event would cost more there. The owners stage the groups
      // (and, in a binade, the value before the first).
      const uint32_t f = (uint32_t)first;
      const uint32_t len =
          min(chunk_end - f, (last_event != 0xffffffffu && f - last_event <= 64u) ? kBurst : 1u);
      last_event = f;
#pragma unroll
      for (int j = 0; j < kPerThread; ++j)
        if (base + j >= f && base + j < f + len) s.seq[base + j - f] = kc[j];
      if (normal && f >= base && f < base + kPerThread) s.t = times_pow2((double)t_bad, e);
      __syncthreads();
      if (tid == 0) run_sequential(mode, f, f + len, f, w, thr, s);
      __syncthreads();
      const int stopped = s.stopped;
      __syncthreads();
      if (stopped) return;
      start = f + len;
    }
    g0 = chunk_end;
  }
}

__global__ void __launch_bounds__(kThreads, 1)
    sample_kernel(const __half* logits, uint32_t n, uint32_t* hist, uint2* g_kc,
                  const uint32_t* opts, unsigned long long* state, uint32_t* token_out,
                  const uint32_t* token_pos) {
  __shared__ Shared s;
  const int tid = threadIdx.x;
  pdl_wait();
  const float top_p = __uint_as_float(opts[1]);
  const uint32_t top_k = opts[2];
  MI_SAMPLE_TRACE_AT(0);
  if (tid == 0) {
    s.ngroups_written = 0;
    s.result = 0xFFFFFFFFu;
  }

  // 1. Groups in descending key order (the first top_k candidates); the
  //    histogram is cleared for the next draw. Thread t owns the block of 64
  //    keys below 65536 - 64 t: its coarse count, then (for the blocks before
  //    the top_k cut) its 64 bins, scanned twice (candidates, groups).
  const unsigned long long cut = top_k > 0 ? (unsigned long long)top_k : ~0ull;
  uint32_t* coarse = hist + kSampleBins;
  const int blk = kSampleBlocks - 1 - tid;
  const uint32_t cblk = coarse[blk];
  unsigned long long tot;
  const unsigned long long c_before = scan_u64(cblk, tot, s);  // ends with a barrier
  const unsigned long long cands_total = tot;
  const bool needed = cblk != 0 && c_before < cut;
  uint4* mine = reinterpret_cast<uint4*>(hist + 64 * blk);  // mine[j]: keys 64 blk + 4j .. + 3
  uint32_t ne = 0;
  if (needed) {
#pragma unroll
    for (int j = 0; j < 16; ++j) {
      const uint4 v = mine[j];
      ne += (v.x != 0) + (v.y != 0) + (v.z != 0) + (v.w != 0);
    }
  }
  const unsigned long long g_before = scan_u64(ne, tot, s);
  const uint32_t groups_total = (uint32_t)tot;
  if (needed) {
    unsigned long long g = g_before, cb = c_before;
    for (int j = 15; j >= 0; --j) {
      const uint4 v = mine[j];
      const uint32_t c[4] = {v.w, v.z, v.y, v.x};  // descending keys
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        if (c[i] == 0) continue;
        if (cb < cut) {
          const unsigned long long keep = cut - cb;
          g_kc[g] = make_uint2((uint32_t)(64 * blk + 4 * j + 3 - i),
                               keep < c[i] ? (uint32_t)keep : c[i]);
          if (keep <= c[i]) s.ngroups_written = (uint32_t)(g + 1);  // the group reaching top_k
        }
        ++g;
        cb += c[i];
      }
    }
  }
  if (cblk != 0) {
#pragma unroll
    for (int j = 0; j < 16; ++j) mine[j] = make_uint4(0, 0, 0, 0);
    coarse[blk] = 0;
  }
  __syncthreads();
  MI_SAMPLE_TRACE_AT(1);
  const uint32_t ngroups = cands_total >= cut ? s.ngroups_written : groups_total;
  if (ngroups == 0) {
    if (tid == 0) token_out[token_pos ? *token_pos : 0] = 0xFFFFFFFFu;
    return;
  }
  Weights w;
  w.max_logit = key_value(g_kc[0].x);
  w.inv_temperature = __uint_as_float(opts[0]);
  MI_SAMPLE_TRACE_AT(2);

  // 3. Total.
  run_pass(kAdd, 0.0, 0, ngroups, g_kc, w, 0.0, true, s);
  double total = s.t;
  MI_SAMPLE_TRACE_AT(3);
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
    run_pass(kTopP, t_start, g_start, ngroups, g_kc, w, thr, false, s);
    if (s.stopped) {  // always, as the full sum reaches the threshold
      kept = s.stop_group + 1;
      if (tid == 0) g_kc[s.stop_group].y = s.stop_pos + 1;
      total = s.t;
    }
    __syncthreads();
  }

  MI_SAMPLE_TRACE_AT(4);
  // 5. XorShift64 draw and the walk.
  __shared__ double s_target;
  if (tid == 0) {
    unsigned long long x = *state;
    x ^= x << 13;
    x ^= x >> 7;
    x ^= x << 17;
    *state = x;
    s_target = __dmul_rn(__ull2double_rn(x) * 0x1p-64, total);
  }
  __syncthreads();
  run_pass(kSub, s_target, 0, kept, g_kc, w, 0.0, false, s);
  MI_SAMPLE_TRACE_AT(5);
  if (!s.stopped) {
    if (tid == 0) token_out[token_pos ? *token_pos : 0] = 0xFFFFFFFEu;
    return;
  }
  const uint32_t key = g_kc[s.stop_group].x;
  const uint32_t want = s.stop_pos;
  const uint32_t bits = key_bits(key);

  // 6. The want-th occurrence (index order) of the chosen value: counts over
  //    contiguous per-thread ranges (loads batched), a block scan, then the
  //    owning thread finds it.
  const uint32_t per = (((n + kThreads - 1) / kThreads) + 7) & ~7u;
  const uint32_t begin = min(n, (uint32_t)tid * per);
  const uint32_t end = min(n, begin + per);
  const uint16_t* lb = reinterpret_cast<const uint16_t*>(logits);
  const bool vec = (reinterpret_cast<uintptr_t>(logits) & 15) == 0;
  uint32_t cnt = 0;
  uint32_t i = begin;
  if (vec) {
    const uint32_t bb = bits | (bits << 16);
    for (; i + 64 <= end; i += 64) {
      uint4 q4[8];
#pragma unroll
      for (int q = 0; q < 8; ++q) q4[q] = *reinterpret_cast<const uint4*>(lb + i + 8 * q);
#pragma unroll
      for (int q = 0; q < 8; ++q) {
        const uint32_t x4[4] = {q4[q].x ^ bb, q4[q].y ^ bb, q4[q].z ^ bb, q4[q].w ^ bb};
#pragma unroll
        for (int r = 0; r < 4; ++r) cnt += ((x4[r] & 0xffffu) == 0) + ((x4[r] >> 16) == 0);
      }
    }
    for (; i + 8 <= end; i += 8) {
      const uint4 q4 = *reinterpret_cast<const uint4*>(lb + i);
      const uint32_t x4[4] = {q4.x ^ bb, q4.y ^ bb, q4.z ^ bb, q4.w ^ bb};
#pragma unroll
      for (int r = 0; r < 4; ++r) cnt += ((x4[r] & 0xffffu) == 0) + ((x4[r] >> 16) == 0);
    }
  }
  for (; i < end; ++i) cnt += lb[i] == bits;
  const unsigned long long before = scan_u64(cnt, tot, s);
  if (want >= before && want < before + cnt) {
    uint32_t left = want - (uint32_t)before;
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
  MI_SAMPLE_TRACE_AT(6);
  if (tid == 0) token_out[token_pos ? *token_pos : 0] = s.result;
}

// Blocks of kHistSeg logits: keys sorted in shared memory, one pair of
// atomics per distinct key (no contention on frequent values).
constexpr int kHistSeg = 256;  // keys per block (smaller sorts: more blocks, fewer stages)
__global__ void __launch_bounds__(256) logit_histogram_kernel(const __half* logits, uint32_t n,
                                                              uint32_t* hist) {
  __shared__ __align__(16) uint16_t keys[kHistSeg + 2048];  // keys, then 1024 block counts
  pdl_wait();
  const int first = (int)(blockIdx.x * kHistSeg);
  hist_add_rows(reinterpret_cast<const uint16_t*>(logits), first,
                (int)min(n, (uint32_t)first + kHistSeg), keys, kHistSeg, hist);
}

}  // namespace

#ifdef MI_SAMPLE_TRACE
extern "C" int mi_debug_sample_trace(unsigned long long* out) {
  return cudaMemcpyFromSymbol(out, g_sample_trace, sizeof(g_sample_trace)) == cudaSuccess ? 0 : -1;
}
#endif

void logit_histogram(const Launch& l, const __half* logits, uint32_t n, uint32_t* hist) {
  const int grid = (int)((n + kHistSeg - 1) / kHistSeg);
  if (grid > 0) launch_kernel(l, dim3(grid), dim3(256), 0, logit_histogram_kernel, logits, n, hist);
}

void sample(const Launch& l, const SampleProblem& p) {
  launch_kernel(l, dim3(1), dim3(kThreads), 0, sample_kernel, p.logits, p.n, p.hist,
                reinterpret_cast<uint2*>(p.groups), p.opts,
                reinterpret_cast<unsigned long long*>(p.state), p.token_out, p.token_pos);
}

}  // namespace k
}  // namespace mi
