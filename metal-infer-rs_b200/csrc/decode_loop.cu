// Persistent greedy decode: one cooperative launch runs `steps` decode steps
// of the whole Qwen3 model (decode path of qwen3.rs:412-555) with the same
// five fused stages per layer as the per-kernel chain in qwen3.cu, in the
// same arithmetic, so both give bit-identical logits and ids:
//   QKV   (embedding +) RMSNorm + Q/K/V rows        (matvec3_rms_impl)
//   ATTN  QK-norm + RoPE + K/V append + flash decode (qk_norm_rope_cache_f16,
//         copy_kv_f16, attention_flash_decode_f16)
//   O     O rows
//   GU    residual add + RMSNorm + gate/up rows + SwiGLU (matvec2_add_rms_impl)
//   DOWN  down rows + residual add
// then final RMSNorm + LM head + greedy argmax, whose id feeds the next step.
//
// One CTA per SM: 15 consumer warps and one producer warp. The producer
// walks the static schedule of weight tiles this CTA will reduce (every
// stage of every layer of every step, then the LM head) and streams them
// into a ring of shared-memory slots with 1-D bulk copies that complete on
// "full" mbarriers. It is throttled only by the ring ("empty" mbarriers the
// consumer warps arrive on), never by the grid barriers between stages, so
// HBM keeps streaming weights while the consumers wait on their
// predecessors. Consumers build each stage's input vector in shared memory,
// reduce their rows from the ring and write the outputs to global memory
// (L2-resident activations are read with L1-bypassing loads), then meet at a
// grid barrier (a monotonic counter in global memory).
//
// Every wait is bounded in time: a ring wait, a grid-barrier wait or an
// attention merge that gives up records a code in g_loop_status and raises a
// device-wide abort flag; all warps leave at the next stage boundary and the
// producer waits (bounded) for its copies in flight before the CTA exits.

#include <algorithm>

#include "device.cuh"
#include "pipeline.cuh"

namespace mi {
namespace k {

namespace {

constexpr int HD = 128;
constexpr int kConsumerWarps = 15;  // + 1 producer: 512 threads, 128 registers
constexpr int kConsumers = kConsumerWarps * 32;
constexpr int kThreads = kConsumers + 32;  // + producer warp
constexpr int kStreams = 8;
constexpr int kTile = 64;                  // keys staged per attention tile
constexpr int kAttnThreads = 128;          // warps 0..3 run the attention units
constexpr int kMaxSlots = 16;
constexpr int kMinSlotBytes = 32 * 1024;

static __device__ unsigned g_loop_status = 0;

#ifdef MI_DECODE_TRACE
// Diagnostic build only: %globaltimer stamps of the first and last CTA for
// the first two steps: [cta][step][stage][event], events 0..2 = consumer
// thread 0 after the preceding barrier / after the input / after its rows,
// 3..4 = producer issue of the stage's first / last tile.
constexpr int kTraceStages = 5 * 64 + 1;
constexpr int kTraceEvents = 12;
static __device__ unsigned long long g_trace[2][2][kTraceStages][kTraceEvents];
__device__ int g_trace_step, g_trace_stage;  // set by consumer thread 0 of the traced CTAs
__device__ __forceinline__ void trace(int step, int stage, int ev) {
  const int c = blockIdx.x == 0 ? 0 : (blockIdx.x == gridDim.x - 1 ? 1 : -1);
  if (c < 0 || step >= 2 || stage >= kTraceStages) return;
  g_trace[c][step][stage][ev] = pipe::global_ns();
}
#define MI_TRACE(step, stage, ev) trace(step, stage, ev)
#define MI_TRACE_CUR(ev) trace(g_trace_step, g_trace_stage, ev)
#define MI_TRACE_SET(step, stage) (g_trace_step = (step), g_trace_stage = (stage))
#else
#define MI_TRACE(step, stage, ev) ((void)0)
#define MI_TRACE_CUR(ev) ((void)0)
#define MI_TRACE_SET(step, stage) ((void)0)
#endif

enum Stage : int { kQKV = 0, kO = 1, kGU = 2, kDown = 3, kLM = 4 };

// Failure codes (high byte: place, low byte: stage).
constexpr unsigned kCodeFull = 0x0100;
constexpr unsigned kCodeEmpty = 0x0200;
constexpr unsigned kCodeGrid = 0x0300;
constexpr unsigned kCodeDrain = 0x0400;

struct StageW {
  const __half* w[3];
  int n[3];
  int k;      // reduction length
  int items;  // rows (pairs for GU)
  int pair;   // GU: gate and up rows per item
};

__device__ __forceinline__ StageW stage_weights(const DecodeLoop& p, int layer, int st) {
  StageW s = {};
  const LoopLayer* L = p.layer + (layer < p.layers ? layer : 0);
  switch (st) {
    case kQKV:
      s.w[0] = L->wq;
      s.w[1] = L->wk;
      s.w[2] = L->wv;
      s.n[0] = p.qh * HD;
      s.n[1] = s.n[2] = p.kvh * HD;
      s.k = p.hidden;
      s.items = s.n[0] + 2 * s.n[1];
      break;
    case kO:
      s.w[0] = L->wo;
      s.n[0] = p.hidden;
      s.k = p.qh * HD;
      s.items = p.hidden;
      break;
    case kGU:
      s.w[0] = L->gate;
      s.w[1] = L->up;
      s.n[0] = s.n[1] = p.inter;
      s.k = p.hidden;
      s.items = p.inter;
      s.pair = 1;
      break;
    case kDown:
      s.w[0] = L->down;
      s.n[0] = p.hidden;
      s.k = p.inter;
      s.items = p.hidden;
      break;
    default:
      s.w[0] = p.lm_head;
      s.n[0] = p.vocab;
      s.k = p.hidden;
      s.items = p.vocab;
      break;
  }
  return s;
}

struct Tiles {
  int first, last, per_tile, count;
  uint32_t row_bytes;
};

__device__ __forceinline__ Tiles tiles_of(const DecodeLoop& p, const StageW& s) {
  Tiles t;
  t.first = (int)((long long)s.items * blockIdx.x / gridDim.x);
  t.last = (int)((long long)s.items * (blockIdx.x + 1) / gridDim.x);
  t.row_bytes = (uint32_t)s.k * 2u;
  t.per_tile = p.slot_bytes / (int)(t.row_bytes * (s.pair ? 2u : 1u));
  t.count = t.last > t.first ? (t.last - t.first + t.per_tile - 1) / t.per_tile : 0;
  return t;
}

template <int G>
struct AttnSmem {
  __half k[kTile][HD];
  __half v[kTile][HD];
  __half new_k[HD];
  __half new_v[HD];
  float q[G][HD];
  float m[kStreams][G];
  float l[kStreams][G];
  float acc[kStreams][G][HD];
  int last;
};

struct Shared {
  uint64_t full[kMaxSlots];
  uint64_t empty[kMaxSlots];
  float scale;
  uint32_t best_key[kConsumerWarps];
  uint32_t best_idx[kConsumerWarps];
  uint32_t token;
  volatile int abort;
};

__device__ __forceinline__ void consumers_sync() {
  asm volatile("bar.sync 1, %0;" ::"n"(kConsumers) : "memory");
}
__device__ __forceinline__ void attn_sync() {
  asm volatile("bar.sync 2, %0;" ::"n"(kAttnThreads) : "memory");
}

__device__ __forceinline__ uint32_t ld_acquire(const uint32_t* p) {
  uint32_t v;
  asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(pipe::smem_u32(bar)) : "memory");
}

__device__ void record(unsigned code) { atomicCAS(&g_loop_status, 0u, code); }

// Ring wait that gives up on abort or after kWaitNs.
__device__ bool ring_wait(uint64_t* bar, uint32_t parity, Shared& sh, unsigned code) {
  if (pipe::mbar_try_wait(bar, parity)) return true;
  const uint64_t start = pipe::global_ns();
  while (!pipe::mbar_try_wait(bar, parity)) {
    if (sh.abort) return false;
    if (pipe::global_ns() - start > pipe::kWaitNs) {
      record(code);
      sh.abort = 1;
      return false;
    }
  }
  return true;
}

// Grid barrier over all CTAs (consumer threads only). Returns false when the
// kernel is aborting; the decision is uniform across the CTA.
__device__ bool grid_sync(const DecodeLoop& p, uint32_t& epoch, Shared& sh) {
  ++epoch;
  consumers_sync();
  if (threadIdx.x == 0) {
    volatile uint32_t* abort_flag = p.sync + 1;
    if (sh.abort) {
      *abort_flag = 1u;
    } else {
      __threadfence();
      atomicAdd(p.sync, 1u);
      const uint32_t target = epoch * gridDim.x;
      uint64_t start = 0;
      while (ld_acquire(p.sync) < target) {
        if (*abort_flag) {
          sh.abort = 1;
          break;
        }
        const uint64_t now = pipe::global_ns();
        if (!start) {
          start = now;
        } else if (now - start > pipe::kWaitNs) {
          record(kCodeGrid);
          sh.abort = 1;
          *abort_flag = 1u;
          break;
        }
      }
      __threadfence();
    }
  }
  consumers_sync();
  return !sh.abort;
}

// ---- producer -------------------------------------------------------------------
__device__ void issue_tile(const StageW& s, const Tiles& t, int tile, uint8_t* dst,
                           uint64_t* full) {
  const int i0 = t.first + tile * t.per_tile;
  const int cnt = min(t.per_tile, t.last - i0);
  const uint32_t rb = t.row_bytes;
  if (s.pair) {
    pipe::mbar_expect_tx(full, 2u * cnt * rb);
    pipe::bulk_g2s(dst, s.w[0] + (size_t)i0 * s.k, cnt * rb, full);
    pipe::bulk_g2s(dst + (size_t)cnt * rb, s.w[1] + (size_t)i0 * s.k, cnt * rb, full);
    return;
  }
  pipe::mbar_expect_tx(full, (uint32_t)cnt * rb);
  int seg_start = 0, done = 0;
  for (int seg = 0; seg < 3 && done < cnt; ++seg) {
    const int seg_end = seg_start + s.n[seg];
    const int a = max(i0 + done, seg_start), b = min(i0 + cnt, seg_end);
    if (a < b) {
      pipe::bulk_g2s(dst + (size_t)done * rb, s.w[seg] + (size_t)(a - seg_start) * s.k,
                     (uint32_t)(b - a) * rb, full);
      done += b - a;
    }
    seg_start = seg_end;
  }
}

__device__ void produce(const DecodeLoop& p, uint8_t* ring, Shared& sh) {
  const int S = p.slots;
  uint32_t g = 0;
  bool ok = true;
  for (int step = 0; ok && step < p.steps; ++step) {
    for (int layer = 0; ok && layer <= p.layers; ++layer) {
      const int nst = layer < p.layers ? 4 : 1;
      for (int j = 0; ok && j < nst; ++j) {
        const int st = layer < p.layers ? (j == 0 ? kQKV : j == 1 ? kO : j == 2 ? kGU : kDown)
                                        : kLM;
        const StageW s = stage_weights(p, layer, st);
        const Tiles t = tiles_of(p, s);
        const int trace_stage = layer < p.layers ? layer * 5 + (j == 0 ? 0 : j + 1) : p.layers * 5;
        (void)trace_stage;
        for (int tile = 0; tile < t.count; ++tile, ++g) {
          const int slot = (int)(g % S);
          const uint32_t use = g / S;
          if (!ring_wait(&sh.empty[slot], (use & 1u) ^ 1u, sh, kCodeEmpty | st)) {
            ok = false;
            break;
          }
          issue_tile(s, t, tile, ring + (size_t)slot * p.slot_bytes, &sh.full[slot]);
          if (tile == 0) MI_TRACE(step, trace_stage, 3);
          if (tile == t.count - 1) MI_TRACE(step, trace_stage, 4);
        }
      }
    }
  }
  // Wait for the last copies into this CTA's ring (all of them when
  // aborting: the consumers may have left without consuming them).
  const uint32_t first = g > (uint32_t)S ? g - (uint32_t)S : 0u;
  for (uint32_t q = first; q < g; ++q) {
    const int slot = (int)(q % S);
    const uint32_t parity = (q / S) & 1u;
    const uint64_t start = pipe::global_ns();
    while (!pipe::mbar_try_wait(&sh.full[slot], parity))
      if (pipe::global_ns() - start > pipe::kWaitNs) {
        record(kCodeDrain);
        break;
      }
  }
}

// ---- consumers: stage input -------------------------------------------------------
enum InMode : int { kPlainIn = 0, kNormIn = 1, kEmbedNormIn = 2, kAddNormIn = 3, kAddThenNormIn = 4 };

// Builds the stage input (k halves) in xs with the prologue of the GEMV
// family (gemv.cu build_input): the same roundings and the canonical sum of
// squares by one warp.
__device__ void build_input(int mode, const __half* x, const __half* x2, const __half* norm_w,
                            int k, float eps, __half* write_back, uint4* xs, Shared& sh) {
  const int tid = threadIdx.x;
  const int lane = tid & 31;
  const int kc = k >> 3;
  const uint4* src = reinterpret_cast<const uint4*>(x);
  const uint4* src2 = reinterpret_cast<const uint4*>(x2);
  for (int c = tid; c < kc; c += kConsumers) {
    uint4 v;
    if (mode == kAddNormIn || mode == kAddThenNormIn) {
      uint4 a = __ldcg(src + c);
      uint4 b = __ldcg(src2 + c);
      const __half2* ha = reinterpret_cast<const __half2*>(&a);
      const __half2* hb = reinterpret_cast<const __half2*>(&b);
      __half2* hv = reinterpret_cast<__half2*>(&v);
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        if (mode == kAddNormIn) {
          float2 fa = __half22float2(ha[i]);
          float2 fb = __half22float2(hb[i]);
          hv[i] = __floats2half2_rn(__fadd_rn(fa.x, fb.x), __fadd_rn(fa.y, fb.y));
        } else {
          hv[i] = __hadd2(ha[i], hb[i]);
        }
      }
    } else if (mode == kEmbedNormIn) {
      v = src ? src[c] : make_uint4(0, 0, 0, 0);  // embedding rows are constant
    } else {
      v = __ldcg(src + c);
    }
    if (write_back && blockIdx.x == 0) reinterpret_cast<uint4*>(write_back)[c] = v;
    xs[c] = v;
  }
  consumers_sync();
  if (mode == kPlainIn) return;
  if (tid < 32) {
    float acc = 0.f;
    for (int c = lane; c < kc; c += 32) {
      if (mode == kAddNormIn) {
        // squares of the unrounded sums (matvec2_add_rms_impl)
        uint4 a = __ldcg(src + c);
        uint4 b = __ldcg(src2 + c);
        const __half2* ha = reinterpret_cast<const __half2*>(&a);
        const __half2* hb = reinterpret_cast<const __half2*>(&b);
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          float2 fa = __half22float2(ha[i]);
          float2 fb = __half22float2(hb[i]);
          float s0 = __fadd_rn(fa.x, fb.x), s1 = __fadd_rn(fa.y, fb.y);
          acc = __fmaf_rn(s0, s0, acc);
          acc = __fmaf_rn(s1, s1, acc);
        }
      } else {
        acc = chunk_sq(xs[c], acc);
      }
    }
    float total = canon_reduce(acc, canon_lanes(k));
    if (lane == 0) sh.scale = rms_scale(total, k, eps);
  }
  consumers_sync();
  const float scale = sh.scale;
  const uint4* g4 = reinterpret_cast<const uint4*>(norm_w);
  for (int c = tid; c < kc; c += kConsumers) {
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
  consumers_sync();
}

// ---- consumers: rows from the ring --------------------------------------------------
// Reduces this CTA's rows of stage `st` (local row r goes to warp r mod 15)
// and writes the stage outputs. `g` is the running tile counter.
__device__ void reduce_rows(const DecodeLoop& p, int st, const StageW& s, const uint4* xs,
                            const uint8_t* ring, Shared& sh, uint32_t& g, uint32_t& best_key,
                            uint32_t& best_idx) {
  const int lane = threadIdx.x & 31;
  const int warp = threadIdx.x >> 5;
  const Tiles t = tiles_of(p, s);
  const int kc = s.k >> 3;
  const int lanes = canon_lanes(s.k);
  const int S = p.slots;
  for (int tile = 0; tile < t.count; ++tile, ++g) {
    const int slot = (int)(g % S);
    const uint32_t use = g / S;
    const bool ok = ring_wait(&sh.full[slot], use & 1u, sh, kCodeFull | st);
    if (threadIdx.x == 0 && tile == 0) MI_TRACE_CUR(5);
    const int i0 = t.first + tile * t.per_tile;
    const int cnt = min(t.per_tile, t.last - i0);
    const uint8_t* base = ring + (size_t)slot * p.slot_bytes;
    if (ok) {
      const int lead = (warp - (tile * t.per_tile) % kConsumerWarps + kConsumerWarps) %
                       kConsumerWarps;
      for (int r = lead; r < cnt; r += kConsumerWarps) {
        const uint4* w0 = reinterpret_cast<const uint4*>(base + (size_t)r * t.row_bytes);
        float a0 = 0.f, a1 = 0.f;
        if (st == kGU) {
          const uint4* w1 = reinterpret_cast<const uint4*>(base + (size_t)(cnt + r) * t.row_bytes);
          for (int c = lane; c < kc; c += 32) {
            uint4 xv = xs[c];
            a0 = chunk_dot(xv, w0[c], a0);
            a1 = chunk_dot(xv, w1[c], a1);
          }
          a1 = canon_reduce(a1, lanes);
        } else {
          for (int c = lane; c < kc; c += 32) a0 = chunk_dot(xs[c], w0[c], a0);
        }
        a0 = canon_reduce(a0, lanes);
        if (threadIdx.x == 0 && tile == 0 && r == lead) MI_TRACE_CUR(6);
        if (lane == 0) {
          const int item = i0 + r;
          switch (st) {
            case kQKV: {
              const int nq = s.n[0], nk = s.n[1];
              __half h0 = __float2half_rn(a0);
              if (item < nq) p.q_raw[item] = h0;
              else if (item < nq + nk) p.k_raw[item - nq] = h0;
              else p.v_raw[item - nq - nk] = h0;
              break;
            }
            case kO:
              p.attn_o[item] = __float2half_rn(a0);
              break;
            case kGU: {
              float gv = __half2float(__float2half_rn(a0));
              float uv = __half2float(__float2half_rn(a1));
              p.act[item] = __float2half_rn(silu_mul(gv, uv));
              break;
            }
            case kDown:
              p.hidden_buf[item] = __hadd(__ldcg(p.residual + item), __float2half_rn(a0));
              break;
            default: {
              __half h0 = __float2half_rn(a0);
              p.logits[item] = h0;
              float v = __half2float(h0);
              if (isfinite(v) && argmax_better(argmax_key(v), (uint32_t)item, best_key, best_idx)) {
                best_key = argmax_key(v);
                best_idx = (uint32_t)item;
              }
              break;
            }
          }
        }
      }
    }
    __syncwarp();
    if (lane == 0) mbar_arrive(&sh.empty[slot]);
  }
}

// ---- consumers: attention units (warps 0..3) -------------------------------------------
// Stages keys [j0, j1) of KV head g (cp.async, 16 bytes per copy), skipping
// position `skip` (the new token, taken from shared memory).
template <int G>
__device__ void stage_keys(const LoopLayer& L, int kvh, int g, int j0, int j1, int skip,
                           AttnSmem<G>& sm) {
  const int per_row = HD * 2 / 16;
  const int total = (j1 - j0) * per_row;
  const size_t stride = (size_t)kvh * HD;
  for (int i = threadIdx.x; i < total; i += kAttnThreads) {
    int r = i / per_row, c = i - r * per_row;
    int j = j0 + r;
    if (j == skip) continue;
    pipe::cp_async16(&sm.k[r][8 * c], L.k_cache + (size_t)j * stride + (size_t)g * HD + 8 * c);
    pipe::cp_async16(&sm.v[r][8 * c], L.v_cache + (size_t)j * stride + (size_t)g * HD + 8 * c);
  }
  pipe::cp_async_commit();
}

// One flash-decode unit: KV head g_kv, key block b of nb (attention.cu's
// attention_decode_kernel with the fused front end, run by 128 threads).
template <int G>
__device__ void attention_unit(const DecodeLoop& p, const LoopLayer& L, int g_kv, int b, int nb,
                               int pos, AttnSmem<G>& sm, Shared& sh) {
  const int lane = threadIdx.x & 31;
  const int warp = threadIdx.x >> 5;
  const int li = lane & 15;
  const int hw = warp * 2 + (lane >> 4);
  const int Lk = pos + 1;
  const int begin = b * p.block;
  const int end = min(Lk, begin + p.block);
  const int ntiles = (end - begin + kTile - 1) / kTile;

  if (hw < G) {
    const unsigned mask = (warp * 2 + 1 < G) ? 0xffffffffu : 0x0000ffffu;
    uint4 raw = __ldcg(reinterpret_cast<const uint4*>(p.q_raw + (size_t)(g_kv * G + hw) * HD) + li);
    float qv[8];
    norm_rope_half(raw, L.q_norm, (uint32_t)pos, p.theta, p.eps, p.round_norm != 0, mask, p.rope,
                   qv);
#pragma unroll
    for (int e = 0; e < 8; ++e) sm.q[hw][8 * li + e] = qv[e];
  }
  if (pos >= begin && pos < end && warp == 3 && lane >= 16) {
    uint4 raw = __ldcg(reinterpret_cast<const uint4*>(p.k_raw + (size_t)g_kv * HD) + li);
    float kv[8];
    norm_rope_half(raw, L.k_norm, (uint32_t)pos, p.theta, p.eps, p.round_norm != 0, 0xffff0000u,
                   p.rope, kv);
    uint4 kk;
    __half2* hk = reinterpret_cast<__half2*>(&kk);
#pragma unroll
    for (int i = 0; i < 4; ++i) hk[i] = __floats2half2_rn(kv[2 * i], kv[2 * i + 1]);
    uint4 vv = __ldcg(reinterpret_cast<const uint4*>(p.v_raw + (size_t)g_kv * HD) + li);
    const size_t row = (size_t)pos * p.kvh * HD + (size_t)g_kv * HD;
    reinterpret_cast<uint4*>(L.k_cache + row)[li] = kk;
    reinterpret_cast<uint4*>(L.v_cache + row)[li] = vv;
    reinterpret_cast<uint4*>(sm.new_k)[li] = kk;
    reinterpret_cast<uint4*>(sm.new_v)[li] = vv;
  }

  if (threadIdx.x == 0) MI_TRACE_CUR(5);
  float qreg[G][8];
  float m[G], l[G], acc[G][8];
  attn_sync();
#pragma unroll
  for (int g = 0; g < G; ++g) {
#pragma unroll
    for (int e = 0; e < 8; ++e) {
      qreg[g][e] = sm.q[g][8 * li + e];
      acc[g][e] = 0.f;
    }
    m[g] = -INFINITY;
    l[g] = 0.f;
  }
  const float scale = __frcp_rn(__fsqrt_rn((float)HD));

  for (int t = 0; t < ntiles; ++t) {
    const int j0 = begin + t * kTile;
    const int j1 = min(end, j0 + kTile);
    stage_keys<G>(L, p.kvh, g_kv, j0, j1, pos, sm);
    pipe::cp_async_wait_all();
    attn_sync();
    if (threadIdx.x == 0 && t == 0) MI_TRACE_CUR(6);
    // Stream hw takes block-relative keys hw, hw + 8, ...; both half-warps
    // of a warp run the same trip count.
    const int count = j1 - j0;
    for (int base = warp * 2; base < count; base += kStreams) {
      const int r = base + (lane >> 4);
      const bool valid = r < count;
      const int j = j0 + r;
      uint4 kk = make_uint4(0, 0, 0, 0), vv = make_uint4(0, 0, 0, 0);
      if (valid && j == pos) {
        kk = reinterpret_cast<const uint4*>(sm.new_k)[li];
        vv = reinterpret_cast<const uint4*>(sm.new_v)[li];
      } else if (valid) {
        kk = reinterpret_cast<const uint4*>(sm.k[r])[li];
        vv = reinterpret_cast<const uint4*>(sm.v[r])[li];
      }
      float kf[8], vf[8];
      const __half2* hk = reinterpret_cast<const __half2*>(&kk);
      const __half2* hv = reinterpret_cast<const __half2*>(&vv);
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        float2 fk = __half22float2(hk[i]);
        float2 fv = __half22float2(hv[i]);
        kf[2 * i] = fk.x;
        kf[2 * i + 1] = fk.y;
        vf[2 * i] = fv.x;
        vf[2 * i + 1] = fv.y;
      }
#pragma unroll
      for (int g = 0; g < G; ++g) {
        float d = 0.f;
#pragma unroll
        for (int e = 0; e < 8; ++e) d = __fmaf_rn(qreg[g][e], kf[e], d);
        float s = __fmul_rn(canon_butterfly(d, 16), scale);
        if (!valid) continue;
        float nm = fmaxf(m[g], s);
        float pa = mi_exp(__fsub_rn(m[g], nm));
        float pc = mi_exp(__fsub_rn(s, nm));
#pragma unroll
        for (int e = 0; e < 8; ++e) acc[g][e] = __fmaf_rn(acc[g][e], pa, __fmul_rn(pc, vf[e]));
        l[g] = __fmaf_rn(l[g], pa, pc);
        m[g] = nm;
      }
    }
    attn_sync();
  }

  if (threadIdx.x == 0) MI_TRACE_CUR(7);
  // Stream merge (index order) -> block partial.
#pragma unroll
  for (int g = 0; g < G; ++g) {
    if (li == 0) {
      sm.m[hw][g] = m[g];
      sm.l[hw][g] = l[g];
    }
#pragma unroll
    for (int e = 0; e < 8; ++e) sm.acc[hw][g][8 * li + e] = acc[g][e];
  }
  attn_sync();
  const int stride = HD + 2;
  float* part = p.attn_part + ((size_t)g_kv * p.attn_blocks + b) * G * stride;
  for (int idx = threadIdx.x; idx < G * HD; idx += kAttnThreads) {
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
      p.attn[(size_t)(g_kv * G + g) * HD + d] = __float2half_rn(__fdiv_rn(num, den));
    } else {
      part[g * stride + 2 + d] = num;
      if (d == 0) {
        part[g * stride] = M;
        part[g * stride + 1] = den;
      }
    }
  }
  if (threadIdx.x == 0) MI_TRACE_CUR(8);
  if (nb == 1) {
    attn_sync();  // shared state is reused by the next unit
    return;
  }
  __threadfence();
  attn_sync();
  if (threadIdx.x == 0) sm.last = atomicAdd(p.attn_count + g_kv, 1u) == (uint32_t)nb - 1;
  attn_sync();
  if (sm.last) {
    __threadfence();
    const float* hb = p.attn_part + (size_t)g_kv * p.attn_blocks * G * stride;
    for (int idx = threadIdx.x; idx < G * HD; idx += kAttnThreads) {
      int g = idx / HD, d = idx - g * HD;
      float M = -INFINITY;
      for (int s = 0; s < nb; ++s) M = fmaxf(M, __ldcg(hb + (size_t)(s * G + g) * stride));
      float num = 0.f, den = 0.f;
      for (int s = 0; s < nb; ++s) {
        const float* ps = hb + (size_t)(s * G + g) * stride;
        float mm = __ldcg(ps);
        float f = mm == -INFINITY ? 0.f : mi_exp(__fsub_rn(mm, M));
        den = __fmaf_rn(__ldcg(ps + 1), f, den);
        num = __fmaf_rn(__ldcg(ps + 2 + d), f, num);
      }
      p.attn[(size_t)(g_kv * G + g) * HD + d] = __float2half_rn(__fdiv_rn(num, den));
    }
    if (threadIdx.x == 0) p.attn_count[g_kv] = 0u;
    if (threadIdx.x == 0) MI_TRACE_CUR(10);
  }
  if (threadIdx.x == 0) MI_TRACE_CUR(9);
  attn_sync();
}

template <int G>
__global__ void __launch_bounds__(kThreads, 1) decode_loop_kernel(DecodeLoop p) {
  extern __shared__ __align__(128) uint8_t smem[];
  __shared__ Shared sh;
  uint8_t* ring = smem;
  uint4* xs = reinterpret_cast<uint4*>(smem + (size_t)p.slots * p.slot_bytes);
  AttnSmem<G>& asm_ = *reinterpret_cast<AttnSmem<G>*>(smem + (size_t)p.slots * p.slot_bytes +
                                                        p.x_bytes);
  const int tid = threadIdx.x;
  if (tid == 0) {
    for (int s = 0; s < p.slots; ++s) {
      pipe::mbar_init(&sh.full[s], 1);
      pipe::mbar_init(&sh.empty[s], kConsumerWarps);
    }
    sh.abort = 0;
    pipe::fence_mbar_init();
  }
  __syncthreads();

  if (tid >= kConsumers) {
    if (tid == kConsumers) produce(p, ring, sh);
    return;
  }

  const uint32_t len0 = __ldcg(p.dev_len);
  uint32_t token = __ldcg(p.toks + len0);
  uint32_t g = 0, epoch = 0;
  const int warp = tid >> 5, lane = tid & 31;
  for (int step = 0; step < p.steps; ++step) {
    const int pos = (int)len0 + step;
    for (int layer = 0; layer < p.layers; ++layer) {
      const LoopLayer& L = p.layer[layer];
      uint32_t bk = 0, bi = 0xFFFFFFFFu;
      // QKV
      {
        if (tid == 0) { MI_TRACE(step, layer * 5 + 0, 0); MI_TRACE_SET(step, layer * 5 + 0); }
        StageW s = stage_weights(p, layer, kQKV);
        if (layer == 0) {
          const bool zero = token == 0xFFFFFFFFu || token >= (uint32_t)p.vocab;
          build_input(kEmbedNormIn, zero ? nullptr : p.embedding + (size_t)token * p.hidden,
                      nullptr, L.in_norm, p.hidden, p.eps, p.hidden_buf, xs, sh);
        } else {
          build_input(kNormIn, p.hidden_buf, nullptr, L.in_norm, p.hidden, p.eps, nullptr, xs, sh);
        }
        if (tid == 0) MI_TRACE(step, layer * 5 + 0, 1);
        reduce_rows(p, kQKV, s, xs, ring, sh, g, bk, bi);
        if (tid == 0) MI_TRACE(step, layer * 5 + 0, 2);
        if (!grid_sync(p, epoch, sh)) return;
      }
      // ATTN
      {
        if (tid == 0) { MI_TRACE(step, layer * 5 + 1, 0); MI_TRACE_SET(step, layer * 5 + 1); }
        const int nb = (pos + p.block) / p.block;  // ceil((pos + 1) / block)
        const int units = p.kvh * nb;
        if (tid < kAttnThreads)
          for (int u = blockIdx.x; u < units; u += gridDim.x)
            attention_unit<G>(p, L, u / nb, u % nb, nb, pos, asm_, sh);
        if (tid == 0) MI_TRACE(step, layer * 5 + 1, 2);
        if (!grid_sync(p, epoch, sh)) return;
      }
      // O
      {
        if (tid == 0) { MI_TRACE(step, layer * 5 + 2, 0); MI_TRACE_SET(step, layer * 5 + 2); }
        StageW s = stage_weights(p, layer, kO);
        build_input(kPlainIn, p.attn, nullptr, nullptr, s.k, p.eps, nullptr, xs, sh);
        if (tid == 0) MI_TRACE(step, layer * 5 + 2, 1);
        reduce_rows(p, kO, s, xs, ring, sh, g, bk, bi);
        if (tid == 0) MI_TRACE(step, layer * 5 + 2, 2);
        if (!grid_sync(p, epoch, sh)) return;
      }
      // GU
      {
        if (tid == 0) { MI_TRACE(step, layer * 5 + 3, 0); MI_TRACE_SET(step, layer * 5 + 3); }
        StageW s = stage_weights(p, layer, kGU);
        build_input(p.add_norm ? kAddNormIn : kAddThenNormIn, p.hidden_buf, p.attn_o, L.post_norm,
                    p.hidden, p.eps, p.residual, xs, sh);
        if (tid == 0) MI_TRACE(step, layer * 5 + 3, 1);
        reduce_rows(p, kGU, s, xs, ring, sh, g, bk, bi);
        if (tid == 0) MI_TRACE(step, layer * 5 + 3, 2);
        if (!grid_sync(p, epoch, sh)) return;
      }
      // DOWN
      {
        if (tid == 0) { MI_TRACE(step, layer * 5 + 4, 0); MI_TRACE_SET(step, layer * 5 + 4); }
        StageW s = stage_weights(p, layer, kDown);
        build_input(kPlainIn, p.act, nullptr, nullptr, s.k, p.eps, nullptr, xs, sh);
        if (tid == 0) MI_TRACE(step, layer * 5 + 4, 1);
        reduce_rows(p, kDown, s, xs, ring, sh, g, bk, bi);
        if (tid == 0) MI_TRACE(step, layer * 5 + 4, 2);
        if (!grid_sync(p, epoch, sh)) return;
      }
    }
    // final norm + LM head + argmax
    {
      if (tid == 0) { MI_TRACE(step, p.layers * 5, 0); MI_TRACE_SET(step, p.layers * 5); }
      uint32_t bk = 0, bi = 0xFFFFFFFFu;
      StageW s = stage_weights(p, p.layers, kLM);
      build_input(kNormIn, p.hidden_buf, nullptr, p.final_norm, p.hidden, p.eps, nullptr, xs, sh);
      if (tid == 0) MI_TRACE(step, p.layers * 5, 1);
      reduce_rows(p, kLM, s, xs, ring, sh, g, bk, bi);
      if (tid == 0) MI_TRACE(step, p.layers * 5, 2);
      if (lane == 0) {
        sh.best_key[warp] = bk;
        sh.best_idx[warp] = bi;
      }
      consumers_sync();
      if (tid == 0) {
        uint32_t ck = 0, ci = 0xFFFFFFFFu;
        for (int w = 0; w < kConsumerWarps; ++w)
          if (argmax_better(sh.best_key[w], sh.best_idx[w], ck, ci)) {
            ck = sh.best_key[w];
            ci = sh.best_idx[w];
          }
        p.argmax_key[blockIdx.x] = ck;
        p.argmax_idx[blockIdx.x] = ci;
      }
      if (!grid_sync(p, epoch, sh)) return;
      if (warp == 0) {
        uint32_t ck = 0, ci = 0xFFFFFFFFu;
        for (int b = lane; b < (int)gridDim.x; b += 32) {
          uint32_t k2 = __ldcg(p.argmax_key + b), i2 = __ldcg(p.argmax_idx + b);
          if (argmax_better(k2, i2, ck, ci)) {
            ck = k2;
            ci = i2;
          }
        }
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) {
          uint32_t ok = __shfl_xor_sync(0xffffffffu, ck, o);
          uint32_t oi = __shfl_xor_sync(0xffffffffu, ci, o);
          if (argmax_better(ok, oi, ck, ci)) {
            ck = ok;
            ci = oi;
          }
        }
        if (lane == 0) {
          sh.token = ci;
          if (blockIdx.x == 0) p.toks[pos + 1] = ci;
        }
      }
      consumers_sync();
      token = sh.token;
    }
  }
  if (blockIdx.x == 0 && tid == 0) *p.dev_len = len0 + (uint32_t)p.steps;
}

template <int G>
size_t attn_smem_bytes() {
  return (sizeof(AttnSmem<G>) + 127) / 128 * 128;
}

size_t attn_smem_for(int group) {
  switch (group) {
    case 1: return attn_smem_bytes<1>();
    case 2: return attn_smem_bytes<2>();
    case 4: return attn_smem_bytes<4>();
    case 8: return attn_smem_bytes<8>();
    default: return 0;
  }
}

template <int G>
cudaError_t launch_g(cudaStream_t stream, const DecodeLoop& p, int grid, size_t smem) {
  auto kernel = decode_loop_kernel<G>;
  cudaError_t err =
      cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  if (err != cudaSuccess) return err;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(grid);
  cfg.blockDim = dim3(kThreads);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeCooperative;
  attr[0].val.cooperative = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, kernel, p);
}

}  // namespace

bool decode_loop_plan(DecodeLoop& p, int device) {
  const int group = p.kvh > 0 ? p.qh / p.kvh : 0;
  if (attn_smem_for(group) == 0 || p.qh % p.kvh) return false;
  if (p.hidden % 8 || p.inter % 8 || p.hidden <= 0 || p.inter <= 0) return false;
  const int max_k = std::max(std::max(p.hidden, p.inter), p.qh * HD);
  int max_item = std::max(std::max(p.hidden * 4, p.inter * 2), p.qh * HD * 2);
  p.slot_bytes = std::max(kMinSlotBytes, (max_item + 127) / 128 * 128);
  p.x_bytes = (max_k * 2 + 127) / 128 * 128;
  int optin = 0;
  if (cudaDeviceGetAttribute(&optin, cudaDevAttrMaxSharedMemoryPerBlockOptin, device) !=
      cudaSuccess)
    return false;
  const size_t fixed = (size_t)p.x_bytes + attn_smem_for(group) + sizeof(Shared) + 1024;
  if (fixed >= (size_t)optin) return false;
  p.slots = (int)std::min<size_t>(kMaxSlots, ((size_t)optin - fixed) / p.slot_bytes);
  if (p.slots < 2) return false;
  int sms = 0;
  if (cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, device) != cudaSuccess)
    return false;
  p.grid = sms;
  return true;
}

size_t decode_loop_smem(const DecodeLoop& p) {
  return (size_t)p.slots * p.slot_bytes + p.x_bytes + attn_smem_for(p.qh / p.kvh);
}

void decode_loop(cudaStream_t stream, const DecodeLoop& p) {
  MI_REQUIRE(p.steps > 0 && p.grid > 0 && p.slots >= 2, MI_ERR_INVALID_ARGUMENT,
             "decode loop plan missing");
  MI_CUDA(cudaMemsetAsync(p.sync, 0, 2 * sizeof(uint32_t), stream));
  const size_t smem = decode_loop_smem(p);
  cudaError_t err = cudaErrorInvalidValue;
  switch (p.qh / p.kvh) {
    case 1: err = launch_g<1>(stream, p, p.grid, smem); break;
    case 2: err = launch_g<2>(stream, p, p.grid, smem); break;
    case 4: err = launch_g<4>(stream, p, p.grid, smem); break;
    case 8: err = launch_g<8>(stream, p, p.grid, smem); break;
    default: break;
  }
  if (err != cudaSuccess)
    fail(MI_ERR_COMMAND, "decode loop launch failed: %s", cudaGetErrorString(err));
}

#ifdef MI_DECODE_TRACE
extern "C" int mi_debug_decode_trace(unsigned long long* out, size_t n) {
  if (n < sizeof(g_trace) / 8) return -1;  // [2][2][321][12]
  return cudaMemcpyFromSymbol(out, g_trace, sizeof(g_trace)) == cudaSuccess ? 0 : -2;
}
#endif

unsigned decode_loop_status(bool reset) {
  unsigned v = 0;
  cudaMemcpyFromSymbol(&v, g_loop_status, sizeof v);
  if (reset && v) {
    unsigned z = 0;
    cudaMemcpyToSymbol(g_loop_status, &z, sizeof z);
  }
  return v;
}

}  // namespace k
}  // namespace mi
