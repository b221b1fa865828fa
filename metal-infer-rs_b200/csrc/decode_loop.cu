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
// One CTA per SM: 11 consumer warps and one producer warp. The producer
// walks the static schedule of weight tiles this CTA will reduce (every
// stage of every layer of every step, then the LM head) and streams them
// into a ring of shared-memory slots with 1-D bulk copies that complete on
// "full" mbarriers. It is throttled only by the ring ("empty" mbarriers the
// consumer warps arrive on), never by the grid barriers between stages, so
// HBM keeps streaming weights while the consumers wait on their
// predecessors; a second cursor over the same schedule prefetches the tiles
// a few slots beyond the ring into L2, so the stream goes on while the ring
// is full. Consumers build each stage's input vector in shared memory,
// reduce their rows from the ring and write the outputs to global memory.
// The kernel is instantiated twice: for one GPU, and for tensor parallelism
// (the mailbox exchanges), so that neither carries the other's code.
//
// There are no grid barriers. Activations that cross CTAs are stored as
// epoch-tagged words (tag << 16 | FP16 bits) that validate themselves: after
// one L2 round trip of delay a CTA reads the words of the stage it consumes
// and re-polls those whose tag is not there yet (no completion counters; under
// tensor parallelism every rank polls the tagged partials the others store
// into its mailbox the same way).
// Attention units publish their block partials with a release reduction,
// and the O stage merges the partials of every head while building its input.
//
// Every wait is bounded in time: a ring wait, a counter or tag poll that
// gives up records a code in g_loop_status and raises a device-wide abort
// flag; all warps leave at the next stage boundary and the producer waits
// (bounded) for its copies in flight before the CTA exits.

#include <algorithm>

#include "device.cuh"
#include "pipeline.cuh"


namespace mi {
namespace k {

namespace {

constexpr int HD = 128;
// 11 consumer warps + 1 producer: 384 threads, 168 registers (15 consumer
// warps at 128 registers measured 1.5% slower on Qwen3-0.6B)
constexpr int kConsumerWarps = 11;
constexpr int kConsumers = kConsumerWarps * 32;
constexpr int kThreads = kConsumers + 32;  // + producer warp
constexpr int kStreams = 8;
constexpr int kTile = 64;                  // keys staged per attention tile
constexpr int kAttnThreads = 256;          // the last 8 consumer warps run the attention units
constexpr int kAttnBase = kConsumerWarps * 32 - kAttnThreads;  // warps 3..10
constexpr int kMaxSlots = 16;
// sync[]: [1] abort flag, [2] attention units finished (cumulative over the
// launch), [kStageDone + st] a word the stage hand-off loads (its delay).
constexpr int kUnitsDone = 2;
constexpr int kStageDone = 8;
constexpr int kPart = HD + 4;  // partial record: max, denominator, 2 pad, 128 numerators
constexpr int kSyncWords = 512;
constexpr int kWaitWord0 = 256;  // per-CTA mailbox wait time (64 ns units)
constexpr int kMaxKvHeads = 64;
constexpr int kMaxDownRows = 64;
constexpr int kMaxGrid = 256;
constexpr int kMinSlotBytes = 32 * 1024;  // 24 / 40 / 64 KB measured slower

static __device__ unsigned g_loop_status = 0;

#ifdef MI_DECODE_TRACE
// Diagnostic build only: %globaltimer stamps of the first and last CTA for
// the first two steps: [cta][step][stage][event], events 0..2 = consumer
// thread 0 after the preceding barrier / after the input / after its rows,
// 3..4 = producer issue of the stage's first / last tile.
constexpr int kTraceStages = 5 * 64 + 1;
constexpr int kTraceEvents = 16;
static __device__ unsigned long long g_trace[2][2][kTraceStages][kTraceEvents];
__shared__ int g_trace_cur[2];  // step, stage of the running stage (traced CTAs)
__shared__ int g_trace_alt;     // events 9 / 10 / 15 of build_input recorded as 11 / 12 / 13
__device__ __forceinline__ void trace(int step, int stage, int ev) {
  const int c = blockIdx.x == 0 ? 0 : (blockIdx.x == gridDim.x - 1 ? 1 : -1);
  if (c < 0 || step >= 2 || stage >= kTraceStages) return;
  g_trace[c][step][stage][ev] = pipe::global_ns();
}
// every CTA: arrival at / release from the grid barriers of step 1, layer 3
static __device__ unsigned long long g_arrive[256][5][2];
__device__ __forceinline__ void trace_arrive(int step, int stage, int ev) {
  if (step == 1 && stage >= 15 && stage < 20 && blockIdx.x < 256)
    g_arrive[blockIdx.x][stage - 15][ev] = pipe::global_ns();
}
#define MI_TRACE(step, stage, ev) trace(step, stage, ev)
#define MI_TRACE_ARRIVE(ev) trace_arrive(g_trace_cur[0], g_trace_cur[1], ev)
#define MI_TRACE_CUR(ev) trace(g_trace_cur[0], g_trace_cur[1], ev)
#define MI_TRACE_IN(ev) \
  trace(g_trace_cur[0], g_trace_cur[1], g_trace_alt ? ((ev) == 9 ? 11 : (ev) == 10 ? 12 : 13) : (ev))
#define MI_TRACE_SET(step, stage) (g_trace_cur[0] = (step), g_trace_cur[1] = (stage))
#else
#define MI_TRACE(step, stage, ev) ((void)0)
#define MI_TRACE_CUR(ev) ((void)0)
#define MI_TRACE_IN(ev) ((void)0)
#define MI_TRACE_ARRIVE(ev) ((void)0)
#define MI_TRACE_SET(step, stage) ((void)0)
#endif

enum Stage : int { kQKV = 0, kO = 1, kGU = 2, kDown = 3, kLM = 4 };

// Failure codes (high byte: place, low byte: stage).
constexpr unsigned kCodeFull = 0x0100;
constexpr unsigned kCodeEmpty = 0x0200;
constexpr unsigned kCodeDrain = 0x0400;
constexpr unsigned kCodeHead = 0x0500;
constexpr unsigned kCodeTag = 0x0600;
constexpr unsigned kCodeKv = 0x0700;

struct StageW {
  const __half* w[3];
  int n[3];
  int k;      // reduction length
  int items;  // rows (pairs for GU)
  int pair;   // GU: gate and up rows per item
};

__device__ __forceinline__ StageW stage_weights(const DecodeLoop& p, const LoopLayer* layers,
                                                int layer, int st) {
  StageW s = {};
  const LoopLayer* L = layers + (layer < p.layers ? layer : 0);
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

// Shared state of the attention units. K and V tiles arrive by TMA as two
// 64-column halves of kTile rows each, 128-byte swizzled (16-byte chunk c of
// row j sits at chunk position c ^ (j & 7) of the row's 128 bytes), so one
// thread per key reads its row without bank conflicts. After a unit's last
// tile the tile region holds the stream accumulators of the stream merge.
template <int G>
struct AttnSmem {
  __half k[2][kTile][64];  // 1024-byte aligned (the swizzle atom)
  __half v[2][kTile][64];
  __half new_k[HD];        // this step's K / V row (the tile's copy is stale)
  __half new_v[HD];
  __half qn_w[HD];         // QK-norm weights of the layer (prefetched)
  __half kn_w[HD];
  float2 rope[HD / 2];     // (cos, sin) at the step's position (prefetched)
  __half q[G][HD];         // normed, rotated, FP16-rounded queries
  float sc[G][kTile];      // scaled scores of the tile
  float pa[G][kTile];      // exp(m_prev - m), exp(s - m) per key
  float pc[G][kTile];
  float m[2][kStreams][G]; // running max per stream, by tile parity
  float l[kStreams][G];
  float f[kStreams][G];    // stream merge factors
  float M[G];
};
static_assert(sizeof(float) * kStreams * 8 * HD <= 2 * 2 * kTile * 64 * sizeof(__half),
              "stream accumulators must fit in the tile region");

struct Shared {
  uint64_t full[kMaxSlots];
  uint64_t empty[kMaxSlots];
  uint64_t kv_full;  // the attention prefetch (first key tile, norms, RoPE row)
  uint64_t kv_tile;  // the attention units' other key tiles
  Tiles tiles[5];  // this CTA's tiling of each stage (the same in every layer)
  float scale;
  __half res[kMaxDownRows];         // DOWN: residual values of this CTA's rows
  uint32_t best_key[kConsumerWarps];
  uint32_t best_idx[kConsumerWarps];
  uint32_t token;
  unsigned long long mbox_ns;  // thread 0: time spent on inputs fed by the other ranks
  volatile int abort;  // raised by any warp (or the producer) that gives up
  int stop;            // the consumers' uniform decision, written by one thread between barriers
  int astop;           // the same for the attention warps
};

__device__ __forceinline__ void consumers_sync() {
  asm volatile("bar.sync 1, %0;" ::"n"(kConsumers) : "memory");
}
// The consumers' barrier with an OR of `pred` over its threads: every thread
// gets the same answer, so a decision taken on it stays uniform.
__device__ __forceinline__ bool consumers_any(bool pred) {
  uint32_t r;
  asm volatile(
      "{\n .reg .pred p, q;\n setp.ne.u32 p, %1, 0;\n bar.red.or.pred q, 1, %2, p;\n"
      " selp.u32 %0, 1, 0, q;\n}"
      : "=r"(r)
      : "r"((uint32_t)pred), "n"(kConsumers)
      : "memory");
  return r != 0;
}
__device__ __forceinline__ void attn_sync() {
  asm volatile("bar.sync 2, %0;" ::"n"(kAttnThreads) : "memory");
}

__device__ __forceinline__ uint32_t ld_relaxed(const uint32_t* p) {
  uint32_t v;
  asm volatile("ld.relaxed.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}


__device__ __forceinline__ void red_release_add(uint32_t* p, uint32_t v) {
  asm volatile("red.release.gpu.global.add.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
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

// 2-D TMA tile load (no multicast) from a tensor map in global memory.
__device__ __forceinline__ void tma_load_2d(void* dst, const void* map, uint64_t* bar, int c0,
                                            int c1) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, "
      "{%3, %4}], [%2];" ::"r"(pipe::smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(pipe::smem_u32(bar)), "r"(c0), "r"(c1)
      : "memory");
}

// Wait for bulk copies this CTA issued (bounded in time, but not cut short
// by an abort: the copies must land before the CTA may leave).
__device__ void copies_wait(uint64_t* bar, uint32_t parity, unsigned code) {
  if (pipe::mbar_try_wait(bar, parity)) return;
  const uint64_t start = pipe::global_ns();
  while (!pipe::mbar_try_wait(bar, parity))
    if (pipe::global_ns() - start > pipe::kWaitNs) {
      record(code);
      return;
    }
}

// ---- epoch-tagged activations ----------------------------------------------------
// Every activation vector that crosses CTAs is stored as one u32 per FP16
// value: (16-bit tag << 16) | value bits, written with a single store. A
// reader polls the words it needs until all carry the tag of the layer-step
// it wants, so each word validates itself and no grid barrier is needed.
// Overwrites are ordered by the data dependencies of the stages: a buffer is
// written again only by a stage that first consumed complete vectors from
// every CTA, each of which had finished reading the previous contents.
// tag(e, slot): e = layer-step counter (host base + step * layers + layer),
// slot 1 marks the DOWN output, which shares the hidden buffer with the
// embedding written at layer 0.
__device__ __forceinline__ uint32_t tagv(uint32_t e, int slot) {
  return ((e * 2u + (uint32_t)slot) & 0xFFFFu) << 16;
}
__device__ __forceinline__ uint4 ld_relaxed_v4(const uint32_t* p) {
  uint4 v;
  asm volatile("ld.relaxed.gpu.global.v4.u32 {%0,%1,%2,%3}, [%4];"
               : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
               : "l"(p)
               : "memory");
  return v;
}
__device__ __forceinline__ void st_relaxed(uint32_t* p, uint32_t v) {
  asm volatile("st.relaxed.gpu.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ void st_relaxed_v4(uint32_t* p, uint4 v) {
  asm volatile("st.relaxed.gpu.global.v4.u32 [%0], {%1,%2,%3,%4};" ::"l"(p), "r"(v.x), "r"(v.y),
               "r"(v.z), "r"(v.w)
               : "memory");
}
__device__ __forceinline__ void st_relaxed_u64(unsigned long long* p, unsigned long long v) {
  asm volatile("st.relaxed.gpu.global.u64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}

// Bounded-poll bookkeeping shared by the tag waits: false once the kernel
// is aborting (the caller then continues on zeros until the next decision).
struct PollClock {
  uint64_t start = 0;
  __device__ __forceinline__ bool keep_going(const DecodeLoop& p, Shared& sh) {
    if (sh.abort || *reinterpret_cast<volatile uint32_t*>(p.sync + 1)) {
      sh.abort = 1;
      return false;
    }
    const uint64_t now = pipe::global_ns();
    if (!start) {
      start = now;
    } else if (now - start > pipe::kWaitNs) {
      record(kCodeTag);
      sh.abort = 1;
      *reinterpret_cast<volatile uint32_t*>(p.sync + 1) = 1u;
      return false;
    }
    return true;
  }
};

// Chunk c (8 FP16 values) of a tagged vector, once all 8 carry `tag`.
__device__ uint4 take8(const DecodeLoop& p, const uint32_t* src, int c, uint32_t tag,
                                   Shared& sh) {
  const uint32_t* q = src + 8 * c;
  PollClock clock;
  while (true) {
    const uint4 a = ld_relaxed_v4(q), b = ld_relaxed_v4(q + 4);
    const uint32_t miss = (a.x ^ tag) | (a.y ^ tag) | (a.z ^ tag) | (a.w ^ tag) | (b.x ^ tag) |
                          (b.y ^ tag) | (b.z ^ tag) | (b.w ^ tag);
    if ((miss >> 16) == 0)
      return make_uint4((a.x & 0xFFFFu) | (a.y << 16), (a.z & 0xFFFFu) | (a.w << 16),
                        (b.x & 0xFFFFu) | (b.y << 16), (b.z & 0xFFFFu) | (b.w << 16));
    if (!clock.keep_going(p, sh)) return make_uint4(0, 0, 0, 0);
  }
}

// Two-phase form for batching: issue the raw loads of several chunks first,
// then validate (re-polling only chunks whose tags were not there yet).
struct Raw8 {
  uint4 a, b;
};
__device__ __forceinline__ Raw8 raw8(const uint32_t* src, int c) {
  return {ld_relaxed_v4(src + 8 * c), ld_relaxed_v4(src + 8 * c + 4)};
}
__device__ __forceinline__ uint4 take8_from(const DecodeLoop& p, const Raw8& r,
                                            const uint32_t* src, int c, uint32_t tag,
                                            Shared& sh) {
  const uint32_t miss = (r.a.x ^ tag) | (r.a.y ^ tag) | (r.a.z ^ tag) | (r.a.w ^ tag) |
                        (r.b.x ^ tag) | (r.b.y ^ tag) | (r.b.z ^ tag) | (r.b.w ^ tag);
  if ((miss >> 16) == 0)
    return make_uint4((r.a.x & 0xFFFFu) | (r.a.y << 16), (r.a.z & 0xFFFFu) | (r.a.w << 16),
                      (r.b.x & 0xFFFFu) | (r.b.y << 16), (r.b.z & 0xFFFFu) | (r.b.w << 16));
  return take8(p, src, c, tag, sh);
}

// Element i of a tagged vector.
__device__ __half take1(const DecodeLoop& p, const uint32_t* src, int i, uint32_t tag, Shared& sh) {
  PollClock clock;
  while (true) {
    const uint32_t w = ld_relaxed(src + i);
    if ((w >> 16) == (tag >> 16)) return __ushort_as_half((unsigned short)(w & 0xFFFFu));
    if (!clock.keep_going(p, sh)) return __float2half_rn(0.f);
  }
}

__device__ __forceinline__ void put1(uint32_t* dst, int i, __half h, uint32_t tag) {
  st_relaxed(dst + i, tag | __half_as_ushort(h));
}
__device__ __forceinline__ void put8(uint32_t* dst, int c, const uint4& v, uint32_t tag) {
  st_relaxed_v4(dst + 8 * c, make_uint4(tag | (v.x & 0xFFFFu), tag | (v.x >> 16),
                                         tag | (v.y & 0xFFFFu), tag | (v.y >> 16)));
  st_relaxed_v4(dst + 8 * c + 4, make_uint4(tag | (v.z & 0xFFFFu), tag | (v.z >> 16),
                                             tag | (v.w & 0xFFFFu), tag | (v.w >> 16)));
}

// ---- tensor-parallel exchange through peer memory ------------------------------------
// Partials are pushed with plain stores into every rank's mailbox (NVLink
// peer mappings); readers poll their own mailbox. System-scope relaxed
// accesses: the tags validate every word. (Counting every CTA of every rank
// into one counter per rank, 1,184 remote reductions per exchange at TP8,
// cost more than the exchange itself.)
__device__ __forceinline__ void st_sys_u64(unsigned long long* p, unsigned long long v) {
  asm volatile("st.relaxed.sys.global.u64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}
__device__ __forceinline__ unsigned long long ld_sys_u64(const unsigned long long* p) {
  unsigned long long v;
  asm volatile("ld.relaxed.sys.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
  return v;
}

// This rank's FP32 partial of row `item` into region `region` of every rank.
__device__ __forceinline__ void push_partial(const DecodeLoop& p, size_t region, int item,
                                             float v, uint32_t tag) {
  const unsigned long long w = ((unsigned long long)tag << 32) | __float_as_uint(v);
  for (int r = 0; r < p.tp; ++r) st_sys_u64(p.peers[r] + region + (size_t)p.rank * p.hidden + item, w);
}

// Chunk c (8 values) of the ranks' partials in region `region`, summed in
// rank order in FP32 and rounded once to FP16 (the row-parallel result).
__device__ uint4 take_partials8(const DecodeLoop& p, size_t region, int c, uint32_t tag,
                                Shared& sh) {
  float acc[8];
  for (int r = 0; r < p.tp; ++r) {
    const unsigned long long* q = p.mbox + region + (size_t)r * p.hidden + 8 * c;
    unsigned long long w[8];
    PollClock clock;
    while (true) {
      bool ok = true;
#pragma unroll
      for (int e = 0; e < 8; ++e) {
        w[e] = ld_sys_u64(q + e);
        ok &= (uint32_t)(w[e] >> 32) == tag;
      }
      if (ok || !clock.keep_going(p, sh)) break;
    }
#pragma unroll
    for (int e = 0; e < 8; ++e) {
      const float v = __uint_as_float((uint32_t)w[e]);
      acc[e] = r == 0 ? v : __fadd_rn(acc[e], v);
    }
  }
  uint4 out;
  __half2* ho = reinterpret_cast<__half2*>(&out);
#pragma unroll
  for (int i = 0; i < 4; ++i) ho[i] = __floats2half2_rn(acc[2 * i], acc[2 * i + 1]);
  return out;
}

// Single-thread bounded wait until *ctr >= target (a cumulative counter);
// false when the kernel is aborting.
__device__ bool wait_counter(const DecodeLoop& p, const uint32_t* ctr, uint32_t target,
                             Shared& sh) {
  volatile uint32_t* abort_flag = p.sync + 1;
  uint64_t start = 0;
  while (ld_relaxed(ctr) < target) {
    if (*abort_flag || sh.abort) {
      sh.abort = 1;
      return false;
    }
    const uint64_t now = pipe::global_ns();
    if (!start) {
      start = now;
    } else if (now - start > pipe::kWaitNs) {
      record(kCodeHead);
      sh.abort = 1;
      *abort_flag = 1u;
      return false;
    }
  }
  __threadfence();
  return true;
}

// Start of the O stage: wait until `units` attention units (cumulative over
// the launch) have published their block partials. While this CTA's own
// attention warps work, the other warps wait at a barrier rather than have
// one of them spin on the counter beside them.
__device__ bool wait_units(const DecodeLoop& p, uint32_t units, bool ran_units, Shared& sh) {
  if (ran_units) consumers_sync();
  if (threadIdx.x == 0) {
    const bool ok = !sh.abort && wait_counter(p, p.sync + kUnitsDone, units, sh);
    sh.stop = ok ? 0 : 1;
  }
  consumers_sync();
  return !sh.stop;
}

// End of a stage: every warp has issued its tagged stores (the readers
// validate each word by its tag, here and in the other ranks' mailboxes).
__device__ __forceinline__ void stage_done(const DecodeLoop& p, int st) {
  (void)p;
  (void)st;
  consumers_sync();
  if (threadIdx.x == 0) MI_TRACE_ARRIVE(0);
}

// Thread 0, before a stage reads another stage's tagged outputs: one L2 round
// trip of delay, then the tagged reads poll their words (each word carries
// its layer-step, so no completion counter is needed; each CTA starts only
// after finishing its own previous stage, so the polls are short). Measured
// on Qwen3-0.6B (tokens/s): waiting for a counter of all CTAs 1,387; polling
// at once 1,387 (the early polls slow the writers); one load's delay 1,466;
// two loads 1,446; a 300 / 700 ns sleep 1,454 / 1,345; backoff between polls
// slower still. Under tensor parallelism the readers of the other ranks'
// partials do the same on their own mailbox.
__device__ __forceinline__ bool stage_ready(const DecodeLoop& p, int st, Shared& sh) {
  const uint32_t v = ld_relaxed(p.sync + kStageDone + st);
  if (v == 0x9E3779B9u) sh.stop = sh.stop;  // a use of the value: the load completes
  return true;
}

// O-stage input: the attention output of every query head, the log-sum-exp
// merge of its nb block partials in block order (the arithmetic of
// attention.cu's final merge), written to xs as FP16.
// Blocks of a batch whose records (max, denominator, 8 numerators) one
// thread loads together.
constexpr int kMergeBatch = 4;

struct MergeRec {
  float m[kMergeBatch], l[kMergeBatch];
  float4 n0[kMergeBatch], n1[kMergeBatch];
};

// Records of blocks [b0, b0 + kMergeBatch) that exist (< nb), loads issued together.
__device__ __forceinline__ void merge_load(const float* hb, size_t block_stride, int d0, int b0,
                                           int nb, MergeRec& r) {
#pragma unroll
  for (int i = 0; i < kMergeBatch; ++i)
    if (b0 + i < nb) {
      const float* rec = hb + (size_t)(b0 + i) * block_stride;
      r.m[i] = __ldcg(rec);
      r.l[i] = __ldcg(rec + 1);
      r.n0[i] = __ldcg(reinterpret_cast<const float4*>(rec + 4 + d0));
      r.n1[i] = __ldcg(reinterpret_cast<const float4*>(rec + 8 + d0));
    }
}

// The block-order accumulation of loaded records (the arithmetic of the
// generic loop below).
__device__ __forceinline__ void merge_apply(const MergeRec& r, int b0, int nb, float M,
                                            float (&num)[8], float& den) {
#pragma unroll
  for (int i = 0; i < kMergeBatch; ++i)
    if (b0 + i < nb) {
      const float f = r.m[i] == -INFINITY ? 0.f : mi_exp(__fsub_rn(r.m[i], M));
      den = __fmaf_rn(r.l[i], f, den);
      num[0] = __fmaf_rn(r.n0[i].x, f, num[0]);
      num[1] = __fmaf_rn(r.n0[i].y, f, num[1]);
      num[2] = __fmaf_rn(r.n0[i].z, f, num[2]);
      num[3] = __fmaf_rn(r.n0[i].w, f, num[3]);
      num[4] = __fmaf_rn(r.n1[i].x, f, num[4]);
      num[5] = __fmaf_rn(r.n1[i].y, f, num[5]);
      num[6] = __fmaf_rn(r.n1[i].z, f, num[6]);
      num[7] = __fmaf_rn(r.n1[i].w, f, num[7]);
    }
}

__device__ void build_attn_input(const DecodeLoop& p, int nb, uint4* xs) {
  const int G = p.qh / p.kvh;
  const int kc = p.qh * HD / 8;
  const size_t block_stride = (size_t)G * kPart;
  for (int c = threadIdx.x; c < kc; c += kConsumers) {
    const int qi = c / (HD / 8);
    const int d0 = (c % (HD / 8)) * 8;
    const float* hb = p.attn_part + ((size_t)(qi / G) * p.attn_blocks * G + qi % G) * kPart;
    float M = -INFINITY;
    float num[8], den = 0.f;
#pragma unroll
    for (int e = 0; e < 8; ++e) num[e] = 0.f;
    if (nb <= 2 * kMergeBatch) {
      // Short caches: the maxima of every block and the first batch's
      // records are loaded together (one L2 round trip up to 4 blocks, two
      // up to 8; the loop below takes two to four).
      MergeRec r;
      float m2[kMergeBatch];
      merge_load(hb, block_stride, d0, 0, nb, r);
#pragma unroll
      for (int i = 0; i < kMergeBatch; ++i)
        if (kMergeBatch + i < nb) m2[i] = __ldcg(hb + (size_t)(kMergeBatch + i) * block_stride);
#pragma unroll
      for (int i = 0; i < kMergeBatch; ++i) {
        if (i < nb) M = fmaxf(M, r.m[i]);
        if (kMergeBatch + i < nb) M = fmaxf(M, m2[i]);
      }
      merge_apply(r, 0, nb, M, num, den);
      if (nb > kMergeBatch) {
        merge_load(hb, block_stride, d0, kMergeBatch, nb, r);
        merge_apply(r, kMergeBatch, nb, M, num, den);
      }
      uint4 v;
      __half2* hv = reinterpret_cast<__half2*>(&v);
#pragma unroll
      for (int i = 0; i < 4; ++i)
        hv[i] = __halves2half2(__float2half_rn(__fdiv_rn(num[2 * i], den)),
                               __float2half_rn(__fdiv_rn(num[2 * i + 1], den)));
      xs[c] = v;
      continue;
    }
#pragma unroll 4
    for (int b = 0; b < nb; ++b) M = fmaxf(M, __ldcg(hb + b * block_stride));
#pragma unroll 4
    for (int b = 0; b < nb; ++b) {
      const float* rec = hb + b * block_stride;
      const float mm = __ldcg(rec);
      const float f = mm == -INFINITY ? 0.f : mi_exp(__fsub_rn(mm, M));
      den = __fmaf_rn(__ldcg(rec + 1), f, den);
      const float4 n0 = __ldcg(reinterpret_cast<const float4*>(rec + 4 + d0));
      const float4 n1 = __ldcg(reinterpret_cast<const float4*>(rec + 8 + d0));
      num[0] = __fmaf_rn(n0.x, f, num[0]);
      num[1] = __fmaf_rn(n0.y, f, num[1]);
      num[2] = __fmaf_rn(n0.z, f, num[2]);
      num[3] = __fmaf_rn(n0.w, f, num[3]);
      num[4] = __fmaf_rn(n1.x, f, num[4]);
      num[5] = __fmaf_rn(n1.y, f, num[5]);
      num[6] = __fmaf_rn(n1.z, f, num[6]);
      num[7] = __fmaf_rn(n1.w, f, num[7]);
    }
    uint4 v;
    __half2* hv = reinterpret_cast<__half2*>(&v);
#pragma unroll
    for (int i = 0; i < 4; ++i)
      hv[i] = __halves2half2(__float2half_rn(__fdiv_rn(num[2 * i], den)),
                             __float2half_rn(__fdiv_rn(num[2 * i + 1], den)));
    xs[c] = v;
  }
  consumers_sync();
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

// L2 prefetch of tile `tile` of stage weights s (the byte ranges issue_tile
// copies): a hint with no completion, so HBM keeps streaming the weights
// ahead of the ring while the ring is full.
__device__ void prefetch_tile(const StageW& s, const Tiles& t, int tile) {
  const int i0 = t.first + tile * t.per_tile;
  const int cnt = min(t.per_tile, t.last - i0);
  const uint32_t rb = t.row_bytes;
  auto pf = [](const void* src, uint32_t bytes) {
    asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(src), "r"(bytes) : "memory");
  };
  if (s.pair) {
    pf(s.w[0] + (size_t)i0 * s.k, cnt * rb);
    pf(s.w[1] + (size_t)i0 * s.k, cnt * rb);
    return;
  }
  int seg_start = 0, done = 0;
  for (int seg = 0; seg < 3 && done < cnt; ++seg) {
    const int seg_end = seg_start + s.n[seg];
    const int a = max(i0 + done, seg_start), b = min(i0 + cnt, seg_end);
    if (a < b) {
      pf(s.w[seg] + (size_t)(a - seg_start) * s.k, (uint32_t)(b - a) * rb);
      done += b - a;
    }
    seg_start = seg_end;
  }
}

// A position in the producer's static schedule of weight tiles (every stage
// of every layer of every step, then the LM head).
struct TileCursor {
  int step = 0, layer = 0, j = 0, tile = -1;
  __device__ __forceinline__ static int stage_of(const DecodeLoop& p, int layer, int j) {
    return layer < p.layers ? (j == 0 ? kQKV : j == 1 ? kO : j == 2 ? kGU : kDown) : kLM;
  }
  // Moves to the next tile; false past the end of the schedule.
  __device__ bool next(const DecodeLoop& p, const Shared& sh) {
    ++tile;
    while (step < p.steps) {
      if (tile < sh.tiles[stage_of(p, layer, j)].count) return true;
      tile = 0;
      if (++j >= (layer < p.layers ? 4 : 1)) {
        j = 0;
        if (++layer > p.layers) {
          layer = 0;
          ++step;
        }
      }
    }
    return false;
  }
};

__device__ void produce(const DecodeLoop& p, const LoopLayer* layers, uint8_t* ring, Shared& sh) {
  const int S = p.slots;
  uint32_t g = 0;
  bool ok = true;
  // The L2 prefetch cursor runs p.l2_ahead tiles ahead of the copies.
  TileCursor pf;
  bool pf_live = true;
  for (int i = 0; i < p.l2_ahead && pf_live; ++i)
    if ((pf_live = pf.next(p, sh)))
      prefetch_tile(stage_weights(p, layers, pf.layer, TileCursor::stage_of(p, pf.layer, pf.j)),
                    sh.tiles[TileCursor::stage_of(p, pf.layer, pf.j)], pf.tile);
  for (int step = 0; ok && step < p.steps; ++step) {
    for (int layer = 0; ok && layer <= p.layers; ++layer) {
      const int nst = layer < p.layers ? 4 : 1;
      for (int j = 0; ok && j < nst; ++j) {
        const int st = layer < p.layers ? (j == 0 ? kQKV : j == 1 ? kO : j == 2 ? kGU : kDown)
                                        : kLM;
        const StageW s = stage_weights(p, layers, layer, st);
        const Tiles t = sh.tiles[st];
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
          if (pf_live && p.l2_ahead > 0 && (pf_live = pf.next(p, sh))) {
            const int pst = TileCursor::stage_of(p, pf.layer, pf.j);
            prefetch_tile(stage_weights(p, layers, pf.layer, pst), sh.tiles[pst], pf.tile);
          }
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

// A stage input: tagged vector x (+ x2 for the residual adds, or an
// embedding row), the norm weights, and where CTA 0 writes back the
// un-normalized input (hidden stream / residual).
struct StageIn {
  int mode;
  int k;
  const uint32_t* x;
  uint32_t xtag;
  const uint32_t* x2;
  uint32_t x2tag;
  long long x2_part;  // >= 0: x2 is the ranks' summed partials in this mailbox region
  int exchange;       // tensor parallelism: x2 comes from the other ranks (timed)
  const __half* embed;  // kEmbedNormIn: table row, null for an out-of-range token
  const __half* norm_w;
  uint32_t* wb;
  uint32_t wbtag;
  // DOWN on one GPU: the residual values of this CTA's rows, polled into
  // sh.res by the last res_n consumer threads beside the stage input
  const uint32_t* res;
  int res_first, res_n;
  uint32_t res_tag;
};

__device__ __forceinline__ uint4 add_chunk(int mode, const uint4& a, const uint4& b) {
  const __half2* ha = reinterpret_cast<const __half2*>(&a);
  const __half2* hb = reinterpret_cast<const __half2*>(&b);
  uint4 v;
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
  return v;
}

// Chunk c of the stage input before the norm (gemv.cu build_input roundings).
__device__ __forceinline__ uint4 input_chunk(const DecodeLoop& p, const StageIn& in, int c,
                                             Shared& sh) {
  if (in.mode == kAddNormIn || in.mode == kAddThenNormIn) {
    const Raw8 ra = raw8(in.x, c), rb = raw8(in.x2, c);
    return add_chunk(in.mode, take8_from(p, ra, in.x, c, in.xtag, sh),
                     take8_from(p, rb, in.x2, c, in.x2tag, sh));
  }
  if (in.mode == kEmbedNormIn)
    return in.embed ? __ldg(reinterpret_cast<const uint4*>(in.embed) + c) : make_uint4(0, 0, 0, 0);
  return take8(p, in.x, c, in.xtag, sh);
}

// One staged chunk's contribution to the canonical sum of squares
// (gemv.cu build_input): kAddNormIn squares the unrounded float sums
// (matvec2_add_rms_impl), kAddThenNormIn the rounded FP16 sums.
__device__ __forceinline__ float sq_chunk(int mode, const uint4& a, const uint4& b, float acc) {
  if (mode == kAddNormIn) {
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
    return acc;
  }
  if (mode == kAddThenNormIn) return chunk_sq(add_chunk(mode, a, b), acc);
  return chunk_sq(a, acc);
}

// Every warp, from the staged input in shared memory: the canonical sum of
// squares (lane l accumulates chunks l, l + 32, ... in order, loaded four at
// a time), reduced over the canonical lanes, and the RMSNorm scale, returned
// to every lane. Each warp computes the same value, so no barrier is needed
// to share it.
__device__ float warp_scale(const DecodeLoop& p, int mode, const uint4* xs, const uint4* xs2,
                            int k) {
  const int lane = threadIdx.x & 31;
  const int kc = k >> 3;
  const bool two = mode == kAddNormIn || mode == kAddThenNormIn;
  float acc = 0.f;
  int c = lane;
  for (; c + 96 < kc; c += 128) {
    uint4 a[4], b[4];
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      a[j] = xs[c + 32 * j];
      b[j] = two ? xs2[c + 32 * j] : a[j];
    }
#pragma unroll
    for (int j = 0; j < 4; ++j) acc = sq_chunk(mode, a[j], b[j], acc);
  }
  for (; c < kc; c += 32) acc = sq_chunk(mode, xs[c], two ? xs2[c] : xs[c], acc);
  return rms_scale(canon_reduce(acc, canon_lanes(k)), k, p.eps);
}

__device__ __forceinline__ uint4 normalize_chunk(const uint4& v, const uint4& g, float scale) {
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
  return o;
}

// Tensor parallelism, the sliced exchange input: see build_input. `part` is
// shared-memory scratch (the normalized-input buffer, free until the
// normalization). Kept out of line so that the one-GPU input code keeps its
// register allocation.
__device__ __noinline__ void tp_slice_sum(const DecodeLoop& p, const StageIn& in, int kc,
                                          float* part, Shared& sh) {
  const int tid = threadIdx.x;
  // Tensor parallelism, sliced: this CTA sums only its slice of the
  // ranks' partials (one thread per (chunk, rank), every load in flight
  // together, then the rank-order sum: the same additions as
  // take_partials8) and publishes it as tagged FP16 in t_attn_o, which
  // nothing else writes under tensor parallelism. Every CTA then stages
  // the summed vector from there like a one-GPU input: a CTA reads its
  // slice's tp partials and the hidden vector once, instead of tp copies
  // of the vector.
  const int c0 = (int)((long long)kc * blockIdx.x / gridDim.x);
  const int c1 = (int)((long long)kc * (blockIdx.x + 1) / gridDim.x);
  const int pairs = (c1 - c0) * p.tp;
  for (int i = tid; i < pairs; i += kConsumers) {
    const int c = c0 + i / p.tp, r = i - (i / p.tp) * p.tp;
    const unsigned long long* q = p.mbox + (size_t)in.x2_part + (size_t)r * p.hidden + 8 * c;
    unsigned long long w[8];
    PollClock clock;
    while (true) {
      bool ok = true;
#pragma unroll
      for (int e = 0; e < 8; ++e) {
        w[e] = ld_sys_u64(q + e);
        ok &= (uint32_t)(w[e] >> 32) == in.x2tag;
      }
      if (ok || !clock.keep_going(p, sh)) break;
    }
#pragma unroll
    for (int e = 0; e < 8; ++e) part[8 * i + e] = __uint_as_float((uint32_t)w[e]);
  }
  consumers_sync();
  for (int cc = tid; cc < c1 - c0; cc += kConsumers) {
    float acc[8];
    for (int r = 0; r < p.tp; ++r)
#pragma unroll
      for (int e = 0; e < 8; ++e) {
        const float v = part[8 * (cc * p.tp + r) + e];
        acc[e] = r == 0 ? v : __fadd_rn(acc[e], v);
      }
    uint4 v;
    __half2* hv = reinterpret_cast<__half2*>(&v);
#pragma unroll
    for (int i = 0; i < 4; ++i) hv[i] = __floats2half2_rn(acc[2 * i], acc[2 * i + 1]);
    put8(p.t_attn_o, c0 + cc, v, in.x2tag);
  }
}

// Builds the stage input (k halves) with the prologue of the GEMV family
// (gemv.cu build_input): the same roundings and the canonical sum of
// squares. Every thread stages its chunks of the tagged vector(s) into xs
// (xs2) in shared memory (one L2 round trip; the tags validate each word);
// one barrier, which also takes the CTA's uniform decision to continue
// (false when the kernel is aborting); then, for the norm modes, every warp
// computes the scale itself and the chunks are normalized into xn, followed
// by a second barrier. Stages without a norm read xs directly.
template <bool TP>
__device__ bool build_input(const DecodeLoop& p, const StageIn& in, int wait_st, uint4* xs,
                            uint4* xs2, uint4* xn, Shared& sh) {
  const int tid = threadIdx.x;
  const int kc = in.k >> 3;
  const bool two = in.mode == kAddNormIn || in.mode == kAddThenNormIn;
  const bool norm = in.mode != kPlainIn;
  const uint4* g4 = reinterpret_cast<const uint4*>(in.norm_w);
  // thread 0 times the input of a stage fed by the other ranks' partials
  // (this rank's wait on the exchange, read back by mi_qwen3_exchange_wait)
  const uint64_t t_in = (in.exchange && tid == 0) ? pipe::global_ns() : 0;
  if (wait_st >= 0 && tid < kc) stage_ready(p, wait_st, sh);  // one L2 round trip of delay before the polls
  if (tid == 0) MI_TRACE_IN(9);
  if (in.res && tid >= kConsumers - in.res_n) {
    const int i = tid - (kConsumers - in.res_n);
    sh.res[i] = take1(p, in.res, in.res_first + i, in.res_tag, sh);
  }
  uint4 g_first = make_uint4(0, 0, 0, 0);
  if (norm && tid < kc) g_first = __ldg(g4 + tid);
  const bool wb = in.wb && blockIdx.x == 0;
  const uint32_t* x2 = in.x2;
  if (TP && two && in.x2_part >= 0 && p.xslice) {
    tp_slice_sum(p, in, kc, reinterpret_cast<float*>(xn), sh);
    x2 = p.t_attn_o;
  }
  if (two && in.x2_part >= 0 && !(TP && p.xslice)) {
    for (int c = tid; c < kc; c += kConsumers) {
      const Raw8 ra = raw8(in.x, c);
      const uint4 b = take_partials8(p, (size_t)in.x2_part, c, in.x2tag, sh);
      const uint4 a = take8_from(p, ra, in.x, c, in.xtag, sh);
      xs[c] = a;
      xs2[c] = b;
      if (wb) put8(in.wb, c, add_chunk(in.mode, a, b), in.wbtag);
    }
  } else if (two) {
    for (int c = tid; c < kc; c += kConsumers) {
      const Raw8 ra = raw8(in.x, c), rb = raw8(x2, c);
      const uint4 a = take8_from(p, ra, in.x, c, in.xtag, sh);
      const uint4 b = take8_from(p, rb, x2, c, in.x2tag, sh);
      xs[c] = a;
      xs2[c] = b;
      if (wb) put8(in.wb, c, add_chunk(in.mode, a, b), in.wbtag);
    }
  } else if (in.mode == kEmbedNormIn) {
    for (int c = tid; c < kc; c += kConsumers) {
      const uint4 v = input_chunk(p, in, c, sh);
      xs[c] = v;
      if (wb) put8(in.wb, c, v, in.wbtag);
    }
  } else {
    for (int c = tid; c < kc; c += kConsumers) {
      const uint4 v = take8(p, in.x, c, in.xtag, sh);
      xs[c] = v;
      if (wb) put8(in.wb, c, v, in.wbtag);
    }
  }
  if (consumers_any(sh.abort)) return false;
  if (in.exchange && tid == 0) sh.mbox_ns += pipe::global_ns() - t_in;
  if (tid == 0) MI_TRACE_IN(10);
  if (norm) {
    // every warp computes the scale when a lane's chain is short; for wide
    // inputs one warp does and shares it (the redundant shared-memory reads
    // of every consumer warp would cost more than the extra barrier)
    const bool every_warp = kc <= 4 * 32;
    float scale = 0.f;
    if (every_warp || tid < 32) scale = warp_scale(p, in.mode, xs, xs2, in.k);
    if (!every_warp) {
      if (tid == 0) sh.scale = scale;
      consumers_sync();
      scale = sh.scale;
    }
    if (tid == 0) MI_TRACE_IN(15);
    for (int c = tid; c < kc; c += kConsumers) {
      const uint4 v = two ? add_chunk(in.mode, xs[c], xs2[c]) : xs[c];
      xn[c] = normalize_chunk(v, c == tid ? g_first : __ldg(g4 + c), scale);
    }
    consumers_sync();
  }
  return true;
}

// ---- consumers: rows from the ring --------------------------------------------------
// Stage output of one reduced item (lane-local).
template <int ST>
__device__ __forceinline__ void put_item(const DecodeLoop& p, const StageW& s, int item, float a0,
                                         float a1, const __half* res, int res_first,
                                         uint32_t tag, uint32_t& best_key, uint32_t& best_idx) {
  if (ST == kQKV) {
    put1(p.t_qkv, item, __float2half_rn(a0), tag);
  } else if (ST == kO) {
    if (p.tp > 1) {
      const MailboxLayout mb = mailbox_layout(p.tp, p.hidden, gridDim.x);
      push_partial(p, mb.o, item, a0, tag);
    } else {
      put1(p.t_attn_o, item, __float2half_rn(a0), tag);
    }
  } else if (ST == kGU) {
    const float gv = __half2float(__float2half_rn(a0));
    const float uv = __half2float(__float2half_rn(a1));
    put1(p.t_act, item, __float2half_rn(silu_mul(gv, uv)), tag);
  } else if (ST == kDown) {
    if (p.tp > 1) {
      const MailboxLayout mb = mailbox_layout(p.tp, p.hidden, gridDim.x);
      push_partial(p, mb.d, item, a0, tag);
    } else {
      const int local = item - res_first;
      put1(p.t_hidden, item, __hadd(res[local], __float2half_rn(a0)), tag);
    }
  } else {
    const __half h0 = __float2half_rn(a0);
    p.logits[item] = h0;
    const float v = __half2float(h0);
    if (isfinite(v) && argmax_better(argmax_key(v), (uint32_t)item, best_key, best_idx)) {
      best_key = argmax_key(v);
      best_idx = (uint32_t)item;
    }
  }
}

// P consecutive rows (gate/up pairs for GU) reduced together: P independent
// canonical FMA chains per lane and interleaved butterflies. Lane q writes
// row q. Rows past `nr` repeat row 0 and are dropped.
template <int ST, int P>
__device__ __forceinline__ void rows_group(const DecodeLoop& p, const StageW& s, const uint4* xs,
                                           const __half* res, int res_first, uint32_t tag,
                                           const uint8_t* base, int r0, int nr, int cnt,
                                           uint32_t row_bytes, int item0, int kc, int lanes,
                                           uint32_t& best_key, uint32_t& best_idx) {
  constexpr bool kPair = ST == kGU;
  const int lane = threadIdx.x & 31;
  const uint4* w[P];
  const uint4* u[P];
#pragma unroll
  for (int q = 0; q < P; ++q) {
    const int r = r0 + (q < nr ? q : 0);
    w[q] = reinterpret_cast<const uint4*>(base + (size_t)r * row_bytes);
    u[q] = reinterpret_cast<const uint4*>(base + (size_t)(cnt + r) * row_bytes);
  }
  float a[P], b[P];
#pragma unroll
  for (int q = 0; q < P; ++q) a[q] = b[q] = 0.f;
  // Full blocks of kB chunks per lane with every shared-memory load issued
  // before the block's FMA chains, then single chunks (chunk order per lane
  // is unchanged).
  constexpr int kB = (P == 1 && !kPair) ? 4 : (P == 2 && !kPair) ? 2 : 1;
  int c = lane;
  for (; c + 32 * (kB - 1) < kc; c += 32 * kB) {
    uint4 xv[kB], wv[P][kB], uv[P][kB];
#pragma unroll
    for (int j = 0; j < kB; ++j) {
      xv[j] = xs[c + 32 * j];
#pragma unroll
      for (int q = 0; q < P; ++q) {
        wv[q][j] = w[q][c + 32 * j];
        if (kPair) uv[q][j] = u[q][c + 32 * j];
      }
    }
#pragma unroll
    for (int j = 0; j < kB; ++j)
#pragma unroll
      for (int q = 0; q < P; ++q) {
        a[q] = chunk_dot(xv[j], wv[q][j], a[q]);
        if (kPair) b[q] = chunk_dot(xv[j], uv[q][j], b[q]);
      }
  }
  for (; c < kc; c += 32) {
    const uint4 xv = xs[c];
#pragma unroll
    for (int q = 0; q < P; ++q) {
      a[q] = chunk_dot(xv, w[q][c], a[q]);
      if (kPair) b[q] = chunk_dot(xv, u[q][c], b[q]);
    }
  }
  for (int o = lanes >> 1; o >= 1; o >>= 1) {
#pragma unroll
    for (int q = 0; q < P; ++q) {
      a[q] = __fadd_rn(a[q], __shfl_xor_sync(0xffffffffu, a[q], o));
      if (kPair) b[q] = __fadd_rn(b[q], __shfl_xor_sync(0xffffffffu, b[q], o));
    }
  }
  if (lanes < 32) {
#pragma unroll
    for (int q = 0; q < P; ++q) {
      a[q] = __shfl_sync(0xffffffffu, a[q], 0);
      if (kPair) b[q] = __shfl_sync(0xffffffffu, b[q], 0);
    }
  }
#pragma unroll
  for (int q = 0; q < P; ++q)
    if (lane == q && q < nr)
      put_item<ST>(p, s, item0 + q, a[q], b[q], res, res_first, tag, best_key, best_idx);
}

// Reduces this CTA's rows of stage ST from the ring: groups of P local rows
// (never straddling a tile) go round-robin to the consumer warps; every
// warp waits for every tile in order and releases it when done. `g` is the
// running tile counter.
template <int ST, int P>
__device__ void reduce_rows_p(const DecodeLoop& p, const StageW& s, const Tiles& t,
                              const uint4* xs, const uint8_t* ring, Shared& sh, uint32_t& g,
                              uint32_t tag, uint32_t& best_key, uint32_t& best_idx) {
  const int lane = threadIdx.x & 31;
  const int warp = threadIdx.x >> 5;
  const int kc = s.k >> 3;
  const int lanes = canon_lanes(s.k);
  const int S = p.slots;
  const int rows = t.last - t.first;
  for (int tile = 0; tile < t.count; ++tile, ++g) {
    const int slot = (int)(g % S);
    const uint32_t use = g / S;
    if (threadIdx.x == 0 && tile == 0) MI_TRACE_CUR(14);
    const bool ok = ring_wait(&sh.full[slot], use & 1u, sh, kCodeFull | ST);
    if (threadIdx.x == 0 && tile == 0) MI_TRACE_CUR(5);
    const int l0 = tile * t.per_tile;
    const int cnt = min(t.per_tile, rows - l0);
    if (ok) {
      const uint8_t* base = ring + (size_t)slot * p.slot_bytes;
      const int g0 = l0 / P;
      const int g1 = (l0 + cnt + P - 1) / P;
      for (int gi = g0 + (warp - g0 % kConsumerWarps + kConsumerWarps) % kConsumerWarps; gi < g1;
           gi += kConsumerWarps) {
        const int r0 = gi * P - l0;
        rows_group<ST, P>(p, s, xs, sh.res, t.first, tag, base, r0, min(P, cnt - r0), cnt, t.row_bytes,
                          t.first + l0 + r0,
                          kc, lanes, best_key, best_idx);
      }
    }
    __syncwarp();
    if (threadIdx.x == 0 && tile == 0) MI_TRACE_CUR(6);
    if (lane == 0) mbar_arrive(&sh.empty[slot]);
  }
  if (threadIdx.x == 0) MI_TRACE_CUR(7);
}

template <int ST>
__device__ void reduce_rows(const DecodeLoop& p, const StageW& s, const uint4* xs,
                            const uint8_t* ring, Shared& sh, uint32_t& g, uint32_t tag,
                            uint32_t& best_key, uint32_t& best_idx) {
  const Tiles t = sh.tiles[ST];
  const int rows = t.last - t.first;
  if (ST == kLM && t.per_tile % 4 == 0 && rows >= 4 * kConsumerWarps)
    reduce_rows_p<ST, 4>(p, s, t, xs, ring, sh, g, tag, best_key, best_idx);
  else if (t.per_tile % 2 == 0 && rows >= 16)
    reduce_rows_p<ST, 2>(p, s, t, xs, ring, sh, g, tag, best_key, best_idx);
  else
    reduce_rows_p<ST, 1>(p, s, t, xs, ring, sh, g, tag, best_key, best_idx);
}

// ---- consumers: attention units (warps 3..10) -------------------------------------------
// Thread index within the attention warps.
__device__ __forceinline__ int atid() { return (int)threadIdx.x - kAttnBase; }

// One thread: TMA loads of the K and V tile of KV head g_kv at positions
// [j0, j0 + kTile) (four 64-column halves), completing on `bar`, whose
// expected bytes the caller has registered. The proxy fence orders the
// generic-proxy writes before it (K/V rows written in earlier steps, and the
// stream accumulators this CTA kept in the tile region) before the copies.
template <int G>
__device__ __forceinline__ void issue_kv_tile(const DecodeLoop& p, int layer, int g_kv, int j0,
                                              AttnSmem<G>& sm, uint64_t* bar) {
  asm volatile("fence.proxy.async;" ::: "memory");
  const uint8_t* maps = static_cast<const uint8_t*>(p.kv_maps) + (size_t)layer * 256;
  tma_load_2d(&sm.k[0][0][0], maps, bar, g_kv * HD, j0);
  tma_load_2d(&sm.k[1][0][0], maps, bar, g_kv * HD + 64, j0);
  tma_load_2d(&sm.v[0][0][0], maps + 128, bar, g_kv * HD, j0);
  tma_load_2d(&sm.v[1][0][0], maps + 128, bar, g_kv * HD + 64, j0);
}
constexpr uint32_t kKvTileBytes = 2u * kTile * HD * 2u;

// After its QKV input, a CTA that owns attention unit blockIdx.x prefetches
// that unit's first key tile (final: written in earlier steps; the row of
// the new position is stale and is taken from this step's K/V instead), the
// layer's QK-norm weights and the RoPE terms of the position into shared
// memory, so the attention stage finds them there: one thread issues the
// TMA tile loads and 1-D bulk copies of the rest, all completing on
// sh.kv_full. Returns whether this CTA issued them (uniform over the CTA).
template <int G>
__device__ bool attention_prefetch(const DecodeLoop& p, int layer, const LoopLayer& L, int pos,
                                   AttnSmem<G>& sm, Shared& sh) {
  const int nb = (pos + p.block) / p.block;
  if ((int)blockIdx.x >= p.kvh * nb) return false;
  if (threadIdx.x != kAttnBase) return true;
  const int g_kv = blockIdx.x / nb, b = blockIdx.x % nb;
  pipe::mbar_expect_tx(&sh.kv_full, kKvTileBytes + 2u * (HD * 2u) +
                                        (p.rope ? (uint32_t)sizeof(sm.rope) : 0u));
  issue_kv_tile<G>(p, layer, g_kv, b * p.block, sm, &sh.kv_full);
  pipe::bulk_g2s(sm.qn_w, L.q_norm, HD * 2, &sh.kv_full);
  pipe::bulk_g2s(sm.kn_w, L.k_norm, HD * 2, &sh.kv_full);
  if (p.rope)
    pipe::bulk_g2s(sm.rope, p.rope + (size_t)pos * (HD / 2), (uint32_t)sizeof(sm.rope),
                   &sh.kv_full);
  return true;
}

// QK-norm + RoPE of one head half-warp from the prefetched shared copies
// (the RoPE row of `pos` is passed as a one-row table at position 0).
template <int G>
__device__ __forceinline__ void head_rope(const DecodeLoop& p, const AttnSmem<G>& sm,
                                          const uint4& raw, const __half* w, int pos,
                                          unsigned mask, float (&out)[8]) {
  if (p.rope)
    norm_rope_half(raw, w, 0u, p.theta, p.eps, p.round_norm != 0, mask, sm.rope, out);
  else
    norm_rope_half(raw, w, (uint32_t)pos, p.theta, p.eps, p.round_norm != 0, mask, nullptr, out);
}

// Row j of a swizzled tile half-pair as 16-byte chunks: chunk c (0..15).
__device__ __forceinline__ uint4 tile_chunk(const __half (*t)[kTile][64], int j, int c) {
  return reinterpret_cast<const uint4*>(&t[c >> 3][j][0])[(c & 7) ^ (j & 7)];
}

// Canonical score of FP16 query q (16 chunks) with the K row of tile key j
// (or the new row): one partial per chunk (8 sequential mixed-precision
// FMAs; both operands are FP16 values, so this is the FP32 FMA of the
// widened operands), then the 16-lane butterfly tree in registers.
template <int G>
__device__ __forceinline__ float key_score(const AttnSmem<G>& sm, int g, int j, bool fresh) {
  const uint4* q = reinterpret_cast<const uint4*>(sm.q[g]);
  const uint4* nk = reinterpret_cast<const uint4*>(sm.new_k);
  float d[8];
#pragma unroll
  for (int c = 0; c < 8; ++c) d[c] = chunk_dot(q[c], fresh ? nk[c] : tile_chunk(sm.k, j, c), 0.f);
#pragma unroll
  for (int c = 0; c < 8; ++c)  // the tree's first level as the upper partials arrive
    d[c] = __fadd_rn(d[c], chunk_dot(q[c + 8], fresh ? nk[c + 8] : tile_chunk(sm.k, j, c + 8), 0.f));
#pragma unroll
  for (int step = 4; step >= 1; step >>= 1)
#pragma unroll
    for (int c = 0; c < step; ++c) d[c] = __fadd_rn(d[c], d[c + step]);
  return d[0];
}

// One flash-decode unit: KV head g_kv, key block b of nb, run by the 256
// attention threads (warps 3..10). The arithmetic is attention.cu's
// attention_decode_kernel with the fused front end: kStreams interleaved
// online-softmax streams per block (stream s takes the block's keys s,
// s + 8, ... in order), merged in stream order into the block partial. The
// work is laid out for latency: one thread per (key, head) score; a key's
// running maximum is its stream's prefix maximum (exact in any order), so
// every key's pair of exponentials is computed independently; only the
// accumulations stay sequential in key order, one thread per (stream, head,
// 8 dims). Tiles past the prefetched one arrive by TMA on sh.kv_tile.
template <int G>
__device__ void attention_unit(const DecodeLoop& p, int layer, const LoopLayer& L, int g_kv,
                               int b, int nb, int pos, bool prefetched, uint32_t kv_parity,
                               uint32_t& tile_uses, uint32_t qkv_tag, AttnSmem<G>& sm,
                               Shared& sh) {
  constexpr int R = (kStreams * G * 16 + kAttnThreads - 1) / kAttnThreads;  // accumulators per thread
  const int t = atid();
  const int li = t & 15;
  const int begin = b * p.block;
  const int end = min(pos + 1, begin + p.block);
  const int ntiles = (end - begin + kTile - 1) / kTile;

  // every CTA's QKV rows are out (the tags then validate each word); the
  // prefetched copies (norms, RoPE row, first key tile) have landed
  if (t == 0) stage_ready(p, kQKV, sh);
  if (prefetched) copies_wait(&sh.kv_full, kv_parity, kCodeKv);
  attn_sync();
  {
    const int hq = t >> 4;  // one query head per half-warp
    if (hq < G) {
      const unsigned mask = ((t >> 5) * 2 + 1 < G) ? 0xffffffffu : 0x0000ffffu;
      const uint4 raw = take8(p, p.t_qkv, (g_kv * G + hq) * (HD / 8) + li, qkv_tag, sh);
      float qv[8];
      head_rope<G>(p, sm, raw, sm.qn_w, pos, mask, qv);
      uint4 qq;
      __half2* hq2 = reinterpret_cast<__half2*>(&qq);
#pragma unroll
      for (int i = 0; i < 4; ++i) hq2[i] = __floats2half2_rn(qv[2 * i], qv[2 * i + 1]);
      reinterpret_cast<uint4*>(sm.q[hq])[li] = qq;
    }
  }
  if (pos >= begin && pos < end && t >= kAttnThreads - 16) {
    const int kc0 = (p.qh * HD + g_kv * HD) / 8;
    const uint4 raw = take8(p, p.t_qkv, kc0 + li, qkv_tag, sh);
    const uint4 vv = take8(p, p.t_qkv, kc0 + p.kvh * HD / 8 + li, qkv_tag, sh);
    float kv[8];
    head_rope<G>(p, sm, raw, sm.kn_w, pos, 0xffff0000u, kv);
    uint4 kk;
    __half2* hk = reinterpret_cast<__half2*>(&kk);
#pragma unroll
    for (int i = 0; i < 4; ++i) hk[i] = __floats2half2_rn(kv[2 * i], kv[2 * i + 1]);
    const size_t row = (size_t)pos * p.kvh * HD + (size_t)g_kv * HD;
    reinterpret_cast<uint4*>(L.k_cache + row)[li] = kk;
    reinterpret_cast<uint4*>(L.v_cache + row)[li] = vv;
    reinterpret_cast<uint4*>(sm.new_k)[li] = kk;
    reinterpret_cast<uint4*>(sm.new_v)[li] = vv;
  }
  if (t < kStreams * G) sm.m[0][t / G][t % G] = -INFINITY;
  if (t == 0) MI_TRACE_CUR(5);

  float acc[R][8], l[R];
#pragma unroll
  for (int r = 0; r < R; ++r) {
    l[r] = 0.f;
#pragma unroll
    for (int e = 0; e < 8; ++e) acc[r][e] = 0.f;
  }
  const float scale = __frcp_rn(__fsqrt_rn((float)HD));

  for (int tl = 0; tl < ntiles; ++tl) {
    const int j0 = begin + tl * kTile;
    const int cnt = min(end, j0 + kTile) - j0;
    const int cur = tl & 1;
    attn_sync();  // the front (tl = 0) or the previous tile's reads are done
    if (tl > 0 || !prefetched) {
      if (t == 0) {
        pipe::mbar_expect_tx(&sh.kv_tile, kKvTileBytes);
        issue_kv_tile<G>(p, layer, g_kv, j0, sm, &sh.kv_tile);
      }
      copies_wait(&sh.kv_tile, tile_uses & 1u, kCodeKv | 1u);
      ++tile_uses;
    }
    if (t == 0 && tl == 0) MI_TRACE_CUR(6);
    // scores, one thread per (key, head)
    for (int idx = t; idx < kTile * G; idx += kAttnThreads) {
      const int j = idx & (kTile - 1), g = idx / kTile;
      if (j < cnt) sm.sc[g][j] = __fmul_rn(key_score<G>(sm, g, j, j0 + j == pos), scale);
    }
    attn_sync();
    if (t == 0 && tl == 0) MI_TRACE_CUR(11);
    // prefix maxima and the two exponentials of every key
    for (int idx = t; idx < kTile * G; idx += kAttnThreads) {
      const int j = idx & (kTile - 1), g = idx / kTile, st = j & (kStreams - 1);
      if (j < cnt) {
        // the stream's earlier keys of the tile, loaded together
        float prev[kTile / kStreams];
#pragma unroll
        for (int i = 0; i < kTile / kStreams; ++i) prev[i] = sm.sc[g][st + kStreams * i];
        float mp = sm.m[cur][st][g];
#pragma unroll
        for (int i = 0; i < kTile / kStreams; ++i)
          if (st + kStreams * i < j) mp = fmaxf(mp, prev[i]);
        const float sc = sm.sc[g][j];
        const float mn = fmaxf(mp, sc);
        sm.pa[g][j] = mi_exp(__fsub_rn(mp, mn));
        sm.pc[g][j] = mi_exp(__fsub_rn(sc, mn));
        if (j + kStreams >= cnt) sm.m[cur ^ 1][st][g] = mn;  // the stream's last key here
      } else if (j < kStreams) {
        sm.m[cur ^ 1][j][g] = sm.m[cur][j][g];  // a stream with no key in this tile
      }
    }
    attn_sync();
    if (t == 0 && tl == 0) MI_TRACE_CUR(12);
    // accumulations in key order, one thread per (stream, head, 8 dims)
#pragma unroll
    for (int r = 0; r < R; ++r) {
      const int idx = t + r * kAttnThreads;
      const int st = (idx >> 4) & (kStreams - 1), g = idx >> 7;
      if (g < G) {
#pragma unroll
        for (int i = 0; i < kTile / kStreams; ++i) {
          const int j = st + kStreams * i;
          if (j >= cnt) break;
          const float a = sm.pa[g][j], c = sm.pc[g][j];
          const uint4 vv = j0 + j == pos ? reinterpret_cast<const uint4*>(sm.new_v)[li]
                                         : tile_chunk(sm.v, j, li);
          const __half2* hv = reinterpret_cast<const __half2*>(&vv);
#pragma unroll
          for (int i = 0; i < 4; ++i) {
            const float2 f = __half22float2(hv[i]);
            acc[r][2 * i] = __fmaf_rn(acc[r][2 * i], a, __fmul_rn(c, f.x));
            acc[r][2 * i + 1] = __fmaf_rn(acc[r][2 * i + 1], a, __fmul_rn(c, f.y));
          }
          l[r] = __fmaf_rn(l[r], a, c);
        }
      }
    }
    if (t == 0 && tl == 0) MI_TRACE_CUR(13);
  }
  attn_sync();  // every tile read is done: the tile region takes the accumulators
  if (t == 0) MI_TRACE_CUR(7);

  // Stream merge (stream order) -> block partial; the factors once per (stream, head).
  float* accs = reinterpret_cast<float*>(&sm.k[0][0][0]);  // [kStreams][G][HD]
  const int fin = ntiles & 1;
#pragma unroll
  for (int r = 0; r < R; ++r) {
    const int idx = t + r * kAttnThreads;
    const int st = (idx >> 4) & (kStreams - 1), g = idx >> 7;
    if (g < G) {
#pragma unroll
      for (int e = 0; e < 8; ++e) accs[(st * G + g) * HD + 8 * li + e] = acc[r][e];
      if (li == 0) sm.l[st][g] = l[r];
    }
  }
  attn_sync();
  if (t < kStreams * G) {
    const int st = t / G, g = t % G;
    float M = -INFINITY;
#pragma unroll
    for (int u = 0; u < kStreams; ++u) M = fmaxf(M, sm.m[fin][u][g]);
    const float ms = sm.m[fin][st][g];
    sm.f[st][g] = ms == -INFINITY ? 0.f : mi_exp(__fsub_rn(ms, M));
    if (st == 0) sm.M[g] = M;
  }
  attn_sync();
  // Block partial (max, denominator, numerators) of every head; the O stage
  // merges the blocks.
  float* part = p.attn_part + ((size_t)g_kv * p.attn_blocks + b) * G * kPart;
  for (int idx = t; idx < G * HD; idx += kAttnThreads) {
    const int g = idx / HD, d = idx - g * HD;
    float num = 0.f, den = 0.f;
#pragma unroll
    for (int st = 0; st < kStreams; ++st) {
      num = __fmaf_rn(accs[(st * G + g) * HD + d], sm.f[st][g], num);
      den = __fmaf_rn(sm.l[st][g], sm.f[st][g], den);
    }
    part[g * kPart + 4 + d] = num;
    if (d == 0) {
      part[g * kPart] = sm.M[g];
      part[g * kPart + 1] = den;
    }
  }
  if (t == 0) MI_TRACE_CUR(8);
  attn_sync();  // partial written; shared state is reused by the next unit
  if (t == 0) red_release_add(p.sync + kUnitsDone, 1u);
}

// Bytes of one hidden-size FP16 vector in shared memory.
__host__ __device__ size_t x2_bytes(int hidden) { return ((size_t)hidden * 2 + 127) / 128 * 128; }

// Bytes of the shared-memory copy of the layer table.
__host__ __device__ size_t layer_table_bytes(int layers) {
  return ((size_t)layers * sizeof(LoopLayer) + 127) / 128 * 128;
}

// TP: the tensor-parallel instantiation (mailbox exchanges); the one-GPU one
// carries none of that code.
template <int G, bool TP>
__global__ void __launch_bounds__(kThreads, 1) decode_loop_kernel(DecodeLoop params) {
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  __shared__ Shared sh;
  // Parameters live in shared memory: a persistent kernel would otherwise
  // miss the constant cache on them at every stage.
  __shared__ DecodeLoop p;
  if (threadIdx.x == 0) p = params;
  __syncthreads();
  // 1024-byte aligned base (the swizzled attention tiles need it; the plan
  // reserves the slack)
  uint8_t* smem = smem_raw + ((1024u - (pipe::smem_u32(smem_raw) & 1023u)) & 1023u);
  uint8_t* ring = smem;
  uint4* xs = reinterpret_cast<uint4*>(smem + (size_t)p.slots * p.slot_bytes);
  AttnSmem<G>& asm_ = *reinterpret_cast<AttnSmem<G>*>(smem + (size_t)p.slots * p.slot_bytes +
                                                        p.x_bytes);
  LoopLayer* lay = reinterpret_cast<LoopLayer*>(smem + (size_t)p.slots * p.slot_bytes + p.x_bytes +
                                                (sizeof(AttnSmem<G>) + 127) / 128 * 128);
  // second operand of the residual-add inputs (hidden halves)
  uint4* xs2 = reinterpret_cast<uint4*>(reinterpret_cast<uint8_t*>(lay) +
                                        layer_table_bytes(p.layers));
  // normalized stage input of the norm stages (hidden halves)
  uint4* xn = reinterpret_cast<uint4*>(reinterpret_cast<uint8_t*>(xs2) + x2_bytes(p.hidden));
  const int tid = threadIdx.x;
  {
    // per-layer pointer table -> shared memory (read at every stage)
    const int words = p.layers * (int)(sizeof(LoopLayer) / 8);
    const unsigned long long* src = reinterpret_cast<const unsigned long long*>(p.layer);
    unsigned long long* dst = reinterpret_cast<unsigned long long*>(lay);
    for (int i = tid; i < words; i += kThreads) dst[i] = src[i];
  }
  if (tid == 0) {
#ifdef MI_TRACE_TWICE
    g_trace_alt = 0;
#endif
    for (int st = 0; st < 5; ++st) sh.tiles[st] = tiles_of(p, stage_weights(p, lay, 0, st));
    sh.stop = 0;
    sh.astop = 0;
    sh.mbox_ns = 0;
    for (int s = 0; s < p.slots; ++s) {
      pipe::mbar_init(&sh.full[s], 1);
      pipe::mbar_init(&sh.empty[s], kConsumerWarps);
    }
    pipe::mbar_init(&sh.kv_full, 1);
    pipe::mbar_init(&sh.kv_tile, 1);
    sh.abort = 0;
    pipe::fence_mbar_init();
  }
  __syncthreads();

  if (tid >= kConsumers) {
    if (tid == kConsumers) produce(p, lay, ring, sh);
    return;
  }

  const uint32_t len0 = __ldcg(p.dev_len);
  uint32_t token = __ldcg(p.toks + len0);
  uint32_t g = 0;
  uint32_t units_total = 0;  // attention units published so far (all CTAs agree)
  uint32_t kv_uses = 0;      // attention prefetches completed on sh.kv_full
  uint32_t tile_uses = 0;    // key tiles completed on sh.kv_tile (attention warps)
  const uint32_t grid = gridDim.x;
  const int warp = tid >> 5, lane = tid & 31;
  for (int step = 0; step < p.steps; ++step) {
    const int pos = (int)len0 + step;
    const int nb = (pos + p.block) / p.block;  // key blocks: ceil((pos + 1) / block)
    for (int layer = 0; layer < p.layers; ++layer) {
      const LoopLayer& L = lay[layer];
      const uint32_t ls = (uint32_t)(step * p.layers + layer);  // layer-step of this launch
      const uint32_t e = p.epoch0 + ls;                             // its tag epoch
      // hidden stream read by GU: under tensor parallelism every QKV stage
      // writes it back (it is assembled from the ranks' down partials there)
      const uint32_t hidden_in = (layer == 0 || p.tp > 1) ? tagv(e, 0) : tagv(e - 1u, 1);
      uint32_t bk = 0, bi = 0xFFFFFFFFu;
      bool kv_issued = false;  // this CTA's attention prefetch of the layer
      // QKV (layer 0: the embedding row, written back as the hidden stream)
      {
        if (tid == 0) { MI_TRACE(step, layer * 5 + 0, 0); MI_TRACE_SET(step, layer * 5 + 0); }
        const StageW s = stage_weights(p, lay, layer, kQKV);
        StageIn in = {};
        in.x2_part = -1;
        in.k = p.hidden;
        in.norm_w = L.in_norm;
        if (layer == 0) {
          const bool zero = token == 0xFFFFFFFFu || token >= p.vocab_full;
          in.mode = kEmbedNormIn;
          in.embed = zero ? nullptr : p.embedding + (size_t)token * p.hidden;
          in.wb = p.t_hidden;
          in.wbtag = tagv(e, 0);
        } else if (p.tp > 1) {
          // hidden = residual + half(sum of the ranks' down partials)
          in.mode = kAddThenNormIn;
          in.x = p.t_res;
          in.xtag = tagv(e - 1u, 0);
          in.x2_part = (long long)mailbox_layout(p.tp, p.hidden, grid).d;
          in.x2tag = tagv(e - 1u, 1);  // as the DOWN stage tagged its partials
          in.exchange = 1;
          in.wb = p.t_hidden;
          in.wbtag = tagv(e, 0);
        } else {
          in.mode = kNormIn;
          in.x = p.t_hidden;
          in.xtag = hidden_in;
        }
        if (!build_input<TP>(p, in, layer == 0 ? -1 : kDown, xs, xs2, xn, sh)) return;
#ifdef MI_TRACE_TWICE
        if (tid == 0) g_trace_alt = 1;
        if (!build_input<TP>(p, in, layer == 0 ? -1 : kDown, xs, xs2, xn, sh)) return;
        if (tid == 0) g_trace_alt = 0;
#endif
        if (tid == 0) MI_TRACE(step, layer * 5 + 0, 1);
        kv_issued = attention_prefetch<G>(p, layer, L, pos, asm_, sh);
        reduce_rows<kQKV>(p, s, xn, ring, sh, g, tagv(e, 0), bk, bi);
        stage_done(p, kQKV);
        if (tid == 0) MI_TRACE(step, layer * 5 + 0, 2);
      }
      // ATTN (units read their head's tagged Q/K/V rows)
      {
        if (tid == 0) { MI_TRACE(step, layer * 5 + 1, 0); MI_TRACE_SET(step, layer * 5 + 1); }
        const int units = p.kvh * nb;
        if (tid >= kAttnBase && tid < kAttnBase + kAttnThreads)
          for (int u = blockIdx.x; u < units; u += gridDim.x)
            attention_unit<G>(p, layer, L, u / nb, u % nb, nb, pos, u == (int)blockIdx.x,
                              kv_uses & 1u, tile_uses, tagv(e, 0), asm_, sh);
        kv_uses += kv_issued ? 1u : 0u;
        if (tid == 0) MI_TRACE(step, layer * 5 + 1, 2);
      }
      // O (waits for every attention unit's partial, merges them as its input)
      {
        units_total += (uint32_t)(p.kvh * nb);
        if (!wait_units(p, units_total, (int)blockIdx.x < p.kvh * nb, sh)) return;
        if (tid == 0) { MI_TRACE(step, layer * 5 + 2, 0); MI_TRACE_SET(step, layer * 5 + 2); }
        if (tid == 0) MI_TRACE_ARRIVE(1);
        const StageW s = stage_weights(p, lay, layer, kO);
        build_attn_input(p, nb, xs);
        if (tid == 0) MI_TRACE(step, layer * 5 + 2, 1);
        reduce_rows<kO>(p, s, xs, ring, sh, g, tagv(e, 0), bk, bi);
        stage_done(p, kO);
        if (tid == 0) MI_TRACE(step, layer * 5 + 2, 2);
      }
      // GU
      {
        if (tid == 0) { MI_TRACE(step, layer * 5 + 3, 0); MI_TRACE_SET(step, layer * 5 + 3); }
        const StageW s = stage_weights(p, lay, layer, kGU);
        StageIn in = {};
        in.x2_part = -1;
        in.mode = p.add_norm ? kAddNormIn : kAddThenNormIn;
        in.k = p.hidden;
        in.x = p.t_hidden;
        in.xtag = hidden_in;
        in.x2 = p.t_attn_o;
        in.x2tag = tagv(e, 0);
        if (p.tp > 1) {
          // attention output = half(sum of the ranks' O partials)
          in.x2_part = (long long)mailbox_layout(p.tp, p.hidden, grid).o;
          in.x2tag = tagv(e, 0);  // as the O stage tagged its partials
          in.exchange = 1;
        }
        in.norm_w = L.post_norm;
        in.wb = p.t_res;
        in.wbtag = tagv(e, 0);
        if (!build_input<TP>(p, in, kO, xs, xs2, xn, sh)) return;
#ifdef MI_TRACE_TWICE
        if (tid == 0) g_trace_alt = 1;
        if (!build_input<TP>(p, in, kO, xs, xs2, xn, sh)) return;
        if (tid == 0) g_trace_alt = 0;
#endif
        if (tid == 0) MI_TRACE(step, layer * 5 + 3, 1);
        reduce_rows<kGU>(p, s, xn, ring, sh, g, tagv(e, 0), bk, bi);
        stage_done(p, kGU);
        if (tid == 0) MI_TRACE(step, layer * 5 + 3, 2);
      }
      // DOWN
      {
        if (tid == 0) { MI_TRACE(step, layer * 5 + 4, 0); MI_TRACE_SET(step, layer * 5 + 4); }
        const StageW s = stage_weights(p, lay, layer, kDown);
        StageIn in = {};
        in.x2_part = -1;
        in.mode = kPlainIn;
        in.k = p.inter;
        in.x = p.t_act;
        in.xtag = tagv(e, 0);
        if (p.tp == 1) {
          // residuals of this CTA's rows (written back by CTA 0 in GU); under
          // tensor parallelism the next QKV stage adds them
          const Tiles& td = sh.tiles[kDown];
          in.res = p.t_res;
          in.res_first = td.first;
          in.res_n = td.last - td.first;
          in.res_tag = tagv(e, 0);
        }
        if (!build_input<TP>(p, in, kGU, xs, xs2, xn, sh)) return;
        if (tid == 0) MI_TRACE(step, layer * 5 + 4, 1);
        reduce_rows<kDown>(p, s, xs, ring, sh, g, tagv(e, 1), bk, bi);
        stage_done(p, kDown);
        if (tid == 0) MI_TRACE(step, layer * 5 + 4, 2);
      }
    }
    // final norm + LM head + argmax
    {
      if (tid == 0) { MI_TRACE(step, p.layers * 5, 0); MI_TRACE_SET(step, p.layers * 5); }
      const uint32_t e = p.epoch0 + (uint32_t)(step * p.layers + p.layers - 1);
      uint32_t bk = 0, bi = 0xFFFFFFFFu;
      const StageW s = stage_weights(p, lay, p.layers, kLM);
      StageIn in = {};
      in.x2_part = -1;
      in.mode = kNormIn;
      in.k = p.hidden;
      in.x = p.t_hidden;
      in.xtag = tagv(e, 1);
      in.norm_w = p.final_norm;
      if (p.tp > 1) {
        in.mode = kAddThenNormIn;
        in.x = p.t_res;
        in.xtag = tagv(e, 0);
        in.x2_part = (long long)mailbox_layout(p.tp, p.hidden, grid).d;
        in.x2tag = tagv(e, 1);
        in.exchange = 1;
      }
      if (!build_input<TP>(p, in, kDown, xs, xs2, xn, sh)) return;
      if (tid == 0) MI_TRACE(step, p.layers * 5, 1);
      reduce_rows<kLM>(p, s, xn, ring, sh, g, 0u, bk, bi);
      if (tid == 0) MI_TRACE(step, p.layers * 5, 2);
      // per-lane bests -> warp best -> CTA best -> tagged record per CTA
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) {
        const uint32_t ok = __shfl_xor_sync(0xffffffffu, bk, o);
        const uint32_t oi = __shfl_xor_sync(0xffffffffu, bi, o);
        if (argmax_better(ok, oi, bk, bi)) {
          bk = ok;
          bi = oi;
        }
      }
      if (lane == 0) {
        sh.best_key[warp] = bk;
        sh.best_idx[warp] = bi;
      }
      consumers_sync();
      const unsigned long long rtag = e & 0x3FFFu;
      if (tid == 0) {
        uint32_t ck = 0, ci = 0xFFFFFFFFu;
        for (int w = 0; w < kConsumerWarps; ++w)
          if (argmax_better(sh.best_key[w], sh.best_idx[w], ck, ci)) {
            ck = sh.best_key[w];
            ci = sh.best_idx[w];
          }
        const unsigned long long idx =
            ci == 0xFFFFFFFFu ? 0x3FFFFull : (unsigned long long)(ci + p.vocab0);
        const unsigned long long rec = ((unsigned long long)ck << 32) | (idx << 14) | rtag;
        if (p.tp > 1) {
          // vocab-parallel: the record goes to every rank's mailbox
          const MailboxLayout mb = mailbox_layout(p.tp, p.hidden, grid);
          for (int r = 0; r < p.tp; ++r)
            st_sys_u64(p.peers[r] + mb.rec + (size_t)p.rank * grid + blockIdx.x, rec);
        } else {
          st_relaxed_u64(p.t_argmax + blockIdx.x, rec);
        }
        stage_ready(p, kLM, sh);  // one L2 round trip of delay before the polls
      }
      consumers_sync();
      // Every CTA reduces all records (argmax order is total: any order).
      // Each consumer thread loads its records together (one poll round
      // trip when they are there), the CTA then reduces in shared memory.
      {
        const uint64_t t_rec = (p.tp > 1 && tid == 0) ? pipe::global_ns() : 0;
        const unsigned long long* recs =
            p.tp > 1 ? p.mbox + mailbox_layout(p.tp, p.hidden, grid).rec : p.t_argmax;
        const int nrec = p.tp * (int)gridDim.x;
        uint32_t ck = 0, ci = 0xFFFFFFFFu;
        constexpr int kRecBatch = 4;
        for (int b0 = tid; b0 < nrec; b0 += kRecBatch * kConsumers) {
          unsigned long long r[kRecBatch];
#pragma unroll
          for (int i = 0; i < kRecBatch; ++i)
            if (b0 + i * kConsumers < nrec) r[i] = ld_sys_u64(recs + b0 + i * kConsumers);
#pragma unroll
          for (int i = 0; i < kRecBatch; ++i) {
            const int b = b0 + i * kConsumers;
            if (b >= nrec) break;
            PollClock clock;
            while ((r[i] & 0x3FFFull) != rtag && clock.keep_going(p, sh)) r[i] = ld_sys_u64(recs + b);
            const uint32_t k2 = (uint32_t)(r[i] >> 32);
            uint32_t i2 = (uint32_t)((r[i] >> 14) & 0x3FFFFull);
            if (i2 == 0x3FFFFu) i2 = 0xFFFFFFFFu;
            if (argmax_better(k2, i2, ck, ci)) {
              ck = k2;
              ci = i2;
            }
          }
        }
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) {
          const uint32_t ok = __shfl_xor_sync(0xffffffffu, ck, o);
          const uint32_t oi = __shfl_xor_sync(0xffffffffu, ci, o);
          if (argmax_better(ok, oi, ck, ci)) {
            ck = ok;
            ci = oi;
          }
        }
        consumers_sync();  // the CTA-best slots are free again
        if (lane == 0) {
          sh.best_key[warp] = ck;
          sh.best_idx[warp] = ci;
        }
        consumers_sync();
        if (tid == 0) {
          uint32_t gk = 0, gi = 0xFFFFFFFFu;
          for (int w = 0; w < kConsumerWarps; ++w)
            if (argmax_better(sh.best_key[w], sh.best_idx[w], gk, gi)) {
              gk = sh.best_key[w];
              gi = sh.best_idx[w];
            }
          sh.token = gi;
          if (blockIdx.x == 0) p.toks[pos + 1] = gi;
          sh.stop = sh.abort ? 1 : 0;
          if (p.tp > 1) sh.mbox_ns += pipe::global_ns() - t_rec;
        }
      }
      consumers_sync();
      if (sh.stop) return;
      token = sh.token;
    }
  }
  if (blockIdx.x == 0 && tid == 0) *p.dev_len = len0 + (uint32_t)p.steps;
  if (tid == 0 && p.tp > 1)
    p.sync[kWaitWord0 + blockIdx.x] = (uint32_t)min(sh.mbox_ns >> 6, 0xFFFFFFFFull);
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
  auto kernel = p.tp > 1 ? decode_loop_kernel<G, true> : decode_loop_kernel<G, false>;
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
  if (p.kvh > kMaxKvHeads) return false;
  if (p.vocab_full >= 0x3FFFF) return false;  // argmax records carry an 18-bit index
  const int max_k = std::max(std::max(p.hidden, p.inter), p.qh * HD);
  int max_item = std::max(std::max(p.hidden * 4, p.inter * 2), p.qh * HD * 2);
  p.slot_bytes = std::max(kMinSlotBytes, (max_item + 127) / 128 * 128);
  p.x_bytes = (max_k * 2 + 1023) / 1024 * 1024;  // keeps the attention tiles 1024-aligned
  int optin = 0;
  if (cudaDeviceGetAttribute(&optin, cudaDevAttrMaxSharedMemoryPerBlockOptin, device) !=
      cudaSuccess)
    return false;
  const size_t fixed = (size_t)p.x_bytes + attn_smem_for(group) + layer_table_bytes(p.layers) +
                       2 * x2_bytes(p.hidden) + sizeof(Shared) + 2048;
  if (fixed >= (size_t)optin) return false;
  p.slots = (int)std::min<size_t>(kMaxSlots, ((size_t)optin - fixed) / p.slot_bytes);
  if (p.slots < 2) return false;
  int sms = 0;
  if (cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, device) != cudaSuccess)
    return false;
  p.grid = std::min(sms, kMaxGrid);
  if ((p.hidden + p.grid - 1) / p.grid > kMaxDownRows) return false;  // DOWN residual cache
  return true;
}

size_t decode_loop_smem(const DecodeLoop& p) {
  return (size_t)p.slots * p.slot_bytes + p.x_bytes + attn_smem_for(p.qh / p.kvh) +
         layer_table_bytes(p.layers) + 2 * x2_bytes(p.hidden) + 1024;  // + alignment slack
}

void decode_loop(cudaStream_t stream, const DecodeLoop& p) {
  MI_REQUIRE(p.steps > 0 && p.grid > 0 && p.slots >= 2, MI_ERR_INVALID_ARGUMENT,
             "decode loop plan missing");
  MI_CUDA(cudaMemsetAsync(p.sync, 0, kSyncWords * sizeof(uint32_t), stream));
  static_assert(kSyncWords == decode_loop_sync_words(), "sync buffer size");
  static_assert(kWaitWord0 == decode_loop_wait_word0() && kWaitWord0 + kMaxGrid <= kSyncWords,
                "sync buffer layout");
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
  if (n < (sizeof(g_trace) + sizeof(g_arrive)) / 8) return -1;  // [2][2][321][16] + [256][5][2]
  if (cudaMemcpyFromSymbol(out, g_trace, sizeof(g_trace)) != cudaSuccess) return -2;
  return cudaMemcpyFromSymbol(out + sizeof(g_trace) / 8, g_arrive, sizeof(g_arrive)) == cudaSuccess
             ? 0 : -2;
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
