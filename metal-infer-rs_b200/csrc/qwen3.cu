// Qwen3 model: weights, KV cache and the forward plans
// (crates/metal-infer-models/src/qwen3.rs).
//
// Prefill (T > 1) follows forward_layer's unfused prefill path
// (qwen3.rs:647-796): rms_norm -> Q/K/V GEMMs -> qk_norm_rope_cache ->
// copy_into_cache -> attention -> O GEMM -> add_rms_norm -> gate/up GEMMs ->
// swiglu -> down GEMM -> add.
//
// Decode (T = 1) runs five fused kernels per layer:
//   1. RMSNorm + Q/K/V GEMV            (layer 0 also gathers the embedding)
//   2. QK-norm + RoPE + K/V append + split-K attention + merge
//   3. O GEMV
//   4. residual add + RMSNorm + gate/up GEMV + SwiGLU
//   5. down GEMV + residual add
// and one final RMSNorm + LM-head GEMV + greedy argmax. The cache keeps its
// length and a token ring on the device (toks[pos] is the token at cache
// position pos), so one captured CUDA graph serves every decode step: the
// step reads toks[len], writes its argmax to toks[len + 1] and increments
// len. Kernels after the first are launched with programmatic dependent
// launch so each one streams its weights while its predecessor finishes.
//
// By default the decode steps of a call run instead in one persistent
// cooperative kernel (decode_loop.cu) with the same stages and arithmetic.

#include <cstring>
#include <functional>
#include <map>
#include <memory>

#ifdef MI_HAVE_NCCL
#include <nccl.h>
#endif

#include "kernels.h"
#include "loader.h"
#include "mi_internal.h"

using namespace mi;

namespace {

enum Role {
  kEmbedding = 0,
  kQ = 1,
  kK = 2,
  kV = 3,
  kO = 4,
  kQNorm = 5,
  kKNorm = 6,
  kGate = 7,
  kUp = 8,
  kDown = 9,
  kInputNorm = 10,
  kPostNorm = 11,
  kFinalNorm = 12,
  kLmHead = 13,
};

struct TensorRef {
  mi_tensor* t = nullptr;
  TensorRef() = default;
  explicit TensorRef(mi_tensor* x) : t(x) {}
  TensorRef(const TensorRef&) = delete;
  TensorRef& operator=(const TensorRef&) = delete;
  TensorRef(TensorRef&& o) noexcept : t(o.t) { o.t = nullptr; }
  TensorRef& operator=(TensorRef&& o) noexcept {
    if (this != &o) {
      reset();
      t = o.t;
      o.t = nullptr;
    }
    return *this;
  }
  ~TensorRef() { reset(); }
  void reset() {
    if (t) mi_tensor_release(t);
    t = nullptr;
  }
  __half* h() const { return t->f16(); }
};

struct Layer {
  TensorRef w[16];
};

// Decode workspace, sized once per model.
struct Workspace {
  TensorRef q_raw, k_raw, v_raw, attn, attn_o, residual, hidden, act, logits;
  TensorRef argmax_pv, argmax_pi, counters, attn_scratch;
  // tensor parallelism: FP32 partials of this rank, all ranks' partials,
  // the rounded sum, this rank's greedy candidate and all ranks' candidates
  TensorRef tp_part, tp_gather, tp_sum, tp_best, tp_best_all, tp_logits;
  TensorRef loop_sync;  // persistent decode: abort flag + attention-unit counter
  TensorRef loop_part;  // persistent decode: attention block partials
  // persistent decode: epoch-tagged activations and per-CTA argmax records
  TensorRef t_hidden, t_res, t_qkv, t_attn_o, t_act, t_argmax;
  // sampling: key histogram, group scratch, options, XorShift64 state and
  // (tensor parallelism) the gathered full-vocabulary logits
  TensorRef smp_hist, smp_groups, smp_opts, smp_state, smp_logits;
  uint64_t loop_epoch = 1;  // layer-steps run through the tagged buffers + 1
  int attn_splits = 0;  // flash-decode blocks for the largest cache seen
  int attn_block = 64;  // keys per flash-decode block
  size_t attn_cap = 0;
};

}  // namespace

struct mi_kv_cache;

struct mi_qwen3 {
  // Released by mi_qwen3_destroy and by each KV cache of the model.
  std::atomic<int> refs{1};
  mi_context* ctx = nullptr;
  mi_qwen3_config cfg{};
  TensorRef embedding, final_norm, lm_head_own;
  const mi_tensor* lm_head = nullptr;
  std::vector<Layer> layers;
  mi_attention_kind attention_kind = MI_ATTENTION_TILED;
  mi_fusion_options fusion{1, 1, 1, 1};
  bool graphs = true;
  // Tensor parallelism: cfg holds this rank's shard (heads, intermediate,
  // vocabulary divided by tp); full_cfg the model's configuration.
  int tp = 1, rank = 0;
  mi_qwen3_config full_cfg{};
#ifdef MI_HAVE_NCCL
  ncclComm_t comm = nullptr;
#endif
  // Tensor-parallel persistent decode: this rank's mailbox (cudaMalloc, IPC
  // exported) and every rank's mailbox mapped here (peer[rank] = local).
  struct Mailbox {
    void* local = nullptr;
    std::vector<void*> peer;
    TensorRef table;  // device array of the tp mailbox pointers
    int grid = 0;
  } mbox;
  bool persistent = true;  // decode through the persistent kernel when it fits
  bool sampling = false;   // LM heads draw tokens (generate_with, temperature > 0)
  int loop_state = 0;      // 0 unplanned, 1 planned, -1 not admitted
  int last_loop_steps = 0; // decode steps of the most recent persistent launch
  k::DecodeLoop loop;
  Workspace ws;
  uint64_t plan_version = 1;  // bumps invalidate captured graphs
};

struct mi_kv_cache {
  mi_qwen3* model = nullptr;
  size_t capacity = 0;
  size_t filled = 0;
  std::vector<TensorRef> key, value;
  TensorRef toks;     // u32 [capacity + 1]
  TensorRef dev_len;  // u32 [1]
  TensorRef rope;     // f32 [capacity, head_dim / 2, 2]: (cos, sin) per position and pair
  const float2* rope_table() const { return reinterpret_cast<const float2*>(rope.t->f32()); }
  cudaGraphExec_t graph = nullptr;  // decode step: [0] greedy, [1] sampled
  uint64_t graph_version = 0;
  cudaGraphExec_t graph_sampled = nullptr;
  uint64_t graph_sampled_version = 0;
  std::vector<k::LoopLayer> loop_host;  // layer table of the persistent decode
  TensorRef loop_layers;                // its device copy
  std::vector<uint8_t> kv_maps_host;    // [layers][K, V] CUtensorMap bytes
  TensorRef kv_maps;                    // their device copy (256-byte aligned)
  ~mi_kv_cache() {
    if (graph) cudaGraphExecDestroy(graph);
    if (graph_sampled) cudaGraphExecDestroy(graph_sampled);
  }
};

namespace {

void require(const void* p, const char* what) {
  MI_REQUIRE(p != nullptr, MI_ERR_INVALID_ARGUMENT, "%s is NULL", what);
}

void model_release(mi_qwen3* m) {
  if (!m || m->refs.fetch_sub(1) != 1) return;
  mi_context* ctx = m->ctx;
  cudaSetDevice(ctx->device);
  cudaStreamSynchronize(ctx->stream);
  for (size_t r = 0; r < m->mbox.peer.size(); ++r)
    if ((int)r != m->rank && m->mbox.peer[r]) cudaIpcCloseMemHandle(m->mbox.peer[r]);
  m->mbox.table = TensorRef();
  if (m->mbox.local) cudaFree(m->mbox.local);
#ifdef MI_HAVE_NCCL
  if (m->comm) ncclCommDestroy(m->comm);
#endif
  delete m;
  context_release(ctx);
}

// Qwen3Config::validate (config.rs:23-57)
void validate_config(const mi_qwen3_config& c) {
  if (!c.hidden_size || !c.intermediate_size || !c.num_hidden_layers || !c.num_attention_heads ||
      !c.num_key_value_heads || !c.head_dim || !c.vocab_size || c.head_dim % 2)
    fail(MI_ERR_CONFIG,
         "invalid model configuration: model dimensions must be non-zero and head_dim even");
  if (c.num_attention_heads % c.num_key_value_heads)
    fail(MI_ERR_CONFIG,
         "invalid model configuration: num_attention_heads must be divisible by "
         "num_key_value_heads");
}

k::Launch launch(mi_qwen3* m, bool pdl) {
  k::Launch l;
  l.stream = m->ctx->stream;
  l.pdl = pdl;
  l.sm_count = m->ctx->sm_count;
  return l;
}

// Decode launches: PDL unless per-kernel profiling is on (events between
// launches would serialise them anyway) or MI_DECODE_PDL=0.
bool pdl_enabled() {
  static int on = -1;
  if (on < 0) {
    const char* e = getenv("MI_DECODE_PDL");
    on = (e && *e == '0') ? 0 : 1;
  }
  return on == 1;
}

// Weight tiles (32 KB each per SM) the persistent decode kernel's producer
// prefetches into L2 beyond its shared-memory copies (same-box A/B,
// Qwen3-0.6B / 8B tokens/s: 0 → 1,467 / 208.0, 4 → 1,512 / 213.9, 6 → 1,500 /
// 211.9, 16 → 1,347 / 166.1). MI_L2_AHEAD=n overrides (0..64).
constexpr int kL2AheadTiles = 4;
int l2_ahead_tiles() {
  static int n = -1;
  if (n < 0) {
    const char* e = getenv("MI_L2_AHEAD");
    n = e ? std::min(std::max(atoi(e), 0), 64) : kL2AheadTiles;
  }
  return n;
}

// Tensor parallelism: each CTA sums its slice of the ranks' partials;
// MI_TP_SLICE=0 has every CTA sum all of them itself.
bool tp_slice_enabled() {
  static int on = -1;
  if (on < 0) {
    const char* e = getenv("MI_TP_SLICE");
    on = (e && *e == '0') ? 0 : 1;
  }
  return on == 1;
}

k::Launch dlaunch(mi_qwen3* m, bool pdl) {
  return launch(m, pdl && !m->ctx->profiling && pdl_enabled() && m->tp == 1);
}

// Prefill launches: PDL on one GPU unless profiling (every kernel waits for
// its predecessor before it reads an operand; nothing is read early, as the
// prefill's decode-attention path reads K / V rows its predecessor appends).
k::Launch plaunch(mi_qwen3* m) {
  k::Launch l = launch(m, !m->ctx->profiling && pdl_enabled() && m->tp == 1);
  l.early = false;
  return l;
}

size_t qwidth(const mi_qwen3_config& c) { return c.num_attention_heads * c.head_dim; }
size_t kvwidth(const mi_qwen3_config& c) { return c.num_key_value_heads * c.head_dim; }

// Tokens index the full vocabulary (the embedding is replicated).
uint32_t vocab_full(const mi_qwen3* m) { return (uint32_t)m->full_cfg.vocab_size; }

// All-gather of `count` elements per rank on the engine stream.
void tp_allgather(mi_qwen3* m, const void* send, void* recv, size_t count, int dtype_bytes) {
#ifdef MI_HAVE_NCCL
  ncclDataType_t t = dtype_bytes == 4 ? ncclFloat32 : ncclFloat16;
  ncclResult_t r = ncclAllGather(send, recv, count, t, m->comm, m->ctx->stream);
  if (r != ncclSuccess)
    fail(MI_ERR_COLLECTIVE, "NCCL all-gather failed: %s", ncclGetErrorString(r));
#else
  (void)m, (void)send, (void)recv, (void)count, (void)dtype_bytes;
  fail(MI_ERR_UNSUPPORTED, "built without NCCL: tensor parallelism is unavailable");
#endif
}

// Row-parallel projection result: the sum of the ranks' FP32 partials
// `part` ([n] each) in rank order, rounded once to FP16 into `out` ([n]).
// Large results (prefill) are reduced slice by slice: rank r receives only
// slice r (n / tp elements) of every other rank's partials (grouped NCCL
// send / receive into `gather`, [tp, n / tp]), sums its slice in rank order
// and the FP16 slices are all-gathered in place, so a rank receives
// (tp - 1) * n / tp * 6 bytes instead of (tp - 1) * n * 4. Small results
// (the per-kernel decode chain) gather the full partials ([tp, n]) and sum
// them; both give the same bits.
constexpr size_t kSliceReduceMin = 1 << 16;

void tp_reduce(mi_qwen3* m, const float* part, size_t n, float* gather, __half* out) {
  const int tp = m->tp, rank = m->rank;
  if (n < kSliceReduceMin || n % (size_t)tp != 0) {
    tp_allgather(m, part, gather, n, 4);
    k::rank_sum_round(m->ctx->stream, gather, tp, n, out);
    return;
  }
#ifdef MI_HAVE_NCCL
  const size_t chunk = n / (size_t)tp;
  cudaStream_t s = m->ctx->stream;
  ncclResult_t r = ncclGroupStart();
  for (int q = 0; q < tp && r == ncclSuccess; ++q) {
    if (q == rank) continue;
    r = ncclSend(part + (size_t)q * chunk, chunk, ncclFloat32, q, m->comm, s);
    if (r == ncclSuccess)
      r = ncclRecv(gather + (size_t)q * chunk, chunk, ncclFloat32, q, m->comm, s);
  }
  const ncclResult_t e = ncclGroupEnd();
  if (r == ncclSuccess) r = e;
  if (r != ncclSuccess)
    fail(MI_ERR_COLLECTIVE, "NCCL partial-slice exchange failed: %s", ncclGetErrorString(r));
  k::rank_sum_round_slice(s, gather, part + (size_t)rank * chunk, rank, tp, chunk,
                          out + (size_t)rank * chunk);
  r = ncclAllGather(out + (size_t)rank * chunk, out, chunk, ncclFloat16, m->comm, s);
  if (r != ncclSuccess)
    fail(MI_ERR_COLLECTIVE, "NCCL all-gather of the reduced slices failed: %s",
         ncclGetErrorString(r));
#else
  (void)rank, (void)gather, (void)out, (void)part;
  fail(MI_ERR_UNSUPPORTED, "built without NCCL: tensor parallelism is unavailable");
#endif
}

// Vocab-parallel greedy id: the ranks' {key, index} candidates in
// w.tp_best are gathered and the best goes to tokens[*pos + 1] (or
// tokens[0] without pos); *step_counter advances when given.
void tp_argmax(mi_qwen3* m, uint32_t* tokens, const uint32_t* pos, uint32_t* step_counter) {
  auto& w = m->ws;
  tp_allgather(m, w.tp_best.t->u32(), w.tp_best_all.t->u32(), 2, 4);
  k::argmax_combine(m->ctx->stream, w.tp_best_all.t->u32(), m->tp, tokens, pos, step_counter);
}

// Sampling buffers (the histogram starts zeroed; the sampler clears it).
void ensure_sampling(mi_qwen3* m) {
  auto& w = m->ws;
  if (w.smp_hist.t) return;
  mi_context* ctx = m->ctx;
  w.smp_hist = TensorRef(new_tensor(ctx, {(size_t)k::kSampleHistWords}, MI_U32, true));
  w.smp_groups = TensorRef(new_tensor(ctx, {2 * (size_t)k::kSampleBins}, MI_U32, true));
  w.smp_opts = TensorRef(new_tensor(ctx, {4}, MI_U32, true));
  w.smp_state = TensorRef(new_tensor(ctx, {2}, MI_U32, true));
  if (m->tp > 1)
    w.smp_logits = TensorRef(new_tensor(ctx, {m->full_cfg.vocab_size}, MI_F16, true));
  MI_CUDA(cudaMemsetAsync(w.smp_hist.t->base(), 0, w.smp_hist.t->bytes(), ctx->stream));
}

// The lm_head's logits -> tokens[*pos] (tokens[0] without pos), drawn by the
// sampler. One GPU: the lm_head GEMV filled the key histogram (hist_built),
// else the histogram kernel builds it. Tensor parallelism: every rank gathers
// the full logits and draws the same token.
void encode_sample(mi_qwen3* m, uint32_t* tokens, const uint32_t* pos, bool hist_built) {
  auto& w = m->ws;
  k::SampleProblem sp;
  sp.logits = w.logits.h();
  sp.n = (uint32_t)m->cfg.vocab_size;
  sp.hist = w.smp_hist.t->u32();
  if (m->tp > 1) {
    tp_allgather(m, w.logits.t->base(), w.smp_logits.t->base(), m->cfg.vocab_size, 2);
    sp.logits = w.smp_logits.h();
    sp.n = (uint32_t)m->full_cfg.vocab_size;
    ProfileScope ph(m->ctx, "sample_histogram");
    k::logit_histogram(launch(m, false), sp.logits, sp.n, sp.hist);
  } else if (!hist_built) {
    ProfileScope ph(m->ctx, "sample_histogram");
    k::logit_histogram(launch(m, false), sp.logits, sp.n, sp.hist);
  }
  sp.groups = w.smp_groups.t->u32();
  sp.opts = w.smp_opts.t->u32();
  sp.state = reinterpret_cast<uint64_t*>(w.smp_state.t->u32());
  sp.token_out = tokens;
  sp.token_pos = pos;
  ProfileScope ps(m->ctx, "sample");
  k::sample(launch(m, false), sp);
}

bool fused_decode_supported(const mi_qwen3* m) {
  const auto& c = m->cfg;
  size_t g = c.num_attention_heads / c.num_key_value_heads;
  return c.head_dim == 128 && (g == 1 || g == 2 || g == 4 || g == 8) &&
         m->attention_kind != MI_ATTENTION_REFERENCE && c.hidden_size % 8 == 0 &&
         c.intermediate_size % 8 == 0 && c.hidden_size <= 16384 && c.intermediate_size <= 16384;
}

void ensure_workspace(mi_qwen3* m, size_t capacity) {
  auto& w = m->ws;
  const auto& c = m->cfg;
  mi_context* ctx = m->ctx;
  if (!w.q_raw.t) {
    w.q_raw = TensorRef(new_tensor(ctx, {qwidth(c)}, MI_F16, true));
    w.k_raw = TensorRef(new_tensor(ctx, {kvwidth(c)}, MI_F16, true));
    w.v_raw = TensorRef(new_tensor(ctx, {kvwidth(c)}, MI_F16, true));
    w.attn = TensorRef(new_tensor(ctx, {qwidth(c)}, MI_F16, true));
    w.attn_o = TensorRef(new_tensor(ctx, {c.hidden_size}, MI_F16, true));
    w.residual = TensorRef(new_tensor(ctx, {c.hidden_size}, MI_F16, true));
    w.hidden = TensorRef(new_tensor(ctx, {c.hidden_size}, MI_F16, true));
    w.act = TensorRef(new_tensor(ctx, {c.intermediate_size}, MI_F16, true));
    w.logits = TensorRef(new_tensor(ctx, {1, c.vocab_size}, MI_F16, true));
    size_t parts = (size_t)ctx->sm_count * 4;
    w.argmax_pv = TensorRef(new_tensor(ctx, {parts}, MI_F32, true));
    w.argmax_pi = TensorRef(new_tensor(ctx, {parts}, MI_U32, true));
    w.counters = TensorRef(new_tensor(ctx, {1 + c.num_key_value_heads}, MI_U32, true));
    if (m->tp > 1) {
      w.tp_part = TensorRef(new_tensor(ctx, {c.hidden_size}, MI_F32, true));
      w.tp_sum = TensorRef(new_tensor(ctx, {c.hidden_size}, MI_F16, true));
      w.tp_best = TensorRef(new_tensor(ctx, {2}, MI_U32, true));
      w.tp_best_all = TensorRef(new_tensor(ctx, {2 * (size_t)m->tp}, MI_U32, true));
      // fixed for the captured decode graph (prefill gathers into its own)
      w.tp_gather = TensorRef(new_tensor(ctx, {(size_t)m->tp * c.hidden_size}, MI_F32, true));
    }
  }
  const int cap_block = k::decode_block_for((int)capacity);
  const int cap_splits = ((int)capacity + cap_block - 1) / cap_block;
  if (capacity > w.attn_cap || cap_splits > w.attn_splits) {
    int kvh = (int)c.num_key_value_heads;
    int block = cap_block;
    int splits = std::max(cap_splits, w.attn_splits);
    int group = (int)(c.num_attention_heads / c.num_key_value_heads);
    size_t bytes = k::attention_decode_scratch(kvh, splits, group, (int)c.head_dim);
    w.attn_scratch = TensorRef(new_tensor(ctx, {bytes / 4}, MI_F32, true));
    w.attn_splits = splits;
    w.attn_block = block;
    w.attn_cap = std::max(capacity, w.attn_cap);
    m->plan_version++;
  }
}

// Sets the device-side cache length (stream-ordered).
__global__ void set_u32_kernel(uint32_t* p, uint32_t v) { *p = v; }

void set_dev_len(mi_kv_cache* c, size_t v) {
  set_u32_kernel<<<1, 1, 0, c->model->ctx->stream>>>(c->dev_len.t->u32(), (uint32_t)v);
  MI_CUDA(cudaGetLastError());
}

// ---- decode step ------------------------------------------------------------
void encode_decode_step(mi_qwen3* m, mi_kv_cache* c) {
  const auto& cfg = m->cfg;
  auto& w = m->ws;
  const int h = (int)cfg.hidden_size, I = (int)cfg.intermediate_size;
  const int qw = (int)qwidth(cfg), kw = (int)kvwidth(cfg);
  uint32_t* len = c->dev_len.t->u32();
  for (size_t li = 0; li < m->layers.size(); ++li) {
    const Layer& L = m->layers[li];
    // 1. (embedding +) RMSNorm + QKV
    {
      k::GemvProblem p;
      p.k = h;
      p.segments = 3;
      p.w[0] = L.w[kQ].h();
      p.w[1] = L.w[kK].h();
      p.w[2] = L.w[kV].h();
      p.n[0] = qw;
      p.n[1] = kw;
      p.n[2] = kw;
      p.out[0] = w.q_raw.h();
      p.out[1] = w.k_raw.h();
      p.out[2] = w.v_raw.h();
      p.norm_w = L.w[kInputNorm].h();
      p.eps = cfg.rms_norm_eps;
      if (li == 0) {
        p.in_mode = k::kInEmbedNorm;
        p.token = c->toks.t->u32();
        p.token_pos = len;
        p.table = m->embedding.h();
        p.table_rows = vocab_full(m);
        p.embed_out = w.hidden.h();
      } else {
        p.in_mode = k::kInNorm;
        p.x = w.hidden.h();
      }
      ProfileScope ps(m->ctx, "qkv_gemv");
      k::gemv(dlaunch(m, li != 0), p);
    }
    // 2. QK-norm + RoPE + KV append + attention
    {
      k::DecodeFused d;
      d.q_raw = w.q_raw.h();
      d.k_raw = w.k_raw.h();
      d.v_raw = w.v_raw.h();
      d.q_norm = L.w[kQNorm].h();
      d.k_norm = L.w[kKNorm].h();
      d.theta = cfg.rope_theta;
      d.eps = cfg.rms_norm_eps;
      d.round_norm = !m->fusion.qk_rope_cache;
      d.key_cache = c->key[li].h();
      d.value_cache = c->value[li].h();
      d.out = w.attn.h();
      d.qh = (int)cfg.num_attention_heads;
      d.kvh = (int)cfg.num_key_value_heads;
      d.hd = (int)cfg.head_dim;
      d.pos.dev = len;
      d.rope = c->rope_table();
      ProfileScope ps(m->ctx, "attention_decode");
      k::attention_decode_fused(dlaunch(m, true), d, w.attn_splits, w.attn_scratch.t->f32(),
                                w.counters.t->u32() + 1, k::decode_block_for((int)c->capacity));
    }
    // 3. O projection (row-parallel under tensor parallelism)
    {
      k::GemvProblem p;
      p.k = qw;
      p.x = w.attn.h();
      p.w[0] = L.w[kO].h();
      p.n[0] = h;
      p.out[0] = w.attn_o.h();
      if (m->tp > 1) {
        p.out_mode = k::kOutF32;
        p.outf = w.tp_part.t->f32();
      }
      ProfileScope ps(m->ctx, "o_gemv");
      k::gemv(dlaunch(m, true), p);
      if (m->tp > 1) tp_reduce(m, w.tp_part.t->f32(), (size_t)h, w.tp_gather.t->f32(), w.attn_o.h());
    }
    // 4. residual + RMSNorm + gate/up + SwiGLU
    {
      k::GemvProblem p;
      p.k = h;
      p.segments = 2;
      p.in_mode = m->fusion.add_rms_norm ? k::kInAddNorm : k::kInAddThenNorm;
      p.x = w.hidden.h();
      p.x2 = w.attn_o.h();
      p.norm_w = L.w[kPostNorm].h();
      p.eps = cfg.rms_norm_eps;
      p.residual_out = w.residual.h();
      p.w[0] = L.w[kGate].h();
      p.w[1] = L.w[kUp].h();
      p.n[0] = I;
      p.n[1] = I;
      p.out_mode = k::kOutSwiglu;
      p.out[0] = w.act.h();
      ProfileScope ps(m->ctx, "gate_up_gemv");
      k::gemv(dlaunch(m, true), p);
    }
    // 5. down + residual (row-parallel under tensor parallelism)
    {
      k::GemvProblem p;
      p.k = I;
      p.x = w.act.h();
      p.w[0] = L.w[kDown].h();
      p.n[0] = h;
      p.out_mode = k::kOutResidual;
      p.res = w.residual.h();
      p.out[0] = w.hidden.h();
      if (m->tp > 1) {
        p.out_mode = k::kOutF32;
        p.outf = w.tp_part.t->f32();
      }
      ProfileScope ps(m->ctx, "down_gemv");
      k::gemv(dlaunch(m, true), p);
      if (m->tp > 1) {
        tp_reduce(m, w.tp_part.t->f32(), (size_t)h, w.tp_gather.t->f32(), w.tp_sum.h());
        k::add(launch(m, false), w.residual.h(), w.tp_sum.h(), w.hidden.h(), (size_t)h);
      }
    }
  }
  // final norm + LM head + argmax; advances the device length.
  {
    k::GemvProblem p;
    p.k = h;
    p.in_mode = k::kInNorm;
    p.x = w.hidden.h();
    p.norm_w = m->final_norm.h();
    p.eps = cfg.rms_norm_eps;
    p.w[0] = m->lm_head->f16();
    p.n[0] = (int)cfg.vocab_size;
    p.out_mode = k::kOutArgmax;
    p.out[0] = w.logits.h();
    p.token_out = c->toks.t->u32();
    p.token_pos = len;
    p.argmax_partial = w.argmax_pv.t->f32();
    p.argmax_index = w.argmax_pi.t->u32();
    p.counter = w.counters.t->u32();
    p.step_counter = len;
    if (m->tp > 1) {
      // vocab-parallel: this rank's candidate, then the combine over ranks
      p.best_out = w.tp_best.t->u32();
      p.index_base = (uint32_t)(m->rank * cfg.vocab_size);
      p.step_counter = nullptr;
    }
    if (m->sampling && m->tp == 1) p.hist = w.smp_hist.t->u32();
    {
      ProfileScope ps(m->ctx, "lm_head_argmax");
      k::gemv(dlaunch(m, true), p);
    }
    if (m->tp > 1) tp_argmax(m, c->toks.t->u32(), len, len);
    // the step counter has advanced: the token goes to toks[*len]
    if (m->sampling) encode_sample(m, c->toks.t->u32(), len, true);
  }
}

// Persistent decode (decode_loop.cu) unless disabled per model or by
// MI_DECODE_LOOP=0; the planner rejects shapes it cannot hold on chip.
bool persistent_env() {
  static int on = -1;
  if (on < 0) {
    const char* e = getenv("MI_DECODE_LOOP");
    on = (e && *e == '0') ? 0 : 1;
  }
  return on == 1;
}

bool decode_loop_ready(mi_qwen3* m) {
  if ((m->tp > 1 && !m->mbox.local) || !m->persistent || !persistent_env() ||
      !fused_decode_supported(m))
    return false;
  if (m->loop_state == 0) {
    const auto& c = m->cfg;
    k::DecodeLoop p;
    p.hidden = (int)c.hidden_size;
    p.inter = (int)c.intermediate_size;
    p.qh = (int)c.num_attention_heads;
    p.kvh = (int)c.num_key_value_heads;
    p.vocab = (int)c.vocab_size;
    p.layers = (int)c.num_hidden_layers;
    p.eps = c.rms_norm_eps;
    p.theta = c.rope_theta;
    p.vocab_full = (uint32_t)m->full_cfg.vocab_size;
    m->loop_state = k::decode_loop_plan(p, m->ctx->device) ? 1 : -1;
    if (m->tp > 1 && p.grid != m->mbox.grid) m->loop_state = -1;  // mailbox sized for another grid
    m->loop = p;
  }
  return m->loop_state == 1;
}

// `steps` decode steps from the cache's device position in persistent
// launches (at most 2048 steps each, which bounds the grid-barrier counter).
void run_decode_loop(mi_qwen3* m, mi_kv_cache* c, size_t steps) {
  mi_context* ctx = m->ctx;
  ensure_workspace(m, c->capacity);
  auto& w = m->ws;
  if (!w.loop_sync.t)
    w.loop_sync = TensorRef(new_tensor(ctx, {k::decode_loop_sync_words()}, MI_U32, true));
  if (!c->loop_layers.t) {
    c->loop_host.resize(m->layers.size());
    for (size_t li = 0; li < m->layers.size(); ++li) {
      const Layer& L = m->layers[li];
      k::LoopLayer& d = c->loop_host[li];
      d.wq = L.w[kQ].h();
      d.wk = L.w[kK].h();
      d.wv = L.w[kV].h();
      d.wo = L.w[kO].h();
      d.q_norm = L.w[kQNorm].h();
      d.k_norm = L.w[kKNorm].h();
      d.gate = L.w[kGate].h();
      d.up = L.w[kUp].h();
      d.down = L.w[kDown].h();
      d.in_norm = L.w[kInputNorm].h();
      d.post_norm = L.w[kPostNorm].h();
      d.k_cache = c->key[li].h();
      d.v_cache = c->value[li].h();
    }
    const size_t bytes = sizeof(k::LoopLayer) * c->loop_host.size();
    c->loop_layers = TensorRef(new_tensor(ctx, {(bytes + 3) / 4}, MI_U32, false));
    MI_CUDA(cudaMemcpyAsync(c->loop_layers.t->base(), c->loop_host.data(), bytes,
                            cudaMemcpyHostToDevice, ctx->stream));
    // K / V tile maps of every layer for the attention prefetch (TMA 2-D)
    const int kvh = (int)m->cfg.num_key_value_heads;
    c->kv_maps_host.assign(m->layers.size() * 2 * 128, 0);
    for (size_t li = 0; li < m->layers.size(); ++li)
      for (int v = 0; v < 2; ++v)
        if (!k::make_kv_tile_map(c->kv_maps_host.data() + (li * 2 + v) * 128,
                                 v ? c->value[li].h() : c->key[li].h(), (int)c->capacity, kvh,
                                 64))
          fail(MI_ERR_KERNEL, "cannot encode the KV cache tile map of layer %zu", li);
    c->kv_maps = TensorRef(new_tensor(ctx, {c->kv_maps_host.size() / 4}, MI_U32, false));
    MI_CUDA(cudaMemcpyAsync(c->kv_maps.t->base(), c->kv_maps_host.data(), c->kv_maps_host.size(),
                            cudaMemcpyHostToDevice, ctx->stream));
  }
  k::DecodeLoop p = m->loop;
  p.round_norm = m->fusion.qk_rope_cache ? 0 : 1;
  p.add_norm = m->fusion.add_rms_norm ? 1 : 0;
  p.block = k::decode_block_for((int)c->capacity);
  p.attn_blocks = w.attn_splits;
  p.layer = reinterpret_cast<const k::LoopLayer*>(c->loop_layers.t->base());
  p.kv_maps = c->kv_maps.t->base();
  p.embedding = m->embedding.h();
  p.final_norm = m->final_norm.h();
  p.lm_head = m->lm_head->f16();
  p.rope = c->rope_table();
  p.toks = c->toks.t->u32();
  p.dev_len = c->dev_len.t->u32();
  if (!w.t_hidden.t) {
    const auto& c = m->cfg;
    w.t_hidden = TensorRef(new_tensor(ctx, {c.hidden_size}, MI_U32, true));
    w.t_res = TensorRef(new_tensor(ctx, {c.hidden_size}, MI_U32, true));
    w.t_qkv = TensorRef(new_tensor(ctx, {qwidth(c) + 2 * kvwidth(c)}, MI_U32, true));
    w.t_attn_o = TensorRef(new_tensor(ctx, {c.hidden_size}, MI_U32, true));
    w.t_act = TensorRef(new_tensor(ctx, {c.intermediate_size}, MI_U32, true));
    w.t_argmax = TensorRef(new_tensor(ctx, {2 * (size_t)p.grid}, MI_U32, true));
  }
  p.t_hidden = w.t_hidden.t->u32();
  p.t_res = w.t_res.t->u32();
  p.t_qkv = w.t_qkv.t->u32();
  p.t_attn_o = w.t_attn_o.t->u32();
  p.t_act = w.t_act.t->u32();
  p.t_argmax = reinterpret_cast<unsigned long long*>(w.t_argmax.t->u32());
  p.logits = w.logits.h();
  const size_t part = k::decode_loop_part_floats(p.kvh, w.attn_splits, p.qh / p.kvh);
  if (!w.loop_part.t || w.loop_part.t->len() < part)
    // zeroed: block records are validated by their epoch tags, so the
    // buffer must not start with tags a previous user left there
    w.loop_part = TensorRef(new_tensor(ctx, {part}, MI_F32, true));
  p.attn_part = w.loop_part.t->f32();
  p.sync = w.loop_sync.t->u32();
  p.tp = m->tp;
  p.xslice = tp_slice_enabled() ? 1 : 0;
  p.l2_ahead = l2_ahead_tiles();
  p.rank = m->rank;
  p.vocab0 = (uint32_t)(m->rank * m->cfg.vocab_size);
  if (m->tp > 1) {
    p.peers = reinterpret_cast<unsigned long long* const*>(m->mbox.table.t->base());
    p.mbox = static_cast<unsigned long long*>(m->mbox.local);
  }
  for (size_t done = 0; done < steps;) {
    p.steps = (int)std::min<size_t>(steps - done, 2048);
    p.epoch0 = (uint32_t)w.loop_epoch;
    ProfileScope ps(ctx, "decode_loop");
    k::decode_loop(ctx->stream, p);
    m->last_loop_steps = p.steps;
    w.loop_epoch += (uint64_t)p.steps * (uint64_t)p.layers;
    done += (size_t)p.steps;
  }
}

// `n` steps through the persistent kernel: one launch when greedy; when
// sampling, one launch per step, each followed by the histogram and the
// sampler, which overwrite the greedy id at toks[*dev_len] before the next
// launch embeds it.
void run_persistent_steps(mi_qwen3* m, mi_kv_cache* c, size_t n) {
  if (!m->sampling) {
    run_decode_loop(m, c, n);
    c->filled += n;
    return;
  }
  for (size_t i = 0; i < n; ++i) {
    run_decode_loop(m, c, 1);
    encode_sample(m, c->toks.t->u32(), c->dev_len.t->u32(), false);
    c->filled += 1;
  }
}

// Runs (or replays) one decode step at the cache's device position.
void run_decode_step(mi_qwen3* m, mi_kv_cache* c) {
  mi_context* ctx = m->ctx;
  if (!m->graphs || ctx->profiling) {
    encode_decode_step(m, c);
    return;
  }
  cudaGraphExec_t& graph = m->sampling ? c->graph_sampled : c->graph;
  uint64_t& version = m->sampling ? c->graph_sampled_version : c->graph_version;
  if (!graph || version != m->plan_version) {
    if (graph) {
      cudaGraphExecDestroy(graph);
      graph = nullptr;
    }
    cudaGraph_t g = nullptr;
    MI_CUDA(cudaStreamBeginCapture(ctx->stream, cudaStreamCaptureModeThreadLocal));
    try {
      encode_decode_step(m, c);
    } catch (...) {
      cudaStreamEndCapture(ctx->stream, &g);
      if (g) cudaGraphDestroy(g);
      throw;
    }
    MI_CUDA(cudaStreamEndCapture(ctx->stream, &g));
    cudaError_t err = cudaGraphInstantiate(&graph, g, 0);
    cudaGraphDestroy(g);
    if (err != cudaSuccess) {
      graph = nullptr;
      fail(MI_ERR_COMMAND, "graph instantiation failed: %s", cudaGetErrorString(err));
    }
    version = m->plan_version;
  }
  MI_CUDA(cudaGraphLaunch(graph, ctx->stream));
}

// ---- prefill / eager forward ---------------------------------------------------
struct Scratch {
  std::vector<TensorRef> owned;
  mi_context* ctx;
  explicit Scratch(mi_context* c) : ctx(c) {}
  __half* f16(std::vector<size_t> shape) {
    owned.emplace_back(new_tensor(ctx, shape, MI_F16));
    return owned.back().h();
  }
};

mi_attention_kind prefill_kind(mi_attention_kind configured, size_t tokens) {
  // attention_kind_for_tokens (qwen3.rs:799-822) for tokens > 1
  switch (configured) {
    case MI_ATTENTION_TILED:
      return tokens >= 32 ? MI_ATTENTION_FLASH_PREFILL : MI_ATTENTION_TILED;
    case MI_ATTENTION_DECODE_SPLIT_KV:
    case MI_ATTENTION_FLASH_DECODE:
      return MI_ATTENTION_TILED;
    default:
      return configured;
  }
}

// out[t, n] of a row-parallel projection: the plain GEMM on one GPU; under
// tensor parallelism each rank's canonical FP32 partials over its slice of
// the input columns, summed in rank order and rounded once.
void row_parallel_gemm(mi_qwen3* m, const k::Launch& l, const __half* x, const __half* w,
                       __half* out, int t, int n, int k_local) {
  if (m->tp == 1) {
    k::gemm(l, x, w, out, t, n, k_local, n);
    return;
  }
  TensorRef part(new_tensor(m->ctx, {(size_t)t * n}, MI_F32, false));
  TensorRef gather(new_tensor(m->ctx, {(size_t)m->tp * t * n}, MI_F32, false));
  k::gemm_partial_f32(l, x, w, part.t->f32(), t, n, k_local);
  tp_reduce(m, part.t->f32(), (size_t)t * n, gather.t->f32(), out);
}

// One layer on hidden [T, h] at cache offset `off` (prefill semantics).
void layer_prefill(mi_qwen3* m, mi_kv_cache* c, size_t li, __half* hidden, size_t T, size_t off,
                   Scratch& s) {
  const auto& cfg = m->cfg;
  const Layer& L = m->layers[li];
  k::Launch l = plaunch(m);
  const int h = (int)cfg.hidden_size, I = (int)cfg.intermediate_size;
  const int qw = (int)qwidth(cfg), kw = (int)kvwidth(cfg);
  const int t = (int)T;
  const float eps = cfg.rms_norm_eps;
  __half* normalized = s.f16({T, (size_t)h});
  __half* q = s.f16({T, (size_t)qw});
  __half* kk = s.f16({T, (size_t)kw});
  __half* v = s.f16({T, (size_t)kw});
  k::rms_norm(l, hidden, L.w[kInputNorm].h(), normalized, t, h, eps);
  {
    const __half* w3[3] = {L.w[kQ].h(), L.w[kK].h(), L.w[kV].h()};
    __half* o3[3] = {q, kk, v};
    const int n3[3] = {qw, kw, kw};
    k::gemm_multi(l, normalized, t, h, 3, w3, o3, n3);
  }
  __half* query = s.f16({T, (size_t)qw});
  k::Pos pos;
  pos.base = (uint32_t)off;
  k::qk_norm_rope_cache(l, q, kk, L.w[kQNorm].h(), L.w[kKNorm].h(), query, c->key[li].h(), t,
                        (int)cfg.num_attention_heads, (int)cfg.num_key_value_heads,
                        (int)cfg.head_dim, pos, cfg.rope_theta, eps, !m->fusion.qk_rope_cache,
                        c->rope_table());
  k::copy_kv(l, v, c->value[li].h(), t, kw, pos);
  __half* attn = s.f16({T, (size_t)qw});
  k::AttnProblem a;
  a.q = query;
  a.k = c->key[li].h();
  a.v = c->value[li].h();
  a.out = attn;
  a.tokens = t;
  a.qh = (int)cfg.num_attention_heads;
  a.kvh = (int)cfg.num_key_value_heads;
  a.hd = (int)cfg.head_dim;
  a.kv_len = (int)(off + T);
  a.causal = 1;
  a.query_offset = (int)off;
  mi_attention_kind kind = T == 1 ? MI_ATTENTION_DECODE_SPLIT_KV
                                  : prefill_kind(m->attention_kind, T);
  if (m->attention_kind == MI_ATTENTION_REFERENCE) kind = MI_ATTENTION_REFERENCE;
  if (kind == MI_ATTENTION_REFERENCE) {
    k::attention_reference(l, a);
  } else if (kind == MI_ATTENTION_DECODE_SPLIT_KV) {
    auto& w = m->ws;
    int block = k::decode_block_for((int)c->capacity);
    k::attention_decode(l, a, ((int)(off + T) + block - 1) / block, block,
                        w.attn_scratch.t->f32(), w.counters.t->u32() + 1);
  } else {
    a.round_p = kind == MI_ATTENTION_FLASH_PREFILL ? 1 : 0;
    k::attention_prefill(l, a);
  }
  __half* attn_o = s.f16({T, (size_t)h});
  row_parallel_gemm(m, l, attn, L.w[kO].h(), attn_o, t, h, qw);
  __half* residual = s.f16({T, (size_t)h});
  if (m->fusion.add_rms_norm) {
    k::add_rms_norm(l, hidden, attn_o, L.w[kPostNorm].h(), residual, normalized, t, h, eps);
  } else {
    k::add(l, hidden, attn_o, residual, T * h);
    k::rms_norm(l, residual, L.w[kPostNorm].h(), normalized, t, h, eps);
  }
  __half* gate = s.f16({T, (size_t)I});
  __half* up = s.f16({T, (size_t)I});
  {
    const __half* w2[2] = {L.w[kGate].h(), L.w[kUp].h()};
    __half* o2[2] = {gate, up};
    const int n2[2] = {I, I};
    k::gemm_multi(l, normalized, t, h, 2, w2, o2, n2);
  }
  __half* act = s.f16({T, (size_t)I});
  k::swiglu(l, gate, up, act, T * I);
  __half* down = s.f16({T, (size_t)h});
  row_parallel_gemm(m, l, act, L.w[kDown].h(), down, t, h, I);
  k::add(l, residual, down, hidden, T * h);
}

void check_capacity(mi_kv_cache* c, size_t count) {
  size_t requested = c->filled + count;
  if (requested > c->capacity)
    fail(MI_ERR_CACHE_CAPACITY, "KV cache capacity %zu exceeded by requested length %zu",
         c->capacity, requested);
}

// Forward of T >= 1 tokens already in toks[filled .. filled + T): logits of
// the last row into ws.logits, greedy id into toks[filled + T], length
// advanced on host and device.
void forward_tokens(mi_qwen3* m, mi_kv_cache* c, size_t T) {
  const auto& cfg = m->cfg;
  ensure_workspace(m, c->capacity);
  size_t off = c->filled;
  if (T == 1 && decode_loop_ready(m)) {
    run_persistent_steps(m, c, 1);
    return;
  }
  if (T == 1 && fused_decode_supported(m)) {
    run_decode_step(m, c);
    c->filled += 1;
    return;
  }
  Scratch s(m->ctx);
  k::Launch l = plaunch(m);
  const int h = (int)cfg.hidden_size;
  __half* hidden = s.f16({T, (size_t)h});
  k::embedding(l, c->toks.t->u32() + off, m->embedding.h(), hidden, (int)T, h, vocab_full(m));
  for (size_t li = 0; li < m->layers.size(); ++li) layer_prefill(m, c, li, hidden, T, off, s);
  auto& w = m->ws;
  k::GemvProblem p;
  p.k = h;
  p.in_mode = k::kInNorm;
  p.x = hidden + (T - 1) * h;
  p.norm_w = m->final_norm.h();
  p.eps = cfg.rms_norm_eps;
  p.w[0] = m->lm_head->f16();
  p.n[0] = (int)cfg.vocab_size;
  p.out_mode = k::kOutArgmax;
  p.out[0] = w.logits.h();
  p.token_out = c->toks.t->u32() + off + T;
  p.argmax_partial = w.argmax_pv.t->f32();
  p.argmax_index = w.argmax_pi.t->u32();
  p.counter = w.counters.t->u32();
  if (m->tp > 1) {
    p.best_out = w.tp_best.t->u32();
    p.index_base = (uint32_t)(m->rank * cfg.vocab_size);
  }
  if (m->sampling && m->tp == 1) p.hist = w.smp_hist.t->u32();
  k::gemv(l, p);
  if (m->tp > 1) tp_argmax(m, c->toks.t->u32() + off + T, nullptr, nullptr);
  if (m->sampling) encode_sample(m, c->toks.t->u32() + off + T, nullptr, true);
  c->filled = off + T;
  set_dev_len(c, c->filled);
}

void upload_tokens(mi_kv_cache* c, const uint32_t* tokens, size_t count, size_t at) {
  MI_CUDA(cudaMemcpyAsync(c->toks.t->u32() + at, tokens, count * 4, cudaMemcpyHostToDevice,
                          c->model->ctx->stream));
}

// The last logits over the full vocabulary (gathered from the vocab shards
// under tensor parallelism).
mi_tensor* copy_logits(mi_qwen3* m) {
  mi_tensor* out = new_tensor(m->ctx, {1, m->full_cfg.vocab_size}, MI_F16);
  if (m->tp > 1) {
    tp_allgather(m, m->ws.logits.t->base(), out->base(), m->cfg.vocab_size, 2);
    return out;
  }
  MI_CUDA(cudaMemcpyAsync(out->base(), m->ws.logits.t->base(), out->bytes(),
                          cudaMemcpyDeviceToDevice, m->ctx->stream));
  return out;
}

struct Timer {
  cudaEvent_t a = nullptr, b = nullptr;
  std::chrono::steady_clock::time_point w;
  cudaStream_t s;
  explicit Timer(cudaStream_t st) : s(st) {
    cudaEventCreate(&a);
    cudaEventCreate(&b);
    cudaEventRecord(a, s);
    w = std::chrono::steady_clock::now();
  }
  void finish(mi_dispatch_stats* st) {
    cudaEventRecord(b, s);
    cudaError_t err = cudaEventSynchronize(b);
    float ms = 0;
    cudaEventElapsedTime(&ms, a, b);
    if (err != cudaSuccess) fail(MI_ERR_COMMAND, "command failed: %s", cudaGetErrorString(err));
    if (st) {
      st->gpu_time = ms * 1e-3;
      st->wall_time =
          std::chrono::duration<double>(std::chrono::steady_clock::now() - w).count();
    }
  }
  ~Timer() {
    cudaEventDestroy(a);
    cudaEventDestroy(b);
  }
};

void check_cache(mi_qwen3* m, mi_kv_cache* c) {
  require(m, "model");
  require(c, "cache");
  if (c->model != m)
    fail(MI_ERR_CONFIG, "invalid model configuration: KV cache layer count differs from model");
}

}  // namespace

extern "C" {

mi_status mi_qwen3_config_validate(const mi_qwen3_config* config) {
  return guard([&] {
    require(config, "config");
    validate_config(*config);
  });
}

mi_status mi_tp_shard(const mi_qwen3_config* config, int tp, int rank, mi_tp_shard_info* out) {
  return guard([&] {
    require(config, "config");
    require(out, "out");
    validate_config(*config);
    const auto& c = *config;
    if (tp < 1 || rank < 0 || rank >= tp)
      fail(MI_ERR_CONFIG, "invalid model configuration: rank %d outside tensor-parallel size %d",
           rank, tp);
    if (c.num_attention_heads % tp || c.num_key_value_heads % tp || c.intermediate_size % tp ||
        c.vocab_size % tp)
      fail(MI_ERR_CONFIG,
           "invalid model configuration: heads, KV heads, intermediate size and vocabulary must "
           "divide by the tensor-parallel size %d", tp);
    if (tp > 1 && ((c.intermediate_size / tp) % 8 || (c.num_attention_heads / tp * c.head_dim) % 8))
      fail(MI_ERR_CONFIG,
           "invalid model configuration: per-rank input slices must be multiples of 8");
    mi_tp_shard_info s{};
    s.q_heads = c.num_attention_heads / tp;
    s.kv_heads = c.num_key_value_heads / tp;
    s.intermediate = c.intermediate_size / tp;
    s.vocab = c.vocab_size / tp;
    s.q_head0 = (size_t)rank * s.q_heads;
    s.kv_head0 = (size_t)rank * s.kv_heads;
    s.inter0 = (size_t)rank * s.intermediate;
    s.vocab0 = (size_t)rank * s.vocab;
    *out = s;
  });
}

mi_status mi_nccl_unique_id(uint8_t* out, size_t len) {
  return guard([&] {
    require(out, "out");
#ifdef MI_HAVE_NCCL
    MI_REQUIRE(len >= sizeof(ncclUniqueId), MI_ERR_INVALID_ARGUMENT,
               "the NCCL id needs %zu bytes", sizeof(ncclUniqueId));
    ncclUniqueId id;
    ncclResult_t r = ncclGetUniqueId(&id);
    if (r != ncclSuccess) fail(MI_ERR_COLLECTIVE, "ncclGetUniqueId: %s", ncclGetErrorString(r));
    std::memcpy(out, &id, sizeof id);
#else
    (void)len;
    fail(MI_ERR_UNSUPPORTED, "built without NCCL: tensor parallelism is unavailable");
#endif
  });
}

}  // extern "C"

namespace {

// Persistent tensor-parallel decode: allocate this rank's mailbox, export it
// (CUDA IPC), gather every rank's handle over NCCL and map the peers'
// mailboxes here. The mailbox starts zeroed (no tag matches zero).
void setup_mailbox(mi_qwen3* m) {
#ifdef MI_HAVE_NCCL
  mi_context* ctx = m->ctx;
  auto& mb = m->mbox;
  mb.grid = std::min(ctx->sm_count, 256);
  const k::MailboxLayout lay =
      k::mailbox_layout(m->tp, (int)m->full_cfg.hidden_size, mb.grid);
  const size_t bytes = lay.words * 8;
  MI_CUDA(cudaMalloc(&mb.local, bytes));
  MI_CUDA(cudaMemset(mb.local, 0, bytes));
  cudaIpcMemHandle_t mine;
  MI_CUDA(cudaIpcGetMemHandle(&mine, mb.local));
  TensorRef dev_mine(new_tensor(ctx, {sizeof mine}, MI_F16, false));  // byte carrier
  TensorRef dev_all(new_tensor(ctx, {sizeof mine * (size_t)m->tp}, MI_F16, false));
  MI_CUDA(cudaMemcpy(dev_mine.t->base(), &mine, sizeof mine, cudaMemcpyHostToDevice));
  ncclResult_t r = ncclAllGather(dev_mine.t->base(), dev_all.t->base(), sizeof mine, ncclUint8,
                                 m->comm, ctx->stream);
  if (r != ncclSuccess)
    fail(MI_ERR_COLLECTIVE, "NCCL all-gather of IPC handles: %s", ncclGetErrorString(r));
  std::vector<cudaIpcMemHandle_t> all(m->tp);
  MI_CUDA(cudaMemcpyAsync(all.data(), dev_all.t->base(), sizeof mine * m->tp,
                          cudaMemcpyDeviceToHost, ctx->stream));
  MI_CUDA(cudaStreamSynchronize(ctx->stream));
  mb.peer.assign(m->tp, nullptr);
  for (int q = 0; q < m->tp; ++q) {
    if (q == m->rank) {
      mb.peer[q] = mb.local;
      continue;
    }
    MI_CUDA(cudaIpcOpenMemHandle(&mb.peer[q], all[q], cudaIpcMemLazyEnablePeerAccess));
  }
  mb.table = TensorRef(new_tensor(ctx, {(size_t)m->tp * 2}, MI_U32, false));
  MI_CUDA(cudaMemcpy(mb.table.t->base(), mb.peer.data(), sizeof(void*) * m->tp,
                     cudaMemcpyHostToDevice));
#else
  (void)m;
#endif
}

// Fills `dst` ([rows, cols] FP16) with the block at (row0, col0) of the full
// [*, full_cols] weight (layer, role); 1-D norms come as one row.
using WeightFill = std::function<void(int layer, int role, __half* dst, size_t rows, size_t cols,
                                      size_t full_cols, size_t row0, size_t col0)>;

// A model, or this rank's shard of it under tensor parallelism (tp ranks):
// every shard is the corresponding block of the full tensors, taken from
// `fill`. Embedding and norms are replicated; a tied LM head is a view of
// the embedding rows of the rank's vocabulary shard.
mi_qwen3* build_model(mi_context* ctx, const mi_qwen3_config& config, int tp, int rank,
                      const uint8_t* nccl_id, const WeightFill& fill) {
  validate_config(config);
  mi_tp_shard_info sh{};
  {
    mi_status st = mi_tp_shard(&config, tp, rank, &sh);
    if (st != MI_OK) fail(st, "%s", mi_last_error_message());
  }
  auto m = std::make_unique<mi_qwen3>();
  m->ctx = ctx;
  m->full_cfg = config;
  m->cfg = config;
  m->cfg.num_attention_heads = (uint32_t)sh.q_heads;
  m->cfg.num_key_value_heads = (uint32_t)sh.kv_heads;
  m->cfg.intermediate_size = (uint32_t)sh.intermediate;
  m->cfg.vocab_size = (uint32_t)sh.vocab;
  m->tp = tp;
  m->rank = rank;
  context_retain(ctx);
  struct CtxGuard {
    mi_qwen3* m;
    ~CtxGuard() {
      if (m) context_release(m->ctx);
    }
  } ctx_guard{m.get()};
  const auto& fc = m->full_cfg;
  const size_t h = fc.hidden_size, hd = fc.head_dim, V = fc.vocab_size;
  const size_t qw = qwidth(fc), I = fc.intermediate_size;
  const size_t qw_l = qwidth(m->cfg), kw_l = kvwidth(m->cfg), I_l = m->cfg.intermediate_size;
  auto block = [&](int layer, int role, size_t rows, size_t cols, size_t full_cols, size_t row0,
                   size_t col0) {
    TensorRef t(new_tensor(ctx, {rows, cols}, MI_F16));
    fill(layer, role, t.h(), rows, cols, full_cols, row0, col0);
    return t;
  };
  auto vec = [&](int layer, int role, size_t n) {
    TensorRef t(new_tensor(ctx, {n}, MI_F16));
    fill(layer, role, t.h(), 1, n, n, 0, 0);
    return t;
  };
  m->embedding = block(-1, kEmbedding, V, h, h, 0, 0);
  m->final_norm = vec(-1, kFinalNorm, h);
  if (fc.tie_word_embeddings) {
    if (tp == 1) {
      m->lm_head = m->embedding.t;
    } else {
      m->lm_head_own = TensorRef(view(m->embedding.t, {sh.vocab, h}, sh.vocab0 * h * 2));
      m->lm_head = m->lm_head_own.t;
    }
  } else {
    m->lm_head_own = block(-1, kLmHead, sh.vocab, h, h, sh.vocab0, 0);
    m->lm_head = m->lm_head_own.t;
  }
  m->layers.resize(fc.num_hidden_layers);
  for (size_t l = 0; l < fc.num_hidden_layers; ++l) {
    Layer& L = m->layers[l];
    const int li = (int)l;
    L.w[kQ] = block(li, kQ, qw_l, h, h, sh.q_head0 * hd, 0);
    L.w[kK] = block(li, kK, kw_l, h, h, sh.kv_head0 * hd, 0);
    L.w[kV] = block(li, kV, kw_l, h, h, sh.kv_head0 * hd, 0);
    L.w[kO] = block(li, kO, h, qw_l, qw, 0, sh.q_head0 * hd);
    L.w[kQNorm] = vec(li, kQNorm, hd);
    L.w[kKNorm] = vec(li, kKNorm, hd);
    L.w[kGate] = block(li, kGate, I_l, h, h, sh.inter0, 0);
    L.w[kUp] = block(li, kUp, I_l, h, h, sh.inter0, 0);
    L.w[kDown] = block(li, kDown, h, I_l, I, 0, sh.inter0);
    L.w[kInputNorm] = vec(li, kInputNorm, h);
    L.w[kPostNorm] = vec(li, kPostNorm, h);
  }
  if (tp > 1) {
#ifdef MI_HAVE_NCCL
    require(nccl_id, "nccl_id");
    ncclUniqueId id;
    std::memcpy(&id, nccl_id, sizeof id);
    MI_CUDA(cudaSetDevice(ctx->device));
    ncclResult_t r = ncclCommInitRank(&m->comm, tp, id, rank);
    if (r != ncclSuccess)
      fail(MI_ERR_COLLECTIVE, "ncclCommInitRank (rank %d of %d): %s", rank, tp,
           ncclGetErrorString(r));
    setup_mailbox(m.get());
#else
    (void)nccl_id;
    fail(MI_ERR_UNSUPPORTED, "built without NCCL: tensor parallelism is unavailable");
#endif
  }
  sync_context(ctx);
  ctx_guard.m = nullptr;
  return m.release();
}

// Seeded N(0, std) matrices and unit norm gains (mi_qwen3_create_random).
WeightFill random_fill(cudaStream_t st, uint64_t seed, double std_dev) {
  return [=](int layer, int role, __half* dst, size_t rows, size_t cols, size_t full_cols,
             size_t row0, size_t col0) {
    if (role == kQNorm || role == kKNorm || role == kInputNorm || role == kPostNorm ||
        role == kFinalNorm) {
      k::fill_f16(st, dst, rows * cols, 0x3c00);
      return;
    }
    k::fill_normal_f16_block(st, dst, rows, cols, full_cols, row0, col0, seed,
                             (uint64_t)((layer + 1) * 16 + role), std_dev);
  };
}

// Weights from a safetensors checkpoint (qwen3.rs:155-240): each tensor is
// checked against the full config's shape, then the shard block is read.
WeightFill checkpoint_fill(const load::Checkpoint& ck, cudaStream_t st) {
  const mi_qwen3_config& c = ck.config();
  const size_t h = c.hidden_size, hd = c.head_dim, V = c.vocab_size, I = c.intermediate_size;
  const size_t qw = qwidth(c), kw = kvwidth(c);
  return [&ck, st, h, hd, V, I, qw, kw](int layer, int role, __half* dst, size_t rows,
                                          size_t cols, size_t, size_t row0, size_t col0) {
    std::vector<size_t> shape;
    switch (role) {
      case kEmbedding: case kLmHead: shape = {V, h}; break;
      case kQ: shape = {qw, h}; break;
      case kK: case kV: shape = {kw, h}; break;
      case kO: shape = {h, qw}; break;
      case kQNorm: case kKNorm: shape = {hd}; break;
      case kGate: case kUp: shape = {I, h}; break;
      case kDown: shape = {h, I}; break;
      default: shape = {h}; break;
    }
    const std::string name = load::weight_name(layer, role);
    ck.expect(name, shape);
    ck.read_block(name, rows, cols, row0, col0, dst, st);
  };
}

mi_qwen3* build_random(mi_context* ctx, const mi_qwen3_config& config, uint64_t seed,
                       double std_dev, int tp, int rank, const uint8_t* nccl_id) {
  return build_model(ctx, config, tp, rank, nccl_id, random_fill(ctx->stream, seed, std_dev));
}

mi_qwen3* build_loaded(mi_context* ctx, const char* directory, int tp, int rank,
                       const uint8_t* nccl_id) {
  auto ck = load::Checkpoint::open(directory);
  return build_model(ctx, ck->config(), tp, rank, nccl_id, checkpoint_fill(*ck, ctx->stream));
}

}  // namespace

extern "C" {

mi_status mi_qwen3_create_random(mi_context* ctx, const mi_qwen3_config* config, uint64_t seed,
                                 double std_dev, mi_qwen3** out) {
  return guard([&] {
    require(ctx, "ctx");
    require(config, "config");
    require(out, "out");
    *out = build_random(ctx, *config, seed, std_dev, 1, 0, nullptr);
  });
}

mi_status mi_qwen3_create_random_tp(mi_context* ctx, const mi_qwen3_config* config,
                                    uint64_t seed, double std_dev, int tp, int rank,
                                    const uint8_t* nccl_id, mi_qwen3** out) {
  return guard([&] {
    require(ctx, "ctx");
    require(config, "config");
    require(out, "out");
    *out = build_random(ctx, *config, seed, std_dev, tp, rank, nccl_id);
  });
}

void mi_qwen3_destroy(mi_qwen3* m) { model_release(m); }

mi_status mi_qwen3_get_config(const mi_qwen3* m, mi_qwen3_config* out) {
  return guard([&] {
    require(m, "model");
    require(out, "out");
    *out = m->full_cfg;
  });
}

mi_status mi_qwen3_set_attention_kind(mi_qwen3* m, mi_attention_kind kind) {
  return guard([&] {
    require(m, "model");
    MI_REQUIRE(kind >= MI_ATTENTION_REFERENCE && kind <= MI_ATTENTION_FLASH_DECODE,
               MI_ERR_INVALID_ARGUMENT, "unknown attention kind %d", (int)kind);
    m->attention_kind = kind;
    m->plan_version++;
  });
}

mi_status mi_qwen3_set_fusion_options(mi_qwen3* m, mi_fusion_options options) {
  return guard([&] {
    require(m, "model");
    m->fusion = options;
    m->plan_version++;
  });
}

mi_fusion_options mi_qwen3_fusion_options(const mi_qwen3* m) {
  return m ? m->fusion : mi_fusion_options{1, 1, 1, 1};
}

mi_status mi_qwen3_set_decode_graphs(mi_qwen3* m, int enabled) {
  return guard([&] {
    require(m, "model");
    m->graphs = enabled != 0;
  });
}

mi_status mi_qwen3_set_decode_persistent(mi_qwen3* m, int enabled) {
  return guard([&] {
    require(m, "model");
    m->persistent = enabled != 0;
  });
}

mi_status mi_qwen3_exchange_wait(mi_qwen3* m, double* mean_seconds, double* max_seconds,
                                 size_t* steps) {
  return guard([&] {
    require(m, "model");
    require(mean_seconds, "mean_seconds");
    require(max_seconds, "max_seconds");
    require(steps, "steps");
    *mean_seconds = *max_seconds = 0.0;
    *steps = (size_t)m->last_loop_steps;
    if (m->tp == 1 || !m->ws.loop_sync.t || m->last_loop_steps == 0) return;
    const int grid = m->loop.grid;
    std::vector<uint32_t> words((size_t)grid);
    MI_CUDA(cudaMemcpyAsync(words.data(), m->ws.loop_sync.t->u32() + k::decode_loop_wait_word0(),
                            words.size() * 4, cudaMemcpyDeviceToHost, m->ctx->stream));
    MI_CUDA(cudaStreamSynchronize(m->ctx->stream));
    double sum = 0.0, mx = 0.0;
    for (uint32_t v : words) {
      const double sec = (double)v * 64e-9;
      sum += sec;
      mx = std::max(mx, sec);
    }
    *mean_seconds = sum / grid;
    *max_seconds = mx;
  });
}

mi_status mi_qwen3_decode_persistent(mi_qwen3* m, int* active) {
  return guard([&] {
    require(m, "model");
    require(active, "active");
    *active = decode_loop_ready(m) ? 1 : 0;
  });
}

mi_status mi_kv_cache_create(mi_qwen3* m, size_t capacity, mi_kv_cache** out) {
  return guard([&] {
    require(m, "model");
    require(out, "out");
    if (capacity == 0)
      fail(MI_ERR_CONFIG, "invalid model configuration: KV cache capacity must be non-zero");
    MI_REQUIRE(capacity < 0x7FFFFFFF, MI_ERR_CONFIG, "KV cache capacity too large");
    auto c = std::make_unique<mi_kv_cache>();
    c->model = m;
    m->refs.fetch_add(1);
    c->capacity = capacity;
    size_t kvh = m->cfg.num_key_value_heads, hd = m->cfg.head_dim;
    for (size_t l = 0; l < m->cfg.num_hidden_layers; ++l) {
      c->key.emplace_back(new_tensor(m->ctx, {capacity, kvh, hd}, MI_F16, true));
      c->value.emplace_back(new_tensor(m->ctx, {capacity, kvh, hd}, MI_F16, true));
    }
    c->toks = TensorRef(new_tensor(m->ctx, {capacity + 1}, MI_U32, true));
    c->dev_len = TensorRef(new_tensor(m->ctx, {1}, MI_U32, true));
    c->rope = TensorRef(new_tensor(m->ctx, {capacity, hd / 2, 2}, MI_F32));
    k::rope_table(m->ctx->stream, reinterpret_cast<float2*>(c->rope.t->f32()), (int)capacity,
                  (int)hd, m->cfg.rope_theta);
    ensure_workspace(m, capacity);
    sync_context(m->ctx);
    *out = c.release();
  });
}

void mi_kv_cache_destroy(mi_kv_cache* c) {
  if (!c) return;
  mi_qwen3* m = c->model;
  cudaSetDevice(m->ctx->device);
  cudaStreamSynchronize(m->ctx->stream);
  delete c;
  model_release(m);
}

size_t mi_kv_cache_len(const mi_kv_cache* c) { return c ? c->filled : 0; }
size_t mi_kv_cache_capacity(const mi_kv_cache* c) { return c ? c->capacity : 0; }

void mi_kv_cache_reset(mi_kv_cache* c) {
  if (!c) return;
  c->filled = 0;
  try {
    set_dev_len(c, 0);
  } catch (...) {
  }
}

mi_status mi_kv_cache_layer(mi_kv_cache* c, size_t layer, mi_tensor** key, mi_tensor** value) {
  return guard([&] {
    require(c, "cache");
    MI_REQUIRE(layer < c->key.size(), MI_ERR_INVALID_ARGUMENT, "layer %zu out of range", layer);
    if (key) *key = view(c->key[layer].t, c->key[layer].t->shape, 0);
    if (value) *value = view(c->value[layer].t, c->value[layer].t->shape, 0);
  });
}

// prefill_with_stats (qwen3.rs:356-373)
mi_status mi_qwen3_prefill(mi_qwen3* m, const uint32_t* tokens, size_t count, mi_kv_cache* cache,
                           mi_tensor** logits, mi_dispatch_stats* stats) {
  return guard([&] {
    check_cache(m, cache);
    if (count == 0) fail(MI_ERR_CONFIG, "invalid model configuration: prefill requires at least one token");
    require(tokens, "tokens");
    cache->filled = 0;  // KvCache::reset, then the capacity check (qwen3.rs:366, 617-624)
    set_dev_len(cache, 0);
    check_capacity(cache, count);
    Timer t(m->ctx->stream);
    upload_tokens(cache, tokens, count, 0);
    try {
      forward_tokens(m, cache, count);
      t.finish(stats);
    } catch (...) {
      cache->filled = 0;
      throw;
    }
    if (logits) *logits = copy_logits(m);
  });
}

// decode_with_stats (qwen3.rs:375-386)
mi_status mi_qwen3_decode(mi_qwen3* m, uint32_t token, mi_kv_cache* cache, mi_tensor** logits,
                          mi_dispatch_stats* stats) {
  return guard([&] {
    check_cache(m, cache);
    check_capacity(cache, 1);
    size_t previous = cache->filled;
    Timer t(m->ctx->stream);
    uint32_t tok = token;
    upload_tokens(cache, &tok, 1, previous);
    try {
      forward_tokens(m, cache, 1);
      t.finish(stats);
    } catch (...) {
      cache->filled = previous;
      set_dev_len(cache, previous);
      throw;
    }
    if (logits) *logits = copy_logits(m);
  });
}

// prefill_argmax (qwen3.rs:388-410)
mi_status mi_qwen3_prefill_argmax(mi_qwen3* m, const uint32_t* tokens, size_t count,
                                  mi_kv_cache* cache, mi_tensor* output, mi_tensor** logits,
                                  mi_dispatch_stats* stats) {
  return guard([&] {
    check_cache(m, cache);
    if (count == 0) fail(MI_ERR_CONFIG, "invalid model configuration: prefill requires at least one token");
    require(tokens, "tokens");
    require(output, "output");
    if (output->dtype != MI_U32 || output->len() != 1)
      fail(MI_ERR_CONFIG, "invalid model configuration: argmax output must be one u32");
    cache->filled = 0;  // KvCache::reset, then the capacity check (qwen3.rs:366, 617-624)
    set_dev_len(cache, 0);
    check_capacity(cache, count);
    Timer t(m->ctx->stream);
    upload_tokens(cache, tokens, count, 0);
    try {
      forward_tokens(m, cache, count);
      MI_CUDA(cudaMemcpyAsync(output->base(), cache->toks.t->u32() + count, 4,
                              cudaMemcpyDeviceToDevice, m->ctx->stream));
      t.finish(stats);
    } catch (...) {
      cache->filled = 0;
      throw;
    }
    if (logits) *logits = copy_logits(m);
  });
}

// decode_argmax (qwen3.rs:412-422)
mi_status mi_qwen3_decode_argmax(mi_qwen3* m, const mi_tensor* token, mi_kv_cache* cache,
                                 mi_tensor* output, mi_tensor** logits, mi_pending** pending) {
  return guard([&] {
    check_cache(m, cache);
    require(token, "token");
    require(output, "output");
    require(pending, "pending");
    if (token->shape != std::vector<size_t>{1} || token->dtype != MI_U32)
      fail(MI_ERR_CONFIG, "invalid model configuration: decode token must be one u32");
    if (output->dtype != MI_U32 || output->len() != 1)
      fail(MI_ERR_CONFIG, "invalid model configuration: argmax output must be one u32");
    check_capacity(cache, 1);
    mi_batch* b = nullptr;
    mi_status s = mi_context_begin_batch(m->ctx, &b);
    if (s != MI_OK) fail(s, "%s", mi_last_error_message());
    size_t previous = cache->filled;
    try {
      MI_CUDA(cudaMemcpyAsync(cache->toks.t->u32() + previous, token->base(), 4,
                              cudaMemcpyDeviceToDevice, m->ctx->stream));
      forward_tokens(m, cache, 1);
      MI_CUDA(cudaMemcpyAsync(output->base(), cache->toks.t->u32() + previous + 1, 4,
                              cudaMemcpyDeviceToDevice, m->ctx->stream));
      if (logits) *logits = copy_logits(m);
    } catch (...) {
      mi_batch_abandon(b);
      cache->filled = previous;
      throw;
    }
    s = mi_batch_commit(b, pending);
    if (s != MI_OK) fail(s, "%s", mi_last_error_message());
  });
}

}  // extern "C"

namespace {

// `n` decode steps from the cache's device position.
void decode_steps(mi_qwen3* m, mi_kv_cache* c, size_t n) {
  if (n == 0) return;
  if (decode_loop_ready(m)) {
    run_persistent_steps(m, c, n);
    return;
  }
  for (size_t i = 0; i < n; ++i) forward_tokens(m, c, 1);
}

// generate_greedy (qwen3.rs:475-555): prefill, then decode steps enqueued
// back to back on the device. Without stop tokens or a callback all steps are
// launched before the single readback; otherwise steps are checked in chunks
// and the cache length is rolled back past a stop.
size_t generate_greedy(mi_qwen3* m, mi_kv_cache* c, const uint32_t* prompt, size_t prompt_len,
                       size_t max_tokens, const uint32_t* stops, size_t nstops,
                       mi_token_callback cb, void* user, uint32_t* out_ids, size_t capacity) {
  if (max_tokens == 0) return 0;
  if (prompt_len == 0)
    fail(MI_ERR_CONFIG, "invalid model configuration: prefill requires at least one token");
  c->filled = 0;
  set_dev_len(c, 0);
  check_capacity(c, prompt_len);
  // Decode steps needed: max_tokens - 1 (the first id comes from prefill).
  size_t steps = max_tokens - 1;
  if (prompt_len + steps > c->capacity)
    fail(MI_ERR_CACHE_CAPACITY, "KV cache capacity %zu exceeded by requested length %zu",
         c->capacity, prompt_len + steps);
  upload_tokens(c, prompt, prompt_len, 0);
  forward_tokens(m, c, prompt_len);
  std::vector<uint32_t> ids(max_tokens);
  size_t produced = 0;
  size_t stop_index = max_tokens;  // index of the token that ended generation
  const bool checks = nstops > 0 || cb != nullptr;
  const size_t chunk = checks ? 16 : max_tokens;
  size_t launched = 0;  // decode steps enqueued
  size_t have = 0;      // ids copied to host
  size_t seen = 0;      // ids examined
  while (stop_index == max_tokens && seen < max_tokens) {
    size_t n_new = std::min(chunk, steps - launched);
    decode_steps(m, c, n_new);
    launched += n_new;
    size_t avail = 1 + launched;  // ids at toks[prompt_len .. prompt_len + avail)
    MI_CUDA(cudaMemcpyAsync(ids.data() + have, c->toks.t->u32() + prompt_len + have,
                            (avail - have) * 4, cudaMemcpyDeviceToHost, m->ctx->stream));
    MI_CUDA(cudaStreamSynchronize(m->ctx->stream));
    // a launch whose bounded wait expired left early: its ids are not valid
    check_device_waits("generate");
    have = avail;
    for (; seen < have && stop_index == max_tokens; ++seen) {
      uint32_t tok = ids[seen];
      if (tok == 0xFFFFFFFFu)
        fail(MI_ERR_CONFIG, "invalid model configuration: logits contain no finite value");
      if (tok == 0xFFFFFFFEu)
        fail(MI_ERR_CONFIG, "invalid model configuration: failed to sample a token");
      bool is_stop = false;
      for (size_t s = 0; s < nstops; ++s) is_stop |= stops[s] == tok;
      if (is_stop) {
        stop_index = seen;
        break;
      }
      if (produced < capacity) out_ids[produced] = tok;
      ++produced;
      if (cb && !cb(tok, user)) stop_index = seen;
    }
  }
  if (stop_index < max_tokens) {
    // As generate_greedy's rollback: the cache keeps the prompt and the
    // tokens fed back before the one that ended generation.
    size_t keep = prompt_len + stop_index;
    if (keep < c->filled) {
      c->filled = keep;
      set_dev_len(c, keep);
    }
  }
  return produced;
}

}  // namespace

extern "C" {

mi_status mi_qwen3_decode_steps(mi_qwen3* m, mi_kv_cache* cache, size_t steps) {
  return guard([&] {
    check_cache(m, cache);
    if (cache->filled == 0)
      fail(MI_ERR_CONFIG, "invalid model configuration: decode needs a prefilled cache");
    check_capacity(cache, steps);
    decode_steps(m, cache, steps);
  });
}

mi_status mi_kv_cache_tokens(mi_kv_cache* cache, size_t start, size_t count, uint32_t* out) {
  return guard([&] {
    require(cache, "cache");
    if (count) require(out, "out");
    MI_REQUIRE(start <= cache->capacity + 1 && count <= cache->capacity + 1 - start,
               MI_ERR_SHAPE, "token range %zu..%zu is outside the cache", start, start + count);
    mi_context* ctx = cache->model->ctx;
    MI_CUDA(cudaMemcpyAsync(out, cache->toks.t->u32() + start, count * 4, cudaMemcpyDeviceToHost,
                            ctx->stream));
    MI_CUDA(cudaStreamSynchronize(ctx->stream));
    // decode_steps is asynchronous: a timed-out launch is reported here,
    // at the first call that reads its ids
    check_device_waits("kv_cache_tokens");
  });
}

// generate (qwen3.rs:424-439)
mi_status mi_qwen3_generate(mi_qwen3* m, const uint32_t* prompt, size_t prompt_len,
                            size_t max_tokens, mi_kv_cache* cache, uint32_t* out_ids,
                            size_t* out_count) {
  return guard([&] {
    check_cache(m, cache);
    require(out_count, "out_count");
    if (max_tokens) require(out_ids, "out_ids");
    require(prompt, "prompt");
    *out_count = generate_greedy(m, cache, prompt, prompt_len, max_tokens, nullptr, 0, nullptr,
                                 nullptr, out_ids, max_tokens);
  });
}

// generate_with (qwen3.rs:441-473)
mi_status mi_qwen3_generate_with(mi_qwen3* m, const uint32_t* prompt, size_t prompt_len,
                                 const mi_generation_options* options, mi_kv_cache* cache,
                                 mi_token_callback on_token, void* user, uint32_t* out_ids,
                                 size_t capacity, size_t* out_count) {
  return guard([&] {
    check_cache(m, cache);
    require(options, "options");
    require(out_count, "out_count");
    require(prompt, "prompt");
    if (!std::isfinite(options->temperature) || options->temperature < 0.f)
      fail(MI_ERR_CONFIG, "invalid model configuration: temperature must be finite and non-negative");
    // validate_generation_options (qwen3.rs:897-907)
    if (!std::isfinite(options->top_p) || !(options->top_p >= 0.f && options->top_p <= 1.f))
      fail(MI_ERR_CONFIG, "invalid model configuration: top_p must be between 0 and 1");
    if (options->temperature == 0.f || options->max_tokens == 0) {
      *out_count = generate_greedy(m, cache, prompt, prompt_len, options->max_tokens,
                                   options->stop_token_ids, options->stop_token_count, on_token,
                                   user, out_ids, capacity);
      return;
    }
    // Sampled (qwen3.rs:455-472): the same pipelined loop, each lm_head
    // followed by the sampler, one XorShift64 stream for the whole call.
    if (options->top_k > 0xFFFFFFFFull)
      fail(MI_ERR_CONFIG, "invalid model configuration: top_k does not fit in u32");
    ensure_sampling(m);
    const float inv = 1.0f / options->temperature;
    uint32_t opts[4];
    std::memcpy(&opts[0], &inv, 4);
    std::memcpy(&opts[1], &options->top_p, 4);
    opts[2] = (uint32_t)options->top_k;
    opts[3] = 0;
    const uint64_t state = options->seed == 0 ? 0x9e3779b97f4a7c15ull : options->seed;
    MI_CUDA(cudaMemcpyAsync(m->ws.smp_opts.t->base(), opts, sizeof(opts), cudaMemcpyHostToDevice,
                            m->ctx->stream));
    MI_CUDA(cudaMemcpyAsync(m->ws.smp_state.t->base(), &state, 8, cudaMemcpyHostToDevice,
                            m->ctx->stream));
    // the host copies above read pageable memory before returning
    struct Scope {
      mi_qwen3* m;
      ~Scope() { m->sampling = false; }
    } scope{m};
    m->sampling = true;
    *out_count = generate_greedy(m, cache, prompt, prompt_len, options->max_tokens,
                                 options->stop_token_ids, options->stop_token_count, on_token,
                                 user, out_ids, capacity);
  });
}

// run_first_block (qwen3.rs:557-583)
mi_status mi_qwen3_run_first_block(mi_qwen3* m, const uint32_t* tokens, size_t count,
                                   mi_tensor** out) {
  return guard([&] {
    require(m, "model");
    require(out, "out");
    if (count == 0) fail(MI_ERR_CONFIG, "invalid model configuration: block benchmark requires tokens");
    require(tokens, "tokens");
    mi_kv_cache* c = nullptr;
    mi_status s = mi_kv_cache_create(m, count, &c);
    if (s != MI_OK) fail(s, "%s", mi_last_error_message());
    std::unique_ptr<mi_kv_cache, void (*)(mi_kv_cache*)> guard_cache(c, mi_kv_cache_destroy);
    upload_tokens(c, tokens, count, 0);
    const int h = (int)m->cfg.hidden_size;
    TensorRef hidden(new_tensor(m->ctx, {count, (size_t)h}, MI_F16));
    k::embedding(launch(m, false), c->toks.t->u32(), m->embedding.h(), hidden.h(), (int)count, h,
                 vocab_full(m));
    Scratch sc(m->ctx);
    layer_prefill(m, c, 0, hidden.h(), count, 0, sc);
    sync_context(m->ctx);
    *out = hidden.t;
    hidden.t = nullptr;
  });
}

// Every layer on given hidden states (no embedding, no head).
mi_status mi_qwen3_forward_hidden(mi_qwen3* m, const mi_tensor* hidden, mi_kv_cache* cache,
                                  mi_tensor** out) {
  return guard([&] {
    check_cache(m, cache);
    require(hidden, "hidden");
    require(out, "out");
    if (hidden->dtype != MI_F16 || hidden->shape.size() != 2 ||
        hidden->shape[1] != m->cfg.hidden_size || hidden->shape[0] == 0)
      fail(MI_ERR_SHAPE, "invalid tensor shape: hidden must be [tokens, hidden_size] f16");
    size_t T = hidden->shape[0];
    check_capacity(cache, T);
    ensure_workspace(m, cache->capacity);
    TensorRef x(new_tensor(m->ctx, hidden->shape, MI_F16));
    MI_CUDA(cudaMemcpyAsync(x.h(), hidden->base(), hidden->bytes(), cudaMemcpyDeviceToDevice,
                            m->ctx->stream));
    Scratch sc(m->ctx);
    size_t off = cache->filled;
    for (size_t li = 0; li < m->layers.size(); ++li) layer_prefill(m, cache, li, x.h(), T, off, sc);
    cache->filled = off + T;
    set_dev_len(cache, cache->filled);
    sync_context(m->ctx);
    *out = x.t;
    x.t = nullptr;
  });
}

mi_status mi_qwen3_weight(mi_qwen3* m, int layer, int role, mi_tensor** out) {
  return guard([&] {
    require(m, "model");
    require(out, "out");
    const mi_tensor* t = nullptr;
    if (layer < 0) {
      if (role == kEmbedding) t = m->embedding.t;
      else if (role == kFinalNorm) t = m->final_norm.t;
      else if (role == kLmHead) t = m->lm_head;
    } else if ((size_t)layer < m->layers.size() && role > 0 && role < 16) {
      t = m->layers[layer].w[role].t;
    }
    if (!t) fail(MI_ERR_MISSING_TENSOR, "missing model tensor (layer %d, role %d)", layer, role);
    *out = view(t, t->shape, 0);
  });
}

mi_status mi_qwen3_load(mi_context* ctx, const char* directory, mi_qwen3** out) {
  return guard([&] {
    require(ctx, "ctx");
    require(directory, "directory");
    require(out, "out");
    *out = build_loaded(ctx, directory, 1, 0, nullptr);
  });
}

mi_status mi_qwen3_load_tp(mi_context* ctx, const char* directory, int tp, int rank,
                           const uint8_t* nccl_id, mi_qwen3** out) {
  return guard([&] {
    require(ctx, "ctx");
    require(directory, "directory");
    require(out, "out");
    *out = build_loaded(ctx, directory, tp, rank, nccl_id);
  });
}

}  // extern "C"
