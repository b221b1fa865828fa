// Kernel launch interfaces shared by the op layer (ops.cu) and the Qwen3
// forward plans (qwen3.cu). Every launcher takes a Launch describing the
// stream and whether the launch may overlap its predecessor through
// programmatic dependent launch (PDL): such kernels issue their
// predecessor-independent loads (weights) first and block on
// griddepcontrol.wait before touching activations.
#pragma once

#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <cstdint>

namespace mi {
namespace k {

struct Launch {
  cudaStream_t stream;
  bool pdl = false;
  // Kernels may read operands no predecessor writes (weights, cached K/V
  // rows) before their dependency wait. True inside the model's launches;
  // the op API, whose operands may be any earlier op's outputs, clears it.
  bool early = true;
  int sm_count = 148;
};

// Position of a step: kernels read `*dev + base` when dev is non-null (decode
// graphs keep the cache length on the device), else `base`.
struct Pos {
  const uint32_t* dev = nullptr;
  uint32_t base = 0;
};

// ---- decode GEMV family (M = 1) -------------------------------------------
enum GemvIn : int {
  kInPlain = 0,    // x as given
  kInNorm = 1,     // half(x * rsqrt(mean(x^2) + eps) * g)       (matvec3_rms)
  kInAddNorm = 2,  // r = x + x2; half(half(r) * scale * g)       (matvec2_add_rms)
  kInEmbedNorm = 3, // x = table[token] (0 for 0xFFFFFFFF), then kInNorm
  kInAddThenNorm = 4 // r = half(x + x2) (half add); half(r * scale(r) * g)  (add_f16 + rms_norm_f16)
};
enum GemvOut : int {
  kOutPlain = 0,     // out[s][row] = half(dot)
  kOutResidual = 1,  // out0[row] = res[row] + half(dot)  (half add)
  kOutSwiglu = 2,    // out0[i] = half(silu(g) * u), g/u = half dots of rows i of w0/w1
  kOutArgmax = 3,    // out0 = logits; greedy id of the logits -> token_out
  kOutF32 = 4        // outf[row] = dot (FP32, unrounded: a tensor-parallel partial)
};

struct GemvProblem {
  const __half* w[3] = {nullptr, nullptr, nullptr};
  int n[3] = {0, 0, 0};
  int segments = 1;
  int k = 0;
  // prologue
  int in_mode = kInPlain;
  const __half* x = nullptr;
  const __half* x2 = nullptr;
  const __half* norm_w = nullptr;
  float eps = 1e-6f;
  __half* residual_out = nullptr;     // kInAddNorm (block 0 writes)
  const uint32_t* token = nullptr;    // kInEmbedNorm: token = token[token_pos ? *token_pos : 0]
  const uint32_t* token_pos = nullptr;
  const __half* table = nullptr;      // kInEmbedNorm
  uint32_t table_rows = 0;
  __half* embed_out = nullptr;        // kInEmbedNorm: block 0 stores the embedded row
  // epilogue
  int out_mode = kOutPlain;
  __half* out[3] = {nullptr, nullptr, nullptr};
  const __half* res = nullptr;        // kOutResidual
  uint32_t* token_out = nullptr;      // kOutArgmax: token_out[token_pos ? *token_pos + 1 : 0]
  float* argmax_partial = nullptr;    // kOutArgmax: [grid] values
  uint32_t* argmax_index = nullptr;   // kOutArgmax: [grid] indices
  uint32_t* counter = nullptr;        // kOutArgmax: zero before, zero after
  uint32_t* step_counter = nullptr;   // kOutArgmax: optional +1 of a decode state
  uint32_t* best_out = nullptr;       // kOutArgmax: optional {key, index + index_base}
  uint32_t index_base = 0;            // kOutArgmax: global index of row 0 (vocab shard)
  float* outf = nullptr;              // kOutF32
  uint32_t* hist = nullptr;           // kOutArgmax: optional +1 per finite logit at its order key
};
// True when the fast kernel accepts the problem (K % 8 == 0, 16-byte
// aligned pointers, K <= 16384); otherwise gemv() uses the generic kernel.
bool gemv_fast_ok(const GemvProblem& p);
void gemv(const Launch& l, const GemvProblem& p);
// ---- sampling (sample_token_f16, qwen3.rs:927-1005) -----------------------
// Order key of a finite FP16 logit: total_cmp order as an unsigned 16-bit key.
constexpr int kSampleBins = 65536;
constexpr int kSampleBlocks = kSampleBins / 64;
// Histogram words: kSampleBins counts per order key, then kSampleBlocks
// counts per block of 64 keys.
constexpr int kSampleHistWords = kSampleBins + kSampleBlocks;
struct SampleProblem {
  const __half* logits = nullptr;
  uint32_t n = 0;
  uint32_t* hist = nullptr;     // [kSampleHistWords], zero before; cleared by sample()
  uint32_t* groups = nullptr;   // scratch [2 * kSampleBins]: {key, count} per group
  // device words: {bits of 1 / temperature (FP32, correctly rounded), bits of
  // top_p, top_k (0: all)}; read at run time, so a captured graph serves any
  const uint32_t* opts = nullptr;
  uint64_t* state = nullptr;    // XorShift64 state, advanced once per token drawn
  // token_out[token_pos ? *token_pos : 0] = token, 0xFFFFFFFF when no logit is
  // finite, 0xFFFFFFFE when the walk ends without a token
  uint32_t* token_out = nullptr;
  const uint32_t* token_pos = nullptr;
};
// hist[key(logit)] += 1 for every finite logit (hist zero before).
void logit_histogram(const Launch& l, const __half* logits, uint32_t n, uint32_t* hist);
// One CTA: draws one token from the histogram and the logits.
void sample(const Launch& l, const SampleProblem& p);

// Plain tiled reference kernel (MatmulBackend::Reference), any shape, M rows.
void matmul_reference(const Launch& l, const __half* x, const __half* w, __half* out, int m,
                      int n, int k);
// Prefill GEMM (M > 1): out[m, n] = x[m, :] . w[n, :], FP32 accumulate.
void gemm(const Launch& l, const __half* x, const __half* w, __half* out, int m, int n, int k,
          int ldo);
// The same over `count` weight matrices that share x (Q / K / V, gate / up):
// out[i][m, n] = x[m, :] . w[i][n, :], one launch for the canonical path.
void gemm_multi(const Launch& l, const __half* x, int m, int k, int count,
                const __half* const* w, __half* const* out, const int* n);
// Tensor-parallel partial product: out[m, n] = DOT(x[m], w[n]) in FP32 with
// the canonical reduction (any m), unrounded.
void gemm_partial_f32(const Launch& l, const __half* x, const __half* w, float* out, int m, int n,
                      int k);
// Expired-wait code of the tensor-core GEMM (0 = none); optionally cleared.
unsigned gemm_tc_status(bool reset);
bool gemm_tc_available();
// A 2-D TMA tensor map (128 bytes, written to `map`) over one layer's K or V
// cache [capacity, kv_heads, 128] FP16 whose box is 64 consecutive values
// (half of one KV head's row) of `box_rows` consecutive positions, 128-byte
// swizzled (rows past the capacity read as zeros). False when the driver's
// encoder is unavailable.
bool make_kv_tile_map(void* map, const __half* cache, int capacity, int kv_heads, int box_rows);

// ---- row / elementwise kernels ---------------------------------------------
void add(const Launch& l, const __half* a, const __half* b, __half* out, size_t n);
void rms_norm(const Launch& l, const __half* x, const __half* w, __half* out, int rows,
              int width, float eps);
void add_rms_norm(const Launch& l, const __half* left, const __half* right, const __half* w,
                  __half* residual, __half* normalized, int rows, int width, float eps);
void swiglu(const Launch& l, const __half* gate, const __half* up, __half* out, size_t n);
void embedding(const Launch& l, const uint32_t* tokens, const __half* table, __half* out,
               int count, int width, uint32_t rows);
void rope(const Launch& l, const __half* in, __half* out, int tokens, int heads, int head_dim,
          Pos pos, float theta);
// round_norm: round the normalized row to FP16 before RoPE (unfused path).
// `rope` (optional) is a rope_table of the same theta and head_dim.
void qk_norm_rope_cache(const Launch& l, const __half* q, const __half* k, const __half* qw,
                        const __half* kw, __half* q_out, __half* key_cache, int tokens,
                        int q_heads, int kv_heads, int head_dim, Pos pos, float theta,
                        float eps, bool round_norm, const float2* rope = nullptr);
void copy_kv(const Launch& l, const __half* src, __half* cache, int tokens, int stride, Pos pos);
// Greedy argmax; partials sized by argmax_partials(n).
int argmax_partials(size_t n);
void argmax(const Launch& l, const __half* logits, size_t n, float* pv, uint32_t* pi,
            uint32_t* out);

// ---- attention ----------------------------------------------------------------
struct AttnProblem {
  const __half* q = nullptr;  // [tokens, qh, hd]
  const __half* k = nullptr;  // [kv_len, kvh, hd]
  const __half* v = nullptr;
  __half* out = nullptr;      // [tokens, qh, hd]
  int tokens = 1, qh = 1, kvh = 1, hd = 128;
  int kv_len = 0;             // used when kv_len_dev is null
  const uint32_t* kv_len_dev = nullptr;  // decode graphs: *kv_len_dev + kv_len_add
  int kv_len_add = 0;
  int causal = 1;
  int query_offset = 0;       // ignored for decode-from-device (offset = len - 1)
  int round_p = 1;            // prefill: round probabilities to FP16 (FlashPrefill)
};
// Two-pass reference semantics (attention_reference_f16), any head_dim.
void attention_reference(const Launch& l, const AttnProblem& p);
// Single-query split-K decode attention for any GQA ratio; partial states in
// `scratch` (attention_decode_scratch bytes) and per-kv-head counters that
// must be zero on entry (they are zero again on exit).
size_t attention_decode_scratch(int kvh, int splits, int group, int hd);
int attention_decode_splits(int kv_len_max, int kvh, int sm_count, int block_keys);
void attention_decode(const Launch& l, const AttnProblem& p, int splits, int block_keys,
                      float* scratch, uint32_t* counters);
// Fused decode front end + attention for the model: per-head RMSNorm + RoPE
// of the query and the new key, K/V append at position len-1, split-K
// attention over the cache.
struct DecodeFused {
  const __half* q_raw = nullptr;  // [qh, hd]
  const __half* k_raw = nullptr;  // [kvh, hd]
  const __half* v_raw = nullptr;  // [kvh, hd]
  const __half* q_norm = nullptr;
  const __half* k_norm = nullptr;
  float theta = 1e6f, eps = 1e-6f;
  bool round_norm = false;
  __half* key_cache = nullptr;    // [cap, kvh, hd]
  __half* value_cache = nullptr;
  __half* out = nullptr;          // [qh, hd]
  int qh = 16, kvh = 8, hd = 128;
  Pos pos;                        // position of the new token (= len - 1)
  const float2* rope = nullptr;   // RoPE table [cap, hd / 2] of (cos, sin), or null
};
// RoPE table of (cos, sin) for positions [0, positions) and pairs [0, hd/2),
// entry p * (hd / 2) + i; the values are those of rope_cs (numerics.cuh).
void rope_table(cudaStream_t s, float2* out, int positions, int head_dim, float theta);
void attention_decode_fused(const Launch& l, const DecodeFused& p, int splits, float* scratch,
                            uint32_t* counters, int block_keys);
// Keys per flash-decode block for a cache of `capacity` positions (64 up to
// 8192 positions, then doubled until at most 128 blocks).
int decode_block_for(int capacity);
// Expired-wait codes of the staged kernels (0 = none), optionally cleared.
unsigned gemv_status(bool reset);
unsigned attention_status(bool reset);
// Prefill attention in 32-key blocks, any GQA ratio, head_dim <= 256: with
// round_p the flash-prefill semantics (FP16 probabilities), without it the
// FP32 online softmax of the tiled kernel.
void attention_prefill(const Launch& l, const AttnProblem& p);
// Prompts of at least this many tokens (head_dim 128, FP16 probabilities)
// take the tensor-core prefill attention (attention_mma.cu): per-op
// tolerance instead of the canonical kernel's bit-exact arithmetic.
constexpr int kMmaPrefillMinTokens = 512;
// The tensor-core prefill attention; false when the problem does not fit it.
bool attention_prefill_mma(const Launch& l, const AttnProblem& p);

// ---- tensor parallelism -----------------------------------------------------------
// out[i] = half(parts[0][i] + parts[1][i] + ... + parts[tp-1][i]), summed in
// rank order in FP32 (parts: [tp, n] as gathered from the ranks).
void rank_sum_round(cudaStream_t s, const float* parts, int tp, size_t n, __half* out);
// Slice `rank` ([n]) of that sum from the other ranks' slices (`pieces`,
// [tp, n], row q from rank q) and this rank's own slice `mine`.
void rank_sum_round_slice(cudaStream_t s, const float* pieces, const float* mine, int rank, int tp,
                          size_t n, __half* out);
// Greedy id over the ranks' {key, index} pairs ([tp, 2]): writes it to
// token_out[*token_pos + 1] (or token_out[0] without token_pos) and adds one
// to *step_counter when given.
void argmax_combine(cudaStream_t s, const uint32_t* pairs, int tp, uint32_t* token_out,
                    const uint32_t* token_pos, uint32_t* step_counter);

// ---- persistent decode loop -------------------------------------------------------
// Per-layer weights and cache of the persistent decode kernel (device array).
struct LoopLayer {
  const __half* wq;
  const __half* wk;
  const __half* wv;
  const __half* wo;
  const __half* q_norm;
  const __half* k_norm;
  const __half* gate;
  const __half* up;
  const __half* down;
  const __half* in_norm;
  const __half* post_norm;
  __half* k_cache;  // [capacity, kvh, 128]
  __half* v_cache;
};
// `steps` greedy decode steps of the whole model in one cooperative launch:
// reads toks[*dev_len], writes each step's id to toks[pos + 1] and the last
// step's logits, advances *dev_len by `steps`. The stage arithmetic is that
// of the per-kernel decode chain (bit-identical results).
struct DecodeLoop {
  int hidden = 0, inter = 0, qh = 0, kvh = 0, vocab = 0, layers = 0;
  float eps = 1e-6f, theta = 1e6f;
  int round_norm = 0;  // FusionOptions::qk_rope_cache off: round the normed q/k
  int add_norm = 1;    // FusionOptions::add_rms_norm: sum of squares of the unrounded sum
  int block = 64;      // flash-decode keys per block
  int attn_blocks = 0; // blocks per head the partial buffer holds
  int steps = 0;
  const LoopLayer* layer = nullptr;
  // [layers][2] CUtensorMap (K, V) of the cache, 64-byte aligned: boxes of
  // 64 values x 64 positions (128-byte swizzle) for the attention tiles
  const void* kv_maps = nullptr;
  const __half* embedding = nullptr;
  const __half* final_norm = nullptr;
  const __half* lm_head = nullptr;
  const float2* rope = nullptr;
  uint32_t* toks = nullptr;
  uint32_t* dev_len = nullptr;
  // Activations that cross CTAs, one u32 per FP16 value: (16-bit epoch tag
  // << 16) | bits, so readers validate every word (no grid barriers).
  uint32_t epoch0 = 1;               // tag base: layer-steps run on these buffers + 1
  uint32_t* t_hidden = nullptr;      // [hidden] residual stream
  uint32_t* t_res = nullptr;         // [hidden] after the attention add
  uint32_t* t_qkv = nullptr;         // [qh * 128 + 2 * kvh * 128]
  uint32_t* t_attn_o = nullptr;      // [hidden]
  uint32_t* t_act = nullptr;         // [inter]
  unsigned long long* t_argmax = nullptr;  // [grid]: key << 32 | index << 14 | 14-bit tag
  __half* logits = nullptr;
  float* attn_part = nullptr;     // [kvh, attn_blocks, G, 132] block partials
  uint32_t* sync = nullptr;       // [decode_loop_sync_words()]: abort flag, attention-unit counter
  // Tensor parallelism (tp > 1): the shapes above are this rank's shard.
  // The row-parallel O and down products leave the kernel as FP32 partials
  // stored straight into every rank's mailbox over NVLink (u64 words: 32-bit
  // epoch tag << 32 | float bits); readers poll their own mailbox until every
  // word carries the tag it wants and sum the ranks' partials in rank order.
  int tp = 1, rank = 0;
  uint32_t vocab0 = 0;                        // global id of this rank's first LM-head row
  uint32_t vocab_full = 0;                    // rows of the (replicated) embedding
  unsigned long long* const* peers = nullptr; // [tp] device pointers to each rank's mailbox
  unsigned long long* mbox = nullptr;         // this rank's mailbox (peers[rank])
  // plan (decode_loop_plan)
  int slot_bytes = 0, slots = 0, x_bytes = 0, grid = 0;
  int xslice = 1;  // tensor parallelism: each CTA sums a slice of the partials (else all)
  int l2_ahead = 0; // the producer's L2 prefetches run this many weight tiles ahead of its copies
};
// Mailbox layout in u64 words for `tp` ranks, hidden size h and grid CTAs:
// [tp][h] O partials, [tp][h] down partials, [tp][grid] argmax records.
struct MailboxLayout {
  size_t o, d, rec, words;
};
__host__ __device__ inline MailboxLayout mailbox_layout(int tp, int h, int grid) {
  MailboxLayout m;
  m.o = 0;
  m.d = (size_t)tp * h;
  m.rec = m.d + (size_t)tp * h;
  m.words = m.rec + (size_t)tp * grid;
  return m;
}
// Fills the plan fields for `device`; false when the model shape or the
// device's shared memory does not admit the persistent kernel.
bool decode_loop_plan(DecodeLoop& p, int device);
void decode_loop(cudaStream_t stream, const DecodeLoop& p);
// Floats of DecodeLoop::attn_part for kvh KV heads, `blocks` key blocks and
// `group` query heads per KV head.
inline size_t decode_loop_part_floats(int kvh, int blocks, int group) {
  return (size_t)kvh * blocks * group * (128 + 4);
}
// u32 words of DecodeLoop::sync: 256 control words, then one word per CTA
// (at most 256 CTAs) with the time its mailbox waits took in the launch
// (tensor parallelism only), in units of 64 ns.
constexpr size_t decode_loop_sync_words() { return 512; }
constexpr size_t decode_loop_wait_word0() { return 256; }
// Expired-wait code of the persistent kernel (0 = none), optionally cleared.
unsigned decode_loop_status(bool reset);

// ---- synthetic data ------------------------------------------------------------
void fill_normal_f16(cudaStream_t s, __half* out, size_t n, uint64_t seed, uint64_t stream,
                     uint64_t offset, double std_dev);
// Fills a [rows, cols] block of a larger [*, full_cols] matrix whose element
// (r, c) is generator index (row0 + r) * full_cols + col0 + c.
void fill_normal_f16_block(cudaStream_t s, __half* out, size_t rows, size_t cols,
                           size_t full_cols, size_t row0, size_t col0, uint64_t seed,
                           uint64_t stream, double std_dev);
void fill_tokens(cudaStream_t s, uint32_t* out, size_t n, uint64_t seed, uint64_t stream,
                 uint32_t vocab);
void fill_f16(cudaStream_t s, __half* out, size_t n, uint16_t bits);

}  // namespace k
}  // namespace mi
