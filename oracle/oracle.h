/*
 * CPU oracle for the Qwen3 hot path of stratorys/metal-infer-rs.
 *
 * TEST INFRASTRUCTURE ONLY. This library restates, on the host, the arithmetic
 * of the reference's Metal kernels
 * (crates/metal-infer-core/src/kernels/transformer.metal) and the model
 * orchestration of crates/metal-infer-models/src/qwen3.rs. It exists to check
 * the CUDA engine and to serve as the timed CPU baseline. Nothing in the
 * engine links it, and only tests/, __graft_entry__.smoke() and bench.py's CPU
 * legs load it.
 *
 * Parity pinning: the reference has no CPU path and no stored outputs. The
 * oracle is pinned against the known-answer vectors and CPU formulas written
 * inline in crates/metal-infer-core/tests/gpu.rs (see tests/test_oracle.py).
 * Beyond those formulas, model-level outputs are "parity unpinned": they are
 * the oracle's own, committed as golden fixtures under tests/golden/.
 *
 * Conventions: all FP16 buffers are IEEE binary16 bit patterns (uint16_t),
 * row-major; weights are [out, in] and products are x * W^T.
 */
#ifndef MI_ORACLE_H
#define MI_ORACLE_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* ---- numerics helpers ------------------------------------------------- */
void or_f16_from_f32(const float* in, uint16_t* out, size_t n);
void or_f32_from_f16(const uint16_t* in, float* out, size_t n);
/* Accumulate dot products in double instead of FP32 (sensitivity studies). */
void or_set_accumulate_f64(int enabled);
int or_num_threads(void);

/* ---- seeded synthetic inputs (SplitMix64 + Box-Muller) ---------------- */
/* Element i of stream `stream` under `seed`, for i in [offset, offset+n). */
void or_gen_normal_f16(uint64_t seed, uint64_t stream, uint64_t offset, size_t n,
                       double std_dev, uint16_t* out);
void or_gen_tokens(uint64_t seed, uint64_t stream, size_t n, uint32_t vocab,
                   uint32_t* out);

/* ---- single ops (one entry per reference kernel family) --------------- */
/* out[m,n] = half(sum_k x[m,k] w[n,k]); transformer.metal:70-94, 274-347 */
void or_matmul(const uint16_t* x, size_t m, size_t k, const uint16_t* w,
               size_t n, uint16_t* out);
/* out = a + b in half arithmetic; transformer.metal:61-68 */
void or_add(const uint16_t* a, const uint16_t* b, size_t n, uint16_t* out);
/* transformer.metal:1318-1340 */
void or_rms_norm(const uint16_t* x, size_t rows, size_t width,
                 const uint16_t* w, float eps, uint16_t* out);
/* transformer.metal:1342-1369 */
void or_add_rms_norm(const uint16_t* left, const uint16_t* right, size_t rows,
                     size_t width, const uint16_t* w, float eps,
                     uint16_t* residual, uint16_t* normalized);
/* transformer.metal:937-1009 (one row) */
void or_rms_norm_matmul3(const uint16_t* x, size_t k, const uint16_t* norm_w,
                         const uint16_t* w0, size_t n0, const uint16_t* w1,
                         size_t n1, const uint16_t* w2, size_t n2, float eps,
                         uint16_t* out0, uint16_t* out1, uint16_t* out2);
/* transformer.metal:1091-1160 (one row) */
void or_add_rms_norm_matmul2(const uint16_t* left, const uint16_t* right,
                             size_t k, const uint16_t* norm_w,
                             const uint16_t* w0, size_t n0, const uint16_t* w1,
                             size_t n1, float eps, uint16_t* residual,
                             uint16_t* out0, uint16_t* out1);
/* transformer.metal:1371-1380 */
void or_swiglu(const uint16_t* gate, const uint16_t* up, size_t n,
               uint16_t* out);
/* transformer.metal:1382-1394; token 0xFFFFFFFF embeds as zeros */
void or_embedding(const uint32_t* tokens, size_t count, const uint16_t* table,
                  size_t rows, size_t width, uint16_t* out);
/* transformer.metal:1396-1512; returns 0xFFFFFFFF when nothing is finite */
uint32_t or_argmax(const uint16_t* logits, size_t n);
/* sample_token / sample_token_f16 + sample_candidates (qwen3.rs:909-1005)
 * with the XorShift64 stream of qwen3.rs:1011-1034 (`state` in/out, already
 * seeded: see or_xorshift_seed). Temperature 0 is the argmax of sample_token.
 * Candidates are ordered by descending total_cmp value; equal bit patterns
 * in ascending index (slice::sort_unstable_by leaves their order open); the
 * exponential is the engine's exp. Returns the token, 0xFFFFFFFF when no
 * logit is finite, 0xFFFFFFFE when the walk ends without a token ("failed to
 * sample a token"). */
uint32_t or_sample_f16(const uint16_t* logits, size_t n, float temperature,
                       float top_p, size_t top_k, uint64_t* state);
/* XorShift64::new (qwen3.rs:1016-1024): seed 0 becomes 0x9e3779b97f4a7c15. */
uint64_t or_xorshift_seed(uint64_t seed);
/* transformer.metal:1514-1531 */
void or_rope(const uint16_t* in, size_t tokens, size_t heads, size_t head_dim,
             size_t offset, float theta, uint16_t* out);
/* transformer.metal:1533-1577; writes K rows into key_cache[offset + t] */
void or_qk_norm_rope_cache(const uint16_t* q, const uint16_t* k, size_t tokens,
                           size_t q_heads, size_t kv_heads, size_t head_dim,
                           const uint16_t* q_w, const uint16_t* k_w,
                           size_t offset, float theta, float eps,
                           size_t cache_capacity, uint16_t* q_out,
                           uint16_t* key_cache);
/* transformer.metal:2318-2325 */
void or_copy_into_cache(const uint16_t* src, size_t tokens, size_t stride,
                        size_t offset, uint16_t* cache);

/* Attention semantics. OR_ATTN_REFERENCE is the two-pass FP32 softmax of
 * attention_reference_f16 (transformer.metal:1579-1612). OR_ATTN_TILED and
 * OR_ATTN_FLASH_PREFILL process keys in 32-key blocks with an online softmax
 * (transformer.metal:1614-1822); flash prefill rounds the probabilities to
 * FP16 before they weight V. */
enum { OR_ATTN_REFERENCE = 0, OR_ATTN_FLASH_PREFILL = 1, OR_ATTN_TILED = 2 };
void or_attention(const uint16_t* q, const uint16_t* k, const uint16_t* v,
                  size_t tokens, size_t q_heads, size_t kv_heads,
                  size_t head_dim, size_t kv_length, int causal,
                  size_t query_offset, int semantics, uint16_t* out);
/* One-query flash decode (transformer.metal:2127-2316) over `length` keys:
 * blocks of `block` keys, `streams` interleaved online-softmax streams per
 * block, log-sum-exp merges in index order. */
void or_attention_decode(const uint16_t* q, const uint16_t* k, const uint16_t* v,
                         size_t q_heads, size_t kv_heads, size_t head_dim,
                         size_t length, size_t block, size_t streams,
                         uint16_t* out);
/* Decode block size used for a cache of `capacity` positions, and the
 * stream count for a head dimension. */
size_t or_decode_block(size_t capacity);
size_t or_decode_streams(size_t head_dim);

/* ---- numerics primitives (for direct checks) ---------------------------- */
void or_exp(const float* in, float* out, size_t n);
float or_dot(const float* x, const float* y, size_t n);
void or_rope_cs(size_t position, size_t pair, size_t head_dim, float theta,
                float* c, float* s);

/* ---- Qwen3 model (qwen3.rs:602-796) ----------------------------------- */
typedef struct or_qwen3_config {
  uint32_t hidden_size;
  uint32_t intermediate_size;
  uint32_t num_hidden_layers;
  uint32_t num_attention_heads;
  uint32_t num_key_value_heads;
  uint32_t head_dim;
  float rms_norm_eps;
  float rope_theta;
  uint32_t vocab_size;
  uint32_t tie_word_embeddings;
} or_qwen3_config;

typedef struct or_qwen3 or_qwen3;

/* Random-init weights: matrices N(0, std) from (seed, stream); norms 1.0.
 * Stream numbering is documented in oracle.cpp (weight_stream). */
or_qwen3* or_qwen3_create_random(const or_qwen3_config* cfg, uint64_t seed,
                                 double std_dev, size_t cache_capacity);
void or_qwen3_destroy(or_qwen3* m);
/* FusionOptions flags that change rounding (qwen3.rs:42-66). */
void or_qwen3_set_fusion(or_qwen3* m, int qk_rope_cache, int add_rms_norm);
/* Tensor-parallel arithmetic of the engine's TP path (no counterpart in the
 * reference, which runs on one GPU): the O and down products become the sum,
 * in rank order, of each rank's canonical DOT over its 1/tp slice of the
 * input columns, rounded once to FP16. Everything else is unchanged. */
void or_qwen3_set_tp(or_qwen3* m, size_t tp);
void or_qwen3_reset(or_qwen3* m);
/* Keeps the first len cached positions (len <= the current length), as the
 * reference's generate_greedy rolls its cache back; -1 otherwise. */
int or_qwen3_truncate(or_qwen3* m, size_t len);
size_t or_qwen3_len(const or_qwen3* m);
/* Embeds tokens and runs the model; logits of the last row (half[vocab]).
 * Returns 0 on success, -1 on cache overflow. */
int or_qwen3_forward(or_qwen3* m, const uint32_t* tokens, size_t count,
                     uint16_t* logits);
/* Runs every layer on given hidden states [count, hidden] (no embedding, no
 * head) and returns the final hidden states; used for the one-block config. */
int or_qwen3_forward_hidden(or_qwen3* m, const uint16_t* hidden, size_t count,
                            uint16_t* out_hidden);
/* Greedy generation as generate_greedy (qwen3.rs:475-555) without stop
 * tokens: prefill, then max_tokens-1 decode steps. Returns count written. */
size_t or_qwen3_generate_greedy(or_qwen3* m, const uint32_t* prompt,
                                size_t prompt_len, size_t max_tokens,
                                uint32_t* out_ids);
/* Sampled generation as generate_with with temperature > 0 (qwen3.rs:441-473)
 * without stop tokens: token 0 from the prefill logits, each later token from
 * the logits of decoding the previous one, one XorShift64 stream seeded by
 * `seed`. Stops early (returning the count) on a sampling failure. */
size_t or_qwen3_generate_sampled(or_qwen3* m, const uint32_t* prompt,
                                 size_t prompt_len, size_t max_tokens,
                                 float temperature, float top_p, size_t top_k,
                                 uint64_t seed, uint32_t* out_ids);
/* Access to one weight tensor by stream role (for op-level checks). */
const uint16_t* or_qwen3_weight(const or_qwen3* m, int layer, int role);
const uint16_t* or_qwen3_cache(const or_qwen3* m, int layer, int value);

#ifdef __cplusplus
}
#endif
#endif
