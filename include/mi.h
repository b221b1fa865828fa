/*
 * mi.h - C ABI of the B200 (sm_100a) Qwen3 engine.
 *
 * This is the drop-in boundary for the hot path of stratorys/metal-infer-rs.
 * Each declaration names the reference item it replaces (file:line relative
 * to the reference repository). The Rust crates keep their API by binding
 * these symbols; the Metal runtime (objc2-metal device,
 * buffers, command encoders) becomes a CUDA stream, stream-ordered device
 * memory and CUDA graphs behind these calls.
 *
 * Conventions
 *  - Every function returns mi_status; MI_OK is 0. On failure,
 *    mi_last_error_message() gives a thread-local description. No C++
 *    exception crosses this boundary.
 *  - Handles are opaque. Tensors are reference-counted views of device
 *    buffers (tensor.rs:35-42): views share the buffer; each handle is
 *    released with mi_tensor_release.
 *  - A context owns one CUDA stream and is not thread-safe, like MetalContext
 *    (context.rs:192-213). Work encoded into a batch starts as it is
 *    encoded; commit records completion and wait blocks on it.
 *  - FP16 is IEEE binary16; weights are [out, in] and products are x * W^T.
 */
#ifndef MI_H
#define MI_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* ---- status and types --------------------------------------------------- */

/* CoreError (crates/metal-infer-core/src/error.rs:6-32) and ModelError
 * (crates/metal-infer-models/src/error.rs:4-29) as status codes. */
typedef enum mi_status {
  MI_OK = 0,
  MI_ERR_NO_DEVICE = 1,       /* CoreError::NoDevice */
  MI_ERR_RESOURCE = 2,        /* CoreError::Resource (allocation, stream) */
  MI_ERR_KERNEL = 3,          /* CoreError::Shader/Pipeline/MissingKernel */
  MI_ERR_COMMAND = 4,         /* CoreError::Command/UnknownCommand */
  MI_ERR_SHAPE = 5,           /* CoreError::Shape */
  MI_ERR_DTYPE = 6,           /* CoreError::DType */
  MI_ERR_DATA_LENGTH = 7,     /* CoreError::DataLength */
  MI_ERR_PROFILING = 8,       /* CoreError::Profiling */
  MI_ERR_CACHE_CAPACITY = 9,  /* ModelError::CacheCapacity */
  MI_ERR_CONFIG = 10,         /* ModelError::Config */
  MI_ERR_UNSUPPORTED = 11,    /* ModelError::Unsupported */
  MI_ERR_IO = 12,             /* ModelError::Io / Json / Safetensors */
  MI_ERR_MISSING_TENSOR = 13, /* ModelError::MissingTensor */
  MI_ERR_TIMEOUT = 14,        /* a bounded device wait gave up */
  MI_ERR_INVALID_ARGUMENT = 15,
  MI_ERR_COLLECTIVE = 16      /* NCCL or peer-exchange failure */
} mi_status;

/* DType (tensor.rs:12-32) */
typedef enum mi_dtype { MI_F16 = 0, MI_F32 = 1, MI_U32 = 2 } mi_dtype;

/* MatmulBackend (context.rs:117-153). MI_MATMUL_MPS has no CUDA
 * counterpart and is rejected with MI_ERR_UNSUPPORTED. */
typedef enum mi_matmul_backend {
  MI_MATMUL_AUTO = 0,
  MI_MATMUL_REFERENCE = 1, /* ReferenceMsl: plain tiled kernel */
  MI_MATMUL_NATIVE = 2,    /* NativeMsl: the tuned kernels */
  MI_MATMUL_MPS = 3
} mi_matmul_backend;

/* AttentionKind (ops.rs:13-19) */
typedef enum mi_attention_kind {
  MI_ATTENTION_REFERENCE = 0,
  MI_ATTENTION_TILED = 1,
  MI_ATTENTION_FLASH_PREFILL = 2,
  MI_ATTENTION_DECODE_SPLIT_KV = 3,
  MI_ATTENTION_FLASH_DECODE = 4
} mi_attention_kind;

/* AttentionConfig (ops.rs:30-36) */
typedef struct mi_attention_config {
  size_t query_heads;
  size_t kv_heads;
  size_t head_dim;
  int causal;
  size_t query_offset;
} mi_attention_config;

/* QkNormRopeCacheConfig (ops.rs:39-43) */
typedef struct mi_qk_config {
  size_t offset;
  float theta;
  float epsilon;
} mi_qk_config;

/* DispatchStats (context.rs:32-36), in seconds. */
typedef struct mi_dispatch_stats {
  double gpu_time;
  double wall_time;
} mi_dispatch_stats;

/* KernelDispatchProfile (context.rs:38-42). */
typedef struct mi_kernel_profile {
  char kernel[64];
  double gpu_time;
} mi_kernel_profile;

typedef struct mi_context mi_context;
typedef struct mi_tensor mi_tensor;
typedef struct mi_batch mi_batch;
typedef struct mi_pending mi_pending;

/* Thread-local message of the last failure (empty after success). */
const char* mi_last_error_message(void);
/* Library version string. */
const char* mi_version(void);

/* ---- context (MetalContext, context.rs:216-872) --------------------------- */

/* MetalContext::new (context.rs:216-248); `device` is the CUDA ordinal. */
mi_status mi_context_create(int device, mi_context** out);
void mi_context_destroy(mi_context* ctx);
/* MetalContext::device_name (context.rs:250-252) */
mi_status mi_context_device_name(const mi_context* ctx, char* buf, size_t len);
/* MetalContext::allocated_bytes (context.rs:340-342) */
size_t mi_context_allocated_bytes(const mi_context* ctx);
/* MetalContext::set_matmul_backend / matmul_backend (context.rs:344-353) */
mi_status mi_context_set_matmul_backend(mi_context* ctx, mi_matmul_backend b);
mi_matmul_backend mi_context_matmul_backend(const mi_context* ctx);
/* MetalContext::set_kernel_profiling / take_kernel_profiles
 * (context.rs:604-701). Profiles are CUDA-event timings per launch. */
mi_status mi_context_set_kernel_profiling(mi_context* ctx, int enabled);
mi_status mi_context_take_kernel_profiles(mi_context* ctx, mi_kernel_profile* out,
                                          size_t capacity, size_t* count);
/* Blocks until all work of the context's stream is done. */
mi_status mi_context_synchronize(mi_context* ctx);
/* Synchronizes, then reports (and clears) the code of a bounded device wait
 * that expired since the last call: 0 = none; otherwise MI_ERR_TIMEOUT is
 * returned and *code names the wait (tensor-core GEMM pipeline: 1 producer,
 * 2 MMA issuer, 3 epilogue, 4 drain). No reference counterpart: Metal
 * command-buffer errors (context.rs:1058-1063) have no device-side waits. */
mi_status mi_context_kernel_status(mi_context* ctx, uint32_t* code);
/* The context's CUDA stream (cudaStream_t) for interop. */
void* mi_context_stream(mi_context* ctx);

/* ---- tensors (context.rs:740-872, tensor.rs:35-261) ----------------------- */

/* MetalContext::empty (context.rs:740-754); contents are zeroed. */
mi_status mi_context_empty(mi_context* ctx, const size_t* shape, size_t rank,
                           mi_dtype dtype, mi_tensor** out);
/* MetalContext::tensor_f16 (context.rs:756-774): FP32 values rounded to FP16. */
mi_status mi_context_tensor_f16(mi_context* ctx, const float* values, size_t count,
                                const size_t* shape, size_t rank, mi_tensor** out);
/* MetalContext::tensor_f16_bits (context.rs:776-793) */
mi_status mi_context_tensor_f16_bits(mi_context* ctx, const uint16_t* bits, size_t count,
                                     const size_t* shape, size_t rank, mi_tensor** out);
/* MetalContext::tensor_f16_bytes (context.rs:795-820): little-endian FP16. */
mi_status mi_context_tensor_f16_bytes(mi_context* ctx, const uint8_t* bytes, size_t nbytes,
                                      const size_t* shape, size_t rank, mi_tensor** out);
/* MetalContext::tensor_bf16_as_f16_bytes (context.rs:822-853) */
mi_status mi_context_tensor_bf16_as_f16_bytes(mi_context* ctx, const uint8_t* bytes,
                                              size_t nbytes, const size_t* shape, size_t rank,
                                              mi_tensor** out);
/* MetalContext::tensor_u32 (context.rs:855-872) */
mi_status mi_context_tensor_u32(mi_context* ctx, const uint32_t* values, size_t count,
                                const size_t* shape, size_t rank, mi_tensor** out);
/* A view of caller-owned device memory (not freed by the engine). */
mi_status mi_context_tensor_from_device(mi_context* ctx, void* device_ptr, const size_t* shape,
                                        size_t rank, mi_dtype dtype, mi_tensor** out);

/* Tensor::clone (shares the buffer) and drop. */
mi_status mi_tensor_clone(const mi_tensor* t, mi_tensor** out);
void mi_tensor_release(mi_tensor* t);
/* Tensor::shape / dtype / len / byte_len (tensor.rs:89-107) */
size_t mi_tensor_rank(const mi_tensor* t);
size_t mi_tensor_shape(const mi_tensor* t, size_t* shape, size_t capacity);
mi_dtype mi_tensor_dtype(const mi_tensor* t);
size_t mi_tensor_len(const mi_tensor* t);
size_t mi_tensor_byte_len(const mi_tensor* t);
void* mi_tensor_device_ptr(const mi_tensor* t);
/* Tensor::reshape / prefix / row / slice_1d (tensor.rs:108-207) */
mi_status mi_tensor_reshape(const mi_tensor* t, const size_t* shape, size_t rank,
                            mi_tensor** out);
mi_status mi_tensor_prefix(const mi_tensor* t, size_t first_dimension, mi_tensor** out);
mi_status mi_tensor_row(const mi_tensor* t, size_t row, mi_tensor** out);
mi_status mi_tensor_slice_1d(const mi_tensor* t, size_t start, size_t len, mi_tensor** out);
/* Tensor::with_f16_bits / to_f32_vec / to_u32_vec (tensor.rs:209-260).
 * They synchronize the context stream first; `count` must equal len. */
mi_status mi_tensor_f16_bits(const mi_tensor* t, uint16_t* out, size_t count);
mi_status mi_tensor_to_f32(const mi_tensor* t, float* out, size_t count);
mi_status mi_tensor_to_u32(const mi_tensor* t, uint32_t* out, size_t count);
/* Overwrite a tensor's contents from host memory (bytes must match). */
mi_status mi_tensor_write(mi_tensor* t, const void* host, size_t nbytes);

/* ---- batches (CommandBatch / PendingBatch, context.rs:703-738, 1032-1082) - */

mi_status mi_context_begin_batch(mi_context* ctx, mi_batch** out);
/* CommandBatch::commit: consumes the batch. */
mi_status mi_batch_commit(mi_batch* b, mi_pending** out);
/* CommandBatch::finish: commit + wait; consumes the batch. */
mi_status mi_batch_finish(mi_batch* b, mi_dispatch_stats* stats);
/* Dropping an uncommitted batch. */
void mi_batch_abandon(mi_batch* b);
/* PendingBatch::wait: consumes the pending handle; stats may be NULL.
 * Returns MI_ERR_TIMEOUT when a kernel's bounded device wait expired (its
 * outputs are not valid), as mi_context_kernel_status reports it. */
mi_status mi_pending_wait(mi_pending* p, mi_dispatch_stats* stats);
/* Non-consuming completion query: 1 done, 0 running. */
int mi_pending_is_complete(const mi_pending* p);

/* ---- ops (CommandBatch methods, ops.rs:221-1285) -------------------------- */
/* Outputs are new tensors owned by the caller (release them); their memory
 * is stream-ordered, so releasing before completion is safe. */

/* ops.rs:222-240 */
mi_status mi_batch_add(mi_batch* b, const mi_tensor* left, const mi_tensor* right,
                       mi_tensor** out);
/* ops.rs:242-373 */
mi_status mi_batch_matmul(mi_batch* b, const mi_tensor* input, const mi_tensor* weight,
                          mi_tensor** out);
/* ops.rs:444-500 */
mi_status mi_batch_matmul2(mi_batch* b, const mi_tensor* input, const mi_tensor* w0,
                           const mi_tensor* w1, mi_tensor** out0, mi_tensor** out1);
/* ops.rs:502-566 */
mi_status mi_batch_matmul3(mi_batch* b, const mi_tensor* input, const mi_tensor* w0,
                           const mi_tensor* w1, const mi_tensor* w2, mi_tensor** out0,
                           mi_tensor** out1, mi_tensor** out2);
/* ops.rs:568-642 */
mi_status mi_batch_rms_norm_matmul3(mi_batch* b, const mi_tensor* input,
                                    const mi_tensor* norm_weight, const mi_tensor* w0,
                                    const mi_tensor* w1, const mi_tensor* w2, float epsilon,
                                    mi_tensor** out0, mi_tensor** out1, mi_tensor** out2);
/* ops.rs:644-720 */
mi_status mi_batch_add_rms_norm_matmul2(mi_batch* b, const mi_tensor* left,
                                        const mi_tensor* right, const mi_tensor* norm_weight,
                                        const mi_tensor* w0, const mi_tensor* w1, float epsilon,
                                        mi_tensor** residual, mi_tensor** out0,
                                        mi_tensor** out1);
/* ops.rs:722-755 */
mi_status mi_batch_rms_norm(mi_batch* b, const mi_tensor* input, const mi_tensor* weight,
                            float epsilon, mi_tensor** out);
/* ops.rs:757-798 */
mi_status mi_batch_add_rms_norm(mi_batch* b, const mi_tensor* left, const mi_tensor* right,
                                const mi_tensor* weight, float epsilon, mi_tensor** residual,
                                mi_tensor** normalized);
/* ops.rs:800-818 */
mi_status mi_batch_swiglu(mi_batch* b, const mi_tensor* gate, const mi_tensor* up,
                          mi_tensor** out);
/* ops.rs:820-845 */
mi_status mi_batch_embedding(mi_batch* b, const mi_tensor* tokens, const mi_tensor* table,
                             mi_tensor** out);
/* ops.rs:847-880: writes one u32 into `output` (0xFFFFFFFF if none finite). */
mi_status mi_batch_argmax(mi_batch* b, const mi_tensor* logits, mi_tensor* output);
/* ops.rs:882-915 */
mi_status mi_batch_rope(mi_batch* b, const mi_tensor* input, size_t offset, float theta,
                        mi_tensor** out);
/* ops.rs:917-977: returns the rotated query; rotated keys are written into
 * key_cache rows [offset, offset + tokens). */
mi_status mi_batch_qk_norm_rope_cache(mi_batch* b, const mi_tensor* query, const mi_tensor* key,
                                      const mi_tensor* query_weight,
                                      const mi_tensor* key_weight, mi_tensor* key_cache,
                                      mi_qk_config config, mi_tensor** out);
/* ops.rs:979-994 */
mi_status mi_batch_attention(mi_batch* b, const mi_tensor* query, const mi_tensor* key,
                             const mi_tensor* value, mi_attention_config config,
                             mi_attention_kind kind, mi_tensor** out);
/* ops.rs:996-1048: split-K flash decode with an explicit key-block size
 * (32, 64, 128 or 256) and thread count (128 or 256). */
mi_status mi_batch_attention_flash_decode_with_configuration(
    mi_batch* b, const mi_tensor* query, const mi_tensor* key, const mi_tensor* value,
    mi_attention_config config, size_t block_keys, size_t threads, mi_tensor** out);
/* ops.rs:1249-1285 */
mi_status mi_batch_copy_into_cache(mi_batch* b, const mi_tensor* source, mi_tensor* cache,
                                   size_t offset);

/* One-query flash decode that allocates nothing. No counterpart in the
 * reference: it serves callers that cannot allocate device memory at the
 * call — hosts that reserve the whole GPU for their own memory pool, and
 * latency-critical loops where cudaMalloc/cudaFree would synchronize the
 * device. Same result as mi_batch_attention_flash_decode_with_configuration
 * on [1, query_heads, 128] queries and [length, kv_heads, 128] FP16 keys and
 * values (all keys visible); the caller passes every input and the output as
 * 16-byte aligned device pointers and the cudaStream_t to run on.
 * Scratch: a fixed device array inside the library (1 MiB of FP32 block
 * partials plus 64 merge counters), held by every GPU that loads the library
 * until exit. Limits: head_dim 128, GQA ratio 1/2/4/8, block_keys 32/64/
 * 128/256, kv_heads <= 64, kv_heads * ceil(length / block_keys) * ratio *
 * 130 * 4 <= 1 MiB; larger sizes return MI_ERR_SHAPE. The first call in a
 * CUDA context looks up the array's device address in that context (make it
 * before any stream capture); `stream` must belong to the current context
 * (else MI_ERR_INVALID_ARGUMENT). Calls share the array: calls that overlap
 * on the GPU race. */
mi_status mi_attention_flash_decode_noalloc(const void* query, const void* key,
                                            const void* value, void* out, size_t query_heads,
                                            size_t kv_heads, size_t head_dim, size_t length,
                                            size_t block_keys, void* stream);

/* ---- Qwen3 model (crates/metal-infer-models/src/qwen3.rs) ----------------- */

/* Qwen3Config (crates/metal-infer-models/src/config.rs:5-21) */
typedef struct mi_qwen3_config {
  size_t hidden_size;
  size_t intermediate_size;
  size_t num_hidden_layers;
  size_t num_attention_heads;
  size_t num_key_value_heads;
  size_t head_dim;
  float rms_norm_eps;
  float rope_theta;
  size_t vocab_size;
  int tie_word_embeddings;
} mi_qwen3_config;

/* FusionOptions (qwen3.rs:42-66) */
typedef struct mi_fusion_options {
  int qkv;
  int gate_up;
  int add_rms_norm;
  int qk_rope_cache;
} mi_fusion_options;

/* GenerationOptions (qwen3.rs:132-152). Temperature 0 is greedy; a
 * temperature > 0 samples on the device (mi_sample_logits). */
typedef struct mi_generation_options {
  size_t max_tokens;
  float temperature;
  float top_p;
  size_t top_k;
  uint64_t seed;
  const uint32_t* stop_token_ids;
  size_t stop_token_count;
} mi_generation_options;

/* sample_token (qwen3.rs:909-925) / sample_token_f16 + sample_candidates
 * (qwen3.rs:927-1005) on the device: one token from FP16 logits ([n] or
 * [1, n]) under temperature / top_p / top_k as GenerationOptions, drawing
 * from the XorShift64 state *state (in/out, qwen3.rs:1011-1034; seed it with
 * mi_xorshift_seed). Temperature 0 is the greedy argmax and leaves *state.
 * Candidates are ordered by descending value, equal logits by ascending
 * index; every FP64 sum is the reference's sequential one. Synchronous.
 * Errors: MI_ERR_CONFIG "logits contain no finite value" / "failed to sample
 * a token" and the validate_generation_options messages. */
mi_status mi_sample_logits(mi_context* ctx, const mi_tensor* logits, float temperature,
                           float top_p, size_t top_k, uint64_t* state, uint32_t* token);
/* XorShift64::new (qwen3.rs:1016-1024): seed 0 becomes 0x9e3779b97f4a7c15. */
uint64_t mi_xorshift_seed(uint64_t seed);

typedef struct mi_qwen3 mi_qwen3;
typedef struct mi_kv_cache mi_kv_cache;

/* Qwen3Config::validate (config.rs:23-57) */
mi_status mi_qwen3_config_validate(const mi_qwen3_config* config);
/* Random-init weights for benchmarks (no checkpoint): every matrix is
 * N(0, std) from the counter-based SplitMix64 + Box-Muller generator keyed by
 * (seed, stream); norm gains are 1.0. Stream of layer l, role r is
 * (l + 1) * 16 + r (roles: 0 embedding, 1 q, 2 k, 3 v, 4 o, 7 gate, 8 up,
 * 9 down, 13 lm_head). Replaces Qwen3Model::load (qwen3.rs:155-240) for
 * synthetic runs. */
mi_status mi_qwen3_create_random(mi_context* ctx, const mi_qwen3_config* config, uint64_t seed,
                                 double std_dev, mi_qwen3** out);
/* ---- tensor parallelism (no counterpart in the reference, which runs on
 * one GPU). Megatron-style sharding over tp ranks, one process (context)
 * per GPU: rank r holds query heads [q_head0, q_head0 + q_heads), KV heads
 * [kv_head0, ...), MLP columns [inter0, ...) and LM-head rows (vocabulary)
 * [vocab0, ...); the O and down projections are row-parallel: each rank's
 * FP32 partial products are gathered over NCCL and summed in rank order,
 * then rounded once to FP16; the greedy id is the best of the ranks'
 * candidates. Every rank calls the same model functions in the same order
 * (prefill, decode, generate return identical ids on all ranks; logits are
 * gathered over the full vocabulary). */
typedef struct mi_tp_shard_info {
  size_t q_heads, kv_heads, intermediate, vocab;
  size_t q_head0, kv_head0, inter0, vocab0;
} mi_tp_shard_info;
/* This rank's shard of `config` (host only; no device needed). */
mi_status mi_tp_shard(const mi_qwen3_config* config, int tp, int rank, mi_tp_shard_info* out);
/* A fresh NCCL unique id (128 bytes) for rank 0 to share with the others. */
mi_status mi_nccl_unique_id(uint8_t* out, size_t len);
/* mi_qwen3_create_random's model, this rank's shard of it; joins the NCCL
 * communicator of `nccl_id` (collective: every rank must call it). tp = 1
 * is mi_qwen3_create_random. */
mi_status mi_qwen3_create_random_tp(mi_context* ctx, const mi_qwen3_config* config,
                                    uint64_t seed, double std_dev, int tp, int rank,
                                    const uint8_t* nccl_id, mi_qwen3** out);
/* Qwen3Model::load from a directory with config.json + model.safetensors
 * or the shards named by model.safetensors.index.json (qwen3.rs:155-240,
 * weights.rs:21-75, config.rs:23-57). F16 tensors are used as stored, BF16
 * ones converted to FP16 through FP32 with round-to-nearest-even; other
 * dtypes, model_type other than qwen3 and attention biases return
 * MI_ERR_UNSUPPORTED, a missing tensor MI_ERR_MISSING_TENSOR, a wrong shape
 * MI_ERR_CONFIG, unreadable files MI_ERR_IO. Tensor names as the
 * reference's (model.layers.{i}.self_attn.q_proj.weight, ...). */
mi_status mi_qwen3_load(mi_context* ctx, const char* directory, mi_qwen3** out);
/* No counterpart in the reference: mi_qwen3_load reading only this rank's
 * tensor-parallel shard of every weight (see mi_qwen3_create_random_tp). */
mi_status mi_qwen3_load_tp(mi_context* ctx, const char* directory, int tp, int rank,
                           const uint8_t* nccl_id, mi_qwen3** out);
void mi_qwen3_destroy(mi_qwen3* m);
mi_status mi_qwen3_get_config(const mi_qwen3* m, mi_qwen3_config* out);
/* Qwen3Model::set_attention_kind / set_fusion_options (qwen3.rs:330-346) */
mi_status mi_qwen3_set_attention_kind(mi_qwen3* m, mi_attention_kind kind);
mi_status mi_qwen3_set_fusion_options(mi_qwen3* m, mi_fusion_options options);
mi_fusion_options mi_qwen3_fusion_options(const mi_qwen3* m);
/* Decode steps run as one CUDA graph (default on); 0 launches eagerly. */
mi_status mi_qwen3_set_decode_graphs(mi_qwen3* m, int enabled);
/* Tensor-parallel diagnostics (no reference counterpart: the reference is
 * single-device). Synchronizes, then reports how long the CTAs of the most
 * recent persistent decode launch spent on inputs fed by the other ranks
 * (from the start of such a stage input until the O / DOWN partials that
 * arrived over NVLink, and the LM-head argmax records, had all validated,
 * staging included): the mean and the maximum over CTAs in seconds, and
 * that launch's decode steps. Zeros when tp = 1 or no persistent launch
 * ran. */
mi_status mi_qwen3_exchange_wait(mi_qwen3* m, double* mean_seconds, double* max_seconds,
                                 size_t* steps);
/* No counterpart in the reference (its decode encodes one command buffer per
 * step). Greedy decode steps run in one persistent cooperative kernel per
 * call (default on, also off with the environment variable
 * MI_DECODE_LOOP=0); 0 selects the per-kernel chain above. Both give the
 * same ids and logits. mi_qwen3_decode_persistent reports whether the
 * persistent kernel is in use for this model on this device. */
mi_status mi_qwen3_set_decode_persistent(mi_qwen3* m, int enabled);
mi_status mi_qwen3_decode_persistent(mi_qwen3* m, int* active);

/* KvCache::new / len / capacity / reset (qwen3.rs:75-117) */
mi_status mi_kv_cache_create(mi_qwen3* m, size_t capacity, mi_kv_cache** out);
void mi_kv_cache_destroy(mi_kv_cache* c);
size_t mi_kv_cache_len(const mi_kv_cache* c);
size_t mi_kv_cache_capacity(const mi_kv_cache* c);
void mi_kv_cache_reset(mi_kv_cache* c);
/* Layer cache tensors [capacity, kv_heads, head_dim] (views). */
mi_status mi_kv_cache_layer(mi_kv_cache* c, size_t layer, mi_tensor** key, mi_tensor** value);

/* Qwen3Model::prefill / prefill_with_stats (qwen3.rs:348-373): resets the
 * cache, runs the prompt, returns logits [1, vocab]. */
mi_status mi_qwen3_prefill(mi_qwen3* m, const uint32_t* tokens, size_t count, mi_kv_cache* cache,
                           mi_tensor** logits, mi_dispatch_stats* stats);
/* Qwen3Model::decode / decode_with_stats (qwen3.rs:375-386) */
mi_status mi_qwen3_decode(mi_qwen3* m, uint32_t token, mi_kv_cache* cache, mi_tensor** logits,
                          mi_dispatch_stats* stats);
/* Qwen3Model::prefill_argmax (qwen3.rs:388-410): writes the greedy id into
 * `output` (one u32); logits may be NULL. */
mi_status mi_qwen3_prefill_argmax(mi_qwen3* m, const uint32_t* tokens, size_t count,
                                  mi_kv_cache* cache, mi_tensor* output, mi_tensor** logits,
                                  mi_dispatch_stats* stats);
/* Qwen3Model::decode_argmax (qwen3.rs:412-422): reads the token from a
 * device u32, writes the next greedy id to `output`, returns a pending
 * handle without waiting. */
mi_status mi_qwen3_decode_argmax(mi_qwen3* m, const mi_tensor* token, mi_kv_cache* cache,
                                 mi_tensor* output, mi_tensor** logits, mi_pending** pending);
/* The pipelined greedy decode loop of generate_greedy (qwen3.rs:475-555)
 * and bench.rs run_pipelined_decode (bench.rs:1850-1895): enqueues `steps`
 * decode steps, each feeding the previous step's argmax (kept on the
 * device), without waiting. The cache must hold a prefilled prompt. Ids are
 * read back with mi_kv_cache_tokens. A launch whose bounded device wait
 * expired (it then leaves early and its ids are not valid) is reported as
 * MI_ERR_TIMEOUT by the next synchronizing call: mi_kv_cache_tokens,
 * mi_qwen3_generate*, mi_pending_wait or mi_context_kernel_status. */
mi_status mi_qwen3_decode_steps(mi_qwen3* m, mi_kv_cache* cache, size_t steps);
/* Copies cache positions [start, start + count) of the token ring (prompt
 * ids, then the greedy ids fed back; position len holds the next id) to the
 * host; synchronizes the context stream, then returns MI_ERR_TIMEOUT if a
 * bounded device wait expired in the work before it. */
mi_status mi_kv_cache_tokens(mi_kv_cache* cache, size_t start, size_t count, uint32_t* out);
/* Qwen3Model::generate (qwen3.rs:424-439): greedy, max_tokens ids;
 * MI_ERR_TIMEOUT if a bounded device wait of its launches expired. */
mi_status mi_qwen3_generate(mi_qwen3* m, const uint32_t* prompt, size_t prompt_len,
                            size_t max_tokens, mi_kv_cache* cache, uint32_t* out_ids,
                            size_t* out_count);
/* Qwen3Model::generate_with (qwen3.rs:441-473): on_token returns non-zero
 * to continue; it may be NULL. Temperature > 0 draws every token on the
 * device (prefill and decode lm_heads followed by the sampler, one
 * XorShift64 stream per call) through the same pipelined loop as greedy; the
 * persistent decode kernel is greedy-only, so sampled decode steps run the
 * per-kernel chain (captured as its own CUDA graph). */
typedef int (*mi_token_callback)(uint32_t token, void* user);
mi_status mi_qwen3_generate_with(mi_qwen3* m, const uint32_t* prompt, size_t prompt_len,
                                 const mi_generation_options* options, mi_kv_cache* cache,
                                 mi_token_callback on_token, void* user, uint32_t* out_ids,
                                 size_t capacity, size_t* out_count);
/* Qwen3Model::run_first_block (qwen3.rs:557-583): first layer on the
 * embedded tokens with a scratch cache; returns hidden [T, hidden]. */
mi_status mi_qwen3_run_first_block(mi_qwen3* m, const uint32_t* tokens, size_t count,
                                   mi_tensor** out);
/* Every layer on caller-given hidden states [count, hidden] at the cache's
 * position (no embedding and no head); appends to the cache. The one-block
 * benchmark config feeds hidden states directly. */
mi_status mi_qwen3_forward_hidden(mi_qwen3* m, const mi_tensor* hidden, mi_kv_cache* cache,
                                  mi_tensor** out);
/* A weight tensor by role (see mi_qwen3_create_random); layer -1 for
 * model-level tensors. */
mi_status mi_qwen3_weight(mi_qwen3* m, int layer, int role, mi_tensor** out);

/* ---- synthetic inputs ----------------------------------------------------- */
/* The generator of mi_qwen3_create_random, on the device: element i of
 * stream (seed, stream) for i in [offset, offset + len). */
mi_status mi_fill_normal_f16(mi_context* ctx, mi_tensor* t, uint64_t seed, uint64_t stream,
                             uint64_t offset, double std_dev);
mi_status mi_fill_tokens_u32(mi_context* ctx, mi_tensor* t, uint64_t seed, uint64_t stream,
                             uint32_t vocab);

#ifdef __cplusplus
}
#endif
#endif /* MI_H */
