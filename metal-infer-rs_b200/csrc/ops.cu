// Op layer of the C ABI: one mi_batch_* entry per CommandBatch method
// (crates/metal-infer-core/src/ops.rs:221-1285) with the same shape and dtype
// validation and error messages; outputs are new stream-ordered tensors.

#include <cmath>
#include <cstring>

#include "kernels.h"
#include "mi_internal.h"

using namespace mi;

namespace {

// Op launches use programmatic dependent launch (each kernel waits for its
// predecessor before it reads any operand, so back-to-back ops overlap only
// their launch latency), unless per-kernel profiling puts events between them.
k::Launch launch_of(mi_context* ctx) {
  k::Launch l;
  l.stream = ctx->stream;
  l.pdl = !ctx->profiling;
  l.early = false;
  l.sm_count = ctx->sm_count;
  return l;
}

void require(const void* p, const char* what) {
  MI_REQUIRE(p != nullptr, MI_ERR_INVALID_ARGUMENT, "%s is NULL", what);
}

mi_context* ctx_of(mi_batch* b) {
  require(b, "batch");
  return b->ctx;
}

// require_f16 (ops.rs:1334-1344)
void require_f16(const mi_tensor* t) {
  require(t, "tensor");
  if (t->dtype != MI_F16)
    fail(MI_ERR_DTYPE, "unsupported dtype: expected f16, got %s", dtype_name(t->dtype));
}

std::string shape_str(const std::vector<size_t>& s) {
  std::string r = "[";
  for (size_t i = 0; i < s.size(); ++i) r += (i ? ", " : "") + std::to_string(s[i]);
  return r + "]";
}

// require_same_shape (ops.rs:1346-1360)
void require_same_shape(const mi_tensor* a, const mi_tensor* b) {
  if (a->shape != b->shape)
    fail(MI_ERR_SHAPE, "invalid tensor shape: shape mismatch: %s and %s",
         shape_str(a->shape).c_str(), shape_str(b->shape).c_str());
}

// matrix_shape (ops.rs:1362-1367)
std::pair<size_t, size_t> matrix_shape(const mi_tensor* t) {
  if (t->shape.size() != 2)
    fail(MI_ERR_SHAPE, "invalid tensor shape: expected matrix, got %s",
         shape_str(t->shape).c_str());
  return {t->shape[0], t->shape[1]};
}

// to_u32 (ops.rs:1369-1376)
uint32_t to_u32(size_t v, const char* label) {
  if (v > 0xFFFFFFFFull) fail(MI_ERR_SHAPE, "invalid tensor shape: %s does not fit in u32", label);
  return (uint32_t)v;
}

int to_int(size_t v, const char* label) {
  if (v > 0x7FFFFFFFull) fail(MI_ERR_SHAPE, "invalid tensor shape: %s does not fit in i32", label);
  return (int)v;
}

struct Out {
  mi_tensor* t = nullptr;
  ~Out() {
    if (t) mi_tensor_release(t);
  }
  mi_tensor* release() {
    mi_tensor* r = t;
    t = nullptr;
    return r;
  }
};

bool use_reference(mi_context* ctx) { return ctx->backend == MI_MATMUL_REFERENCE; }

// x [m, k] . w^T for every weight; m == 1 fuses all weights into one GEMV.
void matmul_n(mi_batch* b, const mi_tensor* input, const mi_tensor* const* w, int count,
              mi_tensor** outs) {
  mi_context* ctx = ctx_of(b);
  require_f16(input);
  for (int i = 0; i < count; ++i) require_f16(w[i]);
  auto [m, kk] = matrix_shape(input);
  Out o[3];
  size_t n[3] = {0, 0, 0};
  for (int i = 0; i < count; ++i) {
    auto [ni, ki] = matrix_shape(w[i]);
    if (ki != kk)
      fail(MI_ERR_SHAPE, "invalid tensor shape: matmul inner dimensions differ: %zu and %zu", kk,
           ki);
    n[i] = ni;
  }
  for (int i = 0; i < count; ++i) o[i].t = new_tensor(ctx, {m, n[i]}, MI_F16);
  k::Launch l = launch_of(ctx);
  int mi_ = to_int(m, "m"), ki = to_int(kk, "k");
  if (m == 0 || kk == 0) {
    for (int i = 0; i < count; ++i)
      if (m && n[i]) MI_CUDA(cudaMemsetAsync(o[i].t->base(), 0, o[i].t->bytes(), ctx->stream));
  } else if (use_reference(ctx)) {
    ProfileScope ps(ctx, "matmul_reference");
    for (int i = 0; i < count; ++i)
      k::matmul_reference(l, input->f16(), w[i]->f16(), o[i].t->f16(), mi_, to_int(n[i], "n"),
                          ki);
  } else if (m == 1) {
    ProfileScope ps(ctx, count == 1 ? "gemv" : count == 2 ? "gemv2" : "gemv3");
    k::GemvProblem p;
    p.k = ki;
    p.segments = count;
    p.x = input->f16();
    for (int i = 0; i < count; ++i) {
      p.w[i] = w[i]->f16();
      p.n[i] = to_int(n[i], "n");
      p.out[i] = o[i].t->f16();
    }
    k::gemv(l, p);
  } else {
    ProfileScope ps(ctx, "gemm");
    for (int i = 0; i < count; ++i)
      k::gemm(l, input->f16(), w[i]->f16(), o[i].t->f16(), mi_, to_int(n[i], "n"), ki,
              to_int(n[i], "n"));
  }
  for (int i = 0; i < count; ++i) outs[i] = o[i].release();
}

}  // namespace

extern "C" {

mi_status mi_batch_add(mi_batch* b, const mi_tensor* left, const mi_tensor* right,
                       mi_tensor** out) {
  return guard([&] {
    mi_context* ctx = ctx_of(b);
    require(out, "out");
    require_f16(left);
    require_f16(right);
    require_same_shape(left, right);
    Out o;
    o.t = new_tensor(ctx, left->shape, MI_F16);
    ProfileScope ps(ctx, "add");
    k::add(launch_of(ctx), left->f16(), right->f16(), o.t->f16(), left->len());
    *out = o.release();
  });
}

mi_status mi_batch_matmul(mi_batch* b, const mi_tensor* input, const mi_tensor* weight,
                          mi_tensor** out) {
  return guard([&] {
    require(out, "out");
    const mi_tensor* w[1] = {weight};
    matmul_n(b, input, w, 1, out);
  });
}

mi_status mi_batch_matmul2(mi_batch* b, const mi_tensor* input, const mi_tensor* w0,
                           const mi_tensor* w1, mi_tensor** out0, mi_tensor** out1) {
  return guard([&] {
    require(out0, "out0");
    require(out1, "out1");
    const mi_tensor* w[2] = {w0, w1};
    mi_tensor* outs[2];
    matmul_n(b, input, w, 2, outs);
    *out0 = outs[0];
    *out1 = outs[1];
  });
}

mi_status mi_batch_matmul3(mi_batch* b, const mi_tensor* input, const mi_tensor* w0,
                           const mi_tensor* w1, const mi_tensor* w2, mi_tensor** out0,
                           mi_tensor** out1, mi_tensor** out2) {
  return guard([&] {
    require(out0, "out0");
    require(out1, "out1");
    require(out2, "out2");
    const mi_tensor* w[3] = {w0, w1, w2};
    mi_tensor* outs[3];
    matmul_n(b, input, w, 3, outs);
    *out0 = outs[0];
    *out1 = outs[1];
    *out2 = outs[2];
  });
}

// rms_norm_matmul3 (ops.rs:568-642)
mi_status mi_batch_rms_norm_matmul3(mi_batch* b, const mi_tensor* input,
                                    const mi_tensor* norm_weight, const mi_tensor* w0,
                                    const mi_tensor* w1, const mi_tensor* w2, float epsilon,
                                    mi_tensor** out0, mi_tensor** out1, mi_tensor** out2) {
  return guard([&] {
    mi_context* ctx = ctx_of(b);
    require(out0, "out0");
    require(out1, "out1");
    require(out2, "out2");
    for (const mi_tensor* t : {input, norm_weight, w0, w1, w2}) require_f16(t);
    auto [rows, width] = matrix_shape(input);
    auto [n0, k0] = matrix_shape(w0);
    auto [n1, k1] = matrix_shape(w1);
    auto [n2, k2] = matrix_shape(w2);
    if (rows != 1 || width % 256 != 0 || norm_weight->shape != std::vector<size_t>{width} ||
        k0 != width || k1 != width || k2 != width)
      fail(MI_ERR_SHAPE,
           "invalid tensor shape: rms_norm_matmul3 requires one row and matching widths "
           "divisible by 256");
    Out o[3];
    o[0].t = new_tensor(ctx, {1, n0}, MI_F16);
    o[1].t = new_tensor(ctx, {1, n1}, MI_F16);
    o[2].t = new_tensor(ctx, {1, n2}, MI_F16);
    k::GemvProblem p;
    p.k = to_int(width, "width");
    p.segments = 3;
    p.in_mode = k::kInNorm;
    p.x = input->f16();
    p.norm_w = norm_weight->f16();
    p.eps = epsilon;
    const mi_tensor* ws[3] = {w0, w1, w2};
    size_t ns[3] = {n0, n1, n2};
    for (int i = 0; i < 3; ++i) {
      p.w[i] = ws[i]->f16();
      p.n[i] = to_int(ns[i], "n");
      p.out[i] = o[i].t->f16();
    }
    ProfileScope ps(ctx, "rms_norm_gemv3");
    k::gemv(launch_of(ctx), p);
    *out0 = o[0].release();
    *out1 = o[1].release();
    *out2 = o[2].release();
  });
}

// add_rms_norm_matmul2 (ops.rs:644-720)
mi_status mi_batch_add_rms_norm_matmul2(mi_batch* b, const mi_tensor* left,
                                        const mi_tensor* right, const mi_tensor* norm_weight,
                                        const mi_tensor* w0, const mi_tensor* w1, float epsilon,
                                        mi_tensor** residual, mi_tensor** out0,
                                        mi_tensor** out1) {
  return guard([&] {
    mi_context* ctx = ctx_of(b);
    require(residual, "residual");
    require(out0, "out0");
    require(out1, "out1");
    for (const mi_tensor* t : {left, right, norm_weight, w0, w1}) require_f16(t);
    require_same_shape(left, right);
    auto [rows, width] = matrix_shape(left);
    auto [n0, k0] = matrix_shape(w0);
    auto [n1, k1] = matrix_shape(w1);
    if (rows != 1 || width % 256 != 0 || norm_weight->shape != std::vector<size_t>{width} ||
        k0 != width || k1 != width)
      fail(MI_ERR_SHAPE,
           "invalid tensor shape: add_rms_norm_matmul2 requires one row and matching widths "
           "divisible by 256");
    Out r, o0, o1;
    r.t = new_tensor(ctx, {1, width}, MI_F16);
    o0.t = new_tensor(ctx, {1, n0}, MI_F16);
    o1.t = new_tensor(ctx, {1, n1}, MI_F16);
    k::GemvProblem p;
    p.k = to_int(width, "width");
    p.segments = 2;
    p.in_mode = k::kInAddNorm;
    p.x = left->f16();
    p.x2 = right->f16();
    p.norm_w = norm_weight->f16();
    p.eps = epsilon;
    p.residual_out = r.t->f16();
    p.w[0] = w0->f16();
    p.w[1] = w1->f16();
    p.n[0] = to_int(n0, "n0");
    p.n[1] = to_int(n1, "n1");
    p.out[0] = o0.t->f16();
    p.out[1] = o1.t->f16();
    ProfileScope ps(ctx, "add_rms_norm_gemv2");
    k::gemv(launch_of(ctx), p);
    *residual = r.release();
    *out0 = o0.release();
    *out1 = o1.release();
  });
}

// rms_norm (ops.rs:722-755)
mi_status mi_batch_rms_norm(mi_batch* b, const mi_tensor* input, const mi_tensor* weight,
                            float epsilon, mi_tensor** out) {
  return guard([&] {
    mi_context* ctx = ctx_of(b);
    require(out, "out");
    require_f16(input);
    require_f16(weight);
    if (input->shape.empty()) fail(MI_ERR_SHAPE, "invalid tensor shape: rms_norm requires rank >= 1");
    size_t width = input->shape.back();
    if (weight->shape != std::vector<size_t>{width})
      fail(MI_ERR_SHAPE, "invalid tensor shape: rms_norm weight must have shape [%zu]", width);
    Out o;
    o.t = new_tensor(ctx, input->shape, MI_F16);
    size_t rows = width ? input->len() / width : 0;
    ProfileScope ps(ctx, "rms_norm");
    k::rms_norm(launch_of(ctx), input->f16(), weight->f16(), o.t->f16(), to_int(rows, "rows"),
                to_int(width, "width"), epsilon);
    *out = o.release();
  });
}

// add_rms_norm (ops.rs:757-798)
mi_status mi_batch_add_rms_norm(mi_batch* b, const mi_tensor* left, const mi_tensor* right,
                                const mi_tensor* weight, float epsilon, mi_tensor** residual,
                                mi_tensor** normalized) {
  return guard([&] {
    mi_context* ctx = ctx_of(b);
    require(residual, "residual");
    require(normalized, "normalized");
    require_f16(left);
    require_f16(right);
    require_f16(weight);
    require_same_shape(left, right);
    if (left->shape.empty())
      fail(MI_ERR_SHAPE, "invalid tensor shape: add_rms_norm requires rank >= 1");
    size_t width = left->shape.back();
    if (weight->shape != std::vector<size_t>{width})
      fail(MI_ERR_SHAPE, "invalid tensor shape: add_rms_norm weight must have shape [%zu]", width);
    Out r, n;
    r.t = new_tensor(ctx, left->shape, MI_F16);
    n.t = new_tensor(ctx, left->shape, MI_F16);
    size_t rows = width ? left->len() / width : 0;
    ProfileScope ps(ctx, "add_rms_norm");
    k::add_rms_norm(launch_of(ctx), left->f16(), right->f16(), weight->f16(), r.t->f16(),
                    n.t->f16(), to_int(rows, "rows"), to_int(width, "width"), epsilon);
    *residual = r.release();
    *normalized = n.release();
  });
}

// swiglu (ops.rs:800-818)
mi_status mi_batch_swiglu(mi_batch* b, const mi_tensor* gate, const mi_tensor* up,
                          mi_tensor** out) {
  return guard([&] {
    mi_context* ctx = ctx_of(b);
    require(out, "out");
    require_f16(gate);
    require_f16(up);
    require_same_shape(gate, up);
    Out o;
    o.t = new_tensor(ctx, gate->shape, MI_F16);
    ProfileScope ps(ctx, "swiglu");
    k::swiglu(launch_of(ctx), gate->f16(), up->f16(), o.t->f16(), gate->len());
    *out = o.release();
  });
}

// embedding (ops.rs:820-845)
mi_status mi_batch_embedding(mi_batch* b, const mi_tensor* tokens, const mi_tensor* table,
                             mi_tensor** out) {
  return guard([&] {
    mi_context* ctx = ctx_of(b);
    require(out, "out");
    require(tokens, "tokens");
    if (tokens->dtype != MI_U32 || tokens->shape.size() != 1)
      fail(MI_ERR_SHAPE, "invalid tensor shape: tokens must be a rank-1 u32 tensor");
    require_f16(table);
    auto [rows, width] = matrix_shape(table);
    Out o;
    o.t = new_tensor(ctx, {tokens->len(), width}, MI_F16);
    ProfileScope ps(ctx, "embedding");
    k::embedding(launch_of(ctx), tokens->u32(), table->f16(), o.t->f16(),
                 to_int(tokens->len(), "token count"), to_int(width, "embedding width"),
                 to_u32(rows, "rows"));
    *out = o.release();
  });
}

// argmax (ops.rs:847-880)
mi_status mi_batch_argmax(mi_batch* b, const mi_tensor* logits, mi_tensor* output) {
  return guard([&] {
    mi_context* ctx = ctx_of(b);
    require_f16(logits);
    require(output, "output");
    if (logits->shape.size() != 1 || logits->len() == 0)
      fail(MI_ERR_SHAPE, "invalid tensor shape: argmax logits must be a nonempty vector");
    if (output->dtype != MI_U32 || output->shape != std::vector<size_t>{1})
      fail(MI_ERR_SHAPE, "invalid tensor shape: argmax output must be one u32");
    to_u32(logits->len(), "argmax logits count");
    int groups = k::argmax_partials(logits->len());
    Out pv, pi;
    pv.t = new_tensor(ctx, {(size_t)groups}, MI_F32);
    pi.t = new_tensor(ctx, {(size_t)groups}, MI_U32);
    ProfileScope ps(ctx, "argmax");
    k::argmax(launch_of(ctx), logits->f16(), logits->len(), pv.t->f32(), pi.t->u32(),
              output->u32());
  });
}

// rope (ops.rs:882-915)
mi_status mi_batch_rope(mi_batch* b, const mi_tensor* input, size_t offset, float theta,
                        mi_tensor** out) {
  return guard([&] {
    mi_context* ctx = ctx_of(b);
    require(out, "out");
    require_f16(input);
    if (input->shape.size() != 3)
      fail(MI_ERR_SHAPE, "invalid tensor shape: RoPE expects [tokens, heads, head_dim]");
    size_t tokens = input->shape[0], heads = input->shape[1], hd = input->shape[2];
    if (hd % 2) fail(MI_ERR_SHAPE, "invalid tensor shape: RoPE head_dim must be even");
    Out o;
    o.t = new_tensor(ctx, input->shape, MI_F16);
    k::Pos pos;
    pos.base = to_u32(offset, "offset");
    ProfileScope ps(ctx, "rope");
    k::rope(launch_of(ctx), input->f16(), o.t->f16(), to_int(tokens, "tokens"),
            to_int(heads, "heads"), to_int(hd, "head_dim"), pos, theta);
    *out = o.release();
  });
}

// qk_norm_rope_cache (ops.rs:917-977)
mi_status mi_batch_qk_norm_rope_cache(mi_batch* b, const mi_tensor* query, const mi_tensor* key,
                                      const mi_tensor* query_weight,
                                      const mi_tensor* key_weight, mi_tensor* key_cache,
                                      mi_qk_config config, mi_tensor** out) {
  return guard([&] {
    mi_context* ctx = ctx_of(b);
    require(out, "out");
    for (const mi_tensor* t : {query, key, query_weight, key_weight, (const mi_tensor*)key_cache})
      require_f16(t);
    if (query->shape.size() != 3) fail(MI_ERR_SHAPE, "invalid tensor shape: query must have rank 3");
    if (key->shape.size() != 3) fail(MI_ERR_SHAPE, "invalid tensor shape: key must have rank 3");
    if (key_cache->shape.size() != 3)
      fail(MI_ERR_SHAPE, "invalid tensor shape: key cache must have rank 3");
    size_t tokens = query->shape[0], qh = query->shape[1], hd = query->shape[2];
    size_t kt = key->shape[0], kvh = key->shape[1], kd = key->shape[2];
    size_t cap = key_cache->shape[0], ch = key_cache->shape[1], cd = key_cache->shape[2];
    if (tokens != kt || hd != kd || kvh != ch || hd != cd ||
        query_weight->shape != std::vector<size_t>{hd} ||
        key_weight->shape != std::vector<size_t>{hd})
      fail(MI_ERR_SHAPE, "invalid tensor shape: Q/K transform tensor shapes are incompatible");
    if (hd % 2 || config.offset + tokens > cap)
      fail(MI_ERR_SHAPE, "invalid tensor shape: Q/K transform has invalid head_dim or cache offset");
    Out o;
    o.t = new_tensor(ctx, query->shape, MI_F16);
    k::Pos pos;
    pos.base = to_u32(config.offset, "offset");
    ProfileScope ps(ctx, "qk_norm_rope_cache");
    k::qk_norm_rope_cache(launch_of(ctx), query->f16(), key->f16(), query_weight->f16(),
                          key_weight->f16(), o.t->f16(), key_cache->f16(),
                          to_int(tokens, "tokens"), to_int(qh, "query heads"),
                          to_int(kvh, "KV heads"), to_int(hd, "head dim"), pos, config.theta,
                          config.epsilon, false);
    *out = o.release();
  });
}

}  // extern "C"

namespace {

// attention_with_flash_configuration (ops.rs:1050-1247)
mi_tensor* attention_impl(mi_batch* b, const mi_tensor* query, const mi_tensor* key,
                          const mi_tensor* value, mi_attention_config config,
                          mi_attention_kind kind, size_t block_keys, size_t threads,
                          bool explicit_flash) {
  mi_context* ctx = ctx_of(b);
  require_f16(query);
  require_f16(key);
  require_f16(value);
  if (query->shape.size() != 3) fail(MI_ERR_SHAPE, "invalid tensor shape: query must have rank 3");
  if (key->shape.size() != 3) fail(MI_ERR_SHAPE, "invalid tensor shape: key must have rank 3");
  if (value->shape.size() != 3) fail(MI_ERR_SHAPE, "invalid tensor shape: value must have rank 3");
  size_t tokens = query->shape[0], qh = query->shape[1], qd = query->shape[2];
  size_t kv_len = key->shape[0], kh = key->shape[1], kd = key->shape[2];
  if (qh != config.query_heads || qd != config.head_dim || kh != config.kv_heads ||
      kd != config.head_dim || value->shape[0] != kv_len || value->shape[1] != kh ||
      value->shape[2] != kd)
    fail(MI_ERR_SHAPE, "invalid tensor shape: attention tensor shapes do not match config");
  if (config.kv_heads == 0 || config.query_heads % config.kv_heads != 0)
    fail(MI_ERR_SHAPE, "invalid tensor shape: query_heads must be divisible by kv_heads");
  size_t hd = config.head_dim;
  bool pow2 = hd && (hd & (hd - 1)) == 0;
  if (kind != MI_ATTENTION_REFERENCE && (!pow2 || hd > 256))
    fail(MI_ERR_SHAPE, "invalid tensor shape: tiled attention requires a power-of-two head_dim <= 256");
  if (kind == MI_ATTENTION_FLASH_DECODE) {
    if (!explicit_flash) {
      block_keys = 64;
      threads = 256;
    }
    if (!(block_keys == 32 || block_keys == 64 || block_keys == 128 || block_keys == 256))
      fail(MI_ERR_SHAPE, "invalid tensor shape: flash decode block size must be 32, 64, 128, or 256");
    if (!(threads == 128 || threads == 256))
      fail(MI_ERR_SHAPE, "invalid tensor shape: flash decode threadgroup size must be 128 or 256");
  }
  if ((kind == MI_ATTENTION_DECODE_SPLIT_KV || kind == MI_ATTENTION_FLASH_DECODE) && tokens != 1)
    fail(MI_ERR_SHAPE, "invalid tensor shape: decode attention requires exactly one query token");
  Out o;
  o.t = new_tensor(ctx, query->shape, MI_F16);
  k::AttnProblem p;
  p.q = query->f16();
  p.k = key->f16();
  p.v = value->f16();
  p.out = o.t->f16();
  p.tokens = to_int(tokens, "tokens");
  p.qh = to_int(qh, "query_heads");
  p.kvh = to_int(kh, "kv_heads");
  p.hd = to_int(hd, "head_dim");
  p.kv_len = to_int(kv_len, "kv_length");
  p.causal = config.causal ? 1 : 0;
  p.query_offset = to_int(config.query_offset, "query_offset");
  k::Launch l = launch_of(ctx);
  if (tokens == 0) return o.release();
  switch (kind) {
    case MI_ATTENTION_REFERENCE: {
      ProfileScope ps(ctx, "attention_reference");
      k::attention_reference(l, p);
      break;
    }
    case MI_ATTENTION_TILED:
    case MI_ATTENTION_FLASH_PREFILL: {
      ProfileScope ps(ctx, kind == MI_ATTENTION_TILED ? "attention_tiled" : "attention_flash_prefill");
      p.round_p = kind == MI_ATTENTION_FLASH_PREFILL ? 1 : 0;
      k::attention_prefill(l, p);
      break;
    }
    case MI_ATTENTION_DECODE_SPLIT_KV:
    case MI_ATTENTION_FLASH_DECODE: {
      if (kind == MI_ATTENTION_FLASH_DECODE) {
        if (qh / kh != 2)
          fail(MI_ERR_SHAPE, "invalid tensor shape: flash decode requires two query heads per KV head");
        size_t available = config.causal ? std::min(kv_len, config.query_offset + 1) : kv_len;
        if (available == 0)
          fail(MI_ERR_SHAPE, "invalid tensor shape: flash decode requires at least one available key");
      }
      size_t available = config.causal ? std::min(kv_len, config.query_offset + 1) : kv_len;
      if (kind == MI_ATTENTION_DECODE_SPLIT_KV) {
        // attention_decode_f16 (transformer.metal:1824-1909): one block over
        // all keys, interleaved streams merged at the end.
        block_keys = std::max<size_t>(64, (available + 63) / 64 * 64);
      }
      int splits = (int)std::max<size_t>(1, std::min<size_t>((available + block_keys - 1) / block_keys,
                                                              4096));
      int group = (int)(qh / kh);
      size_t scratch = k::attention_decode_scratch(p.kvh, splits, group, p.hd);
      Out sc, cnt;
      sc.t = new_tensor(ctx, {scratch / 4}, MI_F32);
      cnt.t = new_tensor(ctx, {kh}, MI_U32, true);
      ProfileScope ps(ctx, kind == MI_ATTENTION_FLASH_DECODE ? "attention_flash_decode"
                                                             : "attention_decode_split_kv");
      k::attention_decode(l, p, splits, (int)block_keys, sc.t->f32(), cnt.t->u32());
      break;
    }
    default:
      fail(MI_ERR_INVALID_ARGUMENT, "unknown attention kind %d", (int)kind);
  }
  return o.release();
}

}  // namespace

extern "C" {

mi_status mi_batch_attention(mi_batch* b, const mi_tensor* query, const mi_tensor* key,
                             const mi_tensor* value, mi_attention_config config,
                             mi_attention_kind kind, mi_tensor** out) {
  return guard([&] {
    require(out, "out");
    *out = attention_impl(b, query, key, value, config, kind, 0, 0, false);
  });
}

mi_status mi_batch_attention_flash_decode_with_configuration(
    mi_batch* b, const mi_tensor* query, const mi_tensor* key, const mi_tensor* value,
    mi_attention_config config, size_t block_keys, size_t threads, mi_tensor** out) {
  return guard([&] {
    require(out, "out");
    *out = attention_impl(b, query, key, value, config, MI_ATTENTION_FLASH_DECODE, block_keys,
                          threads, true);
  });
}

// copy_into_cache (ops.rs:1249-1285)
mi_status mi_batch_copy_into_cache(mi_batch* b, const mi_tensor* source, mi_tensor* cache,
                                   size_t offset) {
  return guard([&] {
    mi_context* ctx = ctx_of(b);
    require_f16(source);
    require_f16(cache);
    if (source->shape.size() != 3)
      fail(MI_ERR_SHAPE, "invalid tensor shape: KV source must have rank 3");
    if (cache->shape.size() != 3)
      fail(MI_ERR_SHAPE, "invalid tensor shape: KV cache must have rank 3");
    if (source->shape[1] != cache->shape[1] || source->shape[2] != cache->shape[2])
      fail(MI_ERR_SHAPE, "invalid tensor shape: KV source/cache shapes are incompatible");
    if (offset + source->shape[0] > cache->shape[0])
      fail(MI_ERR_SHAPE, "invalid tensor shape: KV cache capacity exceeded");
    k::Pos pos;
    pos.base = to_u32(offset, "offset");
    ProfileScope ps(ctx, "copy_kv");
    k::copy_kv(launch_of(ctx), source->f16(), cache->f16(), to_int(source->shape[0], "tokens"),
               to_int(source->shape[1] * source->shape[2], "stride"), pos);
  });
}

// sample_token (qwen3.rs:909-925) / sample_token_f16 (qwen3.rs:927-939) on
// the device, synchronous: the key histogram, then the one-CTA sampler.
mi_status mi_sample_logits(mi_context* ctx, const mi_tensor* logits, float temperature,
                           float top_p, size_t top_k, uint64_t* state, uint32_t* token) {
  return guard([&] {
    require(ctx, "ctx");
    require_f16(logits);
    require(state, "state");
    require(token, "token");
    if (!std::isfinite(temperature) || temperature < 0.f)
      fail(MI_ERR_CONFIG, "invalid model configuration: temperature must be finite and non-negative");
    if (!std::isfinite(top_p) || !(top_p >= 0.f && top_p <= 1.f))
      fail(MI_ERR_CONFIG, "invalid model configuration: top_p must be between 0 and 1");
    const size_t n = logits->len();
    const bool vector_shape = logits->shape.size() == 1 ||
                              (logits->shape.size() == 2 && logits->shape[0] == 1);
    if (!vector_shape || n == 0)
      fail(MI_ERR_SHAPE, "invalid tensor shape: sampling expects nonempty logits [n] or [1, n]");
    MI_REQUIRE(n < 0x80000000ull, MI_ERR_SHAPE, "invalid tensor shape: %zu logits exceed 2^31", n);
    if (top_k > 0xFFFFFFFFull)
      fail(MI_ERR_CONFIG, "invalid model configuration: top_k does not fit in u32");
    Out out;
    out.t = new_tensor(ctx, {2}, MI_U32);
    if (temperature == 0.f) {
      int groups = k::argmax_partials(n);
      Out pv, pi;
      pv.t = new_tensor(ctx, {(size_t)groups}, MI_F32);
      pi.t = new_tensor(ctx, {(size_t)groups}, MI_U32);
      k::argmax(launch_of(ctx), logits->f16(), n, pv.t->f32(), pi.t->u32(), out.t->u32());
    } else {
      Out hist, groups, opts, st;
      hist.t = new_tensor(ctx, {(size_t)k::kSampleHistWords}, MI_U32);
      groups.t = new_tensor(ctx, {2 * (size_t)k::kSampleBins}, MI_U32);
      opts.t = new_tensor(ctx, {4}, MI_U32);
      st.t = new_tensor(ctx, {2}, MI_U32);
      const float inv = 1.0f / temperature;
      uint32_t host_opts[4];
      std::memcpy(&host_opts[0], &inv, 4);
      std::memcpy(&host_opts[1], &top_p, 4);
      host_opts[2] = (uint32_t)top_k;
      host_opts[3] = 0;
      MI_CUDA(cudaMemsetAsync(hist.t->base(), 0, hist.t->bytes(), ctx->stream));
      MI_CUDA(cudaMemcpyAsync(opts.t->base(), host_opts, sizeof(host_opts),
                              cudaMemcpyHostToDevice, ctx->stream));
      MI_CUDA(cudaMemcpyAsync(st.t->base(), state, 8, cudaMemcpyHostToDevice, ctx->stream));
      ProfileScope ps(ctx, "sample");
      k::logit_histogram(launch_of(ctx), logits->f16(), (uint32_t)n, hist.t->u32());
      k::SampleProblem p;
      p.logits = logits->f16();
      p.n = (uint32_t)n;
      p.hist = hist.t->u32();
      p.groups = groups.t->u32();
      p.opts = opts.t->u32();
      p.state = reinterpret_cast<uint64_t*>(st.t->u32());
      p.token_out = out.t->u32();
      k::sample(launch_of(ctx), p);
      MI_CUDA(cudaMemcpyAsync(state, st.t->base(), 8, cudaMemcpyDeviceToHost, ctx->stream));
    }
    uint32_t tok = 0;
    MI_CUDA(cudaMemcpyAsync(&tok, out.t->base(), 4, cudaMemcpyDeviceToHost, ctx->stream));
    MI_CUDA(cudaStreamSynchronize(ctx->stream));
    if (tok == 0xFFFFFFFFu)
      fail(MI_ERR_CONFIG, "invalid model configuration: logits contain no finite value");
    if (tok == 0xFFFFFFFEu)
      fail(MI_ERR_CONFIG, "invalid model configuration: failed to sample a token");
    *token = tok;
  });
}

uint64_t mi_xorshift_seed(uint64_t seed) { return seed == 0 ? 0x9e3779b97f4a7c15ull : seed; }

mi_status mi_fill_normal_f16(mi_context* ctx, mi_tensor* t, uint64_t seed, uint64_t stream,
                             uint64_t offset, double std_dev) {
  return guard([&] {
    require(ctx, "ctx");
    require_f16(t);
    k::fill_normal_f16(ctx->stream, t->f16(), t->len(), seed, stream, offset, std_dev);
  });
}

mi_status mi_fill_tokens_u32(mi_context* ctx, mi_tensor* t, uint64_t seed, uint64_t stream,
                             uint32_t vocab) {
  return guard([&] {
    require(ctx, "ctx");
    require(t, "tensor");
    if (t->dtype != MI_U32) fail(MI_ERR_DTYPE, "unsupported dtype: expected u32, got %s",
                                 dtype_name(t->dtype));
    MI_REQUIRE(vocab > 0, MI_ERR_INVALID_ARGUMENT, "vocab must be non-zero");
    k::fill_tokens(ctx->stream, t->u32(), t->len(), seed, stream, vocab);
  });
}

}  // extern "C"
