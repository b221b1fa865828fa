// CPU oracle for the Qwen3 hot path of stratorys/metal-infer-rs.
//
// TEST INFRASTRUCTURE ONLY: the engine never links or calls this file. It is
// the checker for the CUDA kernels and the timed CPU baseline.
//
// Each function restates one reference kernel of
// crates/metal-infer-core/src/kernels/transformer.metal (cited per function)
// with the same FP16 rounding points. Reductions use FP32 like the reference;
// the reference leaves the summation order to the hardware (simd_sum), so the
// oracle fixes its own order: eight interleaved partial sums combined as a
// tree. Transcendentals come from the host libm. The reference's `half + half`
// (add_f16) is a correctly rounded half addition; it is computed here exactly
// in double and rounded once.
//
// Parity pinning: the reference has no CPU implementation and no stored
// outputs; the oracle is pinned against the inline CPU formulas and
// known-answer vectors of crates/metal-infer-core/tests/gpu.rs.

#include "oracle.h"

#include <immintrin.h>
#include <omp.h>

#include <algorithm>
#include <cmath>
#include <cstring>
#include <limits>
#include <vector>

namespace {

// ---------------------------------------------------------------------------
// IEEE binary16 conversions, round to nearest even.
// ---------------------------------------------------------------------------
inline uint64_t bits_of(double d) {
  uint64_t b;
  std::memcpy(&b, &d, 8);
  return b;
}

// Direct double -> half rounding (one rounding step).
uint16_t f64_to_f16(double d) {
  uint64_t b = bits_of(d);
  uint16_t sign = static_cast<uint16_t>((b >> 48) & 0x8000u);
  int exp = static_cast<int>((b >> 52) & 0x7ff);
  uint64_t mant = b & ((1ull << 52) - 1);
  if (exp == 0x7ff) return mant ? static_cast<uint16_t>(sign | 0x7e00u)
                                : static_cast<uint16_t>(sign | 0x7c00u);
  if (exp == 0) return sign;  // double subnormals are far below half range
  int e = exp - 1023;
  uint64_t full = mant | (1ull << 52);
  if (e > 15) return static_cast<uint16_t>(sign | 0x7c00u);
  if (e >= -14) {
    uint64_t m = full >> 42;
    uint64_t rem = full & ((1ull << 42) - 1);
    uint64_t half_way = 1ull << 41;
    if (rem > half_way || (rem == half_way && (m & 1))) ++m;
    if (m == (1ull << 11)) {
      m >>= 1;
      ++e;
    }
    if (e > 15) return static_cast<uint16_t>(sign | 0x7c00u);
    return static_cast<uint16_t>(sign | ((e + 15) << 10) | (m & 0x3ff));
  }
  if (e < -25) return sign;
  int shift = 28 - e;  // 43..53
  uint64_t m = full >> shift;
  uint64_t rem = full & ((1ull << shift) - 1);
  uint64_t half_way = 1ull << (shift - 1);
  if (rem > half_way || (rem == half_way && (m & 1))) ++m;
  return static_cast<uint16_t>(sign | m);
}

inline uint16_t h(float f) { return f64_to_f16(static_cast<double>(f)); }

inline float f(uint16_t x) { return _cvtsh_ss(x); }

bool g_acc_f64 = false;

// ---------------------------------------------------------------------------
// Dot products of FP16 vectors with FP32 accumulation. Products of two FP16
// values are exact in FP32, so only the summation order matters: eight
// interleaved partial sums, then a tree (0+4,1+5,2+6,3+7; 0+2,1+3; 0+1).
// ---------------------------------------------------------------------------
inline float tree8(__m256 acc) {
  __m128 lo = _mm256_castps256_ps128(acc);
  __m128 hi = _mm256_extractf128_ps(acc, 1);
  __m128 s = _mm_add_ps(lo, hi);
  __m128 s2 = _mm_add_ps(s, _mm_movehl_ps(s, s));
  __m128 s3 = _mm_add_ss(s2, _mm_shuffle_ps(s2, s2, 1));
  return _mm_cvtss_f32(s3);
}

// x is FP32 (already widened), w is FP16.
float dot_xf_w16(const float* x, const uint16_t* w, size_t k) {
  if (g_acc_f64) {
    double s = 0.0;
    for (size_t i = 0; i < k; ++i) s += static_cast<double>(x[i]) * f(w[i]);
    return static_cast<float>(s);
  }
  __m256 acc = _mm256_setzero_ps();
  size_t i = 0;
  for (; i + 8 <= k; i += 8) {
    __m256 wv = _mm256_cvtph_ps(
        _mm_loadu_si128(reinterpret_cast<const __m128i*>(w + i)));
    __m256 xv = _mm256_loadu_ps(x + i);
    acc = _mm256_add_ps(acc, _mm256_mul_ps(xv, wv));
  }
  float s = tree8(acc);
  for (; i < k; ++i) s += x[i] * f(w[i]);
  return s;
}

float dot_f32(const float* a, const float* b, size_t k) {
  if (g_acc_f64) {
    double s = 0.0;
    for (size_t i = 0; i < k; ++i) s += static_cast<double>(a[i]) * b[i];
    return static_cast<float>(s);
  }
  __m256 acc = _mm256_setzero_ps();
  size_t i = 0;
  for (; i + 8 <= k; i += 8)
    acc = _mm256_add_ps(acc, _mm256_mul_ps(_mm256_loadu_ps(a + i),
                                           _mm256_loadu_ps(b + i)));
  float s = tree8(acc);
  for (; i < k; ++i) s += a[i] * b[i];
  return s;
}

void widen(const uint16_t* in, float* out, size_t n) {
  size_t i = 0;
  for (; i + 8 <= n; i += 8)
    _mm256_storeu_ps(out + i, _mm256_cvtph_ps(_mm_loadu_si128(
                                  reinterpret_cast<const __m128i*>(in + i))));
  for (; i < n; ++i) out[i] = f(in[i]);
}

// Sum of squares in FP32 (same fixed order as the dot products).
float sum_squares(const float* x, size_t n) { return dot_f32(x, x, n); }

// rsqrt(total / width + eps) of the reference, as a correctly rounded
// reciprocal of a correctly rounded square root.
inline float rms_scale(float total, size_t width, float eps) {
  return 1.0f / std::sqrt(total / static_cast<float>(width) + eps);
}

// out[m,n] for x already widened to FP32 ([m,k]); parallel over weight rows.
void matmul_xf(const float* xf, size_t m, size_t k, const uint16_t* w,
               size_t n, uint16_t* out) {
#pragma omp parallel for schedule(static)
  for (long long row = 0; row < static_cast<long long>(n); ++row) {
    const uint16_t* wr = w + static_cast<size_t>(row) * k;
    for (size_t r = 0; r < m; ++r)
      out[r * n + row] = h(dot_xf_w16(xf + r * k, wr, k));
  }
}

// ---------------------------------------------------------------------------
// SplitMix64 (Steele, Lea and Flood, 2014) as a counter-based generator: the
// i-th output of the stream is mix64(state0 + (i + 1) * gamma). Normals come
// from the Box-Muller transform (1958) on pairs (2j, 2j + 1).
// ---------------------------------------------------------------------------
constexpr uint64_t kGamma = 0x9E3779B97F4A7C15ull;

inline uint64_t mix64(uint64_t z) {
  z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
  z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
  return z ^ (z >> 31);
}

inline uint64_t stream_state(uint64_t seed, uint64_t stream) {
  return mix64(seed ^ mix64(stream * kGamma + 0x632BE59BD9B4E019ull));
}

inline uint64_t stream_at(uint64_t state, uint64_t i) {
  return mix64(state + (i + 1) * kGamma);
}

// Uniform in (0, 1].
inline double unit_open0(uint64_t z) {
  return static_cast<double>((z >> 11) + 1) * (1.0 / 9007199254740992.0);
}

constexpr double kTwoPi = 6.283185307179586476925286766559;

inline double normal_at(uint64_t state, uint64_t i) {
  uint64_t pair = i >> 1;
  double u1 = unit_open0(stream_at(state, 2 * pair));
  double u2 = unit_open0(stream_at(state, 2 * pair + 1));
  double r = std::sqrt(-2.0 * std::log(u1));
  double t = kTwoPi * u2;
  return (i & 1) ? r * std::sin(t) : r * std::cos(t);
}

// ---------------------------------------------------------------------------
// Attention. Reference semantics: attention_reference_f16
// (transformer.metal:1579-1612): scale = rsqrt(head_dim), two passes (max,
// then exp-sum and P.V), FP32 throughout, output rounded once.
// ---------------------------------------------------------------------------
void attention_reference(const uint16_t* q, const uint16_t* k,
                         const uint16_t* v, size_t tokens, size_t qh,
                         size_t kvh, size_t hd, size_t kv_length, int causal,
                         size_t offset, uint16_t* out) {
  size_t group = qh / kvh;
  float scale = 1.0f / std::sqrt(static_cast<float>(hd));
#pragma omp parallel for collapse(2) schedule(static)
  for (long long qi = 0; qi < static_cast<long long>(tokens); ++qi) {
    for (long long head = 0; head < static_cast<long long>(qh); ++head) {
      size_t kv = static_cast<size_t>(head) / group;
      size_t available =
          causal ? std::min(kv_length, offset + static_cast<size_t>(qi) + 1)
                 : kv_length;
      std::vector<float> qf(hd), kf(hd), scores(available), num(hd, 0.0f);
      widen(q + (qi * qh + head) * hd, qf.data(), hd);
      float maximum = -std::numeric_limits<float>::infinity();
      for (size_t j = 0; j < available; ++j) {
        widen(k + (j * kvh + kv) * hd, kf.data(), hd);
        scores[j] = dot_f32(qf.data(), kf.data(), hd) * scale;
        maximum = std::max(maximum, scores[j]);
      }
      float denominator = 0.0f;
      for (size_t j = 0; j < available; ++j) {
        float p = std::exp(scores[j] - maximum);
        denominator += p;
        const uint16_t* vr = v + (j * kvh + kv) * hd;
        for (size_t d = 0; d < hd; ++d) num[d] += p * f(vr[d]);
      }
      uint16_t* o = out + (qi * qh + head) * hd;
      for (size_t d = 0; d < hd; ++d) o[d] = h(num[d] / denominator);
    }
  }
}

// Flash-prefill semantics (transformer.metal:1669-1822): keys in blocks of
// 32; per block the running max is updated from the available keys, the
// weights exp(s - max) are summed unrounded into the row sum, and rounded to
// FP16 before they multiply V; the accumulator is rescaled by
// alpha = exp(old_max - new_max) (0 while the old max is -inf).
void attention_flash_prefill(const uint16_t* q, const uint16_t* k,
                             const uint16_t* v, size_t tokens, size_t qh,
                             size_t kvh, size_t hd, size_t kv_length,
                             int causal, size_t offset, uint16_t* out) {
  constexpr size_t tile = 32;
  size_t group = qh / kvh;
  float scale = 1.0f / std::sqrt(static_cast<float>(hd));
#pragma omp parallel for collapse(2) schedule(static)
  for (long long qi = 0; qi < static_cast<long long>(tokens); ++qi) {
    for (long long head = 0; head < static_cast<long long>(qh); ++head) {
      size_t kv = static_cast<size_t>(head) / group;
      size_t available =
          causal ? std::min(kv_length, offset + static_cast<size_t>(qi) + 1)
                 : kv_length;
      std::vector<float> qf(hd), kf(hd), acc(hd, 0.0f);
      widen(q + (qi * qh + head) * hd, qf.data(), hd);
      float row_max = -std::numeric_limits<float>::infinity();
      float row_sum = 0.0f;
      float scores[tile];
      for (size_t base = 0; base < available; base += tile) {
        size_t count = std::min(tile, available - base);
        float block_max = -std::numeric_limits<float>::infinity();
        for (size_t c = 0; c < count; ++c) {
          widen(k + ((base + c) * kvh + kv) * hd, kf.data(), hd);
          scores[c] = dot_f32(qf.data(), kf.data(), hd) * scale;
          block_max = std::max(block_max, scores[c]);
        }
        float next_max = std::max(row_max, block_max);
        float alpha = std::isinf(row_max) ? 0.0f : std::exp(row_max - next_max);
        float block_sum = 0.0f;
        for (size_t d = 0; d < hd; ++d) acc[d] *= alpha;
        for (size_t c = 0; c < count; ++c) {
          float weight = std::exp(scores[c] - next_max);
          block_sum += weight;
          float p = f(h(weight));
          const uint16_t* vr = v + ((base + c) * kvh + kv) * hd;
          for (size_t d = 0; d < hd; ++d) acc[d] += p * f(vr[d]);
        }
        row_sum = row_sum * alpha + block_sum;
        row_max = next_max;
      }
      uint16_t* o = out + (qi * qh + head) * hd;
      for (size_t d = 0; d < hd; ++d) o[d] = h(acc[d] / row_sum);
    }
  }
}

// Fused per-head RMSNorm + RoPE (transformer.metal:1533-1577) on one row;
// with round_norm the normalized row is rounded to FP16 first, which is the
// unfused rms_norm -> rope path (transformer.metal:1318-1340, 1514-1531).
void norm_rope_row(const uint16_t* in, const uint16_t* w, size_t hd,
                   size_t position, float theta, float eps, bool apply_norm,
                   bool round_norm, uint16_t* out) {
  std::vector<float> xf(hd), normed(hd);
  widen(in, xf.data(), hd);
  if (apply_norm) {
    float scale = rms_scale(sum_squares(xf.data(), hd), hd, eps);
    for (size_t i = 0; i < hd; ++i) {
      float val = xf[i] * scale * f(w[i]);
      normed[i] = round_norm ? f(h(val)) : val;
    }
  } else {
    normed = xf;
  }
  size_t half_dim = hd / 2;
  for (size_t pair = 0; pair < half_dim; ++pair) {
    float x = normed[pair];
    float y = normed[pair + half_dim];
    float frequency = std::pow(theta, -static_cast<float>(pair * 2) /
                                          static_cast<float>(hd));
    float angle = static_cast<float>(position) * frequency;
    float c = std::cos(angle), s = std::sin(angle);
    out[pair] = h(x * c - y * s);
    out[pair + half_dim] = h(x * s + y * c);
  }
}

}  // namespace

// ===========================================================================
// C API
// ===========================================================================
extern "C" {

void or_f16_from_f32(const float* in, uint16_t* out, size_t n) {
  for (size_t i = 0; i < n; ++i) out[i] = h(in[i]);
}

void or_f32_from_f16(const uint16_t* in, float* out, size_t n) {
  widen(in, out, n);
}

void or_set_accumulate_f64(int enabled) { g_acc_f64 = enabled != 0; }

int or_num_threads(void) { return omp_get_max_threads(); }

void or_gen_normal_f16(uint64_t seed, uint64_t stream, uint64_t offset,
                       size_t n, double std_dev, uint16_t* out) {
  uint64_t state = stream_state(seed, stream);
#pragma omp parallel for schedule(static)
  for (long long i = 0; i < static_cast<long long>(n); ++i)
    out[i] = f64_to_f16(std_dev * normal_at(state, offset + i));
}

void or_gen_tokens(uint64_t seed, uint64_t stream, size_t n, uint32_t vocab,
                   uint32_t* out) {
  uint64_t state = stream_state(seed, stream);
  for (size_t i = 0; i < n; ++i) {
    uint64_t z = stream_at(state, i);
    out[i] = static_cast<uint32_t>(((z >> 32) * vocab) >> 32);
  }
}

void or_matmul(const uint16_t* x, size_t m, size_t k, const uint16_t* w,
               size_t n, uint16_t* out) {
  std::vector<float> xf(m * k);
  widen(x, xf.data(), m * k);
  matmul_xf(xf.data(), m, k, w, n, out);
}

void or_add(const uint16_t* a, const uint16_t* b, size_t n, uint16_t* out) {
  for (size_t i = 0; i < n; ++i)
    out[i] = f64_to_f16(static_cast<double>(f(a[i])) + f(b[i]));
}

void or_rms_norm(const uint16_t* x, size_t rows, size_t width,
                 const uint16_t* w, float eps, uint16_t* out) {
#pragma omp parallel for schedule(static)
  for (long long r = 0; r < static_cast<long long>(rows); ++r) {
    std::vector<float> xf(width);
    widen(x + r * width, xf.data(), width);
    float scale = rms_scale(sum_squares(xf.data(), width), width, eps);
    for (size_t i = 0; i < width; ++i)
      out[r * width + i] = h(xf[i] * scale * f(w[i]));
  }
}

void or_add_rms_norm(const uint16_t* left, const uint16_t* right, size_t rows,
                     size_t width, const uint16_t* w, float eps,
                     uint16_t* residual, uint16_t* normalized) {
#pragma omp parallel for schedule(static)
  for (long long r = 0; r < static_cast<long long>(rows); ++r) {
    std::vector<float> sum(width);
    size_t base = r * width;
    for (size_t i = 0; i < width; ++i) {
      sum[i] = f(left[base + i]) + f(right[base + i]);
      residual[base + i] = h(sum[i]);
    }
    float scale = rms_scale(sum_squares(sum.data(), width), width, eps);
    for (size_t i = 0; i < width; ++i)
      normalized[base + i] = h(f(residual[base + i]) * scale * f(w[i]));
  }
}

void or_rms_norm_matmul3(const uint16_t* x, size_t k, const uint16_t* norm_w,
                         const uint16_t* w0, size_t n0, const uint16_t* w1,
                         size_t n1, const uint16_t* w2, size_t n2, float eps,
                         uint16_t* out0, uint16_t* out1, uint16_t* out2) {
  std::vector<uint16_t> normalized(k);
  or_rms_norm(x, 1, k, norm_w, eps, normalized.data());
  or_matmul(normalized.data(), 1, k, w0, n0, out0);
  or_matmul(normalized.data(), 1, k, w1, n1, out1);
  or_matmul(normalized.data(), 1, k, w2, n2, out2);
}

void or_add_rms_norm_matmul2(const uint16_t* left, const uint16_t* right,
                             size_t k, const uint16_t* norm_w,
                             const uint16_t* w0, size_t n0, const uint16_t* w1,
                             size_t n1, float eps, uint16_t* residual,
                             uint16_t* out0, uint16_t* out1) {
  std::vector<uint16_t> normalized(k);
  or_add_rms_norm(left, right, 1, k, norm_w, eps, residual, normalized.data());
  or_matmul(normalized.data(), 1, k, w0, n0, out0);
  or_matmul(normalized.data(), 1, k, w1, n1, out1);
}

void or_swiglu(const uint16_t* gate, const uint16_t* up, size_t n,
               uint16_t* out) {
  for (size_t i = 0; i < n; ++i) {
    float x = f(gate[i]);
    out[i] = h((x / (1.0f + std::exp(-x))) * f(up[i]));
  }
}

void or_embedding(const uint32_t* tokens, size_t count, const uint16_t* table,
                  size_t rows, size_t width, uint16_t* out) {
  for (size_t t = 0; t < count; ++t) {
    if (tokens[t] == 0xFFFFFFFFu || tokens[t] >= rows) {
      std::memset(out + t * width, 0, width * sizeof(uint16_t));
    } else {
      std::memcpy(out + t * width, table + static_cast<size_t>(tokens[t]) * width,
                  width * sizeof(uint16_t));
    }
  }
}

// Greedy argmax of argmax_f16_partial/_reduce (transformer.metal:1396-1512):
// non-finite values are skipped; values compare by the sign-flipped bit key
// (so -0 < +0); equal keys go to the larger index.
uint32_t or_argmax(const uint16_t* logits, size_t n) {
  uint32_t best_index = 0xFFFFFFFFu;
  uint32_t best_key = 0;
  for (size_t i = 0; i < n; ++i) {
    float value = f(logits[i]);
    if (!std::isfinite(value)) continue;
    uint32_t b;
    std::memcpy(&b, &value, 4);
    uint32_t key = (b & 0x80000000u) ? ~b : (b ^ 0x80000000u);
    if (best_index == 0xFFFFFFFFu || key >= best_key) {
      best_key = key;
      best_index = static_cast<uint32_t>(i);
    }
  }
  return best_index;
}

void or_rope(const uint16_t* in, size_t tokens, size_t heads, size_t head_dim,
             size_t offset, float theta, uint16_t* out) {
  for (size_t t = 0; t < tokens; ++t)
    for (size_t hh = 0; hh < heads; ++hh) {
      size_t base = (t * heads + hh) * head_dim;
      norm_rope_row(in + base, nullptr, head_dim, t + offset, theta, 0.0f,
                    false, false, out + base);
    }
}

void or_qk_norm_rope_cache(const uint16_t* q, const uint16_t* k, size_t tokens,
                           size_t q_heads, size_t kv_heads, size_t head_dim,
                           const uint16_t* q_w, const uint16_t* k_w,
                           size_t offset, float theta, float eps,
                           size_t cache_capacity, uint16_t* q_out,
                           uint16_t* key_cache) {
  (void)cache_capacity;
  for (size_t t = 0; t < tokens; ++t) {
    for (size_t hh = 0; hh < q_heads; ++hh) {
      size_t base = (t * q_heads + hh) * head_dim;
      norm_rope_row(q + base, q_w, head_dim, t + offset, theta, eps, true,
                    false, q_out + base);
    }
    for (size_t hh = 0; hh < kv_heads; ++hh) {
      size_t base = (t * kv_heads + hh) * head_dim;
      size_t cache_base = ((offset + t) * kv_heads + hh) * head_dim;
      norm_rope_row(k + base, k_w, head_dim, t + offset, theta, eps, true,
                    false, key_cache + cache_base);
    }
  }
}

void or_copy_into_cache(const uint16_t* src, size_t tokens, size_t stride,
                        size_t offset, uint16_t* cache) {
  std::memcpy(cache + offset * stride, src, tokens * stride * sizeof(uint16_t));
}

void or_attention(const uint16_t* q, const uint16_t* k, const uint16_t* v,
                  size_t tokens, size_t q_heads, size_t kv_heads,
                  size_t head_dim, size_t kv_length, int causal,
                  size_t query_offset, int semantics, uint16_t* out) {
  if (semantics == OR_ATTN_FLASH_PREFILL)
    attention_flash_prefill(q, k, v, tokens, q_heads, kv_heads, head_dim,
                            kv_length, causal, query_offset, out);
  else
    attention_reference(q, k, v, tokens, q_heads, kv_heads, head_dim,
                        kv_length, causal, query_offset, out);
}

// ===========================================================================
// Qwen3 model. Weight roles and their generator streams: a tensor of layer l
// with role r uses stream (l + 1) * 16 + r; model-level tensors use layer -1
// (embedding: stream 0, lm_head: stream 13). Matrices are N(0, std); norm
// gains are 1.0.
// ===========================================================================
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

}  // extern "C"

struct or_qwen3 {
  or_qwen3_config c;
  std::vector<uint16_t> embedding, final_norm, lm_head;
  struct Layer {
    std::vector<uint16_t> w[16];
    std::vector<uint16_t> key_cache, value_cache;
  };
  std::vector<Layer> layers;
  size_t capacity = 0;
  size_t filled = 0;
  bool fuse_qk_rope_cache = true;
  bool fuse_add_rms_norm = true;
};

namespace {

std::vector<uint16_t> random_matrix(uint64_t seed, int layer, int role,
                                    size_t count, double std_dev) {
  std::vector<uint16_t> out(count);
  or_gen_normal_f16(seed, static_cast<uint64_t>((layer + 1) * 16 + role), 0,
                    count, std_dev, out.data());
  return out;
}

std::vector<uint16_t> ones(size_t n) { return std::vector<uint16_t>(n, 0x3c00); }

// One transformer layer on hidden [T, h] (qwen3.rs:647-796), fusion options
// RECOMMENDED (= ALL) unless changed.
void layer_forward(or_qwen3* m, or_qwen3::Layer& L, std::vector<uint16_t>& hidden,
                   size_t T, size_t offset) {
  const auto& c = m->c;
  size_t hs = c.hidden_size, hd = c.head_dim, qh = c.num_attention_heads,
         kvh = c.num_key_value_heads, I = c.intermediate_size;
  size_t qw = qh * hd, kw = kvh * hd;
  float eps = c.rms_norm_eps;
  std::vector<uint16_t> normalized(T * hs), q(T * qw), k(T * kw), v(T * kw);
  or_rms_norm(hidden.data(), T, hs, L.w[kInputNorm].data(), eps,
              normalized.data());
  {
    std::vector<float> xf(T * hs);
    widen(normalized.data(), xf.data(), T * hs);
    matmul_xf(xf.data(), T, hs, L.w[kQ].data(), qw, q.data());
    matmul_xf(xf.data(), T, hs, L.w[kK].data(), kw, k.data());
    matmul_xf(xf.data(), T, hs, L.w[kV].data(), kw, v.data());
  }
  std::vector<uint16_t> query(T * qw);
  if (m->fuse_qk_rope_cache) {
    or_qk_norm_rope_cache(q.data(), k.data(), T, qh, kvh, hd,
                          L.w[kQNorm].data(), L.w[kKNorm].data(), offset,
                          c.rope_theta, eps, m->capacity, query.data(),
                          L.key_cache.data());
  } else {
    for (size_t t = 0; t < T; ++t) {
      for (size_t hh = 0; hh < qh; ++hh) {
        size_t base = (t * qh + hh) * hd;
        norm_rope_row(q.data() + base, L.w[kQNorm].data(), hd, t + offset,
                      c.rope_theta, eps, true, true, query.data() + base);
      }
      for (size_t hh = 0; hh < kvh; ++hh) {
        size_t base = (t * kvh + hh) * hd;
        norm_rope_row(k.data() + base, L.w[kKNorm].data(), hd, t + offset,
                      c.rope_theta, eps, true, true,
                      L.key_cache.data() + ((offset + t) * kvh + hh) * hd);
      }
    }
  }
  or_copy_into_cache(v.data(), T, kw, offset, L.value_cache.data());
  size_t active = offset + T;
  std::vector<uint16_t> attn(T * qw);
  // attention_kind_for_tokens (qwen3.rs:799-822): FlashPrefill for T >= 32,
  // otherwise tiled / split-KV / flash-decode, all FP32-softmax semantics.
  or_attention(query.data(), L.key_cache.data(), L.value_cache.data(), T, qh,
               kvh, hd, active, 1, offset,
               T >= 32 ? OR_ATTN_FLASH_PREFILL : OR_ATTN_REFERENCE,
               attn.data());
  std::vector<uint16_t> attn_o(T * hs);
  or_matmul(attn.data(), T, qw, L.w[kO].data(), hs, attn_o.data());
  std::vector<uint16_t> residual(T * hs);
  if (m->fuse_add_rms_norm) {
    or_add_rms_norm(hidden.data(), attn_o.data(), T, hs,
                    L.w[kPostNorm].data(), eps, residual.data(),
                    normalized.data());
  } else {
    or_add(hidden.data(), attn_o.data(), T * hs, residual.data());
    or_rms_norm(residual.data(), T, hs, L.w[kPostNorm].data(), eps,
                normalized.data());
  }
  std::vector<uint16_t> gate(T * I), up(T * I), act(T * I);
  {
    std::vector<float> xf(T * hs);
    widen(normalized.data(), xf.data(), T * hs);
    matmul_xf(xf.data(), T, hs, L.w[kGate].data(), I, gate.data());
    matmul_xf(xf.data(), T, hs, L.w[kUp].data(), I, up.data());
  }
  or_swiglu(gate.data(), up.data(), T * I, act.data());
  std::vector<uint16_t> down(T * hs);
  or_matmul(act.data(), T, I, L.w[kDown].data(), hs, down.data());
  or_add(residual.data(), down.data(), T * hs, hidden.data());
}

}  // namespace

extern "C" {

or_qwen3* or_qwen3_create_random(const or_qwen3_config* cfg, uint64_t seed,
                                 double std_dev, size_t cache_capacity) {
  auto* m = new or_qwen3();
  m->c = *cfg;
  const auto& c = m->c;
  size_t hs = c.hidden_size, hd = c.head_dim, qw = c.num_attention_heads * hd,
         kw = c.num_key_value_heads * hd, I = c.intermediate_size,
         V = c.vocab_size;
  m->embedding = random_matrix(seed, -1, kEmbedding, V * hs, std_dev);
  m->final_norm = ones(hs);
  if (!c.tie_word_embeddings)
    m->lm_head = random_matrix(seed, -1, kLmHead, V * hs, std_dev);
  m->layers.resize(c.num_hidden_layers);
  for (uint32_t l = 0; l < c.num_hidden_layers; ++l) {
    auto& L = m->layers[l];
    int li = static_cast<int>(l);
    L.w[kQ] = random_matrix(seed, li, kQ, qw * hs, std_dev);
    L.w[kK] = random_matrix(seed, li, kK, kw * hs, std_dev);
    L.w[kV] = random_matrix(seed, li, kV, kw * hs, std_dev);
    L.w[kO] = random_matrix(seed, li, kO, hs * qw, std_dev);
    L.w[kQNorm] = ones(hd);
    L.w[kKNorm] = ones(hd);
    L.w[kGate] = random_matrix(seed, li, kGate, I * hs, std_dev);
    L.w[kUp] = random_matrix(seed, li, kUp, I * hs, std_dev);
    L.w[kDown] = random_matrix(seed, li, kDown, hs * I, std_dev);
    L.w[kInputNorm] = ones(hs);
    L.w[kPostNorm] = ones(hs);
    L.key_cache.assign(cache_capacity * kw, 0);
    L.value_cache.assign(cache_capacity * kw, 0);
  }
  m->capacity = cache_capacity;
  return m;
}

void or_qwen3_destroy(or_qwen3* m) { delete m; }

void or_qwen3_set_fusion(or_qwen3* m, int qk_rope_cache, int add_rms_norm) {
  m->fuse_qk_rope_cache = qk_rope_cache != 0;
  m->fuse_add_rms_norm = add_rms_norm != 0;
}

void or_qwen3_reset(or_qwen3* m) { m->filled = 0; }

size_t or_qwen3_len(const or_qwen3* m) { return m->filled; }

int or_qwen3_forward_hidden(or_qwen3* m, const uint16_t* hidden, size_t count,
                            uint16_t* out_hidden) {
  if (count == 0 || m->filled + count > m->capacity) return -1;
  std::vector<uint16_t> x(hidden, hidden + count * m->c.hidden_size);
  for (auto& L : m->layers) layer_forward(m, L, x, count, m->filled);
  m->filled += count;
  std::memcpy(out_hidden, x.data(), x.size() * sizeof(uint16_t));
  return 0;
}

int or_qwen3_forward(or_qwen3* m, const uint32_t* tokens, size_t count,
                     uint16_t* logits) {
  const auto& c = m->c;
  if (count == 0 || m->filled + count > m->capacity) return -1;
  size_t hs = c.hidden_size;
  std::vector<uint16_t> x(count * hs);
  or_embedding(tokens, count, m->embedding.data(), c.vocab_size, hs, x.data());
  for (auto& L : m->layers) layer_forward(m, L, x, count, m->filled);
  m->filled += count;
  // Final norm over every row, then the last row through the LM head
  // (qwen3.rs:636-638).
  std::vector<uint16_t> normalized(count * hs);
  or_rms_norm(x.data(), count, hs, m->final_norm.data(), c.rms_norm_eps,
              normalized.data());
  const uint16_t* head =
      c.tie_word_embeddings ? m->embedding.data() : m->lm_head.data();
  or_matmul(normalized.data() + (count - 1) * hs, 1, hs, head, c.vocab_size,
            logits);
  return 0;
}

size_t or_qwen3_generate_greedy(or_qwen3* m, const uint32_t* prompt,
                                size_t prompt_len, size_t max_tokens,
                                uint32_t* out_ids) {
  if (max_tokens == 0) return 0;
  std::vector<uint16_t> logits(m->c.vocab_size);
  m->filled = 0;
  if (or_qwen3_forward(m, prompt, prompt_len, logits.data()) != 0) return 0;
  size_t produced = 0;
  uint32_t token = or_argmax(logits.data(), logits.size());
  for (size_t step = 0; step < max_tokens; ++step) {
    if (token == 0xFFFFFFFFu) break;
    out_ids[produced++] = token;
    if (step + 1 == max_tokens) break;
    if (or_qwen3_forward(m, &token, 1, logits.data()) != 0) break;
    token = or_argmax(logits.data(), logits.size());
  }
  return produced;
}

const uint16_t* or_qwen3_weight(const or_qwen3* m, int layer, int role) {
  if (layer < 0) {
    if (role == kEmbedding) return m->embedding.data();
    if (role == kFinalNorm) return m->final_norm.data();
    if (role == kLmHead)
      return m->c.tie_word_embeddings ? m->embedding.data() : m->lm_head.data();
    return nullptr;
  }
  if (static_cast<size_t>(layer) >= m->layers.size() || role < 0 || role >= 16)
    return nullptr;
  return m->layers[layer].w[role].data();
}

const uint16_t* or_qwen3_cache(const or_qwen3* m, int layer, int value) {
  if (layer < 0 || static_cast<size_t>(layer) >= m->layers.size()) return nullptr;
  return value ? m->layers[layer].value_cache.data()
               : m->layers[layer].key_cache.data();
}

}  // extern "C"
