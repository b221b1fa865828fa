// CPU oracle for the Qwen3 hot path of stratorys/metal-infer-rs.
//
// TEST INFRASTRUCTURE ONLY: the engine never links or calls this file. It is
// the checker for the CUDA kernels and the timed CPU baseline.
//
// Each function restates one reference kernel of
// crates/metal-infer-core/src/kernels/transformer.metal (cited per function)
// with the same FP16 rounding points. Where the reference leaves the
// arithmetic to the hardware, the oracle fixes it as follows (the CUDA engine
// follows the same definitions, so the decode path is bit-exact):
//
//  * Reductions (simd_sum in the reference). DOT(x, y, n): the n elements
//    form chunks of 8; chunk c belongs to lane c mod L with
//    L = min(32, next_pow2(ceil(n / 8))); each lane accumulates its chunks in
//    increasing order, 8 sequential fused multiply-adds per chunk, starting
//    from 0; the L lane sums are combined by a butterfly (step L/2, ..., 1:
//    v[l] = v[l] + v[l + step]). Sums of squares are DOT(x, x).
//  * exp: Cody-Waite reduction n = rint(x * log2 e), r = x - n ln2 (two
//    parts), e^r by the degree-7 Taylor polynomial in Horner form with fused
//    multiply-adds, scaled by 2^n (mi_exp below).
//  * rsqrt: correctly rounded 1 / sqrt.
//  * RoPE: frequency = float(pow(theta, -2i / d)) and cos / sin of the FP32
//    angle evaluated in double precision, each rounded once to FP32.
//  * Decode attention (flash decode, transformer.metal:2127-2316): keys in
//    blocks of B; inside a block, keys are dealt round-robin to S streams;
//    each stream keeps an online-softmax state; streams then blocks are
//    merged by log-sum-exp in index order.
//  * Prefill attention (transformer.metal:1614-1822): per query, keys in
//    blocks of 32 from 0; block sums by a 32-lane butterfly; probabilities
//    rounded to FP16 before weighting V for flash prefill (T >= 32).
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

inline uint16_t h(float v) { return f64_to_f16(static_cast<double>(v)); }

inline float f(uint16_t x) { return _cvtsh_ss(x); }

inline float fr(float v) { return f(h(v)); }  // round through FP16

void widen(const uint16_t* in, float* out, size_t n) {
  size_t i = 0;
  for (; i + 8 <= n; i += 8)
    _mm256_storeu_ps(out + i, _mm256_cvtph_ps(_mm_loadu_si128(
                                  reinterpret_cast<const __m128i*>(in + i))));
  for (; i < n; ++i) out[i] = f(in[i]);
}

bool g_acc_f64 = false;

// ---------------------------------------------------------------------------
// exp: Cody-Waite range reduction and a degree-7 Taylor polynomial.
// ---------------------------------------------------------------------------
inline float pow2i(int e) {  // 2^e for e in [-126, 127]
  uint32_t b = static_cast<uint32_t>(e + 127) << 23;
  float r;
  std::memcpy(&r, &b, 4);
  return r;
}

float mi_exp(float x) {
  if (x != x) return x;
  if (x > 89.0f) return std::numeric_limits<float>::infinity();
  if (x < -104.0f) return 0.0f;
  const float kLog2e = 0x1.715476p+0f;
  const float kLn2Hi = 0x1.62e4p-1f;
  const float kLn2Lo = 0x1.7f7d1cp-20f;
  float n = std::nearbyint(x * kLog2e);
  float r = std::fma(n, -kLn2Hi, x);
  r = std::fma(n, -kLn2Lo, r);
  float p = 0x1.a01a02p-13f;           // 1/5040
  p = std::fma(p, r, 0x1.6c16c2p-10f);  // 1/720
  p = std::fma(p, r, 0x1.111112p-7f);   // 1/120
  p = std::fma(p, r, 0x1.555556p-5f);   // 1/24
  p = std::fma(p, r, 0x1.555556p-3f);   // 1/6
  p = std::fma(p, r, 0.5f);
  p = std::fma(p, r, 1.0f);
  p = std::fma(p, r, 1.0f);
  int ni = static_cast<int>(n);
  if (ni < -126) return (p * pow2i(ni + 64)) * pow2i(-64);
  if (ni > 127) return (p * pow2i(127)) * 2.0f;
  return p * pow2i(ni);
}

// ---------------------------------------------------------------------------
// Canonical reductions.
// ---------------------------------------------------------------------------
inline size_t lanes_for(size_t n) {
  size_t chunks = (n + 7) / 8;
  size_t l = 1;
  while (l < chunks && l < 32) l <<= 1;
  return l;
}

inline float butterfly(float* v, size_t lanes) {
  for (size_t step = lanes / 2; step >= 1; step /= 2)
    for (size_t l = 0; l < step; ++l) v[l] = v[l] + v[l + step];
  return v[0];
}

// Scalar canonical DOT of two FP32 vectors.
float dot_canon(const float* x, const float* y, size_t n) {
  if (g_acc_f64) {
    double s = 0.0;
    for (size_t i = 0; i < n; ++i) s += static_cast<double>(x[i]) * y[i];
    return static_cast<float>(s);
  }
  size_t lanes = lanes_for(n);
  float v[32] = {0};
  size_t chunks = (n + 7) / 8;
  for (size_t c = 0; c < chunks; ++c) {
    float& acc = v[c % lanes];
    size_t end = std::min(n, 8 * c + 8);
    for (size_t i = 8 * c; i < end; ++i) acc = std::fma(x[i], y[i], acc);
  }
  return butterfly(v, lanes);
}

// x pre-arranged for the vector path: for round i (32 chunks) and element j,
// the 32 lanes' values are contiguous: xt[(i * 8 + j) * 32 + lane].
void transpose_lanes(const float* x, size_t n, float* xt) {
  size_t rounds = n / 256;
  for (size_t i = 0; i < rounds; ++i)
    for (size_t lane = 0; lane < 32; ++lane)
      for (size_t j = 0; j < 8; ++j) xt[(i * 8 + j) * 32 + lane] = x[(i * 32 + lane) * 8 + j];
}

// Canonical DOT of a transposed FP32 vector with an FP16 row, n % 256 == 0.
float dot_canon_t(const float* xt, const uint16_t* w, size_t n) {
  __m256 acc[4] = {_mm256_setzero_ps(), _mm256_setzero_ps(), _mm256_setzero_ps(),
                   _mm256_setzero_ps()};
  size_t rounds = n / 256;
  for (size_t i = 0; i < rounds; ++i) {
    for (int g = 0; g < 4; ++g) {
      // chunks of lanes 8g .. 8g + 7 of this round
      const uint16_t* base = w + (i * 32 + 8 * g) * 8;
      __m256 r[8];
      for (int c = 0; c < 8; ++c)
        r[c] = _mm256_cvtph_ps(_mm_loadu_si128(reinterpret_cast<const __m128i*>(base + 8 * c)));
      // 8x8 transpose: t[j] = element j of the 8 chunks
      __m256 t0 = _mm256_unpacklo_ps(r[0], r[1]), t1 = _mm256_unpackhi_ps(r[0], r[1]);
      __m256 t2 = _mm256_unpacklo_ps(r[2], r[3]), t3 = _mm256_unpackhi_ps(r[2], r[3]);
      __m256 t4 = _mm256_unpacklo_ps(r[4], r[5]), t5 = _mm256_unpackhi_ps(r[4], r[5]);
      __m256 t6 = _mm256_unpacklo_ps(r[6], r[7]), t7 = _mm256_unpackhi_ps(r[6], r[7]);
      __m256 s0 = _mm256_shuffle_ps(t0, t2, 0x44), s1 = _mm256_shuffle_ps(t0, t2, 0xEE);
      __m256 s2 = _mm256_shuffle_ps(t1, t3, 0x44), s3 = _mm256_shuffle_ps(t1, t3, 0xEE);
      __m256 s4 = _mm256_shuffle_ps(t4, t6, 0x44), s5 = _mm256_shuffle_ps(t4, t6, 0xEE);
      __m256 s6 = _mm256_shuffle_ps(t5, t7, 0x44), s7 = _mm256_shuffle_ps(t5, t7, 0xEE);
      __m256 e[8];
      e[0] = _mm256_permute2f128_ps(s0, s4, 0x20);
      e[1] = _mm256_permute2f128_ps(s1, s5, 0x20);
      e[2] = _mm256_permute2f128_ps(s2, s6, 0x20);
      e[3] = _mm256_permute2f128_ps(s3, s7, 0x20);
      e[4] = _mm256_permute2f128_ps(s0, s4, 0x31);
      e[5] = _mm256_permute2f128_ps(s1, s5, 0x31);
      e[6] = _mm256_permute2f128_ps(s2, s6, 0x31);
      e[7] = _mm256_permute2f128_ps(s3, s7, 0x31);
      const float* xr = xt + (i * 8) * 32 + 8 * g;
      for (int j = 0; j < 8; ++j)
        acc[g] = _mm256_fmadd_ps(_mm256_loadu_ps(xr + j * 32), e[j], acc[g]);
    }
  }
  alignas(32) float v[32];
  for (int g = 0; g < 4; ++g) _mm256_store_ps(v + 8 * g, acc[g]);
  return butterfly(v, 32);
}

// DOT of an FP32 input with an FP16 weight row (canonical order).
struct RowDot {
  size_t n;
  std::vector<float> x, xt;
  bool fast;
  RowDot(const float* in, size_t k) : n(k), x(in, in + k), fast(k % 256 == 0 && !g_acc_f64) {
    if (fast) {
      xt.resize(k);
      transpose_lanes(x.data(), k, xt.data());
    }
  }
  float operator()(const uint16_t* w) const {
    if (fast) return dot_canon_t(xt.data(), w, n);
    std::vector<float> wf(n);
    widen(w, wf.data(), n);
    return dot_canon(x.data(), wf.data(), n);
  }
};

float sum_squares(const float* x, size_t n) { return dot_canon(x, x, n); }

// rsqrt(total / width + eps) of the reference, as a correctly rounded
// reciprocal of a correctly rounded square root.
inline float rms_scale(float total, size_t width, float eps) {
  return 1.0f / std::sqrt(total / static_cast<float>(width) + eps);
}

// out[m, n] = half(DOT(x[m], w[n])), x already widened ([m, k]).
void matmul_xf(const float* xf, size_t m, size_t k, const uint16_t* w, size_t n, uint16_t* out) {
  std::vector<RowDot> rows;
  rows.reserve(m);
  for (size_t r = 0; r < m; ++r) rows.emplace_back(xf + r * k, k);
#pragma omp parallel for schedule(static)
  for (long long row = 0; row < static_cast<long long>(n); ++row) {
    const uint16_t* wr = w + static_cast<size_t>(row) * k;
    for (size_t r = 0; r < m; ++r) out[r * n + row] = h(rows[r](wr));
  }
}

// ---------------------------------------------------------------------------
// RoPE angle terms (double-precision trig of the FP32 angle).
// ---------------------------------------------------------------------------
inline void rope_cs(size_t position, size_t pair, size_t hd, float theta, float* c, float* s) {
  float exponent = -static_cast<float>(pair * 2) / static_cast<float>(hd);
  float frequency = static_cast<float>(std::pow(static_cast<double>(theta),
                                                static_cast<double>(exponent)));
  float angle = static_cast<float>(position) * frequency;
  *c = static_cast<float>(std::cos(static_cast<double>(angle)));
  *s = static_cast<float>(std::sin(static_cast<double>(angle)));
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

inline uint64_t stream_at(uint64_t state, uint64_t i) { return mix64(state + (i + 1) * kGamma); }

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
// Attention.
// ---------------------------------------------------------------------------
inline float attn_scale(size_t hd) { return 1.0f / std::sqrt(static_cast<float>(hd)); }

// attention_reference_f16 (transformer.metal:1579-1612): two passes (max,
// then exp-sum and P.V), FP32 throughout, output rounded once.
void attention_reference(const uint16_t* q, const uint16_t* k, const uint16_t* v, size_t tokens,
                         size_t qh, size_t kvh, size_t hd, size_t kv_length, int causal,
                         size_t offset, uint16_t* out) {
  size_t group = qh / kvh;
  float scale = attn_scale(hd);
#pragma omp parallel for collapse(2) schedule(static)
  for (long long qi = 0; qi < static_cast<long long>(tokens); ++qi) {
    for (long long head = 0; head < static_cast<long long>(qh); ++head) {
      size_t kv = static_cast<size_t>(head) / group;
      size_t available =
          causal ? std::min(kv_length, offset + static_cast<size_t>(qi) + 1) : kv_length;
      std::vector<float> qf(hd), kf(hd), scores(available), num(hd, 0.0f);
      widen(q + (qi * qh + head) * hd, qf.data(), hd);
      float maximum = -std::numeric_limits<float>::infinity();
      for (size_t j = 0; j < available; ++j) {
        widen(k + (j * kvh + kv) * hd, kf.data(), hd);
        scores[j] = dot_canon(qf.data(), kf.data(), hd) * scale;
        maximum = std::max(maximum, scores[j]);
      }
      float denominator = 0.0f;
      for (size_t j = 0; j < available; ++j) {
        float p = mi_exp(scores[j] - maximum);
        denominator += p;
        const uint16_t* vr = v + (j * kvh + kv) * hd;
        for (size_t d = 0; d < hd; ++d) num[d] += p * f(vr[d]);
      }
      uint16_t* o = out + (qi * qh + head) * hd;
      for (size_t d = 0; d < hd; ++d) o[d] = h(num[d] / denominator);
    }
  }
}

// Prefill attention (attention_tiled_f16 / attention_flash_prefill_f16,
// transformer.metal:1614-1822): keys in blocks of 32 from 0; the block max
// updates the running max; weights exp(s - max) are summed unrounded (32-lane
// butterfly) into the row sum and, with round_p, rounded to FP16 before they
// weight V; the accumulator is rescaled by alpha = exp(old - new) (0 while
// the old max is -inf).
void attention_prefill(const uint16_t* q, const uint16_t* k, const uint16_t* v, size_t tokens,
                       size_t qh, size_t kvh, size_t hd, size_t kv_length, int causal,
                       size_t offset, bool round_p, uint16_t* out) {
  constexpr size_t tile = 32;
  size_t group = qh / kvh;
  float scale = attn_scale(hd);
  const float ninf = -std::numeric_limits<float>::infinity();
#pragma omp parallel for collapse(2) schedule(static)
  for (long long qi = 0; qi < static_cast<long long>(tokens); ++qi) {
    for (long long head = 0; head < static_cast<long long>(qh); ++head) {
      size_t kv = static_cast<size_t>(head) / group;
      size_t available =
          causal ? std::min(kv_length, offset + static_cast<size_t>(qi) + 1) : kv_length;
      std::vector<float> qf(hd), kf(hd), acc(hd, 0.0f);
      widen(q + (qi * qh + head) * hd, qf.data(), hd);
      float row_max = ninf, row_sum = 0.0f;
      float s[tile], w[tile];
      for (size_t base = 0; base < available; base += tile) {
        size_t count = std::min(tile, available - base);
        float block_max = ninf;
        for (size_t c = 0; c < tile; ++c) {
          s[c] = ninf;
          if (c < count) {
            widen(k + ((base + c) * kvh + kv) * hd, kf.data(), hd);
            s[c] = dot_canon(qf.data(), kf.data(), hd) * scale;
          }
          block_max = std::max(block_max, s[c]);
        }
        float next_max = std::max(row_max, block_max);
        float alpha = std::isinf(row_max) ? 0.0f : mi_exp(row_max - next_max);
        for (size_t c = 0; c < tile; ++c) w[c] = c < count ? mi_exp(s[c] - next_max) : 0.0f;
        float tmp[tile];
        std::memcpy(tmp, w, sizeof tmp);
        float block_sum = butterfly(tmp, tile);
        row_sum = std::fma(row_sum, alpha, block_sum);
        row_max = next_max;
        for (size_t d = 0; d < hd; ++d) acc[d] *= alpha;
        for (size_t c = 0; c < count; ++c) {
          float p = round_p ? fr(w[c]) : w[c];
          const uint16_t* vr = v + ((base + c) * kvh + kv) * hd;
          for (size_t d = 0; d < hd; ++d) acc[d] = std::fma(p, f(vr[d]), acc[d]);
        }
      }
      uint16_t* o = out + (qi * qh + head) * hd;
      for (size_t d = 0; d < hd; ++d) o[d] = h(acc[d] / row_sum);
    }
  }
}

// Flash-decode attention for one query row (attention_flash_decode_*,
// transformer.metal:2127-2316): blocks of B keys; inside a block key j goes
// to stream (j - block start) mod S; per stream and head the online softmax
//   m' = max(m, s); a = exp(m - m'); c = exp(s - m');
//   acc = fma(acc, a, c * v); l = fma(l, a, c)
// then streams merge (index order) with f = exp(m_s - M) (0 for an empty
// stream): num = fma(acc_s, f, num), den = fma(l_s, f, den); blocks merge the
// same way; out = half(num / den).
struct SoftmaxState {
  float m, l;
  std::vector<float> acc;
};

void merge_states(const std::vector<SoftmaxState>& parts, size_t hd, SoftmaxState* out) {
  const float ninf = -std::numeric_limits<float>::infinity();
  float M = ninf;
  for (const auto& p : parts) M = std::max(M, p.m);
  out->m = M;
  out->l = 0.0f;
  out->acc.assign(hd, 0.0f);
  for (const auto& p : parts) {
    float fct = p.m == ninf ? 0.0f : mi_exp(p.m - M);
    out->l = std::fma(p.l, fct, out->l);
    for (size_t d = 0; d < hd; ++d) out->acc[d] = std::fma(p.acc[d], fct, out->acc[d]);
  }
}

void attention_decode(const uint16_t* q, const uint16_t* k, const uint16_t* v, size_t qh,
                      size_t kvh, size_t hd, size_t length, size_t block, size_t streams,
                      uint16_t* out) {
  size_t group = qh / kvh;
  float scale = attn_scale(hd);
  const float ninf = -std::numeric_limits<float>::infinity();
  size_t blocks = (length + block - 1) / block;
#pragma omp parallel for schedule(static)
  for (long long head = 0; head < static_cast<long long>(qh); ++head) {
    size_t kv = static_cast<size_t>(head) / group;
    std::vector<float> qf(hd), kf(hd);
    widen(q + head * hd, qf.data(), hd);
    std::vector<SoftmaxState> block_states(blocks);
    for (size_t b = 0; b < blocks; ++b) {
      std::vector<SoftmaxState> st(streams, SoftmaxState{ninf, 0.0f, std::vector<float>(hd, 0.0f)});
      size_t begin = b * block, end = std::min(length, begin + block);
      for (size_t j = begin; j < end; ++j) {
        SoftmaxState& S = st[(j - begin) % streams];
        widen(k + (j * kvh + kv) * hd, kf.data(), hd);
        float s = dot_canon(qf.data(), kf.data(), hd) * scale;
        float nm = std::max(S.m, s);
        float a = mi_exp(S.m - nm);
        float c = mi_exp(s - nm);
        const uint16_t* vr = v + (j * kvh + kv) * hd;
        for (size_t d = 0; d < hd; ++d) S.acc[d] = std::fma(S.acc[d], a, c * f(vr[d]));
        S.l = std::fma(S.l, a, c);
        S.m = nm;
      }
      merge_states(st, hd, &block_states[b]);
    }
    SoftmaxState total;
    merge_states(block_states, hd, &total);
    for (size_t d = 0; d < hd; ++d) out[head * hd + d] = h(total.acc[d] / total.l);
  }
}

// Fused per-head RMSNorm + RoPE (transformer.metal:1533-1577) on one row;
// with round_norm the normalized row is rounded to FP16 first, which is the
// unfused rms_norm -> rope path (transformer.metal:1318-1340, 1514-1531).
void norm_rope_row(const uint16_t* in, const uint16_t* w, size_t hd, size_t position,
                   float theta, float eps, bool apply_norm, bool round_norm, uint16_t* out) {
  std::vector<float> xf(hd), normed(hd);
  widen(in, xf.data(), hd);
  if (apply_norm) {
    float scale = rms_scale(sum_squares(xf.data(), hd), hd, eps);
    for (size_t i = 0; i < hd; ++i) {
      float val = xf[i] * scale * f(w[i]);
      normed[i] = round_norm ? fr(val) : val;
    }
  } else {
    normed = xf;
  }
  size_t half_dim = hd / 2;
  for (size_t pair = 0; pair < half_dim; ++pair) {
    float x = normed[pair];
    float y = normed[pair + half_dim];
    float c, s;
    rope_cs(position, pair, hd, theta, &c, &s);
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

void or_f32_from_f16(const uint16_t* in, float* out, size_t n) { widen(in, out, n); }

void or_set_accumulate_f64(int enabled) { g_acc_f64 = enabled != 0; }

int or_num_threads(void) { return omp_get_max_threads(); }

void or_exp(const float* in, float* out, size_t n) {
  for (size_t i = 0; i < n; ++i) out[i] = mi_exp(in[i]);
}

float or_dot(const float* x, const float* y, size_t n) { return dot_canon(x, y, n); }

void or_rope_cs(size_t position, size_t pair, size_t hd, float theta, float* c, float* s) {
  rope_cs(position, pair, hd, theta, c, s);
}

size_t or_decode_block(size_t capacity) {
  if (capacity <= 8192) return 64;
  size_t b = 64;
  while (b * 128 < capacity) b <<= 1;
  return b;
}

size_t or_decode_streams(size_t head_dim) { return 4 * (32 / lanes_for(head_dim)); }

void or_gen_normal_f16(uint64_t seed, uint64_t stream, uint64_t offset, size_t n, double std_dev,
                       uint16_t* out) {
  uint64_t state = stream_state(seed, stream);
#pragma omp parallel for schedule(static)
  for (long long i = 0; i < static_cast<long long>(n); ++i)
    out[i] = f64_to_f16(std_dev * normal_at(state, offset + i));
}

void or_gen_tokens(uint64_t seed, uint64_t stream, size_t n, uint32_t vocab, uint32_t* out) {
  uint64_t state = stream_state(seed, stream);
  for (size_t i = 0; i < n; ++i) {
    uint64_t z = stream_at(state, i);
    out[i] = static_cast<uint32_t>(((z >> 32) * vocab) >> 32);
  }
}

// matmul_f16 / matvec_* (transformer.metal:70-94, 274-347)
void or_matmul(const uint16_t* x, size_t m, size_t k, const uint16_t* w, size_t n,
               uint16_t* out) {
  std::vector<float> xf(m * k);
  widen(x, xf.data(), m * k);
  matmul_xf(xf.data(), m, k, w, n, out);
}

// add_f16 (transformer.metal:61-68): a correctly rounded half addition.
void or_add(const uint16_t* a, const uint16_t* b, size_t n, uint16_t* out) {
  for (size_t i = 0; i < n; ++i) out[i] = f64_to_f16(static_cast<double>(f(a[i])) + f(b[i]));
}

// rms_norm_f16 (transformer.metal:1318-1340)
void or_rms_norm(const uint16_t* x, size_t rows, size_t width, const uint16_t* w, float eps,
                 uint16_t* out) {
#pragma omp parallel for schedule(static)
  for (long long r = 0; r < static_cast<long long>(rows); ++r) {
    std::vector<float> xf(width);
    widen(x + r * width, xf.data(), width);
    float scale = rms_scale(sum_squares(xf.data(), width), width, eps);
    for (size_t i = 0; i < width; ++i) out[r * width + i] = h(xf[i] * scale * f(w[i]));
  }
}

// add_rms_norm_f16 (transformer.metal:1342-1369): residual = half(l + r);
// squares of the unrounded sums; normalized from the rounded residual.
void or_add_rms_norm(const uint16_t* left, const uint16_t* right, size_t rows, size_t width,
                     const uint16_t* w, float eps, uint16_t* residual, uint16_t* normalized) {
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

// matvec3_rms_impl (transformer.metal:937-1009)
void or_rms_norm_matmul3(const uint16_t* x, size_t k, const uint16_t* norm_w, const uint16_t* w0,
                         size_t n0, const uint16_t* w1, size_t n1, const uint16_t* w2, size_t n2,
                         float eps, uint16_t* out0, uint16_t* out1, uint16_t* out2) {
  std::vector<uint16_t> normalized(k);
  or_rms_norm(x, 1, k, norm_w, eps, normalized.data());
  or_matmul(normalized.data(), 1, k, w0, n0, out0);
  or_matmul(normalized.data(), 1, k, w1, n1, out1);
  or_matmul(normalized.data(), 1, k, w2, n2, out2);
}

// matvec2_add_rms_impl (transformer.metal:1091-1160)
void or_add_rms_norm_matmul2(const uint16_t* left, const uint16_t* right, size_t k,
                             const uint16_t* norm_w, const uint16_t* w0, size_t n0,
                             const uint16_t* w1, size_t n1, float eps, uint16_t* residual,
                             uint16_t* out0, uint16_t* out1) {
  std::vector<uint16_t> normalized(k);
  or_add_rms_norm(left, right, 1, k, norm_w, eps, residual, normalized.data());
  or_matmul(normalized.data(), 1, k, w0, n0, out0);
  or_matmul(normalized.data(), 1, k, w1, n1, out1);
}

// swiglu_f16 (transformer.metal:1371-1380)
void or_swiglu(const uint16_t* gate, const uint16_t* up, size_t n, uint16_t* out) {
  for (size_t i = 0; i < n; ++i) {
    float x = f(gate[i]);
    out[i] = h((x / (1.0f + mi_exp(-x))) * f(up[i]));
  }
}

// embedding_f16 (transformer.metal:1382-1394)
void or_embedding(const uint32_t* tokens, size_t count, const uint16_t* table, size_t rows,
                  size_t width, uint16_t* out) {
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

// XorShift64::new (qwen3.rs:1016-1024)
uint64_t or_xorshift_seed(uint64_t seed) { return seed == 0 ? 0x9e3779b97f4a7c15ull : seed; }

// sample_token (qwen3.rs:909-925), sample_token_f16 (qwen3.rs:927-939) and
// sample_candidates (qwen3.rs:941-1005) as one sequential pass:
//  * finite logits become candidates; they are ordered by descending
//    total_cmp (the sign-flipped bit key below, so +0 precedes -0) and, among
//    equal bit patterns, by ascending index (the reference's unstable sort
//    leaves that order open; both of its top-k branches reduce to "the first
//    top_k in this order");
//  * weights exp((v - max) * (1 / temperature)) in FP32, summed in FP64 in
//    that order; with top_p < 1 the prefix whose running sum first reaches
//    total * top_p is kept and its running sum becomes the total;
//  * target = next_f64() * total; the first candidate at which
//    target -= weight drops to <= 0 is the token.
uint32_t or_sample_f16(const uint16_t* logits, size_t n, float temperature, float top_p,
                       size_t top_k, uint64_t* state) {
  if (temperature == 0.0f) return or_argmax(logits, n);
  struct Cand {
    uint16_t key;
    uint32_t index;
  };
  std::vector<Cand> cand;
  cand.reserve(n);
  for (size_t i = 0; i < n; ++i) {
    uint16_t b = logits[i];
    if ((b & 0x7c00u) == 0x7c00u) continue;  // infinity or NaN
    uint16_t key = (b & 0x8000u) ? static_cast<uint16_t>(~b) : static_cast<uint16_t>(b | 0x8000u);
    cand.push_back({key, static_cast<uint32_t>(i)});
  }
  if (cand.empty()) return 0xFFFFFFFFu;
  std::stable_sort(cand.begin(), cand.end(),
                   [](const Cand& a, const Cand& b) { return a.key > b.key; });
  if (top_k > 0 && cand.size() > top_k) cand.resize(top_k);
  auto value = [&](const Cand& c) {
    uint16_t b = (c.key & 0x8000u) ? static_cast<uint16_t>(c.key & 0x7fffu)
                                    : static_cast<uint16_t>(~c.key);
    return f(b);
  };
  const float max_logit = value(cand[0]);
  const float inverse = 1.0f / temperature;
  std::vector<float> weight(cand.size());
  double total = 0.0;
  for (size_t i = 0; i < cand.size(); ++i) {
    weight[i] = mi_exp((value(cand[i]) - max_logit) * inverse);
    total += static_cast<double>(weight[i]);
  }
  size_t keep = cand.size();
  if (top_p < 1.0f) {
    const double threshold = total * static_cast<double>(top_p);
    double cumulative = 0.0;
    keep = 0;
    for (size_t i = 0; i < cand.size(); ++i) {
      cumulative += static_cast<double>(weight[i]);
      ++keep;
      if (cumulative >= threshold) break;
    }
    total = 0.0;
    for (size_t i = 0; i < keep; ++i) total += static_cast<double>(weight[i]);
  }
  uint64_t v = *state;
  v ^= v << 13;
  v ^= v >> 7;
  v ^= v << 17;
  *state = v;
  double target = (static_cast<double>(v) / 18446744073709551616.0) * total;
  for (size_t i = 0; i < keep; ++i) {
    target -= static_cast<double>(weight[i]);
    if (target <= 0.0) return cand[i].index;
  }
  return 0xFFFFFFFEu;
}

// rope_f16 (transformer.metal:1514-1531)
void or_rope(const uint16_t* in, size_t tokens, size_t heads, size_t head_dim, size_t offset,
             float theta, uint16_t* out) {
  for (size_t t = 0; t < tokens; ++t)
    for (size_t hh = 0; hh < heads; ++hh) {
      size_t base = (t * heads + hh) * head_dim;
      norm_rope_row(in + base, nullptr, head_dim, t + offset, theta, 0.0f, false, false,
                    out + base);
    }
}

// qk_norm_rope_cache_f16 (transformer.metal:1533-1577)
void or_qk_norm_rope_cache(const uint16_t* q, const uint16_t* k, size_t tokens, size_t q_heads,
                           size_t kv_heads, size_t head_dim, const uint16_t* q_w,
                           const uint16_t* k_w, size_t offset, float theta, float eps,
                           size_t cache_capacity, uint16_t* q_out, uint16_t* key_cache) {
  (void)cache_capacity;
  for (size_t t = 0; t < tokens; ++t) {
    for (size_t hh = 0; hh < q_heads; ++hh) {
      size_t base = (t * q_heads + hh) * head_dim;
      norm_rope_row(q + base, q_w, head_dim, t + offset, theta, eps, true, false, q_out + base);
    }
    for (size_t hh = 0; hh < kv_heads; ++hh) {
      size_t base = (t * kv_heads + hh) * head_dim;
      size_t cache_base = ((offset + t) * kv_heads + hh) * head_dim;
      norm_rope_row(k + base, k_w, head_dim, t + offset, theta, eps, true, false,
                    key_cache + cache_base);
    }
  }
}

// copy_kv_f16 (transformer.metal:2318-2325)
void or_copy_into_cache(const uint16_t* src, size_t tokens, size_t stride, size_t offset,
                        uint16_t* cache) {
  std::memcpy(cache + offset * stride, src, tokens * stride * sizeof(uint16_t));
}

void or_attention(const uint16_t* q, const uint16_t* k, const uint16_t* v, size_t tokens,
                  size_t q_heads, size_t kv_heads, size_t head_dim, size_t kv_length, int causal,
                  size_t query_offset, int semantics, uint16_t* out) {
  if (semantics == OR_ATTN_FLASH_PREFILL || semantics == OR_ATTN_TILED)
    attention_prefill(q, k, v, tokens, q_heads, kv_heads, head_dim, kv_length, causal,
                      query_offset, semantics == OR_ATTN_FLASH_PREFILL, out);
  else
    attention_reference(q, k, v, tokens, q_heads, kv_heads, head_dim, kv_length, causal,
                        query_offset, out);
}

void or_attention_decode(const uint16_t* q, const uint16_t* k, const uint16_t* v, size_t q_heads,
                         size_t kv_heads, size_t head_dim, size_t length, size_t block,
                         size_t streams, uint16_t* out) {
  attention_decode(q, k, v, q_heads, kv_heads, head_dim, length, block, streams, out);
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
  size_t decode_block = 64;
  bool fuse_qk_rope_cache = true;
  bool fuse_add_rms_norm = true;
  size_t tp = 1;  // tensor-parallel ranks whose arithmetic the row-parallel products follow
};

namespace {

std::vector<uint16_t> random_matrix(uint64_t seed, int layer, int role, size_t count,
                                    double std_dev) {
  std::vector<uint16_t> out(count);
  or_gen_normal_f16(seed, static_cast<uint64_t>((layer + 1) * 16 + role), 0, count, std_dev,
                    out.data());
  return out;
}

std::vector<uint16_t> ones(size_t n) { return std::vector<uint16_t>(n, 0x3c00); }

// Row-parallel product of tensor parallelism over `tp` ranks: rank t owns
// input columns [t k / tp, (t + 1) k / tp) and produces the canonical DOT
// over its slice in FP32; the partials are summed in rank order and the sum
// is rounded once to FP16. tp = 1 is or_matmul.
void row_parallel_matmul(const uint16_t* x, size_t m, size_t k, const uint16_t* w, size_t n,
                         size_t tp, uint16_t* out) {
  if (tp <= 1) {
    or_matmul(x, m, k, w, n, out);
    return;
  }
  const size_t ks = k / tp;
  std::vector<float> xf(m * k);
  widen(x, xf.data(), m * k);
#pragma omp parallel for schedule(static)
  for (long long row = 0; row < static_cast<long long>(n); ++row) {
    std::vector<float> wf(k);
    widen(w + static_cast<size_t>(row) * k, wf.data(), k);
    for (size_t r = 0; r < m; ++r) {
      float acc = 0.f;
      for (size_t t = 0; t < tp; ++t) {
        const float part = dot_canon(xf.data() + r * k + t * ks, wf.data() + t * ks, ks);
        acc = t == 0 ? part : acc + part;
      }
      out[r * n + static_cast<size_t>(row)] = h(acc);
    }
  }
}

// One transformer layer on hidden [T, h] (qwen3.rs:647-796), fusion options
// RECOMMENDED (= ALL) unless changed.
void layer_forward(or_qwen3* m, or_qwen3::Layer& L, std::vector<uint16_t>& hidden, size_t T,
                   size_t offset) {
  const auto& c = m->c;
  size_t hs = c.hidden_size, hd = c.head_dim, qh = c.num_attention_heads,
         kvh = c.num_key_value_heads, I = c.intermediate_size;
  size_t qw = qh * hd, kw = kvh * hd;
  float eps = c.rms_norm_eps;
  std::vector<uint16_t> normalized(T * hs), q(T * qw), k(T * kw), v(T * kw);
  or_rms_norm(hidden.data(), T, hs, L.w[kInputNorm].data(), eps, normalized.data());
  {
    std::vector<float> xf(T * hs);
    widen(normalized.data(), xf.data(), T * hs);
    matmul_xf(xf.data(), T, hs, L.w[kQ].data(), qw, q.data());
    matmul_xf(xf.data(), T, hs, L.w[kK].data(), kw, k.data());
    matmul_xf(xf.data(), T, hs, L.w[kV].data(), kw, v.data());
  }
  std::vector<uint16_t> query(T * qw);
  if (m->fuse_qk_rope_cache) {
    or_qk_norm_rope_cache(q.data(), k.data(), T, qh, kvh, hd, L.w[kQNorm].data(),
                          L.w[kKNorm].data(), offset, c.rope_theta, eps, m->capacity,
                          query.data(), L.key_cache.data());
  } else {
    for (size_t t = 0; t < T; ++t) {
      for (size_t hh = 0; hh < qh; ++hh) {
        size_t base = (t * qh + hh) * hd;
        norm_rope_row(q.data() + base, L.w[kQNorm].data(), hd, t + offset, c.rope_theta, eps,
                      true, true, query.data() + base);
      }
      for (size_t hh = 0; hh < kvh; ++hh) {
        size_t base = (t * kvh + hh) * hd;
        norm_rope_row(k.data() + base, L.w[kKNorm].data(), hd, t + offset, c.rope_theta, eps,
                      true, true, L.key_cache.data() + ((offset + t) * kvh + hh) * hd);
      }
    }
  }
  or_copy_into_cache(v.data(), T, kw, offset, L.value_cache.data());
  size_t active = offset + T;
  std::vector<uint16_t> attn(T * qw);
  // attention_kind_for_tokens (qwen3.rs:799-822): one query -> flash decode;
  // 32 or more -> flash prefill; otherwise tiled.
  if (T == 1)
    attention_decode(query.data(), L.key_cache.data(), L.value_cache.data(), qh, kvh, hd, active,
                     m->decode_block, or_decode_streams(hd), attn.data());
  else
    attention_prefill(query.data(), L.key_cache.data(), L.value_cache.data(), T, qh, kvh, hd,
                      active, 1, offset, T >= 32, attn.data());
  std::vector<uint16_t> attn_o(T * hs);
  row_parallel_matmul(attn.data(), T, qw, L.w[kO].data(), hs, m->tp, attn_o.data());
  std::vector<uint16_t> residual(T * hs);
  if (m->fuse_add_rms_norm) {
    or_add_rms_norm(hidden.data(), attn_o.data(), T, hs, L.w[kPostNorm].data(), eps,
                    residual.data(), normalized.data());
  } else {
    or_add(hidden.data(), attn_o.data(), T * hs, residual.data());
    or_rms_norm(residual.data(), T, hs, L.w[kPostNorm].data(), eps, normalized.data());
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
  row_parallel_matmul(act.data(), T, I, L.w[kDown].data(), hs, m->tp, down.data());
  or_add(residual.data(), down.data(), T * hs, hidden.data());
}

}  // namespace

extern "C" {

or_qwen3* or_qwen3_create_random(const or_qwen3_config* cfg, uint64_t seed, double std_dev,
                                 size_t cache_capacity) {
  auto* m = new or_qwen3();
  m->c = *cfg;
  const auto& c = m->c;
  size_t hs = c.hidden_size, hd = c.head_dim, qw = c.num_attention_heads * hd,
         kw = c.num_key_value_heads * hd, I = c.intermediate_size, V = c.vocab_size;
  m->embedding = random_matrix(seed, -1, kEmbedding, V * hs, std_dev);
  m->final_norm = ones(hs);
  if (!c.tie_word_embeddings) m->lm_head = random_matrix(seed, -1, kLmHead, V * hs, std_dev);
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
  m->decode_block = or_decode_block(cache_capacity);
  return m;
}

void or_qwen3_destroy(or_qwen3* m) { delete m; }

void or_qwen3_set_fusion(or_qwen3* m, int qk_rope_cache, int add_rms_norm) {
  m->fuse_qk_rope_cache = qk_rope_cache != 0;
  m->fuse_add_rms_norm = add_rms_norm != 0;
}

void or_qwen3_set_tp(or_qwen3* m, size_t tp) { m->tp = tp ? tp : 1; }

void or_qwen3_reset(or_qwen3* m) { m->filled = 0; }

// KvCache rollback of generate_greedy (qwen3.rs:475-555): keep the first
// `len` positions (the cached rows past them are overwritten later).
int or_qwen3_truncate(or_qwen3* m, size_t len) {
  if (len > m->filled) return -1;
  m->filled = len;
  return 0;
}

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

int or_qwen3_forward(or_qwen3* m, const uint32_t* tokens, size_t count, uint16_t* logits) {
  const auto& c = m->c;
  if (count == 0 || m->filled + count > m->capacity) return -1;
  size_t hs = c.hidden_size;
  std::vector<uint16_t> x(count * hs);
  or_embedding(tokens, count, m->embedding.data(), c.vocab_size, hs, x.data());
  for (auto& L : m->layers) layer_forward(m, L, x, count, m->filled);
  m->filled += count;
  // Final norm, then the last row through the LM head (qwen3.rs:636-638).
  std::vector<uint16_t> normalized(hs);
  or_rms_norm(x.data() + (count - 1) * hs, 1, hs, m->final_norm.data(), c.rms_norm_eps,
              normalized.data());
  const uint16_t* head = c.tie_word_embeddings ? m->embedding.data() : m->lm_head.data();
  or_matmul(normalized.data(), 1, hs, head, c.vocab_size, logits);
  return 0;
}

size_t or_qwen3_generate_greedy(or_qwen3* m, const uint32_t* prompt, size_t prompt_len,
                                size_t max_tokens, uint32_t* out_ids) {
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

// generate_with, temperature > 0 branch (qwen3.rs:455-472), no stop tokens.
size_t or_qwen3_generate_sampled(or_qwen3* m, const uint32_t* prompt, size_t prompt_len,
                                 size_t max_tokens, float temperature, float top_p,
                                 size_t top_k, uint64_t seed, uint32_t* out_ids) {
  if (max_tokens == 0) return 0;
  std::vector<uint16_t> logits(m->c.vocab_size);
  m->filled = 0;
  if (or_qwen3_forward(m, prompt, prompt_len, logits.data()) != 0) return 0;
  uint64_t state = or_xorshift_seed(seed);
  size_t produced = 0;
  for (size_t step = 0; step < max_tokens; ++step) {
    uint32_t token = or_sample_f16(logits.data(), logits.size(), temperature, top_p, top_k, &state);
    if (token >= 0xFFFFFFFEu) break;
    out_ids[produced++] = token;
    if (step + 1 == max_tokens) break;
    if (or_qwen3_forward(m, &token, 1, logits.data()) != 0) break;
  }
  return produced;
}

const uint16_t* or_qwen3_weight(const or_qwen3* m, int layer, int role) {
  if (layer < 0) {
    if (role == kEmbedding) return m->embedding.data();
    if (role == kFinalNorm) return m->final_norm.data();
    if (role == kLmHead) return m->c.tie_word_embeddings ? m->embedding.data() : m->lm_head.data();
    return nullptr;
  }
  if (static_cast<size_t>(layer) >= m->layers.size() || role < 0 || role >= 16) return nullptr;
  return m->layers[layer].w[role].data();
}

const uint16_t* or_qwen3_cache(const or_qwen3* m, int layer, int value) {
  if (layer < 0 || static_cast<size_t>(layer) >= m->layers.size()) return nullptr;
  return value ? m->layers[layer].value_cache.data() : m->layers[layer].key_cache.data();
}

}  // extern "C"
