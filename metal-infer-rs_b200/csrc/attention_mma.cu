// Long-prompt prefill attention on the tensor cores (head_dim 128): causal
// GQA flash attention with QK^T and PV as FP16 MMAs accumulating in FP32,
// the online softmax in FP32 and the probabilities rounded to FP16 before
// the PV product, as attention_flash_prefill_f16 does
// (transformer.metal:1669-1822, whose 32 x 32 simdgroup-matrix tiles become
// 64 x 64 tiles here).
//
// A CTA (4 warps) takes 64 queries of one query head; each warp owns 16
// query rows. K and V tiles of 64 keys are staged in shared memory with
// 16-byte cp.async copies, double buffered so the next tile streams in
// while the current one is used. The MMAs are mma.sync m16n8k16 with
// ldmatrix fragment loads (rows padded to 272 bytes: conflict-free).
// Accumulation order inside an MMA is the hardware's, so results match the
// reference semantics within the per-op tolerance, not bit for bit; the
// engine keeps the canonical kernel (attention.cu) for prompts below
// kMmaPrefillMinTokens.

#include "device.cuh"

namespace mi {
namespace k {

namespace {

constexpr int D = 128;
constexpr int BQ = 64;          // queries per CTA
constexpr int BKEYS = 64;       // keys per tile
constexpr int kWarps = 4;
constexpr int kRow = D + 8;     // halves per padded shared row (272 bytes)

struct MmaSmem {
  __half q[BQ][kRow];
  __half k[2][BKEYS][kRow];
  __half v[2][BKEYS][kRow];
};

__device__ __forceinline__ uint32_t sm_addr(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ void ldsm_x4(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2,
                                        uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(addr));
}

__device__ __forceinline__ void ldsm_x4_t(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2,
                                          uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(addr));
}

// D (16x8 FP32) += A (16x16 FP16, row) * B (16x8 FP16, col)
__device__ __forceinline__ void mma16816(float (&d)[4], const uint32_t (&a)[4], uint32_t b0,
                                         uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%0,%1,%2,%3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

// 2^x by the hardware's approximate exponential (ex2.approx; 2^-inf = 0).
__device__ __forceinline__ float exp2_approx(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

__device__ __forceinline__ uint32_t pack_half2(float lo, float hi) {
  __half2 h = __floats2half2_rn(lo, hi);
  return *reinterpret_cast<uint32_t*>(&h);
}

__device__ __forceinline__ void cp16(void* dst, const void* src) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(sm_addr(dst)), "l"(src)
               : "memory");
}

// Stages keys [j0, j0 + BKEYS) of KV head `kvh_i` into buffer `buf` (rows at
// or past `limit` are zero-filled and masked later).
__device__ __forceinline__ void stage_kv(const AttnProblem& p, MmaSmem& sm, int buf, int kvh_i,
                                         int j0, int limit) {
  const size_t stride = (size_t)p.kvh * D;
  for (int i = threadIdx.x; i < BKEYS * (D / 8); i += kWarps * 32) {
    const int r = i >> 4, c = i & 15;
    const int j = j0 + r;
    if (j < limit) {
      const size_t src = (size_t)j * stride + (size_t)kvh_i * D + 8 * c;
      cp16(&sm.k[buf][r][8 * c], p.k + src);
      cp16(&sm.v[buf][r][8 * c], p.v + src);
    } else {
      *reinterpret_cast<uint4*>(&sm.k[buf][r][8 * c]) = make_uint4(0, 0, 0, 0);
      *reinterpret_cast<uint4*>(&sm.v[buf][r][8 * c]) = make_uint4(0, 0, 0, 0);
    }
  }
  asm volatile("cp.async.commit_group;" ::: "memory");
}

__global__ void __launch_bounds__(kWarps * 32) attention_prefill_mma_kernel(AttnProblem p) {
  extern __shared__ __align__(16) uint8_t smem_raw[];
  MmaSmem& sm = *reinterpret_cast<MmaSmem*>(smem_raw);
  const int lane = threadIdx.x & 31;
  const int warp = threadIdx.x >> 5;
  const int g = lane >> 2, t = lane & 3;
  // heaviest (latest) query tiles first under causal masking
  const int qt = gridDim.x - 1 - blockIdx.x;
  const int h = blockIdx.y;
  const int kvh_i = h / (p.qh / p.kvh);
  const int q0 = qt * BQ;
  pdl_wait();
  const int L = p.kv_len;
  const int last_q = min(p.tokens, q0 + BQ) - 1;
  const int limit = p.causal ? min(L, p.query_offset + last_q + 1) : L;
  const int ntiles = (limit + BKEYS - 1) / BKEYS;

  // Q tile (rows past the prompt are zeros)
  for (int i = threadIdx.x; i < BQ * (D / 8); i += kWarps * 32) {
    const int r = i >> 4, c = i & 15;
    uint4 v = make_uint4(0, 0, 0, 0);
    if (q0 + r < p.tokens)
      v = *reinterpret_cast<const uint4*>(p.q + ((size_t)(q0 + r) * p.qh + h) * D + 8 * c);
    *reinterpret_cast<uint4*>(&sm.q[r][8 * c]) = v;
  }
  if (ntiles > 0) stage_kv(p, sm, 0, kvh_i, 0, limit);
  __syncthreads();

  // Q fragments of this warp's 16 rows, all 8 k-steps
  uint32_t qa[D / 16][4];
  {
    const int mat = lane >> 3, r = lane & 7;
    const int row = warp * 16 + r + 8 * (mat & 1);
#pragma unroll
    for (int kk = 0; kk < D / 16; ++kk)
      ldsm_x4(sm_addr(&sm.q[row][16 * kk + 8 * (mat >> 1)]), qa[kk][0], qa[kk][1], qa[kk][2],
              qa[kk][3]);
  }

  const float sl2 = __frcp_rn(__fsqrt_rn((float)D)) * 1.4426950408889634f;  // scale * log2(e)
  float o[D / 8][4];
#pragma unroll
  for (int j = 0; j < D / 8; ++j) o[j][0] = o[j][1] = o[j][2] = o[j][3] = 0.f;
  float m_row[2] = {-INFINITY, -INFINITY}, l_row[2] = {0.f, 0.f};
  const int qpos0 = p.query_offset + q0 + warp * 16 + g;  // absolute positions of rows g, g + 8

  for (int it = 0; it < ntiles; ++it) {
    const int buf = it & 1;
    const int j0 = it * BKEYS;
    if (it + 1 < ntiles) {
      stage_kv(p, sm, buf ^ 1, kvh_i, j0 + BKEYS, limit);
      asm volatile("cp.async.wait_group 1;" ::: "memory");
    } else {
      asm volatile("cp.async.wait_group 0;" ::: "memory");
    }
    __syncthreads();

    // S = Q K^T for 16 rows x 64 keys
    float s[BKEYS / 8][4];
#pragma unroll
    for (int j = 0; j < BKEYS / 8; ++j) s[j][0] = s[j][1] = s[j][2] = s[j][3] = 0.f;
    {
      const int mat = lane >> 3, r = lane & 7;
#pragma unroll
      for (int kk = 0; kk < D / 16; ++kk)
#pragma unroll
        for (int j = 0; j < BKEYS / 8; j += 2) {
          uint32_t b0, b1, b2, b3;
          ldsm_x4(sm_addr(&sm.k[buf][8 * (j + (mat >> 1)) + r][16 * kk + 8 * (mat & 1)]), b0, b1,
                  b2, b3);
          mma16816(s[j], qa[kk], b0, b1);
          mma16816(s[j + 1], qa[kk], b2, b3);
        }
    }
    // mask, online softmax (FP32), probabilities rounded to FP16
    float mx[2] = {-INFINITY, -INFINITY};
#pragma unroll
    for (int j = 0; j < BKEYS / 8; ++j)
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const int key = j0 + 8 * j + 2 * t + (e & 1);
        const int qpos = qpos0 + 8 * (e >> 1);
        const bool ok = key < limit && (!p.causal || key <= qpos) && key < L;
        s[j][e] = ok ? s[j][e] : -INFINITY;
        mx[e >> 1] = fmaxf(mx[e >> 1], s[j][e]);
      }
    float alpha[2], mnew[2];
#pragma unroll
    for (int r = 0; r < 2; ++r) {
      mx[r] = fmaxf(mx[r], __shfl_xor_sync(0xffffffffu, mx[r], 1));
      mx[r] = fmaxf(mx[r], __shfl_xor_sync(0xffffffffu, mx[r], 2));
      mnew[r] = fmaxf(m_row[r], mx[r]);
      alpha[r] = mnew[r] == -INFINITY ? 1.f : exp2_approx((m_row[r] - mnew[r]) * sl2);
      m_row[r] = mnew[r];
    }
    float rs[2] = {0.f, 0.f};
    uint32_t pa[BKEYS / 16][4];
#pragma unroll
    for (int j = 0; j < BKEYS / 8; ++j) {
      float pv[4];
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const float mr = mnew[e >> 1];
        pv[e] = mr == -INFINITY ? 0.f : exp2_approx((s[j][e] - mr) * sl2);
        rs[e >> 1] += pv[e];
      }
      // C fragments of key tiles 2kk, 2kk + 1 are the A fragment of step kk
      const int kk = j >> 1, hi = j & 1;
      pa[kk][2 * hi] = pack_half2(pv[0], pv[1]);
      pa[kk][2 * hi + 1] = pack_half2(pv[2], pv[3]);
    }
#pragma unroll
    for (int r = 0; r < 2; ++r) {
      rs[r] += __shfl_xor_sync(0xffffffffu, rs[r], 1);
      rs[r] += __shfl_xor_sync(0xffffffffu, rs[r], 2);
      l_row[r] = l_row[r] * alpha[r] + rs[r];
    }
#pragma unroll
    for (int j = 0; j < D / 8; ++j) {
      o[j][0] *= alpha[0];
      o[j][1] *= alpha[0];
      o[j][2] *= alpha[1];
      o[j][3] *= alpha[1];
    }
    // O += P V
    {
      const int mat = lane >> 3, r = lane & 7;
#pragma unroll
      for (int kk = 0; kk < BKEYS / 16; ++kk)
#pragma unroll
        for (int j = 0; j < D / 8; j += 2) {
          uint32_t b0, b1, b2, b3;
          ldsm_x4_t(sm_addr(&sm.v[buf][16 * kk + 8 * (mat & 1) + r][8 * (j + (mat >> 1))]), b0,
                    b1, b2, b3);
          mma16816(o[j], pa[kk], b0, b1);
          mma16816(o[j + 1], pa[kk], b2, b3);
        }
    }
    __syncthreads();  // the buffer is staged again two tiles on
  }

  // O / l -> FP16
#pragma unroll
  for (int r = 0; r < 2; ++r) {
    const int q = q0 + warp * 16 + g + 8 * r;
    if (q >= p.tokens) continue;
    const float inv = l_row[r] > 0.f ? 1.f / l_row[r] : 0.f;
    __half* dst = p.out + ((size_t)q * p.qh + h) * D;
#pragma unroll
    for (int j = 0; j < D / 8; ++j)
      *reinterpret_cast<__half2*>(dst + 8 * j + 2 * t) =
          __floats2half2_rn(o[j][2 * r] * inv, o[j][2 * r + 1] * inv);
  }
}

}  // namespace

bool attention_prefill_mma(const Launch& l, const AttnProblem& p) {
  if (p.hd != D || p.kv_len_dev || p.tokens < kMmaPrefillMinTokens || !p.round_p) return false;
  if (((reinterpret_cast<uintptr_t>(p.q) | reinterpret_cast<uintptr_t>(p.k) |
        reinterpret_cast<uintptr_t>(p.v) | reinterpret_cast<uintptr_t>(p.out)) & 15) != 0)
    return false;
  if (p.qh % p.kvh) return false;
  auto kernel = attention_prefill_mma_kernel;
  allow_dynamic_smem(kernel, sizeof(MmaSmem));
  launch_kernel(l, dim3((p.tokens + BQ - 1) / BQ, p.qh), dim3(kWarps * 32), sizeof(MmaSmem),
                kernel, p);
  return true;
}

}  // namespace k
}  // namespace mi
