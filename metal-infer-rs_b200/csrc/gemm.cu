// Prefill projections (M > 1): out[m, n] = sum_k x[m, k] * w[n, k] with FP32
// accumulation and one FP16 rounding (matmul_simd_db_f16,
// transformer.metal:174-272).
//
//   gemm_canon  CUDA-core kernel with the canonical reduction of numerics.cuh
//               (each output is DOT(x[m], w[n]) exactly as the decode GEMV
//               computes it); used for prompts up to kCanonRows rows, where
//               the weight stream, not the arithmetic, bounds the time
//   gemm_tc     tcgen05 tensor-core kernel (gemm_tc.cu) for longer prompts
//   gemm_simt   tiled fallback for ragged K or unaligned operands

#include "device.cuh"

namespace mi {
namespace k {

namespace {

constexpr int kCanonRows = 512;

// Warp tile: 8 rows of x by 8 rows of w; CTA: 2 x 4 warp tiles (16 x 32).
// Lane l reduces chunks l, l + 32, ... of every pair, then the canonical
// butterfly completes each of the 64 dots.
__global__ void __launch_bounds__(256) gemm_canon_kernel(const __half* x, const __half* w,
                                                         __half* out, int m, int n, int k,
                                                         int ldo, float* outf) {
  pdl_wait();
  const int lane = threadIdx.x & 31;
  const int warp = threadIdx.x >> 5;
  const int m0 = blockIdx.y * 16 + (warp & 1) * 8;
  const int n0 = blockIdx.x * 32 + (warp >> 1) * 8;
  const int kc = k >> 3;
  const int lanes = canon_lanes(k);
  float acc[8][8];
#pragma unroll
  for (int i = 0; i < 8; ++i)
#pragma unroll
    for (int j = 0; j < 8; ++j) acc[i][j] = 0.f;
  const uint4 zero = make_uint4(0, 0, 0, 0);
  for (int c = lane; c < kc; c += 32) {
    uint4 xv[8], wv[8];
#pragma unroll
    for (int i = 0; i < 8; ++i)
      xv[i] = m0 + i < m ? __ldg(reinterpret_cast<const uint4*>(x + (size_t)(m0 + i) * k) + c)
                         : zero;
#pragma unroll
    for (int j = 0; j < 8; ++j)
      wv[j] = n0 + j < n ? __ldg(reinterpret_cast<const uint4*>(w + (size_t)(n0 + j) * k) + c)
                         : zero;
#pragma unroll
    for (int i = 0; i < 8; ++i)
#pragma unroll
      for (int j = 0; j < 8; ++j) acc[i][j] = chunk_dot(xv[i], wv[j], acc[i][j]);
  }
#pragma unroll
  for (int i = 0; i < 8; ++i)
#pragma unroll
    for (int j = 0; j < 8; ++j) acc[i][j] = canon_reduce(acc[i][j], lanes);
  // Lane l writes outputs (l / 8, l % 8) and (l / 8 + 4, l % 8).
#pragma unroll
  for (int half = 0; half < 2; ++half) {
    int i = lane / 8 + 4 * half, j = lane % 8;
    float v = 0.f;
#pragma unroll
    for (int ii = 0; ii < 8; ++ii)
#pragma unroll
      for (int jj = 0; jj < 8; ++jj)
        if (ii == i && jj == j) v = acc[ii][jj];
    if (m0 + i < m && n0 + j < n) {
      if (outf) outf[(size_t)(m0 + i) * ldo + n0 + j] = v;
      else out[(size_t)(m0 + i) * ldo + n0 + j] = __float2half_rn(v);
    }
  }
}

// Staged canonical kernel (K >= 256, so every dot spans all 32 lanes): the
// CTA's 16 x rows and 32 w rows are staged 256 elements (one chunk per lane)
// at a time in shared memory by a three-stage 16-byte cp.async pipeline; the
// warp tiles and each lane's FMA chains are those of gemm_canon_kernel. The
// final butterflies of the 64 dots run as a transpose-reduce: at each level a
// lane keeps half of its dots and adds its partner's copies (the same operand
// pairs as the butterfly), so each lane ends with two finished dots and the
// warp issues 62 shuffles instead of 320. Up to three weight matrices that
// share the input (Q / K / V, gate / up) run as one launch: the grid's
// columns walk their rows back to back, each 32-row tile inside one of them.
constexpr int kSM = 16, kSN = 32, kSK = 256, kStages = 3;

struct CanonSmem {
  __half x[kStages][kSM][kSK];
  __half w[kStages][kSN][kSK];
};

struct CanonSeg {
  const __half* w = nullptr;
  __half* out = nullptr;
  float* outf = nullptr;  // FP32 output instead of FP16 (tensor-parallel partials)
  int n = 0;              // rows of w (a multiple of kSN unless it is the only one)
  int ldo = 0;
};
struct CanonSegs {
  CanonSeg s[3];
  int count = 0;
};

// One thread's six 16-byte copies of a stage: column chunk c = lane of rows
// r = warp + 8 j (j < 2: x rows, j >= 2: w rows), addresses computed once;
// a stage at k0 adds k0 to the sources and the buffer offset to the
// destinations.
struct CanonCopies {
  static constexpr int kPer = (kSM + kSN) * (kSK / 8) / 256;
  const __half* src[kPer];  // null: outside the matrix (the chunk is zeroed)
  uint32_t dst[kPer];       // shared address in buffer 0
};
static_assert((kSM + kSN) * (kSK / 8) % 256 == 0 && kSK / 8 == 32, "stage copy layout");

__device__ __forceinline__ CanonCopies canon_copies(const __half* x, const __half* w, int m,
                                                    int n, int k, int m0, int n0,
                                                    CanonSmem& sm) {
  CanonCopies cp;
  const int c = threadIdx.x & 31, r0 = threadIdx.x >> 5;
#pragma unroll
  for (int j = 0; j < CanonCopies::kPer; ++j) {
    const int r = r0 + 8 * j;
    const bool is_x = r < kSM;
    const int row = is_x ? m0 + r : n0 + (r - kSM);
    __half* dst = is_x ? &sm.x[0][r][8 * c] : &sm.w[0][r - kSM][8 * c];
    cp.dst[j] = static_cast<uint32_t>(__cvta_generic_to_shared(dst));
    cp.src[j] = (is_x ? row < m : row < n) ? (is_x ? x : w) + (size_t)row * k + 8 * c : nullptr;
  }
  return cp;
}

__device__ __forceinline__ void canon_stage(const CanonCopies& cp, int k, int k0, int buf) {
  const bool in_k = k0 + 8 * (int)(threadIdx.x & 31) < k;
  const uint32_t off = (uint32_t)buf * (uint32_t)(kSM * kSK * 2);
  const uint32_t offw = (uint32_t)buf * (uint32_t)(kSN * kSK * 2);
#pragma unroll
  for (int j = 0; j < CanonCopies::kPer; ++j) {
    const uint32_t dst = cp.dst[j] + (j < kSM / 8 ? off : offw);
    if (cp.src[j] && in_k) {
      asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(dst), "l"(cp.src[j] + k0)
                   : "memory");
    } else {
      asm volatile("st.shared.v4.u32 [%0], {%1, %1, %1, %1};" ::"r"(dst), "r"(0u) : "memory");
    }
  }
  asm volatile("cp.async.commit_group;" ::: "memory");
}

__global__ void __launch_bounds__(256) gemm_canon_staged_kernel(const __half* x, int m, int k,
                                                                CanonSegs segs) {
  extern __shared__ __align__(16) uint8_t canon_smem[];
  CanonSmem& sm = *reinterpret_cast<CanonSmem*>(canon_smem);
  pdl_wait();
  const int lane = threadIdx.x & 31;
  const int warp = threadIdx.x >> 5;
  // this CTA's weight matrix and its 32-row tile there
  int n0 = blockIdx.x * kSN;
  CanonSeg seg = segs.s[0];
  if (segs.count > 1 && n0 >= segs.s[0].n) {
    n0 -= segs.s[0].n;
    seg = segs.s[1];
    if (segs.count > 2 && n0 >= segs.s[1].n) {
      n0 -= segs.s[1].n;
      seg = segs.s[2];
    }
  }
  const __half* w = seg.w;
  const int n = seg.n;
  const int m0 = blockIdx.y * kSM;
  const int wm = (warp & 1) * 8, wn = (warp >> 1) * 8;
  const int steps = (k + kSK - 1) / kSK;
  float acc[64];
#pragma unroll
  for (int a = 0; a < 64; ++a) acc[a] = 0.f;
  const CanonCopies cps = canon_copies(x, w, m, n, k, m0, n0, sm);
  canon_stage(cps, k, 0, 0);
  if (steps > 1) canon_stage(cps, k, kSK, 1);
  for (int st = 0; st < steps; ++st) {
    const int buf = st % kStages;
    if (st + 2 < steps) {
      canon_stage(cps, k, (st + 2) * kSK, (st + 2) % kStages);
      asm volatile("cp.async.wait_group 2;" ::: "memory");
    } else if (st + 1 < steps) {
      asm volatile("cp.async.wait_group 1;" ::: "memory");
    } else {
      asm volatile("cp.async.wait_group 0;" ::: "memory");
    }
    __syncthreads();
    uint4 xv[8];
#pragma unroll
    for (int i = 0; i < 8; ++i) xv[i] = reinterpret_cast<const uint4*>(sm.x[buf][wm + i])[lane];
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const uint4 wv = reinterpret_cast<const uint4*>(sm.w[buf][wn + j])[lane];
#pragma unroll
      for (int i = 0; i < 8; ++i) acc[i * 8 + j] = chunk_dot(xv[i], wv, acc[i * 8 + j]);
    }
    __syncthreads();  // this buffer is staged again at the next step
  }
  // Transpose-reduce: dot d = i * 8 + j; at the level of lane bit b (16, 8,
  // 4, 2, 1) a lane keeps the half of its dots whose matching index bit
  // equals its lane bit and adds the partner's value of the same dot.
#pragma unroll
  for (int half = 32, o = 16; o >= 1; half >>= 1, o >>= 1) {
    const bool up = (lane & o) != 0;
#pragma unroll
    for (int a = 0; a < half; ++a) {
      const float keep = up ? acc[a + half] : acc[a];
      const float send = up ? acc[a] : acc[a + half];
      acc[a] = __fadd_rn(keep, __shfl_xor_sync(0xffffffffu, send, o));
    }
  }
  // lane l holds dots 2l and 2l + 1 (index bits 5..1 = lane bits 4..0)
#pragma unroll
  for (int s2 = 0; s2 < 2; ++s2) {
    const int d = 2 * lane + s2;
    const int i = d >> 3, j = d & 7;
    if (m0 + wm + i < m && n0 + wn + j < n) {
      const size_t o2 = (size_t)(m0 + wm + i) * seg.ldo + n0 + wn + j;
      if (seg.outf) seg.outf[o2] = acc[s2];
      else seg.out[o2] = __float2half_rn(acc[s2]);
    }
  }
}

constexpr int BM = 64, BN = 64, BK = 16;

// 256 threads; each computes a 4x4 block of the 64x64 tile.
__global__ void __launch_bounds__(256) gemm_simt_kernel(const __half* x, const __half* w,
                                                        __half* out, int m, int n, int k,
                                                        int ldo) {
  __shared__ float xs[BK][BM + 4];
  __shared__ float ws[BK][BN + 4];
  pdl_wait();
  const int tid = threadIdx.x;
  const int tx = tid % 16, ty = tid / 16;
  const int m0 = blockIdx.y * BM, n0 = blockIdx.x * BN;
  float acc[4][4] = {};
  for (int k0 = 0; k0 < k; k0 += BK) {
    for (int i = tid; i < BM * BK; i += 256) {
      int r = i / BK, c = i % BK;
      int gm = m0 + r, gk = k0 + c;
      xs[c][r] = (gm < m && gk < k) ? __half2float(x[(size_t)gm * k + gk]) : 0.f;
      int gn = n0 + r;
      ws[c][r] = (gn < n && gk < k) ? __half2float(w[(size_t)gn * k + gk]) : 0.f;
    }
    __syncthreads();
#pragma unroll
    for (int kk = 0; kk < BK; ++kk) {
      float a[4], b[4];
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        a[i] = xs[kk][ty * 4 + i];
        b[i] = ws[kk][tx * 4 + i];
      }
#pragma unroll
      for (int i = 0; i < 4; ++i)
#pragma unroll
        for (int j = 0; j < 4; ++j) acc[i][j] = fmaf(a[i], b[j], acc[i][j]);
    }
    __syncthreads();
  }
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    int gm = m0 + ty * 4 + i;
    if (gm >= m) continue;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      int gn = n0 + tx * 4 + j;
      if (gn < n) out[(size_t)gm * ldo + gn] = __float2half_rn(acc[i][j]);
    }
  }
}

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15) == 0; }

// The canonical GEMM over one to three weight matrices sharing x: the staged
// kernel when every dot spans 32 lanes (K >= 256; matrices whose rows are
// not a multiple of its 32-row tile run as launches of their own), else the
// direct one.
void launch_canon(const Launch& l, const __half* x, int m, int k, const CanonSegs& segs) {
  if (k >= kSK) {
    auto kernel = gemm_canon_staged_kernel;
    allow_dynamic_smem(kernel, sizeof(CanonSmem));
    bool tiled = true;
    int n_total = 0;
    for (int i = 0; i < segs.count; ++i) {
      tiled &= segs.s[i].n % kSN == 0;
      n_total += segs.s[i].n;
    }
    if (segs.count == 1 || tiled) {
      dim3 grid((n_total + kSN - 1) / kSN, (m + kSM - 1) / kSM);
      launch_kernel(l, grid, dim3(256), sizeof(CanonSmem), kernel, x, m, k, segs);
      return;
    }
    for (int i = 0; i < segs.count; ++i) {
      CanonSegs one;
      one.s[0] = segs.s[i];
      one.count = 1;
      dim3 grid((segs.s[i].n + kSN - 1) / kSN, (m + kSM - 1) / kSM);
      launch_kernel(l, grid, dim3(256), sizeof(CanonSmem), kernel, x, m, k, one);
    }
    return;
  }
  for (int i = 0; i < segs.count; ++i) {
    const CanonSeg& g = segs.s[i];
    dim3 grid((g.n + 31) / 32, (m + 15) / 16);
    launch_kernel(l, grid, dim3(256), 0, gemm_canon_kernel, x, g.w, g.out, m, g.n, k, g.ldo,
                  g.outf);
  }
}

CanonSegs one_seg(const __half* w, __half* out, float* outf, int n, int ldo) {
  CanonSegs s;
  s.s[0].w = w;
  s.s[0].out = out;
  s.s[0].outf = outf;
  s.s[0].n = n;
  s.s[0].ldo = ldo;
  s.count = 1;
  return s;
}

}  // namespace

// FP16 `out`, or FP32 `outf` when it is non-null.
bool gemm_tc(const Launch& l, const __half* x, const __half* w, __half* out, int m, int n, int k,
             int ldo, float* outf = nullptr);

void gemm(const Launch& l, const __half* x, const __half* w, __half* out, int m, int n, int k,
          int ldo) {
  if (m <= 0 || n <= 0) return;
  const bool vec = k % 8 == 0 && aligned16(x) && aligned16(w);
  if (vec && m <= kCanonRows) {
    launch_canon(l, x, m, k, one_seg(w, out, nullptr, n, ldo));
    return;
  }
  if (gemm_tc(l, x, w, out, m, n, k, ldo)) return;
  dim3 grid((n + BN - 1) / BN, (m + BM - 1) / BM);
  launch_kernel(l, grid, dim3(256), 0, gemm_simt_kernel, x, w, out, m, n, k, ldo);
}

void gemm_partial_f32(const Launch& l, const __half* x, const __half* w, float* out, int m, int n,
                      int k) {
  if (m <= 0 || n <= 0) return;
  MI_REQUIRE(k % 8 == 0 && aligned16(x) && aligned16(w), MI_ERR_SHAPE,
             "tensor-parallel partial products need K %% 8 == 0 and 16-byte aligned operands");
  // long prompts: the tensor-core GEMM (the per-op tolerance, as without TP)
  if (m > kCanonRows && gemm_tc(l, x, w, nullptr, m, n, k, n, out)) return;
  launch_canon(l, x, m, k, one_seg(w, nullptr, out, n, n));
}

void gemm_multi(const Launch& l, const __half* x, int m, int k, int count,
                const __half* const* w, __half* const* out, const int* n) {
  if (m <= 0 || count <= 0) return;
  bool vec = k % 8 == 0 && aligned16(x);
  for (int i = 0; i < count; ++i) vec &= aligned16(w[i]);
  if (vec && m <= kCanonRows && count <= 3) {
    CanonSegs segs;
    for (int i = 0; i < count; ++i) {
      segs.s[i].w = w[i];
      segs.s[i].out = out[i];
      segs.s[i].n = n[i];
      segs.s[i].ldo = n[i];
    }
    segs.count = count;
    launch_canon(l, x, m, k, segs);
    return;
  }
  for (int i = 0; i < count; ++i) gemm(l, x, w[i], out[i], m, n[i], k, n[i]);
}

}  // namespace k
}  // namespace mi
