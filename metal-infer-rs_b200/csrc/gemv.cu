// Decode GEMV family (M = 1): y = x . W^T over FP16 weights with the
// canonical FP32 reduction (numerics.cuh), fused with the prologues and
// epilogues of the decode step:
//   kInNorm      matvec3_rms_impl      (transformer.metal:937-1009)
//   kInAddNorm   matvec2_add_rms_impl  (transformer.metal:1091-1160)
//   kOutResidual matmul + add_f16      (transformer.metal:274-347, 61-68)
//   kOutSwiglu   matvec2 + swiglu_f16  (transformer.metal:484-542, 1371-1380)
//   kOutArgmax   matvec_vocab + argmax (transformer.metal:473-482, 1396-1512)
//
// Weight staging: each CTA owns a contiguous block of output rows. Thread 0
// streams the block's weights into a one- or two-stage shared-memory ring
// with 1-D bulk copies (TMA engine) that complete on mbarriers. The first
// stages are issued before griddepcontrol.wait, so under programmatic
// dependent launch the weight stream of this kernel overlaps the previous
// kernel; only the activation read and the reductions remain on the
// dependency chain. A warp then reduces a row from shared memory: lane l
// takes chunks l, l + 32, ... (16 bytes each) and the lanes meet in the
// canonical butterfly.

#include "device.cuh"
#include "pipeline.cuh"

namespace mi {
namespace k {

namespace {

constexpr int kThreads = 256;
constexpr int kWarps = kThreads / 32;
constexpr int kSmemBudget = 112 * 1024;  // two GEMV CTAs fit on one SM
constexpr int kMaxStages = 6;
#ifndef MI_GEMV_LARGE_CTAS_PER_SM
#define MI_GEMV_LARGE_CTAS_PER_SM 2
#endif
constexpr int kLargeCtasPerSm = MI_GEMV_LARGE_CTAS_PER_SM;

struct Plan {
  int rpc;      // items per CTA
  int rps;      // items per stage
  int stages;   // ring depth (1 .. kMaxStages)
  int x_bytes;  // shared bytes of the input row
  int stage_bytes;
  int early;    // the weight stream starts before the dependency wait
};

__device__ __forceinline__ int items_of(const GemvProblem& p, int out_mode) {
  return out_mode == kOutSwiglu ? p.n[0] : p.n[0] + p.n[1] + p.n[2];
}

// Issues the bulk copies of `chunk` of this CTA's items into its stage.
template <int OUT>
__device__ void issue_stage(const GemvProblem& p, const Plan& plan, uint8_t* stages,
                            uint64_t* full, int first, int last, int chunk) {
  const int s = chunk % plan.stages;
  const int i0 = first + chunk * plan.rps;
  const int cnt = min(plan.rps, last - i0);
  const uint32_t row_bytes = (uint32_t)p.k * 2u;
  uint8_t* dst = stages + (size_t)s * plan.stage_bytes;
  if (OUT == kOutSwiglu) {
    pipe::mbar_expect_tx(&full[s], 2u * cnt * row_bytes);
    pipe::bulk_g2s(dst, p.w[0] + (size_t)i0 * p.k, cnt * row_bytes, &full[s]);
    pipe::bulk_g2s(dst + (size_t)cnt * row_bytes, p.w[1] + (size_t)i0 * p.k, cnt * row_bytes,
                   &full[s]);
    return;
  }
  pipe::mbar_expect_tx(&full[s], (uint32_t)cnt * row_bytes);
  int seg_start = 0;
  int done = 0;
  for (int seg = 0; seg < 3 && done < cnt; ++seg) {
    int seg_end = seg_start + p.n[seg];
    int a = max(i0 + done, seg_start), b = min(i0 + cnt, seg_end);
    if (a < b) {
      pipe::bulk_g2s(dst + (size_t)done * row_bytes, p.w[seg] + (size_t)(a - seg_start) * p.k,
                     (uint32_t)(b - a) * row_bytes, &full[s]);
      done += b - a;
    }
    seg_start = seg_end;
  }
}

// Builds the GEMV input in shared memory (k halves as k/8 uint4 chunks) with
// the canonical sum of squares (one warp) for the normalizing prologues.
template <int IN>
__device__ void build_input(const GemvProblem& p, uint4* xs, float* s_scale) {
  const int tid = threadIdx.x;
  const int lane = tid & 31;
  const int kc = p.k >> 3;
  const uint4* src = reinterpret_cast<const uint4*>(p.x);
  if (IN == kInEmbedNorm) {
    uint32_t tok = p.token[p.token_pos ? *p.token_pos : 0u];
    bool zero = tok == 0xFFFFFFFFu || tok >= p.table_rows;
    src = zero ? nullptr : reinterpret_cast<const uint4*>(p.table + (size_t)tok * p.k);
  }
  for (int c = tid; c < kc; c += kThreads) {
    uint4 v;
    if (IN == kInAddNorm || IN == kInAddThenNorm) {
      uint4 a = src[c];
      uint4 b = reinterpret_cast<const uint4*>(p.x2)[c];
      const __half2* ha = reinterpret_cast<const __half2*>(&a);
      const __half2* hb = reinterpret_cast<const __half2*>(&b);
      __half2* hv = reinterpret_cast<__half2*>(&v);
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        if (IN == kInAddNorm) {
          float2 fa = __half22float2(ha[i]);
          float2 fb = __half22float2(hb[i]);
          hv[i] = __floats2half2_rn(__fadd_rn(fa.x, fb.x), __fadd_rn(fa.y, fb.y));
        } else {
          hv[i] = __hadd2(ha[i], hb[i]);
        }
      }
      if (blockIdx.x == 0 && p.residual_out) reinterpret_cast<uint4*>(p.residual_out)[c] = v;
    } else {
      v = (IN == kInEmbedNorm && src == nullptr) ? make_uint4(0, 0, 0, 0) : src[c];
      if (IN == kInEmbedNorm && blockIdx.x == 0 && p.embed_out)
        reinterpret_cast<uint4*>(p.embed_out)[c] = v;
    }
    xs[c] = v;
  }
  __syncthreads();
  if (IN == kInPlain) return;
  if (tid < 32) {
    float acc = 0.f;
    for (int c = lane; c < kc; c += 32) {
      if (IN == kInAddNorm) {
        // squares of the unrounded sums (matvec2_add_rms_impl)
        uint4 a = src[c];
        uint4 b = reinterpret_cast<const uint4*>(p.x2)[c];
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
      } else {
        acc = chunk_sq(xs[c], acc);
      }
    }
    float total = canon_reduce(acc, canon_lanes(p.k));
    if (lane == 0) *s_scale = rms_scale(total, p.k, p.eps);
  }
  __syncthreads();
  const float scale = *s_scale;
  const uint4* g4 = reinterpret_cast<const uint4*>(p.norm_w);
  for (int c = tid; c < kc; c += kThreads) {
    uint4 v = xs[c];
    uint4 g = g4[c];
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
    xs[c] = o;
  }
  __syncthreads();
}

__device__ __forceinline__ void argmax_take(float v, uint32_t idx, uint32_t& bk, uint32_t& bi) {
  if (isfinite(v) && argmax_better(argmax_key(v), idx, bk, bi)) {
    bk = argmax_key(v);
    bi = idx;
  }
}

template <int IN, int OUT>
__global__ void __launch_bounds__(kThreads) gemv_staged_kernel(GemvProblem p, Plan plan) {
  extern __shared__ __align__(128) uint8_t smem[];
  __shared__ uint64_t full[kMaxStages];
  __shared__ float s_scale;
  __shared__ uint32_t best_key_s[kWarps];
  __shared__ uint32_t best_idx_s[kWarps];
  __shared__ bool is_last;
  uint4* xs = reinterpret_cast<uint4*>(smem);
  uint8_t* stages = smem + plan.x_bytes;

  const int tid = threadIdx.x;
  const int lane = tid & 31;
  const int warp = tid >> 5;
  const int kc = p.k >> 3;
  const int lanes = canon_lanes(p.k);
  const int items = items_of(p, OUT);
  const int first = blockIdx.x * plan.rpc;
  const int last = min(items, first + plan.rpc);
  const int nchunks = first < last ? (last - first + plan.rps - 1) / plan.rps : 0;
  const uint32_t row_bytes = (uint32_t)p.k * 2u;

  // The weight stream starts before the dependency wait when no predecessor
  // can write the weights (the model's launches), else right after it.
  if (tid == 0) {
    for (int s = 0; s < plan.stages; ++s) pipe::mbar_init(&full[s], 1);
    pipe::fence_mbar_init();
    if (plan.early)
      for (int c = 0; c < plan.stages && c < nchunks; ++c)
        issue_stage<OUT>(p, plan, stages, full, first, last, c);
  }
  pdl_trigger();
  pdl_wait();
  if (!plan.early && tid == 0)
    for (int c = 0; c < plan.stages && c < nchunks; ++c)
      issue_stage<OUT>(p, plan, stages, full, first, last, c);
  build_input<IN>(p, xs, &s_scale);

  uint32_t best_key = 0, best_idx = 0xFFFFFFFFu;
  for (int chunk = 0; chunk < nchunks; ++chunk) {
    const int s = chunk % plan.stages;
    pipe::mbar_wait(&full[s], (uint32_t)((chunk / plan.stages) & 1), 0x100u | IN);
    const int i0 = first + chunk * plan.rps;
    const int cnt = min(plan.rps, last - i0);
    const uint8_t* st = stages + (size_t)s * plan.stage_bytes;
    for (int r = warp; r < cnt; r += kWarps) {
      const uint4* w0 = reinterpret_cast<const uint4*>(st + (size_t)r * row_bytes);
      float a0 = 0.f, a1 = 0.f;
      if (OUT == kOutSwiglu) {
        const uint4* w1 = reinterpret_cast<const uint4*>(st + (size_t)(cnt + r) * row_bytes);
        for (int c = lane; c < kc; c += 32) {
          uint4 xv = xs[c];
          a0 = chunk_dot(xv, w0[c], a0);
          a1 = chunk_dot(xv, w1[c], a1);
        }
        a1 = canon_reduce(a1, lanes);
      } else {
        for (int c = lane; c < kc; c += 32) a0 = chunk_dot(xs[c], w0[c], a0);
      }
      a0 = canon_reduce(a0, lanes);
      if (lane == 0) {
        const int item = i0 + r;
        if (OUT == kOutSwiglu) {
          float g = __half2float(__float2half_rn(a0));
          float u = __half2float(__float2half_rn(a1));
          p.out[0][item] = __float2half_rn(silu_mul(g, u));
        } else if (OUT == kOutResidual) {
          p.out[0][item] = __hadd(p.res[item], __float2half_rn(a0));
        } else if (OUT == kOutF32) {
          p.outf[item] = a0;
        } else {
          int seg = 0, row = item;
          if (row >= p.n[0]) {
            row -= p.n[0];
            seg = 1;
            if (row >= p.n[1]) {
              row -= p.n[1];
              seg = 2;
            }
          }
          __half h0 = __float2half_rn(a0);
          p.out[seg][row] = h0;
          if (OUT == kOutArgmax) argmax_take(__half2float(h0), (uint32_t)item, best_key, best_idx);
        }
      }
    }
    __syncthreads();
    if (tid == 0 && chunk + plan.stages < nchunks)
      issue_stage<OUT>(p, plan, stages, full, first, last, chunk + plan.stages);
  }

  if (OUT == kOutArgmax && p.hist) {
    // sampling: key histogram of this block's logits, sorted in the idle
    // weight ring (the last stage has been consumed)
    __syncthreads();
    const uint32_t ring = (uint32_t)plan.stages * plan.stage_bytes;
    int seg = 4096;
    while (seg > 64 && (uint32_t)seg * 2u + 4096u > ring) seg >>= 1;
    hist_add_rows(reinterpret_cast<const uint16_t*>(p.out[0]), first, last,
                  reinterpret_cast<uint16_t*>(stages), seg, p.hist);
  }
  if (OUT == kOutArgmax) {
    if (lane == 0) {
      best_key_s[warp] = best_key;
      best_idx_s[warp] = best_idx;
    }
    __syncthreads();
    if (tid == 0) {
      uint32_t bk = 0, bi = 0xFFFFFFFFu;
      for (int w = 0; w < kWarps; ++w)
        if (argmax_better(best_key_s[w], best_idx_s[w], bk, bi)) {
          bk = best_key_s[w];
          bi = best_idx_s[w];
        }
      p.argmax_partial[blockIdx.x] = __uint_as_float(bk);
      p.argmax_index[blockIdx.x] = bi;
      __threadfence();
      uint32_t done = atomicAdd(p.counter, 1u);
      is_last = done == gridDim.x - 1;
    }
    __syncthreads();
    if (is_last) {
      __threadfence();
      uint32_t bk = 0, bi = 0xFFFFFFFFu;
      for (int b = tid; b < (int)gridDim.x; b += kThreads) {
        uint32_t ck = __float_as_uint(__ldcg(p.argmax_partial + b));
        uint32_t ci = __ldcg(p.argmax_index + b);
        if (argmax_better(ck, ci, bk, bi)) {
          bk = ck;
          bi = ci;
        }
      }
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) {
        uint32_t ok = __shfl_xor_sync(0xffffffffu, bk, o);
        uint32_t oi = __shfl_xor_sync(0xffffffffu, bi, o);
        if (argmax_better(ok, oi, bk, bi)) {
          bk = ok;
          bi = oi;
        }
      }
      if (lane == 0) {
        best_key_s[warp] = bk;
        best_idx_s[warp] = bi;
      }
      __syncthreads();
      if (tid == 0) {
        for (int w = 0; w < kWarps; ++w)
          if (argmax_better(best_key_s[w], best_idx_s[w], bk, bi)) {
            bk = best_key_s[w];
            bi = best_idx_s[w];
          }
        if (p.best_out) {
          p.best_out[0] = bk;
          p.best_out[1] = bi == 0xFFFFFFFFu ? bi : bi + p.index_base;
        } else {
          p.token_out[p.token_pos ? *p.token_pos + 1u : 0u] = bi;
        }
        __threadfence();
        if (p.step_counter) *p.step_counter += 1u;
        *p.counter = 0u;
      }
    }
  }
}

// Generic GEMV for any K and alignment (plain input and output only): one
// warp per row with the canonical chunk order, scalar loads.
__global__ void gemv_generic_kernel(const __half* x, const __half* w, __half* out, int n, int k) {
  int warp = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  int lane = threadIdx.x & 31;
  pdl_wait();
  if (warp >= n) return;
  const __half* row = w + (size_t)warp * k;
  const int lanes = canon_lanes(k);
  const int chunks = (k + 7) / 8;
  float acc = 0.f;
  if (lane < lanes)
    for (int c = lane; c < chunks; c += lanes)
      for (int i = 8 * c; i < min(k, 8 * c + 8); ++i)
        acc = __fmaf_rn(__half2float(x[i]), __half2float(row[i]), acc);
  acc = canon_reduce(acc, lanes);
  if (lane == 0) out[warp] = __float2half_rn(acc);
}

// Reference tiled kernel of matmul_f16 (transformer.metal:70-94): 16x16
// tiles, FP32 accumulate, any shape.
__global__ void matmul_reference_kernel(const __half* x, const __half* w, __half* out, int m,
                                        int n, int k) {
  __shared__ __half xt[16][16];
  __shared__ __half wt[16][16];
  pdl_wait();
  int col = blockIdx.x * 16 + threadIdx.x;
  int row = blockIdx.y * 16 + threadIdx.y;
  float sum = 0.f;
  for (int base = 0; base < k; base += 16) {
    int inner = base + threadIdx.x;
    xt[threadIdx.y][threadIdx.x] = row < m && inner < k ? x[(size_t)row * k + inner] : __half(0.f);
    int wcol = blockIdx.x * 16 + threadIdx.y;
    wt[threadIdx.y][threadIdx.x] =
        wcol < n && inner < k ? w[(size_t)wcol * k + inner] : __half(0.f);
    __syncthreads();
#pragma unroll
    for (int i = 0; i < 16; ++i)
      sum = fmaf(__half2float(xt[threadIdx.y][i]), __half2float(wt[threadIdx.x][i]), sum);
    __syncthreads();
  }
  if (row < m && col < n) out[(size_t)row * n + col] = __float2half_rn(sum);
}

Plan make_plan(const GemvProblem& p, int items, int grid, bool pair) {
  Plan pl;
  pl.early = 1;
  pl.rpc = (items + grid - 1) / grid;
  pl.x_bytes = ((p.k * 2) + 127) / 128 * 128;
  int item_bytes = p.k * 2 * (pair ? 2 : 1);
  int budget = kSmemBudget - pl.x_bytes;
  if (pl.rpc * item_bytes <= budget) {
    pl.stages = 1;  // the whole block is prefetched before the dependency wait
    pl.rps = pl.rpc;
  } else {
    // Streaming: a ring of kMaxStages stages keeps most of the budget in
    // flight while one stage is consumed.
    pl.rps = budget / kMaxStages / item_bytes;
    if (pl.rps < 1) pl.rps = 1;
    pl.stages = kMaxStages;
    if (pl.rps * pl.stages * item_bytes > budget) pl.stages = budget / (pl.rps * item_bytes);
    if (pl.stages < 1) pl.stages = 1;
  }
  pl.stage_bytes = (pl.rps * item_bytes + 127) / 128 * 128;
  return pl;
}

template <int IN, int OUT>
void launch_staged(const Launch& l, const GemvProblem& p) {
  int items = (OUT == kOutSwiglu) ? p.n[0] : p.n[0] + p.n[1] + p.n[2];
  if (items <= 0) return;
  // large problems (the lm_head) run kLargeCtasPerSm CTAs per SM
  int grid = items < l.sm_count ? items : l.sm_count;
  if (items >= 64 * l.sm_count) grid = kLargeCtasPerSm * l.sm_count;
  Plan plan = make_plan(p, items, grid, OUT == kOutSwiglu);
  plan.early = l.early ? 1 : 0;
  grid = (items + plan.rpc - 1) / plan.rpc;
  size_t smem = (size_t)plan.x_bytes + (size_t)plan.stages * plan.stage_bytes;
  auto kernel = gemv_staged_kernel<IN, OUT>;
  allow_dynamic_smem(kernel, kSmemBudget + 1024);
  launch_kernel(l, dim3(grid), dim3(kThreads), smem, kernel, p, plan);
}

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15) == 0; }

}  // namespace

bool gemv_fast_ok(const GemvProblem& p) {
  if (p.k <= 0 || (p.k & 7) || p.k > 16384) return false;
  for (int s = 0; s < 3; ++s)
    if (p.n[s] > 0 && !aligned16(p.w[s])) return false;
  const void* ins[] = {p.x, p.x2, p.norm_w, p.table, p.residual_out, p.embed_out};
  for (const void* q : ins)
    if (q && !aligned16(q)) return false;
  return true;
}

unsigned gemv_status(bool reset) { return pipe::read_status(reset); }

void gemv(const Launch& l, const GemvProblem& p) {
  if (!gemv_fast_ok(p)) {
    MI_REQUIRE(p.in_mode == kInPlain && p.out_mode == kOutPlain, MI_ERR_SHAPE,
               "fused GEMV needs K %% 8 == 0, K <= 16384 and 16-byte aligned operands");
    for (int s = 0; s < 3; ++s) {
      if (p.n[s] <= 0) continue;
      int grid = (p.n[s] * 32 + 255) / 256;
      launch_kernel(l, dim3(grid), dim3(256), 0, gemv_generic_kernel, p.x, p.w[s], p.out[s],
                    p.n[s], p.k);
    }
    return;
  }
#define MI_GEMV_CASE(IN, OUT)                 \
  if (p.in_mode == IN && p.out_mode == OUT) { \
    launch_staged<IN, OUT>(l, p);             \
    return;                                   \
  }
  MI_GEMV_CASE(kInPlain, kOutPlain)
  MI_GEMV_CASE(kInNorm, kOutPlain)
  MI_GEMV_CASE(kInAddNorm, kOutPlain)
  MI_GEMV_CASE(kInEmbedNorm, kOutPlain)
  MI_GEMV_CASE(kInPlain, kOutResidual)
  MI_GEMV_CASE(kInAddNorm, kOutSwiglu)
  MI_GEMV_CASE(kInAddThenNorm, kOutPlain)
  MI_GEMV_CASE(kInAddThenNorm, kOutSwiglu)
  MI_GEMV_CASE(kInPlain, kOutSwiglu)
  MI_GEMV_CASE(kInNorm, kOutArgmax)
  MI_GEMV_CASE(kInPlain, kOutArgmax)
  MI_GEMV_CASE(kInPlain, kOutF32)
#undef MI_GEMV_CASE
  fail(MI_ERR_SHAPE, "unsupported GEMV fusion (%d, %d)", p.in_mode, p.out_mode);
}

void matmul_reference(const Launch& l, const __half* x, const __half* w, __half* out, int m,
                      int n, int k) {
  dim3 grid((n + 15) / 16, (m + 15) / 16);
  launch_kernel(l, grid, dim3(16, 16), 0, matmul_reference_kernel, x, w, out, m, n, k);
}

}  // namespace k
}  // namespace mi
