// Tensor-parallel helpers (no counterpart in the reference, which runs on
// one GPU): the rank-ordered sum that turns the ranks' FP32 partial
// products of the row-parallel projections (O, down) into the FP16 result,
// and the combination of the ranks' greedy candidates of the vocab-parallel
// LM head. The collectives themselves (NCCL all-gathers) are issued by the
// model (qwen3.cu).

#include "device.cuh"

namespace mi {
namespace k {

namespace {

__global__ void rank_sum_round_kernel(const float* parts, int tp, size_t n, __half* out) {
  pdl_wait();
  for (size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x; i < n;
       i += (size_t)gridDim.x * blockDim.x) {
    float acc = parts[i];
    for (int t = 1; t < tp; ++t) acc = __fadd_rn(acc, parts[(size_t)t * n + i]);
    out[i] = __float2half_rn(acc);
  }
}

// Slice `rank` of the rank-ordered sum: rank q's piece is `mine` for q ==
// rank, else row q of `pieces` ([tp, n]).
__global__ void rank_sum_round_slice_kernel(const float* pieces, const float* mine, int rank,
                                            int tp, size_t n, __half* out) {
  pdl_wait();
  for (size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x; i < n;
       i += (size_t)gridDim.x * blockDim.x) {
    float acc = rank == 0 ? mine[i] : pieces[i];
    for (int t = 1; t < tp; ++t)
      acc = __fadd_rn(acc, t == rank ? mine[i] : pieces[(size_t)t * n + i]);
    out[i] = __float2half_rn(acc);
  }
}

__global__ void argmax_combine_kernel(const uint32_t* pairs, int tp, uint32_t* token_out,
                                      const uint32_t* token_pos, uint32_t* step_counter) {
  pdl_wait();
  uint32_t bk = 0, bi = 0xFFFFFFFFu;
  for (int t = 0; t < tp; ++t)
    if (argmax_better(pairs[2 * t], pairs[2 * t + 1], bk, bi)) {
      bk = pairs[2 * t];
      bi = pairs[2 * t + 1];
    }
  token_out[token_pos ? *token_pos + 1u : 0u] = bi;
  if (step_counter) *step_counter += 1u;
}

}  // namespace

void rank_sum_round(cudaStream_t s, const float* parts, int tp, size_t n, __half* out) {
  if (n == 0) return;
  const int grid = (int)std::min<size_t>((n + 255) / 256, 1024);
  rank_sum_round_kernel<<<grid, 256, 0, s>>>(parts, tp, n, out);
  MI_CUDA(cudaGetLastError());
}

void rank_sum_round_slice(cudaStream_t s, const float* pieces, const float* mine, int rank, int tp,
                          size_t n, __half* out) {
  if (n == 0) return;
  const int grid = (int)std::min<size_t>((n + 255) / 256, 1024);
  rank_sum_round_slice_kernel<<<grid, 256, 0, s>>>(pieces, mine, rank, tp, n, out);
  MI_CUDA(cudaGetLastError());
}

void argmax_combine(cudaStream_t s, const uint32_t* pairs, int tp, uint32_t* token_out,
                    const uint32_t* token_pos, uint32_t* step_counter) {
  argmax_combine_kernel<<<1, 1, 0, s>>>(pairs, tp, token_out, token_pos, step_counter);
  MI_CUDA(cudaGetLastError());
}

}  // namespace k
}  // namespace mi
