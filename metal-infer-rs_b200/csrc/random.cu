// Synthetic weights and token ids for benchmark runs without a checkpoint.
//
// Counter-based SplitMix64 (Steele, Lea and Flood, "Fast splittable
// pseudorandom number generators", OOPSLA 2014): the i-th output of stream s
// under seed S is mix64(state0 + (i + 1) * gamma) with
// state0 = mix64(S ^ mix64(s * gamma + c)). Normals come from the Box-Muller
// transform on the pair (2j, 2j + 1) computed in double precision and rounded
// once to FP16 (round to nearest even). Being counter-based, any block of a
// tensor (a tensor-parallel shard) is generated independently.

#include "device.cuh"

namespace mi {
namespace k {

namespace {

constexpr uint64_t kGamma = 0x9E3779B97F4A7C15ull;

__host__ __device__ __forceinline__ uint64_t mix64(uint64_t z) {
  z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
  z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
  return z ^ (z >> 31);
}

__host__ __device__ __forceinline__ uint64_t stream_state(uint64_t seed, uint64_t stream) {
  return mix64(seed ^ mix64(stream * kGamma + 0x632BE59BD9B4E019ull));
}

__device__ __forceinline__ double unit_open0(uint64_t z) {
  return (double)((z >> 11) + 1) * (1.0 / 9007199254740992.0);
}

__device__ __forceinline__ double normal_at(uint64_t state, uint64_t i) {
  uint64_t pair = i >> 1;
  double u1 = unit_open0(mix64(state + (2 * pair + 1) * kGamma));
  double u2 = unit_open0(mix64(state + (2 * pair + 2) * kGamma));
  double r = sqrt(-2.0 * log(u1));
  double t = 6.283185307179586476925286766559 * u2;
  return (i & 1) ? r * sin(t) : r * cos(t);
}

__global__ void fill_normal_kernel(__half* out, size_t rows, size_t cols, size_t full_cols,
                                   size_t row0, size_t col0, uint64_t state, uint64_t offset,
                                   double std_dev) {
  size_t n = rows * cols;
  for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < n;
       i += (size_t)gridDim.x * blockDim.x) {
    size_t r = i / cols, c = i - r * cols;
    uint64_t idx = offset + (uint64_t)(row0 + r) * full_cols + col0 + c;
    out[i] = __double2half(std_dev * normal_at(state, idx));
  }
}

__global__ void fill_tokens_kernel(uint32_t* out, size_t n, uint64_t state, uint32_t vocab) {
  for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < n;
       i += (size_t)gridDim.x * blockDim.x) {
    uint64_t z = mix64(state + (i + 1) * kGamma);
    out[i] = (uint32_t)(((z >> 32) * vocab) >> 32);
  }
}

__global__ void fill_bits_kernel(uint16_t* out, size_t n, uint16_t bits) {
  for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < n;
       i += (size_t)gridDim.x * blockDim.x)
    out[i] = bits;
}

int grid_of(size_t n) {
  size_t g = (n + 255) / 256;
  return g > 65536 ? 65536 : (g < 1 ? 1 : (int)g);
}

}  // namespace

void fill_normal_f16(cudaStream_t s, __half* out, size_t n, uint64_t seed, uint64_t stream,
                     uint64_t offset, double std_dev) {
  if (!n) return;
  fill_normal_kernel<<<grid_of(n), 256, 0, s>>>(out, 1, n, n, 0, 0, stream_state(seed, stream),
                                                offset, std_dev);
  MI_CUDA(cudaGetLastError());
}

void fill_normal_f16_block(cudaStream_t s, __half* out, size_t rows, size_t cols,
                           size_t full_cols, size_t row0, size_t col0, uint64_t seed,
                           uint64_t stream, double std_dev) {
  if (!rows || !cols) return;
  fill_normal_kernel<<<grid_of(rows * cols), 256, 0, s>>>(
      out, rows, cols, full_cols, row0, col0, stream_state(seed, stream), 0, std_dev);
  MI_CUDA(cudaGetLastError());
}

void fill_tokens(cudaStream_t s, uint32_t* out, size_t n, uint64_t seed, uint64_t stream,
                 uint32_t vocab) {
  if (!n) return;
  fill_tokens_kernel<<<grid_of(n), 256, 0, s>>>(out, n, stream_state(seed, stream), vocab);
  MI_CUDA(cudaGetLastError());
}

void fill_f16(cudaStream_t s, __half* out, size_t n, uint16_t bits) {
  if (!n) return;
  fill_bits_kernel<<<grid_of(n), 256, 0, s>>>(reinterpret_cast<uint16_t*>(out), n, bits);
  MI_CUDA(cudaGetLastError());
}

}  // namespace k
}  // namespace mi
