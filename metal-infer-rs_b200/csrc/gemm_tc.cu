// tcgen05 tensor-core GEMM for the prefill projections (placeholder until the
// TMA/TMEM kernel lands: every call falls back to the CUDA-core kernel).
#include "device.cuh"

namespace mi {
namespace k {

bool gemm_tc_available() { return false; }

bool gemm_tc(const Launch&, const __half*, const __half*, __half*, int, int, int, int) {
  return false;
}

}  // namespace k
}  // namespace mi
