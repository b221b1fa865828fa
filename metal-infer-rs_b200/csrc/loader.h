// Safetensors checkpoints (crates/metal-infer-models/src/weights.rs:21-75,
// qwen3.rs:155-240): config.json, model.safetensors or the shards listed by
// model.safetensors.index.json, F16 or BF16 tensors (BF16 converted to FP16
// through FP32 with round-to-nearest-even, as half's f16::from_f32).
#pragma once

#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <map>
#include <memory>
#include <string>
#include <vector>

#include "mi.h"

namespace mi {
namespace load {

struct TensorInfo {
  std::string dtype;  // "F16" or "BF16" (others are rejected when read)
  std::vector<size_t> shape;
  size_t begin = 0, end = 0;  // byte range in the file's data section
  int file = 0;
};

class Checkpoint {
 public:
  // Opens `directory` (config.json + tensor files); throws mi errors.
  static std::unique_ptr<Checkpoint> open(const std::string& directory);
  ~Checkpoint();

  const mi_qwen3_config& config() const { return config_; }
  bool has(const std::string& name) const { return tensors_.count(name) != 0; }
  // Checks presence (MI_ERR_MISSING_TENSOR) and shape (MI_ERR_CONFIG).
  const TensorInfo& expect(const std::string& name, const std::vector<size_t>& shape) const;
  // Rows [row0, row0 + rows) x columns [col0, col0 + cols) of the 2-D (or
  // 1-D: rows = 1) tensor `name` into `dst` as FP16, on `stream`
  // (synchronous with respect to the host buffer it stages through).
  void read_block(const std::string& name, size_t rows, size_t cols, size_t row0, size_t col0,
                  __half* dst, cudaStream_t stream) const;

 private:
  struct File {
    int fd = -1;
    const unsigned char* map = nullptr;
    size_t size = 0;
    size_t data = 0;  // offset of the data section
  };
  mi_qwen3_config config_{};
  std::vector<File> files_;
  std::map<std::string, TensorInfo> tensors_;
};

// Checkpoint name of a weight: layer -1 for model-level tensors; roles as
// mi_qwen3_create_random (0 embedding, 1 q, 2 k, 3 v, 4 o, 5 q_norm,
// 6 k_norm, 7 gate, 8 up, 9 down, 10 input norm, 11 post-attention norm,
// 12 final norm, 13 lm_head).
std::string weight_name(int layer, int role);

}  // namespace load
}  // namespace mi
