// Safetensors checkpoint reader (weights.rs:21-75, qwen3.rs:155-240,
// config.rs:5-57). The format is an 8-byte little-endian header length, a
// JSON header {name: {dtype, shape, data_offsets: [begin, end]}, ...} and
// the raw tensor bytes. Files are memory-mapped; a requested block is
// gathered on the host (rows, or a column slice of each row for
// tensor-parallel shards), copied to the device and converted there.

#include "loader.h"

#include <fcntl.h>
#include <sys/mman.h>
#include <sys/stat.h>
#include <unistd.h>

#include <algorithm>
#include <cstring>
#include <fstream>
#include <set>
#include <sstream>

#include "mi_internal.h"

namespace mi {
namespace load {

namespace {

// ---- a small JSON reader (objects, arrays, strings, numbers, literals) ----
struct Json {
  enum Kind { kNull, kBool, kNum, kStr, kArr, kObj } kind = kNull;
  bool b = false;
  double num = 0;
  std::string str;
  std::vector<Json> arr;
  std::vector<std::pair<std::string, Json>> obj;

  const Json* get(const std::string& key) const {
    for (const auto& kv : obj)
      if (kv.first == key) return &kv.second;
    return nullptr;
  }
};

class Parser {
 public:
  Parser(const char* p, const char* e, const std::string& what) : p_(p), e_(e), what_(what) {}
  Json parse() {
    Json v = value();
    ws();
    if (p_ != e_) bad("trailing characters");
    return v;
  }

 private:
  [[noreturn]] void bad(const char* why) {
    fail(MI_ERR_IO, "invalid JSON in %s: %s", what_.c_str(), why);
  }
  void ws() {
    while (p_ < e_ && (*p_ == ' ' || *p_ == '\n' || *p_ == '\r' || *p_ == '\t')) ++p_;
  }
  bool lit(const char* s) {
    size_t n = std::strlen(s);
    if ((size_t)(e_ - p_) >= n && std::memcmp(p_, s, n) == 0) {
      p_ += n;
      return true;
    }
    return false;
  }
  Json value() {
    ws();
    if (p_ >= e_) bad("unexpected end");
    Json v;
    if (*p_ == '{') {
      v.kind = Json::kObj;
      ++p_;
      ws();
      if (p_ < e_ && *p_ == '}') {
        ++p_;
        return v;
      }
      while (true) {
        ws();
        std::string k = string();
        ws();
        if (p_ >= e_ || *p_ != ':') bad("expected ':'");
        ++p_;
        v.obj.emplace_back(std::move(k), value());
        ws();
        if (p_ < e_ && *p_ == ',') {
          ++p_;
          continue;
        }
        if (p_ < e_ && *p_ == '}') {
          ++p_;
          return v;
        }
        bad("expected ',' or '}'");
      }
    }
    if (*p_ == '[') {
      v.kind = Json::kArr;
      ++p_;
      ws();
      if (p_ < e_ && *p_ == ']') {
        ++p_;
        return v;
      }
      while (true) {
        v.arr.push_back(value());
        ws();
        if (p_ < e_ && *p_ == ',') {
          ++p_;
          continue;
        }
        if (p_ < e_ && *p_ == ']') {
          ++p_;
          return v;
        }
        bad("expected ',' or ']'");
      }
    }
    if (*p_ == '"') {
      v.kind = Json::kStr;
      v.str = string();
      return v;
    }
    if (lit("true")) {
      v.kind = Json::kBool;
      v.b = true;
      return v;
    }
    if (lit("false")) {
      v.kind = Json::kBool;
      return v;
    }
    if (lit("null")) return v;
    const char* start = p_;
    while (p_ < e_ && (std::isdigit((unsigned char)*p_) || *p_ == '-' || *p_ == '+' ||
                       *p_ == '.' || *p_ == 'e' || *p_ == 'E'))
      ++p_;
    if (p_ == start) bad("unexpected character");
    v.kind = Json::kNum;
    v.num = std::strtod(std::string(start, p_).c_str(), nullptr);
    return v;
  }
  std::string string() {
    if (p_ >= e_ || *p_ != '"') bad("expected a string");
    ++p_;
    std::string s;
    while (p_ < e_ && *p_ != '"') {
      char c = *p_++;
      if (c == '\\') {
        if (p_ >= e_) bad("bad escape");
        char n = *p_++;
        switch (n) {
          case 'n': s += '\n'; break;
          case 't': s += '\t'; break;
          case 'r': s += '\r'; break;
          case 'b': s += '\b'; break;
          case 'f': s += '\f'; break;
          case 'u':
            if (e_ - p_ < 4) bad("bad escape");
            p_ += 4;  // names and keys are ASCII; other code points are not needed
            s += '?';
            break;
          default: s += n; break;
        }
      } else {
        s += c;
      }
    }
    if (p_ >= e_) bad("unterminated string");
    ++p_;
    return s;
  }
  const char* p_;
  const char* e_;
  std::string what_;
};

std::string read_text(const std::string& path) {
  std::ifstream f(path, std::ios::binary);
  if (!f) fail(MI_ERR_IO, "cannot read %s", path.c_str());
  std::ostringstream ss;
  ss << f.rdbuf();
  return ss.str();
}

bool exists(const std::string& path) {
  struct stat st;
  return ::stat(path.c_str(), &st) == 0;
}

size_t num_field(const Json& cfg, const char* key) {
  const Json* v = cfg.get(key);
  if (!v || v->kind != Json::kNum || v->num < 0)
    fail(MI_ERR_IO, "config.json: missing or invalid field `%s`", key);
  return (size_t)v->num;
}

// qwen3 Qwen3Config (config.rs:5-57), as read from config.json.
mi_qwen3_config parse_config(const std::string& directory) {
  const std::string text = read_text(directory + "/config.json");
  const Json cfg = Parser(text.data(), text.data() + text.size(), "config.json").parse();
  if (cfg.kind != Json::kObj) fail(MI_ERR_IO, "config.json is not an object");
  const Json* type = cfg.get("model_type");
  if (!type || type->kind != Json::kStr) fail(MI_ERR_IO, "config.json: missing `model_type`");
  if (type->str != "qwen3")
    fail(MI_ERR_UNSUPPORTED, "unsupported model: expected model_type qwen3, got %s",
         type->str.c_str());
  const Json* bias = cfg.get("attention_bias");
  if (bias && bias->kind == Json::kBool && bias->b)
    fail(MI_ERR_UNSUPPORTED, "unsupported model: attention biases are not implemented");
  mi_qwen3_config c{};
  c.hidden_size = (uint32_t)num_field(cfg, "hidden_size");
  c.intermediate_size = (uint32_t)num_field(cfg, "intermediate_size");
  c.num_hidden_layers = (uint32_t)num_field(cfg, "num_hidden_layers");
  c.num_attention_heads = (uint32_t)num_field(cfg, "num_attention_heads");
  c.num_key_value_heads = (uint32_t)num_field(cfg, "num_key_value_heads");
  c.head_dim = (uint32_t)num_field(cfg, "head_dim");
  c.vocab_size = (uint32_t)num_field(cfg, "vocab_size");
  const Json* eps = cfg.get("rms_norm_eps");
  const Json* theta = cfg.get("rope_theta");
  if (!eps || eps->kind != Json::kNum || !theta || theta->kind != Json::kNum)
    fail(MI_ERR_IO, "config.json: missing `rms_norm_eps` or `rope_theta`");
  c.rms_norm_eps = (float)eps->num;
  c.rope_theta = (float)theta->num;
  const Json* tie = cfg.get("tie_word_embeddings");
  c.tie_word_embeddings = (tie && tie->kind == Json::kBool && tie->b) ? 1 : 0;
  return c;
}

// BF16 bits -> FP32 -> FP16 with round-to-nearest-even.
__global__ void bf16_to_f16_kernel(const uint16_t* in, __half* out, size_t n) {
  for (size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x; i < n;
       i += (size_t)gridDim.x * blockDim.x)
    out[i] = __float2half_rn(__uint_as_float((uint32_t)in[i] << 16));
}

}  // namespace

std::string weight_name(int layer, int role) {
  if (layer < 0) {
    switch (role) {
      case 0: return "model.embed_tokens.weight";
      case 12: return "model.norm.weight";
      case 13: return "lm_head.weight";
      default: return "";
    }
  }
  const std::string pre = "model.layers." + std::to_string(layer);
  switch (role) {
    case 1: return pre + ".self_attn.q_proj.weight";
    case 2: return pre + ".self_attn.k_proj.weight";
    case 3: return pre + ".self_attn.v_proj.weight";
    case 4: return pre + ".self_attn.o_proj.weight";
    case 5: return pre + ".self_attn.q_norm.weight";
    case 6: return pre + ".self_attn.k_norm.weight";
    case 7: return pre + ".mlp.gate_proj.weight";
    case 8: return pre + ".mlp.up_proj.weight";
    case 9: return pre + ".mlp.down_proj.weight";
    case 10: return pre + ".input_layernorm.weight";
    case 11: return pre + ".post_attention_layernorm.weight";
    default: return "";
  }
}

std::unique_ptr<Checkpoint> Checkpoint::open(const std::string& directory) {
  auto ck = std::unique_ptr<Checkpoint>(new Checkpoint());
  ck->config_ = parse_config(directory);
  // tensor_files (weights.rs:59-75): the index's files, sorted and unique,
  // else model.safetensors
  std::vector<std::string> names;
  const std::string index = directory + "/model.safetensors.index.json";
  if (exists(index)) {
    const std::string text = read_text(index);
    const Json j = Parser(text.data(), text.data() + text.size(), index).parse();
    const Json* map = j.get("weight_map");
    if (!map || map->kind != Json::kObj) fail(MI_ERR_IO, "%s has no weight_map", index.c_str());
    std::set<std::string> uniq;
    for (const auto& kv : map->obj)
      if (kv.second.kind == Json::kStr) uniq.insert(kv.second.str);
    names.assign(uniq.begin(), uniq.end());
  } else if (exists(directory + "/model.safetensors")) {
    names.push_back("model.safetensors");
  } else {
    fail(MI_ERR_UNSUPPORTED, "unsupported model: %s contains neither model.safetensors nor its index",
         directory.c_str());
  }
  for (const auto& name : names) {
    const std::string path = directory + "/" + name;
    File f;
    f.fd = ::open(path.c_str(), O_RDONLY);
    if (f.fd < 0) fail(MI_ERR_IO, "cannot open %s", path.c_str());
    struct stat st;
    if (::fstat(f.fd, &st) != 0 || st.st_size < 8) {
      ::close(f.fd);
      fail(MI_ERR_IO, "%s is not a safetensors file", path.c_str());
    }
    f.size = (size_t)st.st_size;
    void* m = ::mmap(nullptr, f.size, PROT_READ, MAP_PRIVATE, f.fd, 0);
    if (m == MAP_FAILED) {
      ::close(f.fd);
      fail(MI_ERR_IO, "cannot map %s", path.c_str());
    }
    f.map = static_cast<const unsigned char*>(m);
    uint64_t hlen = 0;
    std::memcpy(&hlen, f.map, 8);  // little-endian hosts
    const int file_index = (int)ck->files_.size();
    ck->files_.push_back(f);
    if (hlen > f.size - 8) fail(MI_ERR_IO, "%s: header length past the end", path.c_str());
    ck->files_.back().data = 8 + hlen;
    const char* h = reinterpret_cast<const char*>(f.map + 8);
    const Json header = Parser(h, h + hlen, path).parse();
    if (header.kind != Json::kObj) fail(MI_ERR_IO, "%s: header is not an object", path.c_str());
    for (const auto& kv : header.obj) {
      if (kv.first == "__metadata__") continue;
      const Json* dt = kv.second.get("dtype");
      const Json* sh = kv.second.get("shape");
      const Json* off = kv.second.get("data_offsets");
      if (!dt || dt->kind != Json::kStr || !sh || sh->kind != Json::kArr || !off ||
          off->kind != Json::kArr || off->arr.size() != 2)
        fail(MI_ERR_IO, "%s: malformed entry for `%s`", path.c_str(), kv.first.c_str());
      TensorInfo t;
      t.dtype = dt->str;
      for (const auto& d : sh->arr) t.shape.push_back((size_t)d.num);
      t.begin = (size_t)off->arr[0].num;
      t.end = (size_t)off->arr[1].num;
      t.file = file_index;
      if (t.end < t.begin || ck->files_.back().data + t.end > f.size)
        fail(MI_ERR_IO, "%s: `%s` lies outside the file", path.c_str(), kv.first.c_str());
      ck->tensors_[kv.first] = t;
    }
  }
  return ck;
}

Checkpoint::~Checkpoint() {
  for (auto& f : files_) {
    if (f.map) ::munmap(const_cast<unsigned char*>(f.map), f.size);
    if (f.fd >= 0) ::close(f.fd);
  }
}

const TensorInfo& Checkpoint::expect(const std::string& name,
                                     const std::vector<size_t>& shape) const {
  auto it = tensors_.find(name);
  if (it == tensors_.end()) fail(MI_ERR_MISSING_TENSOR, "missing tensor `%s`", name.c_str());
  if (it->second.shape != shape) {
    std::string got, want;
    for (size_t d : it->second.shape) got += (got.empty() ? "" : ", ") + std::to_string(d);
    for (size_t d : shape) want += (want.empty() ? "" : ", ") + std::to_string(d);
    fail(MI_ERR_CONFIG, "invalid model configuration: %s has shape [%s], expected [%s]",
         name.c_str(), got.c_str(), want.c_str());
  }
  return it->second;
}

void Checkpoint::read_block(const std::string& name, size_t rows, size_t cols, size_t row0,
                            size_t col0, __half* dst, cudaStream_t stream) const {
  const TensorInfo& t = tensors_.at(name);
  if (t.dtype != "F16" && t.dtype != "BF16")
    fail(MI_ERR_UNSUPPORTED, "unsupported model: tensor `%s` uses %s; only F16 and BF16 are supported",
         name.c_str(), t.dtype.c_str());
  const size_t full_cols = t.shape.size() >= 2 ? t.shape.back() : (t.shape.empty() ? 1 : t.shape[0]);
  const size_t nbytes = (t.end - t.begin);
  const size_t elems = nbytes / 2;
  if (elems * 2 != nbytes || (row0 + rows) * full_cols > elems || col0 + cols > full_cols)
    fail(MI_ERR_DATA_LENGTH, "tensor `%s` holds %zu bytes, too few for the requested block",
         name.c_str(), nbytes);
  const File& f = files_[t.file];
  const unsigned char* src = f.map + f.data + t.begin;
  // gather the block on the host (contiguous when it is whole rows)
  std::vector<uint16_t> host(rows * cols);
  if (col0 == 0 && cols == full_cols) {
    std::memcpy(host.data(), src + row0 * full_cols * 2, rows * cols * 2);
  } else {
    for (size_t r = 0; r < rows; ++r)
      std::memcpy(host.data() + r * cols, src + ((row0 + r) * full_cols + col0) * 2, cols * 2);
  }
  const size_t n = rows * cols;
  if (t.dtype == "F16") {
    MI_CUDA(cudaMemcpyAsync(dst, host.data(), n * 2, cudaMemcpyHostToDevice, stream));
  } else {
    uint16_t* staging = nullptr;
    MI_CUDA(cudaMallocAsync(&staging, n * 2, stream));
    MI_CUDA(cudaMemcpyAsync(staging, host.data(), n * 2, cudaMemcpyHostToDevice, stream));
    const int grid = (int)std::min<size_t>((n + 255) / 256, 4096);
    bf16_to_f16_kernel<<<grid, 256, 0, stream>>>(staging, dst, n);
    MI_CUDA(cudaGetLastError());
    MI_CUDA(cudaFreeAsync(staging, stream));
  }
  // the host staging vector dies here: finish the copies first
  MI_CUDA(cudaStreamSynchronize(stream));
}

}  // namespace load
}  // namespace mi
