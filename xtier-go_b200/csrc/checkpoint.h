// Dory checkpoints on disk: a ModelOpt W4A16_NVFP4 export, a directory holding config.json and model.safetensors
// (the layout packs/dory/dory.cpp reads). Host code only: the file is mapped read-only and tensors are handed out
// as views into the mapping, checked for dtype and shape like engine/src/safetensors.cpp:36-100 does.
#pragma once

#include <stddef.h>
#include <stdint.h>

#include <map>
#include <string>
#include <vector>

namespace xtg {

struct TensorView {
  std::string dtype;              // "U8", "F8_E4M3", "F32", "BF16", ...
  std::vector<int64_t> shape;
  const uint8_t* data = nullptr;  // inside the mapping
  size_t bytes = 0;
};

class SafeTensors {
 public:
  explicit SafeTensors(const std::string& path);
  ~SafeTensors();
  SafeTensors(const SafeTensors&) = delete;
  SafeTensors& operator=(const SafeTensors&) = delete;
  bool has(const std::string& name) const { return t_.count(name) != 0; }
  // the tensor `name`, which must have this dtype and shape (an empty shape: a scalar)
  const TensorView& get(const std::string& name, const char* dtype, const std::vector<int64_t>& shape) const;
  size_t file_size() const { return size_; }

 private:
  std::string path_;
  void* map_ = nullptr;
  size_t size_ = 0;
  std::map<std::string, TensorView> t_;
};

// config.json of a Dory checkpoint (packs/dory/dory.cpp:77-134): shapes, the sublayer kinds, RoPE thetas and the
// constants that fold the stored scales.
struct DoryConfig {
  int hidden = 0, ffn = 0, heads = 0, kv_heads = 0, head_dim = 0, vocab = 0;
  int layers = 0, n_in = 0, n_rec = 0, n_out = 0;
  int window = 0, default_loops = 1;
  std::string kv_mode = "per_loop";
  int64_t max_pos = 0;
  float init_range = 0.f, alpha_init = 0.f, gate_init = 0.f;
  float theta_sliding = 0.f, theta_global = 0.f;
  std::vector<int> kind;   // per physical sublayer: 0 MLP, 1 sliding attention, 2 full attention
};

// Reads and checks dir/config.json (a Dory, W4A16_NVFP4, no biases, SiLU, untied head, known layer types).
DoryConfig read_dory_config(const std::string& dir);

// bf16 bits -> f32 (exact)
inline float bf16_bits_f32(uint16_t h) {
  const uint32_t u = (uint32_t)h << 16;
  float f;
  __builtin_memcpy(&f, &u, 4);
  return f;
}

}  // namespace xtg
