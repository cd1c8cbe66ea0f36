// Dory checkpoint files (checkpoint.h): the safetensors mapping and config.json.
//
// safetensors: an 8-byte little-endian header length N, N bytes of JSON {name: {"dtype", "shape",
// "data_offsets": [begin, end]}, "__metadata__": {...}}, then the data, offsets relative to its start.
#include <fcntl.h>
#include <sys/mman.h>
#include <sys/stat.h>
#include <unistd.h>

#include <cmath>
#include <cstring>
#include <fstream>
#include <sstream>

#include "checkpoint.h"
#include "common.cuh"
#include "json.h"

namespace xtg {

namespace {

std::string shape_str(const std::vector<int64_t>& s) {
  std::string r = "[";
  for (size_t i = 0; i < s.size(); ++i) r += (i ? ", " : "") + std::to_string(s[i]);
  return r + "]";
}

size_t dtype_bytes(const std::string& d) {
  if (d == "U8" || d == "I8" || d == "F8_E4M3" || d == "F8_E5M2" || d == "BOOL") return 1;
  if (d == "BF16" || d == "F16" || d == "I16" || d == "U16") return 2;
  if (d == "F32" || d == "I32" || d == "U32") return 4;
  if (d == "F64" || d == "I64" || d == "U64") return 8;
  return 0;
}

}  // namespace

SafeTensors::SafeTensors(const std::string& path) : path_(path) {
  const int fd = ::open(path.c_str(), O_RDONLY);
  if (fd < 0) throw CudaError(path + ": " + std::strerror(errno));
  struct stat st;
  if (::fstat(fd, &st) != 0) {
    ::close(fd);
    throw CudaError(path + ": " + std::strerror(errno));
  }
  size_ = (size_t)st.st_size;
  if (size_ < 8) {
    ::close(fd);
    throw CudaError(path + ": not a safetensors file (shorter than its header length)");
  }
  map_ = ::mmap(nullptr, size_, PROT_READ, MAP_PRIVATE, fd, 0);
  ::close(fd);
  if (map_ == MAP_FAILED) {
    map_ = nullptr;
    throw CudaError(path + ": mmap failed");
  }
  const uint8_t* base = static_cast<const uint8_t*>(map_);
  uint64_t n = 0;
  for (int i = 0; i < 8; ++i) n |= (uint64_t)base[i] << (8 * i);
  if (n == 0 || n > size_ - 8) {
    ::munmap(map_, size_);
    map_ = nullptr;
    throw CudaError(path + ": bad safetensors header length");
  }
  const uint8_t* data = base + 8 + n;
  const size_t data_bytes = size_ - 8 - n;
  try {
    const Json h = Json::parse(std::string(reinterpret_cast<const char*>(base + 8), (size_t)n));
    if (h.kind != Json::Object) throw CudaError("the header is not a JSON object");
    for (const auto& kv : h.obj) {
      if (kv.first == "__metadata__") continue;
      const Json& e = kv.second;
      TensorView t;
      t.dtype = e.string("dtype", "");
      const Json& sh = e.at("shape");
      const Json& off = e.at("data_offsets");
      if (sh.kind != Json::Array || off.kind != Json::Array || off.arr.size() != 2)
        throw CudaError("tensor " + kv.first + ": no shape or data_offsets");
      size_t elems = 1;
      for (const Json& d : sh.arr) {
        if (d.kind != Json::Number || d.num < 0) throw CudaError("tensor " + kv.first + ": bad shape");
        t.shape.push_back((int64_t)d.num);
        elems *= (size_t)d.num;
      }
      const double b = off.arr[0].num, en = off.arr[1].num;
      if (!(b >= 0 && en >= b && en <= (double)data_bytes))
        throw CudaError("tensor " + kv.first + ": data_offsets outside the file");
      t.data = data + (size_t)b;
      t.bytes = (size_t)(en - b);
      const size_t eb = dtype_bytes(t.dtype);
      if (eb && t.bytes != elems * eb)
        throw CudaError("tensor " + kv.first + ": " + std::to_string(t.bytes) + " bytes for " + t.dtype + " " +
                        shape_str(t.shape));
      t_[kv.first] = std::move(t);
    }
  } catch (const std::exception& e) {
    ::munmap(map_, size_);
    map_ = nullptr;
    throw CudaError(path + ": " + e.what());
  }
}

SafeTensors::~SafeTensors() {
  if (map_) ::munmap(map_, size_);
}

const TensorView& SafeTensors::get(const std::string& name, const char* dtype,
                                   const std::vector<int64_t>& shape) const {
  auto it = t_.find(name);
  if (it == t_.end()) throw CudaError(path_ + ": no tensor " + name);
  const TensorView& t = it->second;
  if (t.dtype != dtype) throw CudaError(path_ + ": " + name + " is " + t.dtype + ", expected " + dtype);
  if (t.shape != shape)
    throw CudaError(path_ + ": " + name + " has shape " + shape_str(t.shape) + ", expected " + shape_str(shape));
  return t;
}

DoryConfig read_dory_config(const std::string& dir) {
  std::ifstream f(dir + "/config.json");
  if (!f) throw CudaError(dir + ": no config.json");
  std::stringstream ss;
  ss << f.rdbuf();
  Json c;
  try {
    c = Json::parse(ss.str());
  } catch (const std::exception& e) {
    throw CudaError(dir + "/config.json: " + e.what());
  }
  auto need = [&](const char* k) -> const Json& {
    if (!c.has(k)) throw CudaError(dir + ": config.json has no " + k);
    return c.at(k);
  };
  auto num = [&](const char* k) {
    const Json& v = need(k);
    if (v.kind != Json::Number) throw CudaError(dir + ": config.json " + k + " is not a number");
    return v.num;
  };
  DoryConfig k;
  if (c.string("model_type", "") != "dory") throw CudaError(dir + ": not a Dory checkpoint");
  k.hidden = (int)num("hidden_size");
  k.ffn = (int)num("intermediate_size");
  k.heads = (int)num("num_attention_heads");
  k.kv_heads = (int)num("num_key_value_heads");
  k.head_dim = (int)num("head_dim");
  k.vocab = (int)num("vocab_size");
  k.layers = (int)num("num_hidden_layers");
  k.n_in = (int)num("n_input_layers");
  k.n_rec = (int)num("n_recurrent_layers");
  k.n_out = (int)num("n_output_layers");
  k.window = (int)c.number("sliding_window", 0);
  k.default_loops = (int)c.number("n_recurrent_loops", 1);
  k.kv_mode = c.string("recurrent_kv_cache_mode", "per_loop");
  k.max_pos = (int64_t)num("max_position_embeddings");
  k.init_range = (float)num("initializer_range");
  k.alpha_init = (float)num("ngpt_alpha_init");
  k.gate_init = c.has("attention_output_gate_logit_scale_init")
                    ? (float)c.number("attention_output_gate_logit_scale_init", 0)
                    : std::sqrt((float)k.hidden);
  if (k.n_in + k.n_rec + k.n_out != k.layers)
    throw CudaError(dir + ": input + recurrent + output layers != " + std::to_string(k.layers));
  if (k.kv_heads <= 0 || k.heads % k.kv_heads || k.head_dim % 2)
    throw CudaError(dir + ": unsupported attention shape");
  if (c.at("attention_bias").kind == Json::Bool && c.at("attention_bias").b)
    throw CudaError(dir + ": Dory has no biases");
  if (c.at("mlp_bias").kind == Json::Bool && c.at("mlp_bias").b) throw CudaError(dir + ": Dory has no biases");
  if (c.string("hidden_act", "silu") != "silu" ||
      (c.at("tie_word_embeddings").kind == Json::Bool && c.at("tie_word_embeddings").b))
    throw CudaError(dir + ": Dory uses SiLU and untied embeddings");
  const Json& types = need("layer_types");
  if (types.kind != Json::Array) throw CudaError(dir + ": layer_types is not a list");
  for (const Json& t : types.arr) {
    if (t.kind != Json::String) throw CudaError(dir + ": layer_types holds a non-string");
    if (t.str == "mlp")
      k.kind.push_back(0);
    else if (t.str == "sliding_attention")
      k.kind.push_back(1);
    else if (t.str == "full_attention")
      k.kind.push_back(2);
    else
      throw CudaError(dir + ": unknown layer type " + t.str);
  }
  if ((int)k.kind.size() != k.layers)
    throw CudaError(dir + ": layer_types has " + std::to_string(k.kind.size()) + " entries");
  const Json& rope = need("rope_parameters");
  const char* keys[2] = {"sliding_attention", "full_attention"};
  float* thetas[2] = {&k.theta_sliding, &k.theta_global};
  for (int i = 0; i < 2; ++i) {
    const Json& r = rope.at(keys[i]);
    if (r.kind == Json::Null) continue;
    if (r.string("rope_type", "default") != "default" || r.number("partial_rotary_factor", 1.0) != 1.0)
      throw CudaError(dir + ": only default full-width RoPE is supported");
    *thetas[i] = (float)r.number("rope_theta", 0);
  }
  for (int t : k.kind)
    if ((t == 1 && !(k.theta_sliding > 0)) || (t == 2 && !(k.theta_global > 0)))
      throw CudaError(dir + ": a layer type has no rope_theta");
  for (int t : k.kind)
    if (t == 1 && k.window <= 0) throw CudaError(dir + ": sliding layers without a window");
  if (c.at("quantization_config").string("quant_algo", "") != "W4A16_NVFP4")
    throw CudaError(dir + ": only the W4A16_NVFP4 (ModelOpt) checkpoint is supported");
  return k;
}

}  // namespace xtg
