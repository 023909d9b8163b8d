// Model configuration and weight container of a Laya checkpoint directory: encoder/config.json
// (a ModernBertConfig), rl_agent_config.json and model.safetensors. Restates the reference loader
// src/laya.hpp:1-50 / src/laya.cpp:5-71 (same keys, same defaults, same derived fields).
#pragma once
#include <cstdint>
#include <map>
#include <string>
#include <vector>

namespace laya {

enum class AttnKind { Global, Sliding };

struct Config {
  int n_layers = 28, d = 1024, n_heads = 16, head_dim = 64, intermediate = 2624;
  int vocab = 50368, max_len = 512, head_max_len = 192, head_layers = 2, n_act = 2;
  int local_attention = 128;  // full window width; |q - k| <= local_attention / 2
  float norm_eps = 1e-5f;
  float rope_theta_global = 160000.f, rope_theta_local = 10000.f;
  int pad_id = 50283, cls_id = 50281, sep_id = 50282, mask_id = 50284;
  std::vector<AttnKind> layer_types;
  std::vector<float> temperature;  // per qtype
  std::map<std::string, float> temp_by_options;
  int head_ffn = 0;  // 4 * d

  // Throws std::runtime_error when the encoder config cannot be read or parsed. A missing agent
  // config keeps the defaults, as in the reference.
  static Config load(const std::string& encoder_cfg, const std::string& agent_cfg);
  void dump() const;
};

struct TensorView {
  const void* data = nullptr;
  std::vector<int64_t> shape;
  std::string dtype;  // F32, F16, BF16
  size_t nbytes = 0;
  int64_t numel() const {
    int64_t n = 1;
    for (auto s : shape) n *= s;
    return n;
  }
};

// Read-only memory map of a safetensors file; tensors are views into the mapping.
class SafeTensors {
 public:
  SafeTensors() = default;
  SafeTensors(const SafeTensors&) = delete;
  SafeTensors& operator=(const SafeTensors&) = delete;
  ~SafeTensors();
  bool open(const std::string& path, std::string* err);
  const TensorView* get(const std::string& name) const;
  // Converts a tensor to fp32 on the host (F32 copy, BF16 / F16 widening).
  bool to_f32(const std::string& name, std::vector<float>* out, std::string* err) const;

 private:
  int fd_ = -1;
  void* base_ = nullptr;
  size_t size_ = 0;
  std::map<std::string, TensorView> tensors_;
};

}  // namespace laya
