// Config parsing and safetensors mapping; see model_files.hpp. Key names and defaults follow the
// reference's Config::load (src/laya.cpp:5-41); rope thetas are also accepted under the older
// transformers key names global_rope_theta / local_rope_theta.
#include "model_files.hpp"

#include <fcntl.h>
#include <sys/mman.h>
#include <sys/stat.h>
#include <unistd.h>

#include <cmath>
#include <cstdio>
#include <cstring>
#include <fstream>
#include <sstream>
#include <stdexcept>

#include "json_lite.hpp"

namespace laya {

namespace {
bool read_file(const std::string& path, std::string* out) {
  std::ifstream f(path, std::ios::binary);
  if (!f) return false;
  std::stringstream ss;
  ss << f.rdbuf();
  *out = ss.str();
  return true;
}
int as_int(const json::Value& j, const char* k, int d) { return static_cast<int>(j.number_or(k, d)); }

float half_to_float(uint16_t h) {
  const uint32_t sign = (h >> 15) & 1, exp = (h >> 10) & 0x1F, man = h & 0x3FF;
  float v;
  if (exp == 0) v = std::ldexp(static_cast<float>(man), -24);
  else if (exp == 31) v = man ? NAN : INFINITY;
  else v = std::ldexp(static_cast<float>(man | 0x400), static_cast<int>(exp) - 25);
  return sign ? -v : v;
}
}  // namespace

Config Config::load(const std::string& encoder_cfg, const std::string& agent_cfg) {
  Config c;
  std::string s;
  if (!read_file(encoder_cfg, &s)) throw std::runtime_error("cannot open " + encoder_cfg);
  const json::Value j = json::parse(s);
  c.n_layers = as_int(j, "num_hidden_layers", 28);
  c.d = as_int(j, "hidden_size", 1024);
  c.n_heads = as_int(j, "num_attention_heads", 16);
  c.head_dim = c.d / c.n_heads;
  c.intermediate = as_int(j, "intermediate_size", 2624);
  c.vocab = as_int(j, "vocab_size", 50368);
  c.local_attention = as_int(j, "local_attention", 128);
  c.norm_eps = static_cast<float>(j.number_or("norm_eps", j.number_or("layer_norm_eps", 1e-5)));
  c.pad_id = as_int(j, "pad_token_id", 50283);
  c.cls_id = as_int(j, "cls_token_id", 50281);
  c.sep_id = as_int(j, "sep_token_id", 50282);
  c.mask_id = as_int(j, "mask_token_id", 50284);
  c.rope_theta_global = static_cast<float>(j.number_or("global_rope_theta", 160000.0));
  c.rope_theta_local = static_cast<float>(j.number_or("local_rope_theta", 10000.0));
  if (const json::Value* rp = j.find("rope_parameters")) {
    if (const json::Value* g = rp->find("full_attention"))
      c.rope_theta_global = static_cast<float>(g->number_or("rope_theta", 160000.0));
    if (const json::Value* l = rp->find("sliding_attention"))
      c.rope_theta_local = static_cast<float>(l->number_or("rope_theta", 10000.0));
  }
  const json::Value* lt = j.find("layer_types");
  if (lt && lt->is_array()) {
    for (const auto& t : lt->arr)
      c.layer_types.push_back(t.str == "full_attention" ? AttnKind::Global : AttnKind::Sliding);
  } else {
    const int every = as_int(j, "global_attn_every_n_layers", 3);
    for (int i = 0; i < c.n_layers; ++i) c.layer_types.push_back(i % every == 0 ? AttnKind::Global : AttnKind::Sliding);
  }
  if ((int)c.layer_types.size() != c.n_layers) throw std::runtime_error("layer_types length != num_hidden_layers");
  if (read_file(agent_cfg, &s)) {
    const json::Value g = json::parse(s);
    c.max_len = as_int(g, "max_len", 512);
    c.head_max_len = as_int(g, "head_max_len", 192);
    c.head_layers = as_int(g, "head_layers", 2);
    if (const json::Value* ac = g.find("act_costs"))
      if (ac->is_array()) c.n_act = static_cast<int>(ac->arr.size()) + 1;
    if (const json::Value* t = g.find("temperature"))
      if (t->is_array())
        for (const auto& v : t->arr) c.temperature.push_back(static_cast<float>(v.num));
    if (const json::Value* t = g.find("temperature_by_options"))
      if (t->is_object())
        for (const auto& kv : t->obj) c.temp_by_options[kv.first] = static_cast<float>(kv.second.num);
  }
  if (c.temperature.empty()) c.temperature = {1.f, 1.f, 1.f};
  c.head_ffn = 4 * c.d;
  return c;
}

void Config::dump() const {
  int ng = 0;
  for (auto k : layer_types) ng += k == AttnKind::Global;
  printf("[laya] layers=%d d=%d heads=%d head_dim=%d ffn=%d vocab=%d max_len=%d\n", n_layers, d, n_heads, head_dim,
         intermediate, vocab, max_len);
  printf("[laya] attn: %d global / %d sliding (window=%d) rope theta g=%.0f l=%.0f eps=%g\n", ng, n_layers - ng,
         local_attention, rope_theta_global, rope_theta_local, norm_eps);
  printf("[laya] head: %d layers ffn=%d n_act=%d temps=[%.4f %.4f %.4f]\n", head_layers, head_ffn, n_act,
         temperature.size() > 0 ? temperature[0] : 1.f, temperature.size() > 1 ? temperature[1] : 1.f,
         temperature.size() > 2 ? temperature[2] : 1.f);
}

SafeTensors::~SafeTensors() {
  if (base_ && base_ != MAP_FAILED) munmap(base_, size_);
  if (fd_ >= 0) ::close(fd_);
}

bool SafeTensors::open(const std::string& path, std::string* err) {
  fd_ = ::open(path.c_str(), O_RDONLY);
  if (fd_ < 0) { *err = "open " + path + " failed"; return false; }
  struct stat st;
  if (fstat(fd_, &st) != 0 || st.st_size < 8) { *err = path + ": not a safetensors file"; return false; }
  size_ = static_cast<size_t>(st.st_size);
  base_ = mmap(nullptr, size_, PROT_READ, MAP_PRIVATE, fd_, 0);
  if (base_ == MAP_FAILED) { base_ = nullptr; *err = "mmap failed"; return false; }
  uint64_t hlen;
  memcpy(&hlen, base_, 8);
  if (8 + hlen > size_) { *err = path + ": bad header length"; return false; }
  const size_t data_off = 8 + hlen;
  json::Value hdr;
  try {
    hdr = json::parse(std::string(static_cast<const char*>(base_) + 8, hlen));
  } catch (const std::exception& e) {
    *err = e.what();
    return false;
  }
  for (const auto& kv : hdr.obj) {
    if (kv.first == "__metadata__") continue;
    TensorView t;
    t.dtype = kv.second.string_or("dtype", "");
    if (const json::Value* sh = kv.second.find("shape"))
      for (const auto& d : sh->arr) t.shape.push_back(static_cast<int64_t>(d.num));
    const json::Value* off = kv.second.find("data_offsets");
    if (!off || off->arr.size() != 2) { *err = kv.first + ": no data_offsets"; return false; }
    const size_t a = static_cast<size_t>(off->arr[0].num), b = static_cast<size_t>(off->arr[1].num);
    if (b < a || data_off + b > size_) { *err = kv.first + ": offsets out of range"; return false; }
    t.nbytes = b - a;
    t.data = static_cast<const char*>(base_) + data_off + a;
    tensors_[kv.first] = t;
  }
  return true;
}

const TensorView* SafeTensors::get(const std::string& name) const {
  auto it = tensors_.find(name);
  return it == tensors_.end() ? nullptr : &it->second;
}

bool SafeTensors::to_f32(const std::string& name, std::vector<float>* out, std::string* err) const {
  const TensorView* t = get(name);
  if (!t) { *err = "missing tensor " + name; return false; }
  const int64_t n = t->numel();
  out->resize(static_cast<size_t>(n));
  if (t->dtype == "F32" && t->nbytes == (size_t)n * 4) {
    memcpy(out->data(), t->data, t->nbytes);
  } else if (t->dtype == "BF16" && t->nbytes == (size_t)n * 2) {
    const uint16_t* p = static_cast<const uint16_t*>(t->data);
    for (int64_t i = 0; i < n; ++i) {
      const uint32_t u = static_cast<uint32_t>(p[i]) << 16;
      memcpy(&(*out)[i], &u, 4);
    }
  } else if (t->dtype == "F16" && t->nbytes == (size_t)n * 2) {
    const uint16_t* p = static_cast<const uint16_t*>(t->data);
    for (int64_t i = 0; i < n; ++i) (*out)[i] = half_to_float(p[i]);
  } else {
    *err = name + ": unsupported dtype " + t->dtype;
    return false;
  }
  return true;
}

}  // namespace laya
