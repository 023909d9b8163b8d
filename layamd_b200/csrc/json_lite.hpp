// A small JSON reader for the two config files and the safetensors header: objects, arrays,
// strings (with escapes), numbers, booleans and null. Parse errors throw std::runtime_error.
#pragma once
#include <cmath>
#include <cstdlib>
#include <map>
#include <memory>
#include <stdexcept>
#include <string>
#include <vector>

namespace laya {
namespace json {

struct Value {
  enum Kind { Null, Bool, Number, String, Array, Object } kind = Null;
  bool b = false;
  double num = 0.0;
  std::string str;
  std::vector<Value> arr;
  std::vector<std::pair<std::string, Value>> obj;  // insertion order kept

  bool is_object() const { return kind == Object; }
  bool is_array() const { return kind == Array; }
  bool is_number() const { return kind == Number; }
  bool is_string() const { return kind == String; }
  const Value* find(const std::string& k) const {
    if (kind != Object) return nullptr;
    for (const auto& kv : obj)
      if (kv.first == k) return &kv.second;
    return nullptr;
  }
  double number_or(const std::string& k, double d) const {
    const Value* v = find(k);
    return v && v->kind == Number ? v->num : d;
  }
  std::string string_or(const std::string& k, const std::string& d) const {
    const Value* v = find(k);
    return v && v->kind == String ? v->str : d;
  }
};

class Parser {
 public:
  explicit Parser(const std::string& s) : s_(s) {}
  Value parse() {
    Value v = value();
    ws();
    if (i_ != s_.size()) fail("trailing characters");
    return v;
  }

 private:
  const std::string& s_;
  size_t i_ = 0;
  [[noreturn]] void fail(const char* why) {
    throw std::runtime_error(std::string("json: ") + why + " at offset " + std::to_string(i_));
  }
  void ws() {
    while (i_ < s_.size() && (s_[i_] == ' ' || s_[i_] == '\n' || s_[i_] == '\r' || s_[i_] == '\t')) ++i_;
  }
  bool eat(char c) {
    ws();
    if (i_ < s_.size() && s_[i_] == c) { ++i_; return true; }
    return false;
  }
  Value value() {
    ws();
    if (i_ >= s_.size()) fail("unexpected end");
    const char c = s_[i_];
    Value v;
    if (c == '{') {
      ++i_;
      v.kind = Value::Object;
      if (eat('}')) return v;
      do {
        ws();
        if (i_ >= s_.size() || s_[i_] != '"') fail("expected key");
        std::string k = string();
        if (!eat(':')) fail("expected ':'");
        v.obj.emplace_back(std::move(k), value());
      } while (eat(','));
      if (!eat('}')) fail("expected '}'");
    } else if (c == '[') {
      ++i_;
      v.kind = Value::Array;
      if (eat(']')) return v;
      do { v.arr.push_back(value()); } while (eat(','));
      if (!eat(']')) fail("expected ']'");
    } else if (c == '"') {
      v.kind = Value::String;
      v.str = string();
    } else if (s_.compare(i_, 4, "true") == 0) {
      i_ += 4; v.kind = Value::Bool; v.b = true;
    } else if (s_.compare(i_, 5, "false") == 0) {
      i_ += 5; v.kind = Value::Bool; v.b = false;
    } else if (s_.compare(i_, 4, "null") == 0) {
      i_ += 4;
    } else if (s_.compare(i_, 3, "NaN") == 0) {
      i_ += 3; v.kind = Value::Number; v.num = NAN;
    } else {
      const char* p = s_.c_str() + i_;
      char* e = nullptr;
      v.num = std::strtod(p, &e);
      if (e == p) fail("bad value");
      i_ += static_cast<size_t>(e - p);
      v.kind = Value::Number;
    }
    return v;
  }
  std::string string() {
    ++i_;  // opening quote
    std::string out;
    while (i_ < s_.size() && s_[i_] != '"') {
      char c = s_[i_++];
      if (c != '\\') { out.push_back(c); continue; }
      if (i_ >= s_.size()) fail("bad escape");
      const char e = s_[i_++];
      switch (e) {
        case 'n': out.push_back('\n'); break;
        case 't': out.push_back('\t'); break;
        case 'r': out.push_back('\r'); break;
        case 'b': out.push_back('\b'); break;
        case 'f': out.push_back('\f'); break;
        case 'u': {
          if (i_ + 4 > s_.size()) fail("bad \\u escape");
          const unsigned cp = static_cast<unsigned>(std::strtoul(s_.substr(i_, 4).c_str(), nullptr, 16));
          i_ += 4;
          if (cp < 0x80) out.push_back(static_cast<char>(cp));
          else if (cp < 0x800) { out.push_back(static_cast<char>(0xC0 | (cp >> 6))); out.push_back(static_cast<char>(0x80 | (cp & 0x3F))); }
          else { out.push_back(static_cast<char>(0xE0 | (cp >> 12))); out.push_back(static_cast<char>(0x80 | ((cp >> 6) & 0x3F))); out.push_back(static_cast<char>(0x80 | (cp & 0x3F))); }
          break;
        }
        default: out.push_back(e);
      }
    }
    if (i_ >= s_.size()) fail("unterminated string");
    ++i_;
    return out;
  }
};

inline Value parse(const std::string& s) { return Parser(s).parse(); }

}  // namespace json
}  // namespace laya
