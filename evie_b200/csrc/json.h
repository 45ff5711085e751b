// Minimal JSON reader for config.json and safetensors headers (objects, arrays, strings, numbers, bools, null).
#pragma once

#include <cstdint>
#include <cstdlib>
#include <map>
#include <memory>
#include <stdexcept>
#include <string>
#include <vector>

namespace evie {
namespace json {

struct Value {
  enum Kind { Null, Bool, Number, String, Array, Object } kind = Null;
  bool b = false;
  double num = 0;
  std::string str;
  std::vector<Value> arr;
  std::map<std::string, Value> obj;

  bool is_null() const { return kind == Null; }
  bool has(const std::string& k) const { return kind == Object && obj.count(k) && !obj.at(k).is_null(); }
  const Value& operator[](const std::string& k) const {
    static const Value null_value;
    if (kind != Object) return null_value;
    auto it = obj.find(k);
    return it == obj.end() ? null_value : it->second;
  }
  double number() const {
    if (kind != Number) throw std::runtime_error("expected a number");
    return num;
  }
  int64_t integer() const { return (int64_t)number(); }
  const std::string& string() const {
    if (kind != String) throw std::runtime_error("expected a string");
    return str;
  }
};

class Parser {
 public:
  Parser(const char* p, const char* end) : p_(p), end_(end) {}
  Value parse() {
    Value v = value();
    ws();
    return v;
  }

 private:
  const char* p_;
  const char* end_;
  [[noreturn]] void error(const char* what) { throw std::runtime_error(std::string("json: ") + what); }
  void ws() {
    while (p_ < end_ && (*p_ == ' ' || *p_ == '\n' || *p_ == '\t' || *p_ == '\r')) p_++;
  }
  bool lit(const char* s) {
    const char* q = p_;
    for (; *s; s++, q++)
      if (q >= end_ || *q != *s) return false;
    p_ = q;
    return true;
  }
  Value value() {
    ws();
    if (p_ >= end_) error("unexpected end");
    Value v;
    char c = *p_;
    if (c == '{') {
      v.kind = Value::Object;
      p_++;
      ws();
      if (p_ < end_ && *p_ == '}') {
        p_++;
        return v;
      }
      for (;;) {
        ws();
        if (p_ >= end_ || *p_ != '"') error("expected key");
        std::string k = string_lit();
        ws();
        if (p_ >= end_ || *p_ != ':') error("expected ':'");
        p_++;
        v.obj[k] = value();
        ws();
        if (p_ < end_ && *p_ == ',') { p_++; continue; }
        if (p_ < end_ && *p_ == '}') { p_++; break; }
        error("expected ',' or '}'");
      }
    } else if (c == '[') {
      v.kind = Value::Array;
      p_++;
      ws();
      if (p_ < end_ && *p_ == ']') {
        p_++;
        return v;
      }
      for (;;) {
        v.arr.push_back(value());
        ws();
        if (p_ < end_ && *p_ == ',') { p_++; continue; }
        if (p_ < end_ && *p_ == ']') { p_++; break; }
        error("expected ',' or ']'");
      }
    } else if (c == '"') {
      v.kind = Value::String;
      v.str = string_lit();
    } else if (lit("true")) {
      v.kind = Value::Bool;
      v.b = true;
    } else if (lit("false")) {
      v.kind = Value::Bool;
    } else if (lit("null")) {
      v.kind = Value::Null;
    } else {
      char* q = nullptr;
      std::string tmp(p_, std::min<size_t>(64, end_ - p_));
      v.num = strtod(tmp.c_str(), &q);
      if (q == tmp.c_str()) error("bad value");
      v.kind = Value::Number;
      p_ += q - tmp.c_str();
    }
    return v;
  }
  std::string string_lit() {
    p_++;  // opening quote
    std::string out;
    while (p_ < end_ && *p_ != '"') {
      if (*p_ == '\\') {
        p_++;
        if (p_ >= end_) error("bad escape");
        char e = *p_++;
        switch (e) {
          case 'n': out += '\n'; break;
          case 't': out += '\t'; break;
          case 'r': out += '\r'; break;
          case 'b': out += '\b'; break;
          case 'f': out += '\f'; break;
          case 'u': {
            if (end_ - p_ < 4) error("bad \\u escape");
            unsigned cp = (unsigned)strtoul(std::string(p_, 4).c_str(), nullptr, 16);
            p_ += 4;
            if (cp < 0x80) out += (char)cp;
            else if (cp < 0x800) { out += (char)(0xC0 | (cp >> 6)); out += (char)(0x80 | (cp & 0x3F)); }
            else { out += (char)(0xE0 | (cp >> 12)); out += (char)(0x80 | ((cp >> 6) & 0x3F)); out += (char)(0x80 | (cp & 0x3F)); }
            break;
          }
          default: out += e;
        }
      } else {
        out += *p_++;
      }
    }
    if (p_ >= end_) error("unterminated string");
    p_++;
    return out;
  }
};

inline Value parse(const std::string& s) { return Parser(s.data(), s.data() + s.size()).parse(); }
inline Value parse(const char* p, size_t n) { return Parser(p, p + n).parse(); }

}  // namespace json
}  // namespace evie
