// Minimal JSON reader for the wire program handed across the C ABI.
// Supports objects, arrays, numbers (kept as double), strings, true/false/null.
#pragma once
#include <cmath>
#include <cstdint>
#include <cstdlib>
#include <cstring>
#include <stdexcept>
#include <string>
#include <utility>
#include <vector>

namespace tgjson {

struct Value {
  enum Kind { Null, Bool, Num, Str, Arr, Obj } kind = Null;
  bool b = false;
  double n = 0;
  std::string s;
  std::vector<Value> a;
  std::vector<std::pair<std::string, Value>> o;  // insertion order preserved

  bool is_null() const { return kind == Null; }
  const Value* find(const std::string& k) const {
    for (auto& kv : o) if (kv.first == k) return &kv.second;
    return nullptr;
  }
  const Value& operator[](const std::string& k) const {
    const Value* v = find(k);
    if (!v) throw std::runtime_error("json: missing key '" + k + "'");
    return *v;
  }
  const Value& operator[](size_t i) const { return a.at(i); }
  double num() const {
    if (kind == Bool) return b ? 1.0 : 0.0;
    if (kind != Num) throw std::runtime_error("json: expected number");
    return n;
  }
  int64_t i64() const { return (int64_t)num(); }
  int i32() const { return (int)num(); }
  const std::string& str() const {
    if (kind != Str) throw std::runtime_error("json: expected string");
    return s;
  }
  size_t size() const { return kind == Arr ? a.size() : o.size(); }
};

class Parser {
 public:
  Parser(const char* p, size_t n) : p_(p), end_(p + n) {}
  Value parse() {
    Value v = value();
    ws();
    if (p_ != end_) throw std::runtime_error("json: trailing characters");
    return v;
  }

 private:
  const char* p_;
  const char* end_;
  void ws() { while (p_ < end_ && (*p_ == ' ' || *p_ == '\n' || *p_ == '\r' || *p_ == '\t')) ++p_; }
  bool lit(const char* s) {
    size_t n = strlen(s);
    if ((size_t)(end_ - p_) >= n && memcmp(p_, s, n) == 0) { p_ += n; return true; }
    return false;
  }
  Value value() {
    ws();
    if (p_ >= end_) throw std::runtime_error("json: unexpected end");
    Value v;
    char c = *p_;
    if (c == '{') {
      v.kind = Value::Obj; ++p_; ws();
      if (p_ < end_ && *p_ == '}') { ++p_; return v; }
      for (;;) {
        ws();
        std::string k = string();
        ws();
        if (p_ >= end_ || *p_ != ':') throw std::runtime_error("json: expected ':'");
        ++p_;
        v.o.emplace_back(std::move(k), value());
        ws();
        if (p_ < end_ && *p_ == ',') { ++p_; continue; }
        if (p_ < end_ && *p_ == '}') { ++p_; return v; }
        throw std::runtime_error("json: expected ',' or '}'");
      }
    }
    if (c == '[') {
      v.kind = Value::Arr; ++p_; ws();
      if (p_ < end_ && *p_ == ']') { ++p_; return v; }
      for (;;) {
        v.a.push_back(value());
        ws();
        if (p_ < end_ && *p_ == ',') { ++p_; continue; }
        if (p_ < end_ && *p_ == ']') { ++p_; return v; }
        throw std::runtime_error("json: expected ',' or ']'");
      }
    }
    if (c == '"') { v.kind = Value::Str; v.s = string(); return v; }
    if (lit("true")) { v.kind = Value::Bool; v.b = true; return v; }
    if (lit("false")) { v.kind = Value::Bool; v.b = false; return v; }
    if (lit("null")) { return v; }
    if (lit("NaN")) { v.kind = Value::Num; v.n = std::nan(""); return v; }
    if (lit("Infinity")) { v.kind = Value::Num; v.n = HUGE_VAL; return v; }
    if (lit("-Infinity")) { v.kind = Value::Num; v.n = -HUGE_VAL; return v; }
    char* e = nullptr;
    v.kind = Value::Num;
    v.n = strtod(p_, &e);
    if (e == p_) throw std::runtime_error("json: bad value");
    p_ = e;
    return v;
  }
  std::string string() {
    if (p_ >= end_ || *p_ != '"') throw std::runtime_error("json: expected string");
    ++p_;
    std::string out;
    while (p_ < end_ && *p_ != '"') {
      if (*p_ == '\\') {
        ++p_;
        if (p_ >= end_) break;
        char e = *p_++;
        switch (e) {
          case 'n': out += '\n'; break;
          case 't': out += '\t'; break;
          case 'r': out += '\r'; break;
          case 'b': out += '\b'; break;
          case 'f': out += '\f'; break;
          case 'u': {
            if (end_ - p_ < 4) throw std::runtime_error("json: bad escape");
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
    if (p_ >= end_) throw std::runtime_error("json: unterminated string");
    ++p_;
    return out;
  }
};

inline Value parse(const char* p, size_t n) { return Parser(p, n).parse(); }

}  // namespace tgjson
