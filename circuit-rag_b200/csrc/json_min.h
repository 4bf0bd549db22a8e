// Minimal JSON reader for the .circuit header (objects, arrays, strings,
// numbers, true/false/null).  The reference native loader finds keys by
// substring search (reference native/src/gpu_index.cpp:13-48); this parses the
// header properly so key order, spacing and nested names cannot confuse it.
#pragma once

#include <cstdint>
#include <cstdlib>
#include <map>
#include <memory>
#include <string>
#include <vector>

namespace cb {
namespace json {

struct Value {
  enum Kind { Null, Bool, Number, String, Array, Object } kind = Null;
  bool b = false;
  double num = 0.0;
  std::string raw_number;  // exact text of a number (for 64-bit integers)
  std::string str;
  std::vector<Value> arr;
  std::map<std::string, Value> obj;

  const Value* get(const std::string& key) const {
    if (kind != Object) return nullptr;
    auto it = obj.find(key);
    return it == obj.end() ? nullptr : &it->second;
  }
  bool as_int64(int64_t* out) const {
    if (kind != Number || raw_number.empty()) return false;
    for (char c : raw_number)
      if (!(c == '-' || (c >= '0' && c <= '9'))) return false;
    char* end = nullptr;
    long long v = std::strtoll(raw_number.c_str(), &end, 10);
    if (!end || *end != '\0') return false;
    *out = (int64_t)v;
    return true;
  }
};

class Parser {
 public:
  Parser(const char* s, size_t n) : p_(s), end_(s + n) {}
  bool parse(Value* out) {
    skip();
    if (!value(out, 0)) return false;
    skip();
    // then only the header block's zero padding (as json.loads of the text
    // with its trailing NULs stripped: whitespace after a NUL is not allowed)
    while (p_ < end_ && *p_ == '\0') ++p_;
    return p_ == end_;
  }

 private:
  const char* p_;
  const char* end_;
  static bool is_ws(char c) { return c == ' ' || c == '\t' || c == '\n' || c == '\r'; }
  void skip() {
    while (p_ < end_ && is_ws(*p_)) ++p_;
  }
  bool lit(const char* w) {
    const char* q = p_;
    for (; *w; ++w, ++q)
      if (q >= end_ || *q != *w) return false;
    p_ = q;
    return true;
  }
  bool value(Value* v, int depth) {
    if (depth > 32 || p_ >= end_) return false;
    char c = *p_;
    if (c == '{') return object(v, depth);
    if (c == '[') return array(v, depth);
    if (c == '"') { v->kind = Value::String; return string(&v->str); }
    if (c == 't') { v->kind = Value::Bool; v->b = true; return lit("true"); }
    if (c == 'f') { v->kind = Value::Bool; v->b = false; return lit("false"); }
    if (c == 'n') { v->kind = Value::Null; return lit("null"); }
    return number(v);
  }
  bool object(Value* v, int depth) {
    v->kind = Value::Object;
    ++p_;
    skip();
    if (p_ < end_ && *p_ == '}') { ++p_; return true; }
    while (true) {
      skip();
      std::string key;
      if (p_ >= end_ || *p_ != '"' || !string(&key)) return false;
      skip();
      if (p_ >= end_ || *p_ != ':') return false;
      ++p_;
      skip();
      Value child;
      if (!value(&child, depth + 1)) return false;
      v->obj[key] = std::move(child);
      skip();
      if (p_ >= end_) return false;
      if (*p_ == ',') { ++p_; continue; }
      if (*p_ == '}') { ++p_; return true; }
      return false;
    }
  }
  bool array(Value* v, int depth) {
    v->kind = Value::Array;
    ++p_;
    skip();
    if (p_ < end_ && *p_ == ']') { ++p_; return true; }
    while (true) {
      skip();
      Value child;
      if (!value(&child, depth + 1)) return false;
      v->arr.push_back(std::move(child));
      skip();
      if (p_ >= end_) return false;
      if (*p_ == ',') { ++p_; continue; }
      if (*p_ == ']') { ++p_; return true; }
      return false;
    }
  }
  bool string(std::string* out) {
    ++p_;  // opening quote
    while (p_ < end_ && *p_ != '"') {
      if (*p_ == '\\') {
        ++p_;
        if (p_ >= end_) return false;
        char e = *p_;
        if (e == 'u') {  // keep \uXXXX escapes verbatim; header names are ASCII
          if (end_ - p_ < 5) return false;
          out->append("\\u");
          out->append(p_ + 1, 4);
          p_ += 5;
          continue;
        }
        const char m = e == 'n' ? '\n' : e == 't' ? '\t' : e == 'r' ? '\r' : e == 'b' ? '\b' : e == 'f' ? '\f' : e;
        out->push_back(m);
        ++p_;
        continue;
      }
      out->push_back(*p_++);
    }
    if (p_ >= end_) return false;
    ++p_;
    return true;
  }
  bool number(Value* v) {
    const char* s = p_;
    if (p_ < end_ && (*p_ == '-' || *p_ == '+')) ++p_;
    bool digits = false;
    while (p_ < end_ && ((*p_ >= '0' && *p_ <= '9') || *p_ == '.' || *p_ == 'e' || *p_ == 'E' || *p_ == '-' ||
                         *p_ == '+')) {
      digits = true;
      ++p_;
    }
    if (!digits) return false;
    v->kind = Value::Number;
    v->raw_number.assign(s, p_ - s);
    v->num = std::strtod(v->raw_number.c_str(), nullptr);
    return true;
  }
};

}  // namespace json
}  // namespace cb
