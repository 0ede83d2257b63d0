// Minimal JSON reader for qgraph.json (objects, arrays, strings, numbers, bools, null).
// Numbers keep both their integer value (when the literal is integral) and a double.
#pragma once
#include <cstdint>
#include <map>
#include <memory>
#include <stdexcept>
#include <string>
#include <vector>

namespace llx::json {

struct Value {
  enum Kind { Null, Bool, Number, String, Array, Object } kind = Null;
  bool b = false;
  bool is_int = false;
  int64_t i = 0;
  double d = 0.0;
  std::string s;
  std::vector<Value> arr;
  std::vector<std::pair<std::string, Value>> obj;  // insertion order kept

  bool has(const std::string& k) const {
    if (kind != Object) return false;
    for (auto& kv : obj)
      if (kv.first == k) return true;
    return false;
  }
  const Value& at(const std::string& k) const {
    if (kind != Object) throw std::runtime_error("json: '" + k + "' looked up in a non-object");
    for (auto& kv : obj)
      if (kv.first == k) return kv.second;
    throw std::runtime_error("json: missing key '" + k + "'");
  }
  const Value* find(const std::string& k) const {
    if (kind != Object) return nullptr;
    for (auto& kv : obj)
      if (kv.first == k) return &kv.second;
    return nullptr;
  }
  int64_t as_int() const {
    if (kind == Bool) return b ? 1 : 0;
    if (kind != Number || !is_int) throw std::runtime_error("json: expected an integer");
    return i;
  }
  double as_double() const {
    if (kind != Number) throw std::runtime_error("json: expected a number");
    return d;
  }
  const std::string& as_str() const {
    if (kind != String) throw std::runtime_error("json: expected a string");
    return s;
  }
  bool is_null() const { return kind == Null; }
};

class Parser {
 public:
  explicit Parser(const std::string& text) : t_(text) {}
  Value parse() {
    Value v = value();
    ws();
    if (p_ != t_.size()) fail("trailing characters");
    return v;
  }

 private:
  const std::string& t_;
  size_t p_ = 0;

  [[noreturn]] void fail(const char* what) {
    throw std::runtime_error(std::string("json: ") + what + " at offset " + std::to_string(p_));
  }
  void ws() {
    while (p_ < t_.size() && (t_[p_] == ' ' || t_[p_] == '\n' || t_[p_] == '\r' || t_[p_] == '\t')) ++p_;
  }
  char peek() {
    ws();
    if (p_ >= t_.size()) fail("unexpected end");
    return t_[p_];
  }
  void expect(char c) {
    if (peek() != c) fail("unexpected character");
    ++p_;
  }
  bool lit(const char* w) {
    size_t n = 0;
    while (w[n]) ++n;
    if (t_.compare(p_, n, w) == 0) {
      p_ += n;
      return true;
    }
    return false;
  }
  Value value() {
    char c = peek();
    Value v;
    if (c == '{') {
      v.kind = Value::Object;
      ++p_;
      if (peek() == '}') {
        ++p_;
        return v;
      }
      for (;;) {
        if (peek() != '"') fail("expected key");
        std::string k = str();
        expect(':');
        v.obj.emplace_back(std::move(k), value());
        char d = peek();
        ++p_;
        if (d == '}') break;
        if (d != ',') fail("expected , or }");
      }
      return v;
    }
    if (c == '[') {
      v.kind = Value::Array;
      ++p_;
      if (peek() == ']') {
        ++p_;
        return v;
      }
      for (;;) {
        v.arr.push_back(value());
        char d = peek();
        ++p_;
        if (d == ']') break;
        if (d != ',') fail("expected , or ]");
      }
      return v;
    }
    if (c == '"') {
      v.kind = Value::String;
      v.s = str();
      return v;
    }
    if (lit("true")) {
      v.kind = Value::Bool;
      v.b = true;
      return v;
    }
    if (lit("false")) {
      v.kind = Value::Bool;
      return v;
    }
    if (lit("null")) return v;
    return number();
  }
  std::string str() {
    expect('"');
    std::string out;
    while (p_ < t_.size() && t_[p_] != '"') {
      char c = t_[p_++];
      if (c == '\\') {
        if (p_ >= t_.size()) fail("bad escape");
        char e = t_[p_++];
        switch (e) {
          case '"': out += '"'; break;
          case '\\': out += '\\'; break;
          case '/': out += '/'; break;
          case 'b': out += '\b'; break;
          case 'f': out += '\f'; break;
          case 'n': out += '\n'; break;
          case 'r': out += '\r'; break;
          case 't': out += '\t'; break;
          case 'u': {
            if (p_ + 4 > t_.size()) fail("bad \\u escape");
            unsigned cp = std::stoul(t_.substr(p_, 4), nullptr, 16);
            p_ += 4;
            if (cp < 0x80) {
              out += char(cp);
            } else if (cp < 0x800) {
              out += char(0xC0 | (cp >> 6));
              out += char(0x80 | (cp & 0x3F));
            } else {
              out += char(0xE0 | (cp >> 12));
              out += char(0x80 | ((cp >> 6) & 0x3F));
              out += char(0x80 | (cp & 0x3F));
            }
            break;
          }
          default: fail("bad escape");
        }
      } else {
        out += c;
      }
    }
    if (p_ >= t_.size()) fail("unterminated string");
    ++p_;
    return out;
  }
  Value number() {
    size_t s = p_;
    if (t_[p_] == '-' || t_[p_] == '+') ++p_;
    bool integral = true;
    while (p_ < t_.size()) {
      char c = t_[p_];
      if (c >= '0' && c <= '9') {
        ++p_;
      } else if (c == '.' || c == 'e' || c == 'E' || c == '+' || c == '-') {
        integral = false;
        ++p_;
      } else {
        break;
      }
    }
    if (s == p_) fail("expected a value");
    Value v;
    v.kind = Value::Number;
    std::string lit = t_.substr(s, p_ - s);
    v.d = std::stod(lit);
    if (integral) {
      try {
        v.i = std::stoll(lit);
        v.is_int = true;
      } catch (...) {
        v.is_int = false;
      }
    }
    return v;
  }
};

inline Value parse(const std::string& text) { return Parser(text).parse(); }

}  // namespace llx::json
