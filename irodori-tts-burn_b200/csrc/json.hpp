// Minimal JSON reader for safetensors headers and the `config_json` metadata.
// Supports objects, arrays, strings (with \uXXXX escapes), numbers, true,
// false and null.  Errors are reported by throwing JsonError.
#pragma once

#include <cstdint>
#include <cstdlib>
#include <map>
#include <memory>
#include <stdexcept>
#include <string>
#include <vector>

namespace irt {

struct JsonError : std::runtime_error {
  using std::runtime_error::runtime_error;
};

struct Json {
  enum Kind { Null, Bool, Number, String, Array, Object } kind = Null;
  bool b = false;
  double num = 0.0;
  std::string str;
  std::vector<Json> arr;
  std::map<std::string, Json> obj;

  bool is_null() const { return kind == Null; }
  bool has(const std::string& k) const { return kind == Object && obj.count(k) != 0; }
  const Json& at(const std::string& k) const {
    auto it = obj.find(k);
    if (kind != Object || it == obj.end()) throw JsonError("missing key '" + k + "'");
    return it->second;
  }
  double as_number() const {
    if (kind != Number) throw JsonError("expected a number");
    return num;
  }
  int64_t as_int() const {
    double v = as_number();
    if (v != (double)(int64_t)v) throw JsonError("expected an integer");
    return (int64_t)v;
  }
  bool as_bool() const {
    if (kind != Bool) throw JsonError("expected a bool");
    return b;
  }
  const std::string& as_string() const {
    if (kind != String) throw JsonError("expected a string");
    return str;
  }
};

class JsonParser {
 public:
  JsonParser(const char* p, size_t n) : p_(p), end_(p + n) {}

  Json parse() {
    Json v = value();
    ws();
    if (p_ != end_) fail("trailing characters");
    return v;
  }

 private:
  const char* p_;
  const char* end_;
  int depth_ = 0;

  [[noreturn]] void fail(const char* what) { throw JsonError(std::string("JSON: ") + what); }
  void ws() {
    while (p_ < end_ && (*p_ == ' ' || *p_ == '\n' || *p_ == '\r' || *p_ == '\t')) ++p_;
  }
  bool lit(const char* s) {
    size_t n = 0;
    while (s[n]) ++n;
    if ((size_t)(end_ - p_) < n) return false;
    for (size_t i = 0; i < n; ++i)
      if (p_[i] != s[i]) return false;
    p_ += n;
    return true;
  }
  Json value() {
    ws();
    if (p_ >= end_) fail("unexpected end");
    if (++depth_ > 256) fail("nesting too deep");
    Json v;
    char c = *p_;
    if (c == '{') {
      v.kind = Json::Object;
      ++p_;
      ws();
      if (p_ < end_ && *p_ == '}') {
        ++p_;
      } else {
        for (;;) {
          ws();
          if (p_ >= end_ || *p_ != '"') fail("expected key");
          std::string k = string();
          ws();
          if (p_ >= end_ || *p_ != ':') fail("expected ':'");
          ++p_;
          v.obj[k] = value();
          ws();
          if (p_ < end_ && *p_ == ',') { ++p_; continue; }
          if (p_ < end_ && *p_ == '}') { ++p_; break; }
          fail("expected ',' or '}'");
        }
      }
    } else if (c == '[') {
      v.kind = Json::Array;
      ++p_;
      ws();
      if (p_ < end_ && *p_ == ']') {
        ++p_;
      } else {
        for (;;) {
          v.arr.push_back(value());
          ws();
          if (p_ < end_ && *p_ == ',') { ++p_; continue; }
          if (p_ < end_ && *p_ == ']') { ++p_; break; }
          fail("expected ',' or ']'");
        }
      }
    } else if (c == '"') {
      v.kind = Json::String;
      v.str = string();
    } else if (lit("true")) {
      v.kind = Json::Bool; v.b = true;
    } else if (lit("false")) {
      v.kind = Json::Bool; v.b = false;
    } else if (lit("null")) {
      v.kind = Json::Null;
    } else {
      v.kind = Json::Number;
      v.num = number();
    }
    --depth_;
    return v;
  }
  double number() {
    const char* s = p_;
    if (p_ < end_ && (*p_ == '-' || *p_ == '+')) ++p_;
    while (p_ < end_ && ((*p_ >= '0' && *p_ <= '9') || *p_ == '.' || *p_ == 'e' || *p_ == 'E' ||
                         *p_ == '-' || *p_ == '+'))
      ++p_;
    if (p_ == s) fail("invalid value");
    std::string tok(s, p_);
    char* e = nullptr;
    double d = std::strtod(tok.c_str(), &e);
    if (!e || *e) fail("invalid number");
    return d;
  }
  static void put_utf8(std::string& o, uint32_t cp) {
    if (cp < 0x80) {
      o += (char)cp;
    } else if (cp < 0x800) {
      o += (char)(0xC0 | (cp >> 6));
      o += (char)(0x80 | (cp & 0x3F));
    } else if (cp < 0x10000) {
      o += (char)(0xE0 | (cp >> 12));
      o += (char)(0x80 | ((cp >> 6) & 0x3F));
      o += (char)(0x80 | (cp & 0x3F));
    } else {
      o += (char)(0xF0 | (cp >> 18));
      o += (char)(0x80 | ((cp >> 12) & 0x3F));
      o += (char)(0x80 | ((cp >> 6) & 0x3F));
      o += (char)(0x80 | (cp & 0x3F));
    }
  }
  uint32_t hex4() {
    if (end_ - p_ < 4) fail("bad \\u escape");
    uint32_t v = 0;
    for (int i = 0; i < 4; ++i) {
      char c = *p_++;
      v <<= 4;
      if (c >= '0' && c <= '9') v |= c - '0';
      else if (c >= 'a' && c <= 'f') v |= c - 'a' + 10;
      else if (c >= 'A' && c <= 'F') v |= c - 'A' + 10;
      else fail("bad \\u escape");
    }
    return v;
  }
  std::string string() {
    ++p_;  // opening quote
    std::string o;
    while (p_ < end_ && *p_ != '"') {
      char c = *p_++;
      if (c != '\\') { o += c; continue; }
      if (p_ >= end_) fail("bad escape");
      char e = *p_++;
      switch (e) {
        case '"': o += '"'; break;
        case '\\': o += '\\'; break;
        case '/': o += '/'; break;
        case 'b': o += '\b'; break;
        case 'f': o += '\f'; break;
        case 'n': o += '\n'; break;
        case 'r': o += '\r'; break;
        case 't': o += '\t'; break;
        case 'u': {
          uint32_t cp = hex4();
          if (cp >= 0xD800 && cp < 0xDC00 && end_ - p_ >= 6 && p_[0] == '\\' && p_[1] == 'u') {
            p_ += 2;
            uint32_t lo = hex4();
            cp = 0x10000 + ((cp - 0xD800) << 10) + (lo - 0xDC00);
          }
          put_utf8(o, cp);
          break;
        }
        default: fail("bad escape");
      }
    }
    if (p_ >= end_) fail("unterminated string");
    ++p_;
    return o;
  }
};

inline Json parse_json(const std::string& s) { return JsonParser(s.data(), s.size()).parse(); }

}  // namespace irt
