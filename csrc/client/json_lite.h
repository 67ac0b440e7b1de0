// Minimal JSON document model for the native front-end tools: parse (RFC 8259, UTF-8 text,
// \u escapes incl. surrogate pairs, nesting limited to 64 levels) and compact serialization.
// Numbers keep their literal text so integers of any size round-trip unchanged.
#pragma once
#include <cmath>
#include <cstdint>
#include <cstdio>
#include <cstdlib>
#include <stdexcept>
#include <string>
#include <utility>
#include <vector>

namespace barqjson {

struct Value {
  enum Type { kNull, kBool, kNumber, kString, kArray, kObject } type = kNull;
  bool b = false;
  double num = 0;
  std::string str;  // string value, or the literal text of a number
  std::vector<Value> arr;
  std::vector<std::pair<std::string, Value>> obj;

  static Value string(std::string s) {
    Value v;
    v.type = kString;
    v.str = std::move(s);
    return v;
  }
  static Value number(double d) {
    Value v;
    v.type = kNumber;
    v.num = d;
    char buf[40];
    if (std::isfinite(d) && d == std::floor(d) && std::fabs(d) < 9.0e15)
      std::snprintf(buf, sizeof buf, "%.0f", d);
    else
      std::snprintf(buf, sizeof buf, "%.17g", d);
    v.str = buf;
    return v;
  }
  static Value boolean(bool x) {
    Value v;
    v.type = kBool;
    v.b = x;
    return v;
  }
  static Value object() {
    Value v;
    v.type = kObject;
    return v;
  }
  static Value array() {
    Value v;
    v.type = kArray;
    return v;
  }

  bool is_null() const { return type == kNull; }
  bool is_string() const { return type == kString; }
  bool is_number() const { return type == kNumber; }
  bool is_array() const { return type == kArray; }
  bool is_object() const { return type == kObject; }
  bool is_integer() const {
    return type == kNumber && str.find_first_of(".eE") == std::string::npos;
  }

  const Value* get(const std::string& key) const {
    if (type != kObject) return nullptr;
    for (const auto& kv : obj)
      if (kv.first == key) return &kv.second;
    return nullptr;
  }
  // Adds or replaces a member (insertion order is kept).
  Value& set(const std::string& key, Value v) {
    for (auto& kv : obj)
      if (kv.first == key) return kv.second = std::move(v);
    obj.emplace_back(key, std::move(v));
    return obj.back().second;
  }
  void push(Value v) { arr.push_back(std::move(v)); }
};

inline void append_utf8(std::string& out, uint32_t cp) {
  if (cp < 0x80) {
    out += (char)cp;
  } else if (cp < 0x800) {
    out += (char)(0xC0 | (cp >> 6));
    out += (char)(0x80 | (cp & 0x3F));
  } else if (cp < 0x10000) {
    out += (char)(0xE0 | (cp >> 12));
    out += (char)(0x80 | ((cp >> 6) & 0x3F));
    out += (char)(0x80 | (cp & 0x3F));
  } else {
    out += (char)(0xF0 | (cp >> 18));
    out += (char)(0x80 | ((cp >> 12) & 0x3F));
    out += (char)(0x80 | ((cp >> 6) & 0x3F));
    out += (char)(0x80 | (cp & 0x3F));
  }
}

class Parser {
 public:
  explicit Parser(const std::string& s) : s_(s) {}

  Value document() {
    ws();
    Value v = value(0);
    ws();
    if (i_ != s_.size()) fail("trailing characters");
    return v;
  }

 private:
  static constexpr int kMaxDepth = 64;

  [[noreturn]] void fail(const char* what) const {
    throw std::runtime_error(std::string("invalid JSON: ") + what + " at byte " + std::to_string(i_));
  }
  char peek() const { return i_ < s_.size() ? s_[i_] : '\0'; }
  char next() {
    if (i_ >= s_.size()) fail("unexpected end");
    return s_[i_++];
  }
  void ws() {
    while (i_ < s_.size() && (s_[i_] == ' ' || s_[i_] == '\t' || s_[i_] == '\n' || s_[i_] == '\r')) ++i_;
  }
  void literal(const char* lit) {
    for (const char* p = lit; *p; ++p)
      if (next() != *p) fail("bad literal");
  }

  Value value(int depth) {
    if (depth > kMaxDepth) fail("nesting too deep");
    const char c = peek();
    if (c == '{') return object(depth);
    if (c == '[') return array(depth);
    if (c == '"') return Value::string(string());
    if (c == 't') {
      literal("true");
      return Value::boolean(true);
    }
    if (c == 'f') {
      literal("false");
      return Value::boolean(false);
    }
    if (c == 'n') {
      literal("null");
      return Value();
    }
    return number();
  }

  Value object(int depth) {
    Value v = Value::object();
    next();  // {
    ws();
    if (peek() == '}') {
      ++i_;
      return v;
    }
    for (;;) {
      ws();
      if (peek() != '"') fail("expected a key");
      std::string key = string();
      ws();
      if (next() != ':') fail("expected :");
      ws();
      v.set(key, value(depth + 1));
      ws();
      const char c = next();
      if (c == '}') return v;
      if (c != ',') fail("expected , or }");
    }
  }

  Value array(int depth) {
    Value v = Value::array();
    next();  // [
    ws();
    if (peek() == ']') {
      ++i_;
      return v;
    }
    for (;;) {
      ws();
      v.push(value(depth + 1));
      ws();
      const char c = next();
      if (c == ']') return v;
      if (c != ',') fail("expected , or ]");
    }
  }

  Value number() {
    const size_t b = i_;
    if (peek() == '-') ++i_;
    if (peek() == '0') {
      ++i_;
    } else if (peek() >= '1' && peek() <= '9') {
      while (peek() >= '0' && peek() <= '9') ++i_;
    } else {
      fail("expected a value");
    }
    if (peek() == '.') {
      ++i_;
      if (!(peek() >= '0' && peek() <= '9')) fail("bad fraction");
      while (peek() >= '0' && peek() <= '9') ++i_;
    }
    if (peek() == 'e' || peek() == 'E') {
      ++i_;
      if (peek() == '+' || peek() == '-') ++i_;
      if (!(peek() >= '0' && peek() <= '9')) fail("bad exponent");
      while (peek() >= '0' && peek() <= '9') ++i_;
    }
    Value v;
    v.type = Value::kNumber;
    v.str = s_.substr(b, i_ - b);
    v.num = std::strtod(v.str.c_str(), nullptr);
    return v;
  }

  uint32_t hex4() {
    uint32_t v = 0;
    for (int k = 0; k < 4; ++k) {
      const char c = next();
      v <<= 4;
      if (c >= '0' && c <= '9') v |= (uint32_t)(c - '0');
      else if (c >= 'a' && c <= 'f') v |= (uint32_t)(c - 'a' + 10);
      else if (c >= 'A' && c <= 'F') v |= (uint32_t)(c - 'A' + 10);
      else fail("bad \\u escape");
    }
    return v;
  }

  std::string string() {
    std::string out;
    if (next() != '"') fail("expected a string");
    for (;;) {
      const char c = next();
      if (c == '"') return out;
      if ((unsigned char)c < 0x20) fail("control character in string");
      if (c != '\\') {
        out += c;
        continue;
      }
      const char e = next();
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
          uint32_t cp = hex4();
          if (cp >= 0xD800 && cp < 0xDC00) {  // high surrogate: a low one must follow
            if (next() != '\\' || next() != 'u') fail("unpaired surrogate");
            const uint32_t lo = hex4();
            if (lo < 0xDC00 || lo >= 0xE000) fail("unpaired surrogate");
            cp = 0x10000 + ((cp - 0xD800) << 10) + (lo - 0xDC00);
          } else if (cp >= 0xDC00 && cp < 0xE000) {
            fail("unpaired surrogate");
          }
          append_utf8(out, cp);
          break;
        }
        default: fail("bad escape");
      }
    }
  }

  const std::string& s_;
  size_t i_ = 0;
};

inline Value parse(const std::string& text) { return Parser(text).document(); }

inline void escape_into(std::string& out, const std::string& s) {
  out += '"';
  for (const char ch : s) {
    const unsigned char c = (unsigned char)ch;
    switch (c) {
      case '"': out += "\\\""; break;
      case '\\': out += "\\\\"; break;
      case '\n': out += "\\n"; break;
      case '\r': out += "\\r"; break;
      case '\t': out += "\\t"; break;
      case '\b': out += "\\b"; break;
      case '\f': out += "\\f"; break;
      default:
        if (c < 0x20) {
          char buf[8];
          std::snprintf(buf, sizeof buf, "\\u%04x", c);
          out += buf;
        } else {
          out += ch;  // UTF-8 bytes pass through
        }
    }
  }
  out += '"';
}

inline void dump_into(std::string& out, const Value& v) {
  switch (v.type) {
    case Value::kNull: out += "null"; break;
    case Value::kBool: out += v.b ? "true" : "false"; break;
    case Value::kNumber: out += v.str; break;
    case Value::kString: escape_into(out, v.str); break;
    case Value::kArray: {
      out += '[';
      for (size_t i = 0; i < v.arr.size(); ++i) {
        if (i) out += ',';
        dump_into(out, v.arr[i]);
      }
      out += ']';
      break;
    }
    case Value::kObject: {
      out += '{';
      for (size_t i = 0; i < v.obj.size(); ++i) {
        if (i) out += ',';
        escape_into(out, v.obj[i].first);
        out += ':';
        dump_into(out, v.obj[i].second);
      }
      out += '}';
      break;
    }
  }
}

inline std::string dump(const Value& v) {
  std::string out;
  dump_into(out, v);
  return out;
}

}  // namespace barqjson
