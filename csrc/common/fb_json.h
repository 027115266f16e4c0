// Minimal JSON value, writer and parser for the archive's text files
// (graph_*.json, allocator events, output-tensor metadata, manifests).
//
// Integers are kept exact as int64/uint64 (device addresses do not fit a
// double); objects preserve insertion order so files are byte-stable across
// SAVE runs. No external dependency (the image has no JSON library for C++).
#pragma once

#include <cstdint>
#include <cstdio>
#include <cstring>
#include <map>
#include <memory>
#include <stdexcept>
#include <string>
#include <utility>
#include <vector>

namespace fb {
namespace json {

class Value;
using Array = std::vector<Value>;

class Object {
 public:
  using Item = std::pair<std::string, Value>;
  Value& operator[](const std::string& key);
  const Value* find(const std::string& key) const;
  bool contains(const std::string& key) const { return find(key) != nullptr; }
  const Value& at(const std::string& key) const;
  void erase(const std::string& key);
  const std::vector<Item>& items() const { return items_; }
  size_t size() const { return items_.size(); }

 private:
  std::vector<Item> items_;
  std::map<std::string, size_t> index_;
};

class Value {
 public:
  enum class Type { Null, Bool, Int, UInt, Double, String, Array, Object };

  Value() : type_(Type::Null), u_(0) {}
  Value(std::nullptr_t) : type_(Type::Null), u_(0) {}
  Value(bool b) : type_(Type::Bool), b_(b) {}
  Value(int v) : type_(Type::Int), i_(v) {}
  Value(long v) : type_(Type::Int), i_(v) {}
  Value(long long v) : type_(Type::Int), i_(v) {}
  Value(unsigned v) : type_(Type::UInt), u_(v) {}
  Value(unsigned long v) : type_(Type::UInt), u_(v) {}
  Value(unsigned long long v) : type_(Type::UInt), u_(v) {}
  Value(double v) : type_(Type::Double), d_(v) {}
  Value(const char* s) : type_(Type::String), s_(std::make_shared<std::string>(s)) {}
  Value(std::string s) : type_(Type::String), s_(std::make_shared<std::string>(std::move(s))) {}
  Value(Array a) : type_(Type::Array), a_(std::make_shared<Array>(std::move(a))) {}
  Value(Object o) : type_(Type::Object), o_(std::make_shared<Object>(std::move(o))) {}

  Type type() const { return type_; }
  bool is_null() const { return type_ == Type::Null; }
  bool is_number() const { return type_ == Type::Int || type_ == Type::UInt || type_ == Type::Double; }
  bool is_string() const { return type_ == Type::String; }
  bool is_array() const { return type_ == Type::Array; }
  bool is_object() const { return type_ == Type::Object; }

  bool as_bool() const {
    if (type_ == Type::Bool) return b_;
    if (is_number()) return as_i64() != 0;
    throw std::runtime_error("json: not a bool");
  }
  int64_t as_i64() const {
    switch (type_) {
      case Type::Int: return i_;
      case Type::UInt: return static_cast<int64_t>(u_);
      case Type::Double: return static_cast<int64_t>(d_);
      case Type::Bool: return b_ ? 1 : 0;
      default: throw std::runtime_error("json: not a number");
    }
  }
  uint64_t as_u64() const {
    switch (type_) {
      case Type::Int: return static_cast<uint64_t>(i_);
      case Type::UInt: return u_;
      case Type::Double: return static_cast<uint64_t>(d_);
      case Type::Bool: return b_ ? 1 : 0;
      default: throw std::runtime_error("json: not a number");
    }
  }
  double as_double() const {
    switch (type_) {
      case Type::Int: return static_cast<double>(i_);
      case Type::UInt: return static_cast<double>(u_);
      case Type::Double: return d_;
      default: throw std::runtime_error("json: not a number");
    }
  }
  const std::string& as_string() const {
    if (type_ != Type::String) throw std::runtime_error("json: not a string");
    return *s_;
  }
  const Array& as_array() const {
    if (type_ != Type::Array) throw std::runtime_error("json: not an array");
    return *a_;
  }
  Array& as_array() {
    if (type_ != Type::Array) throw std::runtime_error("json: not an array");
    return *a_;
  }
  const Object& as_object() const {
    if (type_ != Type::Object) throw std::runtime_error("json: not an object");
    return *o_;
  }
  Object& as_object() {
    if (type_ != Type::Object) throw std::runtime_error("json: not an object");
    return *o_;
  }

  void dump(std::string& out) const;
  std::string dump() const {
    std::string s;
    dump(s);
    return s;
  }

 private:
  Type type_;
  union {
    bool b_;
    int64_t i_;
    uint64_t u_;
    double d_;
  };
  std::shared_ptr<std::string> s_;
  std::shared_ptr<Array> a_;
  std::shared_ptr<Object> o_;
};

inline Value& Object::operator[](const std::string& key) {
  auto it = index_.find(key);
  if (it != index_.end()) return items_[it->second].second;
  index_[key] = items_.size();
  items_.emplace_back(key, Value());
  return items_.back().second;
}
inline const Value* Object::find(const std::string& key) const {
  auto it = index_.find(key);
  return it == index_.end() ? nullptr : &items_[it->second].second;
}
inline const Value& Object::at(const std::string& key) const {
  const Value* v = find(key);
  if (!v) throw std::runtime_error("json: missing key '" + key + "'");
  return *v;
}
inline void Object::erase(const std::string& key) {
  auto it = index_.find(key);
  if (it == index_.end()) return;
  items_.erase(items_.begin() + static_cast<long>(it->second));
  index_.clear();
  for (size_t i = 0; i < items_.size(); ++i) index_[items_[i].first] = i;
}

inline void escape_into(std::string& out, const std::string& s) {
  out.push_back('"');
  for (unsigned char c : s) {
    switch (c) {
      case '"': out += "\\\""; break;
      case '\\': out += "\\\\"; break;
      case '\n': out += "\\n"; break;
      case '\r': out += "\\r"; break;
      case '\t': out += "\\t"; break;
      default:
        if (c < 0x20) {
          char buf[8];
          snprintf(buf, sizeof(buf), "\\u%04x", c);
          out += buf;
        } else {
          out.push_back(static_cast<char>(c));
        }
    }
  }
  out.push_back('"');
}

inline void Value::dump(std::string& out) const {
  char buf[64];
  switch (type_) {
    case Type::Null: out += "null"; break;
    case Type::Bool: out += b_ ? "true" : "false"; break;
    case Type::Int: snprintf(buf, sizeof(buf), "%lld", static_cast<long long>(i_)); out += buf; break;
    case Type::UInt: snprintf(buf, sizeof(buf), "%llu", static_cast<unsigned long long>(u_)); out += buf; break;
    case Type::Double: snprintf(buf, sizeof(buf), "%.17g", d_); out += buf; break;
    case Type::String: escape_into(out, *s_); break;
    case Type::Array: {
      out.push_back('[');
      bool first = true;
      for (const auto& v : *a_) {
        if (!first) out.push_back(',');
        first = false;
        v.dump(out);
      }
      out.push_back(']');
      break;
    }
    case Type::Object: {
      out.push_back('{');
      bool first = true;
      for (const auto& kv : o_->items()) {
        if (!first) out.push_back(',');
        first = false;
        escape_into(out, kv.first);
        out.push_back(':');
        kv.second.dump(out);
      }
      out.push_back('}');
      break;
    }
  }
}

class Parser {
 public:
  Parser(const char* p, size_t n) : p_(p), end_(p + n) {}
  Value parse() {
    Value v = value();
    ws();
    if (p_ != end_) fail("trailing characters");
    return v;
  }

 private:
  const char* p_;
  const char* end_;

  [[noreturn]] void fail(const char* what) { throw std::runtime_error(std::string("json parse: ") + what); }
  void ws() {
    while (p_ < end_ && (*p_ == ' ' || *p_ == '\n' || *p_ == '\t' || *p_ == '\r')) ++p_;
  }
  bool lit(const char* s) {
    size_t n = strlen(s);
    if (static_cast<size_t>(end_ - p_) >= n && memcmp(p_, s, n) == 0) {
      p_ += n;
      return true;
    }
    return false;
  }
  Value value() {
    ws();
    if (p_ >= end_) fail("unexpected end");
    char c = *p_;
    if (c == '{') return object();
    if (c == '[') return array();
    if (c == '"') return Value(string());
    if (lit("true")) return Value(true);
    if (lit("false")) return Value(false);
    if (lit("null")) return Value();
    return number();
  }
  std::string string() {
    ++p_;  // opening quote
    std::string out;
    while (p_ < end_ && *p_ != '"') {
      char c = *p_++;
      if (c != '\\') {
        out.push_back(c);
        continue;
      }
      if (p_ >= end_) fail("bad escape");
      char e = *p_++;
      switch (e) {
        case '"': out.push_back('"'); break;
        case '\\': out.push_back('\\'); break;
        case '/': out.push_back('/'); break;
        case 'b': out.push_back('\b'); break;
        case 'f': out.push_back('\f'); break;
        case 'n': out.push_back('\n'); break;
        case 'r': out.push_back('\r'); break;
        case 't': out.push_back('\t'); break;
        case 'u': {
          if (end_ - p_ < 4) fail("bad \\u escape");
          unsigned cp = static_cast<unsigned>(strtoul(std::string(p_, 4).c_str(), nullptr, 16));
          p_ += 4;
          if (cp < 0x80) {
            out.push_back(static_cast<char>(cp));
          } else if (cp < 0x800) {
            out.push_back(static_cast<char>(0xC0 | (cp >> 6)));
            out.push_back(static_cast<char>(0x80 | (cp & 0x3F)));
          } else {
            out.push_back(static_cast<char>(0xE0 | (cp >> 12)));
            out.push_back(static_cast<char>(0x80 | ((cp >> 6) & 0x3F)));
            out.push_back(static_cast<char>(0x80 | (cp & 0x3F)));
          }
          break;
        }
        default: fail("bad escape");
      }
    }
    if (p_ >= end_) fail("unterminated string");
    ++p_;
    return out;
  }
  Value number() {
    const char* start = p_;
    bool is_float = false, neg = false;
    if (p_ < end_ && (*p_ == '-' || *p_ == '+')) {
      neg = *p_ == '-';
      ++p_;
    }
    while (p_ < end_ && ((*p_ >= '0' && *p_ <= '9') || *p_ == '.' || *p_ == 'e' || *p_ == 'E' ||
                         *p_ == '-' || *p_ == '+')) {
      if (*p_ == '.' || *p_ == 'e' || *p_ == 'E') is_float = true;
      ++p_;
    }
    if (p_ == start) fail("bad value");
    std::string tok(start, p_);
    if (is_float) return Value(strtod(tok.c_str(), nullptr));
    if (neg) return Value(static_cast<long long>(strtoll(tok.c_str(), nullptr, 10)));
    unsigned long long u = strtoull(tok.c_str(), nullptr, 10);
    if (u <= static_cast<unsigned long long>(INT64_MAX)) return Value(static_cast<long long>(u));
    return Value(u);
  }
  Value array() {
    ++p_;
    Array a;
    ws();
    if (p_ < end_ && *p_ == ']') {
      ++p_;
      return Value(std::move(a));
    }
    for (;;) {
      a.push_back(value());
      ws();
      if (p_ < end_ && *p_ == ',') {
        ++p_;
        continue;
      }
      if (p_ < end_ && *p_ == ']') {
        ++p_;
        break;
      }
      fail("expected , or ]");
    }
    return Value(std::move(a));
  }
  Value object() {
    ++p_;
    Object o;
    ws();
    if (p_ < end_ && *p_ == '}') {
      ++p_;
      return Value(std::move(o));
    }
    for (;;) {
      ws();
      if (p_ >= end_ || *p_ != '"') fail("expected key");
      std::string k = string();
      ws();
      if (p_ >= end_ || *p_ != ':') fail("expected :");
      ++p_;
      o[k] = value();
      ws();
      if (p_ < end_ && *p_ == ',') {
        ++p_;
        continue;
      }
      if (p_ < end_ && *p_ == '}') {
        ++p_;
        break;
      }
      fail("expected , or }");
    }
    return Value(std::move(o));
  }
};

inline Value parse(const std::string& s) { return Parser(s.data(), s.size()).parse(); }
inline Value parse(const char* p, size_t n) { return Parser(p, n).parse(); }

}  // namespace json
}  // namespace fb
