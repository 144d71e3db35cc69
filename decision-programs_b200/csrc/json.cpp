#include "json.h"

#include <charconv>
#include <cmath>
#include <cstdio>
#include <cstdlib>
#include <limits>

#include "common.h"

namespace dp::json {


bool Value::as_bool() const {
  if (kind_ == Kind::Bool) return b_;
  if (kind_ == Kind::Number && (d_ == 0.0 || d_ == 1.0)) return d_ != 0.0;
  fail("JSON value is not a boolean");
}
double Value::as_double() const {
  need(kind_ == Kind::Number, "JSON value is not a number");
  return d_;
}
std::int64_t Value::as_int() const {
  need(kind_ == Kind::Number, "JSON value is not a number");
  if (!s_.empty() && s_.find_first_of(".eE") == std::string::npos) {
    std::int64_t v = 0;
    auto r = std::from_chars(s_.data(), s_.data() + s_.size(), v);
    if (r.ec != std::errc{} || r.ptr != s_.data() + s_.size()) fail("JSON integer out of range: " + printable(s_));
    return v;
  }
  need(std::isfinite(d_) && d_ == std::floor(d_) && std::fabs(d_) < 9.0e15, "JSON number is not an integer");
  return std::int64_t(d_);
}
std::uint64_t Value::as_uint() const {
  need(kind_ == Kind::Number, "JSON value is not a number");
  if (!s_.empty() && s_.find_first_of(".eE-") == std::string::npos) {
    std::uint64_t v = 0;
    auto r = std::from_chars(s_.data(), s_.data() + s_.size(), v);
    if (r.ec != std::errc{} || r.ptr != s_.data() + s_.size()) fail("JSON integer out of range: " + printable(s_));
    return v;
  }
  std::int64_t v = as_int();
  need(v >= 0, "JSON integer must be non-negative");
  return std::uint64_t(v);
}
const std::string& Value::as_string() const {
  need(kind_ == Kind::String, "JSON value is not a string");
  return s_;
}
const std::vector<Value>& Value::items() const {
  need(kind_ == Kind::Array, "JSON value is not an array");
  return a_;
}
std::vector<Value>& Value::items() {
  need(kind_ == Kind::Array, "JSON value is not an array");
  return a_;
}
const std::vector<std::pair<std::string, Value>>& Value::members() const {
  need(kind_ == Kind::Object, "JSON value is not an object");
  return o_;
}
bool Value::contains(const std::string& key) const { return find(key) != nullptr; }
const Value* Value::find(const std::string& key) const {
  if (kind_ != Kind::Object) return nullptr;
  for (const auto& kv : o_)
    if (kv.first == key) return &kv.second;
  return nullptr;
}
const Value& Value::at(const std::string& key) const {
  const Value* v = find(key);
  if (v == nullptr) fail("missing JSON key: " + printable(key));
  return *v;
}
size_t Value::size() const {
  if (kind_ == Kind::Array) return a_.size();
  if (kind_ == Kind::Object) return o_.size();
  fail("JSON value has no size");
}
void Value::push(Value v) {
  need(kind_ == Kind::Array, "JSON push on non-array");
  a_.push_back(std::move(v));
}
void Value::set(const std::string& key, Value v) {
  need(kind_ == Kind::Object, "JSON set on non-object");
  for (auto& kv : o_)
    if (kv.first == key) { kv.second = std::move(v); return; }
  o_.emplace_back(key, std::move(v));
}

std::string quote(std::string_view s) {
  std::string out;
  out.reserve(s.size() + 2);
  out.push_back('"');
  for (char c : s) {
    switch (c) {
      case '"': out += "\\\""; break;
      case '\\': out += "\\\\"; break;
      case '\n': out += "\\n"; break;
      case '\r': out += "\\r"; break;
      case '\t': out += "\\t"; break;
      default:
        if (static_cast<unsigned char>(c) < 0x20) {
          char buf[8];
          std::snprintf(buf, sizeof buf, "\\u%04x", unsigned(static_cast<unsigned char>(c)));
          out += buf;
        } else {
          out.push_back(c);
        }
    }
  }
  out.push_back('"');
  return out;
}

std::string format_double(double v) {
  if (std::isnan(v)) return "NaN";
  if (std::isinf(v)) return v > 0 ? "Infinity" : "-Infinity";
  char buf[64];
  auto r = std::to_chars(buf, buf + sizeof buf, v);
  return std::string(buf, r.ptr);
}

void append_float(std::string& o, float v) {
  if (std::isnan(v)) {
    o += "NaN";
    return;
  }
  if (std::isinf(v)) {
    o += v > 0 ? "Infinity" : "-Infinity";
    return;
  }
  // "-0" would read back as the integer 0; keep the sign with a float token
  if (v == 0.0f) {
    o += std::signbit(v) ? "-0.0" : "0";
    return;
  }
  char buf[64];
  auto r = std::to_chars(buf, buf + sizeof buf, v);
  // The shortest float repr read back through a double and narrowed must give
  // v again; otherwise use 9 significant digits, which always do.  (from_chars
  // rounds correctly and ignores the locale, as the reader must.)
  double back = 0.0;
  const auto pr = std::from_chars(buf, r.ptr, back);
  if (pr.ec != std::errc{} || float(back) != v)
    r = std::to_chars(buf, buf + sizeof buf, double(v), std::chars_format::general, 9);
  o.append(buf, r.ptr);
}

void append_int(std::string& o, long long v) {
  char buf[24];
  const auto r = std::to_chars(buf, buf + sizeof buf, v);
  o.append(buf, r.ptr);
}

std::string format_float(float v) {
  std::string s;
  append_float(s, v);
  return s;
}

std::string Value::dump() const {
  switch (kind_) {
    case Kind::Null: return "null";
    case Kind::Bool: return b_ ? "true" : "false";
    case Kind::Number: return !s_.empty() ? s_ : format_double(d_);
    case Kind::String: return quote(s_);
    case Kind::Array: {
      std::string out = "[";
      for (size_t i = 0; i < a_.size(); ++i) {
        if (i) out += ",";
        out += a_[i].dump();
      }
      return out + "]";
    }
    case Kind::Object: {
      std::string out = "{";
      for (size_t i = 0; i < o_.size(); ++i) {
        if (i) out += ",";
        out += quote(o_[i].first) + ":" + o_[i].second.dump();
      }
      return out + "}";
    }
  }
  return "null";
}

namespace {
class Parser {
 public:
  explicit Parser(std::string_view t) : t_(t) {}
  Value parse_document() {
    Value v = value(0);
    ws();
    need(i_ == t_.size(), "trailing characters after JSON document");
    return v;
  }

 private:
  std::string_view t_;
  size_t i_ = 0;

  void ws() {
    while (i_ < t_.size() && (t_[i_] == ' ' || t_[i_] == '\n' || t_[i_] == '\r' || t_[i_] == '\t')) ++i_;
  }
  bool lit(std::string_view w) {
    if (t_.substr(i_, w.size()) == w) { i_ += w.size(); return true; }
    return false;
  }
  Value value(int depth) {
    need(depth < 256, "JSON nesting too deep");
    ws();
    need(i_ < t_.size(), "unexpected end of JSON");
    char c = t_[i_];
    if (c == '{') return object(depth);
    if (c == '[') return array(depth);
    if (c == '"') return Value::string(str());
    if (lit("true")) return Value::boolean(true);
    if (lit("false")) return Value::boolean(false);
    if (lit("null")) return Value::null();
    if (lit("NaN")) return Value::number(std::numeric_limits<double>::quiet_NaN());
    if (lit("Infinity") || lit("+Infinity")) return Value::number(std::numeric_limits<double>::infinity());
    if (lit("-Infinity")) return Value::number(-std::numeric_limits<double>::infinity());
    return num();
  }
  Value object(int depth) {
    ++i_;
    Value o = Value::object();
    ws();
    if (i_ < t_.size() && t_[i_] == '}') { ++i_; return o; }
    for (;;) {
      ws();
      need(i_ < t_.size() && t_[i_] == '"', "JSON object key must be a string");
      std::string k = str();
      ws();
      need(i_ < t_.size() && t_[i_] == ':', "expected ':' in JSON object");
      ++i_;
      o.set(k, value(depth + 1));
      ws();
      need(i_ < t_.size(), "unterminated JSON object");
      if (t_[i_] == ',') { ++i_; continue; }
      need(t_[i_] == '}', "expected ',' or '}' in JSON object");
      ++i_;
      return o;
    }
  }
  Value array(int depth) {
    ++i_;
    Value a = Value::array();
    ws();
    if (i_ < t_.size() && t_[i_] == ']') { ++i_; return a; }
    for (;;) {
      a.push(value(depth + 1));
      ws();
      need(i_ < t_.size(), "unterminated JSON array");
      if (t_[i_] == ',') { ++i_; continue; }
      need(t_[i_] == ']', "expected ',' or ']' in JSON array");
      ++i_;
      return a;
    }
  }
  // The value of four hex digits at `at`.
  unsigned hex4(size_t at) const {
    need(at + 4 <= t_.size(), "bad JSON unicode escape");
    unsigned v = 0;
    for (size_t k = 0; k < 4; ++k) {
      const char h = t_[at + k];
      const int d = (h >= '0' && h <= '9')   ? h - '0'
                    : (h >= 'a' && h <= 'f') ? h - 'a' + 10
                    : (h >= 'A' && h <= 'F') ? h - 'A' + 10
                                             : -1;
      need(d >= 0, "bad JSON unicode escape");
      v = v * 16 + unsigned(d);
    }
    return v;
  }
  std::string str() {
    ++i_;
    std::string out;
    while (i_ < t_.size() && t_[i_] != '"') {
      char c = t_[i_++];
      if (c != '\\') { out.push_back(c); continue; }
      need(i_ < t_.size(), "bad JSON escape");
      char e = t_[i_++];
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
          // four hex digits; a high surrogate must be followed by an escaped
          // low one, and the pair is one code point; a lone surrogate is refused
          unsigned cp = hex4(i_);
          i_ += 4;
          if (cp >= 0xD800 && cp <= 0xDBFF) {
            need(i_ + 2 <= t_.size() && t_[i_] == '\\' && t_[i_ + 1] == 'u', "bad JSON unicode escape");
            const unsigned lo = hex4(i_ + 2);
            need(lo >= 0xDC00 && lo <= 0xDFFF, "bad JSON unicode escape");
            i_ += 6;
            cp = 0x10000 + ((cp - 0xD800) << 10) + (lo - 0xDC00);
          } else {
            need(cp < 0xDC00 || cp > 0xDFFF, "bad JSON unicode escape");
          }
          if (cp < 0x80) {
            out.push_back(char(cp));
          } else if (cp < 0x800) {
            out.push_back(char(0xC0 | (cp >> 6)));
            out.push_back(char(0x80 | (cp & 0x3F)));
          } else if (cp < 0x10000) {
            out.push_back(char(0xE0 | (cp >> 12)));
            out.push_back(char(0x80 | ((cp >> 6) & 0x3F)));
            out.push_back(char(0x80 | (cp & 0x3F)));
          } else {
            out.push_back(char(0xF0 | (cp >> 18)));
            out.push_back(char(0x80 | ((cp >> 12) & 0x3F)));
            out.push_back(char(0x80 | ((cp >> 6) & 0x3F)));
            out.push_back(char(0x80 | (cp & 0x3F)));
          }
          break;
        }
        default: fail("bad JSON escape");
      }
    }
    need(i_ < t_.size(), "unterminated JSON string");
    ++i_;
    return out;
  }
  Value num() {
    size_t b = i_;
    if (i_ < t_.size() && (t_[i_] == '-' || t_[i_] == '+')) ++i_;
    while (i_ < t_.size() && ((t_[i_] >= '0' && t_[i_] <= '9') || t_[i_] == '.' || t_[i_] == 'e' ||
                              t_[i_] == 'E' || t_[i_] == '-' || t_[i_] == '+'))
      ++i_;
    if (i_ <= b) fail("invalid JSON token near: " + printable(t_.substr(b, 16)));
    std::string text(t_.substr(b, i_ - b));
    // from_chars reads the same syntax as strtod apart from a leading '+',
    // and reports values beyond the double range instead of returning +-inf
    // or 0: those (rare) tokens take strtod's reading, so both paths agree.
    double d = 0.0;
    const auto r = std::from_chars(text.data(), text.data() + text.size(), d);
    if (text[0] == '+' || r.ec == std::errc::result_out_of_range) {
      char* end = nullptr;
      d = strtod_c(text.c_str(), &end);
      if (end != text.c_str() + text.size()) fail("invalid JSON number: " + printable(text));
    } else {
      if (r.ec != std::errc{} || r.ptr != text.data() + text.size()) fail("invalid JSON number: " + printable(text));
    }
    return Value::number(d, std::move(text));
  }
};
}  // namespace

Value parse(std::string_view text) { return Parser(text).parse_document(); }

}  // namespace dp::json
