// Minimal JSON document model for the C-ABI strings of libdp_gbdt: array
// interfaces, configs, parameter tokens and model buffers.  It accepts the
// bare NaN / Infinity / -Infinity tokens that XGBoost's text format and the
// reference's `{"missing":NaN}` config use (native/class_native_training.cuh:51,
// native/class_native_model_json.hpp:12-17).
#pragma once
#include <cstdint>
#include <map>
#include <memory>
#include <string>
#include <string_view>
#include <utility>
#include <vector>

namespace dp::json {

class Value {
 public:
  enum class Kind { Null, Bool, Number, String, Array, Object };

  Value() = default;
  static Value null() { return Value(); }
  static Value boolean(bool b) { Value v; v.kind_ = Kind::Bool; v.b_ = b; return v; }
  static Value number(double d, std::string text = {}) {
    Value v; v.kind_ = Kind::Number; v.d_ = d; v.s_ = std::move(text); return v;
  }
  static Value string(std::string s) { Value v; v.kind_ = Kind::String; v.s_ = std::move(s); return v; }
  static Value array() { Value v; v.kind_ = Kind::Array; return v; }
  static Value object() { Value v; v.kind_ = Kind::Object; return v; }

  Kind kind() const { return kind_; }
  bool is_null() const { return kind_ == Kind::Null; }
  bool is_bool() const { return kind_ == Kind::Bool; }
  bool is_number() const { return kind_ == Kind::Number; }
  bool is_string() const { return kind_ == Kind::String; }
  bool is_array() const { return kind_ == Kind::Array; }
  bool is_object() const { return kind_ == Kind::Object; }

  bool as_bool() const;
  double as_double() const;
  // Exact integer value (from the literal's text); throws when not integral.
  std::int64_t as_int() const;
  std::uint64_t as_uint() const;
  const std::string& as_string() const;
  const std::vector<Value>& items() const;
  std::vector<Value>& items();
  const std::vector<std::pair<std::string, Value>>& members() const;

  bool contains(const std::string& key) const;
  const Value& at(const std::string& key) const;
  const Value* find(const std::string& key) const;
  const Value& operator[](size_t i) const { return items().at(i); }
  size_t size() const;

  void push(Value v);
  void set(const std::string& key, Value v);

  std::string dump() const;

 private:
  Kind kind_ = Kind::Null;
  bool b_ = false;
  double d_ = 0.0;
  std::string s_;  // string payload, or the literal text of a number
  std::vector<Value> a_;
  std::vector<std::pair<std::string, Value>> o_;
};

Value parse(std::string_view text);

// Shortest decimal that reads back to the same float through a double
// (the reference parses model numbers as double, then narrows to float:
// native/class_io.hpp:180).
std::string format_float(float v);
// The same texts appended to o without a temporary string (model writing).
void append_float(std::string& o, float v);
void append_int(std::string& o, long long v);
std::string format_double(double v);
std::string quote(std::string_view s);

}  // namespace dp::json
