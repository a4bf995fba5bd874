// A small JSON value and parser for checkpoint headers and model configs (RFC 8259 subset: no
// comments; numbers keep whether they were written as integers).
#pragma once

#include <cstdint>
#include <map>
#include <memory>
#include <string>
#include <utility>
#include <vector>

namespace foa::engine {

class Json {
 public:
  enum class Type { Null, Bool, Number, String, Array, Object };
  Json() = default;
  static Json parse(const std::string& text);  // throws ValueError with the offset

  Type type() const { return type_; }
  bool is_null() const { return type_ == Type::Null; }
  bool is_bool() const { return type_ == Type::Bool; }
  bool is_number() const { return type_ == Type::Number; }
  bool is_int() const { return type_ == Type::Number && integral_; }
  bool is_string() const { return type_ == Type::String; }
  bool is_array() const { return type_ == Type::Array; }
  bool is_object() const { return type_ == Type::Object; }

  bool as_bool() const { return b_; }
  double as_double() const { return num_; }
  int64_t as_int() const { return i_; }
  const std::string& as_string() const { return s_; }
  const std::vector<Json>& items() const { return arr_; }
  const std::vector<std::pair<std::string, Json>>& members() const { return obj_; }

  // Object member access; a missing key reads as null.
  const Json& operator[](const std::string& key) const;
  bool contains(const std::string& key) const;
  const Json& at(size_t i) const { return arr_.at(i); }
  size_t size() const { return is_array() ? arr_.size() : obj_.size(); }

  // Builders.
  static Json null() { return Json(); }
  static Json boolean(bool v);
  static Json number(double v);
  static Json integer(int64_t v);
  static Json string(std::string v);
  static Json array(std::vector<Json> v);
  static Json object(std::vector<std::pair<std::string, Json>> v);
  void set(const std::string& key, Json v);
  std::string dump() const;

 private:
  Type type_ = Type::Null;
  bool b_ = false, integral_ = false;
  double num_ = 0;
  int64_t i_ = 0;
  std::string s_;
  std::vector<Json> arr_;
  std::vector<std::pair<std::string, Json>> obj_;
  friend class JsonParser;
};

}  // namespace foa::engine
