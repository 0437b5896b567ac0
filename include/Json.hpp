// Json.hpp -- the JSON value type of the Stream API.
//
// The reference API aliases nlohmann::json (reference include/Model.hpp:10).
// That library is not part of this build, so Stream::Json is a small
// self-contained value type with the subset the API and its callers use:
// parsing (operator>> / parse), dump(indent), at(key/index), operator[],
// contains, size, iteration over arrays and objects, get<T>() for numbers,
// bools, strings and vectors, equality, and brace construction of objects
// and arrays (Json{{"key", 1}, {"other", "x"}}).
#pragma once

#include <cstdint>
#include <initializer_list>
#include <istream>
#include <map>
#include <memory>
#include <ostream>
#include <stdexcept>
#include <string>
#include <type_traits>
#include <utility>
#include <vector>

namespace Stream {

class Json {
 public:
  enum class Kind { Null, Bool, Int, Float, String, Array, Object };
  using Array = std::vector<Json>;
  using Object = std::map<std::string, Json>;

  Json() = default;
  Json(std::nullptr_t) {}
  Json(bool v) : kind_(Kind::Bool), b_(v) {}
  template <typename T, typename std::enable_if<std::is_integral<T>::value && !std::is_same<T, bool>::value, int>::type = 0>
  Json(T v) : kind_(Kind::Int), i_(static_cast<long long>(v)) {}
  template <typename T, typename std::enable_if<std::is_floating_point<T>::value, int>::type = 0>
  Json(T v) : kind_(Kind::Float), f_(static_cast<double>(v)) {}
  Json(const char* v) : kind_(Kind::String), s_(v) {}
  Json(std::string v) : kind_(Kind::String), s_(std::move(v)) {}
  template <typename T>
  Json(const std::vector<T>& v) : kind_(Kind::Array) {
    for (const auto& x : v) a_.push_back(Json(x));
  }
  // {{"k", v}, ...} builds an object when every element is a [string, value]
  // pair, otherwise an array (the nlohmann convention).
  Json(std::initializer_list<Json> init);

  static Json array() { Json j; j.kind_ = Kind::Array; return j; }
  static Json object() { Json j; j.kind_ = Kind::Object; return j; }
  static Json parse(const std::string& text);
  static Json parse(const char* text) { return parse(std::string(text)); }
  template <typename Bytes>
  static Json parse(const Bytes& bytes) { return parse(std::string(bytes.begin(), bytes.end())); }

  Kind kind() const { return kind_; }
  bool is_null() const { return kind_ == Kind::Null; }
  bool is_number() const { return kind_ == Kind::Int || kind_ == Kind::Float; }
  bool is_string() const { return kind_ == Kind::String; }
  bool is_array() const { return kind_ == Kind::Array; }
  bool is_object() const { return kind_ == Kind::Object; }

  const Json& at(const std::string& key) const;
  Json& at(const std::string& key);
  const Json& at(size_t index) const;
  Json& operator[](const std::string& key);  // inserts null into objects (or null values)
  const Json& operator[](const std::string& key) const { return at(key); }
  Json& operator[](size_t index);
  bool contains(const std::string& key) const { return kind_ == Kind::Object && o_.count(key) > 0; }
  size_t size() const;
  void push_back(Json v);

  template <typename T> T get() const;

  // Implicit read conversions, as nlohmann offers (int n = j["n"];); defined
  // after the get<T> specializations below.
  template <typename T, typename std::enable_if<std::is_arithmetic<T>::value, int>::type = 0>
  operator T() const;
  operator std::string() const;

  const Array& items() const { return a_; }
  const Object& fields() const { return o_; }
  Array::const_iterator begin() const { return a_.begin(); }
  Array::const_iterator end() const { return a_.end(); }

  std::string dump(int indent = -1) const;
  bool operator==(const Json& other) const;
  bool operator!=(const Json& other) const { return !(*this == other); }

 private:
  void dump_to(std::string& out, int indent, int depth) const;
  Kind kind_ = Kind::Null;
  bool b_ = false;
  long long i_ = 0;
  double f_ = 0;
  std::string s_;
  Array a_;
  Object o_;
};

std::istream& operator>>(std::istream& in, Json& j);
std::ostream& operator<<(std::ostream& out, const Json& j);

template <> bool Json::get<bool>() const;
template <> int Json::get<int>() const;
template <> long Json::get<long>() const;
template <> long long Json::get<long long>() const;
template <> unsigned Json::get<unsigned>() const;
template <> unsigned long Json::get<unsigned long>() const;
template <> unsigned long long Json::get<unsigned long long>() const;
template <> float Json::get<float>() const;
template <> double Json::get<double>() const;
template <> std::string Json::get<std::string>() const;
template <> std::vector<int> Json::get<std::vector<int>>() const;
template <> std::vector<size_t> Json::get<std::vector<size_t>>() const;

template <typename T, typename std::enable_if<std::is_arithmetic<T>::value, int>::type>
Json::operator T() const { return get<T>(); }
inline Json::operator std::string() const { return get<std::string>(); }

}  // namespace Stream
