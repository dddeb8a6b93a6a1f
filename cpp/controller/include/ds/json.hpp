// Strict JSON value, parser and serializer for the controller.
//
// Strictness matches the worker protocol: no NaN/Infinity (not JSON), no
// trailing garbage, no duplicate object keys, no control characters in
// strings.  Objects keep their keys sorted (std::map) so every dump is
// deterministic, which the golden-fixture tests rely on.  Numbers remember
// whether they were written as integers so ids and counters print without a
// fractional part.
#pragma once
#include <cstdint>
#include <map>
#include <memory>
#include <stdexcept>
#include <string>
#include <vector>

namespace ds {

class JsonError : public std::runtime_error {
 public:
  using std::runtime_error::runtime_error;
};

class Json {
 public:
  enum class Type { Null, Bool, Number, String, Array, Object };
  using Array = std::vector<Json>;
  using Object = std::map<std::string, Json>;

  Json() = default;
  Json(std::nullptr_t) {}
  Json(bool b) : type_(Type::Bool), bool_(b) {}
  Json(int v) : type_(Type::Number), num_(v), integral_(true) {}
  Json(long v) : type_(Type::Number), num_(static_cast<double>(v)), integral_(true) {}
  Json(long long v) : type_(Type::Number), num_(static_cast<double>(v)), integral_(true) {}
  Json(unsigned v) : type_(Type::Number), num_(v), integral_(true) {}
  Json(unsigned long v) : type_(Type::Number), num_(static_cast<double>(v)), integral_(true) {}
  Json(unsigned long long v) : type_(Type::Number), num_(static_cast<double>(v)), integral_(true) {}
  Json(double v);
  Json(const char* s) : type_(Type::String), str_(std::make_shared<std::string>(s)) {}
  Json(const std::string& s) : type_(Type::String), str_(std::make_shared<std::string>(s)) {}
  Json(const Array& a) : type_(Type::Array), arr_(std::make_shared<Array>(a)) {}
  Json(const Object& o) : type_(Type::Object), obj_(std::make_shared<Object>(o)) {}

  static Json array() { return Json(Array{}); }
  static Json object() { return Json(Object{}); }
  static Json parse(const std::string& text);

  Type type() const { return type_; }
  bool is_null() const { return type_ == Type::Null; }
  bool is_bool() const { return type_ == Type::Bool; }
  bool is_number() const { return type_ == Type::Number; }
  bool is_integer() const { return type_ == Type::Number && integral_; }
  bool is_string() const { return type_ == Type::String; }
  bool is_array() const { return type_ == Type::Array; }
  bool is_object() const { return type_ == Type::Object; }

  bool as_bool() const;
  double as_double() const;
  long long as_int() const;
  const std::string& as_string() const;
  const Array& as_array() const;
  Array& as_array();
  const Object& as_object() const;
  Object& as_object();

  // object access
  bool contains(const std::string& key) const;
  const Json& at(const std::string& key) const;
  Json& operator[](const std::string& key);  // creates (null -> object)
  const Json& operator[](const std::string& key) const { return at(key); }
  // typed lookups with defaults (missing or null -> default)
  double num(const std::string& key, double dflt) const;
  long long integer(const std::string& key, long long dflt) const;
  bool flag(const std::string& key, bool dflt) const;
  std::string str(const std::string& key, const std::string& dflt) const;
  const Json& get(const std::string& key) const;  // null Json when missing

  // array access
  const Json& at(size_t i) const;
  Json& at(size_t i);
  const Json& operator[](size_t i) const { return at(i); }
  Json& operator[](size_t i) { return at(i); }
  void push_back(const Json& v);
  size_t size() const;
  bool empty() const { return size() == 0; }

  std::string dump(int indent = -1) const;
  bool operator==(const Json& o) const;
  bool operator!=(const Json& o) const { return !(*this == o); }

 private:
  void detach();  // copy-on-write for shared containers
  void dump_to(std::string& out, int indent, int depth) const;

  Type type_ = Type::Null;
  bool bool_ = false;
  double num_ = 0.0;
  bool integral_ = false;
  std::shared_ptr<std::string> str_;
  std::shared_ptr<Array> arr_;
  std::shared_ptr<Object> obj_;
};

std::string json_escape(const std::string& s);

}  // namespace ds
