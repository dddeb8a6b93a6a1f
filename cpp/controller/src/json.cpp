#include "ds/json.hpp"

#include <cmath>
#include <cstdio>
#include <cstring>
#include <limits>

namespace ds {

Json::Json(double v) : type_(Type::Number), num_(v), integral_(false) {
  if (!std::isfinite(v)) throw JsonError("JSON numbers must be finite");
}

bool Json::as_bool() const {
  if (type_ != Type::Bool) throw JsonError("expected a boolean");
  return bool_;
}
double Json::as_double() const {
  if (type_ != Type::Number) throw JsonError("expected a number");
  return num_;
}
long long Json::as_int() const {
  if (type_ != Type::Number) throw JsonError("expected a number");
  if (std::floor(num_) != num_ || std::fabs(num_) > 9007199254740992.0) throw JsonError("expected an integer");
  return static_cast<long long>(num_);
}
const std::string& Json::as_string() const {
  if (type_ != Type::String) throw JsonError("expected a string");
  return *str_;
}
const Json::Array& Json::as_array() const {
  if (type_ != Type::Array) throw JsonError("expected an array");
  return *arr_;
}
Json::Array& Json::as_array() {
  if (type_ != Type::Array) throw JsonError("expected an array");
  detach();
  return *arr_;
}
const Json::Object& Json::as_object() const {
  if (type_ != Type::Object) throw JsonError("expected an object");
  return *obj_;
}
Json::Object& Json::as_object() {
  if (type_ != Type::Object) throw JsonError("expected an object");
  detach();
  return *obj_;
}

void Json::detach() {
  if (type_ == Type::Array && arr_ && arr_.use_count() > 1) arr_ = std::make_shared<Array>(*arr_);
  if (type_ == Type::Object && obj_ && obj_.use_count() > 1) obj_ = std::make_shared<Object>(*obj_);
}

bool Json::contains(const std::string& key) const {
  return type_ == Type::Object && obj_->count(key) != 0;
}

const Json& Json::at(const std::string& key) const {
  if (type_ != Type::Object) throw JsonError("expected an object with key '" + key + "'");
  auto it = obj_->find(key);
  if (it == obj_->end()) throw JsonError("missing key '" + key + "'");
  return it->second;
}

Json& Json::operator[](const std::string& key) {
  if (type_ == Type::Null) {
    type_ = Type::Object;
    obj_ = std::make_shared<Object>();
  }
  if (type_ != Type::Object) throw JsonError("not an object");
  detach();
  return (*obj_)[key];
}

const Json& Json::get(const std::string& key) const {
  static const Json null_json;
  if (type_ != Type::Object) return null_json;
  auto it = obj_->find(key);
  return it == obj_->end() ? null_json : it->second;
}

double Json::num(const std::string& key, double dflt) const {
  const Json& v = get(key);
  return v.is_null() ? dflt : v.as_double();
}
long long Json::integer(const std::string& key, long long dflt) const {
  const Json& v = get(key);
  return v.is_null() ? dflt : v.as_int();
}
bool Json::flag(const std::string& key, bool dflt) const {
  const Json& v = get(key);
  return v.is_null() ? dflt : v.as_bool();
}
std::string Json::str(const std::string& key, const std::string& dflt) const {
  const Json& v = get(key);
  return v.is_null() ? dflt : v.as_string();
}

const Json& Json::at(size_t i) const {
  if (type_ != Type::Array) throw JsonError("expected an array");
  if (i >= arr_->size()) throw JsonError("array index out of range");
  return (*arr_)[i];
}
Json& Json::at(size_t i) {
  if (type_ != Type::Array) throw JsonError("expected an array");
  detach();
  if (i >= arr_->size()) throw JsonError("array index out of range");
  return (*arr_)[i];
}
void Json::push_back(const Json& v) {
  if (type_ == Type::Null) {
    type_ = Type::Array;
    arr_ = std::make_shared<Array>();
  }
  if (type_ != Type::Array) throw JsonError("push_back on a non-array");
  detach();
  arr_->push_back(v);
}
size_t Json::size() const {
  switch (type_) {
    case Type::Array: return arr_->size();
    case Type::Object: return obj_->size();
    case Type::String: return str_->size();
    case Type::Null: return 0;
    default: return 1;
  }
}

bool Json::operator==(const Json& o) const {
  if (type_ != o.type_) return false;
  switch (type_) {
    case Type::Null: return true;
    case Type::Bool: return bool_ == o.bool_;
    case Type::Number: return num_ == o.num_;
    case Type::String: return *str_ == *o.str_;
    case Type::Array: return *arr_ == *o.arr_;
    case Type::Object: return *obj_ == *o.obj_;
  }
  return false;
}

std::string json_escape(const std::string& s) {
  std::string out;
  out.reserve(s.size() + 2);
  out.push_back('"');
  for (unsigned char c : s) {
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
          out.push_back(static_cast<char>(c));
        }
    }
  }
  out.push_back('"');
  return out;
}

static std::string format_number(double v, bool integral) {
  char buf[40];
  if (integral && std::fabs(v) < 9.2e18) {
    std::snprintf(buf, sizeof buf, "%lld", static_cast<long long>(v));
    return buf;
  }
  // shortest representation that round-trips
  for (int prec = 15; prec <= 17; ++prec) {
    std::snprintf(buf, sizeof buf, "%.*g", prec, v);
    if (std::strtod(buf, nullptr) == v) break;
  }
  std::string s = buf;
  if (s.find_first_of(".eEn") == std::string::npos) s += ".0";
  return s;
}

void Json::dump_to(std::string& out, int indent, int depth) const {
  auto newline = [&](int d) {
    if (indent < 0) return;
    out.push_back('\n');
    out.append(static_cast<size_t>(indent * d), ' ');
  };
  switch (type_) {
    case Type::Null: out += "null"; break;
    case Type::Bool: out += bool_ ? "true" : "false"; break;
    case Type::Number: out += format_number(num_, integral_); break;
    case Type::String: out += json_escape(*str_); break;
    case Type::Array: {
      out.push_back('[');
      bool first = true;
      for (const auto& v : *arr_) {
        if (!first) out.push_back(',');
        first = false;
        newline(depth + 1);
        v.dump_to(out, indent, depth + 1);
      }
      if (!arr_->empty()) newline(depth);
      out.push_back(']');
      break;
    }
    case Type::Object: {
      out.push_back('{');
      bool first = true;
      for (const auto& kv : *obj_) {
        if (!first) out.push_back(',');
        first = false;
        newline(depth + 1);
        out += json_escape(kv.first);
        out += indent < 0 ? ":" : ": ";
        kv.second.dump_to(out, indent, depth + 1);
      }
      if (!obj_->empty()) newline(depth);
      out.push_back('}');
      break;
    }
  }
}

std::string Json::dump(int indent) const {
  std::string out;
  dump_to(out, indent, 0);
  return out;
}

// ---------------------------------------------------------------------------
namespace {

struct Parser {
  const std::string& s;
  size_t i = 0;
  int depth = 0;

  [[noreturn]] void fail(const std::string& what) const {
    throw JsonError("JSON parse error at offset " + std::to_string(i) + ": " + what);
  }
  void ws() {
    while (i < s.size() && (s[i] == ' ' || s[i] == '\n' || s[i] == '\r' || s[i] == '\t')) ++i;
  }
  bool lit(const char* w) {
    size_t n = std::strlen(w);
    if (s.compare(i, n, w) == 0) {
      i += n;
      return true;
    }
    return false;
  }
  static void utf8(std::string& out, unsigned cp) {
    if (cp < 0x80) {
      out.push_back(static_cast<char>(cp));
    } else if (cp < 0x800) {
      out.push_back(static_cast<char>(0xC0 | (cp >> 6)));
      out.push_back(static_cast<char>(0x80 | (cp & 0x3F)));
    } else if (cp < 0x10000) {
      out.push_back(static_cast<char>(0xE0 | (cp >> 12)));
      out.push_back(static_cast<char>(0x80 | ((cp >> 6) & 0x3F)));
      out.push_back(static_cast<char>(0x80 | (cp & 0x3F)));
    } else {
      out.push_back(static_cast<char>(0xF0 | (cp >> 18)));
      out.push_back(static_cast<char>(0x80 | ((cp >> 12) & 0x3F)));
      out.push_back(static_cast<char>(0x80 | ((cp >> 6) & 0x3F)));
      out.push_back(static_cast<char>(0x80 | (cp & 0x3F)));
    }
  }
  unsigned hex4() {
    if (i + 4 > s.size()) fail("short \\u escape");
    unsigned v = 0;
    for (int k = 0; k < 4; ++k) {
      char c = s[i++];
      v <<= 4;
      if (c >= '0' && c <= '9') v |= c - '0';
      else if (c >= 'a' && c <= 'f') v |= c - 'a' + 10;
      else if (c >= 'A' && c <= 'F') v |= c - 'A' + 10;
      else fail("bad hex digit");
    }
    return v;
  }
  std::string string() {
    if (s[i] != '"') fail("expected string");
    ++i;
    std::string out;
    while (true) {
      if (i >= s.size()) fail("unterminated string");
      unsigned char c = static_cast<unsigned char>(s[i++]);
      if (c == '"') break;
      if (c < 0x20) fail("control character in string");
      if (c != '\\') {
        out.push_back(static_cast<char>(c));
        continue;
      }
      if (i >= s.size()) fail("bad escape");
      char e = s[i++];
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
          unsigned cp = hex4();
          if (cp >= 0xD800 && cp < 0xDC00) {
            if (!(i + 1 < s.size() && s[i] == '\\' && s[i + 1] == 'u')) fail("lone surrogate");
            i += 2;
            unsigned lo = hex4();
            if (lo < 0xDC00 || lo >= 0xE000) fail("bad surrogate pair");
            cp = 0x10000 + ((cp - 0xD800) << 10) + (lo - 0xDC00);
          } else if (cp >= 0xDC00 && cp < 0xE000) {
            fail("lone surrogate");
          }
          utf8(out, cp);
          break;
        }
        default: fail("bad escape");
      }
    }
    return out;
  }
  Json number() {
    size_t start = i;
    bool integral = true;
    if (s[i] == '-') ++i;
    if (i >= s.size()) fail("bad number");
    if (s[i] == '0') {
      ++i;
    } else if (s[i] >= '1' && s[i] <= '9') {
      while (i < s.size() && isdigit(static_cast<unsigned char>(s[i]))) ++i;
    } else {
      fail("bad number");
    }
    if (i < s.size() && s[i] == '.') {
      integral = false;
      ++i;
      if (i >= s.size() || !isdigit(static_cast<unsigned char>(s[i]))) fail("bad fraction");
      while (i < s.size() && isdigit(static_cast<unsigned char>(s[i]))) ++i;
    }
    if (i < s.size() && (s[i] == 'e' || s[i] == 'E')) {
      integral = false;
      ++i;
      if (i < s.size() && (s[i] == '+' || s[i] == '-')) ++i;
      if (i >= s.size() || !isdigit(static_cast<unsigned char>(s[i]))) fail("bad exponent");
      while (i < s.size() && isdigit(static_cast<unsigned char>(s[i]))) ++i;
    }
    const std::string tok = s.substr(start, i - start);
    double v = std::strtod(tok.c_str(), nullptr);
    if (!std::isfinite(v)) fail("number out of range");
    Json j(v);
    if (integral && std::fabs(v) <= 9007199254740992.0) {
      Json k(static_cast<long long>(v));
      return k;
    }
    return j;
  }
  Json value() {
    ws();
    if (i >= s.size()) fail("unexpected end");
    if (++depth > 512) fail("nesting too deep");
    Json out;
    char c = s[i];
    if (c == '{') {
      ++i;
      out = Json::object();
      ws();
      if (i < s.size() && s[i] == '}') {
        ++i;
      } else {
        while (true) {
          ws();
          if (i >= s.size() || s[i] != '"') fail("expected key");
          std::string key = string();
          if (out.contains(key)) fail("duplicate key '" + key + "'");
          ws();
          if (i >= s.size() || s[i] != ':') fail("expected ':'");
          ++i;
          out[key] = value();
          ws();
          if (i < s.size() && s[i] == ',') {
            ++i;
            continue;
          }
          if (i < s.size() && s[i] == '}') {
            ++i;
            break;
          }
          fail("expected ',' or '}'");
        }
      }
    } else if (c == '[') {
      ++i;
      out = Json::array();
      ws();
      if (i < s.size() && s[i] == ']') {
        ++i;
      } else {
        while (true) {
          out.push_back(value());
          ws();
          if (i < s.size() && s[i] == ',') {
            ++i;
            continue;
          }
          if (i < s.size() && s[i] == ']') {
            ++i;
            break;
          }
          fail("expected ',' or ']'");
        }
      }
    } else if (c == '"') {
      out = Json(string());
    } else if (lit("true")) {
      out = Json(true);
    } else if (lit("false")) {
      out = Json(false);
    } else if (lit("null")) {
      out = Json();
    } else if (c == '-' || (c >= '0' && c <= '9')) {
      out = number();
    } else {
      fail("unexpected character");
    }
    --depth;
    return out;
  }
};

}  // namespace

Json Json::parse(const std::string& text) {
  Parser p{text};
  Json v = p.value();
  p.ws();
  if (p.i != text.size()) p.fail("trailing characters");
  return v;
}

}  // namespace ds
