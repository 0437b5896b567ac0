// Json.cpp -- parser, printer and accessors of Stream::Json (include/Json.hpp).
#include "Json.hpp"

#include <cmath>
#include <cstdio>
#include <cstdlib>
#include <sstream>

namespace Stream {

Json::Json(std::initializer_list<Json> init) {
  bool pairs = init.size() > 0;
  for (const auto& e : init)
    if (!(e.kind_ == Kind::Array && e.a_.size() == 2 && e.a_[0].kind_ == Kind::String)) pairs = false;
  if (pairs) {
    kind_ = Kind::Object;
    for (const auto& e : init) o_[e.a_[0].s_] = e.a_[1];
  } else {
    kind_ = Kind::Array;
    a_.assign(init.begin(), init.end());
  }
}

const Json& Json::at(const std::string& key) const {
  if (kind_ != Kind::Object) throw std::runtime_error("JSON value is not an object (key " + key + ")");
  auto it = o_.find(key);
  if (it == o_.end()) throw std::runtime_error("JSON key not found: " + key);
  return it->second;
}
Json& Json::at(const std::string& key) {
  return const_cast<Json&>(static_cast<const Json&>(*this).at(key));
}
const Json& Json::at(size_t index) const {
  if (kind_ != Kind::Array || index >= a_.size()) throw std::runtime_error("JSON array index out of range");
  return a_[index];
}
Json& Json::operator[](const std::string& key) {
  if (kind_ == Kind::Null) kind_ = Kind::Object;
  if (kind_ != Kind::Object) throw std::runtime_error("JSON value is not an object (key " + key + ")");
  return o_[key];
}
Json& Json::operator[](size_t index) {
  if (kind_ != Kind::Array || index >= a_.size()) throw std::runtime_error("JSON array index out of range");
  return a_[index];
}
size_t Json::size() const {
  if (kind_ == Kind::Array) return a_.size();
  if (kind_ == Kind::Object) return o_.size();
  return kind_ == Kind::Null ? 0 : 1;
}
void Json::push_back(Json v) {
  if (kind_ == Kind::Null) kind_ = Kind::Array;
  if (kind_ != Kind::Array) throw std::runtime_error("push_back on a non-array JSON value");
  a_.push_back(std::move(v));
}

namespace {
double number_of(Json::Kind k, long long i, double f, bool b) {
  if (k == Json::Kind::Int) return (double)i;
  if (k == Json::Kind::Float) return f;
  if (k == Json::Kind::Bool) return b ? 1 : 0;
  throw std::runtime_error("JSON value is not a number");
}
}  // namespace

template <> bool Json::get<bool>() const {
  if (kind_ == Kind::Bool) return b_;
  return number_of(kind_, i_, f_, b_) != 0;
}
template <> long long Json::get<long long>() const {
  if (kind_ == Kind::Int) return i_;
  const double v = number_of(kind_, i_, f_, b_);
  if (v != std::floor(v)) throw std::runtime_error("JSON number is not an integer");
  return (long long)v;
}
template <> int Json::get<int>() const { return (int)get<long long>(); }
template <> long Json::get<long>() const { return (long)get<long long>(); }
template <> unsigned Json::get<unsigned>() const { return (unsigned)get<long long>(); }
template <> unsigned long Json::get<unsigned long>() const { return (unsigned long)get<long long>(); }
template <> unsigned long long Json::get<unsigned long long>() const { return (unsigned long long)get<long long>(); }
template <> double Json::get<double>() const { return number_of(kind_, i_, f_, b_); }
template <> float Json::get<float>() const { return (float)get<double>(); }
template <> std::string Json::get<std::string>() const {
  if (kind_ != Kind::String) throw std::runtime_error("JSON value is not a string");
  return s_;
}
template <> std::vector<int> Json::get<std::vector<int>>() const {
  if (kind_ != Kind::Array) throw std::runtime_error("JSON value is not an array");
  std::vector<int> out;
  for (const auto& e : a_) out.push_back(e.get<int>());
  return out;
}
template <> std::vector<size_t> Json::get<std::vector<size_t>>() const {
  if (kind_ != Kind::Array) throw std::runtime_error("JSON value is not an array");
  std::vector<size_t> out;
  for (const auto& e : a_) out.push_back((size_t)e.get<long long>());
  return out;
}

bool Json::operator==(const Json& o) const {
  if (is_number() && o.is_number()) {
    if (kind_ == Kind::Int && o.kind_ == Kind::Int) return i_ == o.i_;
    return get<double>() == o.get<double>();
  }
  if (kind_ != o.kind_) return false;
  switch (kind_) {
    case Kind::Null: return true;
    case Kind::Bool: return b_ == o.b_;
    case Kind::String: return s_ == o.s_;
    case Kind::Array: return a_ == o.a_;
    case Kind::Object: return o_ == o.o_;
    default: return false;
  }
}

namespace {
void escape(std::string& out, const std::string& s) {
  out += '"';
  for (unsigned char c : s) {
    switch (c) {
      case '"': out += "\\\""; break;
      case '\\': out += "\\\\"; break;
      case '\n': out += "\\n"; break;
      case '\r': out += "\\r"; break;
      case '\t': out += "\\t"; break;
      default:
        if (c < 0x20) {
          char b[8];
          std::snprintf(b, sizeof b, "\\u%04x", c);
          out += b;
        } else {
          out += (char)c;
        }
    }
  }
  out += '"';
}
}  // namespace

void Json::dump_to(std::string& out, int indent, int depth) const {
  auto newline = [&](int d) {
    if (indent < 0) return;
    out += '\n';
    out.append((size_t)(indent * d), ' ');
  };
  switch (kind_) {
    case Kind::Null: out += "null"; break;
    case Kind::Bool: out += b_ ? "true" : "false"; break;
    case Kind::Int: out += std::to_string(i_); break;
    case Kind::Float: {
      if (!std::isfinite(f_)) { out += "null"; break; }
      char b[32];
      std::snprintf(b, sizeof b, "%.17g", f_);
      std::string t = b;
      if (t.find_first_of(".eE") == std::string::npos) t += ".0";
      out += t;
      break;
    }
    case Kind::String: escape(out, s_); break;
    case Kind::Array:
      out += '[';
      for (size_t i = 0; i < a_.size(); ++i) {
        if (i) out += ',';
        newline(depth + 1);
        a_[i].dump_to(out, indent, depth + 1);
      }
      if (!a_.empty()) newline(depth);
      out += ']';
      break;
    case Kind::Object: {
      out += '{';
      size_t i = 0;
      for (const auto& kv : o_) {
        if (i++) out += ',';
        newline(depth + 1);
        escape(out, kv.first);
        out += indent < 0 ? ":" : ": ";
        kv.second.dump_to(out, indent, depth + 1);
      }
      if (!o_.empty()) newline(depth);
      out += '}';
      break;
    }
  }
}

std::string Json::dump(int indent) const {
  std::string out;
  dump_to(out, indent, 0);
  return out;
}

namespace {
struct Parser {
  const std::string& t;
  size_t p = 0;
  [[noreturn]] void fail(const char* what) {
    throw std::runtime_error(std::string("JSON parse error: ") + what + " at offset " + std::to_string(p));
  }
  void ws() {
    while (p < t.size() && (t[p] == ' ' || t[p] == '\n' || t[p] == '\r' || t[p] == '\t')) ++p;
  }
  bool take(const char* lit) {
    const size_t n = std::char_traits<char>::length(lit);
    if (t.compare(p, n, lit) == 0) { p += n; return true; }
    return false;
  }
  std::string string() {
    if (t[p] != '"') fail("expected string");
    ++p;
    std::string out;
    while (p < t.size() && t[p] != '"') {
      char c = t[p++];
      if (c == '\\') {
        if (p >= t.size()) fail("bad escape");
        const char e = t[p++];
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
            if (p + 4 > t.size()) fail("bad unicode escape");
            const unsigned cp = (unsigned)std::strtoul(t.substr(p, 4).c_str(), nullptr, 16);
            p += 4;
            if (cp < 0x80) out += (char)cp;
            else if (cp < 0x800) { out += (char)(0xc0 | (cp >> 6)); out += (char)(0x80 | (cp & 0x3f)); }
            else { out += (char)(0xe0 | (cp >> 12)); out += (char)(0x80 | ((cp >> 6) & 0x3f)); out += (char)(0x80 | (cp & 0x3f)); }
            break;
          }
          default: fail("bad escape");
        }
      } else {
        out += c;
      }
    }
    if (p >= t.size()) fail("unterminated string");
    ++p;
    return out;
  }
  Json value() {
    ws();
    if (p >= t.size()) fail("unexpected end");
    const char c = t[p];
    if (c == '{') {
      ++p;
      Json o = Json::object();
      ws();
      if (t[p] == '}') { ++p; return o; }
      while (true) {
        ws();
        std::string k = string();
        ws();
        if (t[p] != ':') fail("expected ':'");
        ++p;
        o[k] = value();
        ws();
        if (t[p] == ',') { ++p; continue; }
        if (t[p] == '}') { ++p; return o; }
        fail("expected ',' or '}'");
      }
    }
    if (c == '[') {
      ++p;
      Json a = Json::array();
      ws();
      if (t[p] == ']') { ++p; return a; }
      while (true) {
        a.push_back(value());
        ws();
        if (t[p] == ',') { ++p; continue; }
        if (t[p] == ']') { ++p; return a; }
        fail("expected ',' or ']'");
      }
    }
    if (c == '"') return Json(string());
    if (take("true")) return Json(true);
    if (take("false")) return Json(false);
    if (take("null")) return Json(nullptr);
    const size_t start = p;
    bool real = false;
    if (t[p] == '-' || t[p] == '+') ++p;
    while (p < t.size() && (isdigit((unsigned char)t[p]) || t[p] == '.' || t[p] == 'e' || t[p] == 'E' || t[p] == '-' || t[p] == '+')) {
      if (t[p] == '.' || t[p] == 'e' || t[p] == 'E') real = true;
      ++p;
    }
    if (p == start) fail("unexpected character");
    const std::string num = t.substr(start, p - start);
    if (real) return Json(std::strtod(num.c_str(), nullptr));
    return Json(std::strtoll(num.c_str(), nullptr, 10));
  }
};
}  // namespace

Json Json::parse(const std::string& text) {
  Parser parser{text};
  Json v = parser.value();
  parser.ws();
  if (parser.p != text.size()) parser.fail("trailing characters");
  return v;
}

std::istream& operator>>(std::istream& in, Json& j) {
  std::stringstream ss;
  ss << in.rdbuf();
  j = Json::parse(ss.str());
  return in;
}

std::ostream& operator<<(std::ostream& out, const Json& j) { return out << j.dump(); }

}  // namespace Stream
