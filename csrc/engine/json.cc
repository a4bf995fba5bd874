#include "json.h"

#include <cmath>
#include <cstdio>
#include <cstdlib>

#include "runtime.h"

namespace foa::engine {

class JsonParser {
 public:
  explicit JsonParser(const std::string& t) : t_(t) {}

  Json parse_all() {
    Json v = value();
    ws();
    if (p_ != t_.size()) fail("trailing characters");
    return v;
  }

 private:
  const std::string& t_;
  size_t p_ = 0;

  [[noreturn]] void fail(const char* what) {
    throw ValueError(std::string("malformed JSON at byte ") + std::to_string(p_) + ": " + what);
  }
  void ws() {
    while (p_ < t_.size() && (t_[p_] == ' ' || t_[p_] == '\n' || t_[p_] == '\r' || t_[p_] == '\t')) ++p_;
  }
  bool eat(char c) {
    ws();
    if (p_ < t_.size() && t_[p_] == c) {
      ++p_;
      return true;
    }
    return false;
  }
  void expect(const char* lit) {
    for (const char* c = lit; *c; ++c) {
      if (p_ >= t_.size() || t_[p_] != *c) fail("unexpected literal");
      ++p_;
    }
  }
  static void utf8(std::string& out, uint32_t cp) {
    if (cp < 0x80) {
      out += static_cast<char>(cp);
    } else if (cp < 0x800) {
      out += static_cast<char>(0xC0 | (cp >> 6));
      out += static_cast<char>(0x80 | (cp & 0x3F));
    } else if (cp < 0x10000) {
      out += static_cast<char>(0xE0 | (cp >> 12));
      out += static_cast<char>(0x80 | ((cp >> 6) & 0x3F));
      out += static_cast<char>(0x80 | (cp & 0x3F));
    } else {
      out += static_cast<char>(0xF0 | (cp >> 18));
      out += static_cast<char>(0x80 | ((cp >> 12) & 0x3F));
      out += static_cast<char>(0x80 | ((cp >> 6) & 0x3F));
      out += static_cast<char>(0x80 | (cp & 0x3F));
    }
  }
  uint32_t hex4() {
    if (p_ + 4 > t_.size()) fail("short escape");
    uint32_t v = 0;
    for (int i = 0; i < 4; ++i) {
      const char c = t_[p_++];
      v <<= 4;
      if (c >= '0' && c <= '9') v |= c - '0';
      else if (c >= 'a' && c <= 'f') v |= c - 'a' + 10;
      else if (c >= 'A' && c <= 'F') v |= c - 'A' + 10;
      else fail("bad escape");
    }
    return v;
  }
  std::string str() {
    if (!eat('"')) fail("expected a string");
    std::string out;
    while (true) {
      if (p_ >= t_.size()) fail("unterminated string");
      const char c = t_[p_++];
      if (c == '"') break;
      if (c != '\\') {
        out += c;
        continue;
      }
      if (p_ >= t_.size()) fail("unterminated escape");
      const char e = t_[p_++];
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
          if (cp >= 0xD800 && cp < 0xDC00 && p_ + 6 <= t_.size() && t_[p_] == '\\' && t_[p_ + 1] == 'u') {
            p_ += 2;
            const uint32_t lo = hex4();
            cp = 0x10000 + ((cp - 0xD800) << 10) + (lo - 0xDC00);
          }
          utf8(out, cp);
          break;
        }
        default: fail("bad escape");
      }
    }
    return out;
  }
  Json value() {
    ws();
    if (p_ >= t_.size()) fail("unexpected end");
    const char c = t_[p_];
    if (c == '{') {
      ++p_;
      Json o = Json::object({});
      if (eat('}')) return o;
      do {
        ws();
        std::string k = str();
        if (!eat(':')) fail("expected ':'");
        o.obj_.emplace_back(std::move(k), value());
      } while (eat(','));
      if (!eat('}')) fail("expected '}'");
      return o;
    }
    if (c == '[') {
      ++p_;
      Json a = Json::array({});
      if (eat(']')) return a;
      do {
        a.arr_.push_back(value());
      } while (eat(','));
      if (!eat(']')) fail("expected ']'");
      return a;
    }
    if (c == '"') return Json::string(str());
    if (c == 't') {
      expect("true");
      return Json::boolean(true);
    }
    if (c == 'f') {
      expect("false");
      return Json::boolean(false);
    }
    if (c == 'n') {
      expect("null");
      return Json();
    }
    if (c == 'N') {
      expect("NaN");
      return Json::number(std::nan(""));
    }
    if (c == 'I') {
      expect("Infinity");
      return Json::number(INFINITY);
    }
    // number
    const size_t start = p_;
    bool integral = true;
    if (t_[p_] == '-') ++p_;
    if (p_ < t_.size() && t_[p_] == 'I') {
      expect("Infinity");
      return Json::number(-INFINITY);
    }
    while (p_ < t_.size()) {
      const char d = t_[p_];
      if (d >= '0' && d <= '9') {
        ++p_;
      } else if (d == '.' || d == 'e' || d == 'E' || d == '+' || d == '-') {
        integral = false;
        ++p_;
      } else {
        break;
      }
    }
    if (p_ == start) fail("unexpected character");
    const std::string num = t_.substr(start, p_ - start);
    if (integral) {
      errno = 0;
      char* end = nullptr;
      const long long v = std::strtoll(num.c_str(), &end, 10);
      if (errno == 0 && end && *end == '\0') return Json::integer(v);
    }
    return Json::number(std::strtod(num.c_str(), nullptr));
  }
};

Json Json::parse(const std::string& text) { return JsonParser(text).parse_all(); }

const Json& Json::operator[](const std::string& key) const {
  static const Json kNull;
  if (type_ != Type::Object) return kNull;
  for (const auto& m : obj_)
    if (m.first == key) return m.second;
  return kNull;
}

bool Json::contains(const std::string& key) const {
  if (type_ != Type::Object) return false;
  for (const auto& m : obj_)
    if (m.first == key) return true;
  return false;
}

Json Json::boolean(bool v) {
  Json j;
  j.type_ = Type::Bool;
  j.b_ = v;
  return j;
}
Json Json::number(double v) {
  Json j;
  j.type_ = Type::Number;
  j.num_ = v;
  j.i_ = static_cast<int64_t>(v);
  j.integral_ = false;
  return j;
}
Json Json::integer(int64_t v) {
  Json j;
  j.type_ = Type::Number;
  j.num_ = static_cast<double>(v);
  j.i_ = v;
  j.integral_ = true;
  return j;
}
Json Json::string(std::string v) {
  Json j;
  j.type_ = Type::String;
  j.s_ = std::move(v);
  return j;
}
Json Json::array(std::vector<Json> v) {
  Json j;
  j.type_ = Type::Array;
  j.arr_ = std::move(v);
  return j;
}
Json Json::object(std::vector<std::pair<std::string, Json>> v) {
  Json j;
  j.type_ = Type::Object;
  j.obj_ = std::move(v);
  return j;
}

void Json::set(const std::string& key, Json v) {
  if (type_ != Type::Object) *this = object({});
  for (auto& m : obj_)
    if (m.first == key) {
      m.second = std::move(v);
      return;
    }
  obj_.emplace_back(key, std::move(v));
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
          char buf[8];
          std::snprintf(buf, sizeof(buf), "\\u%04x", c);
          out += buf;
        } else {
          out += static_cast<char>(c);
        }
    }
  }
  out += '"';
}
}  // namespace

std::string Json::dump() const {
  std::string out;
  switch (type_) {
    case Type::Null: return "null";
    case Type::Bool: return b_ ? "true" : "false";
    case Type::Number: {
      if (integral_) return std::to_string(i_);
      char buf[64];
      std::snprintf(buf, sizeof(buf), "%.17g", num_);
      return buf;
    }
    case Type::String: escape(out, s_); return out;
    case Type::Array:
      out += '[';
      for (size_t i = 0; i < arr_.size(); ++i) {
        if (i) out += ',';
        out += arr_[i].dump();
      }
      return out + ']';
    case Type::Object:
      out += '{';
      for (size_t i = 0; i < obj_.size(); ++i) {
        if (i) out += ',';
        escape(out, obj_[i].first);
        out += ':';
        out += obj_[i].second.dump();
      }
      return out + '}';
  }
  return out;
}

}  // namespace foa::engine
