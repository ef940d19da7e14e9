#include "json.h"

#include <cmath>
#include <cstdio>
#include <cstdlib>
#include <cstring>

namespace rpgb {

namespace {

const Json& NullJson() {
  static const Json kNull;
  return kNull;
}

void AppendUtf8(uint32_t cp, std::string* out) {
  if (cp < 0x80) {
    out->push_back(static_cast<char>(cp));
  } else if (cp < 0x800) {
    out->push_back(static_cast<char>(0xC0 | (cp >> 6)));
    out->push_back(static_cast<char>(0x80 | (cp & 0x3F)));
  } else if (cp < 0x10000) {
    out->push_back(static_cast<char>(0xE0 | (cp >> 12)));
    out->push_back(static_cast<char>(0x80 | ((cp >> 6) & 0x3F)));
    out->push_back(static_cast<char>(0x80 | (cp & 0x3F)));
  } else {
    out->push_back(static_cast<char>(0xF0 | (cp >> 18)));
    out->push_back(static_cast<char>(0x80 | ((cp >> 12) & 0x3F)));
    out->push_back(static_cast<char>(0x80 | ((cp >> 6) & 0x3F)));
    out->push_back(static_cast<char>(0x80 | (cp & 0x3F)));
  }
}

class Parser {
 public:
  explicit Parser(const std::string& t) : t_(t) {}
  bool Run(Json* out, std::string* err) {
    Ws();
    if (!Value(out, 0)) {
      *err = err_.empty() ? "invalid JSON" : err_;
      return false;
    }
    Ws();
    if (p_ != t_.size()) {
      *err = "trailing characters after JSON value at offset " + std::to_string(p_);
      return false;
    }
    return true;
  }

 private:
  void Ws() {
    while (p_ < t_.size() && (t_[p_] == ' ' || t_[p_] == '\t' || t_[p_] == '\n' || t_[p_] == '\r')) ++p_;
  }
  bool Fail(const char* m) {
    if (err_.empty()) err_ = std::string(m) + " at offset " + std::to_string(p_);
    return false;
  }
  bool Lit(const char* s) {
    size_t n = 0;
    while (s[n]) ++n;
    if (t_.compare(p_, n, s) != 0) return Fail("bad literal");
    p_ += n;
    return true;
  }
  bool Hex4(uint32_t* v) {
    if (p_ + 4 > t_.size()) return Fail("short \\u escape");
    *v = 0;
    for (int i = 0; i < 4; ++i) {
      const char c = t_[p_++];
      *v <<= 4;
      if (c >= '0' && c <= '9') *v |= static_cast<uint32_t>(c - '0');
      else if (c >= 'a' && c <= 'f') *v |= static_cast<uint32_t>(c - 'a' + 10);
      else if (c >= 'A' && c <= 'F') *v |= static_cast<uint32_t>(c - 'A' + 10);
      else return Fail("bad hex digit");
    }
    return true;
  }
  bool String(std::string* s) {
    if (t_[p_] != '"') return Fail("expected string");
    ++p_;
    while (p_ < t_.size()) {
      const char c = t_[p_++];
      if (c == '"') return true;
      if (static_cast<unsigned char>(c) < 0x20) return Fail("control character in string");
      if (c != '\\') {
        s->push_back(c);
        continue;
      }
      if (p_ >= t_.size()) break;
      const char e = t_[p_++];
      switch (e) {
        case '"': s->push_back('"'); break;
        case '\\': s->push_back('\\'); break;
        case '/': s->push_back('/'); break;
        case 'b': s->push_back('\b'); break;
        case 'f': s->push_back('\f'); break;
        case 'n': s->push_back('\n'); break;
        case 'r': s->push_back('\r'); break;
        case 't': s->push_back('\t'); break;
        case 'u': {
          uint32_t cp;
          if (!Hex4(&cp)) return false;
          if (cp >= 0xD800 && cp < 0xDC00 && p_ + 6 <= t_.size() && t_[p_] == '\\' && t_[p_ + 1] == 'u') {
            p_ += 2;
            uint32_t lo;
            if (!Hex4(&lo)) return false;
            if (lo >= 0xDC00 && lo < 0xE000) {
              cp = 0x10000 + ((cp - 0xD800) << 10) + (lo - 0xDC00);
            } else {
              AppendUtf8(0xFFFD, s);
              cp = lo;
            }
          }
          if (cp >= 0xD800 && cp < 0xE000) cp = 0xFFFD;
          AppendUtf8(cp, s);
          break;
        }
        default: return Fail("bad escape");
      }
    }
    return Fail("unterminated string");
  }
  bool Value(Json* out, int depth) {
    if (depth > 200) return Fail("nesting too deep");
    if (p_ >= t_.size()) return Fail("unexpected end");
    const char c = t_[p_];
    if (c == 'n') {
      *out = Json();
      return Lit("null");
    }
    if (c == 't') {
      *out = Json::Bool(true);
      return Lit("true");
    }
    if (c == 'f') {
      *out = Json::Bool(false);
      return Lit("false");
    }
    if (c == '"') {
      std::string s;
      if (!String(&s)) return false;
      *out = Json::Str(s);
      return true;
    }
    if (c == '[') {
      ++p_;
      *out = Json::Array();
      Ws();
      if (p_ < t_.size() && t_[p_] == ']') {
        ++p_;
        return true;
      }
      while (true) {
        Json v;
        Ws();
        if (!Value(&v, depth + 1)) return false;
        out->Push(std::move(v));
        Ws();
        if (p_ < t_.size() && t_[p_] == ',') {
          ++p_;
          continue;
        }
        if (p_ < t_.size() && t_[p_] == ']') {
          ++p_;
          return true;
        }
        return Fail("expected , or ]");
      }
    }
    if (c == '{') {
      ++p_;
      *out = Json::Object();
      Ws();
      if (p_ < t_.size() && t_[p_] == '}') {
        ++p_;
        return true;
      }
      while (true) {
        Ws();
        std::string k;
        if (p_ >= t_.size() || !String(&k)) return Fail("expected key");
        Ws();
        if (p_ >= t_.size() || t_[p_] != ':') return Fail("expected :");
        ++p_;
        Ws();
        Json v;
        if (!Value(&v, depth + 1)) return false;
        out->Set(k, std::move(v));
        Ws();
        if (p_ < t_.size() && t_[p_] == ',') {
          ++p_;
          continue;
        }
        if (p_ < t_.size() && t_[p_] == '}') {
          ++p_;
          return true;
        }
        return Fail("expected , or }");
      }
    }
    // number
    const size_t start = p_;
    if (t_[p_] == '-') ++p_;
    while (p_ < t_.size() && (isdigit(static_cast<unsigned char>(t_[p_])) || t_[p_] == '.' || t_[p_] == 'e' ||
                              t_[p_] == 'E' || t_[p_] == '+' || t_[p_] == '-')) {
      ++p_;
    }
    if (p_ == start) return Fail("unexpected character");
    const std::string num = t_.substr(start, p_ - start);
    char* end = nullptr;
    const double d = std::strtod(num.c_str(), &end);
    if (end == nullptr || *end != '\0') return Fail("bad number");
    const bool integral = num.find_first_of(".eE") == std::string::npos;
    *out = integral ? Json::IntLiteral(d) : Json::Number(d);
    return true;
  }

  const std::string& t_;
  size_t p_ = 0;
  std::string err_;
};

std::string PyFloat(double d) {
  char buf[40];
  if (!std::isfinite(d)) return d != d ? "NaN" : (d > 0 ? "Infinity" : "-Infinity");
  if (d == std::floor(d) && std::fabs(d) < 1e16) {
    std::snprintf(buf, sizeof(buf), "%.0f.0", d);
    return buf;
  }
  for (int p = 1; p <= 17; ++p) {
    std::snprintf(buf, sizeof(buf), "%.*g", p, d);
    if (std::strtod(buf, nullptr) == d) break;
  }
  return buf;
}

void Dump(const Json& j, std::string* out, bool py);

void DumpNum(const Json& j, std::string* out, bool py) {
  const double d = j.AsDouble();
  char buf[40];
  if (py && !j.IsIntLiteral()) {
    *out += PyFloat(d);
  } else if (std::isfinite(d) && std::fabs(d) < 9.007199254740992e15 && d == std::floor(d)) {
    std::snprintf(buf, sizeof(buf), "%lld", static_cast<long long>(d));
    *out += buf;
  } else if (std::isfinite(d)) {
    std::snprintf(buf, sizeof(buf), "%.17g", d);
    *out += buf;
  } else {
    *out += "null";
  }
}

void Dump(const Json& j, std::string* out) { Dump(j, out, false); }

void Dump(const Json& j, std::string* out, bool py) {
  switch (j.type()) {
    case Json::Type::kNull: *out += "null"; break;
    case Json::Type::kBool: *out += j.AsBool() ? "true" : "false"; break;
    case Json::Type::kNumber: DumpNum(j, out, py); break;
    case Json::Type::kString: JsonEscape(j.AsString(), out); break;
    case Json::Type::kArray: {
      *out += '[';
      for (size_t i = 0; i < j.size(); ++i) {
        if (i) *out += py ? ", " : ",";
        Dump(j.At(i), out, py);
      }
      *out += ']';
      break;
    }
    case Json::Type::kObject: {
      *out += '{';
      bool first = true;
      for (const auto& kv : j.Items()) {
        if (!first) *out += py ? ", " : ",";
        first = false;
        JsonEscape(kv.first, out);
        *out += py ? ": " : ":";
        Dump(kv.second, out, py);
      }
      *out += '}';
      break;
    }
  }
}

}  // namespace

void JsonEscape(const std::string& s, std::string* out) {
  *out += '"';
  for (unsigned char c : s) {
    switch (c) {
      case '"': *out += "\\\""; break;
      case '\\': *out += "\\\\"; break;
      case '\n': *out += "\\n"; break;
      case '\r': *out += "\\r"; break;
      case '\t': *out += "\\t"; break;
      case '\b': *out += "\\b"; break;
      case '\f': *out += "\\f"; break;
      default:
        if (c < 0x20) {
          char buf[8];
          std::snprintf(buf, sizeof(buf), "\\u%04x", c);
          *out += buf;
        } else {
          out->push_back(static_cast<char>(c));
        }
    }
  }
  *out += '"';
}

Json Json::Bool(bool b) {
  Json j;
  j.type_ = Type::kBool;
  j.b_ = b;
  return j;
}
Json Json::Number(double d) {
  Json j;
  j.type_ = Type::kNumber;
  j.d_ = d;
  return j;
}
Json Json::Str(const std::string& s) {
  Json j;
  j.type_ = Type::kString;
  j.s_ = s;
  return j;
}
Json Json::Array() {
  Json j;
  j.type_ = Type::kArray;
  j.arr_ = std::make_shared<std::vector<Json>>();
  return j;
}
Json Json::Object() {
  Json j;
  j.type_ = Type::kObject;
  j.obj_ = std::make_shared<std::map<std::string, Json>>();
  j.order_ = std::make_shared<std::vector<std::pair<std::string, Json>>>();
  return j;
}

Json Json::Parse(const std::string& text, std::string* err) {
  Json out;
  std::string e;
  Parser p(text);
  if (!p.Run(&out, &e)) {
    if (err) *err = e;
    return Json();
  }
  if (err) err->clear();
  return out;
}

std::string Json::Dump() const {
  std::string s;
  rpgb::Dump(*this, &s, false);
  return s;
}

std::string Json::DumpPython() const {
  std::string s;
  rpgb::Dump(*this, &s, true);
  return s;
}

Json Json::IntLiteral(double d) {
  Json j = Number(d);
  j.int_lit_ = true;
  return j;
}

const Json& Json::Get(const std::string& k) const {
  if (!IsObject()) return NullJson();
  const auto it = obj_->find(k);
  return it == obj_->end() ? NullJson() : it->second;
}

Json& Json::Set(const std::string& k, Json v) {
  if (!IsObject()) *this = Object();
  auto it = obj_->find(k);
  if (it == obj_->end()) {
    order_->emplace_back(k, v);
    return (*obj_)[k] = std::move(v);
  }
  for (auto& kv : *order_) {
    if (kv.first == k) kv.second = v;
  }
  it->second = std::move(v);
  return it->second;
}

size_t Json::size() const {
  if (IsArray()) return arr_->size();
  if (IsObject()) return obj_->size();
  return 0;
}

const Json& Json::At(size_t i) const {
  if (!IsArray() || i >= arr_->size()) return NullJson();
  return (*arr_)[i];
}

void Json::Push(Json v) {
  if (!IsArray()) *this = Array();
  arr_->push_back(std::move(v));
}

const std::vector<std::pair<std::string, Json>>& Json::Items() const {
  static const std::vector<std::pair<std::string, Json>> kEmpty;
  return IsObject() ? *order_ : kEmpty;
}

}  // namespace rpgb
