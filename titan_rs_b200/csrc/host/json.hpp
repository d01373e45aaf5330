// JSON text in the form Python's json module reads and writes, for the host-side
// stores and compilers of libtitan_b200 (the `.tune` file, the graph compiler).
//
// The parser accepts what json.loads accepts in strict mode: whitespace " \t\n\r",
// NaN/Infinity/-Infinity, ASCII-digit numbers, no control characters inside strings,
// \uXXXX escapes with surrogate pairs joined. `emit` writes the canonical form,
// byte-identical to json.dumps(obj, sort_keys=True, separators=(",", ":")): members
// sorted by code point, ASCII only with lowercase \uXXXX escapes, integers as written
// ("-0" as "0"), floats as Python's repr, NaN/Infinity/-Infinity as bare words.
#pragma once

#include <charconv>
#include <cmath>
#include <cstdint>
#include <cstdlib>
#include <cstring>
#include <map>
#include <string>
#include <vector>

namespace tb {
namespace json {

// ---------------------------------------------------------------- UTF-8

// Length of the UTF-8 sequence at p (strict: no overlongs, no surrogates, <= U+10FFFF),
// or 0 when it is invalid.
inline size_t utf8_len(const uint8_t* p, const uint8_t* end) {
  uint8_t b = p[0];
  if (b < 0x80) return 1;
  auto cont = [&](size_t i) { return p + i < end && (p[i] & 0xC0) == 0x80; };
  if (b >= 0xC2 && b <= 0xDF) return cont(1) ? 2 : 0;
  if (b >= 0xE0 && b <= 0xEF) {
    if (!cont(1) || !cont(2)) return 0;
    if (b == 0xE0 && p[1] < 0xA0) return 0;  // overlong
    if (b == 0xED && p[1] >= 0xA0) return 0;  // surrogate
    return 3;
  }
  if (b >= 0xF0 && b <= 0xF4) {
    if (!cont(1) || !cont(2) || !cont(3)) return 0;
    if (b == 0xF0 && p[1] < 0x90) return 0;
    if (b == 0xF4 && p[1] >= 0x90) return 0;
    return 4;
  }
  return 0;
}

inline bool valid_utf8(const std::string& s) {
  const uint8_t* p = (const uint8_t*)s.data();
  const uint8_t* end = p + s.size();
  while (p < end) {
    size_t n = utf8_len(p, end);
    if (!n) return false;
    p += n;
  }
  return true;
}

// Code point at p of a string this file produced or validated (UTF-8 that may hold
// surrogate code points, which \u escapes can introduce); advances p.
inline uint32_t decode_cp(const uint8_t*& p) {
  uint8_t b = *p++;
  if (b < 0x80) return b;
  if (b < 0xE0) { uint32_t c = (b & 0x1Fu) << 6 | (*p & 0x3Fu); p += 1; return c; }
  if (b < 0xF0) { uint32_t c = (b & 0x0Fu) << 12 | (p[0] & 0x3Fu) << 6 | (p[1] & 0x3Fu); p += 2; return c; }
  uint32_t c = (b & 0x07u) << 18 | (p[0] & 0x3Fu) << 12 | (p[1] & 0x3Fu) << 6 | (p[2] & 0x3Fu);
  p += 3;
  return c;
}

inline void encode_cp(std::string& out, uint32_t c) {
  if (c < 0x80) {
    out += (char)c;
  } else if (c < 0x800) {
    out += (char)(0xC0 | (c >> 6));
    out += (char)(0x80 | (c & 0x3F));
  } else if (c < 0x10000) {
    out += (char)(0xE0 | (c >> 12));
    out += (char)(0x80 | ((c >> 6) & 0x3F));
    out += (char)(0x80 | (c & 0x3F));
  } else {
    out += (char)(0xF0 | (c >> 18));
    out += (char)(0x80 | ((c >> 12) & 0x3F));
    out += (char)(0x80 | ((c >> 6) & 0x3F));
    out += (char)(0x80 | (c & 0x3F));
  }
}

// ---------------------------------------------------------------- JSON

struct Json {
  enum Kind { Null, Bool, Int, Float, String, Array, Object } kind = Null;
  bool flag = false;
  double number = 0.0;
  std::string text;  // Int: decimal digits; String: UTF-8 (surrogates allowed)
  std::vector<Json> items;
  std::map<std::string, Json> members;  // byte order of UTF-8 = code point order
};

// Recursive-descent parser accepting what Python's json.loads accepts (strict mode):
// whitespace " \t\n\r", NaN/Infinity/-Infinity, ASCII-digit numbers, no control
// characters inside strings, \uXXXX escapes with surrogate-pair joining.
class Parser {
 public:
  explicit Parser(const std::string& s) : s_(s) {}

  bool parse(Json& out, std::string& err) {
    skip_ws();
    if (!value(out, 0)) {
      err = err_ + " at char " + std::to_string(pos_);
      return false;
    }
    skip_ws();
    if (pos_ != s_.size()) {
      err = "extra data at char " + std::to_string(pos_);
      return false;
    }
    return true;
  }

 private:
  const std::string& s_;
  size_t pos_ = 0;
  std::string err_;

  bool fail(const char* msg) {
    err_ = msg;
    return false;
  }
  bool at(char c) const { return pos_ < s_.size() && s_[pos_] == c; }
  bool starts(const char* lit) const { return s_.compare(pos_, strlen(lit), lit) == 0; }
  void skip_ws() {
    while (pos_ < s_.size() && (s_[pos_] == ' ' || s_[pos_] == '\t' || s_[pos_] == '\n' || s_[pos_] == '\r')) ++pos_;
  }
  static bool digit(char c) { return c >= '0' && c <= '9'; }

  bool value(Json& v, int depth) {
    if (depth > 512) return fail("nesting too deep");
    if (pos_ >= s_.size()) return fail("expecting value");
    char c = s_[pos_];
    if (c == '{') return object(v, depth);
    if (c == '[') return array(v, depth);
    if (c == '"') {
      v.kind = Json::String;
      return string(v.text);
    }
    if (c == '-' || digit(c)) {
      if (number(v)) return true;
      if (!starts("-Infinity")) return false;
    }
    struct Word { const char* lit; Json::Kind kind; bool flag; double number; };
    static const Word words[] = {{"null", Json::Null, false, 0.0},
                                 {"true", Json::Bool, true, 0.0},
                                 {"false", Json::Bool, false, 0.0},
                                 {"NaN", Json::Float, false, NAN},
                                 {"Infinity", Json::Float, false, INFINITY},
                                 {"-Infinity", Json::Float, false, -INFINITY}};
    for (const Word& w : words) {
      if (starts(w.lit)) {
        pos_ += strlen(w.lit);
        v.kind = w.kind;
        v.flag = w.flag;
        v.number = w.number;
        return true;
      }
    }
    return fail("expecting value");
  }

  // -?(0|[1-9][0-9]*)(\.[0-9]+)?([eE][-+]?[0-9]+)?
  bool number(Json& v) {
    size_t start = pos_, p = pos_;
    if (s_[p] == '-') ++p;
    if (p >= s_.size() || !digit(s_[p])) return fail("expecting value");
    if (s_[p] == '0') ++p;
    else while (p < s_.size() && digit(s_[p])) ++p;
    size_t int_end = p;
    bool is_float = false;
    if (p + 1 < s_.size() && s_[p] == '.' && digit(s_[p + 1])) {
      p += 2;
      while (p < s_.size() && digit(s_[p])) ++p;
      is_float = true;
    }
    if (p < s_.size() && (s_[p] == 'e' || s_[p] == 'E')) {
      size_t q = p + 1;
      if (q < s_.size() && (s_[q] == '+' || s_[q] == '-')) ++q;
      if (q < s_.size() && digit(s_[q])) {
        while (q < s_.size() && digit(s_[q])) ++q;
        p = q;
        is_float = true;
      }
    }
    pos_ = p;
    if (is_float) {
      v.kind = Json::Float;
      std::string lit = s_.substr(start, p - start);
      v.number = strtod(lit.c_str(), nullptr);  // correctly rounded; overflow gives +-inf
      return true;
    }
    v.kind = Json::Int;
    v.text = s_.substr(start, int_end - start);
    if (v.text == "-0") v.text = "0";
    // CPython refuses integer literals above 4300 digits (sys.int_info.default_max_str_digits).
    if (v.text.size() - (v.text[0] == '-') > 4300) return fail("integer literal too long");
    return true;
  }

  bool hex4(size_t p, uint32_t& out) const {
    if (p + 4 > s_.size()) return false;
    out = 0;
    for (size_t i = p; i < p + 4; ++i) {
      char c = s_[i];
      uint32_t d;
      if (c >= '0' && c <= '9') d = (uint32_t)(c - '0');
      else if (c >= 'a' && c <= 'f') d = (uint32_t)(c - 'a' + 10);
      else if (c >= 'A' && c <= 'F') d = (uint32_t)(c - 'A' + 10);
      else return false;
      out = out << 4 | d;
    }
    return true;
  }

  bool string(std::string& out) {
    ++pos_;  // opening quote
    out.clear();
    for (;;) {
      if (pos_ >= s_.size()) return fail("unterminated string");
      uint8_t c = (uint8_t)s_[pos_];
      if (c == '"') {
        ++pos_;
        return true;
      }
      if (c < 0x20) return fail("invalid control character");
      if (c != '\\') {
        out += (char)c;
        ++pos_;
        continue;
      }
      if (pos_ + 1 >= s_.size()) return fail("unterminated string");
      char e = s_[pos_ + 1];
      pos_ += 2;
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
          uint32_t cp;
          if (!hex4(pos_, cp)) return fail("invalid \\uXXXX escape");
          pos_ += 4;
          if (cp >= 0xD800 && cp <= 0xDBFF && pos_ + 6 <= s_.size() && s_[pos_] == '\\' && s_[pos_ + 1] == 'u') {
            uint32_t lo;
            if (!hex4(pos_ + 2, lo)) return fail("invalid \\uXXXX escape");
            if (lo >= 0xDC00 && lo <= 0xDFFF) {
              cp = 0x10000 + ((cp - 0xD800) << 10) + (lo - 0xDC00);
              pos_ += 6;
            }
          }
          encode_cp(out, cp);
          break;
        }
        default:
          return fail("invalid \\escape");
      }
    }
  }

  bool array(Json& v, int depth) {
    v.kind = Json::Array;
    ++pos_;
    skip_ws();
    if (at(']')) {
      ++pos_;
      return true;
    }
    for (;;) {
      v.items.emplace_back();
      if (!value(v.items.back(), depth + 1)) return false;
      skip_ws();
      if (at(']')) {
        ++pos_;
        return true;
      }
      if (!at(',')) return fail("expecting ',' delimiter");
      ++pos_;
      skip_ws();
    }
  }

  bool object(Json& v, int depth) {
    v.kind = Json::Object;
    ++pos_;
    skip_ws();
    if (at('}')) {
      ++pos_;
      return true;
    }
    for (;;) {
      if (!at('"')) return fail("expecting property name enclosed in double quotes");
      std::string name;
      if (!string(name)) return false;
      skip_ws();
      if (!at(':')) return fail("expecting ':' delimiter");
      ++pos_;
      skip_ws();
      Json member;
      if (!value(member, depth + 1)) return false;
      v.members[name] = std::move(member);  // a repeated name keeps the last value
      skip_ws();
      if (at('}')) {
        ++pos_;
        return true;
      }
      if (!at(',')) return fail("expecting ',' delimiter");
      ++pos_;
      skip_ws();
    }
  }
};

// Python's repr(float): the shortest digits that round-trip, positional notation for
// decimal exponents -4 <= e < 16 (with ".0" when there is no fraction), otherwise
// d[.ddd]e+XX with at least two exponent digits.
inline std::string py_float_repr(double v) {
  if (std::isnan(v)) return "NaN";
  if (std::isinf(v)) return v > 0 ? "Infinity" : "-Infinity";
  char buf[64];
  auto res = std::to_chars(buf, buf + sizeof buf, v, std::chars_format::scientific);
  std::string s(buf, res.ptr);
  std::string out;
  if (s[0] == '-') {
    out = "-";
    s.erase(0, 1);
  }
  size_t e = s.find('e');
  std::string digits;
  for (size_t i = 0; i < e; ++i)
    if (s[i] != '.') digits += s[i];
  int decpt = atoi(s.c_str() + e + 1) + 1;  // value = 0.DIGITS * 10^decpt
  if (decpt <= -4 || decpt > 16) {
    out += digits[0];
    if (digits.size() > 1) out += "." + digits.substr(1);
    int x = decpt - 1;
    out += x < 0 ? "e-" : "e+";
    if (std::abs(x) < 10) out += '0';
    out += std::to_string(std::abs(x));
  } else if (decpt <= 0) {
    out += "0." + std::string((size_t)-decpt, '0') + digits;
  } else if ((size_t)decpt >= digits.size()) {
    out += digits + std::string((size_t)decpt - digits.size(), '0') + ".0";
  } else {
    out += digits.substr(0, (size_t)decpt) + "." + digits.substr((size_t)decpt);
  }
  return out;
}

inline void emit_string(std::string& out, const std::string& s) {
  static const char hex[] = "0123456789abcdef";
  auto u4 = [&](uint32_t c) {
    out += "\\u";
    for (int sh = 12; sh >= 0; sh -= 4) out += hex[(c >> sh) & 15];
  };
  out += '"';
  const uint8_t* p = (const uint8_t*)s.data();
  const uint8_t* end = p + s.size();
  while (p < end) {
    uint32_t c = decode_cp(p);
    switch (c) {
      case '"': out += "\\\""; break;
      case '\\': out += "\\\\"; break;
      case '\n': out += "\\n"; break;
      case '\r': out += "\\r"; break;
      case '\t': out += "\\t"; break;
      case '\b': out += "\\b"; break;
      case '\f': out += "\\f"; break;
      default:
        if (c >= 0x20 && c <= 0x7E) {
          out += (char)c;
        } else if (c < 0x10000) {
          u4(c);
        } else {
          c -= 0x10000;
          u4(0xD800 | (c >> 10));
          u4(0xDC00 | (c & 0x3FF));
        }
    }
  }
  out += '"';
}

inline void emit(std::string& out, const Json& v) {
  switch (v.kind) {
    case Json::Null: out += "null"; break;
    case Json::Bool: out += v.flag ? "true" : "false"; break;
    case Json::Int: out += v.text; break;
    case Json::Float: out += py_float_repr(v.number); break;
    case Json::String: emit_string(out, v.text); break;
    case Json::Array: {
      out += '[';
      for (size_t i = 0; i < v.items.size(); ++i) {
        if (i) out += ',';
        emit(out, v.items[i]);
      }
      out += ']';
      break;
    }
    case Json::Object: {
      out += '{';
      bool first = true;
      for (const auto& m : v.members) {
        if (!first) out += ',';
        first = false;
        emit_string(out, m.first);
        out += ':';
        emit(out, m.second);
      }
      out += '}';
      break;
    }
  }
}

inline bool canonical(const std::string& text, std::string& out, std::string& err, Json* parsed = nullptr) {
  if (!valid_utf8(text)) {
    err = "not valid UTF-8";
    return false;
  }
  Json v;
  if (!Parser(text).parse(v, err)) return false;
  out.clear();
  emit(out, v);
  if (parsed) *parsed = std::move(v);
  return true;
}

}  // namespace json
}  // namespace tb
