// Minimal JSON reader shared by the library's host-side parsers (tokenizer,
// safetensors header).  Host code only.
//
// Objects keep their member order; a repeated member name is an error (the
// default of the std.json parser the reference's readers use).  Strings are
// validated UTF-8 with \u escapes (surrogate pairs joined); numbers are
// integers when written without fraction or exponent and within int64,
// else doubles.  Nesting is limited to 256 levels.
#pragma once

#include <cerrno>
#include <cstdint>
#include <cstdlib>
#include <cstring>
#include <string>
#include <string_view>
#include <unordered_set>
#include <utility>
#include <vector>

namespace nnz_json {

constexpr int kMaxJsonDepth = 256;

inline void utf8_append(std::string& s, uint32_t cp) {
  if (cp < 0x80) {
    s += (char)cp;
  } else if (cp < 0x800) {
    s += (char)(0xC0 | (cp >> 6));
    s += (char)(0x80 | (cp & 0x3F));
  } else if (cp < 0x10000) {
    s += (char)(0xE0 | (cp >> 12));
    s += (char)(0x80 | ((cp >> 6) & 0x3F));
    s += (char)(0x80 | (cp & 0x3F));
  } else {
    s += (char)(0xF0 | (cp >> 18));
    s += (char)(0x80 | ((cp >> 12) & 0x3F));
    s += (char)(0x80 | ((cp >> 6) & 0x3F));
    s += (char)(0x80 | (cp & 0x3F));
  }
}

struct JVal {
  enum Kind { NUL, BOOL, INT, DBL, STR, ARR, OBJ } kind = NUL;
  bool b = false;
  int64_t i = 0;
  double d = 0;
  std::string s;
  std::vector<JVal> arr;
  std::vector<std::pair<std::string, JVal>> obj;

  const JVal* get(std::string_view key) const {
    const JVal* hit = nullptr;
    for (const auto& kv : obj)
      if (kv.first == key) hit = &kv.second;
    return hit;
  }
};

class JsonReader {
 public:
  JsonReader(const char* p, size_t n) : p_(p), end_(p + n) {}

  bool parse(JVal& out, std::string& err) {
    ws();
    if (!value(out, 0)) {
      err = err_;
      return false;
    }
    ws();
    if (p_ != end_) {
      err = "trailing characters after the JSON value";
      return false;
    }
    return true;
  }

 private:
  const char* p_;
  const char* end_;
  std::string err_;

  bool bad(const char* m) {
    if (err_.empty()) err_ = m;
    return false;
  }
  void ws() {
    while (p_ < end_ && (*p_ == ' ' || *p_ == '\t' || *p_ == '\n' || *p_ == '\r')) ++p_;
  }
  bool lit(const char* w) {
    const size_t n = strlen(w);
    if ((size_t)(end_ - p_) < n || memcmp(p_, w, n) != 0) return bad("invalid literal");
    p_ += n;
    return true;
  }
  bool value(JVal& v, int depth) {
    if (depth > kMaxJsonDepth) return bad("nesting too deep");
    if (p_ >= end_) return bad("unexpected end of input");
    switch (*p_) {
      case '{': return object(v, depth);
      case '[': return array(v, depth);
      case '"': v.kind = JVal::STR; return string(v.s);
      case 't': v.kind = JVal::BOOL; v.b = true; return lit("true");
      case 'f': v.kind = JVal::BOOL; v.b = false; return lit("false");
      case 'n': v.kind = JVal::NUL; return lit("null");
      default: return number(v);
    }
  }
  bool object(JVal& v, int depth) {
    v.kind = JVal::OBJ;
    ++p_;
    ws();
    if (p_ < end_ && *p_ == '}') { ++p_; return true; }
    for (;;) {
      ws();
      if (p_ >= end_ || *p_ != '"') return bad("expected a member name");
      std::string key;
      if (!string(key)) return false;
      ws();
      if (p_ >= end_ || *p_ != ':') return bad("expected ':'");
      ++p_;
      ws();
      v.obj.emplace_back(std::move(key), JVal{});
      if (!value(v.obj.back().second, depth + 1)) return false;
      ws();
      if (p_ < end_ && *p_ == ',') { ++p_; continue; }
      if (p_ < end_ && *p_ == '}') { ++p_; return unique_members(v); }
      return bad("expected ',' or '}'");
    }
  }
  // A repeated member name is an error, as in the reference's JSON parser
  // (its default duplicate-field behaviour).
  bool unique_members(const JVal& v) {
    const size_t n = v.obj.size();
    if (n < 16) {
      for (size_t i = 1; i < n; ++i)
        for (size_t j = 0; j < i; ++j)
          if (v.obj[i].first == v.obj[j].first) return bad("duplicate member name");
      return true;
    }
    std::unordered_set<std::string_view> seen;
    seen.reserve(2 * n);
    for (const auto& kv : v.obj)
      if (!seen.insert(kv.first).second) return bad("duplicate member name");
    return true;
  }
  bool array(JVal& v, int depth) {
    v.kind = JVal::ARR;
    ++p_;
    ws();
    if (p_ < end_ && *p_ == ']') { ++p_; return true; }
    for (;;) {
      ws();
      v.arr.emplace_back();
      if (!value(v.arr.back(), depth + 1)) return false;
      ws();
      if (p_ < end_ && *p_ == ',') { ++p_; continue; }
      if (p_ < end_ && *p_ == ']') { ++p_; return true; }
      return bad("expected ',' or ']'");
    }
  }
  bool hex4(uint32_t& u) {
    if (end_ - p_ < 4) return bad("short \\u escape");
    u = 0;
    for (int k = 0; k < 4; ++k) {
      const char c = *p_++;
      u <<= 4;
      if (c >= '0' && c <= '9') u |= (uint32_t)(c - '0');
      else if (c >= 'a' && c <= 'f') u |= (uint32_t)(c - 'a' + 10);
      else if (c >= 'A' && c <= 'F') u |= (uint32_t)(c - 'A' + 10);
      else return bad("bad \\u escape");
    }
    return true;
  }
  bool string(std::string& s) {
    ++p_;   // opening quote
    for (;;) {
      if (p_ >= end_) return bad("unterminated string");
      const unsigned char c = (unsigned char)*p_;
      if (c == '"') { ++p_; return true; }
      if (c < 0x20) return bad("control character in string");
      if (c == '\\') {
        ++p_;
        if (p_ >= end_) return bad("unterminated escape");
        const char e = *p_++;
        switch (e) {
          case '"': s += '"'; break;
          case '\\': s += '\\'; break;
          case '/': s += '/'; break;
          case 'b': s += '\b'; break;
          case 'f': s += '\f'; break;
          case 'n': s += '\n'; break;
          case 'r': s += '\r'; break;
          case 't': s += '\t'; break;
          case 'u': {
            uint32_t u;
            if (!hex4(u)) return false;
            if (u >= 0xD800 && u < 0xDC00) {
              uint32_t lo;
              if (end_ - p_ < 2 || p_[0] != '\\' || p_[1] != 'u') return bad("lone high surrogate");
              p_ += 2;
              if (!hex4(lo)) return false;
              if (lo < 0xDC00 || lo >= 0xE000) return bad("bad low surrogate");
              u = 0x10000 + ((u - 0xD800) << 10) + (lo - 0xDC00);
            } else if (u >= 0xDC00 && u < 0xE000) {
              return bad("lone low surrogate");
            }
            utf8_append(s, u);
            break;
          }
          default: return bad("bad escape");
        }
        continue;
      }
      // raw UTF-8: validate the sequence
      int n = c < 0x80 ? 1 : (c >> 5) == 6 ? 2 : (c >> 4) == 14 ? 3 : (c >> 3) == 30 ? 4 : 0;
      if (n == 0 || end_ - p_ < n) return bad("invalid UTF-8 in string");
      uint32_t cp = n == 1 ? c : n == 2 ? (c & 0x1F) : n == 3 ? (c & 0x0F) : (c & 0x07);
      for (int k = 1; k < n; ++k) {
        const unsigned char cc = (unsigned char)p_[k];
        if ((cc & 0xC0) != 0x80) return bad("invalid UTF-8 in string");
        cp = (cp << 6) | (cc & 0x3F);
      }
      static const uint32_t kMin[5] = {0, 0, 0x80, 0x800, 0x10000};
      if (cp < kMin[n] || cp > 0x10FFFF || (cp >= 0xD800 && cp < 0xE000)) return bad("invalid UTF-8 in string");
      s.append(p_, (size_t)n);
      p_ += n;
    }
  }
  bool number(JVal& v) {
    const char* s = p_;
    if (p_ < end_ && *p_ == '-') ++p_;
    if (p_ >= end_ || *p_ < '0' || *p_ > '9') return bad("invalid value");
    if (*p_ == '0') {
      ++p_;
    } else {
      while (p_ < end_ && *p_ >= '0' && *p_ <= '9') ++p_;
    }
    bool is_int = true;
    if (p_ < end_ && *p_ == '.') {
      is_int = false;
      ++p_;
      if (p_ >= end_ || *p_ < '0' || *p_ > '9') return bad("invalid number");
      while (p_ < end_ && *p_ >= '0' && *p_ <= '9') ++p_;
    }
    if (p_ < end_ && (*p_ == 'e' || *p_ == 'E')) {
      is_int = false;
      ++p_;
      if (p_ < end_ && (*p_ == '+' || *p_ == '-')) ++p_;
      if (p_ >= end_ || *p_ < '0' || *p_ > '9') return bad("invalid number");
      while (p_ < end_ && *p_ >= '0' && *p_ <= '9') ++p_;
    }
    const std::string text(s, p_);
    if (is_int) {
      errno = 0;
      char* e = nullptr;
      const long long x = strtoll(text.c_str(), &e, 10);
      if (errno == 0) {
        v.kind = JVal::INT;
        v.i = x;
        return true;
      }
    }
    v.kind = JVal::DBL;
    v.d = strtod(text.c_str(), nullptr);
    return true;
  }
};

}  // namespace nnz_json
