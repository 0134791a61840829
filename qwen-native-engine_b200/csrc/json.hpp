// Minimal JSON reader for index.json and tile profiles (objects, arrays, strings, numbers,
// booleans, null). Throws JsonError with the byte offset on malformed input.
#pragma once

#include <cstdint>
#include <cstdlib>
#include <map>
#include <memory>
#include <stdexcept>
#include <string>
#include <vector>

namespace qne {

struct JsonError : std::runtime_error {
  using std::runtime_error::runtime_error;
};

struct Json {
  enum Type { Null, Bool, Number, String, Array, Object } type = Null;
  bool b = false;
  double num = 0;
  std::string str;
  std::vector<Json> arr;
  std::map<std::string, Json> obj;

  const Json* get(const std::string& key) const {
    if (type != Object) return nullptr;
    auto it = obj.find(key);
    return it == obj.end() ? nullptr : &it->second;
  }
  bool is_number() const { return type == Number; }

  static Json parse(const char* text, size_t n) {
    Parser p{text, n, 0};
    p.ws();
    Json v = p.value(0);
    p.ws();
    if (p.i != n) p.fail("trailing characters");
    return v;
  }

 private:
  struct Parser {
    const char* s;
    size_t n;
    size_t i;
    [[noreturn]] void fail(const char* what) {
      throw JsonError(std::string("index.json: ") + what + " at byte " + std::to_string(i));
    }
    void ws() {
      while (i < n && (s[i] == ' ' || s[i] == '\n' || s[i] == '\r' || s[i] == '\t')) ++i;
    }
    bool lit(const char* w) {
      size_t k = 0;
      while (w[k]) {
        if (i + k >= n || s[i + k] != w[k]) return false;
        ++k;
      }
      i += k;
      return true;
    }
    Json value(int depth) {
      if (depth > 64) fail("nesting too deep");
      if (i >= n) fail("unexpected end");
      Json v;
      const char c = s[i];
      if (c == '{') {
        v.type = Object;
        ++i;
        ws();
        if (i < n && s[i] == '}') { ++i; return v; }
        for (;;) {
          ws();
          if (i >= n || s[i] != '"') fail("expected a key");
          std::string key = string();
          ws();
          if (i >= n || s[i] != ':') fail("expected ':'");
          ++i;
          ws();
          v.obj[key] = value(depth + 1);
          ws();
          if (i < n && s[i] == ',') { ++i; continue; }
          if (i < n && s[i] == '}') { ++i; return v; }
          fail("expected ',' or '}'");
        }
      }
      if (c == '[') {
        v.type = Array;
        ++i;
        ws();
        if (i < n && s[i] == ']') { ++i; return v; }
        for (;;) {
          ws();
          v.arr.push_back(value(depth + 1));
          ws();
          if (i < n && s[i] == ',') { ++i; continue; }
          if (i < n && s[i] == ']') { ++i; return v; }
          fail("expected ',' or ']'");
        }
      }
      if (c == '"') {
        v.type = String;
        v.str = string();
        return v;
      }
      if (lit("true")) { v.type = Bool; v.b = true; return v; }
      if (lit("false")) { v.type = Bool; v.b = false; return v; }
      if (lit("null")) return v;
      // number
      size_t st = i;
      if (i < n && (s[i] == '-' || s[i] == '+')) ++i;
      while (i < n && ((s[i] >= '0' && s[i] <= '9') || s[i] == '.' || s[i] == 'e' || s[i] == 'E' ||
                       s[i] == '-' || s[i] == '+'))
        ++i;
      if (i == st) fail("unexpected character");
      std::string t(s + st, i - st);
      char* end = nullptr;
      v.num = std::strtod(t.c_str(), &end);
      if (!end || *end) fail("malformed number");
      v.type = Number;
      return v;
    }
    static void utf8(std::string& out, uint32_t cp) {
      if (cp < 0x80) out += (char)cp;
      else if (cp < 0x800) { out += (char)(0xC0 | (cp >> 6)); out += (char)(0x80 | (cp & 63)); }
      else if (cp < 0x10000) {
        out += (char)(0xE0 | (cp >> 12)); out += (char)(0x80 | ((cp >> 6) & 63)); out += (char)(0x80 | (cp & 63));
      } else {
        out += (char)(0xF0 | (cp >> 18)); out += (char)(0x80 | ((cp >> 12) & 63));
        out += (char)(0x80 | ((cp >> 6) & 63)); out += (char)(0x80 | (cp & 63));
      }
    }
    uint32_t hex4() {
      if (i + 4 > n) fail("short \\u escape");
      uint32_t v = 0;
      for (int k = 0; k < 4; ++k) {
        const char h = s[i++];
        v <<= 4;
        if (h >= '0' && h <= '9') v |= (uint32_t)(h - '0');
        else if (h >= 'a' && h <= 'f') v |= (uint32_t)(h - 'a' + 10);
        else if (h >= 'A' && h <= 'F') v |= (uint32_t)(h - 'A' + 10);
        else fail("bad \\u escape");
      }
      return v;
    }
    std::string string() {
      ++i;  // opening quote
      std::string out;
      while (i < n && s[i] != '"') {
        char c = s[i++];
        if ((unsigned char)c < 0x20) fail("control character in string");
        if (c != '\\') { out += c; continue; }
        if (i >= n) fail("unterminated escape");
        c = s[i++];
        switch (c) {
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
            if (cp >= 0xD800 && cp < 0xDC00 && i + 1 < n && s[i] == '\\' && s[i + 1] == 'u') {
              i += 2;
              const uint32_t lo = hex4();
              cp = 0x10000 + ((cp - 0xD800) << 10) + (lo - 0xDC00);
            }
            utf8(out, cp);
            break;
          }
          default: fail("unknown escape");
        }
      }
      if (i >= n) fail("unterminated string");
      ++i;
      return out;
    }
  };
};

}  // namespace qne
