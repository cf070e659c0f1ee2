// A small JSON reader for the host side (safetensors headers, tokenizer.json):
// objects keep their key order, numbers are doubles, strings are UTF-8 with
// every escape decoded (\uXXXX including surrogate pairs).
#pragma once

#include <stdint.h>
#include <stdlib.h>
#include <string.h>

#include <string>
#include <utility>
#include <vector>

namespace q3json {

struct Value {
  enum Kind { NUL, NUM, STR, ARR, OBJ, BOOL } kind = NUL;
  double num = 0;
  std::string str;
  std::vector<Value> arr;
  std::vector<std::pair<std::string, Value>> obj;
  const Value *get(const char *k) const {
    for (const auto &kv : obj)
      if (kv.first == k) return &kv.second;
    return nullptr;
  }
};

inline void put_utf8(std::string &out, uint32_t cp) {
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

struct Parser {
  const char *p, *end;
  bool ok = true;
  void ws() { while (p < end && (*p == ' ' || *p == '\n' || *p == '\r' || *p == '\t')) ++p; }
  bool lit(const char *s) {
    const size_t n = strlen(s);
    if (static_cast<size_t>(end - p) >= n && !memcmp(p, s, n)) { p += n; return true; }
    return false;
  }
  bool hex4(uint32_t &v) {
    if (end - p < 4) return false;
    v = 0;
    for (int k = 0; k < 4; ++k) {
      const char c = *p++;
      v <<= 4;
      if (c >= '0' && c <= '9') v |= static_cast<uint32_t>(c - '0');
      else if (c >= 'a' && c <= 'f') v |= static_cast<uint32_t>(c - 'a' + 10);
      else if (c >= 'A' && c <= 'F') v |= static_cast<uint32_t>(c - 'A' + 10);
      else return false;
    }
    return true;
  }
  std::string string() {
    std::string out;
    if (p >= end || *p != '"') { ok = false; return out; }
    ++p;
    while (p < end && *p != '"') {
      if (*p != '\\') { out += *p++; continue; }
      if (++p >= end) break;
      const char c = *p++;
      switch (c) {
        case 'n': out += '\n'; break;
        case 't': out += '\t'; break;
        case 'r': out += '\r'; break;
        case 'b': out += '\b'; break;
        case 'f': out += '\f'; break;
        case 'u': {
          uint32_t cp;
          if (!hex4(cp)) { ok = false; return out; }
          if (cp >= 0xD800 && cp < 0xDC00 && end - p >= 6 && p[0] == '\\' && p[1] == 'u') {
            const char *save = p;
            p += 2;
            uint32_t lo;
            if (hex4(lo) && lo >= 0xDC00 && lo < 0xE000) cp = 0x10000 + ((cp - 0xD800) << 10) + (lo - 0xDC00);
            else p = save;
          }
          put_utf8(out, cp);
          break;
        }
        default: out += c;   // \" \\ \/
      }
    }
    if (p >= end) { ok = false; return out; }
    ++p;
    return out;
  }
  Value value(int depth = 0) {
    Value v;
    ws();
    if (p >= end || depth > 32) { ok = false; return v; }
    if (*p == '{') {
      v.kind = Value::OBJ;
      ++p;
      ws();
      if (p < end && *p == '}') { ++p; return v; }
      while (ok) {
        ws();
        std::string k = string();
        ws();
        if (p >= end || *p != ':') { ok = false; break; }
        ++p;
        v.obj.emplace_back(std::move(k), value(depth + 1));
        ws();
        if (p < end && *p == ',') { ++p; continue; }
        if (p < end && *p == '}') { ++p; break; }
        ok = false;
      }
    } else if (*p == '[') {
      v.kind = Value::ARR;
      ++p;
      ws();
      if (p < end && *p == ']') { ++p; return v; }
      while (ok) {
        v.arr.push_back(value(depth + 1));
        ws();
        if (p < end && *p == ',') { ++p; continue; }
        if (p < end && *p == ']') { ++p; break; }
        ok = false;
      }
    } else if (*p == '"') {
      v.kind = Value::STR;
      v.str = string();
    } else if (lit("true") || lit("false")) {
      v.kind = Value::BOOL;
    } else if (lit("null")) {
      v.kind = Value::NUL;
    } else {
      char *e = nullptr;
      v.num = strtod(p, &e);
      if (e == p) ok = false;
      else { v.kind = Value::NUM; p = e; }
    }
    return v;
  }
};

}  // namespace q3json
