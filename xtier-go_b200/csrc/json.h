// A small JSON reader for the options string of xtg_cuda_open (objects, arrays, numbers, strings, booleans, null).
#pragma once

#include <cstdlib>
#include <map>
#include <memory>
#include <stdexcept>
#include <string>
#include <vector>

namespace xtg {

struct Json {
  enum Kind { Null, Bool, Number, String, Array, Object } kind = Null;
  bool b = false;
  double num = 0;
  std::string str;
  std::vector<Json> arr;
  std::map<std::string, Json> obj;

  bool has(const std::string& k) const { return kind == Object && obj.count(k) && obj.at(k).kind != Null; }
  const Json& at(const std::string& k) const {
    static const Json none;
    if (kind != Object) return none;
    auto it = obj.find(k);
    return it == obj.end() ? none : it->second;
  }
  double number(const std::string& k, double def) const {
    const Json& v = at(k);
    if (v.kind == Null) return def;
    if (v.kind == Number) return v.num;
    if (v.kind == Bool) return v.b ? 1 : 0;
    if (v.kind == String) {
      char* end = nullptr;
      const double d = std::strtod(v.str.c_str(), &end);
      if (end && *end == 0 && !v.str.empty()) return d;
    }
    throw std::runtime_error("option " + k + ": not a number");
  }
  std::string string(const std::string& k, const std::string& def) const {
    const Json& v = at(k);
    if (v.kind == Null) return def;
    if (v.kind != String) throw std::runtime_error("option " + k + ": not a string");
    return v.str;
  }

  static Json parse(const std::string& text) {
    size_t i = 0;
    Json j = value(text, i);
    ws(text, i);
    if (i != text.size()) throw std::runtime_error("options: trailing characters in JSON");
    return j;
  }

 private:
  static void ws(const std::string& s, size_t& i) {
    while (i < s.size() && (s[i] == ' ' || s[i] == '\n' || s[i] == '\t' || s[i] == '\r')) ++i;
  }
  static Json value(const std::string& s, size_t& i) {
    ws(s, i);
    if (i >= s.size()) throw std::runtime_error("options: unexpected end of JSON");
    Json j;
    const char c = s[i];
    if (c == '{') {
      j.kind = Object;
      ++i;
      ws(s, i);
      if (i < s.size() && s[i] == '}') {
        ++i;
        return j;
      }
      while (true) {
        ws(s, i);
        Json key = value(s, i);
        if (key.kind != String) throw std::runtime_error("options: object key is not a string");
        ws(s, i);
        if (i >= s.size() || s[i] != ':') throw std::runtime_error("options: ':' expected");
        ++i;
        j.obj[key.str] = value(s, i);
        ws(s, i);
        if (i < s.size() && s[i] == ',') {
          ++i;
          continue;
        }
        if (i < s.size() && s[i] == '}') {
          ++i;
          return j;
        }
        throw std::runtime_error("options: ',' or '}' expected");
      }
    }
    if (c == '[') {
      j.kind = Array;
      ++i;
      ws(s, i);
      if (i < s.size() && s[i] == ']') {
        ++i;
        return j;
      }
      while (true) {
        j.arr.push_back(value(s, i));
        ws(s, i);
        if (i < s.size() && s[i] == ',') {
          ++i;
          continue;
        }
        if (i < s.size() && s[i] == ']') {
          ++i;
          return j;
        }
        throw std::runtime_error("options: ',' or ']' expected");
      }
    }
    if (c == '"') {
      j.kind = String;
      ++i;
      while (i < s.size() && s[i] != '"') {
        if (s[i] == '\\' && i + 1 < s.size()) {
          ++i;
          const char e = s[i];
          j.str += e == 'n' ? '\n' : e == 't' ? '\t' : e;
        } else {
          j.str += s[i];
        }
        ++i;
      }
      if (i >= s.size()) throw std::runtime_error("options: unterminated string");
      ++i;
      return j;
    }
    if (s.compare(i, 4, "true") == 0) {
      j.kind = Bool;
      j.b = true;
      i += 4;
      return j;
    }
    if (s.compare(i, 5, "false") == 0) {
      j.kind = Bool;
      i += 5;
      return j;
    }
    if (s.compare(i, 4, "null") == 0) {
      i += 4;
      return j;
    }
    char* end = nullptr;
    j.num = std::strtod(s.c_str() + i, &end);
    if (end == s.c_str() + i) throw std::runtime_error("options: bad JSON value");
    j.kind = Number;
    i = size_t(end - s.c_str());
    return j;
  }
};

}  // namespace xtg
