// Minimal JSON reader for model specs and open options (objects, arrays,
// numbers, strings, booleans, null).  Throws std::runtime_error on bad input.
#pragma once

#include <cstdlib>
#include <map>
#include <memory>
#include <stdexcept>
#include <string>
#include <vector>

namespace vd {

struct Json {
  enum Kind { Null, Bool, Number, String, Array, Object } kind = Null;
  bool b = false;
  double num = 0.0;
  std::string str;
  std::vector<Json> arr;
  std::map<std::string, Json> obj;

  bool has(const std::string& k) const { return kind == Object && obj.count(k) != 0; }
  const Json& at(const std::string& k) const {
    auto it = obj.find(k);
    if (kind != Object || it == obj.end()) throw std::runtime_error("missing key \"" + k + "\"");
    return it->second;
  }
  double number(const std::string& k) const {
    const Json& v = at(k);
    if (v.kind != Number) throw std::runtime_error("key \"" + k + "\" is not a number");
    return v.num;
  }
  double number_or(const std::string& k, double dflt) const { return has(k) && at(k).kind == Number ? at(k).num : dflt; }
  long long integer(const std::string& k) const { return static_cast<long long>(number(k)); }
  long long integer_or(const std::string& k, long long dflt) const {
    return has(k) && at(k).kind == Number ? static_cast<long long>(at(k).num) : dflt;
  }
  bool boolean_or(const std::string& k, bool dflt) const {
    if (!has(k)) return dflt;
    const Json& v = at(k);
    if (v.kind == Bool) return v.b;
    if (v.kind == Number) return v.num != 0.0;
    return dflt;
  }
  std::string string_or(const std::string& k, const std::string& dflt) const {
    return has(k) && at(k).kind == String ? at(k).str : dflt;
  }
};

class JsonParser {
 public:
  explicit JsonParser(const std::string& s) : s_(s) {}
  Json parse() {
    Json v = value();
    ws();
    if (i_ != s_.size()) fail("trailing characters");
    return v;
  }

 private:
  const std::string& s_;
  size_t i_ = 0;

  [[noreturn]] void fail(const char* what) {
    throw std::runtime_error(std::string("JSON: ") + what + " at offset " + std::to_string(i_));
  }
  void ws() {
    while (i_ < s_.size() && (s_[i_] == ' ' || s_[i_] == '\n' || s_[i_] == '\t' || s_[i_] == '\r')) ++i_;
  }
  bool lit(const char* w) {
    size_t n = std::char_traits<char>::length(w);
    if (s_.compare(i_, n, w) == 0) {
      i_ += n;
      return true;
    }
    return false;
  }
  Json value() {
    ws();
    if (i_ >= s_.size()) fail("unexpected end");
    Json v;
    char c = s_[i_];
    if (c == '{') {
      v.kind = Json::Object;
      ++i_;
      ws();
      if (i_ < s_.size() && s_[i_] == '}') {
        ++i_;
        return v;
      }
      while (true) {
        ws();
        if (i_ >= s_.size() || s_[i_] != '"') fail("expected key");
        std::string k = string();
        ws();
        if (i_ >= s_.size() || s_[i_] != ':') fail("expected ':'");
        ++i_;
        v.obj[k] = value();
        ws();
        if (i_ < s_.size() && s_[i_] == ',') {
          ++i_;
          continue;
        }
        if (i_ < s_.size() && s_[i_] == '}') {
          ++i_;
          return v;
        }
        fail("expected ',' or '}'");
      }
    }
    if (c == '[') {
      v.kind = Json::Array;
      ++i_;
      ws();
      if (i_ < s_.size() && s_[i_] == ']') {
        ++i_;
        return v;
      }
      while (true) {
        v.arr.push_back(value());
        ws();
        if (i_ < s_.size() && s_[i_] == ',') {
          ++i_;
          continue;
        }
        if (i_ < s_.size() && s_[i_] == ']') {
          ++i_;
          return v;
        }
        fail("expected ',' or ']'");
      }
    }
    if (c == '"') {
      v.kind = Json::String;
      v.str = string();
      return v;
    }
    if (lit("true")) {
      v.kind = Json::Bool;
      v.b = true;
      return v;
    }
    if (lit("false")) {
      v.kind = Json::Bool;
      return v;
    }
    if (lit("null")) return v;
    if (lit("NaN")) fail("NaN is not supported");
    const char* begin = s_.c_str() + i_;
    char* end = nullptr;
    v.num = std::strtod(begin, &end);
    if (end == begin) fail("bad value");
    v.kind = Json::Number;
    i_ += static_cast<size_t>(end - begin);
    return v;
  }
  std::string string() {
    ++i_;  // opening quote
    std::string out;
    while (i_ < s_.size() && s_[i_] != '"') {
      char c = s_[i_++];
      if (c == '\\') {
        if (i_ >= s_.size()) fail("bad escape");
        char e = s_[i_++];
        switch (e) {
          case 'n': out += '\n'; break;
          case 't': out += '\t'; break;
          case 'r': out += '\r'; break;
          case 'b': out += '\b'; break;
          case 'f': out += '\f'; break;
          case 'u': {
            if (i_ + 4 > s_.size()) fail("bad \\u escape");
            unsigned cp = static_cast<unsigned>(std::strtoul(s_.substr(i_, 4).c_str(), nullptr, 16));
            i_ += 4;
            if (cp < 0x80) {
              out += static_cast<char>(cp);
            } else if (cp < 0x800) {
              out += static_cast<char>(0xC0 | (cp >> 6));
              out += static_cast<char>(0x80 | (cp & 0x3F));
            } else {
              out += static_cast<char>(0xE0 | (cp >> 12));
              out += static_cast<char>(0x80 | ((cp >> 6) & 0x3F));
              out += static_cast<char>(0x80 | (cp & 0x3F));
            }
            break;
          }
          default: out += e;
        }
      } else {
        out += c;
      }
    }
    if (i_ >= s_.size()) fail("unterminated string");
    ++i_;
    return out;
  }
};

inline Json parse_json(const std::string& s) { return JsonParser(s).parse(); }

}  // namespace vd
