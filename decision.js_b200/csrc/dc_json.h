// A small JSON reader for manifest.json (objects, arrays, strings, numbers, true/false/null). Enough for the
// reference's export format (scripts/export_common.py:17-61); not a general-purpose parser.
#pragma once
#include <map>
#include <memory>
#include <string>
#include <vector>

namespace dcj {

struct Value {
  enum Kind { Null, Bool, Num, Str, Arr, Obj } kind = Null;
  bool b = false;
  double num = 0;
  std::string str;
  std::vector<Value> arr;
  std::map<std::string, Value> obj;

  const Value *get(const std::string &k) const {
    if (kind != Obj) return nullptr;
    auto it = obj.find(k);
    return it == obj.end() ? nullptr : &it->second;
  }
  bool is_num() const { return kind == Num; }
};

class Parser {
 public:
  explicit Parser(const std::string &s) : s_(s) {}
  bool parse(Value &out, std::string &err) {
    pos_ = 0;
    if (!value(out, err)) return false;
    ws();
    if (pos_ != s_.size()) return fail(err, "trailing characters");
    return true;
  }

 private:
  const std::string &s_;
  size_t pos_ = 0;

  bool fail(std::string &err, const char *what) {
    err = std::string(what) + " at byte " + std::to_string(pos_);
    return false;
  }
  void ws() {
    while (pos_ < s_.size() && (s_[pos_] == ' ' || s_[pos_] == '\n' || s_[pos_] == '\r' || s_[pos_] == '\t')) pos_++;
  }
  bool lit(const char *w) {
    size_t n = 0;
    while (w[n]) n++;
    if (s_.compare(pos_, n, w) != 0) return false;
    pos_ += n;
    return true;
  }
  bool string(std::string &out, std::string &err) {
    if (s_[pos_] != '"') return fail(err, "expected string");
    pos_++;
    out.clear();
    while (pos_ < s_.size() && s_[pos_] != '"') {
      char c = s_[pos_++];
      if (c == '\\') {
        if (pos_ >= s_.size()) return fail(err, "bad escape");
        char e = s_[pos_++];
        switch (e) {
          case 'n': out += '\n'; break;
          case 't': out += '\t'; break;
          case 'r': out += '\r'; break;
          case 'b': out += '\b'; break;
          case 'f': out += '\f'; break;
          case 'u': {
            if (pos_ + 4 > s_.size()) return fail(err, "bad \\u escape");
            unsigned cp = std::stoul(s_.substr(pos_, 4), nullptr, 16);
            pos_ += 4;
            if (cp < 0x80) out += (char)cp;
            else if (cp < 0x800) out += (char)(0xC0 | (cp >> 6)), out += (char)(0x80 | (cp & 63));
            else out += (char)(0xE0 | (cp >> 12)), out += (char)(0x80 | ((cp >> 6) & 63)), out += (char)(0x80 | (cp & 63));
            break;
          }
          default: out += e;
        }
      } else {
        out += c;
      }
    }
    if (pos_ >= s_.size()) return fail(err, "unterminated string");
    pos_++;
    return true;
  }
  bool value(Value &v, std::string &err) {
    ws();
    if (pos_ >= s_.size()) return fail(err, "unexpected end");
    char c = s_[pos_];
    if (c == '{') {
      v.kind = Value::Obj;
      pos_++;
      ws();
      if (s_[pos_] == '}') { pos_++; return true; }
      for (;;) {
        ws();
        std::string k;
        if (!string(k, err)) return false;
        ws();
        if (s_[pos_] != ':') return fail(err, "expected ':'");
        pos_++;
        if (!value(v.obj[k], err)) return false;
        ws();
        if (s_[pos_] == ',') { pos_++; continue; }
        if (s_[pos_] == '}') { pos_++; return true; }
        return fail(err, "expected ',' or '}'");
      }
    }
    if (c == '[') {
      v.kind = Value::Arr;
      pos_++;
      ws();
      if (s_[pos_] == ']') { pos_++; return true; }
      for (;;) {
        v.arr.emplace_back();
        if (!value(v.arr.back(), err)) return false;
        ws();
        if (s_[pos_] == ',') { pos_++; continue; }
        if (s_[pos_] == ']') { pos_++; return true; }
        return fail(err, "expected ',' or ']'");
      }
    }
    if (c == '"') { v.kind = Value::Str; return string(v.str, err); }
    if (lit("true")) { v.kind = Value::Bool; v.b = true; return true; }
    if (lit("false")) { v.kind = Value::Bool; v.b = false; return true; }
    if (lit("null")) { v.kind = Value::Null; return true; }
    if (lit("NaN")) { v.kind = Value::Num; v.num = 0.0 / 0.0; return true; }
    if (lit("Infinity")) { v.kind = Value::Num; v.num = 1.0 / 0.0; return true; }
    if (c == '-' || (c >= '0' && c <= '9')) {
      size_t end = pos_;
      while (end < s_.size() && (std::string("+-.eE0123456789").find(s_[end]) != std::string::npos)) end++;
      v.kind = Value::Num;
      v.num = std::stod(s_.substr(pos_, end - pos_));
      pos_ = end;
      return true;
    }
    return fail(err, "unexpected character");
  }
};

}  // namespace dcj
