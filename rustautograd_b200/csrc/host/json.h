// Minimal JSON value for structured diagnostics and reports.
//
// rg reports every failure as a JSON object (graph.rs:203-212 `diag`) and its compile report is
// JSON too (validate.rs:854-872). This value type builds those objects and prints them compactly;
// Python parses the text with `json.loads`, exactly as the reference's PyO3 layer does
// (python.rs:14-22).
#pragma once
#include <cmath>
#include <cstdint>
#include <cstdio>
#include <cstdlib>
#include <map>
#include <memory>
#include <string>
#include <utility>
#include <vector>

namespace rg {

class Json {
 public:
  enum class Kind { Null, Bool, Int, Num, Str, Arr, Obj };

  Json() : kind_(Kind::Null) {}
  Json(std::nullptr_t) : kind_(Kind::Null) {}
  Json(bool b) : kind_(Kind::Bool), b_(b) {}
  Json(int v) : kind_(Kind::Int), i_(v) {}
  Json(long v) : kind_(Kind::Int), i_(v) {}
  Json(long long v) : kind_(Kind::Int), i_(v) {}
  Json(unsigned v) : kind_(Kind::Int), i_(v) {}
  Json(unsigned long v) : kind_(Kind::Int), i_((long long)v) {}
  Json(unsigned long long v) : kind_(Kind::Int), i_((long long)v) {}
  Json(double v) : kind_(Kind::Num), d_(v) {}
  Json(const char* s) : kind_(Kind::Str), s_(s) {}
  Json(std::string s) : kind_(Kind::Str), s_(std::move(s)) {}
  template <typename T>
  Json(const std::vector<T>& v) : kind_(Kind::Arr) {
    for (const auto& x : v) arr_.push_back(Json(x));
  }

  static Json array() {
    Json j;
    j.kind_ = Kind::Arr;
    return j;
  }
  static Json object() {
    Json j;
    j.kind_ = Kind::Obj;
    return j;
  }

  Kind kind() const { return kind_; }
  bool is_null() const { return kind_ == Kind::Null; }
  bool is_str() const { return kind_ == Kind::Str; }
  bool is_arr() const { return kind_ == Kind::Arr; }
  bool is_obj() const { return kind_ == Kind::Obj; }
  const std::string& str() const { return s_; }
  double num() const { return kind_ == Kind::Int ? (double)i_ : d_; }
  bool boolean() const { return b_; }

  // Object access; creates the key (and turns null into an object) like serde_json's IndexMut.
  Json& operator[](const std::string& k) {
    if (kind_ == Kind::Null) kind_ = Kind::Obj;
    for (auto& kv : obj_)
      if (kv.first == k) return kv.second;
    obj_.emplace_back(k, Json());
    return obj_.back().second;
  }
  const Json* get(const std::string& k) const {
    for (auto& kv : obj_)
      if (kv.first == k) return &kv.second;
    return nullptr;
  }
  std::vector<Json>& items() { return arr_; }
  const std::vector<Json>& items() const { return arr_; }
  void push(Json v) {
    if (kind_ == Kind::Null) kind_ = Kind::Arr;
    arr_.push_back(std::move(v));
  }
  size_t size() const { return kind_ == Kind::Arr ? arr_.size() : obj_.size(); }

  bool operator==(const char* s) const { return kind_ == Kind::Str && s_ == s; }

  std::string dump() const {
    std::string out;
    write(out);
    return out;
  }

 private:
  static void esc(std::string& out, const std::string& s) {
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
            snprintf(b, sizeof b, "\\u%04x", c);
            out += b;
          } else {
            out += (char)c;
          }
      }
    }
    out += '"';
  }
  void write(std::string& out) const {
    switch (kind_) {
      case Kind::Null: out += "null"; break;
      case Kind::Bool: out += b_ ? "true" : "false"; break;
      case Kind::Int: out += std::to_string(i_); break;
      case Kind::Num: {
        if (!std::isfinite(d_)) {
          out += "null";  // JSON has no Inf/NaN; callers encode those as strings first.
        } else {
          char b[40];
          snprintf(b, sizeof b, "%.17g", d_);
          std::string t = b;
          // Shortest round-trip form, so 0.1 prints as 0.1 like serde_json does.
          for (int p = 1; p <= 17; ++p) {
            snprintf(b, sizeof b, "%.*g", p, d_);
            if (strtod(b, nullptr) == d_) {
              t = b;
              break;
            }
          }
          if (t.find_first_of(".eEn") == std::string::npos) t += ".0";
          out += t;
        }
        break;
      }
      case Kind::Str: esc(out, s_); break;
      case Kind::Arr: {
        out += '[';
        for (size_t i = 0; i < arr_.size(); ++i) {
          if (i) out += ',';
          arr_[i].write(out);
        }
        out += ']';
        break;
      }
      case Kind::Obj: {
        out += '{';
        for (size_t i = 0; i < obj_.size(); ++i) {
          if (i) out += ',';
          esc(out, obj_[i].first);
          out += ':';
          obj_[i].second.write(out);
        }
        out += '}';
        break;
      }
    }
  }

  Kind kind_;
  bool b_ = false;
  long long i_ = 0;
  double d_ = 0;
  std::string s_;
  std::vector<Json> arr_;
  std::vector<std::pair<std::string, Json>> obj_;
};

// JSON cannot carry Inf/NaN as numbers (validate.rs:28-38 `num`).
inline Json jnum(double x) {
  if (std::isfinite(x)) return Json(x);
  if (std::isnan(x)) return Json("nan");
  return Json(x > 0 ? "inf" : "-inf");
}

}  // namespace rg
