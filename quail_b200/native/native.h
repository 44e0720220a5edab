// Shared declarations of the C++ host runtime (module quail_b200._native).
#pragma once

#include <cstdint>
#include <map>
#include <memory>
#include <stdexcept>
#include <string>
#include <utility>
#include <vector>

namespace qbn {

// A minimal ordered JSON value used to hand trees and plans to Python.
class Json {
 public:
  enum class Kind { Null, Bool, Int, Float, String, Array, Object };
  Json() : kind_(Kind::Null) {}
  Json(bool b) : kind_(Kind::Bool), b_(b) {}                      // NOLINT
  Json(int i) : kind_(Kind::Int), i_(i) {}                        // NOLINT
  Json(long long i) : kind_(Kind::Int), i_(i) {}                  // NOLINT
  Json(double d) : kind_(Kind::Float), d_(d) {}                   // NOLINT
  Json(const char* s) : kind_(Kind::String), s_(s) {}             // NOLINT
  Json(std::string s) : kind_(Kind::String), s_(std::move(s)) {}  // NOLINT
  static Json array() {
    Json j;
    j.kind_ = Kind::Array;
    return j;
  }
  static Json object() {
    Json j;
    j.kind_ = Kind::Object;
    return j;
  }
  void push(Json v) { arr_.push_back(std::move(v)); }
  void set(const std::string& k, Json v) {
    for (auto& kv : obj_)
      if (kv.first == k) {
        kv.second = std::move(v);
        return;
      }
    obj_.emplace_back(k, std::move(v));
  }
  size_t size() const { return kind_ == Kind::Array ? arr_.size() : obj_.size(); }
  std::string dump() const;

 private:
  Kind kind_;
  bool b_ = false;
  long long i_ = 0;
  double d_ = 0;
  std::string s_;
  std::vector<Json> arr_;
  std::vector<std::pair<std::string, Json>> obj_;
};

std::string json_escape(const std::string& s);

struct SqlError : std::runtime_error {
  size_t pos;
  SqlError(const std::string& m, size_t p) : std::runtime_error(m), pos(p) {}
};

// SQL text -> JSON syntax tree (throws SqlError)
std::string parse_sql(const std::string& text);

}  // namespace qbn
