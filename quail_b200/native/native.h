// Shared declarations of the C++ host runtime (module quail_b200._native).
#pragma once

#include <cstdint>
#include <map>
#include <memory>
#include <stdexcept>
#include <mutex>
#include <string>
#include <unordered_map>
#include <unordered_set>
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

// Byte-level BPE (HF tokenizer.json, GPT-2 / Qwen2 pre-tokenizer): tokenizer.cpp.
class BpeTokenizer {
 public:
  BpeTokenizer(const std::unordered_map<std::string, int>& vocab,
               const std::vector<std::pair<std::string, std::string>>& merges,
               const std::unordered_map<std::string, int>& added, bool ignore_merges);
  std::vector<int> encode(const std::string& text);
  // threads <= 0: one per hardware thread (fewer for small batches)
  std::vector<std::vector<int>> encode_batch(const std::vector<std::string>& texts, int threads);
  std::string decode(const std::vector<int>& ids, bool skip_special) const;
  int token_to_id(const std::string& token) const;
  size_t vocab_size() const { return id_tok_.size(); }

 private:
  using Cache = std::unordered_map<std::string, std::vector<int>>;
  void encode_into(const std::string& text, std::vector<int>& out, Cache& cache) const;
  void encode_plain(const std::string& text, std::vector<int>& out, Cache& cache) const;
  void bpe(const std::string& word, std::vector<int>& out, Cache& cache) const;
  std::unordered_map<std::string, int> vocab_, added_;
  bool ignore_merges_;
  std::string byte_sym_[256];
  std::unordered_map<uint32_t, uint8_t> sym_byte_;
  std::unordered_map<std::string, int> ranks_;
  std::vector<std::string> id_tok_;
  std::unordered_set<int> added_ids_;
  std::vector<std::string> added_sorted_;  // longest first
  bool added_first_[256] = {};
  Cache cache_;
  std::mutex mu_;  // encode mutates the cache; callers may release the GIL
};

}  // namespace qbn
