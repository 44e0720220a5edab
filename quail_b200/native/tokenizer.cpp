// Byte-level BPE tokenizer for HF tokenizer.json models of the GPT-2 / Qwen2
// family (model "BPE", byte-level pre-tokenizer, the Qwen2 split pattern).
//
//   encode: split out added tokens (exact strings, longest first) -> split the
//   rest into pre-tokens with the Qwen2 pattern
//     (?i:'s|'t|'re|'ve|'m|'ll|'d)|[^\r\n\p{L}\p{N}]?\p{L}+|\p{N}
//     | ?[^\s\p{L}\p{N}]+[\r\n]*|\s*[\r\n]+|\s+(?!\S)|\s+
//   (matched by hand on code points, first alternative that matches, greedy
//   with the regex's backtracking where it matters) -> map each pre-token's
//   UTF-8 bytes to the byte-level alphabet -> merge adjacent symbols by merge
//   rank (lowest rank first, leftmost first) -> ids. Results per pre-token
//   are cached.
//   decode: ids -> token strings -> byte-level alphabet back to bytes.
//
// The input is taken as already NFC-normalized (the normalizer of these
// tokenizers); \p{L} / \p{N} come from the generated unicode_tables.h and \s
// is the Unicode White_Space property.
//
// Reference: the reference tokenizes with the HF `tokenizers` crate
// (crates/quail/src/inputs/tokenizer.rs).
#include <algorithm>
#include <cstdint>
#include <atomic>
#include <mutex>
#include <thread>
#include <stdexcept>
#include <string>
#include <unordered_map>
#include <utility>
#include <vector>

#include "native.h"
#include "unicode_tables.h"

namespace qbn {

namespace {

bool in_ranges(uint32_t cp, const uint32_t (*r)[2], int n) {
  int lo = 0, hi = n - 1;
  while (lo <= hi) {
    const int mid = (lo + hi) / 2;
    if (cp < r[mid][0]) hi = mid - 1;
    else if (cp > r[mid][1]) lo = mid + 1;
    else return true;
  }
  return false;
}

bool is_letter(uint32_t cp) { return in_ranges(cp, kLetterRanges, kLetterRangesCount); }
bool is_number(uint32_t cp) { return in_ranges(cp, kNumberRanges, kNumberRangesCount); }
bool is_space(uint32_t cp) {
  // Unicode White_Space
  return (cp >= 0x9 && cp <= 0xD) || cp == 0x20 || cp == 0x85 || cp == 0xA0 || cp == 0x1680 ||
         (cp >= 0x2000 && cp <= 0x200A) || cp == 0x2028 || cp == 0x2029 || cp == 0x202F || cp == 0x205F ||
         cp == 0x3000;
}
bool is_crlf(uint32_t cp) { return cp == '\r' || cp == '\n'; }

// UTF-8 -> code points with the byte offset of each (malformed bytes pass as U+FFFD, one byte each)
void decode_utf8(const std::string& s, std::vector<uint32_t>& cps, std::vector<size_t>& offs) {
  size_t i = 0;
  while (i < s.size()) {
    const unsigned char c = s[i];
    uint32_t cp = 0xFFFD;
    size_t len = 1;
    if (c < 0x80) {
      cp = c;
    } else if ((c >> 5) == 6 && i + 1 < s.size()) {
      cp = ((c & 0x1F) << 6) | (s[i + 1] & 0x3F);
      len = 2;
    } else if ((c >> 4) == 14 && i + 2 < s.size()) {
      cp = ((c & 0x0F) << 12) | ((s[i + 1] & 0x3F) << 6) | (s[i + 2] & 0x3F);
      len = 3;
    } else if ((c >> 3) == 30 && i + 3 < s.size()) {
      cp = ((c & 0x07) << 18) | ((s[i + 1] & 0x3F) << 12) | ((s[i + 2] & 0x3F) << 6) | (s[i + 3] & 0x3F);
      len = 4;
    }
    cps.push_back(cp);
    offs.push_back(i);
    i += len;
  }
  offs.push_back(s.size());
}

void append_utf8(std::string& out, uint32_t cp) {
  if (cp < 0x80) {
    out += (char)cp;
  } else if (cp < 0x800) {
    out += (char)(0xC0 | (cp >> 6));
    out += (char)(0x80 | (cp & 0x3F));
  } else if (cp < 0x10000) {
    out += (char)(0xE0 | (cp >> 12));
    out += (char)(0x80 | ((cp >> 6) & 0x3F));
    out += (char)(0x80 | (cp & 0x3F));
  } else {
    out += (char)(0xF0 | (cp >> 18));
    out += (char)(0x80 | ((cp >> 12) & 0x3F));
    out += (char)(0x80 | ((cp >> 6) & 0x3F));
    out += (char)(0x80 | (cp & 0x3F));
  }
}

uint32_t lower_ascii(uint32_t c) { return (c >= 'A' && c <= 'Z') ? c + 32 : c; }

// length (in code points) of the pre-token starting at i
size_t match_pretoken(const std::vector<uint32_t>& cp, size_t i) {
  const size_t n = cp.size();
  // 1. contractions, ASCII case-insensitive
  if (cp[i] == '\'' && i + 1 < n) {
    const uint32_t a = lower_ascii(cp[i + 1]);
    const uint32_t b = i + 2 < n ? lower_ascii(cp[i + 2]) : 0;
    if (a == 's' || a == 't' || a == 'm' || a == 'd') return 2;
    if ((a == 'r' && b == 'e') || (a == 'v' && b == 'e') || (a == 'l' && b == 'l')) return 3;
  }
  // 2. [^\r\n\p{L}\p{N}]?\p{L}+
  {
    size_t j = i;
    if (!is_crlf(cp[j]) && !is_letter(cp[j]) && !is_number(cp[j]) && j + 1 < n && is_letter(cp[j + 1])) ++j;
    if (is_letter(cp[j])) {
      while (j < n && is_letter(cp[j])) ++j;
      return j - i;
    }
  }
  // 3. \p{N}
  if (is_number(cp[i])) return 1;
  // 4. ' ?[^\s\p{L}\p{N}]+[\r\n]*'
  {
    auto sym = [&](uint32_t c) { return !is_space(c) && !is_letter(c) && !is_number(c); };
    size_t j = i;
    if (cp[j] == ' ' && j + 1 < n && sym(cp[j + 1])) ++j;
    if (sym(cp[j])) {
      while (j < n && sym(cp[j])) ++j;
      while (j < n && is_crlf(cp[j])) ++j;
      return j - i;
    }
  }
  // whitespace alternatives
  size_t end = i;
  while (end < n && is_space(cp[end])) ++end;
  if (end > i) {
    // 5. \s*[\r\n]+ : up to the last CR / LF of the whitespace run
    size_t last = 0;
    for (size_t k = i; k < end; ++k)
      if (is_crlf(cp[k])) last = k + 1;
    if (last > 0) return last - i;
    // 6. \s+(?!\S) : the run, less its last character when a non-space follows
    if (end == n) return end - i;
    if (end - i >= 2) return end - 1 - i;
    // 7. \s+
    return end - i;
  }
  return 1;  // unreachable: every code point is a letter, number, space or symbol
}

}  // namespace

BpeTokenizer::BpeTokenizer(const std::unordered_map<std::string, int>& vocab,
                           const std::vector<std::pair<std::string, std::string>>& merges,
                           const std::unordered_map<std::string, int>& added, bool ignore_merges)
    : vocab_(vocab), added_(added), ignore_merges_(ignore_merges) {
  // the byte-level alphabet: printable bytes map to themselves, the others to U+0100 onwards
  int next = 0;
  for (int b = 0; b < 256; ++b) {
    const bool keep = (b >= '!' && b <= '~') || (b >= 0xA1 && b <= 0xAC) || (b >= 0xAE && b <= 0xFF);
    const uint32_t cp = keep ? (uint32_t)b : 256u + (uint32_t)next++;
    std::string s;
    append_utf8(s, cp);
    byte_sym_[b] = s;
    sym_byte_[cp] = (uint8_t)b;
  }
  for (size_t r = 0; r < merges.size(); ++r) ranks_[merges[r].first + '\x01' + merges[r].second] = (int)r;
  for (const auto& kv : vocab_) {
    if ((size_t)kv.second >= id_tok_.size()) id_tok_.resize(kv.second + 1);
    id_tok_[kv.second] = kv.first;
  }
  for (const auto& kv : added_) {
    if ((size_t)kv.second >= id_tok_.size()) id_tok_.resize(kv.second + 1);
    id_tok_[kv.second] = kv.first;
    added_ids_.insert(kv.second);
    added_sorted_.push_back(kv.first);
    if (!kv.first.empty()) added_first_[(unsigned char)kv.first[0]] = true;
  }
  std::sort(added_sorted_.begin(), added_sorted_.end(),
            [](const std::string& a, const std::string& b) { return a.size() > b.size(); });
}

void BpeTokenizer::bpe(const std::string& word, std::vector<int>& out, Cache& cache) const {
  auto hit = cache.find(word);
  if (hit != cache.end()) {
    out.insert(out.end(), hit->second.begin(), hit->second.end());
    return;
  }
  std::vector<int> ids;
  auto whole = vocab_.find(word);
  if (ignore_merges_ && whole != vocab_.end()) {
    ids.push_back(whole->second);
  } else {
    // symbols: one per byte-level character
    std::vector<std::string> sym;
    std::vector<uint32_t> cps;
    std::vector<size_t> offs;
    decode_utf8(word, cps, offs);
    for (size_t k = 0; k < cps.size(); ++k) sym.push_back(word.substr(offs[k], offs[k + 1] - offs[k]));
    while (sym.size() > 1) {
      int best = -1;
      size_t at = 0;
      for (size_t k = 0; k + 1 < sym.size(); ++k) {
        auto r = ranks_.find(sym[k] + '\x01' + sym[k + 1]);
        if (r != ranks_.end() && (best < 0 || r->second < best)) {
          best = r->second;
          at = k;
        }
      }
      if (best < 0) break;
      sym[at] += sym[at + 1];
      sym.erase(sym.begin() + at + 1);
    }
    for (const auto& s : sym) {
      auto v = vocab_.find(s);
      if (v == vocab_.end()) throw std::runtime_error("BPE symbol missing from the vocabulary: " + s);
      ids.push_back(v->second);
    }
  }
  if (cache.size() < 1 << 20) cache.emplace(word, ids);
  out.insert(out.end(), ids.begin(), ids.end());
}

void BpeTokenizer::encode_plain(const std::string& text, std::vector<int>& out, Cache& cache) const {
  std::vector<uint32_t> cps;
  std::vector<size_t> offs;
  decode_utf8(text, cps, offs);
  size_t i = 0;
  while (i < cps.size()) {
    const size_t len = match_pretoken(cps, i);
    std::string word;
    for (size_t b = offs[i]; b < offs[i + len]; ++b) word += byte_sym_[(unsigned char)text[b]];
    bpe(word, out, cache);
    i += len;
  }
}

void BpeTokenizer::encode_into(const std::string& text, std::vector<int>& out, Cache& cache) const {
  size_t start = 0, i = 0;
  while (i < text.size()) {
    const std::string* found = nullptr;
    if (added_first_[(unsigned char)text[i]])
      for (const auto& a : added_sorted_)
        if (!a.empty() && text.compare(i, a.size(), a) == 0) {
          found = &a;
          break;
        }
    if (found == nullptr) {
      ++i;
      continue;
    }
    if (i > start) encode_plain(text.substr(start, i - start), out, cache);
    out.push_back(added_.at(*found));
    i += found->size();
    start = i;
  }
  if (start < text.size()) encode_plain(text.substr(start), out, cache);
}

std::vector<int> BpeTokenizer::encode(const std::string& text) {
  std::lock_guard<std::mutex> lock(mu_);
  std::vector<int> out;
  encode_into(text, out, cache_);
  return out;
}

std::vector<std::vector<int>> BpeTokenizer::encode_batch(const std::vector<std::string>& texts, int threads) {
  std::vector<std::vector<int>> out(texts.size());
  size_t bytes = 0;
  for (const auto& t : texts) bytes += t.size();
  int n = threads > 0 ? threads : (int)std::thread::hardware_concurrency();
  n = (int)std::min<size_t>((size_t)std::max(n, 1), std::max<size_t>(bytes / (64 << 10), 1));
  n = (int)std::min<size_t>((size_t)n, std::max<size_t>(texts.size(), 1));
  if (n <= 1) {
    std::lock_guard<std::mutex> lock(mu_);
    for (size_t i = 0; i < texts.size(); ++i) encode_into(texts[i], out[i], cache_);
    return out;
  }
  // workers take texts round-robin in blocks of 16, each with a cache of its own
  std::atomic<size_t> next{0};
  std::vector<std::thread> pool;
  for (int w = 0; w < n; ++w)
    pool.emplace_back([&]() {
      Cache local;
      for (;;) {
        const size_t b = next.fetch_add(16);
        if (b >= texts.size()) break;
        for (size_t i = b; i < std::min(b + 16, texts.size()); ++i) encode_into(texts[i], out[i], local);
      }
    });
  for (auto& t : pool) t.join();
  return out;
}

std::string BpeTokenizer::decode(const std::vector<int>& ids, bool skip_special) const {
  std::string bytes;
  for (int id : ids) {
    if (id < 0 || (size_t)id >= id_tok_.size()) continue;
    if (added_ids_.count(id)) {
      if (!skip_special) bytes += id_tok_[id];
      continue;
    }
    std::vector<uint32_t> cps;
    std::vector<size_t> offs;
    decode_utf8(id_tok_[id], cps, offs);
    for (uint32_t cp : cps) {
      auto b = sym_byte_.find(cp);
      if (b != sym_byte_.end()) bytes += (char)b->second;
    }
  }
  return bytes;
}

int BpeTokenizer::token_to_id(const std::string& token) const {
  auto a = added_.find(token);
  if (a != added_.end()) return a->second;
  auto v = vocab_.find(token);
  return v == vocab_.end() ? -1 : v->second;
}

}  // namespace qbn
