#include "bpe.h"

#include <algorithm>
#include <atomic>
#include <cstdio>
#include <cstdlib>
#include <queue>
#include <stdexcept>
#include <thread>
#include <tuple>

#include "pretok.h"

namespace nanogpt_host {

const char* const kSpecialTokens[9] = {
    "<|bos|>",           "<|user_start|>",   "<|user_end|>",
    "<|assistant_start|>", "<|assistant_end|>", "<|python_start|>",
    "<|python_end|>",    "<|output_start|>", "<|output_end|>"};

static const char kB64[] = "ABCDEFGHIJKLMNOPQRSTUVWXYZabcdefghijklmnopqrstuvwxyz0123456789+/";

std::string base64_encode(std::string_view in) {
  std::string out;
  out.reserve((in.size() + 2) / 3 * 4);
  size_t i = 0;
  for (; i + 2 < in.size(); i += 3) {
    uint32_t v = (uint8_t(in[i]) << 16) | (uint8_t(in[i + 1]) << 8) | uint8_t(in[i + 2]);
    out += kB64[v >> 18]; out += kB64[(v >> 12) & 63]; out += kB64[(v >> 6) & 63]; out += kB64[v & 63];
  }
  if (i + 1 == in.size()) {
    uint32_t v = uint8_t(in[i]) << 16;
    out += kB64[v >> 18]; out += kB64[(v >> 12) & 63]; out += "==";
  } else if (i + 2 == in.size()) {
    uint32_t v = (uint8_t(in[i]) << 16) | (uint8_t(in[i + 1]) << 8);
    out += kB64[v >> 18]; out += kB64[(v >> 12) & 63]; out += kB64[(v >> 6) & 63]; out += '=';
  }
  return out;
}

static int b64_val(char c) {
  if (c >= 'A' && c <= 'Z') return c - 'A';
  if (c >= 'a' && c <= 'z') return c - 'a' + 26;
  if (c >= '0' && c <= '9') return c - '0' + 52;
  if (c == '+') return 62;
  if (c == '/') return 63;
  return -1;
}

// Strict padded standard base64, the alphabet tiktoken files use.
std::string base64_decode(std::string_view in) {
  if (in.size() % 4 != 0) throw std::runtime_error("invalid length");
  std::string out;
  for (size_t i = 0; i < in.size(); i += 4) {
    int v[4], pad = 0;
    for (int j = 0; j < 4; ++j) {
      char c = in[i + j];
      if (c == '=' && i + 4 == in.size() && j >= 2) { v[j] = 0; ++pad; continue; }
      if (pad) throw std::runtime_error("invalid padding");
      v[j] = b64_val(c);
      if (v[j] < 0) throw std::runtime_error(std::string("invalid byte ") + c);
    }
    uint32_t w = (v[0] << 18) | (v[1] << 12) | (v[2] << 6) | v[3];
    out += char(w >> 16);
    if (pad < 2) out += char((w >> 8) & 255);
    if (pad < 1) out += char(w & 255);
  }
  return out;
}

static std::string debug_bytes(const std::string& b) {
  std::string s = "[";
  for (size_t i = 0; i < b.size(); ++i) s += (i ? ", " : "") + std::to_string(unsigned(uint8_t(b[i])));
  return s + "]";
}

Tokenizer Tokenizer::from_file(const std::string& path) {
  FILE* f = std::fopen(path.c_str(), "rb");
  if (!f) throw std::runtime_error("cannot open vocab file " + path);
  std::string contents;
  char buf[1 << 16];
  for (size_t n; (n = std::fread(buf, 1, sizeof buf, f)) > 0;) contents.append(buf, n);
  std::fclose(f);

  std::vector<std::pair<uint32_t, std::string>> entries;
  size_t pos = 0, line_no = 0;
  while (pos < contents.size()) {
    size_t nl = contents.find('\n', pos);
    std::string line = contents.substr(pos, nl == std::string::npos ? std::string::npos : nl - pos);
    pos = nl == std::string::npos ? contents.size() : nl + 1;
    ++line_no;
    if (!line.empty() && line.back() == '\r') line.pop_back();
    size_t sp = line.find(' ');
    if (sp == std::string::npos)
      throw std::runtime_error("vocab line " + std::to_string(line_no) + " missing rank: \"" + line + "\"");
    std::string bytes;
    try {
      bytes = base64_decode(std::string_view(line).substr(0, sp));
    } catch (const std::exception& e) {
      throw std::runtime_error("vocab line " + std::to_string(line_no) + " bad base64: " + e.what());
    }
    std::string rank_str = line.substr(sp + 1);
    char* end = nullptr;
    unsigned long r = rank_str.empty() ? 0 : std::strtoul(rank_str.c_str(), &end, 10);
    if (rank_str.empty() || *end != '\0' || rank_str[0] == '-' || r > 0xFFFFFFFFul)
      throw std::runtime_error("vocab line " + std::to_string(line_no) + " bad rank: " + rank_str);
    entries.emplace_back(uint32_t(r), std::move(bytes));
  }
  std::stable_sort(entries.begin(), entries.end(),
                   [](const auto& a, const auto& b) { return a.first < b.first; });
  for (size_t i = 0; i < entries.size(); ++i)
    if (entries[i].first != i)
      throw std::runtime_error("expected rank " + std::to_string(i) + " at position " +
                               std::to_string(i) + ", got " + std::to_string(entries[i].first));
  if (entries.size() < 256)
    throw std::runtime_error("vocab must contain at least 256 single-byte entries, got " +
                             std::to_string(entries.size()));
  for (size_t i = 0; i < 256; ++i)
    if (entries[i].second != std::string(1, char(i))) {
      char hex[16];
      snprintf(hex, sizeof hex, "%#zx", i);
      throw std::runtime_error("rank " + std::to_string(i + 1) + " must encode single byte " + hex +
                               ", got " + debug_bytes(entries[i].second));
    }
  Tokenizer t;
  t.bytes_.reserve(entries.size());
  for (auto& e : entries) t.bytes_.push_back(std::move(e.second));
  t.build();
  return t;
}

Tokenizer Tokenizer::from_merges(const std::vector<std::string>& merges) {
  Tokenizer t;
  for (int i = 0; i < 256; ++i) t.bytes_.emplace_back(1, char(i));
  for (const auto& m : merges) t.bytes_.push_back(m);
  t.build();
  return t;
}

void Tokenizer::build() {
  first_special_ = static_cast<uint32_t>(bytes_.size());
  encoder_.clear();
  encoder_.reserve(bytes_.size() * 2);
  for (uint32_t id = 0; id < bytes_.size(); ++id) encoder_[bytes_[id]] = id;  // later duplicate wins
  // Every way to split a token's bytes into two known tokens maps to that token.
  pair_rank_.clear();
  for (uint32_t id = 256; id < bytes_.size(); ++id) {
    const std::string& b = bytes_[id];
    for (size_t j = 1; j < b.size(); ++j) {
      auto l = encoder_.find(b.substr(0, j));
      if (l == encoder_.end()) continue;
      auto r = encoder_.find(b.substr(j));
      if (r == encoder_.end()) continue;
      uint64_t key = (uint64_t(l->second) << 32) | r->second;
      pair_rank_[key] = encoder_.at(b);
    }
  }
  special_bytes_.clear();
  for (int i = 0; i < kNumSpecial; ++i) special_bytes_.emplace_back(kSpecialTokens[i]);
}

int Tokenizer::special_id(std::string_view name) const {
  for (int i = 0; i < kNumSpecial; ++i)
    if (name == kSpecialTokens[i]) return int(first_special_) + i;
  return -1;
}

const std::string& Tokenizer::token_bytes(uint32_t id) const {
  if (id < first_special_) return bytes_[id];
  uint32_t k = id - first_special_;
  if (k >= uint32_t(kNumSpecial))
    throw std::out_of_range("token id " + std::to_string(id) + " is out of range (vocab_size " +
                            std::to_string(vocab_size()) + ")");
  return special_bytes_[k];
}

std::vector<uint32_t> Tokenizer::token_byte_lengths() const {
  std::vector<uint32_t> out(vocab_size(), 0);
  for (uint32_t id = 0; id < first_special_; ++id) out[id] = uint32_t(bytes_[id].size());
  return out;
}

uint32_t Tokenizer::pair_rank(uint32_t a, uint32_t b) const {
  auto it = pair_rank_.find((uint64_t(a) << 32) | b);
  return it == pair_rank_.end() ? UINT32_MAX : it->second;
}

// Lowest-rank-first merging over a linked list; ties go to the leftmost pair.
// Stale heap entries are detected with per-node generation counters.
void Tokenizer::encode_piece(const unsigned char* p, size_t n, std::vector<uint32_t>& out) const {
  if (n == 0) return;
  if (n == 1) { out.push_back(p[0]); return; }
  thread_local std::vector<uint32_t> id, gen;
  thread_local std::vector<int32_t> nxt, prv;
  id.assign(p, p + n);
  gen.assign(n, 0);
  nxt.resize(n); prv.resize(n);
  for (size_t i = 0; i < n; ++i) { nxt[i] = i + 1 < n ? int32_t(i + 1) : -1; prv[i] = int32_t(i) - 1; }
  using E = std::tuple<uint32_t, uint32_t, uint32_t, uint32_t, uint32_t>;  // rank, left, lgen, right, rgen
  std::priority_queue<E, std::vector<E>, std::greater<E>> heap;
  for (size_t i = 0; i + 1 < n; ++i) {
    uint32_t r = pair_rank(id[i], id[i + 1]);
    if (r != UINT32_MAX) heap.emplace(r, uint32_t(i), 0u, uint32_t(i + 1), 0u);
  }
  while (!heap.empty()) {
    auto [rank, l, lg, r, rg] = heap.top();
    heap.pop();
    if (nxt[l] != int32_t(r) || gen[l] != lg || gen[r] != rg) continue;
    id[l] = rank;
    ++gen[l];
    int32_t after = nxt[r];
    nxt[l] = after;
    nxt[r] = -1;
    if (after >= 0) prv[after] = int32_t(l);
    if (prv[l] >= 0) {
      uint32_t b = uint32_t(prv[l]);
      uint32_t rr = pair_rank(id[b], id[l]);
      if (rr != UINT32_MAX) heap.emplace(rr, b, gen[b], l, gen[l]);
    }
    if (after >= 0) {
      uint32_t rr = pair_rank(id[l], id[after]);
      if (rr != UINT32_MAX) heap.emplace(rr, l, gen[l], uint32_t(after), gen[after]);
    }
  }
  for (int32_t i = 0; i >= 0; i = nxt[i]) out.push_back(id[i]);
}

std::vector<uint32_t> Tokenizer::encode(std::string_view text) const {
  thread_local std::vector<std::pair<uint32_t, uint32_t>> pieces;
  pieces.clear();
  pre_tokenize(text, pieces);
  std::vector<uint32_t> out;
  out.reserve(text.size() / 3 + 4);
  auto* base = reinterpret_cast<const unsigned char*>(text.data());
  for (auto [b, e] : pieces) encode_piece(base + b, e - b, out);
  return out;
}

std::vector<std::vector<uint32_t>> Tokenizer::encode_batch(const std::vector<std::string>& texts,
                                                           int threads) const {
  std::vector<std::vector<uint32_t>> out(texts.size());
  if (threads <= 0) threads = std::max(1u, std::thread::hardware_concurrency());
  size_t total = 0;
  for (auto& t : texts) total += t.size();
  if (threads == 1 || texts.size() < 2 || total < (1u << 16)) {
    for (size_t i = 0; i < texts.size(); ++i) out[i] = encode(texts[i]);
    return out;
  }
  threads = int(std::min<size_t>(threads, texts.size()));
  std::atomic<size_t> next{0};
  std::vector<std::thread> pool;
  for (int t = 0; t < threads; ++t)
    pool.emplace_back([&] {
      for (size_t i; (i = next.fetch_add(1)) < texts.size();) out[i] = encode(texts[i]);
    });
  for (auto& th : pool) th.join();
  return out;
}

std::string Tokenizer::decode_bytes(const std::vector<uint32_t>& ids) const {
  std::string out;
  for (uint32_t id : ids) out += token_bytes(id);
  return out;
}

}  // namespace nanogpt_host
