// Byte-level BPE tokenizer with tiktoken-format vocab I/O.
// Behaviour follows rs-nanogpt src/tokenizer/bpe.rs:37-343 (file format,
// validation rules, special-token block, lowest-rank-first merging).
#pragma once
#include <cstdint>
#include <string>
#include <string_view>
#include <unordered_map>
#include <vector>

namespace nanogpt_host {

extern const char* const kSpecialTokens[9];
constexpr int kNumSpecial = 9;

std::string base64_encode(std::string_view bytes);
// Throws std::runtime_error on malformed input.
std::string base64_decode(std::string_view b64);

class Tokenizer {
 public:
  // Parse a tiktoken file: one `<base64> <rank>` per line, ranks contiguous
  // from 0, the first 256 ranks the single bytes 0x00..0xFF in order.
  static Tokenizer from_file(const std::string& path);
  static Tokenizer from_merges(const std::vector<std::string>& merges);

  uint32_t bos_id() const { return first_special_; }
  uint32_t vocab_size() const { return first_special_ + kNumSpecial; }
  int special_id(std::string_view name) const;  // -1 when unknown
  const std::string& token_bytes(uint32_t id) const;  // specials render as their literal
  std::vector<uint32_t> token_byte_lengths() const;   // 0 for specials

  // Text -> ids. Never emits special ids.
  std::vector<uint32_t> encode(std::string_view text) const;
  // Many texts at once on `threads` worker threads (0 = hardware concurrency).
  std::vector<std::vector<uint32_t>> encode_batch(const std::vector<std::string>& texts,
                                                  int threads) const;
  std::string decode_bytes(const std::vector<uint32_t>& ids) const;

 private:
  void build();
  void encode_piece(const unsigned char* p, size_t n, std::vector<uint32_t>& out) const;
  uint32_t pair_rank(uint32_t a, uint32_t b) const;

  std::vector<std::string> bytes_;                    // id -> bytes (merges included)
  std::unordered_map<std::string, uint32_t> encoder_; // bytes -> id
  // (left id, right id) -> id of the token whose bytes are their concatenation
  std::unordered_map<uint64_t, uint32_t> pair_rank_;
  std::vector<std::string> special_bytes_;
  uint32_t first_special_ = 256;
};

}  // namespace nanogpt_host
