// BPE trainer: counts unique pre-tokens, then learns merges greedily.
// Selection and merge semantics follow rs-nanogpt src/tokenizer/trainer.rs:
//   * best pair = max count, ties broken by the lexicographic max of
//     (bytes(left), bytes(right))  (trainer.rs:117-129);
//   * merging walks the pair's recorded locations in insertion order, skips
//     stale ones, and adjusts neighbour pair counts only for pairs still in
//     the table (trainer.rs:131-224).
// The reference rescans every pair per merge; this version keeps a lazy
// max-heap keyed the same way, which selects the same pair.
#pragma once
#include <cstdint>
#include <string>
#include <unordered_map>
#include <vector>

namespace nanogpt_host {

class BpeTrainer {
 public:
  // Pre-tokenize and count a batch of documents (multi-threaded).
  void count(const std::vector<std::string>& docs, int threads);
  // Learn up to `num_merges` merges from everything counted so far.
  // `progress` > 0 prints "trained N / M merges" every `progress` merges.
  std::vector<std::string> train(size_t num_merges, int progress);
  size_t unique_pretokens() const { return counts_.size(); }

 private:
  std::unordered_map<std::string, uint64_t> counts_;
};

// tiktoken file: 256 single bytes then the merges, `<base64> <rank>` per line.
void write_vocab(const std::string& path, const std::vector<std::string>& merges);

}  // namespace nanogpt_host
