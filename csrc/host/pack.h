// Row packers.
//  * CropPacker: pretraining best-fit crop packing (rs-nanogpt
//    src/data/loader.rs:9-153). A pool of `buffer_size` documents; each row of
//    T+1 tokens takes the largest pooled doc that fits the gap, or crops the
//    shortest doc to fill it exactly. Resumable: when its input queue runs dry
//    it reports that it needs more documents, so a producer thread can feed it
//    without ever changing the packing decisions.
//  * pack_epoch: SFT best-fit pad packing with loss masks and an FNV digest
//    (src/tasks/pack.rs:97-402).
#pragma once
#include <cstdint>
#include <deque>
#include <vector>

namespace nanogpt_host {

class CropPacker {
 public:
  CropPacker(int batch_rows, int tokens_dim, int buffer_size);
  void push(std::vector<uint32_t> doc) { pending_.push_back(std::move(doc)); }
  // Called when the document source is exhausted (input queue must be empty):
  // starts a new pass. Throws if the finished pass produced no documents.
  void end_pass();
  // Advance packing. Returns true when a full batch is ready (fetch with
  // take_rows); false when more input documents are needed first.
  bool step();
  std::vector<uint32_t> take_rows();
  size_t pending() const { return pending_.size(); }

 private:
  bool refill();  // false when the queue ran dry before the pool was full
  std::deque<std::vector<uint32_t>> pending_;
  std::vector<std::vector<uint32_t>> pool_;
  std::vector<uint32_t> rows_;
  int batch_rows_, row_len_, buffer_size_;
  size_t pos_in_row_ = 0;
  size_t produced_this_pass_ = 0;
};

struct PackStats {
  size_t rows = 0, conversations = 0, pad_tokens = 0, total_tokens = 0, scored_tokens = 0;
};

struct PackedEpoch {
  std::vector<uint32_t> rows;
  std::vector<uint8_t> mask;
  size_t row_capacity = 0;
  PackStats stats;
  uint64_t digest() const;
};

struct Rendered {
  std::vector<uint32_t> ids;
  std::vector<uint8_t> mask;
};

PackedEpoch pack_epoch(const std::vector<Rendered>& rendered, size_t row_capacity, uint32_t bos,
                       size_t buffer_size);

}  // namespace nanogpt_host
