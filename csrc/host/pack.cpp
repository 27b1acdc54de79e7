#include "pack.h"

#include <stdexcept>
#include <string>

namespace nanogpt_host {

CropPacker::CropPacker(int batch_rows, int tokens_dim, int buffer_size)
    : batch_rows_(batch_rows), row_len_(tokens_dim + 1), buffer_size_(buffer_size) {
  if (buffer_size <= 0) throw std::invalid_argument("buffer_size must be positive");
  if (batch_rows <= 0 || tokens_dim <= 0) throw std::invalid_argument("batch shape must be positive");
  rows_.reserve(size_t(batch_rows) * row_len_);
}

void CropPacker::end_pass() {
  if (!pending_.empty()) throw std::logic_error("end_pass with undrained input");
  if (produced_this_pass_ == 0)
    throw std::runtime_error(
        "data source produced no documents in a full pass over the source — empty corpus "
        "(under multi-GPU rank striding each rank keeps only every world_size-th document, so a "
        "corpus with fewer documents than ranks starves this rank)");
  produced_this_pass_ = 0;
}

bool CropPacker::refill() {
  while (pool_.size() < size_t(buffer_size_)) {
    if (pending_.empty()) return false;
    pool_.push_back(std::move(pending_.front()));
    pending_.pop_front();
    ++produced_this_pass_;
  }
  return true;
}

bool CropPacker::step() {
  const size_t total = size_t(batch_rows_) * row_len_;
  while (rows_.size() < total) {
    if (!refill()) return false;
    const size_t remaining = size_t(row_len_) - pos_in_row_;
    // Largest doc that fits; on equal lengths the last one wins.
    long best = -1;
    size_t best_len = 0;
    for (size_t i = 0; i < pool_.size(); ++i) {
      size_t len = pool_[i].size();
      if (len <= remaining && (best < 0 || len >= best_len)) { best = long(i); best_len = len; }
    }
    size_t idx, take;
    if (best >= 0) {
      idx = size_t(best);
      take = best_len;
    } else {
      // Nothing fits: crop the shortest doc (first on ties) to fill the gap.
      idx = 0;
      for (size_t i = 1; i < pool_.size(); ++i)
        if (pool_[i].size() < pool_[idx].size()) idx = i;
      take = remaining;
    }
    const auto& doc = pool_[idx];
    rows_.insert(rows_.end(), doc.begin(), doc.begin() + take);
    pos_in_row_ += take;
    if (pos_in_row_ == size_t(row_len_)) pos_in_row_ = 0;
    // swap_remove
    if (idx + 1 != pool_.size()) pool_[idx] = std::move(pool_.back());
    pool_.pop_back();
  }
  return true;
}

std::vector<uint32_t> CropPacker::take_rows() {
  if (rows_.size() != size_t(batch_rows_) * row_len_) throw std::logic_error("batch not ready");
  std::vector<uint32_t> out;
  out.swap(rows_);
  rows_.reserve(size_t(batch_rows_) * row_len_);
  return out;
}

uint64_t PackedEpoch::digest() const {
  uint64_t h = 0xcbf29ce484222325ull;
  for (size_t i = 0; i < rows.size(); ++i) {
    h ^= uint64_t(rows[i]) | (uint64_t(mask[i] ? 1 : 0) << 32);
    h *= 0x100000001b3ull;
  }
  return h >> 20;
}

PackedEpoch pack_epoch(const std::vector<Rendered>& rendered, size_t row_capacity, uint32_t bos,
                       size_t buffer_size) {
  if (row_capacity < 2)
    throw std::invalid_argument("row capacity must be at least 2 (one input/target pair), got " +
                                std::to_string(row_capacity));
  if (buffer_size == 0) throw std::invalid_argument("buffer_size must be positive");
  PackedEpoch ep;
  ep.row_capacity = row_capacity;
  size_t content = 0;
  for (auto& r : rendered) content += r.ids.size();
  ep.rows.reserve(content + content / 8);
  ep.mask.reserve(content + content / 8);

  std::vector<size_t> buf;  // indices into `rendered`, in arrival order
  size_t src = 0;
  auto refill = [&] {
    while (buf.size() < buffer_size && src < rendered.size()) {
      const auto& c = rendered[src];
      if (c.ids.size() != c.mask.size()) throw std::invalid_argument("rendered ids and mask must have equal length");
      if (c.ids.empty() || c.ids.size() > row_capacity)
        throw std::invalid_argument("conversation of " + std::to_string(c.ids.size()) +
                                    " tokens cannot be packed into rows of " + std::to_string(row_capacity) +
                                    " (render the mixture with max_tokens = row_capacity)");
      buf.push_back(src++);
    }
  };
  while (true) {
    refill();
    if (buf.empty()) break;
    size_t row_start = ep.rows.size();
    while (ep.rows.size() - row_start < row_capacity) {
      size_t remaining = row_capacity - (ep.rows.size() - row_start);
      long best = -1;
      size_t best_len = 0;
      for (size_t i = 0; i < buf.size(); ++i) {  // first max wins
        size_t len = rendered[buf[i]].ids.size();
        if (len <= remaining && len > best_len) { best = long(i); best_len = len; }
      }
      if (best >= 0) {
        const auto& c = rendered[buf[size_t(best)]];
        buf.erase(buf.begin() + best);  // order-preserving remove
        ep.rows.insert(ep.rows.end(), c.ids.begin(), c.ids.end());
        ep.mask.insert(ep.mask.end(), c.mask.begin(), c.mask.end());
        ++ep.stats.conversations;
        refill();
      } else {
        ep.rows.insert(ep.rows.end(), remaining, bos);
        ep.mask.insert(ep.mask.end(), remaining, 0);
        ep.stats.pad_tokens += remaining;
        break;
      }
    }
  }
  ep.stats.rows = ep.rows.size() / row_capacity;
  ep.stats.total_tokens = ep.rows.size();
  for (uint8_t m : ep.mask) ep.stats.scored_tokens += m ? 1 : 0;
  return ep;
}

}  // namespace nanogpt_host
