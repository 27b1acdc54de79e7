// ChaCha8 random generator laid out the way Rust's rand_chacha presents it
// (64-bit block counter, stream 0, 4-block output buffer consumed one 32-bit
// word at a time), seeded like rand_core's `seed_from_u64` (a PCG32 stream
// fills the 32-byte key). rs-nanogpt draws from it in src/eval/sample.rs:163-174
// (top-k sampling) and src/tasks/mixture.rs:61-99 (mixture shuffle).
// The ChaCha core follows the public algorithm description (Bernstein 2008;
// RFC 7539 quarter round) with 8 rounds.
#pragma once
#include <cstddef>
#include <cstdint>
#include <utility>
#include <vector>

namespace nanogpt_host {

class ChaCha8 {
 public:
  explicit ChaCha8(uint64_t seed) {
    uint64_t state = seed;
    for (int i = 0; i < 8; ++i) {
      // PCG32 (XSH-RR) step, as rand_core uses to expand a u64 seed.
      state = state * 6364136223846793005ull + 11634580027462260723ull;
      uint32_t xorshifted = uint32_t(((state >> 18) ^ state) >> 27);
      uint32_t rot = uint32_t(state >> 59);
      key_[i] = (xorshifted >> rot) | (xorshifted << ((32 - rot) & 31));
    }
    idx_ = kBufWords;  // empty buffer
  }

  uint32_t next_u32() {
    if (idx_ >= kBufWords) refill();
    return buf_[idx_++];
  }

  uint64_t next_u64() {
    if (idx_ + 1 < kBufWords) {
      uint64_t lo = buf_[idx_], hi = buf_[idx_ + 1];
      idx_ += 2;
      return (hi << 32) | lo;
    }
    if (idx_ >= kBufWords) {
      refill();
      uint64_t lo = buf_[0], hi = buf_[1];
      idx_ = 2;
      return (hi << 32) | lo;
    }
    uint64_t lo = buf_[kBufWords - 1];
    refill();
    uint64_t hi = buf_[0];
    idx_ = 1;
    return (hi << 32) | lo;
  }

  // Uniform in [0, 1) with 53 random bits.
  double next_f64() { return double(next_u64() >> 11) * (1.0 / 9007199254740992.0); }

  // Uniform integer in [0, range) for 0 < range <= 2^32 - 1, using a widening
  // multiply with one extra draw to shrink the bias (Canon's method).
  uint32_t below(uint32_t range) {
    uint64_t m = uint64_t(next_u32()) * range;
    uint32_t result = uint32_t(m >> 32), lo = uint32_t(m);
    if (lo > uint32_t(0u - range)) {
      uint64_t m2 = uint64_t(next_u32()) * range;
      uint32_t hi2 = uint32_t(m2 >> 32);
      if (uint64_t(lo) + hi2 > 0xFFFFFFFFull) result += 1;
    }
    return result;
  }

  // In-place shuffle of `n` elements through `swap(i, j)`: a forward
  // Fisher-Yates that draws several indices from one 32-bit sample
  // (the "increasing uniform" chooser).
  template <class Swap>
  void shuffle(size_t n, Swap swap) {
    if (n <= 1) return;
    uint32_t cur = 0, chunk = 0;
    uint8_t remaining = 1;  // the first index (range 1) needs no draw
    for (size_t i = 0; i < n; ++i) {
      uint32_t next_n = cur + 1;
      uint8_t next_remaining;
      if (remaining > 0) {
        next_remaining = uint8_t(remaining - 1);
      } else {
        uint32_t product = next_n, k = next_n + 1;
        while (true) {
          uint64_t p = uint64_t(product) * k;
          if (p > 0xFFFFFFFFull) break;
          product = uint32_t(p);
          ++k;
        }
        uint8_t count = uint8_t(k - next_n);
        chunk = below(product);
        next_remaining = uint8_t(count - 1);
      }
      size_t j;
      if (next_remaining == 0) {
        j = chunk;
      } else {
        j = chunk % next_n;
        chunk /= next_n;
      }
      remaining = next_remaining;
      cur = next_n;
      swap(i, j);
    }
  }

 private:
  static constexpr int kBufWords = 64;
  static inline uint32_t rotl(uint32_t v, int c) { return (v << c) | (v >> (32 - c)); }

  void refill() {
    for (int blk = 0; blk < 4; ++blk) {
      uint32_t in[16] = {0x61707865u, 0x3320646eu, 0x79622d32u, 0x6b206574u,
                         key_[0], key_[1], key_[2], key_[3], key_[4], key_[5], key_[6], key_[7],
                         uint32_t(counter_), uint32_t(counter_ >> 32), 0u, 0u};
      uint32_t x[16];
      for (int i = 0; i < 16; ++i) x[i] = in[i];
      for (int r = 0; r < 4; ++r) {  // 4 double rounds = 8 rounds
        qr(x, 0, 4, 8, 12); qr(x, 1, 5, 9, 13); qr(x, 2, 6, 10, 14); qr(x, 3, 7, 11, 15);
        qr(x, 0, 5, 10, 15); qr(x, 1, 6, 11, 12); qr(x, 2, 7, 8, 13); qr(x, 3, 4, 9, 14);
      }
      for (int i = 0; i < 16; ++i) buf_[blk * 16 + i] = x[i] + in[i];
      ++counter_;
    }
    idx_ = 0;
  }
  static inline void qr(uint32_t* x, int a, int b, int c, int d) {
    x[a] += x[b]; x[d] ^= x[a]; x[d] = rotl(x[d], 16);
    x[c] += x[d]; x[b] ^= x[c]; x[b] = rotl(x[b], 12);
    x[a] += x[b]; x[d] ^= x[a]; x[d] = rotl(x[d], 8);
    x[c] += x[d]; x[b] ^= x[c]; x[b] = rotl(x[b], 7);
  }

  uint32_t key_[8];
  uint64_t counter_ = 0;
  uint32_t buf_[kBufWords];
  int idx_;
};

}  // namespace nanogpt_host
