#include "trainer.h"

#include <algorithm>
#include <atomic>
#include <cstdio>
#include <queue>
#include <stdexcept>
#include <string_view>
#include <thread>

#include "bpe.h"
#include "pretok.h"

namespace nanogpt_host {

void BpeTrainer::count(const std::vector<std::string>& docs, int threads) {
  if (threads <= 0) threads = std::max(1u, std::thread::hardware_concurrency());
  threads = int(std::min<size_t>(threads, std::max<size_t>(1, docs.size())));
  std::vector<std::unordered_map<std::string, uint64_t>> local(threads);
  std::atomic<size_t> next{0};
  auto work = [&](int t) {
    std::vector<std::pair<uint32_t, uint32_t>> pieces;
    auto& m = local[t];
    for (size_t i; (i = next.fetch_add(1)) < docs.size();) {
      pieces.clear();
      pre_tokenize(docs[i], pieces);
      for (auto [b, e] : pieces) ++m[docs[i].substr(b, e - b)];
    }
  };
  if (threads == 1) {
    work(0);
  } else {
    std::vector<std::thread> pool;
    for (int t = 0; t < threads; ++t) pool.emplace_back(work, t);
    for (auto& th : pool) th.join();
  }
  for (auto& m : local)
    for (auto& [k, v] : m) counts_[k] += v;
}

namespace {

constexpr uint32_t kTomb = UINT32_MAX;

struct State {
  std::vector<uint32_t> tok;
  std::vector<int32_t> next, prev;
  uint64_t count;
};

struct PairInfo {
  uint64_t count = 0;
  std::vector<std::pair<uint32_t, uint32_t>> locations;  // (state, left index)
};

inline uint64_t key_of(uint32_t a, uint32_t b) { return (uint64_t(a) << 32) | b; }

struct HeapEntry {
  uint64_t count;
  uint32_t a, b;
};

}  // namespace

std::vector<std::string> BpeTrainer::train(size_t num_merges, int progress) {
  std::vector<State> states;
  states.reserve(counts_.size());
  for (auto& [s, c] : counts_) {
    State st;
    size_t n = s.size();
    st.tok.resize(n); st.next.resize(n); st.prev.resize(n);
    for (size_t i = 0; i < n; ++i) {
      st.tok[i] = uint8_t(s[i]);
      st.next[i] = i + 1 < n ? int32_t(i + 1) : -1;
      st.prev[i] = int32_t(i) - 1;
    }
    st.count = c;
    states.push_back(std::move(st));
  }

  std::unordered_map<uint64_t, PairInfo> info;
  for (uint32_t si = 0; si < states.size(); ++si) {
    const State& st = states[si];
    for (uint32_t l = 0; l < st.tok.size(); ++l) {
      if (st.next[l] < 0) continue;
      auto& e = info[key_of(st.tok[l], st.tok[st.next[l]])];
      e.count += st.count;
      e.locations.emplace_back(si, l);
    }
  }

  std::vector<std::string> bytes;
  bytes.reserve(256 + num_merges);
  for (int i = 0; i < 256; ++i) bytes.emplace_back(1, char(i));

  auto less = [&bytes](const HeapEntry& x, const HeapEntry& y) {
    if (x.count != y.count) return x.count < y.count;
    int c = bytes[x.a].compare(bytes[y.a]);
    if (c != 0) return c < 0;
    return bytes[x.b].compare(bytes[y.b]) < 0;
  };
  std::priority_queue<HeapEntry, std::vector<HeapEntry>, decltype(less)> heap(less);
  for (auto& [k, e] : info)
    if (e.count > 0) heap.push({e.count, uint32_t(k >> 32), uint32_t(k)});

  std::vector<std::string> merges;
  std::vector<uint64_t> touched;
  while (merges.size() < num_merges) {
    // Pop stale entries until the top reflects a live pair's current count.
    bool found = false;
    HeapEntry best{};
    while (!heap.empty()) {
      best = heap.top();
      auto it = info.find(key_of(best.a, best.b));
      if (it != info.end() && it->second.count == best.count && best.count > 0) { found = true; break; }
      heap.pop();
    }
    if (!found) break;
    heap.pop();

    const uint32_t a = best.a, b = best.b;
    const uint32_t id = uint32_t(bytes.size());
    bytes.push_back(bytes[a] + bytes[b]);
    merges.push_back(bytes.back());

    auto it = info.find(key_of(a, b));
    std::vector<std::pair<uint32_t, uint32_t>> locations = std::move(it->second.locations);
    info.erase(it);
    touched.clear();
    bool merged_any = false;
    for (auto [si, left] : locations) {
      State& st = states[si];
      int32_t right = st.next[left];
      if (right < 0) continue;
      if (st.tok[left] != a || st.tok[right] != b) continue;
      int32_t before = st.prev[left], after = st.next[right];
      uint64_t c = st.count;
      if (before >= 0) {
        auto f = info.find(key_of(st.tok[before], st.tok[left]));
        if (f != info.end()) {
          if (f->second.count < c) throw std::logic_error("pair count underflow (left neighbour)");
          f->second.count -= c;
          touched.push_back(f->first);
        }
      }
      if (after >= 0) {
        auto f = info.find(key_of(st.tok[right], st.tok[after]));
        if (f != info.end()) {
          if (f->second.count < c) throw std::logic_error("pair count underflow (right neighbour)");
          f->second.count -= c;
          touched.push_back(f->first);
        }
      }
      st.tok[left] = id;
      st.tok[right] = kTomb;
      st.next[left] = after;
      if (after >= 0) st.prev[after] = int32_t(left);
      if (before >= 0) {
        uint64_t k = key_of(st.tok[before], id);
        auto& e = info[k];
        e.count += c;
        e.locations.emplace_back(si, uint32_t(before));
        touched.push_back(k);
      }
      if (after >= 0) {
        uint64_t k = key_of(id, st.tok[after]);
        auto& e = info[k];
        e.count += c;
        e.locations.emplace_back(si, left);
        touched.push_back(k);
      }
      merged_any = true;
    }
    if (!merged_any) throw std::logic_error("merge of a pair with no live locations");
    std::sort(touched.begin(), touched.end());
    touched.erase(std::unique(touched.begin(), touched.end()), touched.end());
    for (uint64_t k : touched) {
      auto f = info.find(k);
      if (f != info.end() && f->second.count > 0)
        heap.push({f->second.count, uint32_t(k >> 32), uint32_t(k)});
    }
    if (progress > 0 && merges.size() % size_t(progress) == 0)
      std::fprintf(stderr, "trained %zu / %zu merges\n", merges.size(), num_merges);
  }
  return merges;
}

void write_vocab(const std::string& path, const std::vector<std::string>& merges) {
  // C stdio rather than iostreams: the module shares a process with other
  // native libraries (Arrow) whose C++ runtime state iostreams would touch.
  std::string text;
  size_t rank = 0;
  for (int i = 0; i < 256; ++i) text += base64_encode(std::string(1, char(i))) + ' ' + std::to_string(rank++) + '\n';
  for (const auto& m : merges) text += base64_encode(m) + ' ' + std::to_string(rank++) + '\n';
  FILE* f = std::fopen(path.c_str(), "wb");
  if (!f) throw std::runtime_error("cannot write vocab file " + path);
  const size_t n = std::fwrite(text.data(), 1, text.size(), f);
  const int rc = std::fclose(f);
  if (n != text.size() || rc != 0) throw std::runtime_error("failed writing vocab file " + path);
}

}  // namespace nanogpt_host
