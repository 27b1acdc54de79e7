#include "render.h"

#include <algorithm>
#include <atomic>
#include <stdexcept>
#include <thread>

#include "chacha.h"

namespace nanogpt_host {

static const char* role_name(int r) {
  return r == kSystem ? "system" : r == kUser ? "user" : "assistant";
}

namespace {
struct Renderer {
  const Tokenizer& tok;
  uint32_t user_start, user_end, assistant_start, assistant_end, python_start, python_end,
      output_start, output_end;
  Rendered out;

  explicit Renderer(const Tokenizer& t) : tok(t) {
    user_start = t.special_id("<|user_start|>");
    user_end = t.special_id("<|user_end|>");
    assistant_start = t.special_id("<|assistant_start|>");
    assistant_end = t.special_id("<|assistant_end|>");
    python_start = t.special_id("<|python_start|>");
    python_end = t.special_id("<|python_end|>");
    output_start = t.special_id("<|output_start|>");
    output_end = t.special_id("<|output_end|>");
  }
  void push(uint32_t id, bool scored) { out.ids.push_back(id); out.mask.push_back(scored); }
  void text(const std::string& s, bool scored) {
    auto ids = tok.encode(s);
    out.ids.insert(out.ids.end(), ids.begin(), ids.end());
    out.mask.insert(out.mask.end(), ids.size(), scored ? 1 : 0);
  }
  void user_turn(const std::string& s) { push(user_start, false); text(s, false); push(user_end, false); }
  void assistant_turn(const Message& m) {
    push(assistant_start, false);
    if (!m.has_parts) {
      text(m.text, true);
    } else {
      for (const auto& p : m.parts) {
        if (p.kind == kText) {
          text(p.text, true);
        } else if (p.kind == kPython) {
          push(python_start, true); text(p.text, true); push(python_end, true);
        } else {
          push(output_start, false); text(p.text, false); push(output_end, false);
        }
      }
    }
    push(assistant_end, true);
  }
};
}  // namespace

Rendered render_conversation(const Tokenizer& tok, const Conversation& msgs, size_t max_tokens) {
  auto invalid = [](const std::string& m) { return std::invalid_argument(m); };
  if (msgs.empty()) throw invalid("conversation has no messages");
  Renderer r(tok);
  r.push(tok.bos_id(), false);
  size_t first = 0, logical = 0, offset = 0;
  if (msgs[0].role == kSystem) {
    if (msgs[0].has_parts) throw invalid("system message content must be text");
    if (msgs.size() < 2)
      throw invalid("system message must be followed by a user message, but the conversation ends after it");
    if (msgs[1].role != kUser)
      throw invalid(std::string("system message must be followed by a user message, got ") + role_name(msgs[1].role));
    if (msgs[1].has_parts) throw invalid("message 1: user message content must be text");
    r.user_turn(msgs[0].text + "\n\n" + msgs[1].text);
    first = 2;
    logical = 1;
    offset = 1;
  }
  for (size_t i = first; i < msgs.size(); ++i) {
    const Message& m = msgs[i];
    bool expect_user = logical % 2 == 0;
    int expected = expect_user ? kUser : kAssistant;
    if (m.role != expected)
      throw invalid("message " + std::to_string(logical + offset) + ": expected " + role_name(expected) +
                    ", got " + role_name(m.role));
    if (expect_user) {
      if (m.has_parts)
        throw invalid("message " + std::to_string(logical + offset) + ": user message content must be text");
      r.user_turn(m.text);
    } else {
      r.assistant_turn(m);
    }
    ++logical;
  }
  if (r.out.ids.size() > max_tokens) {
    r.out.ids.resize(max_tokens);
    r.out.mask.resize(max_tokens);
  }
  return std::move(r.out);
}

std::vector<Rendered> render_mixture(const Tokenizer& tok,
                                     const std::vector<std::vector<Conversation>>& sources,
                                     const std::vector<std::string>& names, size_t row_capacity,
                                     uint64_t seed, int threads) {
  std::vector<std::pair<size_t, size_t>> jobs;  // (source, index)
  for (size_t s = 0; s < sources.size(); ++s)
    for (size_t i = 0; i < sources[s].size(); ++i) jobs.emplace_back(s, i);
  std::vector<Rendered> out(jobs.size());
  std::vector<std::string> errors(jobs.size());
  if (threads <= 0) threads = std::max(1u, std::thread::hardware_concurrency());
  std::atomic<size_t> next{0};
  auto work = [&] {
    for (size_t k; (k = next.fetch_add(1)) < jobs.size();) {
      auto [s, i] = jobs[k];
      try {
        out[k] = render_conversation(tok, sources[s][i], row_capacity);
      } catch (const std::exception& e) {
        errors[k] = names[s] + "[" + std::to_string(i) + "]: " + e.what();
      }
    }
  };
  std::vector<std::thread> pool;
  for (int t = 0; t < threads; ++t) pool.emplace_back(work);
  for (auto& th : pool) th.join();
  for (auto& e : errors)
    if (!e.empty()) throw std::invalid_argument(e);  // first failure in mixture order
  ChaCha8 rng(seed);
  rng.shuffle(out.size(), [&](size_t i, size_t j) { std::swap(out[i], out[j]); });
  return out;
}

}  // namespace nanogpt_host
