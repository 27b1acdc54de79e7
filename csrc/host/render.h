// Chat conversation rendering for SFT (rs-nanogpt src/tokenizer/chat.rs:188-300):
// a conversation becomes token ids plus a loss mask that is true exactly on the
// tokens the model must produce (assistant text, python tool-call spans and
// <|assistant_end|>).
#pragma once
#include <cstdint>
#include <string>
#include <vector>

#include "bpe.h"
#include "pack.h"

namespace nanogpt_host {

enum Role : int { kSystem = 0, kUser = 1, kAssistant = 2 };
enum PartKind : int { kText = 0, kPython = 1, kPythonOutput = 2 };

struct Part {
  int kind;
  std::string text;
};

struct Message {
  int role;
  bool has_parts;          // false: `text` holds the content
  std::string text;
  std::vector<Part> parts;
};

using Conversation = std::vector<Message>;

// Throws std::invalid_argument with the reference's messages on malformed input.
Rendered render_conversation(const Tokenizer& tok, const Conversation& conv, size_t max_tokens);

// Render every conversation (in parallel, order preserved), then shuffle once
// with ChaCha8(seed). `names[i]` labels source i in error messages.
std::vector<Rendered> render_mixture(const Tokenizer& tok,
                                     const std::vector<std::vector<Conversation>>& sources,
                                     const std::vector<std::string>& names, size_t row_capacity,
                                     uint64_t seed, int threads);

}  // namespace nanogpt_host
