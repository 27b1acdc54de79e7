// GPT-4-style pre-tokenizer, written as a direct matcher for the one fixed
// pattern rs-nanogpt uses (src/tokenizer/shared.rs:33-58) instead of a general
// regex engine. Leftmost-first alternation semantics of a backtracking engine
// are reproduced branch by branch; see pretok.cpp for the derivation.
#pragma once
#include <cstdint>
#include <string_view>
#include <utility>
#include <vector>

namespace nanogpt_host {

// Split `text` (valid UTF-8) into pre-token pieces. Each piece is returned as
// a [begin, end) byte range; the ranges tile the text exactly.
void pre_tokenize(std::string_view text, std::vector<std::pair<uint32_t, uint32_t>>& out);

// Class flags of one codepoint (UC_* bits from unicode_tables.h).
uint8_t uc_flags(uint32_t cp);

}  // namespace nanogpt_host
