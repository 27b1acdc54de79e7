// Direct matcher for rs-nanogpt's pre-tokenizer pattern
// (src/tokenizer/shared.rs:33-41), the alternation of
//   1. [^\r\n\p{L}\p{N}]?[Lu Lt Lm Lo M]*[Ll Lm Lo M]+(?i:'s|'t|'re|'ve|'m|'ll|'d)?
//   2. [^\r\n\p{L}\p{N}]?[Lu Lt Lm Lo M]+[Ll Lm Lo M]*(?i:'s|'t|'re|'ve|'m|'ll|'d)?
//   3. \p{N}{1,3}
//   4.  ?[^\s\p{L}\p{N}]+[\r\n/]*
//   5. \s*[\r\n]+
//   6. \s+(?!\S)
//   7. \s+
// A backtracking engine tries the branches in order at each start position
// and returns the first that succeeds, with greedy quantifiers backing off one
// character at a time. Each branch below computes that first success in
// closed form:
//   * branch 1: the greedy upper-ish run [s, e) backs off to the largest k in
//     [s, e] whose codepoint is lower-ish; the lower-ish run then extends
//     greedily and the optional contraction is tried.
//   * branch 5: \s* backs off to the last CR/LF inside the whitespace run.
//   * branch 6: the whitespace run either reaches the end of the text or backs
//     off by exactly one character (which is whitespace, so (?!\S) holds).
// Every codepoint is matched by some branch, so pieces tile the input.
#include "pretok.h"

#include "unicode_tables.h"

namespace nanogpt_host {

static uint8_t lookup_slow(uint32_t cp) {
  int lo = 0, hi = kUcRangeCount - 1;
  while (lo <= hi) {
    int mid = (lo + hi) >> 1;
    if (cp < kUcRanges[mid].lo) hi = mid - 1;
    else if (cp > kUcRanges[mid].hi) lo = mid + 1;
    else return kUcRanges[mid].flags;
  }
  return 0;
}

uint8_t uc_flags(uint32_t cp) {
  struct Ascii { uint8_t f[128]; Ascii() { for (uint32_t c = 0; c < 128; ++c) f[c] = lookup_slow(c); } };
  static const Ascii ascii;  // thread-safe one-time init
  if (cp < 128) return ascii.f[cp];
  return lookup_slow(cp);
}

namespace {

struct Cursor {
  std::vector<uint32_t> cp;    // codepoints
  std::vector<uint32_t> off;   // byte offset of each codepoint, plus the end
  std::vector<uint8_t> fl;     // class flags per codepoint
};

void decode_utf8(std::string_view s, Cursor& c) {
  c.cp.clear(); c.off.clear(); c.fl.clear();
  const auto* p = reinterpret_cast<const unsigned char*>(s.data());
  size_t n = s.size(), i = 0;
  while (i < n) {
    uint32_t b = p[i], cp; size_t len;
    if (b < 0x80) { cp = b; len = 1; }
    else if ((b >> 5) == 0x6 && i + 1 < n) { cp = ((b & 0x1F) << 6) | (p[i + 1] & 0x3F); len = 2; }
    else if ((b >> 4) == 0xE && i + 2 < n) {
      cp = ((b & 0x0F) << 12) | ((p[i + 1] & 0x3F) << 6) | (p[i + 2] & 0x3F); len = 3;
    } else if ((b >> 3) == 0x1E && i + 3 < n) {
      cp = ((b & 0x07) << 18) | ((p[i + 1] & 0x3F) << 12) | ((p[i + 2] & 0x3F) << 6) | (p[i + 3] & 0x3F);
      len = 4;
    } else { cp = 0xFFFD; len = 1; }  // invalid input: treat the byte as a symbol
    c.cp.push_back(cp);
    c.off.push_back(static_cast<uint32_t>(i));
    c.fl.push_back(uc_flags(cp));
    i += len;
  }
  c.off.push_back(static_cast<uint32_t>(n));
}

inline bool is_crlf(uint32_t cp) { return cp == '\r' || cp == '\n'; }

struct Matcher {
  const Cursor& c;
  size_t n;
  bool upper(size_t i) const { return i < n && (c.fl[i] & UC_UPPERISH); }
  bool lower(size_t i) const { return i < n && (c.fl[i] & UC_LOWERISH); }
  bool number(size_t i) const { return i < n && (c.fl[i] & UC_NUMBER); }
  bool space(size_t i) const { return i < n && (c.fl[i] & UC_SPACE); }
  // [^\r\n\p{L}\p{N}]
  bool prefix(size_t i) const {
    return i < n && !is_crlf(c.cp[i]) && !(c.fl[i] & (UC_LETTER | UC_NUMBER));
  }
  // [^\s\p{L}\p{N}]
  bool symbol(size_t i) const {
    return i < n && !(c.fl[i] & (UC_LETTER | UC_NUMBER | UC_SPACE));
  }

  static uint32_t fold(uint32_t cp) {
    if (cp >= 'A' && cp <= 'Z') return cp + 32;
    if (cp == 0x17F) return 's';  // LATIN SMALL LETTER LONG S folds to 's'
    return cp;
  }
  // (?i:'s|'t|'re|'ve|'m|'ll|'d)? -> number of codepoints consumed.
  size_t contraction(size_t f) const {
    if (f >= n || c.cp[f] != '\'' || f + 1 >= n) return 0;
    uint32_t a = fold(c.cp[f + 1]);
    if (a == 's' || a == 't') return 2;
    uint32_t b = f + 2 < n ? fold(c.cp[f + 2]) : 0;
    if (a == 'r' && b == 'e') return 3;
    if (a == 'v' && b == 'e') return 3;
    if (a == 'm') return 2;
    if (a == 'l' && b == 'l') return 3;
    if (a == 'd') return 2;
    return 0;
  }

  size_t branch1(size_t i) const {
    for (int p = prefix(i) ? 1 : 0; p >= 0; --p) {
      size_t s = i + p, e = s;
      while (upper(e)) ++e;
      for (size_t k = e + 1; k-- > s;) {
        if (lower(k)) {
          size_t f = k;
          while (lower(f)) ++f;
          return f + contraction(f);
        }
      }
    }
    return 0;
  }

  size_t branch2(size_t i) const {
    for (int p = prefix(i) ? 1 : 0; p >= 0; --p) {
      size_t s = i + p, e = s;
      while (upper(e)) ++e;
      if (e == s) continue;
      size_t f = e;
      while (lower(f)) ++f;
      return f + contraction(f);
    }
    return 0;
  }

  size_t branch3(size_t i) const {
    size_t f = i;
    while (f - i < 3 && number(f)) ++f;
    return f > i ? f : 0;
  }

  size_t branch4(size_t i) const {
    size_t s;
    if (i < n && c.cp[i] == ' ' && symbol(i + 1)) s = i + 1;
    else if (symbol(i)) s = i;
    else return 0;
    size_t f = s;
    while (symbol(f)) ++f;
    while (f < n && (is_crlf(c.cp[f]) || c.cp[f] == '/')) ++f;
    return f;
  }

  size_t branch5(size_t i) const {
    size_t e = i;
    while (space(e)) ++e;
    for (size_t k = e; k-- > i;)
      if (is_crlf(c.cp[k])) return k + 1;
    return 0;
  }

  size_t branch67(size_t i) const {
    size_t e = i;
    while (space(e)) ++e;
    if (e == i) return 0;
    if (e == n) return e;          // (?!\S) holds at end of text
    if (e - 1 > i) return e - 1;   // back off one whitespace char
    return e;                      // branch 7: plain \s+
  }

  size_t match(size_t i) const {
    size_t m;
    if ((m = branch1(i))) return m;
    if ((m = branch2(i))) return m;
    if ((m = branch3(i))) return m;
    if ((m = branch4(i))) return m;
    if ((m = branch5(i))) return m;
    if ((m = branch67(i))) return m;
    return i + 1;  // unreachable for valid input; keeps the scan total
  }
};

}  // namespace

void pre_tokenize(std::string_view text, std::vector<std::pair<uint32_t, uint32_t>>& out) {
  thread_local Cursor c;
  decode_utf8(text, c);
  Matcher m{c, c.cp.size()};
  size_t i = 0;
  while (i < m.n) {
    size_t j = m.match(i);
    out.emplace_back(c.off[i], c.off[j]);
    i = j;
  }
}

}  // namespace nanogpt_host
