// Token masks from a real GBNF grammar: the step after the reference's toy
// Grammar (src/decoder.rs:378-557), whose get_allowed_tokens (:466-529)
// replays the last ten tokens through one-token rule matches. Here a grammar
// in the GBNF notation is compiled into a stack automaton over bytes, the
// vocabulary into a byte trie, and each sequence's state yields the
// bit-packed allowed-token row that rl_sample_batch / rl_grammar_greedy take
// (bit j of word w is token 32w + j).
//
// Grammar notation (one rule per `name ::= ...`; a rule's alternatives may
// continue on lines that start with '|'; inside parentheses newlines are
// free; '#' starts a comment):
//   "literal"   characters, with escapes \n \r \t \\ \" \' \[ \] \- and
//               \xHH \uHHHH \UHHHHHHHH (code points)
//   [a-z_0-9]   one character in the class; [^...] one character outside it
//               (ranges of code points; surrogates excluded)
//   .           any character
//   name        a rule (defined anywhere in the text)
//   ( ... )     a group of alternatives
//   x* x+ x?    repetition of the preceding element (literal, class, rule or
//               group); x{m} x{m,} x{m,n} bounded repetition
// The grammar text is UTF-8. Matching is over the bytes of the tokens' text:
// a character is its UTF-8 encoding, so a class with non-ASCII members
// compiles into a rule whose alternatives are byte-class sequences (the ASCII
// part stays one byte class), and a character may span several tokens.
//
// Automaton: a state is a set of stacks of element positions. A stack's top
// is always a byte class (or the stack is empty: the start rule is complete,
// so the end-of-sequence token is allowed). Consuming a byte advances every
// stack whose top class holds it and expands references until classes are on
// top again; a reference in tail position replaces its caller's frame, so
// right recursion (x* and the like) does not deepen the stacks. Left
// recursion is rejected when the grammar is compiled.
//
// Masks: the vocabulary's token bytes form a trie walked depth first from the
// state; a subtree is cut at the first byte no stack accepts, so the cost is
// the number of trie nodes the grammar allows next, not the vocabulary size.
// Finished rows are cached by state. Accepts walk a lazy automaton (interned
// stack sets, byte transitions computed once) that the grammar's states share.
#include <algorithm>
#include <cstdint>
#include <cstring>
#include <map>
#include <mutex>
#include <string>
#include <thread>
#include <unordered_map>
#include <vector>

#include "internal.h"
#include "rl_sampler.h"

namespace rl {
namespace gbnf {

enum Kind : uint8_t { kChars = 0, kRef = 1, kEnd = 2 };
struct Elem {
  Kind kind;
  uint32_t arg;  // kChars: byte-set index; kRef: rule index
};
struct ByteSet {
  uint64_t w[4] = {0, 0, 0, 0};
  void add(int c) { w[c >> 6] |= 1ull << (c & 63); }
  bool has(int c) const { return (w[c >> 6] >> (c & 63)) & 1ull; }
  void invert() {
    for (auto& x : w) x = ~x;
  }
};

constexpr size_t kMaxStackDepth = 1024;  // frames of one stack
constexpr size_t kMaxStacks = 4096;      // stacks of one state
constexpr int kMaxRepeat = 1000;         // x{m,n}: n at most

using Stack = std::vector<uint32_t>;
using StackSet = std::vector<Stack>;  // sorted, no duplicates

struct Grammar {
  std::vector<Elem> elems;   // every alternative, each closed by a kEnd element
  std::vector<ByteSet> sets;
  std::vector<std::vector<uint32_t>> alts;  // per rule: its alternatives' first elements
  std::vector<std::string> names;
  uint32_t root = 0;
  // vocabulary trie (CSR): node n's children are child_byte / child_node
  // [child_begin[n], child_begin[n + 1]); the tokens whose bytes end at n are
  // tok_ids[tok_begin[n], tok_begin[n + 1])
  std::vector<uint32_t> child_begin, child_node, tok_begin;
  std::vector<uint8_t> child_byte;
  std::vector<int32_t> tok_ids;
  // each token's bytes: tb[tb_begin[t], tb_begin[t + 1])
  std::vector<uint32_t> tb_begin;
  std::vector<uint8_t> tb;
  int V = 0;
  int eos = -1;
};

// ---------------------------------------------------------------------------
// Parser
// ---------------------------------------------------------------------------
using Seq = std::vector<Elem>;  // an alternative without its kEnd

struct Parser {
  const char* p;
  const char* end;
  Grammar& g;
  std::vector<std::vector<Seq>> bodies;  // per rule
  std::vector<int> defined;
  std::unordered_map<std::string, uint32_t> ids;
  std::string err;

  Parser(const char* text, size_t n, Grammar& gr) : p(text), end(text + n), g(gr) {}

  bool fail(const std::string& m) {
    if (err.empty()) err = m;
    return false;
  }
  uint32_t rule_id(const std::string& name) {
    auto it = ids.find(name);
    if (it != ids.end()) return it->second;
    const uint32_t id = static_cast<uint32_t>(g.names.size());
    ids[name] = id;
    g.names.push_back(name);
    bodies.emplace_back();
    defined.push_back(0);
    return id;
  }
  uint32_t new_rule(const std::string& base) {
    std::string n = base + "#" + std::to_string(g.names.size());  // '#' is not a name character
    const uint32_t id = rule_id(n);
    defined[id] = 1;
    return id;
  }
  uint32_t set_of(const ByteSet& s) {
    g.sets.push_back(s);
    return static_cast<uint32_t>(g.sets.size() - 1);
  }
  static bool name_char(char c) {
    return (c >= 'a' && c <= 'z') || (c >= 'A' && c <= 'Z') || (c >= '0' && c <= '9') || c == '_' || c == '-';
  }
  // spaces and comments; newlines too when nl
  void space(bool nl) {
    while (p < end) {
      if (*p == ' ' || *p == '\t' || (nl && (*p == '\n' || *p == '\r'))) {
        ++p;
      } else if (*p == '#') {
        while (p < end && *p != '\n') ++p;
      } else {
        break;
      }
    }
  }
  // after the end of a line at top level: a following line that starts with
  // '|' continues the rule
  bool continues() {
    const char* q = p;
    while (q < end) {
      if (*q == ' ' || *q == '\t' || *q == '\n' || *q == '\r') {
        ++q;
      } else if (*q == '#') {
        while (q < end && *q != '\n') ++q;
      } else {
        break;
      }
    }
    if (q < end && *q == '|') {
      p = q;
      return true;
    }
    return false;
  }
  bool at_rule_start() const {
    const char* q = p;
    while (q < end && name_char(*q)) ++q;
    if (q == p) return false;
    while (q < end && (*q == ' ' || *q == '\t')) ++q;
    return end - q >= 3 && q[0] == ':' && q[1] == ':' && q[2] == '=';
  }
  std::string name() {
    const char* q = p;
    while (p < end && name_char(*p)) ++p;
    return std::string(q, p);
  }
  static int hexval(char c) {
    if (c >= '0' && c <= '9') return c - '0';
    if (c >= 'a' && c <= 'f') return c - 'a' + 10;
    if (c >= 'A' && c <= 'F') return c - 'A' + 10;
    return -1;
  }
  // one (possibly escaped) character of a literal or class, as a code point:
  // the grammar text is UTF-8; \xHH, \uHHHH and \UHHHHHHHH name code points
  bool hex_cp(int digits, uint32_t* out) {
    if (end - p < digits) return fail("bad hexadecimal escape");
    uint32_t v = 0;
    for (int i = 0; i < digits; ++i) {
      const int h = hexval(p[i]);
      if (h < 0) return fail("bad hexadecimal escape");
      v = v * 16 + static_cast<uint32_t>(h);
    }
    p += digits;
    *out = v;
    return true;
  }
  bool cp_of(uint32_t* out) {
    if (p >= end) return fail("unexpected end of grammar");
    const unsigned char c0 = static_cast<unsigned char>(*p);
    if (c0 != '\\') {
      // UTF-8 sequence of the grammar text
      int n = c0 < 0x80 ? 1 : (c0 >> 5) == 6 ? 2 : (c0 >> 4) == 14 ? 3 : (c0 >> 3) == 30 ? 4 : 0;
      if (n == 0 || end - p < n) return fail("invalid UTF-8 in the grammar text");
      uint32_t v = n == 1 ? c0 : (c0 & (0x7Fu >> n));
      for (int i = 1; i < n; ++i) {
        const unsigned char ci = static_cast<unsigned char>(p[i]);
        if ((ci & 0xC0) != 0x80) return fail("invalid UTF-8 in the grammar text");
        v = (v << 6) | (ci & 0x3Fu);
      }
      p += n;
      *out = v;
      return true;
    }
    ++p;
    if (p >= end) return fail("unfinished escape");
    const char c = *p++;
    switch (c) {
      case 'n': *out = '\n'; return true;
      case 'r': *out = '\r'; return true;
      case 't': *out = '\t'; return true;
      case '\\': case '"': case '\'': case '[': case ']': case '-': case '^': *out = static_cast<unsigned char>(c); return true;
      case 'x': return hex_cp(2, out);
      case 'u': return hex_cp(4, out);
      case 'U': return hex_cp(8, out);
      default: return fail(std::string("unknown escape \\") + c);
    }
  }
  static bool valid_cp(uint32_t v) { return v <= 0x10FFFFu && !(v >= 0xD800u && v <= 0xDFFFu); }
  static int utf8_encode(uint32_t v, uint8_t* b) {
    if (v < 0x80u) {
      b[0] = static_cast<uint8_t>(v);
      return 1;
    }
    if (v < 0x800u) {
      b[0] = static_cast<uint8_t>(0xC0u | (v >> 6));
      b[1] = static_cast<uint8_t>(0x80u | (v & 0x3Fu));
      return 2;
    }
    if (v < 0x10000u) {
      b[0] = static_cast<uint8_t>(0xE0u | (v >> 12));
      b[1] = static_cast<uint8_t>(0x80u | ((v >> 6) & 0x3Fu));
      b[2] = static_cast<uint8_t>(0x80u | (v & 0x3Fu));
      return 3;
    }
    b[0] = static_cast<uint8_t>(0xF0u | (v >> 18));
    b[1] = static_cast<uint8_t>(0x80u | ((v >> 12) & 0x3Fu));
    b[2] = static_cast<uint8_t>(0x80u | ((v >> 6) & 0x3Fu));
    b[3] = static_cast<uint8_t>(0x80u | (v & 0x3Fu));
    return 4;
  }
  // The code points [lo, hi] (no surrogates, one encoded length n > 1) as
  // sequences of byte classes: split until every byte position of the
  // encodings ranges freely below a common prefix (the UTF-8 range split
  // that regular-expression engines use, after Russ Cox's utf8 ranges).
  void utf8_seqs(uint32_t lo, uint32_t hi, std::vector<Seq>* out) {
    static const uint32_t kMaxOfLen[4] = {0x7Fu, 0x7FFu, 0xFFFFu, 0x10FFFFu};
    for (int k = 0; k < 3; ++k)
      if (lo <= kMaxOfLen[k] && hi > kMaxOfLen[k]) {
        utf8_seqs(lo, kMaxOfLen[k], out);
        utf8_seqs(kMaxOfLen[k] + 1, hi, out);
        return;
      }
    uint8_t a[4], b[4];
    const int n = utf8_encode(lo, a);
    for (int i = 1; i < n; ++i) {
      const uint32_t m = (1u << (6 * i)) - 1u;
      if ((lo & ~m) != (hi & ~m)) {
        if ((lo & m) != 0u) {
          utf8_seqs(lo, lo | m, out);
          utf8_seqs((lo | m) + 1u, hi, out);
          return;
        }
        if ((hi & m) != m) {
          utf8_seqs(lo, (hi & ~m) - 1u, out);
          utf8_seqs(hi & ~m, hi, out);
          return;
        }
      }
    }
    utf8_encode(hi, b);
    Seq sq;
    for (int i = 0; i < n; ++i) {
      ByteSet bs;
      for (int c = a[i]; c <= b[i]; ++c) bs.add(c);
      sq.push_back({kChars, set_of(bs)});
    }
    out->push_back(std::move(sq));
  }
  // One character from the code-point ranges (sorted, disjoint, valid): a
  // single byte class when they are all ASCII, else a rule whose
  // alternatives are the ASCII byte class and the multi-byte sequences.
  bool char_element(const std::string& rule, const std::vector<std::pair<uint32_t, uint32_t>>& ranges, Seq* seq) {
    ByteSet ascii;
    bool any_ascii = false;
    std::vector<Seq> alts;
    for (const auto& r : ranges) {
      uint32_t lo = r.first, hi = r.second;
      if (lo <= 0x7Fu) {
        for (uint32_t c = lo; c <= std::min(hi, 0x7Fu); ++c) ascii.add(static_cast<int>(c));
        any_ascii = true;
        if (hi <= 0x7Fu) continue;
        lo = 0x80u;
      }
      utf8_seqs(lo, hi, &alts);
    }
    if (alts.empty()) {
      if (!any_ascii) return fail("a class that matches no character in rule " + rule);
      seq->push_back({kChars, set_of(ascii)});
      return true;
    }
    if (any_ascii) {
      Seq a1;
      a1.push_back({kChars, set_of(ascii)});
      alts.insert(alts.begin(), std::move(a1));
    }
    const uint32_t r = new_rule(rule);
    bodies[r] = std::move(alts);
    seq->push_back({kRef, r});
    return true;
  }
  // ranges -> sorted, merged, without surrogates; complemented when neg
  static std::vector<std::pair<uint32_t, uint32_t>> normalize_ranges(std::vector<std::pair<uint32_t, uint32_t>> v,
                                                                     bool neg) {
    std::sort(v.begin(), v.end());
    std::vector<std::pair<uint32_t, uint32_t>> m;
    for (const auto& r : v) {
      if (!m.empty() && r.first <= m.back().second + 1u) m.back().second = std::max(m.back().second, r.second);
      else m.push_back(r);
    }
    if (neg) {
      std::vector<std::pair<uint32_t, uint32_t>> c;
      uint32_t next = 0;
      for (const auto& r : m) {
        if (r.first > next) c.push_back({next, r.first - 1u});
        next = r.second + 1u;
      }
      if (next <= 0x10FFFFu) c.push_back({next, 0x10FFFFu});
      m.swap(c);
    }
    std::vector<std::pair<uint32_t, uint32_t>> out;
    for (const auto& r : m) {
      if (r.first <= 0xDFFFu && r.second >= 0xD800u) {
        if (r.first < 0xD800u) out.push_back({r.first, 0xD7FFu});
        if (r.second > 0xDFFFu) out.push_back({0xE000u, r.second});
      } else {
        out.push_back(r);
      }
    }
    return out;
  }
  bool alternatives(const std::string& rule, bool nested, std::vector<Seq>* out) {
    Seq s;
    if (!sequence(rule, nested, &s)) return false;
    out->push_back(std::move(s));
    while (true) {
      if (p < end && *p == '|') {
        ++p;
        space(true);
        Seq t;
        if (!sequence(rule, nested, &t)) return false;
        out->push_back(std::move(t));
        continue;
      }
      if (!nested && p < end && (*p == '\n' || *p == '\r') && continues()) continue;
      return true;
    }
  }
  bool sequence(const std::string& rule, bool nested, Seq* seq) {
    size_t last = SIZE_MAX;  // first element of the last symbol (for repetition)
    while (true) {
      space(nested);
      if (p >= end || *p == '|' || *p == ')' || *p == '\n' || *p == '\r') return true;
      if (!nested && at_rule_start()) return true;
      const size_t start = seq->size();
      if (*p == '"') {
        ++p;
        while (p < end && *p != '"') {
          uint32_t v;
          if (!cp_of(&v)) return false;
          if (!valid_cp(v)) return fail("a literal's character is not a Unicode scalar value in rule " + rule);
          uint8_t b8[4];
          const int nb = utf8_encode(v, b8);
          for (int i = 0; i < nb; ++i) {
            ByteSet b;
            b.add(b8[i]);
            seq->push_back({kChars, set_of(b)});
          }
        }
        if (p >= end) return fail("unterminated literal in rule " + rule);
        ++p;
        if (seq->size() == start) {  // "": the empty string
          last = SIZE_MAX;
          continue;
        }
      } else if (*p == '[') {
        ++p;
        bool neg = false;
        if (p < end && *p == '^') {
          neg = true;
          ++p;
        }
        std::vector<std::pair<uint32_t, uint32_t>> ranges;
        while (p < end && *p != ']') {
          uint32_t lo;
          if (!cp_of(&lo)) return false;
          uint32_t hi = lo;
          if (p + 1 < end && *p == '-' && p[1] != ']') {
            ++p;
            if (!cp_of(&hi)) return false;
            if (hi < lo) return fail("empty range in a class of rule " + rule);
          }
          if (hi > 0x10FFFFu) return fail("a class range beyond U+10FFFF in rule " + rule);
          ranges.push_back({lo, hi});
        }
        if (p >= end) return fail("unterminated class in rule " + rule);
        ++p;
        if (!char_element(rule, normalize_ranges(std::move(ranges), neg), seq)) return false;
      } else if (*p == '.') {
        ++p;
        if (!char_element(rule, normalize_ranges({{0u, 0x10FFFFu}}, false), seq)) return false;
      } else if (*p == '(') {
        ++p;
        space(true);
        const uint32_t sub = new_rule(rule);
        std::vector<Seq> body;
        if (!alternatives(rule, true, &body)) return false;
        space(true);
        if (p >= end || *p != ')') return fail("missing ')' in rule " + rule);
        ++p;
        bodies[sub] = std::move(body);
        seq->push_back({kRef, sub});
      } else if (name_char(*p)) {
        const std::string n = name();
        seq->push_back({kRef, rule_id(n)});
      } else {
        return fail(std::string("unexpected character '") + *p + "' in rule " + rule);
      }
      last = start;
      // repetition of the symbol just read
      while (p < end && (*p == '*' || *p == '+' || *p == '?' || *p == '{')) {
        if (last == SIZE_MAX) return fail("repetition without an element in rule " + rule);
        int lo = 0, hi = -1;  // hi -1: unbounded
        if (*p == '*') {
          lo = 0;
        } else if (*p == '+') {
          lo = 1;
        } else if (*p == '?') {
          hi = 1;
        } else {
          ++p;
          space(false);
          const char* q = p;
          while (p < end && *p >= '0' && *p <= '9') ++p;
          if (p == q || p - q > 4) return fail("bad {m,n} in rule " + rule);
          lo = std::stoi(std::string(q, p));
          hi = lo;
          space(false);
          if (p < end && *p == ',') {
            ++p;
            space(false);
            q = p;
            while (p < end && *p >= '0' && *p <= '9') ++p;
            hi = (p == q) ? -1 : (p - q > 4 ? kMaxRepeat + 1 : std::stoi(std::string(q, p)));
            space(false);
          }
          if (p >= end || *p != '}') return fail("missing '}' in rule " + rule);
          if (lo > kMaxRepeat || hi > kMaxRepeat || (hi >= 0 && hi < lo)) return fail("bad {m,n} in rule " + rule);
        }
        ++p;
        const Seq x(seq->begin() + static_cast<long>(last), seq->end());
        seq->resize(last);
        // lo copies, then (hi - lo) optional copies or an unbounded tail
        Seq rep;
        for (int i = 0; i < lo; ++i) rep.insert(rep.end(), x.begin(), x.end());
        if (hi < 0) {
          const uint32_t star = new_rule(rule);  // star ::= x star | ""
          Seq a = x;
          a.push_back({kRef, star});
          bodies[star] = {a, Seq()};
          rep.push_back({kRef, star});
        } else if (hi > lo) {
          // nested optional tail: opt_k ::= x opt_{k-1} | ""
          uint32_t inner = UINT32_MAX;
          for (int i = 0; i < hi - lo; ++i) {
            const uint32_t opt = new_rule(rule);
            Seq a = x;
            if (inner != UINT32_MAX) a.push_back({kRef, inner});
            bodies[opt] = {a, Seq()};
            inner = opt;
          }
          rep.push_back({kRef, inner});
        }
        // the repetition becomes one symbol (a rule) so that a further
        // suffix applies to all of it
        const uint32_t r = new_rule(rule);
        bodies[r] = {rep};
        seq->push_back({kRef, r});
      }
    }
  }
  bool parse() {
    while (true) {
      space(true);
      if (p >= end) break;
      const std::string n = name();
      if (n.empty()) return fail(std::string("expected a rule name, found '") + *p + "'");
      space(false);
      if (end - p < 3 || std::strncmp(p, "::=", 3) != 0) return fail("expected '::=' after " + n);
      p += 3;
      space(true);
      const uint32_t id = rule_id(n);
      if (defined[id]) return fail("rule " + n + " defined twice");
      defined[id] = 1;
      std::vector<Seq> body;
      if (!alternatives(n, false, &body)) return false;
      bodies[id] = std::move(body);
    }
    for (size_t i = 0; i < defined.size(); ++i)
      if (!defined[i]) return fail("undefined rule " + g.names[i]);
    return true;
  }
};

// nullable rules (a fixpoint), then a cycle search over "may start with"
bool left_recursive(const Grammar& g, std::string* which) {
  const size_t R = g.alts.size();
  std::vector<char> nullable(R, 0);
  auto alt_nullable = [&](uint32_t a) {
    for (uint32_t e = a;; ++e) {
      const Elem& x = g.elems[e];
      if (x.kind == kEnd) return true;
      if (x.kind == kChars || !nullable[x.arg]) return false;
    }
  };
  for (bool changed = true; changed;) {
    changed = false;
    for (size_t r = 0; r < R; ++r) {
      if (nullable[r]) continue;
      for (uint32_t a : g.alts[r])
        if (alt_nullable(a)) {
          nullable[r] = 1;
          changed = true;
          break;
        }
    }
  }
  std::vector<std::vector<uint32_t>> first(R);
  for (size_t r = 0; r < R; ++r)
    for (uint32_t a : g.alts[r])
      for (uint32_t e = a;; ++e) {
        const Elem& x = g.elems[e];
        if (x.kind != kRef) break;
        first[r].push_back(x.arg);
        if (!nullable[x.arg]) break;
      }
  std::vector<char> color(R, 0);  // 0 new, 1 on the path, 2 done
  std::vector<std::pair<uint32_t, size_t>> st;
  for (size_t r0 = 0; r0 < R; ++r0) {
    if (color[r0]) continue;
    st.push_back({static_cast<uint32_t>(r0), 0});
    color[r0] = 1;
    while (!st.empty()) {
      auto& [r, i] = st.back();
      if (i < first[r].size()) {
        const uint32_t n = first[r][i++];
        if (color[n] == 1) {
          *which = g.names[n];
          return true;
        }
        if (color[n] == 0) {
          color[n] = 1;
          st.push_back({n, 0});
        }
      } else {
        color[r] = 2;
        st.pop_back();
      }
    }
  }
  return false;
}

// ---------------------------------------------------------------------------
// Automaton
// ---------------------------------------------------------------------------
// Pushes s, expanded until a byte class is on top (or s is empty), onto out.
// False when a stack grows beyond kMaxStackDepth or the set beyond kMaxStacks.
bool expand(const Grammar& g, Stack s, StackSet& out) {
  while (true) {
    if (s.empty()) break;
    const uint32_t top = s.back();
    const Elem& e = g.elems[top];
    if (e.kind == kEnd) {
      s.pop_back();
      continue;
    }
    if (e.kind == kChars) break;
    s.pop_back();
    if (g.elems[top + 1].kind != kEnd) s.push_back(top + 1);  // return address (none in tail position)
    if (s.size() >= kMaxStackDepth) return false;
    const auto& alts = g.alts[e.arg];
    for (size_t i = 0; i + 1 < alts.size(); ++i) {
      Stack t = s;
      t.push_back(alts[i]);
      if (!expand(g, std::move(t), out)) return false;
    }
    s.push_back(alts.back());
  }
  if (out.size() >= kMaxStacks) return false;
  out.push_back(std::move(s));
  return true;
}

void normalize(StackSet& s) {
  std::sort(s.begin(), s.end());
  s.erase(std::unique(s.begin(), s.end()), s.end());
}

// The state after byte c (empty: c is not allowed). False on overflow.
bool advance(const Grammar& g, const StackSet& in, int c, StackSet& out) {
  out.clear();
  for (const Stack& s : in) {
    if (s.empty() || !g.sets[g.elems[s.back()].arg].has(c)) continue;
    Stack t = s;
    t.back() += 1;
    if (!expand(g, std::move(t), out)) return false;
  }
  normalize(out);
  return true;
}

bool accepting(const StackSet& s) { return !s.empty() && s.front().empty(); }

}  // namespace gbnf
}  // namespace rl

// The grammar and a cache of finished mask rows by state: a state seen
// before (they recur: the same position inside a string, a value, an array at
// the same depth) is answered by a copy. Bounded (kCacheRows rows, emptied
// when full); guarded by a mutex, so one grammar may serve several threads.
namespace rl {
namespace gbnf {
struct SetHash {
  size_t operator()(const StackSet& s) const {
    uint64_t h = 1469598103934665603ull;
    for (const Stack& st : s) {
      for (uint32_t x : st) h = (h ^ x) * 1099511628211ull;
      h = (h ^ 0xffffffffull) * 1099511628211ull;
    }
    return static_cast<size_t>(h);
  }
};
struct CachedRow {
  std::vector<uint32_t> row;
  int count;
};
constexpr size_t kCacheBytes = 64u << 20;  // rows kept at most: 64 MB of them

// The accept path's lazy automaton: stack sets interned as they are met,
// each (set, byte) transition computed once and kept, so accepting a token
// is a table walk once its bytes have been seen from that state. Bounded
// (kDfaMax sets, about 1 KB of transitions each): when full it is emptied and
// its epoch advances, which tells the states that their ids are stale.
constexpr size_t kDfaMax = 16384;
struct Dfa {
  std::unordered_map<StackSet, int32_t, SetHash> ids;
  std::vector<const StackSet*> sets;  // id -> its set (the map's keys do not move)
  std::vector<int32_t> next;          // [id * 256 + byte]: -2 unknown, -1 refused, else the next id
  uint32_t epoch = 1;
  int32_t intern(const StackSet& st) {
    auto it = ids.find(st);
    if (it != ids.end()) return it->second;
    if (sets.size() >= kDfaMax) {
      ids.clear();
      sets.clear();
      next.clear();
      ++epoch;
    }
    const int32_t id = static_cast<int32_t>(sets.size());
    auto ins = ids.emplace(st, id).first;
    sets.push_back(&ins->first);
    next.resize(next.size() + 256, -2);
    return id;
  }
};
}  // namespace gbnf
}  // namespace rl

struct rl_gbnf {
  rl::gbnf::Grammar g;
  mutable std::mutex mu;
  mutable std::unordered_map<rl::gbnf::StackSet, rl::gbnf::CachedRow, rl::gbnf::SetHash> cache;
  mutable std::mutex dfa_mu;
  mutable rl::gbnf::Dfa dfa;
};
struct rl_gbnf_state {
  rl::gbnf::StackSet set;
  int finished = 0;        // the end-of-sequence token was accepted
  int32_t dfa_id = -1;     // the set's id in the grammar's lazy automaton,
  uint32_t dfa_epoch = 0;  // valid while the automaton's epoch is this one
};

namespace {

using namespace rl::gbnf;

// The states one mask walk meets, interned, with their transitions computed
// once each: within a walk most trie nodes lead to a state already seen
// (inside a JSON string nearly every byte keeps the same state), so the walk
// is table lookups after the first visit.
struct Walk {
  const Grammar& g;
  std::vector<StackSet> sets;
  std::map<StackSet, int32_t> ids;
  std::vector<int32_t> next;  // [state * 256 + byte]: -2 unknown, -1 refused, else the state
  bool ok = true;
  explicit Walk(const Grammar& gr) : g(gr) {}
  int32_t intern(StackSet&& st) {
    auto it = ids.find(st);
    if (it != ids.end()) return it->second;
    const int32_t id = static_cast<int32_t>(sets.size());
    ids.emplace(st, id);
    sets.push_back(std::move(st));
    next.resize(next.size() + 256, -2);
    return id;
  }
  int32_t step(int32_t id, int c) {
    const size_t k = static_cast<size_t>(id) * 256 + static_cast<size_t>(c);
    if (next[k] != -2) return next[k];
    StackSet out;
    if (!advance(g, sets[id], c, out)) {
      ok = false;
      return -1;
    }
    const int32_t n = out.empty() ? -1 : intern(std::move(out));
    next[k] = n;
    return n;
  }
};

// Allowed tokens below trie node n, reached in walk state id.
bool mask_dfs(Walk& w, uint32_t n, int32_t id, uint32_t* row, int* count) {
  const Grammar& g = w.g;
  for (uint32_t k = g.child_begin[n]; k < g.child_begin[n + 1]; ++k) {
    const int32_t nid = w.step(id, g.child_byte[k]);
    if (!w.ok) return false;
    if (nid < 0) continue;
    const uint32_t c = g.child_node[k];
    for (uint32_t t = g.tok_begin[c]; t < g.tok_begin[c + 1]; ++t) {
      const int tid = g.tok_ids[t];
      if (!((row[tid >> 5] >> (tid & 31)) & 1u)) {
        row[tid >> 5] |= 1u << (tid & 31);
        ++*count;
      }
    }
    if (g.child_begin[c + 1] > g.child_begin[c] && !mask_dfs(w, c, nid, row, count)) return false;
  }
  return true;
}

rl_status mask_one(const rl_gbnf* G, const rl_gbnf_state* s, uint32_t* row, int64_t words, int32_t* n_allowed) {
  const Grammar& g = G->g;
  std::fill(row, row + words, 0u);
  int count = 0;
  const int64_t vw = (g.V + 31) / 32;
  if (!s->finished && !s->set.empty()) {
    std::lock_guard<std::mutex> lk(G->mu);
    auto it = G->cache.find(s->set);
    if (it != G->cache.end()) {
      std::copy(it->second.row.begin(), it->second.row.end(), row);
      if (n_allowed) *n_allowed = it->second.count;
      return RL_OK;
    }
  }
  if (!s->finished && !s->set.empty()) {
    Walk w(g);
    StackSet start = s->set;
    const int32_t id0 = w.intern(std::move(start));
    if (!mask_dfs(w, 0, id0, row, &count))
      return rl::set_error(RL_ERR_SHAPE, "rl_gbnf_mask: the grammar's state grew beyond its stack limits");
    if (g.eos >= 0 && accepting(s->set) && !((row[g.eos >> 5] >> (g.eos & 31)) & 1u)) {
      row[g.eos >> 5] |= 1u << (g.eos & 31);
      ++count;
    }
    std::lock_guard<std::mutex> lk(G->mu);
    if ((G->cache.size() + 1) * static_cast<size_t>(vw) * 4u > kCacheBytes) G->cache.clear();
    G->cache[s->set] = CachedRow{std::vector<uint32_t>(row, row + vw), count};
  }
  if (n_allowed) *n_allowed = count;
  return RL_OK;
}

}  // namespace

extern "C" {
#pragma GCC visibility push(default)

rl_status rl_gbnf_create(const char* text, const char* root, int V, const char* const* tokens,
                         const int32_t* token_len, int32_t eos_id, rl_gbnf** out) {
  if (!out) return rl::set_error(RL_ERR_INVALID_ARG, "rl_gbnf_create: out is NULL");
  *out = nullptr;
  if (!text || !root || V <= 0 || !tokens || !token_len)
    return rl::set_error(RL_ERR_INVALID_ARG, "rl_gbnf_create: text, root, tokens and token_len are required, V > 0");
  if (eos_id >= V) return rl::set_error(RL_ERR_INVALID_ARG, "rl_gbnf_create: eos_id >= V");
  try {
    rl_gbnf* G = new rl_gbnf();
    Grammar& g = G->g;
    Parser ps(text, std::strlen(text), g);
    if (!ps.parse()) {
      const std::string m = "rl_gbnf_create: " + ps.err;
      delete G;
      return rl::set_error(RL_ERR_INVALID_ARG, m.c_str());
    }
    auto it = ps.ids.find(root);
    if (it == ps.ids.end()) {
      delete G;
      return rl::set_error(RL_ERR_INVALID_ARG, "rl_gbnf_create: the root rule is not defined");
    }
    g.root = it->second;
    // flatten: every alternative closed by kEnd, so that the successor of a
    // class or reference always exists
    g.alts.resize(ps.bodies.size());
    for (size_t r = 0; r < ps.bodies.size(); ++r)
      for (const Seq& a : ps.bodies[r]) {
        g.alts[r].push_back(static_cast<uint32_t>(g.elems.size()));
        g.elems.insert(g.elems.end(), a.begin(), a.end());
        g.elems.push_back({kEnd, 0});
      }
    std::string lr;
    if (left_recursive(g, &lr)) {
      const std::string m = "rl_gbnf_create: left recursion through rule " + lr;
      delete G;
      return rl::set_error(RL_ERR_UNSUPPORTED, m.c_str());
    }
    // the vocabulary trie
    std::vector<std::map<uint8_t, uint32_t>> kids(1);
    std::vector<std::vector<int32_t>> ends(1);
    for (int t = 0; t < V; ++t) {
      if (t == eos_id || token_len[t] <= 0 || !tokens[t]) continue;  // never matched as bytes
      uint32_t n = 0;
      for (int i = 0; i < token_len[t]; ++i) {
        const uint8_t c = static_cast<uint8_t>(tokens[t][i]);
        auto f = kids[n].find(c);
        if (f == kids[n].end()) {
          const uint32_t m = static_cast<uint32_t>(kids.size());
          kids[n][c] = m;
          kids.emplace_back();
          ends.emplace_back();
          n = m;
        } else {
          n = f->second;
        }
      }
      ends[n].push_back(t);
    }
    const size_t N = kids.size();
    g.child_begin.assign(N + 1, 0);
    g.tok_begin.assign(N + 1, 0);
    for (size_t n = 0; n < N; ++n) {
      g.child_begin[n + 1] = g.child_begin[n] + static_cast<uint32_t>(kids[n].size());
      g.tok_begin[n + 1] = g.tok_begin[n] + static_cast<uint32_t>(ends[n].size());
      for (const auto& kv : kids[n]) {
        g.child_byte.push_back(kv.first);
        g.child_node.push_back(kv.second);
      }
      g.tok_ids.insert(g.tok_ids.end(), ends[n].begin(), ends[n].end());
    }
    g.tb_begin.assign(static_cast<size_t>(V) + 1, 0);
    for (int t = 0; t < V; ++t) {
      const int n = (t == eos_id || !tokens[t] || token_len[t] <= 0) ? 0 : token_len[t];
      g.tb_begin[t + 1] = g.tb_begin[t] + static_cast<uint32_t>(n);
      g.tb.insert(g.tb.end(), reinterpret_cast<const uint8_t*>(tokens[t]),
                  reinterpret_cast<const uint8_t*>(tokens[t]) + n);
    }
    g.V = V;
    g.eos = eos_id;
    *out = G;
    return RL_OK;
  } catch (...) {
    return rl::set_error(RL_ERR_OOM, "rl_gbnf_create: host allocation failed");
  }
}

void rl_gbnf_destroy(rl_gbnf* g) { delete g; }

rl_status rl_gbnf_state_create(const rl_gbnf* G, rl_gbnf_state** out) {
  if (!out) return rl::set_error(RL_ERR_INVALID_ARG, "rl_gbnf_state_create: out is NULL");
  *out = nullptr;
  if (!G) return rl::set_error(RL_ERR_INVALID_ARG, "rl_gbnf_state_create: grammar is NULL");
  try {
    rl_gbnf_state* s = new rl_gbnf_state();
    const Grammar& g = G->g;
    bool ok = true;
    for (uint32_t a : g.alts[g.root]) ok = ok && expand(g, Stack{a}, s->set);
    if (!ok) {
      delete s;
      return rl::set_error(RL_ERR_SHAPE, "rl_gbnf_state_create: the start state grew beyond the stack limits");
    }
    normalize(s->set);
    *out = s;
    return RL_OK;
  } catch (...) {
    return rl::set_error(RL_ERR_OOM, "rl_gbnf_state_create: host allocation failed");
  }
}

void rl_gbnf_state_destroy(rl_gbnf_state* s) { delete s; }

rl_status rl_gbnf_state_copy(const rl_gbnf_state* src, rl_gbnf_state* dst) {
  if (!src || !dst) return rl::set_error(RL_ERR_INVALID_ARG, "rl_gbnf_state_copy: NULL state");
  try {
    *dst = *src;
  } catch (...) {
    return rl::set_error(RL_ERR_OOM, "rl_gbnf_state_copy: host allocation failed");
  }
  return RL_OK;
}

int rl_gbnf_accepting(const rl_gbnf_state* s) { return (s && !s->finished && accepting(s->set)) ? 1 : 0; }

rl_status rl_gbnf_accept(const rl_gbnf* G, rl_gbnf_state* s, int32_t token) {
  if (!G || !s) return rl::set_error(RL_ERR_INVALID_ARG, "rl_gbnf_accept: NULL grammar or state");
  const Grammar& g = G->g;
  if (token < 0 || token >= g.V) return rl::set_error(RL_ERR_INVALID_ARG, "rl_gbnf_accept: token out of range");
  if (s->finished) return rl::set_error(RL_ERR_INVALID_ARG, "rl_gbnf_accept: the sequence already ended");
  try {
    if (token == g.eos) {
      if (!accepting(s->set)) return rl::set_error(RL_ERR_INVALID_ARG, "rl_gbnf_accept: the grammar is not complete");
      s->finished = 1;
      s->set.clear();
      s->dfa_id = -1;
      return RL_OK;
    }
    if (g.tb_begin[token + 1] == g.tb_begin[token])
      return rl::set_error(RL_ERR_INVALID_ARG, "rl_gbnf_accept: the token has no bytes");
    std::lock_guard<std::mutex> lk(G->dfa_mu);
    Dfa& d = G->dfa;
    int32_t id = (s->dfa_epoch == d.epoch && s->dfa_id >= 0) ? s->dfa_id : d.intern(s->set);
    const uint32_t epoch0 = d.epoch;
    for (uint32_t k = g.tb_begin[token]; k < g.tb_begin[token + 1]; ++k) {
      const int c = g.tb[k];
      int32_t n = d.next[static_cast<size_t>(id) * 256 + static_cast<size_t>(c)];
      if (n == -2) {
        StackSet out;
        if (!advance(g, *d.sets[id], c, out))
          return rl::set_error(RL_ERR_SHAPE, "rl_gbnf_accept: the grammar's state grew beyond its stack limits");
        if (out.empty()) {
          n = -1;
        } else {
          n = d.intern(out);
          if (d.epoch != epoch0) {
            // the automaton was emptied to make room: walk this token again
            // from the state's own set, uncached
            StackSet cur = s->set, nx;
            for (uint32_t q = g.tb_begin[token]; q < g.tb_begin[token + 1]; ++q) {
              if (!advance(g, cur, g.tb[q], nx))
                return rl::set_error(RL_ERR_SHAPE, "rl_gbnf_accept: the grammar's state grew beyond its stack limits");
              if (nx.empty())
                return rl::set_error(RL_ERR_INVALID_ARG, "rl_gbnf_accept: the grammar does not allow the token");
              cur.swap(nx);
            }
            s->set.swap(cur);
            s->dfa_id = -1;
            return RL_OK;
          }
        }
        d.next[static_cast<size_t>(id) * 256 + static_cast<size_t>(c)] = n;
      }
      if (n < 0) return rl::set_error(RL_ERR_INVALID_ARG, "rl_gbnf_accept: the grammar does not allow the token");
      id = n;
    }
    s->set = *d.sets[id];
    s->dfa_id = id;
    s->dfa_epoch = d.epoch;
    return RL_OK;
  } catch (...) {
    return rl::set_error(RL_ERR_OOM, "rl_gbnf_accept: host allocation failed");
  }
}

rl_status rl_gbnf_accept_batch(const rl_gbnf* G, rl_gbnf_state* const* states, const int32_t* tokens, int B,
                               int32_t* row_status, int nthreads) {
  if (!G || (B > 0 && (!states || !tokens))) return rl::set_error(RL_ERR_INVALID_ARG, "rl_gbnf_accept_batch: NULL argument");
  if (B < 0) return rl::set_error(RL_ERR_INVALID_ARG, "rl_gbnf_accept_batch: B < 0");
  std::vector<rl_status> st(static_cast<size_t>(B), RL_OK);
  // a few microseconds a row, under the lazy automaton's lock: threads only
  // pay for large batches (measured slower than one thread at 64 rows)
  nthreads = std::max(1, std::min(nthreads, B / 256));
  auto run = [&](int b0, int b1) {
    for (int b = b0; b < b1; ++b) st[b] = rl_gbnf_accept(G, states[b], tokens[b]);
  };
  if (nthreads == 1) {
    run(0, B);
  } else {
    std::vector<std::thread> ts;
    for (int t = 0; t < nthreads; ++t) ts.emplace_back(run, B * t / nthreads, B * (t + 1) / nthreads);
    for (auto& t : ts) t.join();
  }
  rl_status first = RL_OK;
  for (int b = 0; b < B; ++b) {
    if (row_status) row_status[b] = st[b];
    if (first == RL_OK) first = st[b];
  }
  if (first != RL_OK) return rl::set_error(first, "rl_gbnf_accept_batch: a row's token was refused (see row_status)");
  return RL_OK;
}

rl_status rl_gbnf_mask(const rl_gbnf* G, const rl_gbnf_state* s, uint32_t* mask_row, int64_t words,
                       int32_t* n_allowed) {
  if (!G || !s || !mask_row) return rl::set_error(RL_ERR_INVALID_ARG, "rl_gbnf_mask: NULL argument");
  if (words < (G->g.V + 31) / 32) return rl::set_error(RL_ERR_INVALID_ARG, "rl_gbnf_mask: words < ceil(V/32)");
  try {
    return mask_one(G, s, mask_row, words, n_allowed);
  } catch (...) {
    return rl::set_error(RL_ERR_OOM, "rl_gbnf_mask: host allocation failed");
  }
}

rl_status rl_gbnf_mask_batch(const rl_gbnf* G, const rl_gbnf_state* const* states, int B, uint32_t* mask,
                             int64_t mask_stride, int32_t* n_allowed, int nthreads) {
  if (!G || (B > 0 && (!states || !mask))) return rl::set_error(RL_ERR_INVALID_ARG, "rl_gbnf_mask_batch: NULL argument");
  if (B < 0) return rl::set_error(RL_ERR_INVALID_ARG, "rl_gbnf_mask_batch: B < 0");
  if (mask_stride < (G->g.V + 31) / 32)
    return rl::set_error(RL_ERR_INVALID_ARG, "rl_gbnf_mask_batch: mask_stride < ceil(V/32)");
  for (int b = 0; b < B; ++b)
    if (!states[b]) return rl::set_error(RL_ERR_INVALID_ARG, "rl_gbnf_mask_batch: NULL state");
  // rows whose state is cached are copied here; the others are walked, on
  // up to nthreads threads when there are several
  std::vector<rl_status> st(static_cast<size_t>(B), RL_OK);
  std::vector<int> miss;
  {
    const Grammar& g = G->g;
    const int64_t vw = (g.V + 31) / 32;
    std::lock_guard<std::mutex> lk(G->mu);
    for (int b = 0; b < B; ++b) {
      uint32_t* row = mask + static_cast<int64_t>(b) * mask_stride;
      const rl_gbnf_state* s = states[b];
      if (s->finished || s->set.empty()) {
        std::fill(row, row + mask_stride, 0u);
        if (n_allowed) n_allowed[b] = 0;
        continue;
      }
      auto it = G->cache.find(s->set);
      if (it == G->cache.end()) {
        miss.push_back(b);
        continue;
      }
      std::copy(it->second.row.begin(), it->second.row.end(), row);
      std::fill(row + vw, row + mask_stride, 0u);
      if (n_allowed) n_allowed[b] = it->second.count;
    }
  }
  const int M = static_cast<int>(miss.size());
  nthreads = std::max(1, std::min(nthreads, M));
  auto run = [&](int i0, int i1) {
    for (int i = i0; i < i1; ++i) {
      const int b = miss[i];
      try {
        st[b] = mask_one(G, states[b], mask + static_cast<int64_t>(b) * mask_stride, mask_stride,
                         n_allowed ? n_allowed + b : nullptr);
      } catch (...) {
        st[b] = RL_ERR_OOM;
      }
    }
  };
  if (nthreads == 1) {
    run(0, M);
  } else {
    std::vector<std::thread> ts;
    for (int t = 0; t < nthreads; ++t) ts.emplace_back(run, M * t / nthreads, M * (t + 1) / nthreads);
    for (auto& t : ts) t.join();
  }
  for (int b = 0; b < B; ++b)
    if (st[b] != RL_OK) return rl::set_error(st[b], "rl_gbnf_mask_batch: a row's mask failed");
  return RL_OK;
}

#pragma GCC visibility pop
}  // extern "C"
