// Constrained decoding: allowed-token masks for JSON and regular-expression outputs (host C++).
//
// A byte trie over the vocabulary's token strings is built once per tokenizer. A matcher holds the
// parse state of one sequence's output so far; mask() walks the trie depth-first from that state,
// stepping the matcher byte by byte on copies and pruning every prefix that kills it, so the cost
// follows the live prefixes, not the vocabulary size. Masks are cached per matcher state (JSON
// output revisits the same few states, e.g. "inside a string", all the time).
//
//   JsonMatcher   RFC 8259 JSON as a pushdown automaton (object/array stack, string escapes, number
//                 grammar, true/false/null), whitespace between tokens; optionally the top-level
//                 value must be an object (OpenAI json_object mode).
//   RegexMatcher  full-match regular expression: literals, escapes (\d \w \s \. ...), classes
//                 [a-z] [^...], ., groups, |, * + ? {m} {m,} {m,n}; Thompson NFA simulated as a set
//                 of states.
//
// The reference exposes grammar-constrained sampling through llama.cpp's sampler chain
// (runner/llamacpp/gollek-runner-llamacpp/…/LlamaHandles.java:174-203) and structured output in its
// safetensors plugin; the automata here are written from the JSON grammar and the textbook
// Thompson construction.
#include <torch/extension.h>

#include <algorithm>
#include <array>
#include <cctype>
#include <cstdint>
#include <list>
#include <memory>
#include <stdexcept>
#include <string>
#include <unordered_map>
#include <vector>

namespace {

// ------------------------------------------------------------------------------------- trie
struct Trie {
  struct Node {
    std::vector<std::pair<uint8_t, int>> kids;  // sorted by byte
    std::vector<int32_t> tokens;                // tokens whose bytes end here
  };
  std::vector<Node> nodes;
  int vocab = 0;

  explicit Trie(const std::vector<std::string>& toks) : vocab((int)toks.size()) {
    nodes.emplace_back();
    for (int t = 0; t < (int)toks.size(); ++t) {
      const std::string& s = toks[t];
      if (s.empty()) continue;  // special / unmapped tokens are never allowed by a matcher
      int n = 0;
      for (unsigned char c : s) {
        auto& k = nodes[n].kids;
        auto it = std::lower_bound(k.begin(), k.end(), std::make_pair(c, -1));
        if (it != k.end() && it->first == c) {
          n = it->second;
        } else {
          const int id = (int)nodes.size();
          k.insert(it, {c, id});
          nodes.emplace_back();
          n = id;
        }
      }
      nodes[n].tokens.push_back(t);
    }
  }
};

// ------------------------------------------------------------------------------------- JSON
struct JsonState {
  enum Mode : uint8_t {
    VALUE, OBJ_FIRST, OBJ_KEY, COLON, OBJ_NEXT, ARR_FIRST, ARR_NEXT, STR, STR_ESC, STR_U,
    NUM_MINUS, NUM_ZERO, NUM_INT, NUM_DOT, NUM_FRAC, NUM_E, NUM_ESIGN, NUM_EXP, LIT, DONE, DEAD
  };
  std::array<uint8_t, 64> stack{};  // 'o' object, 'a' array (nesting limit 64)
  uint8_t depth = 0;
  uint8_t mode = VALUE;
  uint8_t str_is_key = 0;
  uint8_t u_left = 0;          // hex digits left in \uXXXX
  uint8_t lit = 0, lit_pos = 0;
  uint8_t top_object = 0;      // top-level value must be an object

  bool empty() const { return depth == 0; }
  uint8_t back() const { return stack[depth - 1]; }
  bool push(uint8_t c) {
    if (depth >= stack.size()) return false;
    stack[depth++] = c;
    return true;
  }
  void pop() { --depth; }

  std::string key() const {
    std::string k(stack.begin(), stack.begin() + depth);
    k.push_back('|');
    k.push_back((char)mode);
    k.push_back((char)str_is_key);
    k.push_back((char)u_left);
    k.push_back((char)lit);
    k.push_back((char)lit_pos);
    k.push_back((char)top_object);
    return k;
  }
};

const char* kLits[3] = {"true", "false", "null"};

bool is_ws(unsigned char c) { return c == ' ' || c == '\t' || c == '\n' || c == '\r'; }

struct JsonMachine {
  // after a complete value: where the parser continues
  static void value_done(JsonState& s) {
    if (s.empty()) {
      s.mode = JsonState::DONE;
    } else {
      s.mode = s.back() == 'o' ? JsonState::OBJ_NEXT : JsonState::ARR_NEXT;
    }
  }

  static bool start_value(JsonState& s, unsigned char c) {
    const bool top = s.empty();
    if (top && s.top_object && c != '{') return false;
    switch (c) {
      case '{': s.mode = JsonState::OBJ_FIRST; return s.push('o');
      case '[': s.mode = JsonState::ARR_FIRST; return s.push('a');
      case '"': s.mode = JsonState::STR; s.str_is_key = 0; return true;
      case '-': s.mode = JsonState::NUM_MINUS; return true;
      case '0': s.mode = JsonState::NUM_ZERO; return true;
      case 't': s.mode = JsonState::LIT; s.lit = 0; s.lit_pos = 1; return true;
      case 'f': s.mode = JsonState::LIT; s.lit = 1; s.lit_pos = 1; return true;
      case 'n': s.mode = JsonState::LIT; s.lit = 2; s.lit_pos = 1; return true;
      default:
        if (c >= '1' && c <= '9') { s.mode = JsonState::NUM_INT; return true; }
        return false;
    }
  }

  static bool close(JsonState& s, char want) {
    if (s.empty() || s.back() != want) return false;
    s.pop();
    value_done(s);
    return true;
  }

  static bool step(JsonState& s, unsigned char c) {
    using M = JsonState;
    for (int guard = 0; guard < 2; ++guard) {  // a number ends on the next byte, which is re-read
      switch (s.mode) {
        case M::VALUE:
          if (is_ws(c)) return true;
          return start_value(s, c);
        case M::OBJ_FIRST:
          if (is_ws(c)) return true;
          if (c == '}') return close(s, 'o');
          if (c == '"') { s.mode = M::STR; s.str_is_key = 1; return true; }
          return false;
        case M::OBJ_KEY:
          if (is_ws(c)) return true;
          if (c == '"') { s.mode = M::STR; s.str_is_key = 1; return true; }
          return false;
        case M::COLON:
          if (is_ws(c)) return true;
          if (c == ':') { s.mode = M::VALUE; return true; }
          return false;
        case M::OBJ_NEXT:
          if (is_ws(c)) return true;
          if (c == ',') { s.mode = M::OBJ_KEY; return true; }
          if (c == '}') return close(s, 'o');
          return false;
        case M::ARR_FIRST:
          if (is_ws(c)) return true;
          if (c == ']') return close(s, 'a');
          return start_value(s, c);
        case M::ARR_NEXT:
          if (is_ws(c)) return true;
          if (c == ',') { s.mode = M::VALUE; return true; }
          if (c == ']') return close(s, 'a');
          return false;
        case M::STR:
          if (c == '"') {
            if (s.str_is_key) { s.mode = M::COLON; s.str_is_key = 0; } else { value_done(s); }
            return true;
          }
          if (c == '\\') { s.mode = M::STR_ESC; return true; }
          return c >= 0x20;  // control characters must be escaped; UTF-8 bytes pass through
        case M::STR_ESC:
          if (c == 'u') { s.mode = M::STR_U; s.u_left = 4; return true; }
          if (c == '"' || c == '\\' || c == '/' || c == 'b' || c == 'f' || c == 'n' || c == 'r' || c == 't') {
            s.mode = M::STR;
            return true;
          }
          return false;
        case M::STR_U:
          if (isxdigit(c)) {
            if (--s.u_left == 0) s.mode = M::STR;
            return true;
          }
          return false;
        case M::NUM_MINUS:
          if (c == '0') { s.mode = M::NUM_ZERO; return true; }
          if (c >= '1' && c <= '9') { s.mode = M::NUM_INT; return true; }
          return false;
        case M::NUM_ZERO:
          if (c == '.') { s.mode = M::NUM_DOT; return true; }
          if (c == 'e' || c == 'E') { s.mode = M::NUM_E; return true; }
          value_done(s);
          continue;  // the number ended: read c in the enclosing state
        case M::NUM_INT:
          if (c >= '0' && c <= '9') return true;
          if (c == '.') { s.mode = M::NUM_DOT; return true; }
          if (c == 'e' || c == 'E') { s.mode = M::NUM_E; return true; }
          value_done(s);
          continue;
        case M::NUM_DOT:
          if (c >= '0' && c <= '9') { s.mode = M::NUM_FRAC; return true; }
          return false;
        case M::NUM_FRAC:
          if (c >= '0' && c <= '9') return true;
          if (c == 'e' || c == 'E') { s.mode = M::NUM_E; return true; }
          value_done(s);
          continue;
        case M::NUM_E:
          if (c == '+' || c == '-') { s.mode = M::NUM_ESIGN; return true; }
          if (c >= '0' && c <= '9') { s.mode = M::NUM_EXP; return true; }
          return false;
        case M::NUM_ESIGN:
          if (c >= '0' && c <= '9') { s.mode = M::NUM_EXP; return true; }
          return false;
        case M::NUM_EXP:
          if (c >= '0' && c <= '9') return true;
          value_done(s);
          continue;
        case M::LIT: {
          const char* l = kLits[s.lit];
          if ((unsigned char)l[s.lit_pos] != c) return false;
          if (l[++s.lit_pos] == 0) value_done(s);
          return true;
        }
        case M::DONE:
          return is_ws(c);
        default:
          return false;
      }
    }
    return false;
  }

  static bool accepting(const JsonState& s) {
    using M = JsonState;
    if (s.mode == M::DONE) return true;
    // a top-level number is complete at end of input
    return s.empty() && !s.top_object &&
           (s.mode == M::NUM_ZERO || s.mode == M::NUM_INT || s.mode == M::NUM_FRAC || s.mode == M::NUM_EXP);
  }
};

// ------------------------------------------------------------------------------------- regex
struct Nfa {
  struct St {
    int kind;                   // 0 = byte set, 1 = split (epsilon to out, out2), 2 = match
    std::vector<uint64_t> set;  // 256-bit byte set (kind 0)
    int out = -1, out2 = -1;
  };
  std::vector<St> st;
  int start = -1;

  int add(int kind) {
    st.push_back({kind, std::vector<uint64_t>(kind == 0 ? 4 : 0, 0), -1, -1});
    return (int)st.size() - 1;
  }
};

struct Frag {
  int start;
  std::vector<int*> outs;  // dangling exits (indices resolved through pointers into st vector)
};

class RegexCompiler {
 public:
  explicit RegexCompiler(const std::string& p) : p_(p) {}

  Nfa compile() {
    // fragments store exits as (state, which) pairs to survive vector growth
    auto f = parse_alt();
    if (i_ != p_.size()) throw std::invalid_argument("regex: unexpected '" + std::string(1, p_[i_]) + "'");
    const int m = nfa_.add(2);
    patch(f.second, m);
    nfa_.start = f.first;
    return nfa_;
  }

 private:
  using Exits = std::vector<std::pair<int, int>>;  // (state, 0 = out, 1 = out2)
  using F = std::pair<int, Exits>;

  void patch(const Exits& e, int to) {
    for (auto& x : e) (x.second ? nfa_.st[x.first].out2 : nfa_.st[x.first].out) = to;
  }

  F parse_alt() {
    F a = parse_seq();
    while (i_ < p_.size() && p_[i_] == '|') {
      ++i_;
      F b = parse_seq();
      const int s = nfa_.add(1);
      nfa_.st[s].out = a.first;
      nfa_.st[s].out2 = b.first;
      Exits e = a.second;
      e.insert(e.end(), b.second.begin(), b.second.end());
      a = {s, e};
    }
    return a;
  }

  F empty_frag() {
    const int s = nfa_.add(1);  // epsilon with one dangling exit
    nfa_.st[s].out2 = -2;       // unused branch
    return {s, {{s, 0}}};
  }

  F parse_seq() {
    if (i_ >= p_.size() || p_[i_] == '|' || p_[i_] == ')') return empty_frag();
    F acc = parse_repeat();
    while (i_ < p_.size() && p_[i_] != '|' && p_[i_] != ')') {
      F nxt = parse_repeat();
      patch(acc.second, nxt.first);
      acc.second = nxt.second;
    }
    return acc;
  }

  // Builds a fresh copy of an atom (its text range is re-parsed), for {m,n} expansion.
  F atom_at(size_t pos) {
    const size_t save = i_;
    i_ = pos;
    F f = parse_atom();
    i_ = save;
    return f;
  }

  F star(F a) {
    const int s = nfa_.add(1);
    nfa_.st[s].out = a.first;
    patch(a.second, s);
    return {s, {{s, 1}}};
  }

  F plus(F a) {
    const int s = nfa_.add(1);
    nfa_.st[s].out = a.first;
    patch(a.second, s);
    return {a.first, {{s, 1}}};
  }

  F quest(F a) {
    const int s = nfa_.add(1);
    nfa_.st[s].out = a.first;
    Exits e = a.second;
    e.push_back({s, 1});
    return {s, e};
  }

  F concat(F a, F b) {
    patch(a.second, b.first);
    return {a.first, b.second};
  }

  F parse_repeat() {
    const size_t atom_pos = i_;
    F a = parse_atom();
    while (i_ < p_.size()) {
      const char c = p_[i_];
      if (c == '*') { ++i_; a = star(a); }
      else if (c == '+') { ++i_; a = plus(a); }
      else if (c == '?') { ++i_; a = quest(a); }
      else if (c == '{') {
        size_t j = i_ + 1;
        auto num = [&](int& v) {
          const size_t s0 = j;
          v = 0;
          while (j < p_.size() && isdigit((unsigned char)p_[j])) v = v * 10 + (p_[j++] - '0');
          return j > s0;
        };
        int m = 0, n = 0;
        if (!num(m)) break;  // a literal '{'
        bool unbounded = false;
        if (j < p_.size() && p_[j] == ',') {
          ++j;
          if (!num(n)) unbounded = true;
        } else {
          n = m;
        }
        if (j >= p_.size() || p_[j] != '}') throw std::invalid_argument("regex: bad {m,n}");
        i_ = j + 1;
        if (m > 64 || (!unbounded && (n < m || n > 64))) throw std::invalid_argument("regex: repeat count > 64");
        // a{m,n} = a ... a (m times) then (n - m) optional copies, or a* when unbounded
        F out = m > 0 ? a : empty_frag();
        for (int k = 1; k < m; ++k) out = concat(out, atom_at(atom_pos));
        if (unbounded) {
          out = m > 0 ? concat(out, star(atom_at(atom_pos))) : star(a);
        } else {
          for (int k = m; k < n; ++k) out = concat(out, quest(k == 0 && m == 0 ? a : atom_at(atom_pos)));
        }
        a = out;
      } else {
        break;
      }
    }
    return a;
  }

  void set_bit(std::vector<uint64_t>& s, unsigned c) { s[c >> 6] |= 1ull << (c & 63); }

  void add_class_escape(std::vector<uint64_t>& s, char e) {
    auto range = [&](int a, int b) { for (int c = a; c <= b; ++c) set_bit(s, (unsigned)c); };
    switch (e) {
      case 'd': range('0', '9'); break;
      case 'w': range('0', '9'); range('a', 'z'); range('A', 'Z'); set_bit(s, '_'); break;
      case 's': for (char c : std::string(" \t\n\r\f\v")) set_bit(s, (unsigned char)c); break;
      case 'n': set_bit(s, '\n'); break;
      case 't': set_bit(s, '\t'); break;
      case 'r': set_bit(s, '\r'); break;
      default: set_bit(s, (unsigned char)e);
    }
  }

  F byte_set(const std::vector<uint64_t>& set) {
    const int s = nfa_.add(0);
    nfa_.st[s].set = set;
    return {s, {{s, 0}}};
  }

  F parse_atom() {
    if (i_ >= p_.size()) throw std::invalid_argument("regex: unexpected end");
    const char c = p_[i_++];
    std::vector<uint64_t> set(4, 0);
    if (c == '(') {
      if (i_ + 1 < p_.size() && p_[i_] == '?' && p_[i_ + 1] == ':') i_ += 2;  // non-capturing group
      F f = parse_alt();
      if (i_ >= p_.size() || p_[i_] != ')') throw std::invalid_argument("regex: missing ')'");
      ++i_;
      return f;
    }
    if (c == '.') {
      for (int b = 0; b < 256; ++b)
        if (b != '\n') set_bit(set, (unsigned)b);
      return byte_set(set);
    }
    if (c == '\\') {
      if (i_ >= p_.size()) throw std::invalid_argument("regex: dangling escape");
      const char e = p_[i_++];
      if (e == 'D' || e == 'W' || e == 'S') {
        std::vector<uint64_t> pos(4, 0);
        add_class_escape(pos, (char)tolower(e));
        for (int k = 0; k < 4; ++k) set[k] = ~pos[k];
      } else {
        add_class_escape(set, e);
      }
      return byte_set(set);
    }
    if (c == '[') {
      bool neg = false;
      if (i_ < p_.size() && p_[i_] == '^') { neg = true; ++i_; }
      bool first = true;
      while (i_ < p_.size() && (p_[i_] != ']' || first)) {
        first = false;
        unsigned char a = (unsigned char)p_[i_++];
        if (a == '\\' && i_ < p_.size()) {
          add_class_escape(set, p_[i_++]);
          continue;
        }
        if (i_ + 1 < p_.size() && p_[i_] == '-' && p_[i_ + 1] != ']') {
          unsigned char b = (unsigned char)p_[i_ + 1];
          i_ += 2;
          for (unsigned x = a; x <= b; ++x) set_bit(set, x);
        } else {
          set_bit(set, a);
        }
      }
      if (i_ >= p_.size()) throw std::invalid_argument("regex: missing ']'");
      ++i_;
      if (neg)
        for (int k = 0; k < 4; ++k) set[k] = ~set[k];
      return byte_set(set);
    }
    if (c == '*' || c == '+' || c == '?' || c == ')' || c == '|')
      throw std::invalid_argument(std::string("regex: misplaced '") + c + "'");
    set_bit(set, (unsigned char)c);
    return byte_set(set);
  }

  std::string p_;
  size_t i_ = 0;
  Nfa nfa_;
};

struct RegexState {
  std::vector<uint64_t> on;  // bitset over NFA states
  std::string key() const { return std::string(reinterpret_cast<const char*>(on.data()), on.size() * 8); }
};

// ------------------------------------------------------------------------------------- matchers
// Depth-first trie walk on value copies of a concrete matcher (no allocation per edge for JSON).
template <class M>
void walk_trie(const Trie& trie, int node, const M& m, bool* out) {
  for (const auto& kv : trie.nodes[node].kids) {
    M c = m;
    if (!c.step(kv.first)) continue;
    for (int32_t t : trie.nodes[kv.second].tokens) out[t] = true;
    walk_trie(trie, kv.second, c, out);
  }
}

class Matcher {
 public:
  virtual ~Matcher() = default;
  virtual std::unique_ptr<Matcher> clone() const = 0;
  virtual bool step(unsigned char c) = 0;
  virtual bool accepting() const = 0;
  virtual std::string key() const = 0;
  virtual void mask_into(const Trie& trie, bool* out) const = 0;
};

class JsonMatcher : public Matcher {
 public:
  explicit JsonMatcher(bool top_object) { s_.top_object = top_object ? 1 : 0; }
  std::unique_ptr<Matcher> clone() const override { return std::make_unique<JsonMatcher>(*this); }
  bool step(unsigned char c) override { return JsonMachine::step(s_, c); }
  bool accepting() const override { return JsonMachine::accepting(s_); }
  std::string key() const override { return "j" + s_.key(); }
  void mask_into(const Trie& trie, bool* out) const override { walk_trie(trie, 0, *this, out); }

 private:
  JsonState s_;
};

class RegexMatcher : public Matcher {
 public:
  // id: the pattern's number in its compiler; part of the mask-cache key, since NFA state sets of
  // different patterns are not comparable.
  RegexMatcher(std::shared_ptr<const Nfa> nfa, uint64_t id) : nfa_(std::move(nfa)), id_(id) {
    s_.on.assign((nfa_->st.size() + 63) / 64, 0);
    add(s_, nfa_->start);
  }
  std::unique_ptr<Matcher> clone() const override { return std::make_unique<RegexMatcher>(*this); }

  bool step(unsigned char c) override {
    RegexState nx;
    nx.on.assign(s_.on.size(), 0);
    bool any = false;
    for (size_t w = 0; w < s_.on.size(); ++w) {
      uint64_t bits = s_.on[w];
      while (bits) {
        const int k = (int)(w * 64 + __builtin_ctzll(bits));
        bits &= bits - 1;
        const auto& st = nfa_->st[k];
        if (st.kind == 0 && ((st.set[c >> 6] >> (c & 63)) & 1)) {
          add(nx, st.out);
          any = true;
        }
      }
    }
    s_ = std::move(nx);
    return any;
  }

  bool accepting() const override {
    for (size_t k = 0; k < nfa_->st.size(); ++k)
      if (nfa_->st[k].kind == 2 && ((s_.on[k >> 6] >> (k & 63)) & 1)) return true;
    return false;
  }
  std::string key() const override {
    return "r" + std::string(reinterpret_cast<const char*>(&id_), sizeof(id_)) + s_.key();
  }
  void mask_into(const Trie& trie, bool* out) const override { walk_trie(trie, 0, *this, out); }

 private:
  void add(RegexState& s, int k) const {  // epsilon closure
    if (k < 0 || ((s.on[k >> 6] >> (k & 63)) & 1)) return;
    s.on[k >> 6] |= 1ull << (k & 63);
    const auto& st = nfa_->st[k];
    if (st.kind == 1) {
      add(s, st.out);
      add(s, st.out2);
    }
  }
  std::shared_ptr<const Nfa> nfa_;
  uint64_t id_;
  RegexState s_;
};

// ------------------------------------------------------------------------------------- compiler
class GrammarCompiler {
 public:
  GrammarCompiler(const std::vector<std::string>& token_bytes, int64_t eos) : trie_(token_bytes), eos_(eos) {}

  int vocab() const { return trie_.vocab; }

  // Allowed-token mask for a matcher state (EOS allowed exactly when the output can end here).
  torch::Tensor mask(const Matcher& m) {
    const std::string k = m.key();
    auto it = cache_.find(k);
    if (it != cache_.end()) {
      lru_.splice(lru_.begin(), lru_, it->second.second);
      return it->second.first;
    }
    auto out = torch::zeros({trie_.vocab}, torch::dtype(torch::kBool));
    bool* o = out.data_ptr<bool>();
    {
      pybind11::gil_scoped_release release;
      m.mask_into(trie_, o);
      if (eos_ >= 0 && eos_ < trie_.vocab) o[eos_] = m.accepting();
    }
    lru_.push_front(k);
    cache_[k] = {out, lru_.begin()};
    if (cache_.size() > kCache) {
      cache_.erase(lru_.back());
      lru_.pop_back();
    }
    return out;
  }

  // Compiled NFA and id of a pattern (one per distinct pattern, reused by later requests).
  std::pair<std::shared_ptr<const Nfa>, uint64_t> regex(const std::string& pattern) {
    auto it = patterns_.find(pattern);
    if (it != patterns_.end()) return it->second;
    auto nfa = std::make_shared<const Nfa>(RegexCompiler(pattern).compile());
    if (patterns_.size() >= kPatterns) patterns_.clear();  // ids stay unique: the counter keeps going
    auto v = std::make_pair(nfa, next_id_++);
    patterns_[pattern] = v;
    return v;
  }

  bool advance(Matcher& m, int64_t token, const std::vector<std::string>& token_bytes) const {
    if (token == eos_) return m.accepting();
    if (token < 0 || token >= (int64_t)token_bytes.size()) return false;
    for (unsigned char c : token_bytes[token])
      if (!m.step(c)) return false;
    return !token_bytes[token].empty();
  }

 private:
  static constexpr size_t kCache = 4096;
  static constexpr size_t kPatterns = 256;
  Trie trie_;
  uint64_t next_id_ = 0;
  std::unordered_map<std::string, std::pair<std::shared_ptr<const Nfa>, uint64_t>> patterns_;
  int64_t eos_;
  std::list<std::string> lru_;
  std::unordered_map<std::string, std::pair<torch::Tensor, std::list<std::string>::iterator>> cache_;
};

struct PyCompiler {
  std::shared_ptr<GrammarCompiler> g;
  std::shared_ptr<std::vector<std::string>> bytes;  // shared by every matcher of this vocabulary
};

struct PyMatcher {
  std::shared_ptr<GrammarCompiler> g;
  std::shared_ptr<std::vector<std::string>> bytes;
  std::unique_ptr<Matcher> m;
  bool dead = false;
};

}  // namespace

void register_grammar(pybind11::module& m) {
  namespace py = pybind11;
  py::class_<PyMatcher>(m, "GrammarMatcher")
      .def("mask", [](PyMatcher& s) {
        if (s.dead) throw std::runtime_error("grammar matcher is dead (a disallowed token was accepted)");
        return s.g->mask(*s.m);
      })
      .def("advance", [](PyMatcher& s, int64_t tok) {
        if (s.dead) return false;
        const bool ok = s.g->advance(*s.m, tok, *s.bytes);
        if (!ok) s.dead = true;
        return ok;
      })
      .def("accepting", [](PyMatcher& s) { return !s.dead && s.m->accepting(); })
      .def("clone", [](PyMatcher& s) {
        PyMatcher c{s.g, s.bytes, s.m->clone(), s.dead};
        return c;
      });
  py::class_<PyCompiler>(m, "GrammarCompiler")
      .def(py::init([](std::vector<py::bytes> toks, int64_t eos) {
             std::vector<std::string> b;
             b.reserve(toks.size());
             for (auto& t : toks) b.push_back(std::string(t));
             PyCompiler c;
             c.g = std::make_shared<GrammarCompiler>(b, eos);
             c.bytes = std::make_shared<std::vector<std::string>>(std::move(b));
             return c;
           }),
           py::arg("token_bytes"), py::arg("eos_token_id"))
      .def("vocab_size", [](PyCompiler& c) { return c.g->vocab(); })
      .def("json", [](PyCompiler& c, bool top_object) {
             return PyMatcher{c.g, c.bytes, std::make_unique<JsonMatcher>(top_object)};
           }, py::arg("top_object") = true)
      .def("regex", [](PyCompiler& c, const std::string& pattern) {
        auto nfa = c.g->regex(pattern);
        return PyMatcher{c.g, c.bytes, std::make_unique<RegexMatcher>(nfa.first, nfa.second)};
      });
}
