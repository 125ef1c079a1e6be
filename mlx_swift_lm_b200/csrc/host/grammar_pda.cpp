// Context-free grammar engine for constrained decoding: EBNF rules compiled to
// per-rule automata and matched by a pushdown automaton with a set of stacks.
//
// The reference vendors xgrammar (Libraries/MLXCXGrammar: EBNF front end,
// Earley parser, per-state token-mask cache, matcher with rollback and
// jump-forward). This engine covers the same job for grammars without left
// recursion, with unbounded nesting (recursive JSON schemas, EBNF):
//   * grammar text: `name ::= body` rules; bodies use "literals" (with \n \t
//     \r \\ \" \xHH \uXXXX escapes), byte classes [a-z_\-] / [^...], `.`
//     (any byte), rule names, ( ), |, and the quantifiers * + ? {m} {m,}
//     {m,n}; `#` starts a comment. Classes and `.` work on bytes: a
//     multi-byte UTF-8 character in a class admits the bytes 0x80-0xFF;
//   * every rule body is a Thompson NFA whose consuming edges are a byte
//     class or a call of another rule, determinised per rule (subset
//     construction over bytes and rule symbols);
//   * matcher state: the set of parse stacks (frames (rule, state) hash-consed
//     in an arena, so equal stacks are one node) closed under calls (push the
//     callee's start with the caller's return state beneath) and returns (an
//     accepting frame pops to its caller); a byte advances every stack whose
//     top has an edge for it;
//   * token masks: per (rule, state) a trie walk classifies every token as
//     consumed inside the rule (allowed whatever the stack holds), rejected
//     inside the rule, or undecided below a trie node (the walk met a call or
//     a possible return); these classes live in the compiled grammar, shared
//     by every request using it. A step's mask is the union of its tops'
//     allowed sets plus a trie walk of the undecided subtrees carrying the
//     whole stack set (stack sets interned, byte transitions between them
//     memoised), cached per stack set; EOS is allowed where the root rule
//     can end;
//   * calls in tail position (the return state only accepts) push no return
//     frame, so right-recursive rules (free text up to a trigger, lists
//     written as `x ::= item x | ""`) keep a constant stack depth;
//   * rollback by history of stack sets, forced prefix (jump-forward) while a
//     single byte is possible.
// Left recursion (a rule reaching a call of itself without consuming input)
// makes the closure grow without bound; it is refused with an error.
#include <pybind11/numpy.h>
#include <pybind11/pybind11.h>
#include <pybind11/stl.h>

#include <algorithm>
#include <array>
#include <bitset>
#include <cstdint>
#include <functional>
#include <map>
#include <memory>
#include <stdexcept>
#include <string>
#include <unordered_map>
#include <vector>

#include "grammar_vocab.h"

namespace py = pybind11;

namespace b200host {
namespace cfg {

// ------------------------------------------------------------------ EBNF AST
struct Ast {
  enum Kind { kBytes, kRule, kSeq, kAlt, kRepeat } kind;
  std::bitset<256> cls;          // kBytes
  std::string name;              // kRule (resolved to an index after parsing)
  int rule = -1;
  std::vector<std::unique_ptr<Ast>> kids;  // kSeq / kAlt / kRepeat (one kid)
  int lo = 0, hi = -1;           // kRepeat: hi < 0 = unbounded
};
using AstP = std::unique_ptr<Ast>;

static AstP mk(Ast::Kind k) {
  auto a = std::make_unique<Ast>();
  a->kind = k;
  return a;
}

static void utf8(uint32_t cp, std::string& out) {
  if (cp < 0x80) {
    out.push_back((char)cp);
  } else if (cp < 0x800) {
    out.push_back((char)(0xC0 | (cp >> 6)));
    out.push_back((char)(0x80 | (cp & 0x3F)));
  } else if (cp < 0x10000) {
    out.push_back((char)(0xE0 | (cp >> 12)));
    out.push_back((char)(0x80 | ((cp >> 6) & 0x3F)));
    out.push_back((char)(0x80 | (cp & 0x3F)));
  } else {
    out.push_back((char)(0xF0 | (cp >> 18)));
    out.push_back((char)(0x80 | ((cp >> 12) & 0x3F)));
    out.push_back((char)(0x80 | ((cp >> 6) & 0x3F)));
    out.push_back((char)(0x80 | (cp & 0x3F)));
  }
}

class Parser {
 public:
  explicit Parser(const std::string& src) : s_(src) {}

  // rules in order of appearance; names -> index
  std::vector<std::string> names;
  std::vector<AstP> bodies;

  void parse() {
    skip();
    while (p_ < s_.size()) {
      std::string name = ident();
      if (name.empty()) fail("rule name expected");
      skip();
      if (s_.compare(p_, 3, "::=") != 0) fail("'::=' expected after " + name);
      p_ += 3;
      AstP body = alt();
      auto it = index_.find(name);
      if (it != index_.end()) {  // a repeated rule name adds alternatives
        auto a = mk(Ast::kAlt);
        a->kids.push_back(std::move(bodies[it->second]));
        a->kids.push_back(std::move(body));
        bodies[it->second] = std::move(a);
      } else {
        index_[name] = (int)names.size();
        names.push_back(name);
        bodies.push_back(std::move(body));
      }
      skip();
    }
    for (auto& b : bodies) resolve(b.get());
  }
  int index(const std::string& n) const {
    auto it = index_.find(n);
    return it == index_.end() ? -1 : it->second;
  }

 private:
  const std::string s_;
  size_t p_ = 0;
  std::map<std::string, int> index_;

  [[noreturn]] void fail(const std::string& m) const {
    throw std::invalid_argument("grammar: " + m + " at offset " + std::to_string(p_));
  }
  void skip() {
    while (p_ < s_.size()) {
      if (isspace((unsigned char)s_[p_])) {
        ++p_;
      } else if (s_[p_] == '#') {
        while (p_ < s_.size() && s_[p_] != '\n') ++p_;
      } else {
        break;
      }
    }
  }
  static bool name_char(char c) { return isalnum((unsigned char)c) || c == '_' || c == '-' || c == '.'; }
  std::string ident() {
    size_t q = p_;
    if (q < s_.size() && (isalpha((unsigned char)s_[q]) || s_[q] == '_')) {
      while (q < s_.size() && name_char(s_[q])) ++q;
    }
    std::string out = s_.substr(p_, q - p_);
    p_ = q;
    return out;
  }
  // is the text at p_ the start of a new rule ("name ::=")?
  bool at_rule_start() const {
    size_t q = p_;
    if (q >= s_.size() || !(isalpha((unsigned char)s_[q]) || s_[q] == '_')) return false;
    while (q < s_.size() && name_char(s_[q])) ++q;
    while (q < s_.size() && (s_[q] == ' ' || s_[q] == '\t' || s_[q] == '\n' || s_[q] == '\r')) ++q;
    return s_.compare(q, 3, "::=") == 0;
  }
  uint32_t hexn(int n) {
    if (p_ + n > s_.size()) fail("short escape");
    uint32_t v = (uint32_t)std::stoul(s_.substr(p_, n), nullptr, 16);
    p_ += n;
    return v;
  }
  // one (possibly escaped) character of a literal / class, as a code point
  uint32_t chr() {
    if (p_ >= s_.size()) fail("unterminated literal");
    unsigned char c = (unsigned char)s_[p_++];
    if (c != '\\') {
      if (c < 0x80) return c;
      // decode one UTF-8 sequence
      int n = c >= 0xF0 ? 3 : c >= 0xE0 ? 2 : 1;
      uint32_t cp = c & (0x3F >> n);
      for (int i = 0; i < n && p_ < s_.size(); ++i) cp = (cp << 6) | ((unsigned char)s_[p_++] & 0x3F);
      return cp;
    }
    if (p_ >= s_.size()) fail("dangling escape");
    char e = s_[p_++];
    switch (e) {
      case 'n': return '\n';
      case 't': return '\t';
      case 'r': return '\r';
      case 'f': return '\f';
      case 'v': return '\v';
      case '0': return 0;
      case 'x': return hexn(2);
      case 'u': return hexn(4);
      case 'U': return hexn(8);
      default: return (unsigned char)e;
    }
  }
  AstP literal() {
    ++p_;  // opening quote
    std::string bytes;
    while (true) {
      if (p_ >= s_.size()) fail("unterminated string");
      if (s_[p_] == '"') {
        ++p_;
        break;
      }
      utf8(chr(), bytes);
    }
    auto seq = mk(Ast::kSeq);
    for (unsigned char b : bytes) {
      auto a = mk(Ast::kBytes);
      a->cls.set(b);
      seq->kids.push_back(std::move(a));
    }
    return seq;
  }
  AstP klass() {
    ++p_;  // [
    bool neg = false;
    if (p_ < s_.size() && s_[p_] == '^') {
      neg = true;
      ++p_;
    }
    std::bitset<256> set;
    bool first = true, high = false;
    while (true) {
      if (p_ >= s_.size()) fail("unterminated class");
      if (s_[p_] == ']' && !first) {
        ++p_;
        break;
      }
      first = false;
      uint32_t a = chr(), b = a;
      if (p_ + 1 < s_.size() && s_[p_] == '-' && s_[p_ + 1] != ']') {
        ++p_;
        b = chr();
      }
      if (b < a) fail("reversed range");
      for (uint32_t c = a; c <= b && c < 0x80; ++c) set.set(c);
      if (b >= 0x80) {  // non-ASCII members: admit every UTF-8 byte (byte-level classes)
        high = true;
        for (int c = 0x80; c < 0x100; ++c) set.set(c);
      }
    }
    auto n = mk(Ast::kBytes);
    n->cls = neg ? ~set : set;
    if (neg && !high)  // a negated ASCII class still admits the bytes of multi-byte characters
      for (int c = 0x80; c < 0x100; ++c) n->cls.set(c);
    return n;
  }
  AstP primary() {
    skip();
    if (p_ >= s_.size()) fail("unexpected end");
    char c = s_[p_];
    if (c == '"') return literal();
    if (c == '[') return klass();
    if (c == '.') {
      ++p_;
      auto a = mk(Ast::kBytes);
      a->cls.set();
      return a;
    }
    if (c == '(') {
      ++p_;
      AstP a = alt();
      skip();
      if (p_ >= s_.size() || s_[p_] != ')') fail("')' expected");
      ++p_;
      return a;
    }
    std::string n = ident();
    if (n.empty()) fail(std::string("unexpected '") + c + "'");
    auto a = mk(Ast::kRule);
    a->name = n;
    return a;
  }
  AstP postfix() {
    AstP a = primary();
    while (true) {
      skip();
      if (p_ >= s_.size()) break;
      char c = s_[p_];
      int lo, hi;
      if (c == '*') {
        lo = 0, hi = -1, ++p_;
      } else if (c == '+') {
        lo = 1, hi = -1, ++p_;
      } else if (c == '?') {
        lo = 0, hi = 1, ++p_;
      } else if (c == '{') {
        ++p_;
        size_t q;
        lo = std::stoi(s_.substr(p_), &q);
        p_ += q;
        hi = lo;
        if (p_ < s_.size() && s_[p_] == ',') {
          ++p_;
          if (p_ < s_.size() && s_[p_] == '}') {
            hi = -1;
          } else {
            hi = std::stoi(s_.substr(p_), &q);
            p_ += q;
          }
        }
        if (p_ >= s_.size() || s_[p_] != '}') fail("'}' expected");
        ++p_;
        if (hi >= 0 && hi < lo) fail("bad repetition bounds");
      } else {
        break;
      }
      auto r = mk(Ast::kRepeat);
      r->lo = lo;
      r->hi = hi;
      r->kids.push_back(std::move(a));
      a = std::move(r);
    }
    return a;
  }
  AstP seq() {
    auto s = mk(Ast::kSeq);
    while (true) {
      skip();
      if (p_ >= s_.size() || s_[p_] == '|' || s_[p_] == ')' || at_rule_start()) break;
      s->kids.push_back(postfix());
    }
    return s;
  }
  AstP alt() {
    auto a = mk(Ast::kAlt);
    a->kids.push_back(seq());
    while (true) {
      skip();
      if (p_ < s_.size() && s_[p_] == '|') {
        ++p_;
        a->kids.push_back(seq());
      } else {
        break;
      }
    }
    if (a->kids.size() == 1) return std::move(a->kids[0]);
    return a;
  }
  void resolve(Ast* a) {
    if (a->kind == Ast::kRule) {
      a->rule = index(a->name);
      if (a->rule < 0) throw std::invalid_argument("grammar: undefined rule '" + a->name + "'");
    }
    for (auto& k : a->kids) resolve(k.get());
  }
};

// ------------------------------------------------------------------ per-rule automata
struct NState {
  int sym = -1;  // -1: no consuming edge; else index into the rule's symbol table
  int next = -1;
  int eps1 = -1, eps2 = -1;
};

struct RuleNfa {
  std::vector<NState> st;
  std::vector<std::bitset<256>> byte_syms;  // symbol s < byte_syms.size(): byte class
  std::vector<int> call_syms;               // symbol byte_syms.size() + i: call of rule call_syms[i]
  int start = 0, accept = 0;
  int add() {
    st.push_back(NState{});
    return (int)st.size() - 1;
  }
  int byte_sym(const std::bitset<256>& c) {
    for (size_t i = 0; i < byte_syms.size(); ++i)
      if (byte_syms[i] == c) return (int)i;
    byte_syms.push_back(c);
    return (int)byte_syms.size() - 1;
  }
};

struct Frag {
  int s, e;
};

class NfaBuilder {
 public:
  explicit NfaBuilder(RuleNfa& n) : n_(n) {}
  Frag build(const Ast* a) {
    switch (a->kind) {
      case Ast::kBytes: {
        int s = n_.add(), e = n_.add();
        n_.st[s].sym = n_.byte_sym(a->cls);
        n_.st[s].next = e;
        return {s, e};
      }
      case Ast::kRule: {
        int s = n_.add(), e = n_.add();
        calls_.push_back({s, a->rule});
        n_.st[s].next = e;
        return {s, e};
      }
      case Ast::kSeq: {
        if (a->kids.empty()) {
          int s = n_.add();
          return {s, s};
        }
        Frag f = build(a->kids[0].get());
        for (size_t i = 1; i < a->kids.size(); ++i) {
          Frag g = build(a->kids[i].get());
          n_.st[f.e].eps1 = g.s;
          f.e = g.e;
        }
        return f;
      }
      case Ast::kAlt: {
        int s = n_.add(), e = n_.add();
        int cur = s;
        for (size_t i = 0; i < a->kids.size(); ++i) {
          Frag g = build(a->kids[i].get());
          n_.st[g.e].eps1 = e;
          if (i + 1 == a->kids.size()) {
            n_.st[cur].eps1 = g.s;
          } else {
            int nxt = n_.add();
            n_.st[cur].eps1 = g.s;
            n_.st[cur].eps2 = nxt;
            cur = nxt;
          }
        }
        return {s, e};
      }
      case Ast::kRepeat: {
        const Ast* k = a->kids[0].get();
        int s = n_.add();
        int cur = s;
        for (int i = 0; i < a->lo; ++i) {
          Frag g = build(k);
          n_.st[cur].eps1 = g.s;
          cur = g.e;
        }
        int e = n_.add();
        if (a->hi < 0) {  // star on the tail
          Frag g = build(k);
          n_.st[cur].eps1 = g.s;
          n_.st[cur].eps2 = e;
          n_.st[g.e].eps1 = g.s;
          n_.st[g.e].eps2 = e;
        } else {
          for (int i = a->lo; i < a->hi; ++i) {
            Frag g = build(k);
            n_.st[cur].eps1 = g.s;
            n_.st[cur].eps2 = e;
            cur = g.e;
          }
          n_.st[cur].eps1 = e;
        }
        return {s, e};
      }
    }
    throw std::logic_error("grammar: bad node");
  }
  void finish() {
    for (auto& c : calls_) {
      int idx = -1;
      for (size_t i = 0; i < n_.call_syms.size(); ++i)
        if (n_.call_syms[i] == c.second) idx = (int)i;
      if (idx < 0) {
        n_.call_syms.push_back(c.second);
        idx = (int)n_.call_syms.size() - 1;
      }
      n_.st[c.first].sym = (int)n_.byte_syms.size() + idx;  // byte symbols are all known by now
    }
  }

 private:
  RuleNfa& n_;
  std::vector<std::pair<int, int>> calls_;  // (state, rule) until symbols are numbered
};

struct DState {
  std::array<int, 256> next;           // byte -> state (-1 none)
  std::vector<std::pair<int, int>> calls;  // (callee rule, state after the call)
  bool accept = false;
  bool has_bytes = false;
};

struct RuleDfa {
  std::vector<DState> st;  // state 0 = start
};

static RuleDfa determinise(const RuleNfa& n) {
  const int nb = (int)n.byte_syms.size();
  auto closure = [&](std::vector<int> set) {
    std::vector<char> in(n.st.size(), 0);
    std::vector<int> stack = set;
    for (int s : set) in[s] = 1;
    while (!stack.empty()) {
      int s = stack.back();
      stack.pop_back();
      for (int e : {n.st[s].eps1, n.st[s].eps2})
        if (e >= 0 && !in[e]) {
          in[e] = 1;
          set.push_back(e);
          stack.push_back(e);
        }
    }
    std::sort(set.begin(), set.end());
    return set;
  };
  RuleDfa d;
  std::map<std::vector<int>, int> index;
  std::vector<std::vector<int>> sets;
  auto intern = [&](std::vector<int> set) {
    auto it = index.find(set);
    if (it != index.end()) return it->second;
    int id = (int)sets.size();
    index[set] = id;
    sets.push_back(set);
    return id;
  };
  intern(closure({n.start}));
  for (size_t i = 0; i < sets.size(); ++i) {
    DState ds;
    ds.next.fill(-1);
    const std::vector<int> cur = sets[i];
    for (int s : cur)
      if (s == n.accept) ds.accept = true;
    // byte moves: group target sets per byte
    std::array<std::vector<int>, 256> by;
    std::map<int, std::vector<int>> callt;  // callee rule -> targets
    for (int s : cur) {
      const NState& x = n.st[s];
      if (x.sym < 0) continue;
      if (x.sym < nb) {
        const auto& cls = n.byte_syms[x.sym];
        for (int b = 0; b < 256; ++b)
          if (cls.test(b)) by[b].push_back(x.next);
      } else {
        callt[n.call_syms[x.sym - nb]].push_back(x.next);
      }
    }
    std::map<std::vector<int>, int> memo;
    for (int b = 0; b < 256; ++b) {
      if (by[b].empty()) continue;
      std::vector<int> t = by[b];
      std::sort(t.begin(), t.end());
      t.erase(std::unique(t.begin(), t.end()), t.end());
      auto m = memo.find(t);
      int id;
      if (m != memo.end()) {
        id = m->second;
      } else {
        id = intern(closure(t));
        memo[t] = id;
      }
      ds.next[b] = id;
      ds.has_bytes = true;
    }
    for (auto& kv : callt) ds.calls.push_back({kv.first, intern(closure(kv.second))});
    d.st.push_back(ds);
  }
  return d;
}

// ------------------------------------------------------------------ rule inlining
// Rules that take no part in a recursion cycle are expanded into their
// callers (lexical rules such as a JSON string or number become byte-level
// states of the rule that uses them), so calls remain only where recursion
// needs a stack; this keeps most tokens decidable inside one rule.
static AstP clone(const Ast* a) {
  auto c = std::make_unique<Ast>();
  c->kind = a->kind;
  c->cls = a->cls;
  c->name = a->name;
  c->rule = a->rule;
  c->lo = a->lo;
  c->hi = a->hi;
  for (auto& k : a->kids) c->kids.push_back(clone(k.get()));
  return c;
}

static void refs(const Ast* a, std::vector<int>& out) {
  if (a->kind == Ast::kRule) out.push_back(a->rule);
  for (auto& k : a->kids) refs(k.get(), out);
}

static size_t ast_size(const Ast* a) {
  size_t n = 1;
  for (auto& k : a->kids) n += ast_size(k.get());
  return n;
}

static void inline_rules(std::vector<AstP>& bodies) {
  const int R = (int)bodies.size();
  std::vector<std::vector<int>> edges(R);
  for (int r = 0; r < R; ++r) refs(bodies[r].get(), edges[r]);
  // cyclic[r]: r reaches itself through calls
  std::vector<char> cyclic(R, 0);
  for (int r = 0; r < R; ++r) {
    std::vector<char> seen(R, 0);
    std::vector<int> st = edges[r];
    while (!st.empty() && !cyclic[r]) {
      int x = st.back();
      st.pop_back();
      if (x == r) cyclic[r] = 1;
      if (seen[x]) continue;
      seen[x] = 1;
      for (int y : edges[x]) st.push_back(y);
    }
  }
  // expand references to acyclic rules, bottom-up (memoised expanded bodies)
  std::vector<AstP> expanded(R);
  std::vector<char> state(R, 0);  // 0 new, 1 in progress, 2 done
  constexpr size_t kMaxAst = 1 << 18;
  std::function<void(int)> expand_rule;
  std::function<AstP(const Ast*)> expand = [&](const Ast* a) -> AstP {
    if (a->kind == Ast::kRule && !cyclic[a->rule]) {
      expand_rule(a->rule);
      if (ast_size(expanded[a->rule].get()) <= kMaxAst / 16) return clone(expanded[a->rule].get());
      return clone(a);
    }
    auto c = std::make_unique<Ast>();
    c->kind = a->kind;
    c->cls = a->cls;
    c->name = a->name;
    c->rule = a->rule;
    c->lo = a->lo;
    c->hi = a->hi;
    for (auto& k : a->kids) c->kids.push_back(expand(k.get()));
    return c;
  };
  expand_rule = [&](int r) {
    if (state[r] == 2) return;
    state[r] = 1;
    expanded[r] = expand(bodies[r].get());
    state[r] = 2;
  };
  for (int r = 0; r < R; ++r) expand_rule(r);
  for (int r = 0; r < R; ++r)
    if (ast_size(expanded[r].get()) <= kMaxAst) bodies[r] = std::move(expanded[r]);
}

// ------------------------------------------------------------------ compiled grammar
class Grammar {
 public:
  Grammar(const std::string& text, const std::string& root) {
    Parser p(text);
    p.parse();
    root_ = p.index(root);
    if (root_ < 0) throw std::invalid_argument("grammar: no root rule '" + root + "'");
    names_ = p.names;
    inline_rules(p.bodies);
    for (auto& body : p.bodies) {
      RuleNfa n;
      NfaBuilder b(n);
      Frag f = b.build(body.get());
      b.finish();
      n.start = f.s;
      n.accept = f.e;
      dfas_.push_back(determinise(n));
    }
  }
  int root() const { return root_; }
  const DState& st(int rule, int s) const { return dfas_[rule].st[s]; }
  int num_rules() const { return (int)dfas_.size(); }
  size_t num_states() const {
    size_t n = 0;
    for (auto& d : dfas_) n += d.st.size();
    return n;
  }

 private:
  int root_ = -1;
  std::vector<std::string> names_;
  std::vector<RuleDfa> dfas_;
};

// Token classes of one (rule, state) top: allowed whatever the stack holds,
// and the trie nodes below which the rest of every token is undecided (the
// walk met a call or a possible return before the token's bytes ran out).
struct Local {
  std::vector<uint32_t> allowed;
  std::vector<int> undecided_roots;
};

// A grammar compiled against one vocabulary: shared by every matcher of it,
// so the per-(rule, state) token classes are computed once.
class Compiled {
 public:
  Compiled(std::shared_ptr<Vocab> vocab, const std::string& text, const std::string& root)
      : vocab(std::move(vocab)), g(std::make_shared<Grammar>(text, root)) {}
  std::shared_ptr<Vocab> vocab;
  std::shared_ptr<Grammar> g;

  const Local& local(int rule, int state) {
    auto key = std::make_pair(rule, state);
    auto it = local_.find(key);
    if (it != local_.end()) return it->second;
    Local L;
    L.allowed.assign((vocab->size() + 31) / 32, 0u);
    struct Item {
      int node, state;
      bool branch;
    };
    std::vector<Item> stack{{0, state, false}};
    while (!stack.empty()) {
      Item cur = stack.back();
      stack.pop_back();
      const auto& tn = vocab->nodes_[cur.node];
      if (cur.node != 0)
        for (int id : tn.ids) L.allowed[id >> 5] |= 1u << (id & 31);
      const DState& d = g->st(rule, cur.state);
      const bool branch = cur.branch || !d.calls.empty() || d.accept;
      for (auto& kv : tn.kids) {
        const int nx = d.next[kv.first];
        if (nx >= 0) {
          stack.push_back({kv.second, nx, branch});
        } else if (branch) {
          L.undecided_roots.push_back(kv.second);
        }
      }
    }
    return local_.emplace(key, std::move(L)).first->second;
  }

 private:
  std::map<std::pair<int, int>, Local> local_;
};

// ------------------------------------------------------------------ matcher
constexpr int kMaxClosure = 1 << 16;

class Matcher {
 public:
  explicit Matcher(std::shared_ptr<Compiled> c) : c_(std::move(c)), vocab_(c_->vocab), g_(c_->g) {
    history_.push_back(close({node(g_->root(), 0, -1)}));
  }

  bool is_accepting() const { return accepting(history_.back()); }
  bool is_terminated() const { return terminated_; }
  size_t num_stacks() const { return history_.back().size(); }
  size_t num_states() const { return g_->num_states(); }

  py::array_t<uint32_t> mask() {
    const auto& set = history_.back();
    auto it = mask_cache_.find(set);
    if (it == mask_cache_.end()) it = mask_cache_.emplace(set, compute_mask(set)).first;
    const auto& m = it->second;
    py::array_t<uint32_t> out(m.size());
    std::copy(m.begin(), m.end(), out.mutable_data());
    return out;
  }

  bool accept_token(int id) {
    if (terminated_ || id < 0 || id >= vocab_->size()) return false;
    if (vocab_->is_eos(id)) {
      if (!is_accepting()) return false;
      terminated_ = true;
      history_.push_back(history_.back());
      return true;
    }
    const std::string& b = vocab_->bytes(id);
    if (b.empty()) return false;
    std::vector<int> set = history_.back();
    for (unsigned char c : b) {
      set = advance(set, c);
      if (set.empty()) return false;
    }
    history_.push_back(std::move(set));
    return true;
  }
  bool accept_string(const std::string& s) {
    std::vector<int> set = history_.back();
    for (unsigned char c : s) {
      set = advance(set, c);
      if (set.empty()) return false;
    }
    history_.push_back(std::move(set));
    return true;
  }
  void rollback(int n) {
    for (int i = 0; i < n && history_.size() > 1; ++i) history_.pop_back();
    terminated_ = false;
  }
  std::string forced_prefix(int max_len) {
    std::string out;
    std::vector<int> set = history_.back();
    for (int i = 0; i < max_len; ++i) {
      if (accepting(set)) break;
      int only = -1;
      bool many = false;
      for (int n : set) {
        const Frame& f = arena_[n];
        const DState& d = g_->st(f.rule, f.state);
        if (!d.has_bytes) continue;
        for (int b = 0; b < 256 && !many; ++b)
          if (d.next[b] >= 0) {
            if (only < 0) {
              only = b;
            } else if (only != b) {
              many = true;
            }
          }
        if (many) break;
      }
      if (many || only < 0) break;
      out.push_back((char)only);
      set = advance(set, (unsigned char)only);
    }
    return out;
  }

 private:
  struct Frame {
    int rule, state, parent;
  };

  std::shared_ptr<Compiled> c_;
  std::shared_ptr<Vocab> vocab_;
  std::shared_ptr<Grammar> g_;
  std::vector<Frame> arena_;
  std::unordered_map<uint64_t, std::vector<int>> nodes_;  // (rule, state, parent) hash -> candidate ids
  std::vector<std::vector<int>> history_;
  bool terminated_ = false;
  std::map<std::vector<int>, std::vector<uint32_t>> mask_cache_;
  // stack sets interned to ids, and memoised byte transitions between them
  std::map<std::vector<int>, int> set_ids_;
  std::vector<std::vector<int>> sets_;
  std::unordered_map<uint64_t, int> step_memo_;

  int node(int rule, int state, int parent) {
    const uint64_t key = ((uint64_t)(uint32_t)rule * 1000003ull + (uint32_t)state) * 2654435761ull ^
                         (uint64_t)(uint32_t)(parent + 1);
    auto& bucket = nodes_[key];
    for (int id : bucket) {
      const Frame& f = arena_[id];
      if (f.rule == rule && f.state == state && f.parent == parent) return id;
    }
    arena_.push_back(Frame{rule, state, parent});
    bucket.push_back((int)arena_.size() - 1);
    return (int)arena_.size() - 1;
  }

  // Closure under calls and returns; the result keeps the stacks that can
  // consume a byte or end the parse.
  std::vector<int> close(std::vector<int> set) {
    std::vector<int> out, work = set;
    std::unordered_map<int, char> seen;
    for (int n : set) seen[n] = 1;
    size_t steps = 0;
    while (!work.empty()) {
      if (++steps > (size_t)kMaxClosure)
        throw std::runtime_error("grammar: closure does not terminate (left recursion?)");
      const int n = work.back();
      work.pop_back();
      const Frame f = arena_[n];
      const DState& d = g_->st(f.rule, f.state);
      if (d.has_bytes || (d.accept && f.parent < 0)) out.push_back(n);
      for (auto& c : d.calls) {
        // a call in tail position (its return state only accepts) returns
        // straight to this frame's caller: right-recursive rules run in
        // constant stack depth
        const DState& rs = g_->st(f.rule, c.second);
        const bool tail = rs.accept && !rs.has_bytes && rs.calls.empty();
        const int ret = tail ? f.parent : node(f.rule, c.second, f.parent);
        const int child = node(c.first, 0, ret);
        if (!seen[child]) {
          seen[child] = 1;
          work.push_back(child);
        }
      }
      if (d.accept && f.parent >= 0 && !seen[f.parent]) {
        seen[f.parent] = 1;
        work.push_back(f.parent);
      }
    }
    std::sort(out.begin(), out.end());
    out.erase(std::unique(out.begin(), out.end()), out.end());
    return out;
  }

  std::vector<int> advance(const std::vector<int>& set, unsigned char b) {
    std::vector<int> nxt;
    for (int n : set) {
      const Frame f = arena_[n];
      const int t = g_->st(f.rule, f.state).next[b];
      if (t >= 0) nxt.push_back(node(f.rule, t, f.parent));
    }
    if (nxt.empty()) return nxt;
    std::sort(nxt.begin(), nxt.end());
    nxt.erase(std::unique(nxt.begin(), nxt.end()), nxt.end());
    return close(nxt);
  }

  bool accepting(const std::vector<int>& set) const {
    for (int n : set) {
      const Frame& f = arena_[n];
      if (f.parent < 0 && g_->st(f.rule, f.state).accept) return true;
    }
    return false;
  }

  int set_id(const std::vector<int>& set) {
    auto it = set_ids_.find(set);
    if (it != set_ids_.end()) return it->second;
    set_ids_[set] = (int)sets_.size();
    sets_.push_back(set);
    return (int)sets_.size() - 1;
  }
  // id of the set after byte b (-1: empty), memoised
  int step(int sid, unsigned char b) {
    const uint64_t key = (uint64_t)sid * 256 + b;
    auto it = step_memo_.find(key);
    if (it != step_memo_.end()) return it->second;
    std::vector<int> nx = advance(sets_[sid], b);
    const int r = nx.empty() ? -1 : set_id(nx);
    step_memo_[key] = r;
    return r;
  }

  std::vector<uint32_t> compute_mask(const std::vector<int>& set) {
    std::vector<uint32_t> m((vocab_->size() + 31) / 32, 0u);
    std::vector<int> roots;
    std::map<std::pair<int, int>, char> tops;
    for (int n : set) {
      const Frame& f = arena_[n];
      if (!g_->st(f.rule, f.state).has_bytes) continue;
      if (tops[{f.rule, f.state}]) continue;
      tops[{f.rule, f.state}] = 1;
      const Local& L = c_->local(f.rule, f.state);
      for (size_t w = 0; w < m.size(); ++w) m[w] |= L.allowed[w];
      roots.insert(roots.end(), L.undecided_roots.begin(), L.undecided_roots.end());
    }
    std::sort(roots.begin(), roots.end());
    roots.erase(std::unique(roots.begin(), roots.end()), roots.end());
    // undecided subtrees: walk the trie from each root with the whole stack set,
    // pruning where no stack can take the next byte
    const int s0 = set_id(set);
    std::vector<std::pair<int, int>> work;  // (trie node, set id after its path)
    for (int r : roots) {
      int sid = s0;
      for (unsigned char b : vocab_->path(r)) {
        sid = step(sid, b);
        if (sid < 0) break;
      }
      if (sid >= 0) work.push_back({r, sid});
    }
    while (!work.empty()) {
      auto [t, sid] = work.back();
      work.pop_back();
      const auto& tn = vocab_->nodes_[t];
      for (int id : tn.ids) m[id >> 5] |= 1u << (id & 31);
      for (auto& kv : tn.kids) {
        const int nx = step(sid, kv.first);
        if (nx >= 0) work.push_back({kv.second, nx});
      }
    }
    if (accepting(set))
      for (int e : vocab_->eos()) m[e >> 5] |= 1u << (e & 31);
    return m;
  }
};

}  // namespace cfg
}  // namespace b200host

void register_grammar_pda(py::module_& m) {
  using namespace b200host;
  py::class_<cfg::Compiled, std::shared_ptr<cfg::Compiled>>(m, "CfgGrammar")
      .def(py::init<std::shared_ptr<Vocab>, const std::string&, const std::string&>(), py::arg("vocab"),
           py::arg("grammar"), py::arg("root") = std::string("root"))
      .def_property_readonly("num_states", [](const cfg::Compiled& c) { return c.g->num_states(); });
  py::class_<cfg::Matcher>(m, "CfgMatcher")
      .def(py::init<std::shared_ptr<cfg::Compiled>>(), py::arg("grammar"))
      .def("mask", &cfg::Matcher::mask)
      .def("accept_token", &cfg::Matcher::accept_token)
      .def("accept_string", &cfg::Matcher::accept_string)
      .def("rollback", &cfg::Matcher::rollback)
      .def("forced_prefix", [](cfg::Matcher& m, int max_len) { return py::bytes(m.forced_prefix(max_len)); },
           py::arg("max_len") = 256)
      .def("is_accepting", &cfg::Matcher::is_accepting)
      .def("is_terminated", &cfg::Matcher::is_terminated)
      .def_property_readonly("num_stacks", &cfg::Matcher::num_stacks)
      .def_property_readonly("num_states", &cfg::Matcher::num_states);
}
