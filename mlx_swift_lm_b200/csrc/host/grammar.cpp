// Grammar engine for constrained decoding (native).
//
// The reference vendors xgrammar (Libraries/MLXCXGrammar, ~24k lines of C++:
// EBNF / JSON-schema / regex front ends, Earley parser, per-state token masks,
// matcher with rollback and jump-forward, C API xgrammar_c.h). This engine is
// a compact redesign with the same job:
//   * a regular-expression dialect compiled to a byte-level NFA (Thompson)
//     and determinised lazily (subset construction on demand, states cached);
//   * JSON schema / EBNF front ends (Python side) lower to this dialect, with
//     recursion unrolled to a bounded depth;
//   * a vocabulary trie over the tokens' byte strings; the allowed-token mask
//     of a DFA state is a depth-first walk of the trie that prunes at dead
//     states, computed once per state and cached as a bitmask;
//   * a matcher with accept / rollback / forced-prefix (jump-forward) and an
//     EOS rule (EOS allowed only in accepting states).
// Regex dialect: literals, escapes (\d \w \s \n \t \\ and escaped
// metacharacters), classes [a-z_] / [^...], '.', grouping ( ), alternation |,
// quantifiers * + ? {m} {m,} {m,n}.
#include <pybind11/numpy.h>
#include <pybind11/pybind11.h>
#include <pybind11/stl.h>

#include <algorithm>
#include <bitset>
#include <cstdint>
#include <map>
#include <memory>
#include <stdexcept>
#include <string>
#include <unordered_map>
#include <vector>

#include "grammar_vocab.h"

namespace py = pybind11;

namespace b200host {

// ------------------------------------------------------------------ NFA
struct NState {
  std::bitset<256> cls;  // byte class for a consuming edge
  int next = -1;          // consuming edge target
  int eps1 = -1, eps2 = -1;
};

struct Frag {
  int start, end;  // end state has no edges yet
};

class RegexCompiler {
 public:
  explicit RegexCompiler(const std::string& re) : s_(re) {}
  std::vector<NState> states;
  int compile(int* accept) {
    Frag f = parse_alt();
    if (pos_ != s_.size()) throw std::invalid_argument("regex: unexpected ')' at " + std::to_string(pos_));
    *accept = f.end;
    return f.start;
  }

 private:
  const std::string s_;
  size_t pos_ = 0;
  int add() {
    states.emplace_back();
    return (int)states.size() - 1;
  }
  bool more() const { return pos_ < s_.size(); }
  char peek() const { return s_[pos_]; }

  Frag parse_alt() {
    Frag left = parse_concat();
    while (more() && peek() == '|') {
      ++pos_;
      Frag right = parse_concat();
      int st = add(), en = add();
      states[st].eps1 = left.start;
      states[st].eps2 = right.start;
      states[left.end].eps1 = en;
      states[right.end].eps1 = en;
      left = {st, en};
    }
    return left;
  }
  Frag parse_concat() {
    int st = add();
    Frag cur{st, st};
    while (more() && peek() != '|' && peek() != ')') {
      Frag a = parse_repeat();
      states[cur.end].eps1 = a.start;
      cur.end = a.end;
    }
    return cur;
  }
  Frag clone(const Frag& f) {
    // copy the sub-automaton reachable from f.start up to f.end
    std::map<int, int> m;
    std::vector<int> stack{f.start};
    m[f.start] = add();
    while (!stack.empty()) {
      int u = stack.back();
      stack.pop_back();
      for (int v : {states[u].next, states[u].eps1, states[u].eps2}) {
        if (v < 0 || m.count(v)) continue;
        m[v] = add();
        stack.push_back(v);
      }
    }
    for (auto& kv : m) {
      const NState src = states[kv.first];
      NState& dst = states[kv.second];
      dst.cls = src.cls;
      dst.next = src.next >= 0 ? m[src.next] : -1;
      dst.eps1 = src.eps1 >= 0 ? m[src.eps1] : -1;
      dst.eps2 = src.eps2 >= 0 ? m[src.eps2] : -1;
    }
    return {m[f.start], m[f.end]};
  }
  Frag star(Frag a) {
    int st = add(), en = add();
    states[st].eps1 = a.start;
    states[st].eps2 = en;
    states[a.end].eps1 = a.start;
    states[a.end].eps2 = en;
    return {st, en};
  }
  Frag optional(Frag a) {
    int st = add(), en = add();
    states[st].eps1 = a.start;
    states[st].eps2 = en;
    states[a.end].eps1 = en;
    return {st, en};
  }
  Frag concat(Frag a, Frag b) {
    states[a.end].eps1 = b.start;
    return {a.start, b.end};
  }
  Frag empty() {
    int st = add();
    return {st, st};
  }
  Frag parse_repeat() {
    Frag a = parse_atom();
    while (more()) {
      char c = peek();
      if (c == '*') {
        ++pos_;
        a = star(a);
      } else if (c == '+') {
        ++pos_;
        Frag b = clone(a);
        a = concat(a, star(b));
      } else if (c == '?') {
        ++pos_;
        a = optional(a);
      } else if (c == '{') {
        size_t close = s_.find('}', pos_);
        if (close == std::string::npos) throw std::invalid_argument("regex: unterminated {");
        std::string body = s_.substr(pos_ + 1, close - pos_ - 1);
        pos_ = close + 1;
        int lo, hi;
        size_t comma = body.find(',');
        if (comma == std::string::npos) {
          lo = hi = std::stoi(body);
        } else {
          lo = comma == 0 ? 0 : std::stoi(body.substr(0, comma));
          hi = comma + 1 == body.size() ? -1 : std::stoi(body.substr(comma + 1));
        }
        if (lo > 256 || hi > 256) throw std::invalid_argument("regex: repeat count too large");
        Frag base = a;
        Frag out = empty();
        for (int i = 0; i < lo; ++i) out = concat(out, i == 0 ? base : clone(base));
        if (hi < 0) {
          out = concat(out, star(lo == 0 ? base : clone(base)));
        } else {
          for (int i = lo; i < hi; ++i) out = concat(out, optional((i == 0 && lo == 0) ? base : clone(base)));
        }
        a = out;
      } else {
        break;
      }
    }
    return a;
  }
  static void add_class_escape(std::bitset<256>& b, char c) {
    switch (c) {
      case 'd':
        for (int x = '0'; x <= '9'; ++x) b.set(x);
        break;
      case 'w':
        for (int x = '0'; x <= '9'; ++x) b.set(x);
        for (int x = 'a'; x <= 'z'; ++x) b.set(x);
        for (int x = 'A'; x <= 'Z'; ++x) b.set(x);
        b.set('_');
        break;
      case 's':
        for (char x : {' ', '\t', '\n', '\r', '\f', '\v'}) b.set((unsigned char)x);
        break;
      case 'D': {
        std::bitset<256> t;
        add_class_escape(t, 'd');
        b |= ~t;
        break;
      }
      case 'W': {
        std::bitset<256> t;
        add_class_escape(t, 'w');
        b |= ~t;
        break;
      }
      case 'S': {
        std::bitset<256> t;
        add_class_escape(t, 's');
        b |= ~t;
        break;
      }
      case 'n': b.set('\n'); break;
      case 't': b.set('\t'); break;
      case 'r': b.set('\r'); break;
      case 'f': b.set('\f'); break;
      default: b.set((unsigned char)c);
    }
  }
  // After a backslash: read `\xHH` as one byte. Returns -1 if not a hex escape.
  int hex_escape(char e) {
    if (e != 'x') return -1;
    if (pos_ + 2 > s_.size()) throw std::invalid_argument("regex: truncated \\x escape");
    const int v = std::stoi(s_.substr(pos_, 2), nullptr, 16);
    pos_ += 2;
    return v;
  }
  Frag byte_class(const std::bitset<256>& cls) {
    int st = add(), en = add();
    states[st].cls = cls;
    states[st].next = en;
    return {st, en};
  }
  Frag parse_atom() {
    if (!more()) throw std::invalid_argument("regex: unexpected end");
    char c = s_[pos_++];
    if (c == '(') {
      if (s_.compare(pos_, 2, "?:") == 0) pos_ += 2;
      Frag f = parse_alt();
      if (!more() || peek() != ')') throw std::invalid_argument("regex: missing )");
      ++pos_;
      return f;
    }
    std::bitset<256> cls;
    if (c == '.') {
      cls.set();
      cls.reset('\n');
    } else if (c == '\\') {
      if (!more()) throw std::invalid_argument("regex: trailing backslash");
      char e = s_[pos_++];
      if (e == 'u') {  // \uXXXX -> UTF-8 bytes as a literal sequence
        unsigned cp = std::stoul(s_.substr(pos_, 4), nullptr, 16);
        pos_ += 4;
        return literal_utf8(cp);
      }
      const int hx = hex_escape(e);
      if (hx >= 0) cls.set(hx);
      else add_class_escape(cls, e);
    } else if (c == '[') {
      bool neg = false;
      if (more() && peek() == '^') {
        neg = true;
        ++pos_;
      }
      bool first = true;
      while (more() && (peek() != ']' || first)) {
        first = false;
        unsigned char a = (unsigned char)s_[pos_++];
        if (a == '\\') {
          char e = s_[pos_++];
          if (e == 'd' || e == 'w' || e == 's' || e == 'D' || e == 'W' || e == 'S') {
            add_class_escape(cls, e);
            continue;
          }
          const int hx = hex_escape(e);
          if (hx >= 0) {
            a = (unsigned char)hx;
          } else {
            std::bitset<256> t;
            add_class_escape(t, e);
            for (int x = 0; x < 256; ++x)
              if (t[x]) a = (unsigned char)x;
          }
        }
        if (pos_ + 1 < s_.size() && peek() == '-' && s_[pos_ + 1] != ']') {
          ++pos_;
          unsigned char b = (unsigned char)s_[pos_++];
          if (b == '\\') {
            const char e2 = s_[pos_++];
            const int hx2 = hex_escape(e2);
            if (hx2 >= 0) {
              b = (unsigned char)hx2;
            } else {
              std::bitset<256> t;
              add_class_escape(t, e2);
              for (int x = 0; x < 256; ++x)
                if (t[x]) b = (unsigned char)x;
            }
          }
          for (int x = a; x <= b; ++x) cls.set(x);
        } else {
          cls.set(a);
        }
      }
      if (!more()) throw std::invalid_argument("regex: unterminated [");
      ++pos_;
      if (neg) cls = ~cls;
    } else {
      cls.set((unsigned char)c);
    }
    return byte_class(cls);
  }
  Frag literal_utf8(unsigned cp) {
    std::string u;
    if (cp < 0x80) u.push_back((char)cp);
    else if (cp < 0x800) {
      u.push_back((char)(0xC0 | (cp >> 6)));
      u.push_back((char)(0x80 | (cp & 0x3F)));
    } else {
      u.push_back((char)(0xE0 | (cp >> 12)));
      u.push_back((char)(0x80 | ((cp >> 6) & 0x3F)));
      u.push_back((char)(0x80 | (cp & 0x3F)));
    }
    Frag out = empty();
    for (unsigned char ch : u) {
      std::bitset<256> b;
      b.set(ch);
      out = concat(out, byte_class(b));
    }
    return out;
  }
};

// ------------------------------------------------------------------ lazy DFA
class Dfa {
 public:
  explicit Dfa(const std::string& regex) {
    RegexCompiler rc(regex);
    int accept;
    int start = rc.compile(&accept);
    nfa_ = std::move(rc.states);
    accept_ = accept;
    start_ = intern(closure({start}));
  }
  int start() const { return start_; }
  bool accepting(int d) const { return dstates_[d].accepting; }
  int step(int d, unsigned char b) {
    int& t = dstates_[d].trans[b];
    if (t != -2) return t;
    std::vector<int> next;
    for (int s : dstates_[d].set)
      if (nfa_[s].next >= 0 && nfa_[s].cls[b]) next.push_back(nfa_[s].next);
    if (next.empty()) {
      dstates_[d].trans[b] = -1;
      return -1;
    }
    const int r = intern(closure(next));
    dstates_[d].trans[b] = r;
    return r;
  }
  // true if some byte leaves state d
  bool has_out(int d) {
    for (int s : dstates_[d].set)
      if (nfa_[s].next >= 0 && nfa_[s].cls.any()) return true;
    return false;
  }
  size_t num_states() const { return dstates_.size(); }

 private:
  struct DState {
    std::vector<int> set;
    bool accepting = false;
    std::vector<int> trans = std::vector<int>(256, -2);
  };
  std::vector<NState> nfa_;
  int accept_ = -1, start_ = -1;
  std::vector<DState> dstates_;
  std::map<std::vector<int>, int> index_;

  std::vector<int> closure(std::vector<int> seeds) {
    std::vector<char> seen(nfa_.size(), 0);
    std::vector<int> out, stack = seeds;
    while (!stack.empty()) {
      int u = stack.back();
      stack.pop_back();
      if (u < 0 || seen[u]) continue;
      seen[u] = 1;
      out.push_back(u);
      stack.push_back(nfa_[u].eps1);
      stack.push_back(nfa_[u].eps2);
    }
    std::sort(out.begin(), out.end());
    return out;
  }
  int intern(std::vector<int> set) {
    auto it = index_.find(set);
    if (it != index_.end()) return it->second;
    if (dstates_.size() > 200000) throw std::runtime_error("grammar: DFA state budget exceeded");
    DState d;
    d.accepting = std::binary_search(set.begin(), set.end(), accept_);
    d.set = set;
    dstates_.push_back(std::move(d));
    index_[set] = (int)dstates_.size() - 1;
    return (int)dstates_.size() - 1;
  }
};

class Matcher {
 public:
  Matcher(std::shared_ptr<Vocab> vocab, const std::string& regex)
      : vocab_(std::move(vocab)), dfa_(std::make_shared<Dfa>(regex)) {
    history_.push_back(dfa_->start());
  }
  int state() const { return history_.back(); }
  bool is_accepting() const { return dfa_->accepting(state()); }
  bool is_terminated() const { return terminated_; }

  // Bitmask (uint32 words, bit = token allowed) for the current state.
  py::array_t<uint32_t> mask() {
    const int d = state();
    auto it = cache_.find(d);
    if (it == cache_.end()) it = cache_.emplace(d, compute(d)).first;
    const auto& m = it->second;
    py::array_t<uint32_t> out(m.size());
    std::copy(m.begin(), m.end(), out.mutable_data());
    return out;
  }

  bool accept_token(int id) {
    if (terminated_) return false;
    for (int e : vocab_->eos())
      if (id == e) {
        if (!is_accepting()) return false;
        terminated_ = true;
        history_.push_back(state());
        return true;
      }
    auto bytes = token_bytes(id);
    int d = state();
    for (unsigned char c : bytes) {
      d = dfa_->step(d, c);
      if (d < 0) return false;
    }
    history_.push_back(d);
    return true;
  }
  bool accept_string(const std::string& s) {
    int d = state();
    for (unsigned char c : s) {
      d = dfa_->step(d, c);
      if (d < 0) return false;
    }
    history_.push_back(d);
    return true;
  }
  void rollback(int n) {
    for (int i = 0; i < n && history_.size() > 1; ++i) history_.pop_back();
    terminated_ = false;
  }
  // Bytes forced by the grammar from the current state (single successor chain).
  std::string forced_prefix(int max_len = 256) {
    std::string out;
    int d = state();
    for (int i = 0; i < max_len; ++i) {
      if (dfa_->accepting(d)) break;
      int only = -1, cnt = 0, nxt = -1;
      for (int b = 0; b < 256 && cnt < 2; ++b) {
        int t = dfa_->step(d, (unsigned char)b);
        if (t >= 0) {
          ++cnt;
          only = b;
          nxt = t;
        }
      }
      if (cnt != 1) break;
      out.push_back((char)only);
      d = nxt;
    }
    return out;
  }
  size_t dfa_states() const { return dfa_->num_states(); }

  std::vector<unsigned char> token_bytes(int id) {
    // recover the token's bytes from the trie (built once per vocab)
    if (tok_bytes_.empty()) {
      tok_bytes_.resize(vocab_->size());
      std::vector<std::pair<int, std::string>> stack{{0, ""}};
      while (!stack.empty()) {
        auto [n, s] = stack.back();
        stack.pop_back();
        for (int i : vocab_->nodes_[n].ids) tok_bytes_[i] = s;
        for (auto& kv : vocab_->nodes_[n].kids) stack.push_back({kv.second, s + (char)kv.first});
      }
    }
    const std::string& s = tok_bytes_[id];
    return std::vector<unsigned char>(s.begin(), s.end());
  }

 private:
  std::shared_ptr<Vocab> vocab_;
  std::shared_ptr<Dfa> dfa_;
  std::vector<int> history_;
  bool terminated_ = false;
  std::unordered_map<int, std::vector<uint32_t>> cache_;
  std::vector<std::string> tok_bytes_;

  std::vector<uint32_t> compute(int d) {
    std::vector<uint32_t> m((vocab_->size() + 31) / 32, 0u);
    // DFS over the trie carrying the DFA state
    std::vector<std::pair<int, int>> stack{{0, d}};
    while (!stack.empty()) {
      auto [node, st] = stack.back();
      stack.pop_back();
      if (node != 0)
        for (int id : vocab_->nodes_[node].ids) m[id >> 5] |= 1u << (id & 31);
      for (auto& kv : vocab_->nodes_[node].kids) {
        const int nx = dfa_->step(st, kv.first);
        if (nx >= 0) stack.push_back({kv.second, nx});
      }
    }
    if (dfa_->accepting(d))
      for (int e : vocab_->eos()) m[e >> 5] |= 1u << (e & 31);
    return m;
  }
};

}  // namespace b200host

void register_grammar(py::module_& m) {
  using namespace b200host;
  py::class_<Vocab, std::shared_ptr<Vocab>>(m, "GrammarVocab")
      .def(py::init<const std::vector<py::bytes>&, std::vector<int>>(), py::arg("tokens"), py::arg("eos_ids"))
      .def_property_readonly("size", &Vocab::size);
  py::class_<Matcher>(m, "GrammarMatcher")
      .def(py::init<std::shared_ptr<Vocab>, const std::string&>(), py::arg("vocab"), py::arg("regex"))
      .def("mask", &Matcher::mask)
      .def("accept_token", &Matcher::accept_token)
      .def("accept_string", &Matcher::accept_string)
      .def("rollback", &Matcher::rollback)
      .def("forced_prefix", &Matcher::forced_prefix, py::arg("max_len") = 256)
      .def("is_accepting", &Matcher::is_accepting)
      .def("is_terminated", &Matcher::is_terminated)
      .def_property_readonly("dfa_states", &Matcher::dfa_states)
      .def_property_readonly("state", &Matcher::state);
}
