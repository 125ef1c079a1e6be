// Vocabulary trie shared by the grammar matchers (regex DFA and pushdown):
// every token id's byte string, and a trie over them whose nodes list the ids
// that end there. Special / unrepresentable tokens (empty strings) never match
// text; EOS ids are allowed only where a grammar accepts.
#pragma once
#include <pybind11/pybind11.h>

#include <map>
#include <string>
#include <vector>

namespace b200host {

class Vocab {
 public:
  Vocab(const std::vector<pybind11::bytes>& tokens, std::vector<int> eos) : eos_(std::move(eos)) {
    n_ = (int)tokens.size();
    bytes_.resize(n_);
    nodes_.push_back(Node{});
    parent_.push_back(-1);
    byte_.push_back(0);
    for (int id = 0; id < n_; ++id) {
      std::string s = tokens[id];
      bytes_[id] = s;
      if (s.empty()) continue;
      int cur = 0;
      for (unsigned char c : s) {
        auto it = nodes_[cur].kids.find(c);
        if (it == nodes_[cur].kids.end()) {
          nodes_.push_back(Node{});
          parent_.push_back(cur);
          byte_.push_back(c);
          nodes_[cur].kids[c] = (int)nodes_.size() - 1;
          cur = (int)nodes_.size() - 1;
        } else {
          cur = it->second;
        }
      }
      nodes_[cur].ids.push_back(id);
    }
  }
  int size() const { return n_; }
  const std::vector<int>& eos() const { return eos_; }
  bool is_eos(int id) const {
    for (int e : eos_)
      if (e == id) return true;
    return false;
  }
  const std::string& bytes(int id) const { return bytes_[id]; }
  // bytes from the trie root to trie node `node`
  std::string path(int node) const {
    std::string out;
    for (int n = node; n > 0; n = parent_[n]) out.push_back((char)byte_[n]);
    return std::string(out.rbegin(), out.rend());
  }
  struct Node {
    std::map<unsigned char, int> kids;
    std::vector<int> ids;
  };
  std::vector<Node> nodes_;

 private:
  int n_;
  std::vector<int> eos_;
  std::vector<std::string> bytes_;
  std::vector<int> parent_;
  std::vector<unsigned char> byte_;
};

}  // namespace b200host
