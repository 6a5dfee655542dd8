#include "schema_matcher.h"

#include <algorithm>
#include <cstring>
#include <stdexcept>

namespace bloom {
namespace rt {

namespace {

constexpr uint8_t kMaxWs = 8;  // longest run of insignificant whitespace

bool is_ws(uint8_t c) { return c == ' ' || c == '\t' || c == '\n' || c == '\r'; }
bool is_digit(uint8_t c) { return c >= '0' && c <= '9'; }
bool is_hex(uint8_t c) { return is_digit(c) || (c >= 'a' && c <= 'f') || (c >= 'A' && c <= 'F'); }

bool seen_bit(const MatchFrame& f, int i) { return i < 64 && ((f.seen >> i) & 1ull); }

// number grammar: -? (0 | [1-9][0-9]*) (. [0-9]+)? ([eE] [+-]? [0-9]+)?
// states: 0 start, 1 '-', 2 leading 0, 3 int digits, 4 '.', 5 frac, 6 'e', 7 exp sign, 8 exp digits
int number_next(int st, uint8_t c, bool int_only) {
  switch (st) {
    case 0:
      if (c == '-') return 1;
      if (c == '0') return 2;
      if (c >= '1' && c <= '9') return 3;
      return -1;
    case 1:
      if (c == '0') return 2;
      if (c >= '1' && c <= '9') return 3;
      return -1;
    case 2:
    case 3:
      if (st == 3 && is_digit(c)) return 3;
      if (int_only) return -1;
      if (c == '.') return 4;
      if (c == 'e' || c == 'E') return 6;
      return -1;
    case 4:
      return is_digit(c) ? 5 : -1;
    case 5:
      if (is_digit(c)) return 5;
      if (c == 'e' || c == 'E') return 6;
      return -1;
    case 6:
      if (c == '+' || c == '-') return 7;
      return is_digit(c) ? 8 : -1;
    case 7:
    case 8:
      return is_digit(c) ? 8 : -1;
  }
  return -1;
}
bool number_accepting(int st) { return st == 2 || st == 3 || st == 5 || st == 8; }

}  // namespace

// ---------------------------------------------------------------- trie
VocabTrie::VocabTrie(const std::vector<std::string>& tokens, const std::vector<int32_t>& excluded) {
  vocab_ = static_cast<int>(tokens.size());
  std::vector<uint8_t> skip(tokens.size(), 0);
  for (int32_t e : excluded)
    if (e >= 0 && e < vocab_) skip[e] = 1;
  // sort token ids by bytes, then build the trie in one pass (children in byte order)
  std::vector<int32_t> order;
  order.reserve(tokens.size());
  for (int32_t i = 0; i < vocab_; ++i) {
    if (skip[i]) continue;
    if (tokens[i].empty()) {
      empty_tokens.push_back(i);
      continue;
    }
    order.push_back(i);
  }
  std::sort(order.begin(), order.end(), [&](int32_t a, int32_t b) {
    if (tokens[a] != tokens[b]) return tokens[a] < tokens[b];
    return a < b;
  });
  nodes_.push_back({0, -1, -1, -1, 0});  // root
  std::vector<int32_t> path{0};            // node of each prefix length of the previous token
  std::vector<int32_t> last_child;         // last child of each node (for sibling links)
  last_child.push_back(-1);
  std::string prev;
  // tokens ending at a node are collected afterwards (ids sorted per node)
  std::vector<std::pair<int32_t, int32_t>> ends;  // (node, token id)
  for (int32_t id : order) {
    const std::string& t = tokens[id];
    size_t common = 0;
    while (common < prev.size() && common < t.size() && prev[common] == t[common]) ++common;
    path.resize(common + 1);
    for (size_t k = common; k < t.size(); ++k) {
      const int32_t parent = path[k];
      const int32_t n = static_cast<int32_t>(nodes_.size());
      nodes_.push_back({static_cast<uint8_t>(t[k]), -1, -1, -1, 0});
      last_child.push_back(-1);
      if (nodes_[parent].first_child < 0)
        nodes_[parent].first_child = n;
      else
        nodes_[last_child[parent]].next_sibling = n;
      last_child[parent] = n;
      path.push_back(n);
    }
    ends.emplace_back(path[t.size()], id);
    prev = t;
  }
  std::stable_sort(ends.begin(), ends.end(), [](const auto& a, const auto& b) { return a.first < b.first; });
  token_ids_.reserve(ends.size());
  for (size_t i = 0; i < ends.size(); ++i) {
    Node& nd = nodes_[ends[i].first];
    if (nd.first_token < 0) nd.first_token = static_cast<int32_t>(token_ids_.size());
    ++nd.num_tokens;
    token_ids_.push_back(ends[i].second);
  }
}

// ---------------------------------------------------------------- matcher
SchemaMatcher::SchemaMatcher(std::vector<SchemaNode> nodes, int root) : nodes_(std::move(nodes)), root_(root) {
  if (root_ >= static_cast<int>(nodes_.size())) throw std::invalid_argument("SchemaMatcher: root out of range");
  for (const SchemaNode& n : nodes_) {
    if (n.prop_keys.size() != n.prop_nodes.size() || n.prop_keys.size() != n.prop_required.size())
      throw std::invalid_argument("SchemaMatcher: property arrays differ in length");
    if (n.prop_keys.size() > 64) throw std::invalid_argument("SchemaMatcher: at most 64 properties per object");
    for (int c : n.prop_nodes)
      if (c >= static_cast<int>(nodes_.size())) throw std::invalid_argument("SchemaMatcher: property node out of range");
    if (n.items >= static_cast<int>(nodes_.size())) throw std::invalid_argument("SchemaMatcher: items out of range");
  }
  st_.pending = root_;
}

bool SchemaMatcher::end_scalar(MatchState& s) const {
  s.sk = MatchState::S_NONE;
  s.text.clear();
  s.lit = nullptr;
  s.esc = 0;
  s.num = 0;
  s.phase = s.stack.empty() ? MatchState::P_DONE : MatchState::P_AFTER_VALUE;
  return true;
}

bool SchemaMatcher::start_value(MatchState& s, uint8_t c) const {
  const SchemaNode* n = node(s.pending);
  const uint32_t ty = n ? n->types : 0u;
  auto allows = [&](uint32_t bits) { return ty == 0u || (ty & bits) != 0u; };
  if (s.stack.empty() && c != '{') return false;  // the document is an object
  if (n && !n->enum_lits.empty()) {
    bool any = false;
    for (const std::string& e : n->enum_lits) any |= (!e.empty() && static_cast<uint8_t>(e[0]) == c);
    if (!any) return false;
    s.sk = MatchState::S_ENUM;
    s.text.assign(1, static_cast<char>(c));
    s.phase = MatchState::P_SCALAR;
    // a one-character literal that is self-delimiting cannot occur; numbers end on a delimiter
    return true;
  }
  switch (c) {
    case '{':
      if (!allows(kTypeObject)) return false;
      s.stack.push_back({s.pending, '{', 0ull, -1});
      s.phase = MatchState::P_KEY_OR_END;
      return true;
    case '[':
      if (!allows(kTypeArray)) return false;
      s.stack.push_back({s.pending, '[', 0ull, -1});
      s.phase = MatchState::P_VALUE_OR_END;
      return true;
    case '"':
      if (!allows(kTypeString)) return false;
      s.sk = MatchState::S_STRING;
      s.esc = 0;
      s.phase = MatchState::P_SCALAR;
      return true;
    case 't':
    case 'f':
      if (!allows(kTypeBoolean)) return false;
      s.sk = MatchState::S_LITERAL;
      s.lit = c == 't' ? "rue" : "alse";
      s.phase = MatchState::P_SCALAR;
      return true;
    case 'n':
      if (!allows(kTypeNull)) return false;
      s.sk = MatchState::S_LITERAL;
      s.lit = "ull";
      s.phase = MatchState::P_SCALAR;
      return true;
    default:
      break;
  }
  if (c == '-' || is_digit(c)) {
    if (!allows(kTypeNumber | kTypeInteger)) return false;
    s.int_only = ty != 0u && (ty & kTypeInteger) && !(ty & kTypeNumber);
    const int nx = number_next(0, c, s.int_only);
    if (nx < 0) return false;
    s.sk = MatchState::S_NUMBER;
    s.num = static_cast<uint8_t>(nx);
    s.phase = MatchState::P_SCALAR;
    return true;
  }
  return false;
}

// Characters outside scalars: whitespace, brackets, commas, colons, value starts.
bool SchemaMatcher::structural(MatchState& s, uint8_t c) const {
  using S = MatchState;
  if (is_ws(c)) {
    if (s.ws >= kMaxWs) return false;
    ++s.ws;
    return true;
  }
  s.ws = 0;
  auto close_container = [&](char kind) {
    if (s.stack.empty() || s.stack.back().kind != kind) return false;
    s.stack.pop_back();
    s.phase = s.stack.empty() ? S::P_DONE : S::P_AFTER_VALUE;
    return true;
  };
  auto required_done = [&](const MatchFrame& f) {
    const SchemaNode* n = node(f.node);
    if (!n) return true;
    for (size_t i = 0; i < n->prop_keys.size(); ++i)
      if (n->prop_required[i] && !seen_bit(f, static_cast<int>(i))) return false;
    return true;
  };
  auto key_possible = [&](const MatchFrame& f) {
    const SchemaNode* n = node(f.node);
    if (!n || n->additional) return true;
    for (size_t i = 0; i < n->prop_keys.size(); ++i)
      if (!seen_bit(f, static_cast<int>(i))) return true;
    return false;
  };
  auto start_key = [&]() {
    const MatchFrame& f = s.stack.back();
    if (!key_possible(f)) return false;
    const SchemaNode* n = node(f.node);
    s.sk = S::S_KEY;
    s.key_free = !n || n->additional;
    s.text.clear();
    s.esc = 0;
    s.phase = S::P_SCALAR;
    return true;
  };
  switch (s.phase) {
    case S::P_VALUE:
      return start_value(s, c);
    case S::P_VALUE_OR_END: {
      if (c == ']') return close_container('[');
      const SchemaNode* n = node(s.stack.back().node);
      s.pending = n ? n->items : -1;
      return start_value(s, c);
    }
    case S::P_KEY_OR_END:
      if (c == '}') return required_done(s.stack.back()) && close_container('{');
      return c == '"' && start_key();
    case S::P_KEY:
      return c == '"' && start_key();
    case S::P_COLON: {
      if (c != ':') return false;
      const MatchFrame& f = s.stack.back();
      const SchemaNode* n = node(f.node);
      s.pending = (n && f.cur >= 0) ? n->prop_nodes[f.cur] : -1;
      s.phase = S::P_VALUE;
      return true;
    }
    case S::P_AFTER_VALUE: {
      MatchFrame& f = s.stack.back();
      if (f.kind == '{') {
        if (c == ',') {
          if (!key_possible(f)) return false;
          s.phase = S::P_KEY;
          return true;
        }
        if (c == '}') return required_done(f) && close_container('{');
        return false;
      }
      if (c == ',') {
        const SchemaNode* n = node(f.node);
        s.pending = n ? n->items : -1;
        s.phase = S::P_VALUE;
        return true;
      }
      if (c == ']') return close_container('[');
      return false;
    }
    case S::P_DONE:
    case S::P_SCALAR:
      return false;
  }
  return false;
}

bool SchemaMatcher::step(MatchState& s, uint8_t c) const {
  using S = MatchState;
  if (s.phase != S::P_SCALAR) return structural(s, c);
  switch (s.sk) {
    case S::S_STRING:
    case S::S_KEY: {
      bool closed = false;
      if (s.esc == 0) {
        if (c == '"') {
          closed = true;
        } else if (c == '\\') {
          s.esc = 1;
        } else if (c < 0x20) {
          return false;
        }
      } else if (s.esc == 1) {
        if (c == 'u') {
          s.esc = 6;
        } else if (c == '"' || c == '\\' || c == '/' || c == 'b' || c == 'f' || c == 'n' || c == 'r' || c == 't') {
          s.esc = 0;
        } else {
          return false;
        }
      } else {
        if (!is_hex(c)) return false;
        if (--s.esc == 2) s.esc = 0;
      }
      if (s.sk == S::S_STRING) {
        if (closed) return end_scalar(s);
        return true;
      }
      // object key
      MatchFrame& f = s.stack.back();
      const SchemaNode* n = node(f.node);
      if (!closed) {
        s.text.push_back(static_cast<char>(c));
        if (s.key_free || !n) return true;
        for (size_t i = 0; i < n->prop_keys.size(); ++i)
          if (!seen_bit(f, static_cast<int>(i)) && n->prop_keys[i].compare(0, s.text.size(), s.text) == 0) return true;
        return false;
      }
      if (s.esc != 0) return false;
      int idx = -1;
      if (n)
        for (size_t i = 0; i < n->prop_keys.size(); ++i)
          if (n->prop_keys[i] == s.text) {
            idx = static_cast<int>(i);
            break;
          }
      if (idx >= 0) {
        if (seen_bit(f, idx)) return false;  // duplicate property
        f.seen |= 1ull << idx;
      } else if (!s.key_free) {
        return false;
      }
      f.cur = idx;
      s.sk = S::S_NONE;
      s.text.clear();
      s.phase = S::P_COLON;
      return true;
    }
    case S::S_NUMBER: {
      const int nx = number_next(s.num, c, s.int_only);
      if (nx >= 0) {
        s.num = static_cast<uint8_t>(nx);
        return true;
      }
      if (!number_accepting(s.num)) return false;
      end_scalar(s);
      return structural(s, c);
    }
    case S::S_LITERAL:
      if (s.lit == nullptr || *s.lit != static_cast<char>(c)) return false;
      ++s.lit;
      if (*s.lit == '\0') return end_scalar(s);
      return true;
    case S::S_ENUM: {
      const SchemaNode* n = node(s.pending);
      std::string nt = s.text;
      nt.push_back(static_cast<char>(c));
      bool prefix = false, exact_closed = false, longer = false;
      for (const std::string& e : n->enum_lits) {
        if (e.compare(0, nt.size(), nt) == 0) {
          prefix = true;
          if (e.size() == nt.size()) {
            const char last = e.back();
            exact_closed |= (last == '"' || last == '}' || last == ']');
          } else {
            longer = true;
          }
        }
      }
      if (prefix) {
        s.text.swap(nt);
        if (exact_closed && !longer) return end_scalar(s);
        return true;
      }
      // the literal so far must be complete; c then belongs to the structure
      bool exact = false;
      for (const std::string& e : n->enum_lits) exact |= (e == s.text);
      if (!exact) return false;
      end_scalar(s);
      return structural(s, c);
    }
    case S::S_NONE:
      break;
  }
  return false;
}

bool SchemaMatcher::feed(const std::string& text) {
  MatchState t = st_;
  for (unsigned char c : text)
    if (!step(t, c)) return false;
  st_ = std::move(t);
  return true;
}

std::string SchemaMatcher::state_key() const {
  const MatchState& s = st_;
  std::string k;
  k.reserve(64 + s.stack.size() * 24 + s.text.size());
  auto put = [&](const void* p, size_t n) { k.append(static_cast<const char*>(p), n); };
  const uint8_t hdr[8] = {static_cast<uint8_t>(s.phase), static_cast<uint8_t>(s.sk), s.esc, s.num,
                          static_cast<uint8_t>(s.int_only), static_cast<uint8_t>(s.key_free), s.ws, 0};
  put(hdr, sizeof hdr);
  put(&s.pending, sizeof s.pending);
  const uint32_t depth = static_cast<uint32_t>(s.stack.size());
  put(&depth, sizeof depth);
  for (const MatchFrame& f : s.stack) {
    put(&f.node, sizeof f.node);
    put(&f.kind, 1);
    put(&f.seen, sizeof f.seen);
    put(&f.cur, sizeof f.cur);
  }
  if (s.sk == MatchState::S_LITERAL && s.lit) k.append(s.lit);
  if (s.sk == MatchState::S_ENUM) k.append(s.text);
  if (s.sk == MatchState::S_KEY) {
    // a free key that can no longer become a declared name behaves like any other free key
    bool matters = !s.key_free;
    if (!matters) {
      const SchemaNode* n = node(s.stack.back().node);
      if (n)
        for (const std::string& p : n->prop_keys) matters |= p.compare(0, s.text.size(), s.text) == 0;
    }
    if (matters) {
      k.push_back('\x01');
      k.append(s.text);
    }
  }
  return k;
}

const std::vector<uint32_t>& SchemaMatcher::mask(const VocabTrie& trie, const std::vector<int32_t>& eos) {
  const std::string key = state_key();
  auto it = cache_.find(key);
  if (it != cache_.end()) {
    ++hits_;
    return it->second;
  }
  ++misses_;
  const int V = trie.vocab_size();
  std::vector<uint32_t> m(static_cast<size_t>((V + 31) / 32), 0u);
  const auto& nodes = trie.nodes();
  const auto& ids = trie.token_ids();
  // depth-first walk; states[d] is the state after the first d bytes of the current path
  std::vector<MatchState> states(1, st_);
  struct Item {
    int32_t node;
    int depth;
  };
  std::vector<Item> todo;
  for (int32_t c = nodes[0].first_child; c >= 0; c = nodes[c].next_sibling) todo.push_back({c, 0});
  std::reverse(todo.begin(), todo.end());
  while (!todo.empty()) {
    const Item it2 = todo.back();
    todo.pop_back();
    if (static_cast<int>(states.size()) < it2.depth + 2) states.resize(it2.depth + 2);
    states[it2.depth + 1] = states[it2.depth];
    if (!step(states[it2.depth + 1], nodes[it2.node].byte)) continue;
    const auto& nd = nodes[it2.node];
    for (int32_t j = 0; j < nd.num_tokens; ++j) {
      const int32_t t = ids[nd.first_token + j];
      m[t >> 5] |= 1u << (t & 31);
    }
    const size_t mark = todo.size();
    for (int32_t c = nd.first_child; c >= 0; c = nodes[c].next_sibling) todo.push_back({c, it2.depth + 1});
    std::reverse(todo.begin() + mark, todo.end());
  }
  if (complete())
    for (int32_t e : eos)
      if (e >= 0 && e < V) m[e >> 5] |= 1u << (e & 31);
  auto res = cache_.emplace(key, std::move(m));
  return res.first->second;
}

}  // namespace rt
}  // namespace bloom

// ---------------------------------------------------------------- Python surface
#ifndef BLOOM_NO_PYTHON
#include <pybind11/pybind11.h>
#include <pybind11/stl.h>
#include <torch/extension.h>

namespace py = pybind11;

void register_schema(py::module_& m) {
  using namespace bloom::rt;
  py::class_<SchemaNode>(m, "SchemaNode")
      .def(py::init<>())
      .def_readwrite("types", &SchemaNode::types)
      .def_readwrite("enum_lits", &SchemaNode::enum_lits)
      .def_readwrite("prop_keys", &SchemaNode::prop_keys)
      .def_readwrite("prop_nodes", &SchemaNode::prop_nodes)
      .def_readwrite("prop_required", &SchemaNode::prop_required)
      .def_readwrite("additional", &SchemaNode::additional)
      .def_readwrite("items", &SchemaNode::items);
  py::class_<VocabTrie, std::shared_ptr<VocabTrie>>(m, "VocabTrie")
      .def(py::init([](const std::vector<py::bytes>& toks, const std::vector<int32_t>& excluded) {
             std::vector<std::string> t;
             t.reserve(toks.size());
             for (const py::bytes& b : toks) t.emplace_back(b);
             return std::make_shared<VocabTrie>(t, excluded);
           }),
           py::arg("tokens"), py::arg("excluded") = std::vector<int32_t>{})
      .def_property_readonly("vocab_size", &VocabTrie::vocab_size)
      .def_property_readonly("num_nodes", [](const VocabTrie& t) { return t.nodes().size(); });
  py::class_<SchemaMatcher>(m, "SchemaMatcher")
      .def(py::init<std::vector<SchemaNode>, int>(), py::arg("nodes"), py::arg("root"))
      .def("feed", [](SchemaMatcher& s, const py::bytes& b) { return s.feed(std::string(b)); })
      .def("complete", &SchemaMatcher::complete)
      .def("state_key", [](const SchemaMatcher& s) { return py::bytes(s.state_key()); })
      .def_property_readonly("cache_hits", &SchemaMatcher::cache_hits)
      .def_property_readonly("cache_misses", &SchemaMatcher::cache_misses)
      .def(
          "mask_into",
          [](SchemaMatcher& s, const VocabTrie& trie, const std::vector<int32_t>& eos, torch::Tensor out) {
            TORCH_CHECK(out.device().is_cpu() && out.scalar_type() == at::kInt && out.is_contiguous(),
                        "out must be a contiguous host int32 tensor");
            const std::vector<uint32_t>* m = nullptr;
            {
              py::gil_scoped_release nogil;
              m = &s.mask(trie, eos);
            }
            TORCH_CHECK(out.numel() >= static_cast<int64_t>(m->size()), "out holds fewer words than the mask");
            std::memcpy(out.data_ptr(), m->data(), m->size() * sizeof(uint32_t));
          },
          py::arg("trie"), py::arg("eos"), py::arg("out"));
}
#endif  // BLOOM_NO_PYTHON
