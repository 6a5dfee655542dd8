// Incremental JSON recogniser for structured output (JSON mode).
//
// The state is a small pushdown automaton over characters: a stack of open
// containers plus a scalar-lexer state.  `feed` consumes a candidate token's
// text and fails without changing the state when the text cannot continue a
// valid JSON document; `complete` tells whether the document is finished.
// The decoder keeps one state per request and, at every step, tries the
// highest-scoring candidate tokens in order: the first that keeps the prefix
// valid is emitted; end-of-sequence is allowed only once the document is
// complete; if no candidate is valid the step falls back to the unconstrained
// choice (reference behaviour: crates/engine/src/executor/candle.rs:2884-3243,
// JsonDfa + filter_logits_by_grammar with top-256 candidates and EOS gating).
#include <pybind11/pybind11.h>
#include <pybind11/stl.h>

#include <cstdint>
#include <string>
#include <vector>

namespace py = pybind11;

namespace {

enum Lex : uint8_t {
  L_VALUE,         // expecting a value
  L_AFTER_VALUE,   // a value just ended (expect , } ] or whitespace)
  L_KEY_OR_END,    // after '{' : expecting key string or '}'
  L_KEY,           // after ',' in object: expecting key string
  L_COLON,         // after key: expecting ':'
  L_STRING,        // inside a string
  L_STRING_ESC,    // after backslash
  L_STRING_U,      // inside \uXXXX (count in ucount)
  L_NUMBER,        // inside a number
  L_LITERAL,       // inside true/false/null
  L_DONE,          // top-level value complete
  L_VALUE_OR_END,  // after '[' : expecting value or ']'
};

struct State {
  std::vector<char> stack;  // '{' or '['
  Lex lex = L_VALUE;
  bool string_is_key = false;
  uint8_t ucount = 0;
  std::string lit;       // remaining literal chars
  std::string num;       // number chars so far
};

bool num_can_end(const std::string& n) {
  if (n.empty()) return false;
  const char c = n.back();
  return (c >= '0' && c <= '9');
}

bool num_accept(std::string& n, char c) {
  // grammar: -? (0 | [1-9][0-9]*) (. [0-9]+)? ([eE] [+-]? [0-9]+)?
  const bool has_dot = n.find('.') != std::string::npos;
  const bool has_e = n.find_first_of("eE") != std::string::npos;
  const char last = n.empty() ? '\0' : n.back();
  if (c >= '0' && c <= '9') {
    if ((last == '0') && (n == "0" || n == "-0")) return false;  // no leading zeros
    n.push_back(c);
    return true;
  }
  if (c == '-') {
    if (n.empty() || last == 'e' || last == 'E') {
      n.push_back(c);
      return true;
    }
    return false;
  }
  if (c == '+') {
    if (last == 'e' || last == 'E') {
      n.push_back(c);
      return true;
    }
    return false;
  }
  if (c == '.') {
    if (!has_dot && !has_e && last >= '0' && last <= '9') {
      n.push_back(c);
      return true;
    }
    return false;
  }
  if (c == 'e' || c == 'E') {
    if (!has_e && last >= '0' && last <= '9') {
      n.push_back(c);
      return true;
    }
    return false;
  }
  return false;
}

void value_ended(State& s) { s.lex = s.stack.empty() ? L_DONE : L_AFTER_VALUE; }

bool step(State& s, char c) {
  const bool ws = c == ' ' || c == '\n' || c == '\t' || c == '\r';
  switch (s.lex) {
    case L_DONE:
      return ws;
    case L_VALUE:
    case L_VALUE_OR_END:
      if (ws) return true;
      if (c == ']' && s.lex == L_VALUE_OR_END) {
        s.stack.pop_back();
        value_ended(s);
        return true;
      }
      if (c == '{') {
        s.stack.push_back('{');
        s.lex = L_KEY_OR_END;
        return true;
      }
      if (c == '[') {
        s.stack.push_back('[');
        s.lex = L_VALUE_OR_END;
        return true;
      }
      if (c == '"') {
        s.lex = L_STRING;
        s.string_is_key = false;
        return true;
      }
      if (c == '-' || (c >= '0' && c <= '9')) {
        s.num.clear();
        s.lex = L_NUMBER;
        return num_accept(s.num, c);
      }
      if (c == 't') { s.lit = "rue"; s.lex = L_LITERAL; return true; }
      if (c == 'f') { s.lit = "alse"; s.lex = L_LITERAL; return true; }
      if (c == 'n') { s.lit = "ull"; s.lex = L_LITERAL; return true; }
      return false;
    case L_LITERAL:
      if (!s.lit.empty() && c == s.lit[0]) {
        s.lit.erase(0, 1);
        if (s.lit.empty()) value_ended(s);
        return true;
      }
      return false;
    case L_NUMBER:
      if (num_accept(s.num, c)) return true;
      if (!num_can_end(s.num)) return false;
      value_ended(s);
      return step(s, c);
    case L_STRING:
      if (c == '"') {
        if (s.string_is_key) {
          s.lex = L_COLON;
        } else {
          value_ended(s);
        }
        return true;
      }
      if (c == '\\') {
        s.lex = L_STRING_ESC;
        return true;
      }
      return static_cast<unsigned char>(c) >= 0x20;
    case L_STRING_ESC:
      if (c == 'u') {
        s.lex = L_STRING_U;
        s.ucount = 0;
        return true;
      }
      if (c == '"' || c == '\\' || c == '/' || c == 'b' || c == 'f' || c == 'n' || c == 'r' || c == 't') {
        s.lex = L_STRING;
        return true;
      }
      return false;
    case L_STRING_U:
      if ((c >= '0' && c <= '9') || (c >= 'a' && c <= 'f') || (c >= 'A' && c <= 'F')) {
        if (++s.ucount == 4) s.lex = L_STRING;
        return true;
      }
      return false;
    case L_KEY_OR_END:
    case L_KEY:
      if (ws) return true;
      if (c == '}' && s.lex == L_KEY_OR_END) {
        s.stack.pop_back();
        value_ended(s);
        return true;
      }
      if (c == '"') {
        s.lex = L_STRING;
        s.string_is_key = true;
        return true;
      }
      return false;
    case L_COLON:
      if (ws) return true;
      if (c == ':') {
        s.lex = L_VALUE;
        return true;
      }
      return false;
    case L_AFTER_VALUE:
      if (ws) return true;
      if (c == ',') {
        s.lex = s.stack.back() == '{' ? L_KEY : L_VALUE;
        return true;
      }
      if ((c == '}' && s.stack.back() == '{') || (c == ']' && s.stack.back() == '[')) {
        s.stack.pop_back();
        value_ended(s);
        return true;
      }
      return false;
  }
  return false;
}

class JsonDfa {
 public:
  bool feed(const std::string& text) {
    State t = s_;
    for (char c : text)
      if (!step(t, c)) return false;
    s_ = std::move(t);
    return true;
  }
  bool can_feed(const std::string& text) const {
    State t = s_;
    for (char c : text)
      if (!step(t, c)) return false;
    return true;
  }
  bool complete() const {
    if (s_.lex == L_DONE) return true;
    // a top-level number may end at end of input
    return s_.stack.empty() && s_.lex == L_NUMBER && num_can_end(s_.num);
  }
  bool started() const { return !(s_.lex == L_VALUE && s_.stack.empty()); }
  int depth() const { return static_cast<int>(s_.stack.size()); }

  // First candidate (in the given order) that keeps the prefix valid; eos
  // candidates are accepted only when the document is complete.  -1: none.
  int pick(const std::vector<int>& cand, const std::vector<std::string>& vocab, const std::vector<int>& eos) const {
    for (int t : cand) {
      bool is_eos = false;
      for (int e : eos) is_eos |= (t == e);
      if (is_eos) {
        if (complete()) return t;
        continue;
      }
      if (t < 0 || t >= static_cast<int>(vocab.size())) continue;
      const std::string& s = vocab[t];
      if (s.empty()) continue;
      if (can_feed(s)) return t;
    }
    return -1;
  }

 private:
  State s_;
};

bool is_valid_json(const std::string& text) {
  JsonDfa d;
  return d.feed(text) && d.complete();
}

}  // namespace

void register_json(py::module_& m) {
  py::class_<JsonDfa>(m, "JsonDfa")
      .def(py::init<>())
      .def("feed", &JsonDfa::feed)
      .def("can_feed", &JsonDfa::can_feed)
      .def("complete", &JsonDfa::complete)
      .def("started", &JsonDfa::started)
      .def("depth", &JsonDfa::depth)
      .def("pick", &JsonDfa::pick, py::call_guard<py::gil_scoped_release>());
  m.def("is_valid_json", &is_valid_json);
}
