// JSON Schema constrained decoding: an incremental recogniser of JSON text
// that follows a compiled schema, and the per-step vocabulary mask it allows.
//
// Supported schema subset (the same keywords the HTTP layer accepts):
// type (object, array, string, number, integer, boolean, null), enum
// (canonical JSON literals), properties, required, additionalProperties
// (boolean), items.  A node id of -1 means "any JSON value".
//
// The recogniser is a pushdown automaton over bytes: a stack of open
// containers (each with its schema node, the properties already seen and the
// property whose value is being read) and a scalar lexer (string with
// escapes, number grammar, true/false/null, enum literal or property-name
// prefix matching).  Object keys are restricted to the declared properties
// when additionalProperties is false; '}' is accepted only once every
// required property has appeared; runs of insignificant whitespace are
// bounded so a constrained decoder cannot loop on blanks.
//
// `mask` evaluates every vocabulary token from the current state in one
// depth-first walk of a byte trie of the vocabulary (a subtree is skipped as
// soon as its prefix is rejected) and caches the result by a canonical
// serialisation of the state, so steps that revisit a state (e.g. the inside
// of a free string) cost a hash lookup.  The mask is uploaded and applied to
// the logits on the GPU before sampling.
//
// Reference behaviour: response-format validation and schema checks
// (crates/server/src/helpers.rs:2454-2960) and constrained decoding with a
// JSON DFA (crates/engine/src/executor/candle.rs:2584-3243).
#pragma once

#include <cstdint>
#include <memory>
#include <string>
#include <unordered_map>
#include <vector>

namespace bloom {
namespace rt {

struct SchemaNode {
  uint32_t types = 0;  // bit set of kType*; 0 = any type
  std::vector<std::string> enum_lits;  // canonical JSON texts ("\"red\"", "3", "true"); empty = any
  std::vector<std::string> prop_keys;  // property names as they appear between the quotes (escaped form)
  std::vector<int> prop_nodes;         // schema node of each property (-1 = any)
  std::vector<uint8_t> prop_required;
  bool additional = true;  // additionalProperties
  int items = -1;          // schema node of array items (-1 = any)
};

enum : uint32_t {
  kTypeObject = 1,
  kTypeArray = 2,
  kTypeString = 4,
  kTypeNumber = 8,
  kTypeInteger = 16,
  kTypeBoolean = 32,
  kTypeNull = 64,
};

// Byte trie over the vocabulary (shared by every matcher of one tokenizer).
class VocabTrie {
 public:
  // tokens[i] = the bytes token i decodes to; excluded ids (special tokens)
  // are never allowed by a mask.
  VocabTrie(const std::vector<std::string>& tokens, const std::vector<int32_t>& excluded);
  int vocab_size() const { return vocab_; }
  struct Node {
    uint8_t byte;
    int32_t first_child;  // index into nodes_, -1 none
    int32_t next_sibling;
    int32_t first_token;  // index into token_ids_ of the tokens ending here (-1 none)
    int32_t num_tokens;
  };
  const std::vector<Node>& nodes() const { return nodes_; }
  const std::vector<int32_t>& token_ids() const { return token_ids_; }
  std::vector<int32_t> empty_tokens;  // tokens that decode to no bytes

 private:
  int vocab_;
  std::vector<Node> nodes_;
  std::vector<int32_t> token_ids_;
};

struct MatchFrame {
  int32_t node;   // schema node of the container (-1 any)
  char kind;      // '{' or '['
  uint64_t seen;  // properties already present (bit i = prop_keys[i], i < 64)
  int32_t cur;    // property index of the value being read (-1: additional / unknown key)
};

// Recogniser state (small and copyable: the trie walk copies it per node).
struct MatchState {
  enum Phase : uint8_t {
    P_VALUE,         // a value of node `pending` must start
    P_AFTER_VALUE,   // a value ended inside a container
    P_KEY_OR_END,    // after '{'
    P_KEY,           // after ',' in an object
    P_COLON,         // after a key
    P_VALUE_OR_END,  // after '['
    P_DONE,          // top-level value complete
    P_SCALAR,        // inside a scalar or key (see sk)
  };
  enum Scalar : uint8_t { S_NONE, S_STRING, S_NUMBER, S_LITERAL, S_ENUM, S_KEY };
  std::vector<MatchFrame> stack;
  Phase phase = P_VALUE;
  int32_t pending = -1;   // node of the value about to start / being read
  Scalar sk = S_NONE;
  uint8_t esc = 0;        // string: 1 after a backslash, 2..5 inside \uXXXX
  uint8_t num = 0;        // number grammar state
  bool int_only = false;  // number must be an integer
  bool key_free = false;  // key text is not matched against declared names
  const char* lit = nullptr;  // literal: remaining characters
  std::string text;       // enum literal or key text so far
  uint8_t ws = 0;         // consecutive insignificant whitespace
};

class SchemaMatcher {
 public:
  // root = node id of the top-level schema (-1: any JSON object); the
  // top-level value must be an object either way.
  SchemaMatcher(std::vector<SchemaNode> nodes, int root);

  // Consume text; on failure the state is left unchanged and false returned.
  bool feed(const std::string& text);
  bool complete() const { return st_.phase == MatchState::P_DONE; }
  // Allowed-token bit mask (ceil(V / 32) words, bit t % 32 of word t / 32)
  // from the current state; end-of-sequence ids are allowed only when the
  // document is complete.
  const std::vector<uint32_t>& mask(const VocabTrie& trie, const std::vector<int32_t>& eos);
  int64_t cache_hits() const { return hits_; }
  int64_t cache_misses() const { return misses_; }
  std::string state_key() const;

  // one byte; false (state undefined) if rejected -- callers work on a copy
  bool step(MatchState& s, uint8_t c) const;

 private:
  bool start_value(MatchState& s, uint8_t c) const;
  bool end_scalar(MatchState& s) const;
  bool structural(MatchState& s, uint8_t c) const;
  const SchemaNode* node(int id) const { return id < 0 ? nullptr : &nodes_[id]; }

  std::vector<SchemaNode> nodes_;
  int root_;
  MatchState st_;
  std::unordered_map<std::string, std::vector<uint32_t>> cache_;
  int64_t hits_ = 0, misses_ = 0;
};

}  // namespace rt
}  // namespace bloom
