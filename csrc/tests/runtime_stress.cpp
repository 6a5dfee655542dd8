// Stress driver for the host runtime under sanitizers (no Python, no GPU).
//
//   scheduler   random requests (prompt lengths, priorities, stop tokens),
//               random aborts, failed steps, preemption policies, swap slots
//               and long-context policies, stepped until every request ends;
//               afterwards every KV block must be back in the pool
//   cachemesh   the block manager with pinned-host (here: heap) L2 slots and
//               an L3 directory, prefix reuse across many short requests
//   schema      random byte streams fed to the JSON Schema matcher, and mask
//               computation over a random vocabulary trie
//   pool        many small parallel_for jobs back to back (data races: TSan)
// Built and run by tests/test_sanitizers.py with -fsanitize=address,undefined
// (and the pool part with -fsanitize=thread); any sanitizer report or a
// violated invariant fails the run.
#include <cstdio>
#include <cstdlib>
#include <random>
#include <string>
#include <vector>

#include "../runtime/scheduler.h"
#include "../runtime/schema_matcher.h"
#include "../runtime/thread_pool.h"

using namespace bloom::rt;

#define CHECK(c)                                                     \
  do {                                                               \
    if (!(c)) {                                                      \
      std::fprintf(stderr, "CHECK failed %s:%d: %s\n", __FILE__, __LINE__, #c); \
      std::exit(3);                                                  \
    }                                                                \
  } while (0)

static int scheduler_stress(uint32_t seed, int policy, int swap_slots, int lc_policy) {
  std::mt19937 rng(seed);
  SchedulerConfig cfg;
  cfg.max_num_seqs = 8;
  cfg.max_num_batched_tokens = 96;
  cfg.max_model_len = 256;
  cfg.eos_token_ids = {2};
  cfg.victim_policy = policy;
  cfg.max_preemptions_per_request = policy % 2 ? 2 : 0;
  cfg.swap_slots = swap_slots;
  cfg.priority_preempt_ms = policy == 1 ? 0.0 : -1.0;
  cfg.kv_admission_threshold = policy == 3 ? 0.9 : 1.0;
  cfg.lc_policy = lc_policy;
  cfg.lc_window_tokens = 64;
  cfg.lc_target_free = 4;
  const int blocks = 20;
  Scheduler s(cfg, blocks, 16, seed % 2 == 0);
  const int MB = 16, T = 96 + 8;
  const StepMeta worst = arena_layout(T, 8, 8, T / 64 + 8, T + 8, MB);
  std::vector<int32_t> arena(static_cast<size_t>(worst.used_words) + 64);
  Arena a{arena.data(), static_cast<int64_t>(arena.size()), T, 8, MB};
  s.set_arena(a);
  s.set_clock_ms(0.0);
  std::vector<int64_t> ids;
  int added = 0;
  for (int step = 0; step < 4000 && (added < 60 || s.has_unfinished()); ++step) {
    s.set_clock_ms(step * 5.0);
    if (added < 60 && rng() % 3 == 0) {
      std::vector<int32_t> prompt(1 + rng() % 120);
      for (auto& t : prompt) t = 3 + static_cast<int32_t>(rng() % 40);  // small alphabet: prefix hits
      SamplingParams sp;
      sp.max_tokens = 1 + rng() % 40;
      sp.ignore_eos = rng() % 2;
      ids.push_back(s.add_request(prompt, sp, static_cast<int>(rng() % 4)));
      ++added;
    }
    if (!ids.empty() && rng() % 17 == 0) s.abort(ids[rng() % ids.size()]);
    StepMeta m = s.schedule();
    if (m.num_tokens == 0) continue;
    CHECK(m.used_words <= a.capacity);
    s.take_swap_ins();
    s.take_swap_outs();
    if (rng() % 29 == 0) {
      s.fail_scheduled();
      continue;
    }
    std::vector<int32_t> sampled(static_cast<size_t>(std::max(1, m.num_logits)));
    for (auto& t : sampled) t = rng() % 11 == 0 ? 2 : 3 + static_cast<int32_t>(rng() % 40);
    s.update(sampled.data(), m.num_real_logits);
  }
  CHECK(!s.has_unfinished());
  const PoolMetrics pm = s.blocks().metrics();
  CHECK(pm.active_blocks == 0);
  CHECK(pm.free_blocks + pm.cached_blocks == pm.total_blocks);
  CHECK(s.free_swap_slots() == swap_slots);
  return 0;
}

static int cachemesh_stress(uint32_t seed) {
  std::mt19937 rng(seed);
  const int64_t block_bytes = 256, slots = 6;
  std::vector<uint8_t> l2(static_cast<size_t>(block_bytes * slots));
  char dir[] = "/tmp/bloom-mesh-XXXXXX";
  CHECK(mkdtemp(dir) != nullptr);
  CacheMeshConfig mc;
  mc.l2_slots = slots;
  mc.block_bytes = block_bytes;
  mc.l3_dir = dir;
  mc.l3_max_blocks = 16;
  SchedulerConfig cfg;
  cfg.max_num_seqs = 4;
  cfg.max_num_batched_tokens = 64;
  cfg.max_model_len = 128;
  Scheduler s(cfg, 8, 16, true);
  s.enable_cachemesh(mc, l2.data());
  const StepMeta worst = arena_layout(64 + 4, 4, 4, 64 / 64 + 4, 64 + 4, 8);
  std::vector<int32_t> arena(static_cast<size_t>(worst.used_words) + 64);
  s.set_arena(Arena{arena.data(), static_cast<int64_t>(arena.size()), 68, 4, 8});
  std::vector<std::vector<int32_t>> prompts;
  for (int i = 0; i < 5; ++i) {
    std::vector<int32_t> p(17 + rng() % 60);
    for (auto& t : p) t = 3 + static_cast<int32_t>(rng() % 50);
    prompts.push_back(p);
  }
  for (int round = 0; round < 40; ++round) {
    SamplingParams sp;
    sp.max_tokens = 2;
    sp.ignore_eos = true;
    s.add_request(prompts[rng() % prompts.size()], sp, 0);
    while (s.has_unfinished()) {
      StepMeta m = s.schedule();
      s.blocks().take_restores();
      s.blocks().take_offloads();
      if (m.num_tokens == 0) continue;
      std::vector<int32_t> sampled(static_cast<size_t>(std::max(1, m.num_logits)), 7);
      s.update(sampled.data(), m.num_real_logits);
    }
  }
  CHECK(s.blocks().metrics().active_blocks == 0);
  std::string cmd = std::string("rm -rf ") + dir;
  CHECK(std::system(cmd.c_str()) == 0);
  return 0;
}

static int schema_fuzz(uint32_t seed) {
  std::mt19937 rng(seed);
  // {"name": string, "n": integer, "tags": [string], "ok": boolean} with required name
  std::vector<SchemaNode> nodes(4);
  nodes[0].types = kTypeObject;
  nodes[0].prop_keys = {"name", "n", "tags", "ok"};
  nodes[0].prop_nodes = {1, 2, 3, -1};
  nodes[0].prop_required = {1, 0, 0, 0};
  nodes[0].additional = false;
  nodes[1].types = kTypeString;
  nodes[2].types = kTypeInteger;
  nodes[3].types = kTypeArray;
  nodes[3].items = 1;
  const std::string alphabet = "{}[]\":,. -+eE0123456789abcdefnrtlsu\\\n";
  std::vector<std::string> vocab;
  for (int i = 0; i < 300; ++i) {
    std::string t(1 + rng() % 5, ' ');
    for (auto& c : t) c = alphabet[rng() % alphabet.size()];
    vocab.push_back(t);
  }
  vocab.push_back("");
  VocabTrie trie(vocab, {3});
  for (int round = 0; round < 200; ++round) {
    SchemaMatcher m(nodes, 0);
    for (int i = 0; i < 60; ++i) {
      const std::vector<uint32_t>& mk = m.mask(trie, {5});
      CHECK(mk.size() == (vocab.size() + 31) / 32);
      // follow the mask: pick an allowed token when there is one
      std::vector<int> allowed;
      for (size_t t = 0; t < vocab.size(); ++t)
        if ((mk[t >> 5] >> (t & 31)) & 1u) allowed.push_back(static_cast<int>(t));
      if (allowed.empty()) break;
      const int t = allowed[rng() % allowed.size()];
      if (t == 5) break;
      CHECK(m.feed(vocab[t]));  // a masked-in token always feeds
    }
    SchemaMatcher r(nodes, 0);
    for (int i = 0; i < 200; ++i) {  // arbitrary bytes never crash, rejected ones change nothing
      std::string b(1, static_cast<char>(rng() % 256));
      const std::string before = r.state_key();
      if (!r.feed(b)) CHECK(r.state_key() == before);
    }
  }
  return 0;
}

static int pool_stress() {
  std::vector<int64_t> data(1 << 14);
  for (int iter = 0; iter < 3000; ++iter) {
    const int64_t n = 1 + iter % 700;
    parallel_for(n, [&](int64_t b, int64_t e) {
      for (int64_t i = b; i < e; ++i) data[static_cast<size_t>(i)] += i;
    });
  }
  for (int64_t i = 0; i < 700; ++i) {
    int64_t uses = 0;
    for (int iter = 0; iter < 3000; ++iter) uses += (1 + iter % 700) > i;
    CHECK(data[static_cast<size_t>(i)] == uses * i);
  }
  return 0;
}

int main(int argc, char** argv) {
  const std::string what = argc > 1 ? argv[1] : "all";
  if (what == "pool") return pool_stress();
  for (uint32_t seed = 1; seed <= 12; ++seed)
    scheduler_stress(seed, static_cast<int>(seed % 7), seed % 3 == 0 ? 0 : 12, static_cast<int>(seed % 4));
  cachemesh_stress(7);
  schema_fuzz(11);
  pool_stress();
  std::printf("runtime stress ok\n");
  return 0;
}
