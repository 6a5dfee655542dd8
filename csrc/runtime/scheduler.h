// In-flight batching scheduler (host side, C++).
//
// One step = decode rows for every running sequence that only needs its last
// sampled token computed, then prefill rows (chunked) for partially computed
// and newly admitted sequences with the token budget that is left.  This is
// the step order of the reference scheduler (crates/engine/src/scheduler/
// mod.rs:1795-1845: preempt -> decode micro-batches -> prefill with leftover
// budget; chunked prefill :2042-2217), but here every scheduled row of every
// sequence goes into ONE batched forward: the step's metadata (token ids,
// positions, KV slots, block tables, attention tiles, sampling rows and
// sampling parameters) is written straight into pinned host buffers that the
// model runner copies to the device in one transfer.
//
// Preemption is by recompute (reference mod.rs:2001-2027): when the KV pool
// cannot grow a running sequence, the most recently admitted running
// sequence releases its blocks and goes back to the head of the wait queue.
// Stop conditions come from the model (EOS ids), never a hard-coded token id.
#pragma once

#include <chrono>
#include <cstdint>
#include <deque>
#include <memory>
#include <string>
#include <unordered_map>
#include <vector>

#include "block_manager.h"

namespace bloom {
namespace rt {

struct SamplingParams {
  float temperature = 0.f;  // <= 0: greedy
  float top_p = 1.f;
  int top_k = 0;
  int64_t seed = 0;
  int max_tokens = 128;
  int min_tokens = 0;
  bool ignore_eos = false;
  std::vector<int32_t> stop_token_ids;
};

enum class SeqStatus : int { Waiting = 0, Running = 1, Finished = 2 };
enum class FinishReason : int { None = 0, Stop = 1, Length = 2, Aborted = 3, Error = 4 };

struct Sequence {
  int64_t id = 0;
  std::vector<int32_t> tokens;
  int num_prompt = 0;
  int num_computed = 0;
  int num_cached_prefix = 0;
  std::vector<int32_t> table;
  std::vector<uint64_t> hashes;
  SamplingParams sp;
  SeqStatus status = SeqStatus::Waiting;
  FinishReason finish = FinishReason::None;
  int priority = 0;
  int64_t order = 0;
  std::vector<int32_t> draft;  // speculative proposals for the next verify step
  int num_preemptions = 0;
  bool admitted_once = false;
  bool verifying = false;  // scheduled as a verify group in the current step
  // swap preemption: host slots holding this sequence's first blocks while it waits
  std::vector<int32_t> swap_slots;
  bool swapped = false;
  double arrival_ms = 0.0;          // scheduler clock at add_request
  double last_scheduled_ms = 0.0;   // scheduler clock of the last step that ran it
  int num_generated() const { return static_cast<int>(tokens.size()) - num_prompt; }
};

// Which running sequence gives up its KV blocks when the pool cannot grow
// another one (recompute preemption).  Lower cost is chosen first; ties go to
// the most recently admitted sequence.
//   Newest       most recently admitted (the default)
//   Priority     lowest request priority           (reference PreemptionPolicy::Priority)
//   Oldest       most generated tokens             (PreemptionPolicy::Oldest: cost = -generated)
//   KvCost       fewest KV tokens (cheapest redo)  (PreemptionPolicy::KvCost)
//   AegaeonScore age x value / KV tokens: young sessions holding much KV
//                go first (priority_eviction.rs, Aegaeon section 5.2; value = 1)
//   Lru          longest since last scheduled      (KvEvictionPolicy::Lru)
//   LargestFirst most KV tokens                    (KvEvictionPolicy::LargestFirst)
// (reference: crates/core/src/token_scheduling/preemption.rs:20-64,136-240,
// priority_eviction.rs:38-74,173-312)
enum class VictimPolicy : int { Newest = 0, Priority = 1, Oldest = 2, KvCost = 3, AegaeonScore = 4, Lru = 5,
                                LargestFirst = 6 };

struct SchedulerConfig {
  int max_num_seqs = 256;
  int max_num_batched_tokens = 8192;
  int max_model_len = 4096;
  bool chunked_prefill = true;
  std::vector<int32_t> eos_token_ids;
  // Speculative decoding: every decode row becomes a verify row of
  // spec_len + 1 tokens (the last sampled token followed by spec_len
  // proposals; missing proposals are padded and always rejected).  0 = off.
  int spec_len = 0;
  // Long-context policy (reference: scheduler/paged_cache.rs:58-90, 443-464).
  // Full: attention sees every block.  SlidingWindow: only the blocks of the
  // last lc_window_tokens tokens.  ContextShift: only the blocks of the last
  // max(lc_max_context - lc_shift, block) tokens.  CompactInactive: all
  // blocks visible; before each step cached blocks no sequence holds are
  // evicted until lc_target_free blocks are free.  Visibility is per step
  // and whole blocks; the window never starts inside the tokens of the
  // current step, so every query still sees its own position.
  // Preemption: victim policy (VictimPolicy), per-request cap (a sequence
  // preempted this many times is not chosen again while another candidate
  // exists; 0 = no cap), and priority preemption: a waiting request whose
  // priority is above a running one and that has waited at least
  // priority_preempt_ms (< 0: off) may preempt lower-priority sequences to
  // get its KV blocks.
  int victim_policy = 0;
  int max_preemptions_per_request = 0;
  double priority_preempt_ms = -1.0;
  // KV admission threshold: no waiting request is admitted while the used
  // fraction of the KV pool is at or above it (reference
  // KvEvictionManager::check_admission, default 0.85 there; 1.0 = off here).
  double kv_admission_threshold = 1.0;
  // Swap preemption: host slots (one KV block each) that a preempted
  // sequence's blocks are copied into instead of being recomputed later
  // (0 = recompute preemption only; a victim whose blocks do not fit in the
  // free slots is recomputed).
  int swap_slots = 0;
  int lc_policy = 0;  // 0 full, 1 sliding window, 2 context shift, 3 compact inactive
  int lc_window_tokens = 0;
  int lc_max_context = 0;
  int lc_shift = 0;
  int lc_target_free = 0;
};

// Blocks of a table of `total_blocks` that a policy keeps visible.
int lc_window_blocks(const SchedulerConfig& c, int block_size, int total_blocks);

// The scheduler writes each step's metadata into ONE pinned int32 arena in a
// packed layout, so the runner moves it to the device with a single copy.
// Offsets (in 32-bit words) depend only on the row counts, so a decode-only
// step padded to a batch bucket has the same layout every time and can be
// replayed from a CUDA graph.  Region order:
//   input_ids[T] slot_mapping[T] positions[T] (int64, 8-byte aligned)
//   decode_seq_lens[Bd] decode_block_table[Bd * MB]
//   prefill_ctx_lens[Sp] prefill_cu_q[Sp + 1] prefill_block_table[Sp * MB]
//   tile_seq[NT] tile_start[NT]
//   logits_rows[NL] top_k[NL] temperature[NL] (f32) top_p[NL] (f32)
//   draft_ids[NL] seeds[NL] (int64, aligned) offsets[NL] (int64)
// With speculation on, the decode region holds Bd * q_len token rows
// (q_len = spec_len + 1 consecutive positions per sequence) and every one of
// them is a sampling row; draft_ids[row] is the proposal that row's sample is
// checked against (-1: none, i.e. the bonus row or a padded proposal).
struct Arena {
  int32_t* base = nullptr;
  int64_t capacity = 0;    // words
  int max_tokens = 0;      // T capacity
  int max_seqs = 0;        // rows of a block table / sampling rows
  int max_blocks = 0;      // MB: block-table width
};

struct StepMeta {
  int num_tokens = 0;   // T (including decode padding)
  int num_decode = 0;   // Bd (including padding)
  int decode_q_len = 1; // token rows per decode sequence (spec_len + 1 when speculating)
  int num_real_decode = 0;
  int num_prefill = 0;  // Sp
  int num_tiles = 0;    // NT
  int num_logits = 0;   // NL (including padding)
  int num_real_logits = 0;
  int max_decode_blocks = 0;
  int num_preempted = 0;
  bool all_greedy = true;
  // word offsets into the arena
  int64_t off_input_ids = 0, off_slot_mapping = 0, off_positions = 0;
  int64_t off_decode_seq_lens = 0, off_decode_block_table = 0;
  int64_t off_prefill_ctx_lens = 0, off_prefill_cu_q = 0, off_prefill_block_table = 0;
  int64_t off_tile_seq = 0, off_tile_start = 0;
  int64_t off_logits_rows = 0, off_top_k = 0, off_temperature = 0, off_top_p = 0, off_draft_ids = 0, off_seeds = 0,
          off_offsets = 0;
  int64_t used_words = 0;
};

// Packed layout for the given row counts (shared by the scheduler and the runner).
StepMeta arena_layout(int T, int Bd, int Sp, int NT, int NL, int MB, int q_len = 1);

// Prompt-lookup (n-gram) proposal: the longest suffix of `tokens` of length
// max_order down to min_order that also occurs earlier; returns the k tokens
// that followed its most recent earlier occurrence, continuing periodically
// past the end of the sequence (empty if no suffix recurs).
std::vector<int32_t> ngram_propose(const std::vector<int32_t>& tokens, int k, int max_order, int min_order);

struct Event {
  int64_t seq_id;
  int32_t token;
  bool finished;
  int finish_reason;
};

class Scheduler {
 public:
  Scheduler(const SchedulerConfig& cfg, int num_blocks, int block_size, bool prefix_caching);

  void set_arena(const Arena& a) { arena_ = a; }
  // Decode-only steps are padded up to the smallest bucket >= their batch.
  void set_decode_buckets(const std::vector<int>& b) { buckets_ = b; }
  int64_t add_request(const std::vector<int32_t>& prompt, const SamplingParams& sp, int priority);
  bool abort(int64_t id);
  bool has_unfinished() const { return !waiting_.empty() || !running_.empty(); }
  int num_waiting() const { return static_cast<int>(waiting_.size()); }
  int num_running() const { return static_cast<int>(running_.size()); }

  StepMeta schedule();
  // Policy maintenance outside the forward pass (CompactInactive); returns
  // the number of cache blocks freed.  schedule() runs it first.
  int maintain_long_context();
  // Block ids of a table visible to attention under the policy.
  std::vector<int32_t> visible_blocks(const std::vector<int32_t>& table) const;
  std::vector<Event> update(const int32_t* sampled, int n);
  // The step scheduled last could not be trusted (a kernel reported an
  // error): every sequence it scheduled finishes with FinishReason::Error and
  // releases its KV blocks, and the step's sampling state is dropped.
  // Returns the failed sequence ids.  Sequences that were not part of the
  // step are untouched.  (Reference: fail_scheduled_requests,
  // crates/engine/src/scheduler/mod.rs:1862-1907.)
  std::vector<int64_t> fail_scheduled();

  // ---- speculative decoding
  // Running sequences whose next step is a decode (verify) row, in running order.
  std::vector<int64_t> decode_candidates() const;
  // Proposals for the next step (at most spec_len are used); false if unknown.
  bool set_draft(int64_t id, const std::vector<int32_t>& draft);
  // n-gram proposals for every decode candidate; returns how many got one.
  int propose_ngram(int max_order, int min_order);
  // Replace the token tail: keep the first keep_len tokens, append tail.  KV
  // beyond keep_len is dropped (num_computed clamps).  Used to re-synchronise
  // a draft model's mirror sequence with the target after verification.
  // Blocks this sequence shares with others may not be cut into.
  bool set_tail(int64_t id, int keep_len, const std::vector<int32_t>& tail);

  BlockManager& blocks() { return bm_; }
  // Host (L2) and file (L3) tiers under the prefix cache; l2_base holds
  // cfg.l2_slots * cfg.block_bytes bytes of pinned memory owned by the caller.
  void enable_cachemesh(const CacheMeshConfig& cfg, uint8_t* l2_base) {
    mesh_ = std::make_unique<CacheMesh>(cfg, l2_base);
    bm_.set_cachemesh(mesh_.get());
  }
  CacheMesh* cachemesh() { return mesh_.get(); }
  const Sequence* find(int64_t id) const;
  const SchedulerConfig& config() const { return cfg_; }
  int64_t total_preemptions() const { return total_preemptions_; }
  int64_t admissions_deferred() const { return admissions_deferred_; }
  int64_t priority_preemptions() const { return priority_preemptions_; }
  // ---- swap preemption: block copies the runner issues before the step's
  // forward, swap-ins (host slot -> block) first, then swap-outs (block -> slot)
  std::vector<std::pair<int32_t, int32_t>> take_swap_ins() { return std::move(swap_in_q_); }
  std::vector<std::pair<int32_t, int32_t>> take_swap_outs() { return std::move(swap_out_q_); }
  int free_swap_slots() const { return static_cast<int>(free_swap_.size()); }
  int64_t total_swap_outs() const { return total_swap_outs_; }

  // ---- KV state export / import (reference Model::export_state /
  // import_state, crates/engine/src/core/model.rs:215-238)
  struct SeqState {
    std::vector<int32_t> tokens;
    int num_prompt = 0;
    int num_computed = 0;         // tokens whose KV is in the blocks below
    std::vector<int32_t> blocks;  // block ids holding those tokens, in order
    SamplingParams sp;
    int priority = 0;
  };
  // A running or waiting (not swapped) sequence's state; throws if unknown.
  SeqState export_sequence(int64_t id) const;
  // New waiting sequence that resumes from num_computed tokens of KV: its
  // blocks are allocated now (returned in SeqState::blocks) and the caller
  // copies the pages in before the next step.  Throws if the pool is full.
  std::pair<int64_t, std::vector<int32_t>> import_sequence(const std::vector<int32_t>& tokens, int num_prompt,
                                                           int num_computed, const SamplingParams& sp, int priority);

  // Longest sequence (prompt + generated tokens): max_model_len, or less when
  // the KV pool cannot hold that many tokens of one sequence.
  int length_limit() const;
  // Scheduler clock in milliseconds (steady clock; a test may pin it).
  double now_ms() const;
  void set_clock_ms(double ms) { clock_override_ms_ = ms; }
  // Fraction of the KV pool held by sequences and the prefix cache's active blocks.
  double kv_utilization() const;
  // Cost of choosing `s` as the preemption victim under the configured policy.
  double victim_cost(const Sequence& s, double now) const;
  // speculation counters: verify groups, proposals offered, proposals accepted
  int64_t spec_steps() const { return spec_steps_; }
  int64_t spec_proposed() const { return spec_proposed_; }
  int64_t spec_accepted() const { return spec_accepted_; }
  // Sequence ids of the sampling rows of the last scheduled step, in row order.
  std::vector<int64_t> sampling_ids() const {
    std::vector<int64_t> v;
    v.reserve(last_sampling_.size());
    for (const Sequence* s : last_sampling_) v.push_back(s->id);
    return v;
  }

 private:
  // Recompute preemption: release the blocks and requeue at the head of the
  // wait queue (to_front) or behind the waiting requests of >= priority.
  void preempt(Sequence* s, bool to_front = true);
  // Lowest-cost running sequence that is not `requester` and not already in
  // `scheduled`; sequences at the preemption cap only when nothing else is left.
  Sequence* pick_victim(const Sequence* requester, const std::vector<Sequence*>& scheduled) const;
  bool is_stop(const Sequence& s, int32_t tok) const;
  FinishReason stop_reason(const Sequence& s, int32_t tok) const;
  void finish(Sequence* s, FinishReason r);

  SchedulerConfig cfg_;
  BlockManager bm_;
  std::unique_ptr<CacheMesh> mesh_;
  Arena arena_;
  std::vector<int> buckets_;
  std::unordered_map<int64_t, std::unique_ptr<Sequence>> seqs_;
  std::deque<Sequence*> waiting_;
  std::vector<Sequence*> running_;
  std::vector<Sequence*> last_sampling_;
  std::vector<int32_t> row_draft_;  // per sampling row: proposal to check (-1 none)
  std::vector<int32_t> row_group_;  // per sampling row: rows in its verify group (1 for plain rows)
  std::vector<Sequence*> last_scheduled_;
  int64_t next_id_ = 1;
  int64_t next_order_ = 0;
  int64_t total_preemptions_ = 0;
  int64_t admissions_deferred_ = 0;
  int64_t total_swap_outs_ = 0;
  std::vector<int32_t> free_swap_;
  std::vector<std::pair<int32_t, int32_t>> swap_in_q_, swap_out_q_;
  int64_t priority_preemptions_ = 0;
  double clock_override_ms_ = -1.0;
  int64_t spec_steps_ = 0, spec_proposed_ = 0, spec_accepted_ = 0;
};

}  // namespace rt
}  // namespace bloom
