#include "scheduler.h"

#include <algorithm>
#include <stdexcept>

namespace bloom {
namespace rt {

Scheduler::Scheduler(const SchedulerConfig& cfg, int num_blocks, int block_size, bool prefix_caching)
    : cfg_(cfg), bm_(num_blocks, block_size, prefix_caching) {
  for (int i = cfg.swap_slots - 1; i >= 0; --i) free_swap_.push_back(i);
}

int64_t Scheduler::add_request(const std::vector<int32_t>& prompt, const SamplingParams& sp, int priority) {
  if (prompt.empty()) throw std::invalid_argument("add_request: empty prompt");
  if (static_cast<int>(prompt.size()) >= cfg_.max_model_len)
    throw std::invalid_argument("add_request: prompt longer than max_model_len");
  // a sequence alone must always fit the pool, or it could be preempted and
  // re-admitted forever: prompts past the pool are refused, and generation
  // stops at the pool's token capacity (length_limit)
  if (static_cast<int>(prompt.size()) >= length_limit())
    throw std::invalid_argument("add_request: prompt needs more KV blocks than the pool holds (" +
                                std::to_string(bm_.num_blocks()) + " blocks of " +
                                std::to_string(bm_.block_size()) + " tokens)");
  auto s = std::make_unique<Sequence>();
  s->id = next_id_++;
  s->tokens = prompt;
  s->num_prompt = static_cast<int>(prompt.size());
  s->sp = sp;
  s->priority = priority;
  s->order = next_order_++;
  s->arrival_ms = now_ms();
  s->last_scheduled_ms = s->arrival_ms;
  Sequence* p = s.get();
  seqs_[p->id] = std::move(s);
  // higher priority first, FCFS inside a priority class
  auto it = waiting_.end();
  while (it != waiting_.begin() && (*(it - 1))->priority < priority) --it;
  waiting_.insert(it, p);
  return p->id;
}

const Sequence* Scheduler::find(int64_t id) const {
  auto it = seqs_.find(id);
  return it == seqs_.end() ? nullptr : it->second.get();
}

void Scheduler::finish(Sequence* s, FinishReason r) {
  s->status = SeqStatus::Finished;
  s->finish = r;
  bm_.release(s->table, s->hashes);
  for (int32_t slot : s->swap_slots) free_swap_.push_back(slot);
  s->swap_slots.clear();
  s->swapped = false;
}

bool Scheduler::abort(int64_t id) {
  auto it = seqs_.find(id);
  if (it == seqs_.end()) return false;
  Sequence* s = it->second.get();
  if (s->status == SeqStatus::Finished) return false;
  waiting_.erase(std::remove(waiting_.begin(), waiting_.end(), s), waiting_.end());
  running_.erase(std::remove(running_.begin(), running_.end(), s), running_.end());
  finish(s, FinishReason::Aborted);
  seqs_.erase(it);
  return true;
}

void Scheduler::preempt(Sequence* s, bool to_front) {
  running_.erase(std::remove(running_.begin(), running_.end(), s), running_.end());
  const int bs = bm_.block_size();
  const int keep = (s->num_computed + bs - 1) / bs;  // blocks holding computed KV
  if (keep > 0 && static_cast<int>(free_swap_.size()) >= keep && keep <= static_cast<int>(s->table.size())) {
    // swap: copy the computed blocks to host slots; the sequence keeps its progress
    s->swap_slots.clear();
    for (int b = 0; b < keep; ++b) {
      const int32_t slot = free_swap_.back();
      free_swap_.pop_back();
      swap_out_q_.emplace_back(s->table[b], slot);
      s->swap_slots.push_back(slot);
    }
    s->swapped = true;
    ++total_swap_outs_;
  } else {
    s->num_computed = 0;
  }
  bm_.release(s->table, s->hashes);
  s->status = SeqStatus::Waiting;
  ++s->num_preemptions;
  ++total_preemptions_;
  if (to_front) {
    waiting_.push_front(s);
    return;
  }
  // behind every waiting request of higher or equal priority
  auto it = waiting_.begin();
  while (it != waiting_.end() && (*it)->priority >= s->priority) ++it;
  waiting_.insert(it, s);
}

double Scheduler::now_ms() const {
  if (clock_override_ms_ >= 0.0) return clock_override_ms_;
  using namespace std::chrono;
  return duration<double, std::milli>(steady_clock::now().time_since_epoch()).count();
}

double Scheduler::kv_utilization() const {
  const PoolMetrics pm = bm_.metrics();
  return pm.total_blocks ? static_cast<double>(pm.active_blocks) / static_cast<double>(pm.total_blocks) : 1.0;
}

double Scheduler::victim_cost(const Sequence& s, double now) const {
  const double kv = static_cast<double>(s.num_computed);
  switch (static_cast<VictimPolicy>(cfg_.victim_policy)) {
    case VictimPolicy::Priority:
      return static_cast<double>(s.priority);
    case VictimPolicy::Oldest:
      return -static_cast<double>(s.num_generated());
    case VictimPolicy::KvCost:
      return kv;
    case VictimPolicy::AegaeonScore: {
      const double age_s = std::max(1e-3, (now - s.arrival_ms) / 1e3);
      return age_s / std::max(1.0, kv);
    }
    case VictimPolicy::Lru:
      return -(now - s.last_scheduled_ms);
    case VictimPolicy::LargestFirst:
      return -kv;
    case VictimPolicy::Newest:
    default:
      return -static_cast<double>(s.order);
  }
}

Sequence* Scheduler::pick_victim(const Sequence* requester, const std::vector<Sequence*>& scheduled) const {
  const double now = now_ms();
  const int cap = cfg_.max_preemptions_per_request;
  Sequence* best = nullptr;
  Sequence* best_capped = nullptr;
  double bc = 0.0, bcc = 0.0;
  auto better = [&](Sequence* cand, double c, Sequence* cur, double cur_c) {
    return cur == nullptr || c < cur_c || (c == cur_c && cand->order > cur->order);
  };
  for (Sequence* r : running_) {
    if (r == requester || r->status != SeqStatus::Running) continue;
    if (std::find(scheduled.begin(), scheduled.end(), r) != scheduled.end()) continue;
    const double c = victim_cost(*r, now);
    if (cap > 0 && r->num_preemptions >= cap) {
      if (better(r, c, best_capped, bcc)) best_capped = r, bcc = c;
    } else if (better(r, c, best, bc)) {
      best = r, bc = c;
    }
  }
  return best ? best : best_capped;
}

int Scheduler::length_limit() const {
  return std::min(cfg_.max_model_len, bm_.num_blocks() * bm_.block_size() - cfg_.spec_len);
}

bool Scheduler::is_stop(const Sequence& s, int32_t tok) const {
  if (s.num_generated() >= s.sp.max_tokens) return true;
  if (static_cast<int>(s.tokens.size()) >= length_limit()) return true;
  if (s.num_generated() < s.sp.min_tokens) return false;
  if (!s.sp.ignore_eos)
    for (int32_t e : cfg_.eos_token_ids)
      if (tok == e) return true;
  for (int32_t e : s.sp.stop_token_ids)
    if (tok == e) return true;
  return false;
}

int lc_window_blocks(const SchedulerConfig& c, int block_size, int total_blocks) {
  auto to_blocks = [&](int tokens) { return tokens <= 0 || block_size <= 0 ? 0 : (tokens + block_size - 1) / block_size; };
  switch (c.lc_policy) {
    case 1:
      return to_blocks(c.lc_window_tokens);
    case 2:
      return to_blocks(std::max(std::max(0, c.lc_max_context - c.lc_shift), block_size));
    default:
      return total_blocks;
  }
}

std::vector<int32_t> Scheduler::visible_blocks(const std::vector<int32_t>& table) const {
  const int n = static_cast<int>(table.size());
  const int w = lc_window_blocks(cfg_, bm_.block_size(), n);
  if (w >= n) return table;
  return std::vector<int32_t>(table.end() - w, table.end());
}

int Scheduler::maintain_long_context() {
  if (cfg_.lc_policy != 3) return 0;
  const PoolMetrics pm = bm_.metrics();
  const int need = cfg_.lc_target_free - static_cast<int>(pm.free_blocks);
  return need > 0 ? bm_.evict_cached(need) : 0;
}

StepMeta Scheduler::schedule() {
  if (arena_.base == nullptr) throw std::runtime_error("Scheduler: arena not set");
  if (mesh_) mesh_->begin_step();
  maintain_long_context();
  StepMeta m;
  const int bs = bm_.block_size();
  // verify width: spec_len + 1 rows per decode sequence when any running
  // sequence carries a proposal this step, else plain one-row decode (the
  // speculator may pause proposing when its drafts are not accepted)
  int ql = 1;
  if (cfg_.spec_len > 0)
    for (const Sequence* s : running_)
      if (!s->draft.empty()) {
        ql = cfg_.spec_len + 1;
        break;
      }
  int budget = std::min(cfg_.max_num_batched_tokens, arena_.max_tokens);
  last_sampling_.clear();
  last_scheduled_.clear();

  struct Prefill {
    Sequence* s;
    int start;
    int len;
  };
  std::vector<Sequence*> decodes;
  std::vector<Prefill> prefills;

  // 0) priority preemption (before anything is scheduled): the head of the
  // wait queue outranks running sequences and has waited long enough, but the
  // pool cannot hold its prompt -> lower-priority sequences give up their
  // blocks (lowest priority, newest first) until it fits
  if (cfg_.priority_preempt_ms >= 0.0 && !waiting_.empty()) {
    Sequence* h = waiting_.front();
    if (now_ms() - h->arrival_ms >= cfg_.priority_preempt_ms) {
      const int need_blocks =
          (static_cast<int>(h->tokens.size()) + bs - 1) / bs - static_cast<int>(h->table.size());
      while (static_cast<int>(bm_.num_available()) < need_blocks) {
        Sequence* v = nullptr;
        for (Sequence* r : running_)
          if (r->priority < h->priority &&
              (v == nullptr || r->priority < v->priority || (r->priority == v->priority && r->order > v->order)))
            v = r;
        if (v == nullptr) break;
        preempt(v, /*to_front=*/false);  // h stays at the head of the queue
        ++m.num_preempted;
        ++priority_preemptions_;
      }
    }
  }

  // 1) decode rows: running sequences that need exactly their last token computed.
  const std::vector<Sequence*> snapshot = running_;
  for (Sequence* s : snapshot) {
    if (s->status != SeqStatus::Running) continue;  // preempted earlier in this loop
    const int need = static_cast<int>(s->tokens.size()) - s->num_computed;
    if (need != 1) continue;
    if (budget < ql || static_cast<int>(decodes.size()) >= arena_.max_seqs) break;
    bool ok = bm_.ensure_capacity(s->table, s->num_computed + ql);
    while (!ok) {
      // preempt the policy's victim among running sequences not yet scheduled
      // (the requester itself when the policy ranks it first)
      Sequence* victim = pick_victim(s, decodes);
      if (victim == nullptr) break;
      if (cfg_.victim_policy != static_cast<int>(VictimPolicy::Newest)) {
        const double now = now_ms();
        if (victim_cost(*s, now) < victim_cost(*victim, now)) break;
      }
      preempt(victim);
      ++m.num_preempted;
      ok = bm_.ensure_capacity(s->table, s->num_computed + ql);
    }
    if (!ok) {
      preempt(s);
      ++m.num_preempted;
      continue;
    }
    decodes.push_back(s);
    budget -= ql;
  }

  // 2) partially prefilled running sequences (chunked prefill continues)
  for (Sequence* s : running_) {
    const int need = static_cast<int>(s->tokens.size()) - s->num_computed;
    if (need <= 1) continue;
    if (budget <= 0 || static_cast<int>(prefills.size()) + static_cast<int>(decodes.size()) >= arena_.max_seqs) break;
    const int len = cfg_.chunked_prefill ? std::min(need, budget) : need;
    if (len > budget) break;
    if (!bm_.ensure_capacity(s->table, s->num_computed + len)) break;
    prefills.push_back({s, s->num_computed, len});
    budget -= len;
  }

  // 3) admit waiting sequences (not while the KV pool is above the admission threshold)
  if (!waiting_.empty() && cfg_.kv_admission_threshold < 1.0 && kv_utilization() >= cfg_.kv_admission_threshold &&
      !(running_.empty() && decodes.empty() && prefills.empty())) {
    ++admissions_deferred_;
    budget = 0;
  }
  while (!waiting_.empty() && budget > 0 && static_cast<int>(running_.size()) < cfg_.max_num_seqs &&
         static_cast<int>(prefills.size()) + static_cast<int>(decodes.size()) < arena_.max_seqs) {
    Sequence* s = waiting_.front();
    if (s->table.empty() && !s->swapped) {
      // prefix reuse: whole cached blocks, always leaving the last token to compute
      const int max_cached = ((static_cast<int>(s->tokens.size()) - 1) / bs) * bs;
      s->num_computed = bm_.match_prefix(s->tokens, max_cached, s->table, s->hashes);
      if (!s->admitted_once) s->num_cached_prefix = s->num_computed;
    }
    const int need = static_cast<int>(s->tokens.size()) - s->num_computed;
    int len = cfg_.chunked_prefill ? std::min(need, budget) : need;
    if (len > budget) break;
    const bool fits = bm_.ensure_capacity(s->table, s->num_computed + len);
    if (!fits) {
      if (running_.empty() && decodes.empty() && prefills.empty()) {
        // nothing else holds blocks: this request can never fit
        waiting_.pop_front();
        finish(s, FinishReason::Length);
        continue;
      }
      break;
    }
    waiting_.pop_front();
    if (s->swapped) {
      // swap in: the saved blocks go back into the first blocks of the new table
      for (size_t b = 0; b < s->swap_slots.size(); ++b) {
        swap_in_q_.emplace_back(s->table[b], s->swap_slots[b]);
        free_swap_.push_back(s->swap_slots[b]);  // the runner copies swap-ins before any swap-out
      }
      s->swap_slots.clear();
      s->swapped = false;
    }
    s->status = SeqStatus::Running;
    s->admitted_once = true;
    running_.push_back(s);
    if (len == 1 && need == 1 && ql == 1) {
      decodes.push_back(s);
    } else {
      prefills.push_back({s, s->num_computed, len});
    }
    budget -= len;
  }

  // ---- layout (decode-only steps padded to a bucket)
  int Bd = static_cast<int>(decodes.size());
  const int real_decode = Bd;
  int T_pref = 0;
  for (auto& p : prefills) T_pref += p.len;
  int ntiles = 0;
  for (auto& p : prefills) ntiles += (p.len + 127) / 128;  // 128 query rows per attention tile
  int nl_real = Bd * ql;
  for (auto& p : prefills)
    if (p.start + p.len == static_cast<int>(p.s->tokens.size())) ++nl_real;
  if (prefills.empty() && Bd > 0) {
    for (int b : buckets_)
      if (b >= Bd) {
        Bd = std::min(b, arena_.max_seqs);
        break;
      }
  }
  const int T = Bd * ql + T_pref;
  const int NL = nl_real + (Bd - real_decode) * ql;
  const int mb = arena_.max_blocks;
  m = [&] {
    StepMeta lay = arena_layout(T, Bd, static_cast<int>(prefills.size()), ntiles, NL, mb, ql);
    lay.num_preempted = m.num_preempted;
    return lay;
  }();
  if (m.used_words > arena_.capacity) throw std::runtime_error("Scheduler: step does not fit in the arena");
  int32_t* A = arena_.base;
  int32_t* input_ids = A + m.off_input_ids;
  int32_t* slots = A + m.off_slot_mapping;
  int64_t* positions = reinterpret_cast<int64_t*>(A + m.off_positions);
  int32_t* dsl = A + m.off_decode_seq_lens;
  int32_t* dbt = A + m.off_decode_block_table;
  int32_t* pctx = A + m.off_prefill_ctx_lens;
  int32_t* pcu = A + m.off_prefill_cu_q;
  int32_t* pbt = A + m.off_prefill_block_table;
  int32_t* tseq = A + m.off_tile_seq;
  int32_t* tstart = A + m.off_tile_start;
  int32_t* lrows = A + m.off_logits_rows;
  int32_t* topk = A + m.off_top_k;
  float* temp = reinterpret_cast<float*>(A + m.off_temperature);
  float* topp = reinterpret_cast<float*>(A + m.off_top_p);
  int64_t* seeds = reinterpret_cast<int64_t*>(A + m.off_seeds);
  int64_t* offs = reinterpret_cast<int64_t*>(A + m.off_offsets);
  int32_t* drafts = A + m.off_draft_ids;
  row_draft_.clear();
  row_group_.clear();

  // first block attention sees: the policy's window over the blocks covering
  // the context, never starting after the first token of this step
  auto window_start = [&](int ctx, int first) {
    const int nb = (ctx + bs - 1) / bs;
    const int w = lc_window_blocks(cfg_, bs, nb);
    return std::max(0, std::min(nb - w, first / bs));
  };
  int t = 0;
  int nsample = 0;
  m.all_greedy = true;
  auto add_sample = [&](Sequence* s, int row, int32_t draft, int group, int extra_offset) {
    lrows[nsample] = row;
    temp[nsample] = s ? s->sp.temperature : 0.f;
    topp[nsample] = s ? s->sp.top_p : 1.f;
    topk[nsample] = s ? s->sp.top_k : 0;
    seeds[nsample] = s ? s->sp.seed : 0;
    offs[nsample] = s ? s->num_generated() + extra_offset : 0;
    drafts[nsample] = draft;
    if (s && s->sp.temperature > 0.f) m.all_greedy = false;
    if (s) {
      last_sampling_.push_back(s);
      row_draft_.push_back(draft);
      row_group_.push_back(group);
    }
    ++nsample;
  };
  for (int i = 0; i < Bd; ++i) {
    int32_t* row_bt = dbt + static_cast<int64_t>(i) * mb;
    if (i < real_decode) {
      Sequence* s = decodes[i];
      const int pos = s->num_computed;
      const int nb = static_cast<int>(s->table.size());
      if (nb > mb) throw std::runtime_error("Scheduler: block table wider than the arena");
      const int w0 = window_start(pos + ql, pos);
      std::copy(s->table.begin() + w0, s->table.end(), row_bt);
      dsl[i] = pos + ql - w0 * bs;
      m.max_decode_blocks = std::max(m.max_decode_blocks, (pos + ql + bs - 1) / bs - w0);
      const int nd = std::min<int>(static_cast<int>(s->draft.size()), ql - 1);
      for (int j = 0; j < ql; ++j) {
        const int p = pos + j;
        input_ids[t] = j == 0 ? s->tokens[pos] : (j - 1 < nd ? s->draft[j - 1] : 0);
        positions[t] = p;
        slots[t] = s->table[p / bs] * bs + p % bs;
        add_sample(s, t, j < nd ? s->draft[j] : -1, ql, j);
        ++t;
      }
      s->verifying = ql > 1;
    } else {  // padding rows: read one page of block 0, write no KV, results ignored
      for (int j = 0; j < ql; ++j) {
        input_ids[t] = 0;
        positions[t] = j;
        slots[t] = -1;
        add_sample(nullptr, t, -1, ql, 0);
        ++t;
      }
      row_bt[0] = 0;
      dsl[i] = ql;
    }
  }
  pcu[0] = 0;
  struct TileOrder {
    int seq, start, extent;
  };
  std::vector<TileOrder> tiles;
  tiles.reserve(ntiles);
  for (size_t j = 0; j < prefills.size(); ++j) {
    const Prefill& p = prefills[j];
    Sequence* s = p.s;
    for (int k = 0; k < p.len; ++k) {
      const int pos = p.start + k;
      input_ids[t] = s->tokens[pos];
      positions[t] = pos;
      slots[t] = s->table[pos / bs] * bs + pos % bs;
      ++t;
    }
    const int nb = static_cast<int>(s->table.size());
    if (nb > mb) throw std::runtime_error("Scheduler: block table wider than the arena");
    const int w0 = window_start(p.start + p.len, p.start);
    std::copy(s->table.begin() + w0, s->table.end(), pbt + static_cast<int64_t>(j) * mb);
    pctx[j] = p.start + p.len - w0 * bs;
    pcu[j + 1] = pcu[j] + p.len;
    for (int r = 0; r < p.len; r += 128)
      tiles.push_back({static_cast<int>(j), r, p.start - w0 * bs + std::min(r + 128, p.len)});
    s->num_computed = p.start + p.len;
    if (s->num_computed == static_cast<int>(s->tokens.size())) add_sample(s, t - 1, -1, 1, 0);
  }
  // heavy tiles (long kv extent) first for load balance
  std::stable_sort(tiles.begin(), tiles.end(), [](const TileOrder& a, const TileOrder& b) { return a.extent > b.extent; });
  for (int i = 0; i < static_cast<int>(tiles.size()); ++i) {
    tseq[i] = tiles[i].seq;
    tstart[i] = tiles[i].start;
  }
  const double tnow = now_ms();
  for (Sequence* s : decodes) s->last_scheduled_ms = tnow;
  for (auto& p : prefills) p.s->last_scheduled_ms = tnow;
  for (Sequence* s : decodes) s->num_computed += ql;  // provisional for verify rows: update() rolls back
  for (Sequence* s : decodes) last_scheduled_.push_back(s);
  for (auto& p : prefills) last_scheduled_.push_back(p.s);
  m.num_real_decode = real_decode;
  m.num_real_logits = static_cast<int>(last_sampling_.size());
  m.decode_q_len = ql;
  return m;
}

StepMeta arena_layout(int T, int Bd, int Sp, int NT, int NL, int MB, int q_len) {
  StepMeta m;
  int64_t off = 0;
  auto take = [&](int64_t words) {
    const int64_t o = off;
    off += words;
    return o;
  };
  auto align2 = [&] { off = (off + 1) & ~int64_t(1); };
  m.off_input_ids = take(T);
  m.off_slot_mapping = take(T);
  align2();
  m.off_positions = take(2 * int64_t(T));
  m.off_decode_seq_lens = take(Bd);
  m.off_decode_block_table = take(int64_t(Bd) * MB);
  m.off_prefill_ctx_lens = take(Sp);
  m.off_prefill_cu_q = take(Sp + 1);
  m.off_prefill_block_table = take(int64_t(Sp) * MB);
  m.off_tile_seq = take(NT);
  m.off_tile_start = take(NT);
  m.off_logits_rows = take(NL);
  m.off_top_k = take(NL);
  m.off_temperature = take(NL);
  m.off_top_p = take(NL);
  m.off_draft_ids = take(NL);
  align2();
  m.off_seeds = take(2 * int64_t(NL));
  m.off_offsets = take(2 * int64_t(NL));
  align2();
  m.used_words = off;
  m.num_tokens = T;
  m.num_decode = Bd;
  m.num_prefill = Sp;
  m.num_tiles = NT;
  m.num_logits = NL;
  m.decode_q_len = q_len;
  return m;
}

FinishReason Scheduler::stop_reason(const Sequence& s, int32_t tok) const {
  const bool length =
      s.num_generated() >= s.sp.max_tokens || static_cast<int>(s.tokens.size()) >= length_limit();
  bool eos = false;
  if (!s.sp.ignore_eos)
    for (int32_t e : cfg_.eos_token_ids) eos |= (tok == e);
  for (int32_t e : s.sp.stop_token_ids) eos |= (tok == e);
  return (eos && s.num_generated() >= s.sp.min_tokens) ? FinishReason::Stop
                                                      : (length ? FinishReason::Length : FinishReason::Stop);
}

std::vector<Event> Scheduler::update(const int32_t* sampled, int n) {
  std::vector<Event> ev;
  if (n < static_cast<int>(last_sampling_.size()))
    throw std::invalid_argument("Scheduler::update: fewer sampled tokens than sampling rows");
  n = static_cast<int>(last_sampling_.size());
  for (Sequence* s : last_scheduled_)
    if (!s->verifying) bm_.commit_full_blocks(s->tokens, s->num_computed, s->table, s->hashes);
  int i = 0;
  while (i < n) {
    Sequence* s = last_sampling_[i];
    const int g = s->verifying ? row_group_[i] : 1;
    if (s->status != SeqStatus::Running) {  // aborted meanwhile
      i += g;
      continue;
    }
    if (!s->verifying) {
      const int32_t tok = sampled[i];
      s->tokens.push_back(tok);
      const bool stop = is_stop(*s, tok);
      FinishReason r = FinishReason::None;
      if (stop) {
        r = stop_reason(*s, tok);
        running_.erase(std::remove(running_.begin(), running_.end(), s), running_.end());
        finish(s, r);
      }
      ev.push_back({s->id, tok, stop, static_cast<int>(r)});
      ++i;
      continue;
    }
    // Verify group: rows i .. i+g-1 sampled positions pos .. pos+g-1.  Row j
    // agrees with its proposal => proposal j accepted; the first row that
    // disagrees (or the bonus row) supplies the one new token.  For greedy
    // rows the sample is the argmax; for stochastic rows the sampler already
    // did the accept / residual draw, so equality is the acceptance test.
    const int pos = s->num_computed - g;
    int acc = 0;
    while (acc < g - 1 && sampled[i + acc] == row_draft_[i + acc]) ++acc;
    bool stopped = false;
    FinishReason r = FinishReason::None;
    for (int j = 0; j <= acc; ++j) {
      const int32_t tok = sampled[i + j];
      s->tokens.push_back(tok);
      const bool stop = is_stop(*s, tok);
      if (stop) r = stop_reason(*s, tok);
      ev.push_back({s->id, tok, stop, static_cast<int>(r)});
      if (stop) {
        stopped = true;
        break;
      }
    }
    s->num_computed = std::min<int>(pos + 1 + acc, static_cast<int>(s->tokens.size()));
    ++spec_steps_;
    spec_proposed_ += s->draft.empty() ? 0 : std::min<int>(static_cast<int>(s->draft.size()), g - 1);
    spec_accepted_ += acc;
    s->verifying = false;
    s->draft.clear();
    bm_.commit_full_blocks(s->tokens, s->num_computed, s->table, s->hashes);
    if (stopped) {
      running_.erase(std::remove(running_.begin(), running_.end(), s), running_.end());
      finish(s, r);
    } else {
      bm_.truncate(s->table, s->hashes, static_cast<int>(s->tokens.size()));  // blocks of rejected rows
    }
    i += g;
  }
  for (Sequence* s : last_scheduled_) s->verifying = false;
  last_sampling_.clear();
  last_scheduled_.clear();
  row_draft_.clear();
  row_group_.clear();
  // drop finished sequences
  for (auto it = seqs_.begin(); it != seqs_.end();) {
    if (it->second->status == SeqStatus::Finished)
      it = seqs_.erase(it);
    else
      ++it;
  }
  return ev;
}

std::vector<int64_t> Scheduler::fail_scheduled() {
  std::vector<int64_t> ids;
  for (Sequence* s : last_scheduled_) {
    if (s->status == SeqStatus::Finished) continue;
    ids.push_back(s->id);
    running_.erase(std::remove(running_.begin(), running_.end(), s), running_.end());
    waiting_.erase(std::remove(waiting_.begin(), waiting_.end(), s), waiting_.end());
    s->verifying = false;
    s->draft.clear();
    finish(s, FinishReason::Error);
  }
  last_sampling_.clear();
  last_scheduled_.clear();
  row_draft_.clear();
  row_group_.clear();
  for (int64_t id : ids) seqs_.erase(id);
  return ids;
}

Scheduler::SeqState Scheduler::export_sequence(int64_t id) const {
  const Sequence* s = find(id);
  if (s == nullptr || s->status == SeqStatus::Finished) throw std::invalid_argument("export_sequence: unknown id");
  if (s->swapped) throw std::invalid_argument("export_sequence: sequence is swapped out; export it once resumed");
  SeqState st;
  st.tokens = s->tokens;
  st.num_prompt = s->num_prompt;
  // verify rows of a scheduled step are provisional: export between steps only
  st.num_computed = s->num_computed;
  const int bs = bm_.block_size();
  const int nb = (st.num_computed + bs - 1) / bs;
  st.blocks.assign(s->table.begin(), s->table.begin() + std::min<int>(nb, static_cast<int>(s->table.size())));
  st.num_computed = std::min<int>(st.num_computed, static_cast<int>(st.blocks.size()) * bs);
  st.sp = s->sp;
  st.priority = s->priority;
  return st;
}

std::pair<int64_t, std::vector<int32_t>> Scheduler::import_sequence(const std::vector<int32_t>& tokens,
                                                                    int num_prompt, int num_computed,
                                                                    const SamplingParams& sp, int priority) {
  if (tokens.empty() || num_prompt < 1 || num_prompt > static_cast<int>(tokens.size()))
    throw std::invalid_argument("import_sequence: bad token counts");
  if (static_cast<int>(tokens.size()) >= length_limit())
    throw std::invalid_argument("import_sequence: sequence longer than max_model_len or the KV pool");
  // at least the last token is recomputed, so the first step samples from it
  num_computed = std::max(0, std::min(num_computed, static_cast<int>(tokens.size()) - 1));
  auto s = std::make_unique<Sequence>();
  s->id = next_id_++;
  s->tokens = tokens;
  s->num_prompt = num_prompt;
  s->num_computed = num_computed;
  s->num_cached_prefix = num_computed;
  s->sp = sp;
  s->priority = priority;
  s->order = next_order_++;
  s->arrival_ms = now_ms();
  s->last_scheduled_ms = s->arrival_ms;
  if (num_computed > 0 && !bm_.ensure_capacity(s->table, num_computed))
    throw std::runtime_error("import_sequence: no free KV blocks for the imported state");
  Sequence* p = s.get();
  seqs_[p->id] = std::move(s);
  auto it = waiting_.end();
  while (it != waiting_.begin() && (*(it - 1))->priority < priority) --it;
  waiting_.insert(it, p);
  return {p->id, p->table};
}

// ---------------------------------------------------------------- speculation
std::vector<int64_t> Scheduler::decode_candidates() const {
  std::vector<int64_t> v;
  for (const Sequence* s : running_)
    if (static_cast<int>(s->tokens.size()) - s->num_computed == 1) v.push_back(s->id);
  return v;
}

bool Scheduler::set_draft(int64_t id, const std::vector<int32_t>& draft) {
  auto it = seqs_.find(id);
  if (it == seqs_.end() || it->second->status == SeqStatus::Finished) return false;
  Sequence* s = it->second.get();
  s->draft.assign(draft.begin(), draft.begin() + std::min<size_t>(draft.size(), std::max(cfg_.spec_len, 0)));
  return true;
}

int Scheduler::propose_ngram(int max_order, int min_order) {
  int n = 0;
  for (Sequence* s : running_) {
    if (static_cast<int>(s->tokens.size()) - s->num_computed != 1) continue;
    s->draft = ngram_propose(s->tokens, cfg_.spec_len, max_order, min_order);
    n += !s->draft.empty();
  }
  return n;
}

bool Scheduler::set_tail(int64_t id, int keep_len, const std::vector<int32_t>& tail) {
  auto it = seqs_.find(id);
  if (it == seqs_.end() || it->second->status == SeqStatus::Finished) return false;
  Sequence* s = it->second.get();
  if (keep_len < s->num_prompt || keep_len > static_cast<int>(s->tokens.size())) return false;
  if (keep_len + static_cast<int>(tail.size()) >= length_limit()) return false;
  s->tokens.resize(keep_len);
  s->tokens.insert(s->tokens.end(), tail.begin(), tail.end());
  if (s->num_computed > keep_len) s->num_computed = keep_len;
  if (s->status == SeqStatus::Running) bm_.truncate(s->table, s->hashes, s->num_computed);
  s->draft.clear();
  return true;
}

std::vector<int32_t> ngram_propose(const std::vector<int32_t>& tokens, int k, int max_order, int min_order) {
  std::vector<int32_t> out;
  const int n = static_cast<int>(tokens.size());
  if (k <= 0) return out;
  min_order = std::max(1, min_order);
  for (int order = std::min(max_order, n - 1); order >= min_order; --order) {
    const int32_t* suf = tokens.data() + n - order;
    // most recent earlier occurrence whose continuation exists
    for (int start = n - order - 1; start >= 0; --start) {
      if (tokens[start] != suf[0]) continue;
      bool eq = true;
      for (int j = 1; j < order && eq; ++j) eq = tokens[start + j] == suf[j];
      if (!eq) continue;
      // the continuation runs on into the proposal itself, so a repeating
      // span proposes its period again (from + j - n < j always)
      const int from = start + order;
      for (int j = 0; j < k; ++j) out.push_back(from + j < n ? tokens[from + j] : out[from + j - n]);
      return out;
    }
  }
  return out;
}

}  // namespace rt
}  // namespace bloom
