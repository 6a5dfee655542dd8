// Paged KV-cache block manager (host side; the pages themselves live in HBM).
//
// Semantics follow the reference pool (crates/engine/src/scheduler/mod.rs:219-851,
// BloomKvCachePool): 16-token blocks, a free list, reference counts, a prefix
// table keyed on the hash of the full token prefix up to each full block,
// an LRU of cached blocks that no running sequence holds (reused on a prefix
// hit, evicted for new allocations), and the same pool metrics
// (mod.rs:176-185: total / free / active / cached blocks, hits, misses,
// evictions, reuses).  Victim choice follows the reference's
// age x value x cost score (mod.rs:656-672) restricted to unreferenced
// blocks: the oldest, least-reused cached block goes first.
#pragma once

#include <cstdint>
#include <list>
#include <unordered_map>
#include <vector>

#include "cachemesh.h"

namespace bloom {
namespace rt {

struct PoolMetrics {
  int64_t total_blocks = 0;
  int64_t free_blocks = 0;
  int64_t active_blocks = 0;
  int64_t cached_blocks = 0;
  int64_t hits = 0;
  int64_t misses = 0;
  int64_t evictions = 0;
  int64_t reuses = 0;
};

class BlockManager {
 public:
  BlockManager(int num_blocks, int block_size, bool enable_prefix_caching);

  int block_size() const { return block_size_; }
  int num_blocks() const { return num_blocks_; }
  // Blocks that can be handed out right now (free + evictable cached).
  int num_available() const { return static_cast<int>(free_.size() + lru_.size()); }

  // Look up the longest cached prefix of `tokens` (whole blocks only, and at
  // most max_tokens tokens).  Matching blocks are pinned (refcount++) and
  // appended to `table`; returns the number of cached tokens.
  int match_prefix(const std::vector<int32_t>& tokens, int max_tokens, std::vector<int32_t>& table,
                   std::vector<uint64_t>& hashes);

  // Grow `table` so it covers `num_tokens` tokens.  All-or-nothing.
  bool ensure_capacity(std::vector<int32_t>& table, int num_tokens);

  // Register the hash of every newly completed full block of a sequence
  // (tokens[0 : num_computed]) so later prompts can reuse it.
  void commit_full_blocks(const std::vector<int32_t>& tokens, int num_computed, const std::vector<int32_t>& table,
                          std::vector<uint64_t>& hashes);

  // Drop the sequence's references.  Hashed blocks whose refcount reaches 0
  // stay cached (LRU); unhashed blocks return to the free list.
  void release(std::vector<int32_t>& table, std::vector<uint64_t>& hashes);

  // Shrink a table to cover only `num_tokens` tokens (speculative rollback /
  // context shift); freed tail blocks go back to the pool.
  void truncate(std::vector<int32_t>& table, std::vector<uint64_t>& hashes, int num_tokens);

  // Evict up to n cached blocks (compaction of inactive cache).
  int evict_cached(int n);
  void reset_prefix_cache();

  PoolMetrics metrics() const;

  // ---- CacheMesh (host / file tiers below the HBM prefix cache)
  void set_cachemesh(CacheMesh* mesh) { mesh_ = mesh; }
  CacheMesh* cachemesh() const { return mesh_; }
  struct Copy {
    int32_t block;
    int32_t slot;
  };
  // Copies queued since the last call: HBM block -> host slot (evicted
  // prefix blocks) and host slot -> HBM block (prefix restored from L2/L3).
  // Restores must be issued before offloads (a slot may be reused).
  std::vector<Copy> take_offloads() { return std::move(offloads_); }
  std::vector<Copy> take_restores() { return std::move(restores_); }
  int refcount(int block) const { return refcount_[block]; }

  static uint64_t chain_hash(uint64_t prev, const int32_t* toks, int n);

 private:
  int take_block();  // -1 if none
  void touch_lru(int block);

  int num_blocks_;
  int block_size_;
  bool prefix_caching_;
  std::vector<int32_t> free_;
  std::vector<int32_t> refcount_;
  std::vector<uint64_t> block_hash_;  // 0 = none
  std::vector<int64_t> block_uses_;
  std::unordered_map<uint64_t, int32_t> by_hash_;
  std::list<int32_t> lru_;  // cached, unreferenced; front = oldest
  std::vector<std::list<int32_t>::iterator> lru_pos_;
  std::vector<uint8_t> in_lru_;
  int64_t hits_ = 0, misses_ = 0, evictions_ = 0, reuses_ = 0;
  CacheMesh* mesh_ = nullptr;
  std::vector<Copy> offloads_, restores_;
};

}  // namespace rt
}  // namespace bloom
