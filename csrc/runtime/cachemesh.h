// CacheMesh: hierarchical KV-block cache below the HBM prefix cache.
//
//   L1  paged KV blocks in HBM (BlockManager prefix table)
//   L2  pinned host memory: a slot per block, LRU
//   L3  files in a directory, LRU, surviving the process
//
// When the block manager evicts a cached (hashed, unreferenced) HBM block to
// reuse it, the block's pages are offloaded to an L2 slot: the scheduler
// queues (block, slot) and the model runner copies device -> host on its
// stream before the step's forward can overwrite the block.  An L2 slot that
// is itself evicted spills to an L3 file.  When a prompt's prefix misses in
// HBM, the chain hashes of its next blocks are looked up in L2 and L3; a hit
// takes a fresh HBM block, queues (block, slot) for a host -> device copy
// ahead of the forward, and re-registers the block in the prefix table.
// Keys are the 64-bit chain hashes of the full token prefix that the block
// manager already computes, qualified by a namespace (model + KV layout) in
// L3 file names, so files of another model never match.
//
// Behaviour follows the reference's SGLang-style CacheMesh
// (crates/engine/src/cachemesh/store.rs:375-555: offload_to_l2, restore,
// tier metrics); the tiers here hold the real paged KV bytes of the B200
// cache instead of host f32 copies.
#pragma once

#include <algorithm>
#include <cstdint>
#include <list>
#include <string>
#include <unordered_map>
#include <vector>

namespace bloom {
namespace rt {

struct CacheMeshConfig {
  int64_t l2_slots = 0;       // host slots (0 disables the mesh)
  int64_t block_bytes = 0;    // bytes of one KV block over all layers
  std::string l3_dir;         // empty: no L3
  int64_t l3_max_blocks = 0;  // 0: no L3
  std::string name_space = "default";
};

struct CacheMeshMetrics {
  int64_t l2_used = 0, l2_capacity = 0, l3_used = 0, l3_capacity = 0;
  int64_t offloads = 0, l2_hits = 0, l3_hits = 0, misses = 0, l2_evictions = 0, l3_writes = 0, l3_evictions = 0;
};

class CacheMesh {
 public:
  CacheMesh(const CacheMeshConfig& cfg, uint8_t* l2_base);

  bool enabled() const { return cfg_.l2_slots > 0 && l2_base_ != nullptr; }
  // Start of a scheduler step: the copies queued by the previous step have
  // completed (the runner synchronises every step), so their slots may be
  // reused again.  Slots handed out within a step are never reused within it.
  void begin_step() { std::fill(pending_.begin(), pending_.end(), 0); }
  // Slot that will receive the device copy of the block with this hash
  // (evicting the L2 LRU entry to L3 if needed).  -1: disabled.
  int reserve_offload(uint64_t hash);
  // L2 slot holding this hash, promoting an L3 file into L2 if needed; -1 on miss.
  int lookup(uint64_t hash);
  bool contains(uint64_t hash) const;
  CacheMeshMetrics metrics() const;
  const CacheMeshConfig& config() const { return cfg_; }

 private:
  int take_slot();  // free or evicted (spilled) slot
  void spill_to_l3(uint64_t hash, int slot);
  std::string l3_path(uint64_t hash) const;
  void touch(uint64_t hash);
  void l3_touch(uint64_t hash);
  void scan_l3();

  CacheMeshConfig cfg_;
  uint8_t* l2_base_;
  std::vector<int> free_slots_;
  std::vector<char> pending_;  // slot has a device copy queued in the current step
  std::unordered_map<uint64_t, int> l2_map_;  // hash -> slot
  std::list<uint64_t> l2_lru_;                // front = oldest
  std::unordered_map<uint64_t, std::list<uint64_t>::iterator> l2_pos_;
  std::list<uint64_t> l3_lru_;
  std::unordered_map<uint64_t, std::list<uint64_t>::iterator> l3_pos_;
  CacheMeshMetrics m_;
};

}  // namespace rt
}  // namespace bloom
