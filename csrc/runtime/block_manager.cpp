#include "block_manager.h"

#include <algorithm>
#include <iterator>
#include <stdexcept>

namespace bloom {
namespace rt {

BlockManager::BlockManager(int num_blocks, int block_size, bool enable_prefix_caching)
    : num_blocks_(num_blocks), block_size_(block_size), prefix_caching_(enable_prefix_caching) {
  if (num_blocks <= 0 || block_size <= 0) throw std::invalid_argument("BlockManager: bad sizes");
  free_.reserve(num_blocks);
  // hand out low block ids first (pop_back)
  for (int b = num_blocks - 1; b >= 0; --b) free_.push_back(b);
  refcount_.assign(num_blocks, 0);
  block_hash_.assign(num_blocks, 0);
  block_uses_.assign(num_blocks, 0);
  lru_pos_.resize(num_blocks);
  in_lru_.assign(num_blocks, 0);
}

// FNV-1a over the previous hash and the block's tokens; 0 is reserved for "no hash".
uint64_t BlockManager::chain_hash(uint64_t prev, const int32_t* toks, int n) {
  uint64_t h = 1469598103934665603ull ^ (prev * 0x9E3779B97F4A7C15ull);
  for (int i = 0; i < n; ++i) {
    uint32_t v = static_cast<uint32_t>(toks[i]);
    for (int k = 0; k < 4; ++k) {
      h ^= (v >> (8 * k)) & 0xFFu;
      h *= 1099511628211ull;
    }
  }
  return h == 0 ? 1 : h;
}

void BlockManager::touch_lru(int block) {
  if (in_lru_[block]) {
    lru_.erase(lru_pos_[block]);
    in_lru_[block] = 0;
  }
}

int BlockManager::take_block() {
  if (!free_.empty()) {
    const int b = free_.back();
    free_.pop_back();
    return b;
  }
  if (!lru_.empty()) {
    // victim: oldest unreferenced cached block (age), preferring rarely reused ones (value)
    auto victim = lru_.begin();
    int scanned = 0;
    for (auto it = lru_.begin(); it != lru_.end() && scanned < 8; ++it, ++scanned) {
      if (block_uses_[*it] < block_uses_[*victim]) victim = it;
    }
    const int b = *victim;
    lru_.erase(victim);
    in_lru_[b] = 0;
    if (block_hash_[b] != 0) {
      if (mesh_ != nullptr) {  // keep the prefix one tier down
        const int slot = mesh_->reserve_offload(block_hash_[b]);
        if (slot >= 0) offloads_.push_back({b, slot});
      }
      auto f = by_hash_.find(block_hash_[b]);
      if (f != by_hash_.end() && f->second == b) by_hash_.erase(f);
      block_hash_[b] = 0;
    }
    block_uses_[b] = 0;
    ++evictions_;
    return b;
  }
  return -1;
}

int BlockManager::match_prefix(const std::vector<int32_t>& tokens, int max_tokens, std::vector<int32_t>& table,
                               std::vector<uint64_t>& hashes) {
  if (!prefix_caching_) return 0;
  const int nfull = std::min<int>(static_cast<int>(tokens.size()), max_tokens) / block_size_;
  uint64_t prev = 0;
  int matched = 0;
  for (int i = 0; i < nfull; ++i) {
    const uint64_t h = chain_hash(prev, tokens.data() + i * block_size_, block_size_);
    auto it = by_hash_.find(h);
    if (it == by_hash_.end()) {
      // HBM miss: the block may still be one tier down
      const int slot = (mesh_ != nullptr && mesh_->contains(h)) ? mesh_->lookup(h) : -1;
      const int nb = slot >= 0 ? take_block() : -1;
      if (nb < 0) {
        ++misses_;
        break;
      }
      refcount_[nb] = 1;
      block_uses_[nb] = 1;
      block_hash_[nb] = h;
      by_hash_[h] = nb;
      restores_.push_back({nb, slot});
      ++hits_;
      table.push_back(nb);
      hashes.push_back(h);
      prev = h;
      ++matched;
      continue;
    }
    const int b = it->second;
    touch_lru(b);
    ++refcount_[b];
    ++block_uses_[b];
    ++hits_;
    ++reuses_;
    table.push_back(b);
    hashes.push_back(h);
    prev = h;
    ++matched;
  }
  return matched * block_size_;
}

bool BlockManager::ensure_capacity(std::vector<int32_t>& table, int num_tokens) {
  const int need = (num_tokens + block_size_ - 1) / block_size_ - static_cast<int>(table.size());
  if (need <= 0) return true;
  if (need > num_available()) return false;
  for (int i = 0; i < need; ++i) {
    const int b = take_block();
    if (b < 0) return false;  // unreachable given the check above
    refcount_[b] = 1;
    block_uses_[b] = 1;
    table.push_back(b);
  }
  return true;
}

void BlockManager::commit_full_blocks(const std::vector<int32_t>& tokens, int num_computed,
                                      const std::vector<int32_t>& table, std::vector<uint64_t>& hashes) {
  if (!prefix_caching_) return;
  const int nfull = std::min<int>(num_computed, static_cast<int>(tokens.size())) / block_size_;
  while (static_cast<int>(hashes.size()) < nfull && hashes.size() < table.size()) {
    const int i = static_cast<int>(hashes.size());
    const uint64_t prev = i == 0 ? 0 : hashes[i - 1];
    const uint64_t h = chain_hash(prev, tokens.data() + i * block_size_, block_size_);
    hashes.push_back(h);
    const int b = table[i];
    if (block_hash_[b] == 0 && by_hash_.find(h) == by_hash_.end()) {
      block_hash_[b] = h;
      by_hash_[h] = b;
    }
  }
}

void BlockManager::release(std::vector<int32_t>& table, std::vector<uint64_t>& hashes) {
  // release in reverse so the tail of a prefix is evicted before its head
  for (auto it = table.rbegin(); it != table.rend(); ++it) {
    const int b = *it;
    if (--refcount_[b] > 0) continue;
    if (refcount_[b] < 0) refcount_[b] = 0;
    if (prefix_caching_ && block_hash_[b] != 0) {
      // LRU: front is evicted first.  The tail of the sequence is appended
      // before its head, so a prefix loses its last blocks first.
      lru_.push_back(b);
      lru_pos_[b] = std::prev(lru_.end());
      in_lru_[b] = 1;
    } else {
      free_.push_back(b);
    }
  }
  table.clear();
  hashes.clear();
}

void BlockManager::truncate(std::vector<int32_t>& table, std::vector<uint64_t>& hashes, int num_tokens) {
  const int keep = (num_tokens + block_size_ - 1) / block_size_;
  while (static_cast<int>(table.size()) > keep) {
    const int b = table.back();
    table.pop_back();
    if (--refcount_[b] <= 0) {
      refcount_[b] = 0;
      if (block_hash_[b] != 0) {
        auto f = by_hash_.find(block_hash_[b]);
        if (f != by_hash_.end() && f->second == b) by_hash_.erase(f);
        block_hash_[b] = 0;
      }
      free_.push_back(b);
    }
  }
  const int full = num_tokens / block_size_;
  if (static_cast<int>(table.size()) > full) {
    // the kept partial tail block will be written again: it may no longer
    // stand for a full cached prefix, and it must not be shared
    const int b = table[full];
    if (refcount_[b] > 1) throw std::logic_error("truncate: cannot cut into a block shared by another sequence");
    if (block_hash_[b] != 0) {
      auto f = by_hash_.find(block_hash_[b]);
      if (f != by_hash_.end() && f->second == b) by_hash_.erase(f);
      block_hash_[b] = 0;
    }
  }
  if (static_cast<int>(hashes.size()) > full) hashes.resize(full);
}

int BlockManager::evict_cached(int n) {
  int done = 0;
  while (done < n && !lru_.empty()) {
    const int b = lru_.front();
    lru_.pop_front();
    in_lru_[b] = 0;
    if (block_hash_[b] != 0) {
      auto f = by_hash_.find(block_hash_[b]);
      if (f != by_hash_.end() && f->second == b) by_hash_.erase(f);
      block_hash_[b] = 0;
    }
    free_.push_back(b);
    ++evictions_;
    ++done;
  }
  return done;
}

void BlockManager::reset_prefix_cache() { evict_cached(static_cast<int>(lru_.size())); }

PoolMetrics BlockManager::metrics() const {
  PoolMetrics m;
  m.total_blocks = num_blocks_;
  m.free_blocks = static_cast<int64_t>(free_.size());
  m.cached_blocks = static_cast<int64_t>(lru_.size());
  m.active_blocks = num_blocks_ - m.free_blocks - m.cached_blocks;
  m.hits = hits_;
  m.misses = misses_;
  m.evictions = evictions_;
  m.reuses = reuses_;
  return m;
}

}  // namespace rt
}  // namespace bloom
