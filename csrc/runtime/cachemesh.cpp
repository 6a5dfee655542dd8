#include "cachemesh.h"

#include <cstdio>
#include <cstring>
#include <dirent.h>
#include <stdexcept>
#include <sys/stat.h>
#include <unistd.h>

namespace bloom {
namespace rt {

namespace {
constexpr char kMagic[8] = {'B', 'L', 'M', 'K', 'V', 'L', '3', '1'};
}

CacheMesh::CacheMesh(const CacheMeshConfig& cfg, uint8_t* l2_base) : cfg_(cfg), l2_base_(l2_base) {
  if (cfg_.l2_slots < 0 || cfg_.block_bytes < 0) throw std::invalid_argument("CacheMesh: bad sizes");
  for (int64_t s = cfg_.l2_slots - 1; s >= 0; --s) free_slots_.push_back(static_cast<int>(s));
  pending_.assign(static_cast<size_t>(cfg_.l2_slots), 0);
  m_.l2_capacity = cfg_.l2_slots;
  m_.l3_capacity = cfg_.l3_dir.empty() ? 0 : cfg_.l3_max_blocks;
  if (m_.l3_capacity > 0) {
    ::mkdir(cfg_.l3_dir.c_str(), 0755);
    scan_l3();
  }
}

std::string CacheMesh::l3_path(uint64_t hash) const {
  char name[64];
  std::snprintf(name, sizeof name, "-%016llx.kv", static_cast<unsigned long long>(hash));
  return cfg_.l3_dir + "/" + cfg_.name_space + name;
}

void CacheMesh::scan_l3() {
  DIR* d = ::opendir(cfg_.l3_dir.c_str());
  if (d == nullptr) return;
  const std::string prefix = cfg_.name_space + "-";
  while (dirent* e = ::readdir(d)) {
    const std::string n = e->d_name;
    if (n.size() != prefix.size() + 16 + 3 || n.compare(0, prefix.size(), prefix) != 0 ||
        n.compare(n.size() - 3, 3, ".kv") != 0)
      continue;
    const uint64_t h = std::strtoull(n.substr(prefix.size(), 16).c_str(), nullptr, 16);
    if (l3_pos_.count(h)) continue;
    l3_lru_.push_back(h);
    l3_pos_[h] = std::prev(l3_lru_.end());
  }
  ::closedir(d);
  m_.l3_used = static_cast<int64_t>(l3_lru_.size());
}

void CacheMesh::touch(uint64_t hash) {
  auto it = l2_pos_.find(hash);
  if (it == l2_pos_.end()) return;
  l2_lru_.erase(it->second);
  l2_lru_.push_back(hash);
  it->second = std::prev(l2_lru_.end());
}

void CacheMesh::l3_touch(uint64_t hash) {
  auto it = l3_pos_.find(hash);
  if (it == l3_pos_.end()) return;
  l3_lru_.erase(it->second);
  l3_lru_.push_back(hash);
  it->second = std::prev(l3_lru_.end());
}

void CacheMesh::spill_to_l3(uint64_t hash, int slot) {
  if (m_.l3_capacity <= 0) return;
  if (l3_pos_.count(hash)) {
    l3_touch(hash);
    return;
  }
  while (static_cast<int64_t>(l3_lru_.size()) >= m_.l3_capacity && !l3_lru_.empty()) {
    const uint64_t old = l3_lru_.front();
    l3_lru_.pop_front();
    l3_pos_.erase(old);
    ::unlink(l3_path(old).c_str());
    ++m_.l3_evictions;
  }
  const std::string path = l3_path(hash);
  const std::string tmp = path + ".tmp";
  FILE* f = std::fopen(tmp.c_str(), "wb");
  if (f == nullptr) return;
  const uint64_t bytes = static_cast<uint64_t>(cfg_.block_bytes);
  bool ok = std::fwrite(kMagic, 1, 8, f) == 8 && std::fwrite(&hash, 8, 1, f) == 1 && std::fwrite(&bytes, 8, 1, f) == 1 &&
            std::fwrite(l2_base_ + static_cast<int64_t>(slot) * cfg_.block_bytes, 1, bytes, f) == bytes;
  ok = (std::fclose(f) == 0) && ok;
  if (!ok || std::rename(tmp.c_str(), path.c_str()) != 0) {
    ::unlink(tmp.c_str());
    return;
  }
  l3_lru_.push_back(hash);
  l3_pos_[hash] = std::prev(l3_lru_.end());
  ++m_.l3_writes;
  m_.l3_used = static_cast<int64_t>(l3_lru_.size());
}

int CacheMesh::take_slot() {
  if (!free_slots_.empty()) {
    const int s = free_slots_.back();
    free_slots_.pop_back();
    return s;
  }
  auto it = l2_lru_.begin();
  while (it != l2_lru_.end() && pending_[l2_map_[*it]]) ++it;  // never a slot with a copy queued this step
  if (it == l2_lru_.end()) return -1;
  const uint64_t old = *it;
  l2_lru_.erase(it);
  l2_pos_.erase(old);
  const int s = l2_map_[old];
  l2_map_.erase(old);
  ++m_.l2_evictions;
  spill_to_l3(old, s);  // the slot's bytes are complete: copies of earlier steps were synchronised
  return s;
}

int CacheMesh::reserve_offload(uint64_t hash) {
  if (!enabled()) return -1;
  auto it = l2_map_.find(hash);
  if (it != l2_map_.end()) {  // the same prefix block is already in L2: nothing to copy
    touch(hash);
    return -1;
  }
  const int s = take_slot();
  if (s < 0) return -1;
  pending_[s] = 1;
  l2_map_[hash] = s;
  l2_lru_.push_back(hash);
  l2_pos_[hash] = std::prev(l2_lru_.end());
  ++m_.offloads;
  m_.l2_used = static_cast<int64_t>(l2_map_.size());
  return s;
}

bool CacheMesh::contains(uint64_t hash) const { return l2_map_.count(hash) || l3_pos_.count(hash); }

int CacheMesh::lookup(uint64_t hash) {
  if (!enabled()) return -1;
  auto it = l2_map_.find(hash);
  if (it != l2_map_.end()) {
    touch(hash);
    pending_[it->second] = 1;
    ++m_.l2_hits;
    return it->second;
  }
  if (l3_pos_.count(hash) == 0) {
    ++m_.misses;
    return -1;
  }
  // promote the L3 file into an L2 slot
  FILE* f = std::fopen(l3_path(hash).c_str(), "rb");
  if (f == nullptr) {
    l3_lru_.erase(l3_pos_[hash]);
    l3_pos_.erase(hash);
    ++m_.misses;
    return -1;
  }
  char magic[8];
  uint64_t h = 0, bytes = 0;
  const bool hdr = std::fread(magic, 1, 8, f) == 8 && std::memcmp(magic, kMagic, 8) == 0 &&
                   std::fread(&h, 8, 1, f) == 1 && std::fread(&bytes, 8, 1, f) == 1 && h == hash &&
                   bytes == static_cast<uint64_t>(cfg_.block_bytes);
  int s = -1;
  if (hdr) s = take_slot();
  bool ok = false;
  if (s >= 0) ok = std::fread(l2_base_ + static_cast<int64_t>(s) * cfg_.block_bytes, 1, bytes, f) == bytes;
  std::fclose(f);
  if (!ok) {
    if (s >= 0) free_slots_.push_back(s);
    ++m_.misses;
    return -1;
  }
  l3_touch(hash);
  pending_[s] = 1;
  l2_map_[hash] = s;
  l2_lru_.push_back(hash);
  l2_pos_[hash] = std::prev(l2_lru_.end());
  m_.l2_used = static_cast<int64_t>(l2_map_.size());
  ++m_.l3_hits;
  return s;
}

CacheMeshMetrics CacheMesh::metrics() const {
  CacheMeshMetrics r = m_;
  r.l2_used = static_cast<int64_t>(l2_map_.size());
  r.l3_used = static_cast<int64_t>(l3_lru_.size());
  return r;
}

}  // namespace rt
}  // namespace bloom
