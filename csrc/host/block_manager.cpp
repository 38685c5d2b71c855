#include "block_manager.hpp"

#include <algorithm>
#include <stdexcept>
#include <string>

namespace vmc {

BlockManager::BlockManager(int64_t num_blocks, int block_size, bool enable_prefix_caching)
    : block_size_(block_size), enable_caching_(enable_prefix_caching) {
  if (num_blocks < 2) throw std::runtime_error("BlockManager: need at least 2 blocks (block 0 is the null block)");
  if (block_size <= 0) throw std::runtime_error("BlockManager: block_size must be positive");
  blocks_.resize(static_cast<size_t>(num_blocks));
  // Block 0 is the null block: never handed out, used as padding in block tables.
  for (int32_t b = 1; b < static_cast<int32_t>(num_blocks); ++b) free_append(b);
}

double BlockManager::usage() const {
  int64_t usable = num_blocks() - 1;
  return usable <= 0 ? 0.0 : 1.0 - static_cast<double>(num_free_) / static_cast<double>(usable);
}

void BlockManager::free_remove(int32_t b) {
  Block& blk = blocks_[b];
  if (!blk.in_free) return;
  if (blk.prev >= 0) blocks_[blk.prev].next = blk.next; else head_ = blk.next;
  if (blk.next >= 0) blocks_[blk.next].prev = blk.prev; else tail_ = blk.prev;
  blk.prev = blk.next = -1;
  blk.in_free = false;
  --num_free_;
}

void BlockManager::free_append(int32_t b) {
  Block& blk = blocks_[b];
  if (blk.in_free) return;
  blk.prev = tail_;
  blk.next = -1;
  if (tail_ >= 0) blocks_[tail_].next = b; else head_ = b;
  tail_ = b;
  blk.in_free = true;
  ++num_free_;
}

int32_t BlockManager::free_pop() {
  int32_t b = head_;
  if (b < 0) return -1;
  free_remove(b);
  return b;
}

void BlockManager::unhash(int32_t b) {
  Block& blk = blocks_[b];
  if (!blk.has_hash) return;
  auto it = hash_to_block_.find(blk.hash);
  if (it != hash_to_block_.end() && it->second == b) hash_to_block_.erase(it);
  blk.has_hash = false;
  blk.hash = 0;
}

int64_t BlockManager::blocks_needed(int64_t rid, int64_t num_tokens) const {
  int64_t want = (num_tokens + block_size_ - 1) / block_size_;
  auto it = req_blocks_.find(rid);
  int64_t have = it == req_blocks_.end() ? 0 : static_cast<int64_t>(it->second.size());
  return std::max<int64_t>(0, want - have);
}

bool BlockManager::can_allocate(int64_t rid, int64_t num_tokens) const {
  return blocks_needed(rid, num_tokens) <= num_free_;
}

bool BlockManager::allocate(int64_t rid, int64_t num_tokens, const std::vector<int32_t>& hit_blocks) {
  auto& list = req_blocks_[rid];
  // Count how many of the hit blocks would leave the free pool, to check capacity up front.
  int64_t hits_from_free = 0;
  for (int32_t b : hit_blocks) {
    if (b <= 0 || b >= static_cast<int32_t>(blocks_.size())) throw std::runtime_error("allocate: bad hit block id");
    if (blocks_[b].in_free) ++hits_from_free;
  }
  int64_t want = (num_tokens + block_size_ - 1) / block_size_;
  int64_t have = static_cast<int64_t>(list.size() + hit_blocks.size());
  int64_t fresh = std::max<int64_t>(0, want - have);
  if (fresh + hits_from_free > num_free_) {
    if (list.empty()) req_blocks_.erase(rid);
    return false;
  }
  for (int32_t b : hit_blocks) {
    free_remove(b);
    blocks_[b].ref += 1;
    list.push_back(b);
  }
  for (int64_t k = 0; k < fresh; ++k) {
    int32_t b = free_pop();
    if (b < 0) throw std::runtime_error("allocate: free list corrupted");
    if (blocks_[b].has_hash) unhash(b);  // evict the cached contents
    blocks_[b].ref = 1;
    list.push_back(b);
  }
  return true;
}

void BlockManager::free(int64_t rid) {
  auto it = req_blocks_.find(rid);
  if (it == req_blocks_.end()) return;
  // Return blocks tail-first so that the least useful (latest) prefix blocks are evicted first.
  auto& list = it->second;
  for (auto r = list.rbegin(); r != list.rend(); ++r) {
    Block& blk = blocks_[*r];
    if (--blk.ref <= 0) {
      blk.ref = 0;
      free_append(*r);
    }
  }
  req_blocks_.erase(it);
}

void BlockManager::trim(int64_t rid, int64_t num_tokens) {
  if (num_tokens < 0) throw std::runtime_error("trim: num_tokens must be non-negative");
  auto it = req_blocks_.find(rid);
  if (it == req_blocks_.end()) return;
  auto& list = it->second;
  size_t keep = static_cast<size_t>((num_tokens + block_size_ - 1) / block_size_);
  if (keep >= list.size()) return;
  for (size_t k = list.size(); k-- > keep;) {
    Block& blk = blocks_[list[k]];
    if (--blk.ref <= 0) {
      blk.ref = 0;
      unhash(list[k]);  // partially overwritten speculative blocks must not be served as cache hits
      free_append(list[k]);
    }
  }
  list.resize(keep);
}

const std::vector<int32_t>& BlockManager::blocks_of(int64_t rid) const {
  static const std::vector<int32_t> empty;
  auto it = req_blocks_.find(rid);
  return it == req_blocks_.end() ? empty : it->second;
}

int BlockManager::find_longest_prefix_hit(const std::vector<uint64_t>& hashes, int max_blocks,
                                          std::vector<int32_t>& out) const {
  out.clear();
  if (!enable_caching_) return 0;
  int n = std::min<int>(max_blocks, static_cast<int>(hashes.size()));
  for (int k = 0; k < n; ++k) {
    auto it = hash_to_block_.find(hashes[k]);
    if (it == hash_to_block_.end()) break;
    out.push_back(it->second);
  }
  return static_cast<int>(out.size());
}

void BlockManager::cache_full_blocks(int64_t rid, const std::vector<uint64_t>& hashes, int num_full_blocks) {
  if (!enable_caching_) return;
  auto it = req_blocks_.find(rid);
  if (it == req_blocks_.end()) return;
  auto& list = it->second;
  int n = std::min<int>({num_full_blocks, static_cast<int>(list.size()), static_cast<int>(hashes.size())});
  for (int k = 0; k < n; ++k) {
    Block& blk = blocks_[list[k]];
    if (blk.has_hash) continue;
    if (hash_to_block_.count(hashes[k])) continue;  // identical content already cached elsewhere
    blk.has_hash = true;
    blk.hash = hashes[k];
    hash_to_block_[hashes[k]] = list[k];
  }
}

void BlockManager::reset_prefix_cache() {
  for (auto& kv : hash_to_block_) {
    blocks_[kv.second].has_hash = false;
    blocks_[kv.second].hash = 0;
  }
  hash_to_block_.clear();
}

std::vector<uint64_t> BlockManager::block_hashes(const int32_t* tokens, int64_t n_tokens, int block_size) {
  int64_t nb = n_tokens / block_size;
  std::vector<uint64_t> out(static_cast<size_t>(nb));
  uint64_t h = 0xcbf29ce484222325ULL;  // FNV-1a 64-bit offset basis
  for (int64_t b = 0; b < nb; ++b) {
    for (int i = 0; i < block_size; ++i) {
      h ^= static_cast<uint64_t>(static_cast<int64_t>(tokens[b * block_size + i]));
      h *= 0x100000001b3ULL;  // FNV-1a 64-bit prime
    }
    out[static_cast<size_t>(b)] = h;
  }
  return out;
}

}  // namespace vmc
