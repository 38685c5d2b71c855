// Paged KV block manager with prefix caching.
//
// Same semantics as the reference's KVCacheManager (src/memory/kv_cache_manager.cpp: ctor :174,
// allocate_slots :458, free_slots :513, find_longest_prefix_hit :441, cache_full_blocks :648,
// trim_request_to_tokens :837): a pool of fixed-size blocks, block 0 reserved as the null block,
// an LRU free queue (freed blocks go to the tail in reverse order so that a request's tail blocks
// are evicted first), reference counts for blocks shared through the prefix cache, and a
// hash -> block map whose entry is dropped when a cached block is reused for new data.
// The free queue is an intrusive doubly-linked list over block indices (O(1) remove for prefix
// hits), and request block lists are keyed by integer request ids.
#pragma once
#include <cstdint>
#include <unordered_map>
#include <vector>

namespace vmc {

class BlockManager {
 public:
  BlockManager(int64_t num_blocks, int block_size, bool enable_prefix_caching);

  int block_size() const { return block_size_; }
  int64_t num_blocks() const { return static_cast<int64_t>(blocks_.size()); }
  int64_t num_free_blocks() const { return num_free_; }
  // Fraction of usable (non-null) blocks in use.
  double usage() const;
  bool prefix_caching() const { return enable_caching_; }

  // Ensure request `rid` owns enough blocks for `num_tokens` tokens. `hit_blocks` are prefix-cache
  // hits to append first (their ref counts are bumped). Returns false and changes nothing when the
  // free pool is too small.
  bool allocate(int64_t rid, int64_t num_tokens, const std::vector<int32_t>& hit_blocks = {});
  bool can_allocate(int64_t rid, int64_t num_tokens) const;
  int64_t blocks_needed(int64_t rid, int64_t num_tokens) const;
  void free(int64_t rid);
  // Release blocks beyond those needed for `num_tokens` tokens (speculative rollback).
  void trim(int64_t rid, int64_t num_tokens);
  const std::vector<int32_t>& blocks_of(int64_t rid) const;
  bool has(int64_t rid) const { return req_blocks_.count(rid) != 0; }

  // Prefix cache.
  int find_longest_prefix_hit(const std::vector<uint64_t>& hashes, int max_blocks, std::vector<int32_t>& out) const;
  void cache_full_blocks(int64_t rid, const std::vector<uint64_t>& hashes, int num_full_blocks);
  int64_t num_cached_blocks() const { return static_cast<int64_t>(hash_to_block_.size()); }
  void reset_prefix_cache();

  // Chained FNV-1a over full blocks of `block_size` tokens; hash k covers tokens [0, (k+1)*bs).
  static std::vector<uint64_t> block_hashes(const int32_t* tokens, int64_t n_tokens, int block_size);

 private:
  struct Block {
    int32_t prev = -1, next = -1;
    int32_t ref = 0;
    bool in_free = false;
    bool has_hash = false;
    uint64_t hash = 0;
  };
  void free_remove(int32_t b);
  void free_append(int32_t b);
  int32_t free_pop();
  void unhash(int32_t b);

  int block_size_;
  bool enable_caching_;
  std::vector<Block> blocks_;
  int32_t head_ = -1, tail_ = -1;
  int64_t num_free_ = 0;
  std::unordered_map<int64_t, std::vector<int32_t>> req_blocks_;
  std::unordered_map<uint64_t, int32_t> hash_to_block_;
};

}  // namespace vmc
