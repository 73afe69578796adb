// Paged KV-cache block manager (host side).
//
// Parity: crates/swiftllm-core/src/memory/block_manager.rs (BlockAllocator
// free list + refcounts :107-236, BlockManager allocate/free/fork/copy/swap
// :240-535). Differences by design:
//   * one intrusive doubly-linked LRU free queue per pool, so a block that is
//     free but still holds a prefix-cache hash can be revived in O(1)
//     (the reference declares `prefix_cache` but never uses it, :265-269);
//   * copy-on-write is decided at append time (the reference's `copy_block`
//     only bumps refcounts, :402-426);
//   * the engine thread owns the manager, so there is no lock.
#pragma once
#include <cstdint>
#include <stdexcept>
#include <string>
#include <unordered_map>
#include <utility>
#include <vector>

namespace swift {

// One pool of equally sized blocks (GPU or host swap space).
class BlockPool {
 public:
  BlockPool(int num_blocks, bool enable_caching);

  int num_blocks() const { return num_blocks_; }
  int num_free() const { return num_free_; }
  int refcount(int b) const { return ref_[b]; }
  bool caching() const { return caching_; }

  // Take a block from the head of the free queue (the least recently freed).
  // Drops any cached hash it carried. Returns -1 when nothing is free.
  int allocate();
  void incref(int b);
  // Returns true if the block went back to the free queue.
  bool decref(int b);

  // Prefix cache: find a block holding `h`; takes a reference. -1 on miss.
  int lookup(uint64_t h);
  // Peek without taking a reference.
  bool contains(uint64_t h) const { return cached_.count(h) != 0; }
  // Attach `h` to block `b` if the hash is not cached yet.
  void set_hash(int b, uint64_t h);
  int64_t num_cached() const { return static_cast<int64_t>(cached_.size()); }
  void reset_cache();

 private:
  void push_tail(int b);
  void unlink(int b);

  int num_blocks_;
  bool caching_;
  std::vector<int> ref_, prev_, next_;
  std::vector<uint8_t> in_free_, has_hash_;
  std::vector<uint64_t> hash_;
  int head_ = -1, tail_ = -1, num_free_ = 0;
  std::unordered_map<uint64_t, int> cached_;
};

struct CopyPair {
  int src, dst;
};

class BlockManager {
 public:
  BlockManager(int block_size, int num_gpu_blocks, int num_cpu_blocks,
               double watermark, bool enable_prefix_caching);

  int block_size() const { return block_size_; }
  int blocks_needed(int64_t num_tokens) const {
    return static_cast<int>((num_tokens + block_size_ - 1) / block_size_);
  }
  int num_free_gpu() const { return gpu_.num_free(); }
  int num_free_cpu() const { return cpu_.num_free(); }
  int num_gpu_blocks() const { return gpu_.num_blocks(); }
  int num_cpu_blocks() const { return cpu_.num_blocks(); }
  int watermark_blocks() const { return watermark_blocks_; }
  bool prefix_caching() const { return gpu_.caching(); }
  BlockPool& gpu() { return gpu_; }

  // True if `n` more GPU blocks can be taken (keeping the watermark free if
  // `keep_watermark`).
  bool can_allocate(int n, bool keep_watermark) const;

  // Prefix-cache probe for a new sequence: returns how many leading full
  // blocks of `tokens` are cached (no references taken).
  int count_cached_blocks(const int32_t* tokens, int64_t n) const;
  // Start a table for `seq`, reusing up to `max_blocks` cached prefix blocks.
  // Returns the number of tokens covered by reused blocks.
  int64_t allocate_cached_prefix(int64_t seq, const int32_t* tokens, int64_t n,
                                 int max_blocks);
  // Grow the table of `seq` to cover `total_tokens`. Any write into a shared
  // partial last block first copies it (pairs appended to `cow`).
  // Returns false (and changes nothing) if blocks ran out.
  bool ensure_slots(int64_t seq, int64_t num_computed, int64_t total_tokens,
                    std::vector<CopyPair>* cow);
  int blocks_to_grow(int64_t seq, int64_t num_computed, int64_t total_tokens) const;
  // Register hashes of the full blocks of `seq` covered by `num_tokens`.
  void register_full_blocks(int64_t seq, const int32_t* tokens, int64_t num_tokens);

  void free(int64_t seq);
  void fork(int64_t parent, int64_t child);
  bool has(int64_t seq) const { return tables_.count(seq) != 0; }
  const std::vector<int>& table(int64_t seq) const;

  bool can_swap_out(int64_t seq) const;
  bool can_swap_in(int64_t seq) const;
  // Move every block of `seq` to the host pool; (gpu, cpu) pairs appended.
  void swap_out(int64_t seq, std::vector<CopyPair>* mapping);
  // Move back; (cpu, gpu) pairs appended.
  void swap_in(int64_t seq, std::vector<CopyPair>* mapping);
  bool is_swapped(int64_t seq) const { return cpu_tables_.count(seq) != 0; }

  void reset_prefix_cache() { gpu_.reset_cache(); }

 private:
  static uint64_t chain_hash(uint64_t prev, const int32_t* toks, int n);

  int block_size_;
  int watermark_blocks_;
  BlockPool gpu_, cpu_;
  std::unordered_map<int64_t, std::vector<int>> tables_;
  std::unordered_map<int64_t, std::vector<int>> cpu_tables_;
  // per-seq: number of leading blocks whose hash is registered + last hash
  std::unordered_map<int64_t, std::pair<int, uint64_t>> hashed_;
};

}  // namespace swift
