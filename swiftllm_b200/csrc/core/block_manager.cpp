#include "block_manager.h"

#include <algorithm>

namespace swift {

// ---------------------------------------------------------------- BlockPool

BlockPool::BlockPool(int num_blocks, bool enable_caching)
    : num_blocks_(num_blocks),
      caching_(enable_caching),
      ref_(num_blocks, 0),
      prev_(num_blocks, -1),
      next_(num_blocks, -1),
      in_free_(num_blocks, 0),
      has_hash_(num_blocks, 0),
      hash_(num_blocks, 0) {
  if (num_blocks < 0) throw std::invalid_argument("num_blocks must be >= 0");
  for (int b = 0; b < num_blocks; ++b) push_tail(b);
}

void BlockPool::push_tail(int b) {
  prev_[b] = tail_;
  next_[b] = -1;
  if (tail_ >= 0) next_[tail_] = b; else head_ = b;
  tail_ = b;
  in_free_[b] = 1;
  ++num_free_;
}

void BlockPool::unlink(int b) {
  if (prev_[b] >= 0) next_[prev_[b]] = next_[b]; else head_ = next_[b];
  if (next_[b] >= 0) prev_[next_[b]] = prev_[b]; else tail_ = prev_[b];
  prev_[b] = next_[b] = -1;
  in_free_[b] = 0;
  --num_free_;
}

int BlockPool::allocate() {
  if (head_ < 0) return -1;
  int b = head_;
  unlink(b);
  if (has_hash_[b]) {
    auto it = cached_.find(hash_[b]);
    if (it != cached_.end() && it->second == b) cached_.erase(it);
    has_hash_[b] = 0;
  }
  ref_[b] = 1;
  return b;
}

void BlockPool::incref(int b) {
  if (in_free_[b]) unlink(b);
  ++ref_[b];
}

bool BlockPool::decref(int b) {
  if (ref_[b] <= 0) throw std::logic_error("double free of KV block " + std::to_string(b));
  if (--ref_[b] == 0) {
    push_tail(b);
    return true;
  }
  return false;
}

int BlockPool::lookup(uint64_t h) {
  auto it = cached_.find(h);
  if (it == cached_.end()) return -1;
  incref(it->second);
  return it->second;
}

void BlockPool::set_hash(int b, uint64_t h) {
  if (!caching_ || has_hash_[b]) return;
  if (cached_.count(h)) return;
  cached_[h] = b;
  hash_[b] = h;
  has_hash_[b] = 1;
}

void BlockPool::reset_cache() {
  cached_.clear();
  std::fill(has_hash_.begin(), has_hash_.end(), 0);
}

// ------------------------------------------------------------- BlockManager

BlockManager::BlockManager(int block_size, int num_gpu_blocks, int num_cpu_blocks,
                           double watermark, bool enable_prefix_caching)
    : block_size_(block_size),
      watermark_blocks_(static_cast<int>(watermark * num_gpu_blocks)),
      gpu_(num_gpu_blocks, enable_prefix_caching),
      cpu_(num_cpu_blocks, false) {
  if (block_size <= 0) throw std::invalid_argument("block_size must be > 0");
}

bool BlockManager::can_allocate(int n, bool keep_watermark) const {
  int reserve = keep_watermark ? watermark_blocks_ : 0;
  return gpu_.num_free() - n >= reserve;
}

uint64_t BlockManager::chain_hash(uint64_t prev, const int32_t* toks, int n) {
  // FNV-1a over the previous hash and the block's token ids, then a
  // splitmix64 finaliser to spread the bits.
  uint64_t h = 1469598103934665603ull ^ prev;
  for (int i = 0; i < n; ++i) {
    uint32_t t = static_cast<uint32_t>(toks[i]);
    for (int k = 0; k < 4; ++k) {
      h ^= (t >> (8 * k)) & 0xffu;
      h *= 1099511628211ull;
    }
  }
  h += 0x9e3779b97f4a7c15ull;
  h = (h ^ (h >> 30)) * 0xbf58476d1ce4e5b9ull;
  h = (h ^ (h >> 27)) * 0x94d049bb133111ebull;
  return h ^ (h >> 31);
}

int BlockManager::count_cached_blocks(const int32_t* tokens, int64_t n) const {
  if (!gpu_.caching()) return 0;
  int full = static_cast<int>(n / block_size_);
  uint64_t h = 0;
  int hits = 0;
  for (int i = 0; i < full; ++i) {
    h = chain_hash(h, tokens + static_cast<int64_t>(i) * block_size_, block_size_);
    if (!gpu_.contains(h)) break;
    ++hits;
  }
  return hits;
}

int64_t BlockManager::allocate_cached_prefix(int64_t seq, const int32_t* tokens,
                                             int64_t n, int max_blocks) {
  auto& t = tables_[seq];
  if (!t.empty()) throw std::logic_error("allocate_cached_prefix on a live sequence");
  if (!gpu_.caching()) return 0;
  int full = static_cast<int>(std::min<int64_t>(n / block_size_, max_blocks));
  uint64_t h = 0;
  int hits = 0;
  for (int i = 0; i < full; ++i) {
    uint64_t nh = chain_hash(h, tokens + static_cast<int64_t>(i) * block_size_, block_size_);
    int b = gpu_.lookup(nh);
    if (b < 0) break;
    t.push_back(b);
    h = nh;
    ++hits;
  }
  hashed_[seq] = {hits, h};
  return static_cast<int64_t>(hits) * block_size_;
}

int BlockManager::blocks_to_grow(int64_t seq, int64_t num_computed, int64_t total) const {
  auto it = tables_.find(seq);
  int have = it == tables_.end() ? 0 : static_cast<int>(it->second.size());
  int need = blocks_needed(total) - have;
  if (need < 0) need = 0;
  // a write into a shared partial block costs one more block (copy-on-write)
  if (it != tables_.end() && total > num_computed && num_computed % block_size_ != 0) {
    int last = static_cast<int>(num_computed / block_size_);
    if (last < have && gpu_.refcount(it->second[last]) > 1) ++need;
  }
  return need;
}

bool BlockManager::ensure_slots(int64_t seq, int64_t num_computed, int64_t total,
                                std::vector<CopyPair>* cow) {
  int need = blocks_to_grow(seq, num_computed, total);
  if (need > gpu_.num_free()) return false;
  auto& t = tables_[seq];
  if (total > num_computed && num_computed % block_size_ != 0) {
    int last = static_cast<int>(num_computed / block_size_);
    if (last < static_cast<int>(t.size()) && gpu_.refcount(t[last]) > 1) {
      int nb = gpu_.allocate();
      if (cow) cow->push_back({t[last], nb});
      gpu_.decref(t[last]);
      t[last] = nb;
    }
  }
  int want = blocks_needed(total);
  while (static_cast<int>(t.size()) < want) t.push_back(gpu_.allocate());
  return true;
}

void BlockManager::register_full_blocks(int64_t seq, const int32_t* tokens, int64_t n) {
  if (!gpu_.caching()) return;
  auto it = tables_.find(seq);
  if (it == tables_.end()) return;
  auto& st = hashed_[seq];
  int full = static_cast<int>(std::min<int64_t>(n / block_size_, it->second.size()));
  for (int i = st.first; i < full; ++i) {
    st.second = chain_hash(st.second, tokens + static_cast<int64_t>(i) * block_size_, block_size_);
    gpu_.set_hash(it->second[i], st.second);
    st.first = i + 1;
  }
}

void BlockManager::free(int64_t seq) {
  auto it = tables_.find(seq);
  if (it != tables_.end()) {
    // free in reverse so that prefix blocks (most reusable) are evicted last
    for (auto r = it->second.rbegin(); r != it->second.rend(); ++r) gpu_.decref(*r);
    tables_.erase(it);
  }
  auto ct = cpu_tables_.find(seq);
  if (ct != cpu_tables_.end()) {
    for (int b : ct->second) cpu_.decref(b);
    cpu_tables_.erase(ct);
  }
  hashed_.erase(seq);
}

void BlockManager::fork(int64_t parent, int64_t child) {
  auto it = tables_.find(parent);
  if (it == tables_.end()) throw std::logic_error("fork of unknown sequence");
  std::vector<int> copy = it->second;
  for (int b : copy) gpu_.incref(b);
  tables_[child] = std::move(copy);
  auto h = hashed_.find(parent);
  if (h != hashed_.end()) hashed_[child] = h->second;
}

const std::vector<int>& BlockManager::table(int64_t seq) const {
  static const std::vector<int> empty;
  auto it = tables_.find(seq);
  return it == tables_.end() ? empty : it->second;
}

bool BlockManager::can_swap_out(int64_t seq) const {
  auto it = tables_.find(seq);
  return it != tables_.end() && static_cast<int>(it->second.size()) <= cpu_.num_free();
}

bool BlockManager::can_swap_in(int64_t seq) const {
  auto it = cpu_tables_.find(seq);
  return it != cpu_tables_.end() &&
         can_allocate(static_cast<int>(it->second.size()), true);
}

void BlockManager::swap_out(int64_t seq, std::vector<CopyPair>* mapping) {
  auto it = tables_.find(seq);
  if (it == tables_.end()) throw std::logic_error("swap_out of unknown sequence");
  std::vector<int> ct;
  ct.reserve(it->second.size());
  for (int g : it->second) {
    int c = cpu_.allocate();
    if (c < 0) throw std::runtime_error("host swap space exhausted");
    mapping->push_back({g, c});
    ct.push_back(c);
  }
  for (auto r = it->second.rbegin(); r != it->second.rend(); ++r) gpu_.decref(*r);
  tables_.erase(it);
  hashed_.erase(seq);
  cpu_tables_[seq] = std::move(ct);
}

void BlockManager::swap_in(int64_t seq, std::vector<CopyPair>* mapping) {
  auto it = cpu_tables_.find(seq);
  if (it == cpu_tables_.end()) throw std::logic_error("swap_in of unknown sequence");
  std::vector<int> gt;
  gt.reserve(it->second.size());
  for (int c : it->second) {
    int g = gpu_.allocate();
    if (g < 0) throw std::runtime_error("GPU blocks exhausted during swap-in");
    mapping->push_back({c, g});
    gt.push_back(g);
    cpu_.decref(c);
  }
  cpu_tables_.erase(it);
  tables_[seq] = std::move(gt);
  hashed_[seq] = {0, 0};
}

}  // namespace swift
