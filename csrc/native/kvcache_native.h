// Native paged-KV block pool and radix prefix cache (the engine's per-step bookkeeping).
// Shared by the pybind module (kvcache_native.cpp) and the native scheduler (scheduler_native.cpp).
//
// Parity: the reference's page pool (advanced/src/paged_attention.rs:27-212: alloc / free per
// sequence) and its radix prompt cache (advanced/src/prompt_cache.rs:16-258: longest-prefix match,
// incremental insert, LRU eviction), both Rust.  Here:
//
//   BlockPool   blocks of `block_size` tokens with reference counts; a LIFO free list (block ids
//               come out 0, 1, 2, ... on a fresh pool, freed ids are reused first).
//   RadixCache  a radix tree whose edges are whole blocks of token ids; each node holds the KV block
//               of its edge and a reference on it.  A child is found by hashing (parent, tokens).
//               Eviction walks an ordered set of (last use, node) over the current leaves and frees
//               the least recently used leaf that no running sequence holds (block ref == 1), so an
//               eviction costs O(log n) plus one step per older leaf that a running sequence still
//               holds, instead of a walk over the whole tree.
//
// The Python classes in engine/kv_cache.py and engine/prefix_cache.py implement the same contract
// and serve as the oracle in tests/test_kvcache_native.py (random operation sequences, identical
// block ids, refs, matches and evictions).
#pragma once
#include <algorithm>
#include <cstdint>
#include <cstring>
#include <set>
#include <stdexcept>
#include <string>
#include <unordered_map>
#include <utility>
#include <vector>

namespace barq_native {

class BlockPool {
 public:
  BlockPool(int num_blocks, int block_size) : num_blocks_(num_blocks), block_size_(block_size), ref_(num_blocks, 0) {
    if (num_blocks <= 0 || block_size <= 0) throw std::invalid_argument("BlockPool: sizes must be positive");
    free_.reserve(num_blocks);
    for (int b = num_blocks - 1; b >= 0; --b) free_.push_back(b);
  }

  int n_free() const { return (int)free_.size(); }
  int n_used() const { return num_blocks_ - (int)free_.size(); }
  int num_blocks() const { return num_blocks_; }
  int block_size() const { return block_size_; }
  int blocks_for(long n_tokens) const { return (int)((n_tokens + block_size_ - 1) / block_size_); }
  bool can_allocate(int n) const { return n <= (int)free_.size(); }

  std::vector<int> allocate(int n) {
    if (n > (int)free_.size())
      throw std::out_of_range("need " + std::to_string(n) + " blocks, " + std::to_string(free_.size()) + " free");
    std::vector<int> out;
    out.reserve(n);
    for (int i = 0; i < n; ++i) {
      const int b = free_.back();
      free_.pop_back();
      ref_[b] = 1;
      out.push_back(b);
    }
    return out;
  }

  void retain(const std::vector<int>& blocks) {
    for (int b : blocks) {
      check(b);
      if (ref_[b] <= 0) throw std::invalid_argument("retain of free block " + std::to_string(b));
      ++ref_[b];
    }
  }

  void release(const std::vector<int>& blocks) {
    for (int b : blocks) {
      check(b);
      if (ref_[b] <= 0) throw std::invalid_argument("double free of block " + std::to_string(b));
      if (--ref_[b] == 0) free_.push_back(b);
    }
  }

  int ref(int b) const {
    check(b);
    return ref_[b];
  }
  const std::vector<int>& refs() const { return ref_; }
  const std::vector<int>& free_list() const { return free_; }

 private:
  void check(int b) const {
    if (b < 0 || b >= num_blocks_) throw std::out_of_range("block id " + std::to_string(b) + " out of range");
  }
  int num_blocks_, block_size_;
  std::vector<int> ref_;
  std::vector<int> free_;
};

class RadixCache {
 public:
  explicit RadixCache(BlockPool& pool) : pool_(pool), bs_(pool.block_size()) {
    nodes_.push_back(Node{-1, -1, 0, 0});  // root
  }

  // Longest cached block-aligned prefix of `tokens`: (block ids, tokens covered).
  std::pair<std::vector<int>, int> match(const std::vector<int>& tokens) {
    ++queries_;
    std::vector<int> out;
    int node = 0;
    for (size_t i = 0; i + bs_ <= tokens.size(); i += bs_) {
      auto it = child_.find(key(node, tokens.data() + i));
      if (it == child_.end()) break;
      touch(it->second);
      out.push_back(nodes_[it->second].block);
      node = it->second;
    }
    if (!out.empty()) ++hits_;
    return {out, (int)out.size() * bs_};
  }

  // Donate the full blocks of a finished sequence; the cache takes its own reference on new nodes.
  void insert(const std::vector<int>& tokens, const std::vector<int>& table) {
    int node = 0;
    const size_t n_full = std::min(tokens.size() / bs_, table.size());
    for (size_t j = 0; j < n_full; ++j) {
      const std::string k = key(node, tokens.data() + j * bs_);
      auto it = child_.find(k);
      int c;
      if (it == child_.end()) {
        c = alloc_node(node, table[j]);
        child_.emplace(k, c);
        keys_[c] = k;
        pool_.retain({table[j]});
        ++n_blocks_;
        if (nodes_[node].n_children++ == 0 && node != 0) leaves_.erase({nodes_[node].last_used, node});
        leaves_.insert({0, c});  // a new leaf; touch() below gives it its stamp
      } else {
        c = it->second;
      }
      touch(c);
      node = c;
    }
  }

  // Free up to n blocks from least-recently-used leaves that no running sequence references.
  int evict(int n) {
    int freed = 0;
    while (freed < n) {
      int victim = -1;
      for (const auto& lf : leaves_)
        if (pool_.ref(nodes_[lf.second].block) == 1) {
          victim = lf.second;
          break;
        }
      if (victim < 0) break;
      Node& v = nodes_[victim];
      leaves_.erase({v.last_used, victim});
      child_.erase(keys_[victim]);
      keys_.erase(victim);
      pool_.release({v.block});
      const int p = v.parent;
      free_nodes_.push_back(victim);
      v = Node{-1, -1, 0, 0};
      if (--nodes_[p].n_children == 0 && p != 0) leaves_.insert({nodes_[p].last_used, p});
      --n_blocks_;
      ++freed;
    }
    return freed;
  }

  int n_blocks() const { return n_blocks_; }
  long queries() const { return queries_; }
  long hits() const { return hits_; }

 private:
  struct Node {
    int parent, block;
    long last_used;
    int n_children;
  };

  std::string key(int parent, const int* toks) const {
    std::string k(sizeof(int) * (bs_ + 1), '\0');
    std::memcpy(&k[0], &parent, sizeof(int));
    std::memcpy(&k[sizeof(int)], toks, sizeof(int) * bs_);
    return k;
  }

  int alloc_node(int parent, int block) {
    int c;
    if (!free_nodes_.empty()) {
      c = free_nodes_.back();
      free_nodes_.pop_back();
    } else {
      c = (int)nodes_.size();
      nodes_.push_back(Node{});
    }
    nodes_[c] = Node{parent, block, 0, 0};
    return c;
  }

  // new last-use stamp; a leaf moves in the LRU set
  void touch(int c) {
    Node& nd = nodes_[c];
    const bool leaf = nd.n_children == 0;
    if (leaf) leaves_.erase({nd.last_used, c});
    nd.last_used = ++clock_;
    if (leaf) leaves_.insert({nd.last_used, c});
  }

  BlockPool& pool_;
  int bs_;
  std::vector<Node> nodes_;
  std::vector<int> free_nodes_;
  std::unordered_map<std::string, int> child_;  // (parent, block tokens) -> node
  std::unordered_map<int, std::string> keys_;   // node -> its key (for removal)
  std::set<std::pair<long, int>> leaves_;       // (last use, node) of every leaf
  long clock_ = 0, queries_ = 0, hits_ = 0;
  int n_blocks_ = 0;
};

}  // namespace barq_native
