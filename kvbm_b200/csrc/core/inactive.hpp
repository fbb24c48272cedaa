// Inactive-pool indexes: which registered-but-unused block is evicted next.
//
// An InactiveIndex only sees (SeqHash, block id) pairs; the owning
// BlockPool holds all slot state under its mutex and calls these methods
// with that mutex held.
//
// Backends (parity: crates/kvbm-logical/src/pools/inactive/backends/):
//   LruIndex      - evicts in release order (lru_backend.rs; also the
//                   hashmap+FIFO reuse policy, hashmap_backend.rs/fifo.rs)
//   MultiLruIndex - four LRU tiers chosen by TinyLFU frequency at insert
//                   time, coldest tier evicted first (multi_lru_backend.rs)
//   LineageIndex  - prefix-tree aware: only leaves are evictable, so a
//                   shared prefix outlives every branch hanging off it
//                   (lineage/mod.rs); leaf order by first-insertion tick or
//                   FIFO of becoming a leaf (lineage/eviction.rs)
#pragma once

#include <array>
#include <cstdint>
#include <list>
#include <map>
#include <memory>
#include <optional>
#include <stdexcept>
#include <string>
#include <unordered_map>
#include <utility>
#include <vector>

#include "hash.hpp"
#include "tinylfu.hpp"

namespace kvbm {

using BlockId = int64_t;
using HashBlock = std::pair<SeqHash, BlockId>;

class InactiveIndex {
 public:
  virtual ~InactiveIndex() = default;
  // Remove and return the entry for `h`, if present.
  virtual std::optional<BlockId> take(const SeqHash& h) = 0;
  // Pull `count` entries in eviction order (fewer if not enough).
  virtual std::vector<HashBlock> evict(size_t count) = 0;
  virtual void insert(const SeqHash& h, BlockId id) = 0;
  virtual bool has(const SeqHash& h) const = 0;
  virtual size_t size() const = 0;
  virtual std::string name() const = 0;
};

// ---------------------------------------------------------------------------
class LruIndex : public InactiveIndex {
 public:
  explicit LruIndex(std::string nm = "lru") : name_(std::move(nm)) {}
  std::optional<BlockId> take(const SeqHash& h) override {
    auto it = map_.find(h);
    if (it == map_.end()) return std::nullopt;
    BlockId id = it->second->second;
    order_.erase(it->second);
    map_.erase(it);
    return id;
  }
  std::vector<HashBlock> evict(size_t count) override {
    std::vector<HashBlock> out;
    out.reserve(std::min(count, order_.size()));
    while (count-- > 0 && !order_.empty()) {
      out.push_back(order_.front());
      map_.erase(order_.front().first);
      order_.pop_front();
    }
    return out;
  }
  void insert(const SeqHash& h, BlockId id) override {
    order_.emplace_back(h, id);
    map_[h] = std::prev(order_.end());
  }
  bool has(const SeqHash& h) const override { return map_.count(h) != 0; }
  size_t size() const override { return map_.size(); }
  std::string name() const override { return name_; }

 private:
  std::string name_;
  std::list<HashBlock> order_;
  std::unordered_map<SeqHash, std::list<HashBlock>::iterator, SeqHashHasher> map_;
};

// ---------------------------------------------------------------------------
class MultiLruIndex : public InactiveIndex {
 public:
  MultiLruIndex(std::shared_ptr<TinyLfu> freq, std::array<uint32_t, 3> thresholds = {3, 8, 15})
      : freq_(std::move(freq)), th_(thresholds) {
    if (!(th_[0] < th_[1] && th_[1] < th_[2])) throw std::invalid_argument("thresholds must ascend");
    if (th_[2] > 15) throw std::invalid_argument("max threshold is 15 (4-bit counters)");
    if (th_[0] < 1) throw std::invalid_argument("cold threshold must be >= 1");
  }
  std::optional<BlockId> take(const SeqHash& h) override {
    auto it = where_.find(h);
    if (it == where_.end()) return std::nullopt;
    int tier = it->second;
    where_.erase(it);
    return tiers_[tier].take(h);
  }
  std::vector<HashBlock> evict(size_t count) override {
    std::vector<HashBlock> out;
    for (int t = 0; t < 4 && out.size() < count; ++t) {
      auto got = tiers_[t].evict(count - out.size());
      for (auto& p : got) {
        where_.erase(p.first);
        out.push_back(p);
      }
    }
    return out;
  }
  void insert(const SeqHash& h, BlockId id) override {
    const uint32_t f = freq_ ? freq_->estimate(h.lineage) : 0;
    int tier = f < th_[0] ? 0 : (f < th_[1] ? 1 : (f < th_[2] ? 2 : 3));
    tiers_[tier].insert(h, id);
    where_[h] = tier;
  }
  bool has(const SeqHash& h) const override { return where_.count(h) != 0; }
  size_t size() const override { return where_.size(); }
  std::string name() const override { return "multi_lru"; }
  size_t tier_size(int t) const { return tiers_[t].size(); }

 private:
  std::shared_ptr<TinyLfu> freq_;
  std::array<uint32_t, 3> th_;
  std::array<LruIndex, 4> tiers_;
  std::unordered_map<SeqHash, int, SeqHashHasher> where_;
};

// ---------------------------------------------------------------------------
class LineageIndex : public InactiveIndex {
 public:
  enum class LeafOrder { Tick, Fifo };
  explicit LineageIndex(LeafOrder order = LeafOrder::Tick) : order_(order) {}

  std::optional<BlockId> take(const SeqHash& h) override {
    auto it = nodes_.find(key(h));
    if (it == nodes_.end() || !it->second.real || it->second.hash != h) return std::nullopt;
    BlockId id = it->second.id;
    make_ghost_or_remove(it);
    --real_;
    return id;
  }
  std::vector<HashBlock> evict(size_t count) override {
    std::vector<HashBlock> out;
    while (out.size() < count && !leaves_.empty()) {
      auto lit = leaves_.begin();
      const uint64_t k = lit->second;
      leaves_.erase(lit);
      auto it = nodes_.find(k);
      Node& n = it->second;
      n.in_leaves = false;
      out.emplace_back(n.hash, n.id);
      --real_;
      remove_node(it);
    }
    return out;
  }
  void insert(const SeqHash& h, BlockId id) override {
    const uint64_t k = key(h);
    auto it = nodes_.find(k);
    if (it == nodes_.end()) {
      Node n;
      n.hash = h;
      n.id = id;
      n.real = true;
      n.tick = ++tick_;
      it = nodes_.emplace(k, n).first;
      // link to parent (creating a ghost placeholder if it is not here yet)
      if (h.position > 0) {
        const uint64_t pk = parent_key(h);
        auto pit = nodes_.find(pk);
        if (pit == nodes_.end()) {
          Node g;
          g.real = false;
          g.hash.position = h.position - 1;
          pit = nodes_.emplace(pk, g).first;
        }
        Node& p = pit->second;
        if (p.children++ == 0 && p.in_leaves) {
          leaves_.erase(p.leaf_key);
          p.in_leaves = false;
        }
        it->second.has_parent = true;
        it->second.parent = pk;
      }
    } else {
      // a ghost placeholder becomes real (a re-insert of a real one only
      // refreshes its block id)
      Node& n = it->second;
      if (n.real) {
        n.id = id;
        return;
      }
      n.hash = h;
      n.id = id;
      if (!n.real) {
        n.real = true;
        if (n.tick == 0) n.tick = ++tick_;
      }
      if (!n.has_parent && h.position > 0) {
        const uint64_t pk = parent_key(h);
        auto pit = nodes_.find(pk);
        if (pit == nodes_.end()) {
          Node g;
          g.real = false;
          g.hash.position = h.position - 1;
          pit = nodes_.emplace(pk, g).first;
        }
        Node& p = pit->second;
        if (p.children++ == 0 && p.in_leaves) {
          leaves_.erase(p.leaf_key);
          p.in_leaves = false;
        }
        n.has_parent = true;
        n.parent = pk;
      }
    }
    ++real_;
    Node& n = it->second;
    if (n.children == 0) add_leaf(k, n);
  }
  bool has(const SeqHash& h) const override {
    auto it = nodes_.find(key(h));
    return it != nodes_.end() && it->second.real && it->second.hash == h;
  }
  size_t size() const override { return real_; }
  std::string name() const override { return order_ == LeafOrder::Tick ? "lineage" : "lineage_fifo"; }
  size_t leaf_count() const { return leaves_.size(); }
  size_t node_count() const { return nodes_.size(); }

 private:
  struct Node {
    SeqHash hash;
    BlockId id = -1;
    bool real = false;
    bool in_leaves = false;
    bool has_parent = false;
    uint64_t parent = 0;
    uint64_t tick = 0;
    uint64_t leaf_key = 0;
    uint32_t children = 0;
  };
  static uint64_t key(const SeqHash& h) { return h.lineage; }
  static uint64_t parent_key(const SeqHash& h) { return h.parent; }

  void add_leaf(uint64_t k, Node& n) {
    if (!n.real || n.in_leaves) return;
    n.leaf_key = order_ == LeafOrder::Tick ? n.tick : ++fifo_seq_;
    leaves_.emplace(n.leaf_key, k);
    n.in_leaves = true;
  }
  void make_ghost_or_remove(std::unordered_map<uint64_t, Node>::iterator it) {
    Node& n = it->second;
    if (n.in_leaves) {
      leaves_.erase(n.leaf_key);
      n.in_leaves = false;
    }
    if (n.children > 0) {
      n.real = false;
      n.id = -1;
    } else {
      remove_node(it);
    }
  }
  // Remove a childless node and walk up: a parent that loses its last child
  // becomes a leaf (if real) or disappears (if a ghost).
  void remove_node(std::unordered_map<uint64_t, Node>::iterator it) {
    while (true) {
      Node& n = it->second;
      const bool hp = n.has_parent;
      const uint64_t pk = n.parent;
      nodes_.erase(it);
      if (!hp) return;
      auto pit = nodes_.find(pk);
      if (pit == nodes_.end()) return;
      Node& p = pit->second;
      if (--p.children > 0) return;
      if (p.real) {
        add_leaf(pk, p);
        return;
      }
      it = pit;  // ghost with no children left: remove it too
    }
  }

  LeafOrder order_;
  std::unordered_map<uint64_t, Node> nodes_;
  std::map<uint64_t, uint64_t> leaves_;  // leaf order key -> node key
  uint64_t tick_ = 0;
  uint64_t fifo_seq_ = 0;
  size_t real_ = 0;
};

inline std::unique_ptr<InactiveIndex> make_inactive_index(const std::string& kind, std::shared_ptr<TinyLfu> freq) {
  if (kind == "lru" || kind == "fifo" || kind == "hashmap") return std::make_unique<LruIndex>(kind);
  if (kind == "multi_lru") return std::make_unique<MultiLruIndex>(freq ? freq : std::make_shared<TinyLfu>());
  if (kind == "lineage" || kind == "lineage_tick") return std::make_unique<LineageIndex>(LineageIndex::LeafOrder::Tick);
  if (kind == "lineage_fifo") return std::make_unique<LineageIndex>(LineageIndex::LeafOrder::Fifo);
  throw std::invalid_argument("unknown inactive backend: " + kind);
}

}  // namespace kvbm
