// Branch points of the registered block tree.
//
// Every registered sequence hash names its parent (position - 1, parent
// lineage). A node whose registered children carry more than one distinct
// lineage is a branch point: the place where sequences that share a prefix
// diverge. The tracker keeps, for every parent node that has had a child
// registered, the set of distinct child lineages (the first child inline,
// further ones in a small vector, so the common fanout-1 node costs no heap
// allocation), and a bounded history of branch points scored by
// observations / (ticks since last update + 1); the lowest score is evicted
// when the history is full. One registration is one hash-map probe plus a
// scan of the node's children.
//
// The registry calls on_registered() when a hash becomes present in its
// first tier, outside its own mutex; the tracker's mutex is a leaf.
//
// Parity: crates/kvbm-logical/src/branch_tracker.rs:189-345 (on_block_registered,
// is_branch_point, current_fanout, current_branch_points, hot_branch_points,
// branch_points_on_prefix, branch_point_count, tracked_parent_count,
// history_len) and the BoundedBranchCache score/eviction rule (:57-176).
#pragma once

#include <algorithm>
#include <cstdint>
#include <mutex>
#include <optional>
#include <tuple>
#include <unordered_map>
#include <vector>

#include "hash.hpp"
#include "ranked_mutex.hpp"

namespace kvbm {

struct BranchRecord {
  uint64_t position = 0;
  uint64_t fragment = 0;
  uint32_t current_fanout = 0;
  uint32_t max_fanout = 0;
  uint32_t observations = 0;
  uint64_t last_tick = 0;
};

class BranchTracker {
 public:
  explicit BranchTracker(size_t history_capacity = 1024) : capacity_(history_capacity) {}

  void on_registered(const SeqHash& h) {
    if (h.position == 0) return;  // roots have no parent
    std::lock_guard<RankedMutex> g(mu_);
    const Key pk{uint64_t(h.position) - 1, h.parent};
    Node& n = parents_[pk];
    if (n.add(h.lineage)) {
      const uint32_t f = n.fanout();
      if (f >= 2) note(pk, f);
    }
    ++tick_;
  }

  bool is_branch_point(uint64_t position, uint64_t fragment) const {
    std::lock_guard<RankedMutex> g(mu_);
    auto it = parents_.find(Key{position, fragment});
    return it != parents_.end() && it->second.fanout() > 1;
  }

  std::optional<uint32_t> current_fanout(uint64_t position, uint64_t fragment) const {
    std::lock_guard<RankedMutex> g(mu_);
    auto it = parents_.find(Key{position, fragment});
    if (it == parents_.end()) return std::nullopt;
    return it->second.fanout();
  }

  // (position, fragment, fanout) of every node with fanout > 1, by position then fragment.
  std::vector<std::tuple<uint64_t, uint64_t, uint32_t>> current_branch_points() const {
    std::lock_guard<RankedMutex> g(mu_);
    std::vector<std::tuple<uint64_t, uint64_t, uint32_t>> out;
    for (const auto& [k, n] : parents_)
      if (n.fanout() > 1) out.emplace_back(k.pos, k.frag, n.fanout());
    std::sort(out.begin(), out.end());
    return out;
  }

  // History records, highest score first.
  std::vector<BranchRecord> hot_branch_points(size_t limit) const {
    std::lock_guard<RankedMutex> g(mu_);
    std::vector<std::pair<double, const BranchRecord*>> scored;
    scored.reserve(history_.size());
    for (const auto& [k, r] : history_) scored.emplace_back(score(r), &r);
    std::stable_sort(scored.begin(), scored.end(), [](auto& a, auto& b) { return a.first > b.first; });
    std::vector<BranchRecord> out;
    for (size_t i = 0; i < scored.size() && i < limit; ++i) out.push_back(*scored[i].second);
    return out;
  }

  // Branch points met along a prefix (hash i at position i): the history record when there is
  // one, else a record built from the live fanout with no observations.
  std::vector<BranchRecord> on_prefix(const std::vector<SeqHash>& prefix) const {
    std::lock_guard<RankedMutex> g(mu_);
    std::vector<BranchRecord> out;
    for (const auto& h : prefix) {
      const Key k{h.position, h.lineage};
      auto hit = history_.find(k);
      if (hit != history_.end()) {
        out.push_back(hit->second);
        continue;
      }
      auto it = parents_.find(k);
      if (it != parents_.end() && it->second.fanout() > 1) {
        const uint32_t f = it->second.fanout();
        out.push_back(BranchRecord{k.pos, k.frag, f, f, 0, tick_});
      }
    }
    return out;
  }

  size_t branch_point_count() const {
    std::lock_guard<RankedMutex> g(mu_);
    size_t c = 0;
    for (const auto& [k, n] : parents_) c += n.fanout() > 1;
    return c;
  }
  size_t tracked_parent_count() const {
    std::lock_guard<RankedMutex> g(mu_);
    return parents_.size();
  }
  size_t history_len() const {
    std::lock_guard<RankedMutex> g(mu_);
    return history_.size();
  }
  uint64_t tick() const {
    std::lock_guard<RankedMutex> g(mu_);
    return tick_;
  }

 private:
  struct Key {
    uint64_t pos, frag;
    bool operator==(const Key& o) const { return pos == o.pos && frag == o.frag; }
  };
  struct KeyHash {
    size_t operator()(const Key& k) const { return size_t(k.frag ^ (k.pos * 0x9e3779b97f4a7c15ULL)); }
  };
  struct Node {
    uint64_t first = 0;
    bool has_first = false;
    std::vector<uint64_t> more;
    uint32_t fanout() const { return uint32_t(has_first) + uint32_t(more.size()); }
    bool add(uint64_t c) {
      if (!has_first) {
        first = c;
        has_first = true;
        return true;
      }
      if (first == c || std::find(more.begin(), more.end(), c) != more.end()) return false;
      more.push_back(c);
      return true;
    }
  };

  double score(const BranchRecord& r) const {
    const uint64_t age = (tick_ > r.last_tick ? tick_ - r.last_tick : 0) + 1;
    return double(r.observations) / double(age);
  }

  void note(const Key& k, uint32_t fanout) {
    if (capacity_ == 0) return;
    auto it = history_.find(k);
    if (it != history_.end()) {
      BranchRecord& r = it->second;
      r.current_fanout = fanout;
      r.max_fanout = std::max(r.max_fanout, fanout);
      ++r.observations;
      r.last_tick = tick_;
      return;
    }
    if (history_.size() >= capacity_) {
      auto victim = history_.begin();
      double vs = score(victim->second);
      for (auto h = std::next(history_.begin()); h != history_.end(); ++h) {
        const double s = score(h->second);
        if (s < vs) vs = s, victim = h;
      }
      history_.erase(victim);
    }
    history_.emplace(k, BranchRecord{k.pos, k.frag, fanout, fanout, 1, tick_});
  }

  mutable RankedMutex mu_{kRankBranchTracker, "BranchTracker"};
  size_t capacity_;
  uint64_t tick_ = 0;
  std::unordered_map<Key, Node, KeyHash> parents_;
  std::unordered_map<Key, BranchRecord, KeyHash> history_;
};

}  // namespace kvbm
