// Cross-tier block registry and KV-event emission.
//
// The registry counts, per sequence hash, how many presence-bearing blocks
// (primaries and duplicates) each tier (G1..G4) holds. A hash's first
// presence anywhere emits a Create event, its last absence a Remove event -
// the lifetime the reference ties to the registration handle's RAII
// EventReleaseHandle (crates/kvbm-logical/src/events/protocol.rs:68,
// registry/handle.rs:27). Emission is filtered by a policy: all events, or
// only positions that are powers of two within [min, max]
// (events/policy.rs:25-69, default [16, 65536]). Events are queued in order
// and drained in batches: consecutive events of one kind, Creates sorted by
// ascending position, Removes by descending position, at most `max_batch`
// hashes per batch (events/batcher.rs:22-78, events/protocol.rs:42).
//
// Lock order: a BlockPool never holds its own mutex while calling in here.
#pragma once

#include <algorithm>
#include <array>
#include <atomic>
#include <cstdint>
#include <deque>
#include <memory>
#include <mutex>

#include "ranked_mutex.hpp"
#include <unordered_map>
#include <unordered_set>
#include <vector>

#include "branch_tracker.hpp"
#include "hash.hpp"
#include "tinylfu.hpp"

namespace kvbm {

constexpr int kMaxTiers = 4;

enum class EventKind : int { Create = 0, Remove = 1 };

struct KvEvent {
  EventKind kind;
  SeqHash hash;
};

struct EventPolicy {
  bool all = true;
  uint64_t min_pos = 16;
  uint64_t max_pos = 65536;
  bool should_emit(const SeqHash& h) const {
    if (all) return true;
    const uint64_t p = h.position;
    return p >= min_pos && p <= max_pos && p != 0 && (p & (p - 1)) == 0;
  }
};

class EventQueue {
 public:
  explicit EventQueue(EventPolicy policy = {}) : policy_(policy) {}
  void set_policy(EventPolicy p) {
    std::lock_guard<RankedMutex> g(mu_);
    policy_ = p;
  }
  void on_present(const SeqHash& h) {
    std::lock_guard<RankedMutex> g(mu_);
    if (!enabled_ || !policy_.should_emit(h)) return;
    emitted_.insert(h);
    q_.push_back({EventKind::Create, h});
  }
  void on_absent(const SeqHash& h) {
    std::lock_guard<RankedMutex> g(mu_);
    if (emitted_.erase(h) == 0) return;
    q_.push_back({EventKind::Remove, h});
  }
  std::vector<KvEvent> drain(size_t max = SIZE_MAX) {
    std::lock_guard<RankedMutex> g(mu_);
    std::vector<KvEvent> out;
    while (!q_.empty() && out.size() < max) {
      out.push_back(q_.front());
      q_.pop_front();
    }
    return out;
  }
  // Batches of same-kind events, sorted for radix-tree friendliness.
  std::vector<std::pair<EventKind, std::vector<SeqHash>>> drain_batches(size_t max_batch) {
    auto evs = drain();
    std::vector<std::pair<EventKind, std::vector<SeqHash>>> out;
    for (auto& e : evs) {
      if (out.empty() || out.back().first != e.kind || out.back().second.size() >= max_batch)
        out.push_back({e.kind, {}});
      out.back().second.push_back(e.hash);
    }
    for (auto& [k, v] : out) {
      if (k == EventKind::Create)
        std::stable_sort(v.begin(), v.end(), [](auto& a, auto& b) { return a.position < b.position; });
      else
        std::stable_sort(v.begin(), v.end(), [](auto& a, auto& b) { return a.position > b.position; });
    }
    return out;
  }
  size_t pending() const {
    std::lock_guard<RankedMutex> g(mu_);
    return q_.size();
  }
  void set_enabled(bool e) {
    std::lock_guard<RankedMutex> g(mu_);
    enabled_ = e;
  }

 private:
  mutable RankedMutex mu_{kRankEventQueue, "EventQueue"};
  EventPolicy policy_;
  bool enabled_ = true;
  std::deque<KvEvent> q_;
  std::unordered_set<SeqHash, SeqHashHasher> emitted_;
};

class Registry {
 public:
  explicit Registry(std::shared_ptr<EventQueue> events = nullptr, std::shared_ptr<TinyLfu> freq = nullptr)
      : events_(std::move(events)), freq_(std::move(freq)) {}

  void mark_present(const SeqHash& h, int tier) {
    bool first = false;
    {
      std::lock_guard<RankedMutex> g(mu_);
      auto& e = map_[h];
      first = (e.total == 0);
      ++e.count[tier];
      ++e.total;
    }
    if (first && events_) events_->on_present(h);
    if (first && branches_) branches_->on_registered(h);
  }
  void mark_absent(const SeqHash& h, int tier) {
    bool last = false;
    {
      std::lock_guard<RankedMutex> g(mu_);
      auto it = map_.find(h);
      if (it == map_.end() || it->second.count[tier] == 0) return;
      --it->second.count[tier];
      if (--it->second.total == 0) {
        map_.erase(it);
        last = true;
      }
    }
    if (last && events_) events_->on_absent(h);
  }
  bool is_present(const SeqHash& h, int tier) const {
    std::lock_guard<RankedMutex> g(mu_);
    auto it = map_.find(h);
    if (it == map_.end()) return false;
    return tier < 0 ? it->second.total > 0 : it->second.count[tier] > 0;
  }
  uint32_t presence_mask(const SeqHash& h) const {
    std::lock_guard<RankedMutex> g(mu_);
    auto it = map_.find(h);
    if (it == map_.end()) return 0;
    uint32_t m = 0;
    for (int t = 0; t < kMaxTiers; ++t)
      if (it->second.count[t]) m |= 1u << t;
    return m;
  }
  void touch(const SeqHash& h) {
    if (freq_) freq_->touch(h.lineage);
  }
  uint32_t frequency(const SeqHash& h) const { return freq_ ? freq_->estimate(h.lineage) : 0; }
  size_t size() const {
    std::lock_guard<RankedMutex> g(mu_);
    return map_.size();
  }
  std::shared_ptr<EventQueue> events() const { return events_; }
  std::shared_ptr<TinyLfu> freq() const { return freq_; }
  // Set before the first registration; not synchronised with mark_present.
  void set_branch_tracker(std::shared_ptr<BranchTracker> b) { branches_ = std::move(b); }
  std::shared_ptr<BranchTracker> branch_tracker() const { return branches_; }

 private:
  struct Entry {
    std::array<uint32_t, kMaxTiers> count{};
    uint32_t total = 0;
  };
  mutable RankedMutex mu_{kRankRegistry, "Registry"};
  std::unordered_map<SeqHash, Entry, SeqHashHasher> map_;
  std::shared_ptr<EventQueue> events_;
  std::shared_ptr<TinyLfu> freq_;
  std::shared_ptr<BranchTracker> branches_;
};

}  // namespace kvbm
