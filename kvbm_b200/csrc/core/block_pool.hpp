// BlockPool: the logical block lifecycle of one tier, under one mutex.
//
// Slot states and transitions (parity: crates/kvbm-logical/src/pools/store.rs,
// blocks/{mutable,complete,immutable}.rs):
//
//   Reset --allocate--> Mutable --stage(hash)--> Staged --register--> Primary
//     ^                   |  ^                    |                    |
//     |  release_mutable  |  +-----unstage--------+                    | last release
//     +-------------------+<-------release_staged-+                    v
//     +<----------------------- evict (allocate) ----------------- Inactive
//     +<----------------------- reset_on_release / duplicate --------+
//
// * allocate(n) is all-or-nothing: reset (FIFO) blocks first, then evictions
//   from the inactive index in policy order; evicted hashes are reported.
// * register_block on a hash that is already active or inactive follows the
//   duplication policy: Allow keeps the new block as a Duplicate (which holds
//   a reference on the primary), Reject returns the existing primary and
//   sends the new block back to the reset pool.
// * match_prefix walks the hashes in order and stops at the first miss,
//   taking a reference on each hit (resurrecting inactive primaries) - one
//   lock acquisition for the whole batch. scan() does not stop on a miss.
// * Presence changes are reported to the shared Registry after the pool
//   mutex is released (registry before pool in lock order).
#pragma once

#include <atomic>
#include <cstdint>
#include <deque>
#include <memory>
#include <mutex>

#include "ranked_mutex.hpp"
#include <optional>
#include <stdexcept>
#include <string>
#include <unordered_map>
#include <utility>
#include <vector>

#include "hash.hpp"
#include "inactive.hpp"
#include "registry.hpp"

namespace kvbm {

enum class SlotState : int { Reset = 0, Mutable = 1, Staged = 2, Primary = 3, Duplicate = 4, Inactive = 5 };
enum class DupPolicy : int { Allow = 0, Reject = 1 };

struct PoolMetrics {
  std::atomic<uint64_t> allocations{0}, allocations_from_reset{0}, evictions{0}, registrations{0},
      registration_dedup{0}, duplicate_blocks{0}, match_hashes_requested{0}, match_blocks_returned{0},
      scan_hashes_requested{0}, scan_blocks_returned{0}, allocate_failures{0};
};

struct RegisterResult {
  BlockId block_id;   // block that carries the caller's reference
  int kind;           // 0 new primary, 1 duplicate, 2 deduplicated onto the existing primary
};

class BlockPool {
 public:
  BlockPool(size_t num_blocks, size_t block_size, const std::string& inactive_kind, int tier,
            std::shared_ptr<Registry> registry, DupPolicy policy)
      : block_size_(block_size), tier_(tier), policy_(policy), registry_(std::move(registry)) {
    if (num_blocks == 0) throw std::invalid_argument("num_blocks must be > 0");
    if (tier < 0 || tier >= kMaxTiers) throw std::invalid_argument("tier out of range");
    if (!registry_) registry_ = std::make_shared<Registry>();
    inactive_ = make_inactive_index(inactive_kind, registry_->freq());
    slots_.resize(num_blocks);
    for (size_t i = 0; i < num_blocks; ++i) free_.push_back(static_cast<BlockId>(i));
  }

  // ---------------------------------------------------------------- allocate
  std::optional<std::vector<BlockId>> allocate(size_t count, std::vector<SeqHash>* evicted_out) {
    std::vector<SeqHash> evicted;
    std::vector<BlockId> out;
    {
      std::lock_guard<RankedMutex> g(mu_);
      if (count == 0) return out;
      if (free_.size() + inactive_->size() < count) {
        metrics_.allocate_failures++;
        return std::nullopt;
      }
      const size_t from_reset = std::min(count, free_.size());
      out.reserve(count);
      for (size_t i = 0; i < from_reset; ++i) {
        out.push_back(free_.front());
        free_.pop_front();
      }
      auto ev = inactive_->evict(count - from_reset);
      if (ev.size() != count - from_reset) {
        // backend broke its size contract: roll back, commit nothing
        for (auto& p : ev) inactive_->insert(p.first, p.second);
        for (auto it = out.rbegin(); it != out.rend(); ++it) free_.push_front(*it);
        metrics_.allocate_failures++;
        return std::nullopt;
      }
      for (BlockId id : out) set_mutable(id);
      for (auto& [h, id] : ev) {
        set_mutable(id);
        out.push_back(id);
        evicted.push_back(h);
      }
      metrics_.allocations += count;
      metrics_.allocations_from_reset += from_reset;
      metrics_.evictions += ev.size();
    }
    for (auto& h : evicted) registry_->mark_absent(h, tier_);
    if (evicted_out) *evicted_out = std::move(evicted);
    return out;
  }

  void release_mutable(BlockId id) {
    std::lock_guard<RankedMutex> g(mu_);
    expect(id, SlotState::Mutable, "release_mutable");
    reset_locked(id);
  }

  void stage(BlockId id, const SeqHash& h) {
    std::lock_guard<RankedMutex> g(mu_);
    expect(id, SlotState::Mutable, "stage");
    slots_[id].state = SlotState::Staged;
    slots_[id].hash = h;
  }

  void unstage(BlockId id) {
    std::lock_guard<RankedMutex> g(mu_);
    expect(id, SlotState::Staged, "unstage");
    slots_[id].state = SlotState::Mutable;
  }

  void release_staged(BlockId id) {
    std::lock_guard<RankedMutex> g(mu_);
    expect(id, SlotState::Staged, "release_staged");
    reset_locked(id);
  }

  // -------------------------------------------------------------- register
  RegisterResult register_block(BlockId id) {
    RegisterResult res{id, 0};
    SeqHash h;
    bool presence = false;
    {
      std::lock_guard<RankedMutex> g(mu_);
      expect(id, SlotState::Staged, "register_block");
      h = slots_[id].hash;
      metrics_.registrations++;
      std::optional<BlockId> existing = acquire_locked(h);
      if (existing) {
        if (*existing == id) throw std::logic_error("register_block: collision with same block id");
        if (policy_ == DupPolicy::Allow) {
          Slot& s = slots_[id];
          s.state = SlotState::Duplicate;
          s.refs = 1;
          s.primary = *existing;  // keeps the reference acquired above
          metrics_.duplicate_blocks++;
          presence = true;
          res = {id, 1};
        } else {
          metrics_.registration_dedup++;
          reset_locked(id);
          res = {*existing, 2};
        }
      } else {
        Slot& s = slots_[id];
        s.state = SlotState::Primary;
        s.refs = 1;
        s.primary = -1;
        active_[h] = id;
        presence = true;
        res = {id, 0};
      }
    }
    if (presence) registry_->mark_present(h, tier_);
    registry_->touch(h);
    return res;
  }

  // ---------------------------------------------------------------- lookup
  std::vector<BlockId> match_prefix(const std::vector<SeqHash>& hashes) {
    std::vector<BlockId> out;
    {
      std::lock_guard<RankedMutex> g(mu_);
      metrics_.match_hashes_requested += hashes.size();
      for (auto& h : hashes) {
        auto id = acquire_locked(h);
        if (!id) break;
        out.push_back(*id);
      }
      metrics_.match_blocks_returned += out.size();
    }
    for (size_t i = 0; i < out.size(); ++i) registry_->touch(hashes[i]);
    return out;
  }

  std::vector<std::pair<SeqHash, BlockId>> scan(const std::vector<SeqHash>& hashes, bool touch) {
    std::vector<std::pair<SeqHash, BlockId>> out;
    {
      std::lock_guard<RankedMutex> g(mu_);
      metrics_.scan_hashes_requested += hashes.size();
      for (auto& h : hashes) {
        auto id = acquire_locked(h);
        if (id) out.emplace_back(h, *id);
      }
      metrics_.scan_blocks_returned += out.size();
    }
    if (touch)
      for (auto& p : out) registry_->touch(p.first);
    return out;
  }

  // Number of leading hashes present (active or inactive), no references taken.
  size_t count_prefix(const std::vector<SeqHash>& hashes) const {
    std::lock_guard<RankedMutex> g(mu_);
    size_t n = 0;
    for (auto& h : hashes) {
      if (active_.count(h) == 0 && !inactive_->has(h)) break;
      ++n;
    }
    return n;
  }

  bool contains(const SeqHash& h) const {
    std::lock_guard<RankedMutex> g(mu_);
    return active_.count(h) != 0 || inactive_->has(h);
  }

  // ------------------------------------------------------------ references
  void add_ref(BlockId id) {
    std::lock_guard<RankedMutex> g(mu_);
    check_id(id);
    Slot& s = slots_[id];
    if (s.state != SlotState::Primary && s.state != SlotState::Duplicate)
      throw std::logic_error("add_ref on a block that is not registered");
    ++s.refs;
  }

  void release(BlockId id) {
    std::vector<SeqHash> absent;
    {
      std::lock_guard<RankedMutex> g(mu_);
      release_locked(id, absent);
    }
    for (auto& h : absent) registry_->mark_absent(h, tier_);
  }

  void set_reset_on_release(BlockId id, bool v) {
    std::lock_guard<RankedMutex> g(mu_);
    check_id(id);
    slots_[id].reset_on_release = v;
  }

  // Drain every inactive block back to the reset pool (cache reset).
  size_t reset_inactive() {
    std::vector<SeqHash> absent;
    {
      std::lock_guard<RankedMutex> g(mu_);
      auto all = inactive_->evict(inactive_->size());
      for (auto& [h, id] : all) {
        reset_locked(id);
        absent.push_back(h);
      }
    }
    for (auto& h : absent) registry_->mark_absent(h, tier_);
    return absent.size();
  }

  // ------------------------------------------------------------- accessors
  size_t total_blocks() const { return slots_.size(); }
  size_t block_size() const { return block_size_; }
  int tier() const { return tier_; }
  size_t reset_len() const {
    std::lock_guard<RankedMutex> g(mu_);
    return free_.size();
  }
  size_t inactive_len() const {
    std::lock_guard<RankedMutex> g(mu_);
    return inactive_->size();
  }
  size_t available() const {
    std::lock_guard<RankedMutex> g(mu_);
    return free_.size() + inactive_->size();
  }
  size_t active_len() const {
    std::lock_guard<RankedMutex> g(mu_);
    return active_.size();
  }
  SlotState state(BlockId id) const {
    std::lock_guard<RankedMutex> g(mu_);
    check_id(id);
    return slots_[id].state;
  }
  uint32_t refs(BlockId id) const {
    std::lock_guard<RankedMutex> g(mu_);
    check_id(id);
    return slots_[id].refs;
  }
  SeqHash hash_of(BlockId id) const {
    std::lock_guard<RankedMutex> g(mu_);
    check_id(id);
    return slots_[id].hash;
  }
  std::string inactive_kind() const { return inactive_->name(); }
  const PoolMetrics& metrics() const { return metrics_; }
  std::shared_ptr<Registry> registry() const { return registry_; }

 private:
  struct Slot {
    SlotState state = SlotState::Reset;
    SeqHash hash{};
    uint32_t refs = 0;
    BlockId primary = -1;
    bool reset_on_release = false;
  };

  void check_id(BlockId id) const {
    if (id < 0 || static_cast<size_t>(id) >= slots_.size()) throw std::out_of_range("block id out of range");
  }
  void expect(BlockId id, SlotState st, const char* what) const {
    check_id(id);
    if (slots_[id].state != st) throw std::logic_error(std::string(what) + ": block in wrong state");
  }
  void set_mutable(BlockId id) {
    Slot& s = slots_[id];
    s.state = SlotState::Mutable;
    s.refs = 0;
    s.primary = -1;
    s.reset_on_release = false;
  }
  void reset_locked(BlockId id) {
    Slot& s = slots_[id];
    s.state = SlotState::Reset;
    s.refs = 0;
    s.primary = -1;
    s.reset_on_release = false;
    free_.push_back(id);
  }
  // Take a reference on the block registered under `h`, resurrecting an
  // inactive primary.
  std::optional<BlockId> acquire_locked(const SeqHash& h) {
    auto it = active_.find(h);
    if (it != active_.end()) {
      ++slots_[it->second].refs;
      return it->second;
    }
    auto id = inactive_->take(h);
    if (!id) return std::nullopt;
    Slot& s = slots_[*id];
    s.state = SlotState::Primary;
    s.refs = 1;
    active_[h] = *id;
    return id;
  }
  void release_locked(BlockId id, std::vector<SeqHash>& absent) {
    check_id(id);
    Slot& s = slots_[id];
    if (s.state != SlotState::Primary && s.state != SlotState::Duplicate)
      throw std::logic_error("release on a block that is not registered");
    if (s.refs == 0) throw std::logic_error("release: reference count underflow");
    if (--s.refs > 0) return;
    if (s.state == SlotState::Duplicate) {
      const BlockId p = s.primary;
      absent.push_back(s.hash);
      reset_locked(id);
      release_locked(p, absent);
      return;
    }
    active_.erase(s.hash);
    if (s.reset_on_release) {
      absent.push_back(s.hash);
      reset_locked(id);
    } else {
      s.state = SlotState::Inactive;
      inactive_->insert(s.hash, id);
    }
  }

  size_t block_size_;
  int tier_;
  DupPolicy policy_;
  std::shared_ptr<Registry> registry_;
  mutable RankedMutex mu_{kRankBlockPool, "BlockPool"};
  std::vector<Slot> slots_;
  std::deque<BlockId> free_;
  std::unique_ptr<InactiveIndex> inactive_;
  std::unordered_map<SeqHash, BlockId, SeqHashHasher> active_;
  PoolMetrics metrics_;
};

}  // namespace kvbm
