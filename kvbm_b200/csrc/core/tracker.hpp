// Consolidator tracker and hub positional index.
//
// ConsolidatorTracker dedups KV events from several sources (the engine's
// own G1 events, e.g. vLLM, and KVBM's G2/G3 events) into one stream for a
// KV-aware router: a block is published (STORE) when the first source that
// carries tokens stores it and withdrawn (REMOVE) only when the last source
// drops it. External sources name blocks by opaque string hashes and parents
// by the parent's string hash; the tracker resolves them to sequence hashes
// so the router sees one hash space. Parity:
// crates/kvbm-consolidator/src/tracker.rs:75-364 (handle_store,
// handle_remove, handle_kvbm_store, handle_kvbm_remove, handle_clear_all,
// drain_events) and source.rs (EventSource).
//
// PositionalIndex is the hub's fleet-wide index: per block position, which
// instances hold which sequence hash; a query walks a request's hashes and
// returns the deepest one held anywhere (lineage hashing guarantees that a
// holder of a deep block also holds its ancestors). Parity:
// crates/kvbm-hub/src/features/indexer/index.rs:32-200.
#pragma once

#include <algorithm>
#include <cstdint>
#include <deque>
#include <map>
#include <mutex>

#include "ranked_mutex.hpp"
#include <optional>
#include <set>
#include <string>
#include <unordered_map>
#include <unordered_set>
#include <utility>
#include <vector>

#include "hash.hpp"

namespace kvbm {

enum class EventSource : int { Vllm = 0, Trtllm = 1, Kvbm = 2 };

struct ConsolidatedEvent {
  int kind;  // 0 store, 1 remove, 2 clear_all
  SeqHash hash{};
  std::vector<int32_t> tokens;
  int64_t block_size = 0;
  std::string lora;
  int source = 0;
};

class ConsolidatorTracker {
 public:
  // Returns true if a Store was queued.
  bool handle_store(int source, const std::string& ext, const std::optional<std::string>& parent_ext,
                    const std::vector<int32_t>& tokens, int64_t block_size, const std::string& lora) {
    if (block_size <= 0 || static_cast<int64_t>(tokens.size()) != block_size) return false;
    const SeqHash* parent = nullptr;
    SeqHash ph;
    if (parent_ext) {
      auto pit = ext_.find(key(source, *parent_ext));
      if (pit != ext_.end()) {
        ph = pit->second;
        parent = &ph;
      }
    }
    const uint64_t salt = string_salt(lora);
    const SeqHash h = chain(parent, block_hash(tokens.data(), tokens.size(), salt), salt);
    const std::string k = key(source, ext);
    auto eit = ext_.find(k);
    if (eit != ext_.end() && eit->second == h) return false;  // idempotent repeat
    auto bit = blocks_.find(h);
    if (bit != blocks_.end()) {
      bit->second.sources.insert(source);
      ext_[k] = h;
      if (!bit->second.published) {
        bit->second.published = true;
        q_.push_back({0, h, tokens, block_size, lora, source});
        return true;
      }
      return false;
    }
    State st;
    st.sources.insert(source);
    st.published = true;
    blocks_.emplace(h, std::move(st));
    ext_[k] = h;
    q_.push_back({0, h, tokens, block_size, lora, source});
    return true;
  }

  bool handle_remove(int source, const std::string& ext) {
    auto eit = ext_.find(key(source, ext));
    if (eit == ext_.end()) return false;
    const SeqHash h = eit->second;
    ext_.erase(eit);
    return drop_source(h, source);
  }

  // KVBM events carry sequence hashes but no tokens: they keep a block live
  // without being publishable on their own.
  bool handle_kvbm_store(const SeqHash& h) {
    const int src = static_cast<int>(EventSource::Kvbm);
    auto bit = blocks_.find(h);
    if (bit != blocks_.end()) {
      bit->second.sources.insert(src);
      return false;  // already live: nothing new downstream
    }
    State st;
    st.sources.insert(src);
    st.published = false;
    blocks_.emplace(h, std::move(st));
    return true;
  }

  bool handle_kvbm_remove(const SeqHash& h) { return drop_source(h, static_cast<int>(EventSource::Kvbm)); }

  void handle_clear_all() {
    blocks_.clear();
    ext_.clear();
    q_.push_back({2, {}, {}, 0, "", 0});
  }

  std::vector<ConsolidatedEvent> drain() {
    std::vector<ConsolidatedEvent> out(q_.begin(), q_.end());
    q_.clear();
    return out;
  }

  size_t num_blocks() const { return blocks_.size(); }
  size_t num_external() const { return ext_.size(); }
  bool is_live(const SeqHash& h) const { return blocks_.count(h) != 0; }

 private:
  struct State {
    std::set<int> sources;
    bool published = false;
  };
  static std::string key(int source, const std::string& ext) { return std::to_string(source) + ":" + ext; }
  bool drop_source(const SeqHash& h, int source) {
    auto bit = blocks_.find(h);
    if (bit == blocks_.end()) return false;
    bit->second.sources.erase(source);
    if (!bit->second.sources.empty()) return false;
    const bool pub = bit->second.published;
    blocks_.erase(bit);
    if (pub) q_.push_back({1, h, {}, 0, "", source});
    return pub;
  }

  std::unordered_map<SeqHash, State, SeqHashHasher> blocks_;
  std::unordered_map<std::string, SeqHash> ext_;
  std::deque<ConsolidatedEvent> q_;
};

// ---------------------------------------------------------------------------
using InstanceId = std::pair<uint64_t, uint64_t>;  // 128-bit instance id (hi, lo)

class PositionalIndex {
 public:
  PositionalIndex(uint64_t max_seq_len, uint64_t block_size) : block_size_(block_size) {
    if (block_size == 0) throw std::invalid_argument("block_size must be > 0");
    if (max_seq_len % block_size) throw std::invalid_argument("max_seq_len must be a multiple of block_size");
    max_positions_ = max_seq_len / block_size;
  }
  void grow_to(uint64_t max_seq_len) {
    std::lock_guard<RankedMutex> g(mu_);
    max_positions_ = std::max(max_positions_, max_seq_len / block_size_);
  }
  void apply_create(const InstanceId& inst, const std::vector<SeqHash>& hs) {
    std::lock_guard<RankedMutex> g(mu_);
    for (auto& h : hs) {
      if (h.position >= max_positions_) {
        ++dropped_;
        continue;
      }
      buckets_[h.position][h.lineage].insert(inst);
    }
  }
  void apply_remove(const InstanceId& inst, const std::vector<SeqHash>& hs) {
    std::lock_guard<RankedMutex> g(mu_);
    for (auto& h : hs) {
      auto b = buckets_.find(h.position);
      if (b == buckets_.end()) continue;
      auto e = b->second.find(h.lineage);
      if (e == b->second.end()) continue;
      e->second.erase(inst);
      if (e->second.empty()) b->second.erase(e);
    }
  }
  void remove_instance(const InstanceId& inst) {
    std::lock_guard<RankedMutex> g(mu_);
    for (auto& [pos, m] : buckets_) {
      for (auto it = m.begin(); it != m.end();) {
        it->second.erase(inst);
        it = it->second.empty() ? m.erase(it) : std::next(it);
      }
    }
  }
  // Deepest hash present and its holders.
  std::optional<std::pair<SeqHash, std::vector<InstanceId>>> query(const std::vector<SeqHash>& hs) const {
    std::lock_guard<RankedMutex> g(mu_);
    std::vector<SeqHash> sorted(hs);
    std::sort(sorted.begin(), sorted.end(), [](auto& a, auto& b) { return a.position > b.position; });
    for (auto& h : sorted) {
      auto b = buckets_.find(h.position);
      if (b == buckets_.end()) continue;
      auto e = b->second.find(h.lineage);
      if (e == b->second.end() || e->second.empty()) continue;
      return std::make_pair(h, std::vector<InstanceId>(e->second.begin(), e->second.end()));
    }
    return std::nullopt;
  }
  uint64_t num_positions() const {
    std::lock_guard<RankedMutex> g(mu_);
    return max_positions_;
  }
  uint64_t dropped() const {
    std::lock_guard<RankedMutex> g(mu_);
    return dropped_;
  }
  size_t num_entries() const {
    std::lock_guard<RankedMutex> g(mu_);
    size_t n = 0;
    for (auto& [p, m] : buckets_) n += m.size();
    return n;
  }
  // Every indexed block at one position bucket: (lineage word, holders), sorted by lineage.
  std::vector<std::pair<uint64_t, std::vector<InstanceId>>> at_position(uint64_t position) const {
    std::lock_guard<RankedMutex> g(mu_);
    std::vector<std::pair<uint64_t, std::vector<InstanceId>>> out;
    auto b = buckets_.find(position);
    if (b == buckets_.end()) return out;
    for (auto& [lin, insts] : b->second) out.emplace_back(lin, std::vector<InstanceId>(insts.begin(), insts.end()));
    std::sort(out.begin(), out.end(), [](auto& a, auto& c) { return a.first < c.first; });
    return out;
  }

 private:
  mutable RankedMutex mu_{kRankPositionalIndex, "PositionalIndex"};
  uint64_t block_size_;
  uint64_t max_positions_;
  uint64_t dropped_ = 0;
  std::map<uint64_t, std::unordered_map<uint64_t, std::set<InstanceId>>> buckets_;
};

}  // namespace kvbm
