// TinyLFU frequency sketch (Einziger, Friedman & Manes, "TinyLFU: A Highly
// Efficient Cache Admission Policy", 2015): a count-min sketch of 4-bit
// counters, 16 per 64-bit word, four hash rows, aged by halving every
// counter once `sample_size` increments have been recorded.
//
// Parity: crates/kvbm-logical/src/tinylfu.rs:125-243 (TinyLFUSketch /
// TinyLFUTracker) - the same published algorithm; hashing here is
// splitmix64 with four seeds.
#pragma once

#include <algorithm>
#include <cstdint>
#include <mutex>

#include "ranked_mutex.hpp"
#include <vector>

#include "hash.hpp"

namespace kvbm {

class TinyLfu {
 public:
  explicit TinyLfu(size_t capacity = (1u << 21)) {
    words_ = std::max<size_t>(1, capacity / 4);
    table_.assign(words_, 0);
    sample_size_ = static_cast<uint64_t>(std::max<size_t>(16, capacity)) * 10;
  }

  void touch(uint64_t key) {
    std::lock_guard<RankedMutex> g(mu_);
    bool added = false;
    for (int i = 0; i < 4; ++i) {
      const uint64_t h = splitmix64(key ^ kSeeds[i]);
      added |= inc(h % words_, static_cast<int>(h >> 60));
    }
    if (added && ++size_ >= sample_size_) age();
  }

  uint32_t estimate(uint64_t key) const {
    std::lock_guard<RankedMutex> g(mu_);
    uint32_t m = 15;
    for (int i = 0; i < 4; ++i) {
      const uint64_t h = splitmix64(key ^ kSeeds[i]);
      m = std::min(m, get(h % words_, static_cast<int>(h >> 60)));
    }
    return m;
  }

  uint64_t size() const { return size_; }

 private:
  static constexpr uint64_t kSeeds[4] = {0x243f6a8885a308d3ULL, 0x13198a2e03707344ULL, 0xa4093822299f31d0ULL,
                                         0x082efa98ec4e6c89ULL};
  bool inc(size_t w, int c) {
    const uint64_t mask = 0xFULL << (c * 4);
    if ((table_[w] & mask) == mask) return false;
    table_[w] += 1ULL << (c * 4);
    return true;
  }
  uint32_t get(size_t w, int c) const { return static_cast<uint32_t>((table_[w] >> (c * 4)) & 0xF); }
  void age() {
    for (auto& w : table_) w = (w >> 1) & 0x7777777777777777ULL;
    size_ /= 2;
  }

  mutable RankedMutex mu_{kRankTinyLfu, "TinyLfu"};
  std::vector<uint64_t> table_;
  size_t words_;
  uint64_t size_ = 0;
  uint64_t sample_size_;
};

}  // namespace kvbm
