// Lock-rank checking for the core's mutexes.
//
// Every mutex of the core has a rank; a thread may only acquire a mutex
// whose rank is strictly greater than the rank of every mutex it already
// holds. The hierarchy:
//
//   Registry (10) -> BlockPool (20) -> EventQueue (30), TinyLfu (40), BranchTracker (45)
//   ConsolidatorTracker (50), PositionalIndex (60): independent leaves
//
// (a BlockPool releases its mutex before it calls into the registry; the
// registry may append events and touch frequencies under its own mutex; the
// multi-LRU inactive index reads TinyLFU estimates under the pool mutex).
// With KVBM_LOCK_CHECK=1 in the environment every acquisition is checked
// against a thread-local stack of held ranks and a violation throws
// LockOrderError before the mutex is taken; otherwise the check is one
// predictable branch. The test suite runs with the check on.
//
// Parity: the lock-order DAG enforcement of the reference's test builds
// (crates/kvbm-logical/src/pools/store.rs:28-38, tracing_mutex).
#pragma once

#include <cstdlib>
#include <mutex>
#include <stdexcept>
#include <string>
#include <utility>
#include <vector>

namespace kvbm {

enum LockRank : int {
  kRankRegistry = 10,
  kRankBlockPool = 20,
  kRankEventQueue = 30,
  kRankTinyLfu = 40,
  kRankBranchTracker = 45,
  kRankTracker = 50,
  kRankPositionalIndex = 60,
};

struct LockOrderError : std::logic_error {
  using std::logic_error::logic_error;
};

inline bool lock_check_enabled() {
  static const bool on = [] {
    const char* v = std::getenv("KVBM_LOCK_CHECK");
    return v != nullptr && v[0] != '\0' && v[0] != '0';
  }();
  return on;
}

class RankedMutex {
 public:
  RankedMutex(int rank, const char* name) : rank_(rank), name_(name) {}
  RankedMutex(const RankedMutex&) = delete;
  RankedMutex& operator=(const RankedMutex&) = delete;

  void lock() {
    if (lock_check_enabled()) check();
    mu_.lock();
    if (lock_check_enabled()) held().emplace_back(rank_, name_);
  }
  bool try_lock() {
    if (!mu_.try_lock()) return false;
    if (lock_check_enabled()) held().emplace_back(rank_, name_);
    return true;
  }
  void unlock() {
    if (lock_check_enabled()) {
      auto& h = held();
      for (auto it = h.rbegin(); it != h.rend(); ++it) {
        if (it->second == name_ && it->first == rank_) {
          h.erase(std::next(it).base());
          break;
        }
      }
    }
    mu_.unlock();
  }
  int rank() const { return rank_; }

  // Ranks held by the calling thread (innermost last); for tests.
  static std::vector<std::pair<int, const char*>>& held() {
    static thread_local std::vector<std::pair<int, const char*>> h;
    return h;
  }

 private:
  void check() const {
    for (const auto& [r, n] : held()) {
      if (r >= rank_)
        throw LockOrderError(std::string("lock order violation: acquiring ") + name_ + " (rank " +
                             std::to_string(rank_) + ") while holding " + n + " (rank " + std::to_string(r) + ")");
    }
  }

  std::mutex mu_;
  int rank_;
  const char* name_;
};

}  // namespace kvbm
