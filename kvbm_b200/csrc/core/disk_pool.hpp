// G3 disk tier: a file of num_blocks fixed-size block slots, read and
// written with positional I/O from a small thread pool, directly from/to
// pinned host (G2) buffers.
//
// O_DIRECT is used when requested and supported (4 KiB-aligned buffers,
// offsets and sizes; pinned G2 block slots satisfy this); otherwise buffered
// I/O. A non-persistent pool unlinks its file right after opening it, so the
// space is reclaimed when the process exits (the reference unlinks its G3
// files after NIXL registration for the same reason,
// crates/kvbm-connector/src/connector/disk_cleanup.rs). The reference drives
// G3 through NIXL's POSIX/GDS backends (crates/kvbm-physical/src/transfer/
// strategy.rs:138-205); here it is plain pread/pwrite.
#pragma once

#include <fcntl.h>
#include <sys/stat.h>
#include <unistd.h>

#include <atomic>
#include <cerrno>
#include <condition_variable>
#include <cstdint>
#include <cstring>
#include <functional>
#include <mutex>
#include <queue>
#include <stdexcept>
#include <string>
#include <thread>
#include <vector>

namespace kvbm {

class DiskPool {
 public:
  DiskPool(const std::string& path, uint64_t num_blocks, uint64_t block_bytes, bool direct, bool persistent,
           int threads)
      : path_(path), num_blocks_(num_blocks), block_bytes_(block_bytes), persistent_(persistent) {
    const int flags = O_RDWR | O_CREAT;
    fd_ = ::open(path.c_str(), flags, 0600);
    if (fd_ < 0) throw std::runtime_error("DiskPool: cannot open " + path + ": " + std::strerror(errno));
    // A second descriptor with O_DIRECT serves 4 KiB-aligned buffers; other
    // buffers go through the page cache.
    if (direct && block_bytes % 4096 == 0) {
      fd_direct_ = ::open(path.c_str(), O_RDWR | O_DIRECT);
      direct_ = fd_direct_ >= 0;
    }
    if (::ftruncate(fd_, static_cast<off_t>(num_blocks * block_bytes)) != 0) {
      ::close(fd_);
      throw std::runtime_error("DiskPool: ftruncate failed: " + std::string(std::strerror(errno)));
    }
    if (!persistent_) ::unlink(path.c_str());
    for (int i = 0; i < std::max(1, threads); ++i) workers_.emplace_back([this] { run(); });
  }

  ~DiskPool() {
    {
      std::lock_guard<std::mutex> g(mu_);
      stop_ = true;
    }
    cv_.notify_all();
    for (auto& t : workers_) t.join();
    if (fd_ >= 0) ::close(fd_);
    if (fd_direct_ >= 0) ::close(fd_direct_);
  }

  // Write blocks ids[i] from host buffers ptrs[i] (each block_bytes long).
  void write(const std::vector<int64_t>& ids, const std::vector<uint64_t>& ptrs) { io(ids, ptrs, true); }
  void read(const std::vector<int64_t>& ids, const std::vector<uint64_t>& ptrs) { io(ids, ptrs, false); }

  uint64_t num_blocks() const { return num_blocks_; }
  uint64_t block_bytes() const { return block_bytes_; }
  bool direct() const { return direct_; }
  bool persistent() const { return persistent_; }
  // descriptors of the (possibly already unlinked) file, for other I/O paths such as cuFile
  int fd() const { return fd_; }
  int fd_direct() const { return fd_direct_; }
  const std::string& path() const { return path_; }
  uint64_t bytes_written() const { return written_.load(); }
  uint64_t bytes_read() const { return read_.load(); }

 private:
  void io(const std::vector<int64_t>& ids, const std::vector<uint64_t>& ptrs, bool is_write) {
    if (ids.size() != ptrs.size()) throw std::invalid_argument("ids and ptrs differ in length");
    for (auto id : ids)
      if (id < 0 || static_cast<uint64_t>(id) >= num_blocks_) throw std::out_of_range("disk block id out of range");
    if (ids.empty()) return;
    std::atomic<size_t> remaining{ids.size()};
    std::atomic<int> err{0};
    std::mutex dm;
    std::condition_variable dcv;
    for (size_t i = 0; i < ids.size(); ++i) {
      auto job = [&, i] {
        const off_t off = static_cast<off_t>(ids[i]) * static_cast<off_t>(block_bytes_);
        char* p = reinterpret_cast<char*>(ptrs[i]);
        const int fd = (direct_ && (ptrs[i] % 4096) == 0) ? fd_direct_ : fd_;
        uint64_t done = 0;
        while (done < block_bytes_) {
          ssize_t r = is_write ? ::pwrite(fd, p + done, block_bytes_ - done, off + done)
                               : ::pread(fd, p + done, block_bytes_ - done, off + done);
          if (r < 0) {
            if (errno == EINTR) continue;
            err.store(errno);
            break;
          }
          if (r == 0) {  // reading past EOF of a never-written block: zero fill
            std::memset(p + done, 0, block_bytes_ - done);
            done = block_bytes_;
            break;
          }
          done += static_cast<uint64_t>(r);
        }
        (is_write ? written_ : read_) += done;
        if (--remaining == 0) {
          std::lock_guard<std::mutex> g(dm);
          dcv.notify_all();
        }
      };
      {
        std::lock_guard<std::mutex> g(mu_);
        q_.push(std::move(job));
      }
      cv_.notify_one();
    }
    std::unique_lock<std::mutex> lk(dm);
    dcv.wait(lk, [&] { return remaining.load() == 0; });
    if (err.load() != 0) throw std::runtime_error(std::string("DiskPool I/O failed: ") + std::strerror(err.load()));
  }

  void run() {
    while (true) {
      std::function<void()> job;
      {
        std::unique_lock<std::mutex> lk(mu_);
        cv_.wait(lk, [&] { return stop_ || !q_.empty(); });
        if (stop_ && q_.empty()) return;
        job = std::move(q_.front());
        q_.pop();
      }
      job();
    }
  }

  std::string path_;
  uint64_t num_blocks_, block_bytes_;
  bool persistent_;
  bool direct_ = false;
  int fd_ = -1;
  int fd_direct_ = -1;
  std::atomic<uint64_t> written_{0}, read_{0};
  std::mutex mu_;
  std::condition_variable cv_;
  std::queue<std::function<void()>> q_;
  std::vector<std::thread> workers_;
  bool stop_ = false;
};

}  // namespace kvbm
