#include "source_file.hpp"

#include <fcntl.h>
#include <sys/stat.h>
#include <unistd.h>

#include <algorithm>
#include <cerrno>
#include <chrono>
#include <cstdlib>
#include <cstring>
#include <memory>

#include "errors.hpp"

namespace tsb {

SourceFile::SourceFile(const std::string& path, uint64_t align, bool direct) : path_(path), align_(align) {
  fd_buffered_ = ::open(path.c_str(), O_RDONLY | O_CLOEXEC);
  require(fd_buffered_ >= 0, SS_E_IO, "cannot open source " + path + ": " + std::strerror(errno));
  struct stat st {};
  require(::fstat(fd_buffered_, &st) == 0, SS_E_IO, "cannot stat source " + path);
  size_ = uint64_t(st.st_size);
  if (direct) {
    fd_ = ::open(path.c_str(), O_RDONLY | O_CLOEXEC | O_DIRECT);
    direct_ = fd_ >= 0;  // a file system that refuses O_DIRECT (tmpfs) reads buffered
  }
}

SourceFile::~SourceFile() {
  if (fd_ >= 0) ::close(fd_);
  if (fd_buffered_ >= 0) ::close(fd_buffered_);
}

namespace {
void pread_all(int fd, char* dst, uint64_t off, uint64_t n, const std::string& path) {
  while (n) {
    const ssize_t r = ::pread(fd, dst, size_t(n), off_t(off));
    if (r < 0 && errno == EINTR) continue;
    require(r > 0, SS_E_IO, "short read of " + path + " at offset " + std::to_string(off));
    dst += r;
    off += uint64_t(r);
    n -= uint64_t(r);
  }
}
}  // namespace

void SourceFile::read(void* dst, uint64_t offset, uint64_t bytes) const {
  require(offset <= size_ && bytes <= size_ - offset, SS_E_IO,
          "read past the end of " + path_ + " (offset " + std::to_string(offset) + ", bytes " + std::to_string(bytes) +
              ")");
  if (!bytes) return;
  if (!direct_) {
    pread_all(fd_buffered_, static_cast<char*>(dst), offset, bytes, path_);
    return;
  }
  const uint64_t a = align_ < 4096 ? 4096 : align_;
  if (((reinterpret_cast<uintptr_t>(dst) | offset | bytes) & (a - 1)) == 0) {  // aligned: straight into dst
    char* out = static_cast<char*>(dst);
    uint64_t pos = offset, left = bytes;
    while (left) {
      const ssize_t r = ::pread(fd_, out, size_t(left), off_t(pos));
      if (r < 0 && errno == EINTR) continue;
      if (r < 0 && errno == EINVAL) {  // refused after all: buffered for the rest
        pread_all(fd_buffered_, out, pos, left, path_);
        return;
      }
      require(r > 0, SS_E_IO, "short read of " + path_ + " at offset " + std::to_string(pos));
      out += r;
      pos += uint64_t(r);
      left -= uint64_t(r);
      if (uint64_t(r) % a != 0 && left) {  // a short unaligned piece: the rest buffered
        pread_all(fd_buffered_, out, pos, left, path_);
        return;
      }
    }
    return;
  }
  // unbuffered: aligned covering reads through a bounce buffer (at most 8 MiB per read)
  const uint64_t piece = uint64_t(8) << 20;
  void* raw = nullptr;
  require(::posix_memalign(&raw, size_t(a), size_t(piece + 2 * a)) == 0, SS_E_NOMEM, "bounce buffer");
  std::unique_ptr<void, decltype(&std::free)> bounce(raw, &std::free);
  char* out = static_cast<char*>(dst);
  uint64_t pos = offset, left = bytes;
  while (left) {
    const uint64_t start = pos / a * a, skip = pos - start;
    const uint64_t want = std::min<uint64_t>(left, piece);
    uint64_t span = (skip + want + a - 1) / a * a;
    if (start + span > (size_ + a - 1) / a * a) span = (size_ + a - 1) / a * a - start;
    ssize_t got = 0;
    while (uint64_t(got) < skip + want) {
      const ssize_t r = ::pread(fd_, static_cast<char*>(raw) + got, size_t(span - uint64_t(got)), off_t(start + uint64_t(got)));
      if (r < 0 && errno == EINTR) continue;
      if (r < 0 && errno == EINVAL) {  // refused after all: buffered for this piece
        pread_all(fd_buffered_, out, pos, want, path_);
        got = ssize_t(skip + want);
        std::memcpy(static_cast<char*>(raw) + skip, out, size_t(want));
        break;
      }
      require(r > 0, SS_E_IO, "short read of " + path_ + " at offset " + std::to_string(start + uint64_t(got)));
      got += r;
    }
    std::memcpy(out, static_cast<char*>(raw) + skip, size_t(want));
    out += want;
    pos += want;
    left -= want;
  }
}

AsyncReads::AsyncReads(unsigned threads, std::function<void(uint32_t, char*, unsigned)> read)
    : read_(std::move(read)), limit_(std::max(1u, threads)) {
  for (unsigned i = 0; i < std::max(1u, threads); ++i) th_.emplace_back([this, i] { loop(i); });
}

void AsyncReads::set_depth(std::unique_ptr<ReadDepth> c, uint64_t unit_bytes) {
  {
    std::lock_guard<std::mutex> lk(mu_);
    depth_ = std::move(c);
    unit_bytes_ = unit_bytes;
    const unsigned readers = unsigned(th_.size());
    limit_ = depth_ ? std::min(std::max(depth_->depth(), 1u), readers) : readers;
    busy_ = false;
  }
  cv_.notify_all();
}

AsyncReads::~AsyncReads() {
  {
    std::lock_guard<std::mutex> lk(mu_);
    stop_ = true;
    for (Job* j : land_q_) delete j;  // landing reads never started are dropped
    land_q_.clear();
  }
  cv_.notify_all();
  for (std::thread& t : th_) t.join();
  for (Job* j : running_) delete j;
  for (size_t i = head_; i < q_.size(); ++i) delete q_[i];
}

void AsyncReads::set_landing(unsigned cap, bool reserve) {
  std::lock_guard<std::mutex> lk(mu_);
  land_cap_ = std::max(1u, cap);
  land_reserve_ = reserve;
}

bool AsyncReads::landing_ready() const {
  if (land_q_.empty() || head_ < q_.size()) return false;
  if (!land_reserve_) return reading_ < land_cap_;
  const unsigned readers = unsigned(th_.size());
  if (readers == 1) return reading_ == 0;
  return landing_running_ < land_cap_ && landing_running_ + 1 < readers;
}

void* AsyncReads::begin_landing(uint32_t key, char* dst) {
  Job* j = new Job;
  j->key = key;
  j->dst = dst;
  j->landing = true;
  {
    std::lock_guard<std::mutex> lk(mu_);
    land_q_.push_back(j);
  }
  cv_.notify_one();
  return j;
}

bool AsyncReads::cancel(void* h) {
  std::lock_guard<std::mutex> lk(mu_);
  const auto it = std::find(land_q_.begin(), land_q_.end(), static_cast<Job*>(h));
  if (it == land_q_.end()) return false;  // running or finished: ended as usual
  delete *it;
  land_q_.erase(it);
  return true;
}

void AsyncReads::wait(void* h) {
  Job* j = static_cast<Job*>(h);
  std::unique_lock<std::mutex> lk(mu_);
  const auto queued = std::find(land_q_.begin(), land_q_.end(), j);
  if (queued != land_q_.end()) {  // a landing read not started: it runs now, at the front of the demand reads
    land_q_.erase(queued);
    j->landing = false;
    q_.insert(q_.begin() + std::ptrdiff_t(head_), j);
    cv_.notify_one();
  }
  done_cv_.wait(lk, [&] { return j->done.load(std::memory_order_acquire); });
}

void* AsyncReads::begin(uint32_t key, char* dst) {
  Job* j = new Job;
  j->key = key;
  j->dst = dst;
  {
    std::lock_guard<std::mutex> lk(mu_);
    q_.push_back(j);
  }
  cv_.notify_one();
  return j;
}

bool AsyncReads::done(void* h) const { return static_cast<const Job*>(h)->done.load(std::memory_order_acquire); }

uint64_t AsyncReads::end(void* h) {
  Job* j = static_cast<Job*>(h);
  wait(h);
  {
    std::unique_lock<std::mutex> lk(mu_);
    auto it = std::find(running_.begin(), running_.end(), j);
    require(it != running_.end(), SS_E_BACKEND, "a file read ended twice");
    running_.erase(it);
  }
  std::unique_ptr<Job> own(j);
  if (j->err) std::rethrow_exception(j->err);
  return j->ns;
}

void AsyncReads::loop(unsigned worker) {
  for (;;) {
    Job* j = nullptr;
    {
      std::unique_lock<std::mutex> lk(mu_);
      // (stopping drains the demand queue without the depth limit; landing reads never started are dropped)
      cv_.wait(lk, [&] {
        return ((stop_ || reading_ < limit_) && (head_ < q_.size() || stop_)) || (!stop_ && landing_ready());
      });
      if (head_ < q_.size() && (stop_ || reading_ < limit_)) {
        j = q_[head_++];
        if (head_ == q_.size()) {  // the queue's storage reused once every job was taken
          q_.clear();
          head_ = 0;
        }
      } else if (!stop_ && landing_ready()) {
        j = land_q_.front();
        land_q_.erase(land_q_.begin());
        ++landing_running_;
      } else {
        return;  // (stopping with nothing queued)
      }
      running_.push_back(j);
      ++reading_;
      if (depth_ && !busy_) {  // the pool leaves idle: a busy period begins
        busy_ = true;
        busy_t0_ = std::chrono::steady_clock::now();
        busy_reads_ = 0;
      }
    }
    const auto t0 = std::chrono::steady_clock::now();
    try {
      read_(j->key, j->dst, worker);
    } catch (...) {
      j->err = std::current_exception();
    }
    j->ns = uint64_t(
        std::chrono::duration_cast<std::chrono::nanoseconds>(std::chrono::steady_clock::now() - t0).count());
    bool more = false;
    {
      std::lock_guard<std::mutex> lk(mu_);
      j->done.store(true, std::memory_order_release);
      --reading_;
      landing_running_ -= j->landing ? 1 : 0;
      if (depth_ && busy_) {
        ++busy_reads_;
        if (reading_ == 0 && head_ == q_.size()) {  // idle again: the period measured, the next depth set
          const uint64_t ns = uint64_t(std::chrono::duration_cast<std::chrono::nanoseconds>(
                                           std::chrono::steady_clock::now() - busy_t0_).count());
          busy_ = false;
          const uint32_t d = depth_->on_busy(busy_reads_, busy_reads_ * unit_bytes_, ns);
          limit_ = std::min(std::max(d, 1u), unsigned(th_.size()));
        }
      }
      more = head_ < q_.size() || !land_q_.empty();
    }
    done_cv_.notify_all();
    if (more) cv_.notify_all();  // (a read held back by the depth, the cap or the reserve may start)
  }
}

ReadPool::ReadPool(unsigned threads) {
  for (unsigned i = 1; i < std::max(1u, threads); ++i) th_.emplace_back([this] { loop(); });
}

ReadPool::~ReadPool() {
  {
    std::lock_guard<std::mutex> lk(mu_);
    stop_ = true;
  }
  start_cv_.notify_all();
  for (std::thread& t : th_) t.join();
}

void ReadPool::work() {
  for (;;) {
    const size_t i = next_.fetch_add(1);
    if (i >= n_) return;
    try {
      (*fn_)(i);
    } catch (...) {
      std::lock_guard<std::mutex> lk(mu_);
      if (!err_) err_ = std::current_exception();
    }
  }
}

void ReadPool::loop() {
  uint64_t seen = 0;
  for (;;) {
    {
      std::unique_lock<std::mutex> lk(mu_);
      start_cv_.wait(lk, [&] { return stop_ || gen_ != seen; });
      if (stop_) return;
      seen = gen_;
    }
    work();
    std::lock_guard<std::mutex> lk(mu_);
    if (--busy_ == 0) done_cv_.notify_all();
  }
}

void ReadPool::run(size_t n, const std::function<void(size_t)>& fn) {
  {
    std::lock_guard<std::mutex> lk(mu_);
    fn_ = &fn;
    n_ = n;
    next_ = 0;
    err_ = nullptr;
    busy_ = th_.size();
    ++gen_;
  }
  start_cv_.notify_all();
  work();
  std::exception_ptr err;
  {
    std::unique_lock<std::mutex> lk(mu_);
    done_cv_.wait(lk, [&] { return busy_ == 0; });
    err = err_;
    fn_ = nullptr;
  }
  if (err) std::rethrow_exception(err);
}

}  // namespace tsb
