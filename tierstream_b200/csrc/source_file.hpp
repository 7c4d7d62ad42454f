// A descriptor source file opened for reading: unbuffered (O_DIRECT) when asked and allowed, else buffered. Reads of
// any offset and size; an unbuffered read lands directly in the destination when its address, offset and size are
// aligned, else goes through an aligned bounce buffer of the file's alignment.
#pragma once

#include <atomic>
#include <chrono>
#include <condition_variable>
#include <cstdint>
#include <exception>
#include <functional>
#include <mutex>
#include <string>
#include <thread>
#include <vector>

#include "read_depth.hpp"

namespace tsb {

// A fixed set of reader threads serving one job at a time: run(n, fn) calls fn(i) for every i in [0, n) on the
// threads and the caller, returns once all calls finished and rethrows the first failure. One caller at a time.
// Reads in flight: a fixed set of reader threads, one read each at a time, oldest first. begin queues read(key, dst)
// and returns its handle; done answers without waiting; end waits for it, rethrows its failure and returns its time in
// ns. Every begun read must be ended exactly once, before the destination is reused or freed; queued reads still run
// at destruction.
class AsyncReads {
 public:
  // read(key, dst, worker): runs on reader thread `worker` (0 .. threads - 1), one read per thread at a time
  AsyncReads(unsigned threads, std::function<void(uint32_t, char*, unsigned)> read);
  ~AsyncReads();
  AsyncReads(const AsyncReads&) = delete;
  AsyncReads& operator=(const AsyncReads&) = delete;
  void* begin(uint32_t key, char* dst);
  bool done(void* h) const;
  void wait(void* h);  // until the read finished (it is still ended with end)
  uint64_t end(void* h);
  // Landing reads (dg_landing_blocks): queued behind every demand read; a reader takes one only while no demand read
  // is queued and, with `reserve`, fewer than `cap` landing reads run and one reader stays free of them (a single
  // reader: only while nothing else runs), else while fewer than `cap` reads of either kind run. Landing reads are
  // whole-unit reads here. cancel drops one that has not started (true: the handle is gone); ending one still queued
  // moves it to the front of the demand reads first.
  void set_landing(unsigned cap, bool reserve);
  void* begin_landing(uint32_t key, char* dst);
  bool cancel(void* h);
  // dg_disk_queue_adapt: reads start only while fewer than the controller's depth run (the readers stay allocated),
  // and each busy period of the pool (from idle to idle) is measured and fed to it, each read counted as
  // unit_bytes. Set while idle (the open, reset_open); nullptr: every reader.
  void set_depth(std::unique_ptr<ReadDepth> c, uint64_t unit_bytes);
  template <class F>
  void with_depth(F&& f) const {  // f(const ReadDepth&) under the pool's lock, if a controller is set
    std::lock_guard<std::mutex> lk(mu_);
    if (depth_) f(*depth_);
  }

 private:
  struct Job {
    uint32_t key = 0;
    char* dst = nullptr;
    std::atomic<bool> done{false};
    std::exception_ptr err;
    uint64_t ns = 0;
    bool landing = false;
  };
  bool landing_ready() const;  // (under mu_) a reader may take the oldest landing read
  void loop(unsigned worker);
  std::function<void(uint32_t, char*, unsigned)> read_;
  mutable std::mutex mu_;
  std::condition_variable cv_, done_cv_;
  std::vector<Job*> q_;                    // queued, oldest first (owned)
  std::vector<Job*> running_;              // taken by a reader, not yet ended (owned)
  size_t head_ = 0;                        // the next queued job
  std::vector<std::thread> th_;
  bool stop_ = false;
  unsigned reading_ = 0;                   // reads taken and not finished
  std::vector<Job*> land_q_;               // landing reads not started, oldest first (owned)
  unsigned landing_running_ = 0, land_cap_ = 1;
  bool land_reserve_ = false;
  unsigned limit_ = 0;                     // reads allowed at once (the readers, or the controller's depth)
  std::unique_ptr<ReadDepth> depth_;       // dg_disk_queue_adapt's controller (or none)
  uint64_t unit_bytes_ = 0;
  bool busy_ = false;                      // a busy period is being measured
  std::chrono::steady_clock::time_point busy_t0_;
  uint64_t busy_reads_ = 0;
};

class ReadPool {
 public:
  explicit ReadPool(unsigned threads);
  ~ReadPool();
  ReadPool(const ReadPool&) = delete;
  ReadPool& operator=(const ReadPool&) = delete;
  void run(size_t n, const std::function<void(size_t)>& fn);
  unsigned threads() const { return unsigned(th_.size()) + 1; }

 private:
  void loop();
  void work();
  std::mutex mu_;
  std::condition_variable start_cv_, done_cv_;
  std::vector<std::thread> th_;
  const std::function<void(size_t)>* fn_ = nullptr;
  size_t n_ = 0;
  std::atomic<size_t> next_{0};
  size_t busy_ = 0;
  uint64_t gen_ = 0;
  bool stop_ = false;
  std::exception_ptr err_;
};

class SourceFile {
 public:
  SourceFile(const std::string& path, uint64_t align, bool direct);
  ~SourceFile();
  SourceFile(const SourceFile&) = delete;
  SourceFile& operator=(const SourceFile&) = delete;
  // Reads exactly `bytes` at `offset` into dst (throws SS_E_IO on a short read or an error). Thread-safe.
  void read(void* dst, uint64_t offset, uint64_t bytes) const;
  bool direct() const { return direct_; }
  uint64_t size() const { return size_; }
  const std::string& path() const { return path_; }

 private:
  std::string path_;
  int fd_ = -1, fd_buffered_ = -1;
  bool direct_ = false;
  uint64_t align_ = 4096, size_ = 0;
};

}  // namespace tsb
