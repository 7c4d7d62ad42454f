// tsb_test_read_pool: the reads-in-flight pool's scheduling rules checked with a fake read that blocks until the
// check lets it finish (no file, no device): landing reads wait behind demand reads and, with the reserve, keep one
// reader free of them; cancel drops a landing read that has not started and no other; ending a landing read still
// queued runs it at the front of the demand reads. Test infrastructure: the rules, not their timing, are checked
// (waits for a read to start are bounded at 5 s; a read that must not start is watched for 50 ms).
#include <algorithm>
#include <chrono>
#include <condition_variable>
#include <memory>
#include <mutex>
#include <set>
#include <string>
#include <thread>
#include <vector>

#include "errors.hpp"
#include "source_file.hpp"

namespace tsb {
namespace {

class FakeReads {
 public:
  // the pool's read: recorded when it starts, then held until released
  void read(uint32_t key) {
    std::unique_lock<std::mutex> lk(mu_);
    started_.push_back(key);
    ++running_;
    peak_ = std::max(peak_, running_);
    cv_.notify_all();
    cv_.wait(lk, [&] { return released_.count(key) != 0; });
    --running_;
  }
  void release(uint32_t key) {
    std::lock_guard<std::mutex> lk(mu_);
    released_.insert(key);
    cv_.notify_all();
  }
  void release_all() {  // (a check that failed: every read, held or to come, finishes)
    std::lock_guard<std::mutex> lk(mu_);
    for (uint32_t k = 0; k < 1000; ++k) released_.insert(k);
    cv_.notify_all();
  }
  bool started(uint32_t key, int ms) {
    std::unique_lock<std::mutex> lk(mu_);
    return cv_.wait_for(lk, std::chrono::milliseconds(ms),
                        [&] { return std::find(started_.begin(), started_.end(), key) != started_.end(); });
  }
  std::vector<uint32_t> order() {
    std::lock_guard<std::mutex> lk(mu_);
    return started_;
  }
  unsigned peak() {
    std::lock_guard<std::mutex> lk(mu_);
    return peak_;
  }

 private:
  std::mutex mu_;
  std::condition_variable cv_;
  std::vector<uint32_t> started_;
  std::set<uint32_t> released_;
  unsigned running_ = 0, peak_ = 0;
};

void expect(bool ok, const std::string& rule) { require(ok, SS_E_BACKEND, "tsb_test_read_pool: " + rule); }

// A scenario's fake reads, pool and helper thread; on every exit the reads are let go, the helper joined and the pool
// destroyed, in that order (a failed check never leaves a reader blocked).
struct Scenario {
  FakeReads f;
  std::unique_ptr<AsyncReads> pool;
  std::thread helper;
  explicit Scenario(unsigned readers)
      : pool(std::make_unique<AsyncReads>(readers, [this](uint32_t key, char*, unsigned) { f.read(key); })) {}
  ~Scenario() {
    f.release_all();
    if (helper.joinable()) helper.join();
    pool.reset();
  }
};

// Demand keys are below 100, landing keys from 100.
void landing_waits_and_reserve() {
  Scenario sc(2);
  FakeReads& f = sc.f;
  AsyncReads& pool = *sc.pool;
  pool.set_landing(4, true);
  void* l0 = pool.begin_landing(100, nullptr);
  void* l1 = pool.begin_landing(101, nullptr);
  expect(f.started(100, 5000), "a landing read with idle readers did not start");
  expect(!f.started(101, 50), "a second landing read ran beside the first with two readers and the reserve");
  void* d0 = pool.begin(0, nullptr);
  expect(f.started(0, 5000), "a demand read did not take the reader kept free of landing reads");
  f.release(100);
  pool.end(l0);
  expect(f.started(101, 5000), "the next landing read did not start once the first ended");
  f.release(0);
  f.release(101);
  pool.end(d0);
  pool.end(l1);
  expect(f.peak() <= 2, "more reads ran than the pool has readers");
}

void landing_behind_demand_and_cap() {
  Scenario sc(2);
  FakeReads& f = sc.f;
  AsyncReads& pool = *sc.pool;
  pool.set_landing(1, false);  // no reserve: a landing read only while fewer than 1 read of either kind runs
  void* d0 = pool.begin(0, nullptr);
  expect(f.started(0, 5000), "a demand read did not start");
  void* l0 = pool.begin_landing(100, nullptr);
  expect(!f.started(100, 50), "a landing read started while the cap was taken by a demand read");
  void* d1 = pool.begin(1, nullptr);
  expect(f.started(1, 5000), "a demand read queued after a landing read did not start first");
  f.release(0);
  f.release(1);
  pool.end(d0);
  pool.end(d1);
  expect(f.started(100, 5000), "the landing read did not start once the demand reads ended");
  f.release(100);
  pool.end(l0);
  const std::vector<uint32_t> o = f.order();
  expect(o.size() == 3 && o[2] == 100, "the landing read did not run after the demand reads");
}

void cancel_only_what_has_not_started() {
  Scenario sc(1);
  FakeReads& f = sc.f;
  AsyncReads& pool = *sc.pool;
  pool.set_landing(1, false);
  void* d0 = pool.begin(0, nullptr);
  expect(f.started(0, 5000), "a demand read did not start");
  void* l0 = pool.begin_landing(100, nullptr);
  expect(pool.cancel(l0), "a landing read that had not started was not cancelled");
  void* l1 = pool.begin_landing(101, nullptr);
  f.release(0);
  pool.end(d0);
  expect(f.started(101, 5000), "a landing read did not start on the idle reader");
  expect(!pool.cancel(l1), "a running landing read was cancelled");
  expect(!f.started(100, 50), "a cancelled landing read ran");
  f.release(101);
  pool.end(l1);
}

void ending_a_queued_landing_runs_it_first() {
  Scenario sc(2);
  FakeReads& f = sc.f;
  AsyncReads& pool = *sc.pool;
  pool.set_landing(1, true);
  void* d0 = pool.begin(0, nullptr);
  void* d1 = pool.begin(1, nullptr);
  expect(f.started(0, 5000) && f.started(1, 5000), "two demand reads on two readers did not both start");
  void* l0 = pool.begin_landing(100, nullptr);
  void* d2 = pool.begin(2, nullptr);
  sc.helper = std::thread([&pool, l0] { pool.end(l0); });  // a demand of the landing: it runs before read 2
  std::this_thread::sleep_for(std::chrono::milliseconds(20));
  f.release(0);
  expect(f.started(100, 5000), "the ended landing read did not take the freed reader");
  expect(!f.started(2, 50), "a queued demand read ran before the landing read a demand ended");
  f.release(100);
  sc.helper.join();
  f.release(1);
  f.release(2);
  pool.end(d0);
  pool.end(d1);
  pool.end(d2);
}

}  // namespace

void check_read_pool() {
  landing_waits_and_reserve();
  landing_behind_demand_and_cap();
  cancel_only_what_has_not_started();
  ending_a_queued_landing_runs_it_first();
}

}  // namespace tsb
