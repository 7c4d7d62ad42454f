// Host read-ahead (read_ahead.hpp).
#include "read_ahead.hpp"

#include <algorithm>

#include "errors.hpp"

namespace tsb {

ReadAhead::ReadAhead(std::vector<char*> buffers, unsigned threads, Read read)
    : bufs_(std::move(buffers)), read_(std::move(read)) {
  for (size_t b = bufs_.size(); b-- > 0;) free_.push_back(int32_t(b));
  try {
    for (unsigned t = 0; t < std::max(1u, threads); ++t) th_.emplace_back([this] { loop(); });
  } catch (...) {
    {
      std::lock_guard<std::mutex> lk(mu_);
      stop_ = true;
    }
    cv_.notify_all();
    for (auto& t : th_) t.join();
    throw;
  }
}

ReadAhead::~ReadAhead() {
  {
    std::lock_guard<std::mutex> lk(mu_);
    stop_ = true;
  }
  cv_.notify_all();
  for (auto& t : th_) t.join();
}

bool ReadAhead::requested(int layer, int unit) const {
  std::lock_guard<std::mutex> lk(mu_);
  return entries_.count(key(layer, unit)) != 0;
}

void ReadAhead::request(int layer, int unit) {
  std::lock_guard<std::mutex> lk(mu_);
  if (frozen_ || entries_.count(key(layer, unit))) return;
  auto e = std::make_shared<Entry>();
  e->layer = layer;
  e->unit = unit;
  entries_.emplace(key(layer, unit), e);  // a tombstone until the forward's end: never requested twice
  waiting_.push_back(e);
  start_locked();
}

void ReadAhead::start_locked() {
  while (!frozen_ && !waiting_.empty() && !free_.empty()) {
    EntryPtr e = waiting_.front();
    waiting_.pop_front();
    if (e->st != Entry::Waiting) continue;  // abandoned meanwhile
    e->buf = free_.back();
    free_.pop_back();
    e->st = Entry::Reading;
    queue_.push_back(e);
    cv_.notify_all();
  }
}

void ReadAhead::give_back_locked(Entry& e) {
  if (e.buf < 0 || e.quarantined) return;
  free_.push_back(e.buf);
  e.buf = -1;
  start_locked();
}

void ReadAhead::loop() {
  std::unique_lock<std::mutex> lk(mu_);
  for (;;) {
    cv_.wait(lk, [&] { return stop_ || !queue_.empty(); });
    if (queue_.empty()) return;  // (stop_)
    EntryPtr e = queue_.front();
    queue_.pop_front();
    if (e->st == Entry::Abandoned) {  // dropped before it started: never read
      give_back_locked(*e);
      continue;
    }
    e->started = true;
    ++running_;
    char* dst = bufs_[size_t(e->buf)];
    lk.unlock();
    uint64_t n = 0;
    ss_status err = SS_OK;
    std::string msg;
    try {
      n = read_(e->layer, e->unit, dst);
    } catch (const Error& x) {
      err = x.status();
      msg = x.what();
    } catch (const std::exception& x) {
      err = SS_E_IO;
      msg = x.what();
    }
    lk.lock();
    --running_;
    e->ended = true;
    e->ok = err == SS_OK;
    e->bytes = n;
    e->err = err;
    e->msg = msg;
    if (!e->ok) {  // a failed buffer is never copied from
      give_back_locked(*e);
      if (e->st != Entry::Abandoned) e->st = Entry::Failed;
    } else if (e->st == Entry::Abandoned) {
      give_back_locked(*e);
    } else if (e->st == Entry::Reading) {
      e->st = Entry::Ready;  // kept for its fetch
    }  // Landing: its fetch waits for this end
    cv_.notify_all();
  }
}

ReadAhead::EntryPtr ReadAhead::claim(int layer, int unit) {
  std::lock_guard<std::mutex> lk(mu_);
  auto it = entries_.find(key(layer, unit));
  if (it == entries_.end()) return nullptr;
  Entry& e = *it->second;
  switch (e.st) {
    case Entry::Waiting:  // not started: the file read starts as early
      e.st = Entry::Abandoned;
      return nullptr;
    case Entry::Reading:
    case Entry::Ready:
      e.st = Entry::Landing;
      return it->second;
    case Entry::Failed:
      ++total_.fallback;
      return nullptr;
    default:  // claimed before in this forward, or dropped
      return nullptr;
  }
}

const char* ReadAhead::wait(Entry& e, ss_status* status, std::string* msg) {
  std::unique_lock<std::mutex> lk(mu_);
  cv_.wait(lk, [&] { return e.ended || stop_; });
  if (e.ended && e.ok) return bufs_[size_t(e.buf)];
  if (status) *status = e.ended ? e.err : SS_E_BACKEND;
  if (msg) *msg = e.ended ? "read-ahead: " + e.msg : "read-ahead: stopped";
  return nullptr;
}

void ReadAhead::done(Entry& e, bool ok, bool issued) {
  std::lock_guard<std::mutex> lk(mu_);
  if (!ok && issued) {  // copies out of the buffer may still be in flight: it is never reused
    e.quarantined = true;
    e.st = Entry::Failed;
    return;
  }
  if (e.ended) give_back_locked(e);
  if (e.st == Entry::Landing) e.st = ok ? Entry::Consumed : Entry::Abandoned;
}

RaStats ReadAhead::end_forward() {
  std::unique_lock<std::mutex> lk(mu_);
  frozen_ = true;
  for (auto& kv : entries_) {
    Entry& e = *kv.second;
    if (e.st == Entry::Waiting || e.st == Entry::Reading || e.st == Entry::Ready) e.st = Entry::Abandoned;
  }
  waiting_.clear();
  for (const EntryPtr& e : queue_) give_back_locked(*e);  // given a buffer, never started
  queue_.clear();
  cv_.wait(lk, [&] { return running_ == 0 || stop_; });
  RaStats f;
  for (auto& kv : entries_) {
    Entry& e = *kv.second;
    if (e.ended) give_back_locked(e);  // read and never copied, or its fetch ended without done
    ++f.requested;
    f.bytes += e.bytes;
    if (e.started && e.ended) {
      if (e.ok) {
        ++f.read;
        if (e.st == Entry::Consumed) ++f.landed;
        else ++f.unused;
      } else {
        ++f.failed;
      }
    }
  }
  entries_.clear();
  total_.requested += f.requested;
  total_.read += f.read;
  total_.landed += f.landed;
  total_.unused += f.unused;
  total_.failed += f.failed;
  total_.bytes += f.bytes;
  frozen_ = false;
  return f;
}

RaStats ReadAhead::totals() const {
  std::lock_guard<std::mutex> lk(mu_);
  return total_;
}

}  // namespace tsb
