// The open's fill pipeline (loader.hpp).
#include "loader.hpp"

#include <algorithm>
#include <chrono>
#include <condition_variable>
#include <deque>
#include <exception>
#include <mutex>
#include <thread>
#include <utility>

#include "errors.hpp"

namespace tsb {

LoadStats run_load(const std::vector<LoadUnit>& units, const std::vector<char*>& buffers, uint64_t buffer_bytes,
                   uint64_t stride, unsigned readers, const std::function<void(const LoadUnit&, char*)>& read,
                   const std::function<void(size_t, const std::vector<LoadCopy>&)>& submit,
                   const std::function<void(size_t)>& recycle) {
  using Clock = std::chrono::steady_clock;
  const auto t0 = Clock::now();
  require(stride >= 1 && buffer_bytes >= stride && readers >= 1, SS_E_INVALID,
          "loader: a ring buffer holds no unit, or no reader");
  LoadStats st;
  // batches of consecutive slot units, one ring buffer each; the in-place units
  const size_t per = size_t(buffer_bytes / stride);
  std::vector<std::vector<size_t>> batches;
  std::vector<size_t> in_place;
  for (size_t i = 0; i < units.size(); ++i) {
    if (units[i].slot >= 0) {
      if (batches.empty() || batches.back().size() == per) batches.emplace_back();
      batches.back().push_back(i);
    } else {
      require(units[i].host != nullptr, SS_E_INVALID, "loader: a unit with neither a slot nor a host destination");
      in_place.push_back(i);
    }
  }
  st.slot_units = units.size() - in_place.size();
  st.host_units = in_place.size();
  st.batches = batches.size();
  require(batches.empty() || !buffers.empty(), SS_E_INVALID, "loader: units with slots and no ring buffer");
  if (units.empty()) return st;

  std::mutex mu;
  std::condition_variable reader_cv, caller_cv;
  std::vector<size_t> free_bufs;  // a stack: buffer 0 is taken first
  for (size_t b = buffers.size(); b-- > 0;) free_bufs.push_back(b);
  std::deque<std::pair<size_t, size_t>> done;  // (batch, buffer) read, not yet submitted
  size_t next_batch = 0, next_in_place = 0, waiting = 0, submitted = 0;
  unsigned active = 0;
  bool abort = false;
  std::exception_ptr err;
  auto failed = [&](std::exception_ptr e) {  // under mu
    if (!err) err = e;
    abort = true;
    reader_cv.notify_all();
    caller_cv.notify_all();
  };

  auto reader = [&] {
    std::unique_lock<std::mutex> lk(mu);
    while (!abort) {
      if (next_batch < batches.size() && !free_bufs.empty()) {
        const size_t b = next_batch++, buf = free_bufs.back();
        free_bufs.pop_back();
        lk.unlock();
        try {
          for (size_t k = 0; k < batches[b].size(); ++k) read(units[batches[b][k]], buffers[buf] + k * stride);
        } catch (...) {
          lk.lock();
          failed(std::current_exception());
          break;
        }
        lk.lock();
        done.emplace_back(b, buf);
        caller_cv.notify_one();
      } else if (next_in_place < in_place.size()) {
        const size_t i = in_place[next_in_place++];
        lk.unlock();
        try {
          read(units[i], units[i].host);
        } catch (...) {
          lk.lock();
          failed(std::current_exception());
          break;
        }
        lk.lock();
      } else if (next_batch < batches.size()) {  // every buffer is busy: the opening thread frees the oldest
        ++waiting;
        ++st.reader_waits;
        caller_cv.notify_one();
        reader_cv.wait(lk);
        --waiting;
      } else {
        break;
      }
    }
    --active;
    caller_cv.notify_one();
  };

  std::vector<std::thread> th;
  std::deque<size_t> in_flight;  // submitted, not yet recycled, oldest first
  {
    std::unique_lock<std::mutex> lk(mu);
    const unsigned n = unsigned(std::min<size_t>(readers, batches.size() + in_place.size()));
    for (unsigned t = 0; t < n; ++t) {
      ++active;
      try {
        th.emplace_back(reader);
      } catch (...) {
        --active;
        failed(std::current_exception());
        break;
      }
    }
    while (!abort) {
      if (!done.empty()) {
        const auto [b, buf] = done.front();
        done.pop_front();
        lk.unlock();
        std::vector<LoadCopy> copies;
        try {
          copies.reserve(batches[b].size());
          for (size_t k = 0; k < batches[b].size(); ++k)
            copies.push_back(LoadCopy{units[batches[b][k]].slot, buffers[buf] + k * stride, batches[b][k]});
          submit(buf, copies);
        } catch (...) {
          lk.lock();
          failed(std::current_exception());
          break;
        }
        lk.lock();
        in_flight.push_back(buf);
        st.max_in_flight = std::max<uint64_t>(st.max_in_flight, in_flight.size());
        if (++submitted == batches.size()) st.slot_seconds = std::chrono::duration<double>(Clock::now() - t0).count();
      } else if (waiting > 0 && free_bufs.empty() && !in_flight.empty()) {
        const size_t buf = in_flight.front();
        in_flight.pop_front();
        lk.unlock();
        try {
          recycle(buf);
        } catch (...) {
          lk.lock();
          failed(std::current_exception());
          break;
        }
        lk.lock();
        ++st.recycles;
        free_bufs.push_back(buf);
        reader_cv.notify_all();
      } else if (active == 0) {
        break;
      } else {
        caller_cv.wait(lk);
      }
    }
  }
  for (std::thread& t : th) t.join();
  // no copy may still read a buffer once this returns
  for (size_t buf : in_flight) {
    try {
      recycle(buf);
    } catch (...) {
      if (!err) err = std::current_exception();
    }
  }
  if (err) std::rethrow_exception(err);
  st.seconds = std::chrono::duration<double>(Clock::now() - t0).count();
  return st;
}

}  // namespace tsb
